"""A minimal stand-in for the SGLang objects the migration transactions touch.

adaptive_sparse/migration.py:27-288 reads and writes a HiSparse coordinator
(request -> token / host / hot-buffer tables, the device and host KV pools, the
token allocator) that lives in SGLang.  This module builds the smallest
coordinator those transactions accept, over this package's own parts -- a
VMM ``Backing``, a ``PhysicalPages`` tracker for the chunk-aligned K/V planes
(adaptive_sparse/minimax_vmm.py:210-243) and the ``PinnedHostKVPool`` -- so the
demote / promote path runs end to end without SGLang: in the GPU tests and in
bench.py's round-trip leg.  It allocates and moves no KV data itself.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

CHUNK = 2 << 20


class PagedAllocator:
    """Page-granular physical allocator that maps chunks through the tracker."""

    def __init__(self, tracker, page_size, page_count, device):
        self.tracker, self.page_size, self.device = tracker, page_size, device
        self.free_pages = list(range(1, page_count + 1))

    def alloc(self, need):
        pages = need // self.page_size
        if pages > len(self.free_pages):
            return None
        taken, self.free_pages = self.free_pages[:pages], self.free_pages[pages:]
        self.tracker.acquire(taken)
        base = torch.tensor(taken, dtype=torch.int64, device=self.device) * self.page_size
        return (base[:, None] + torch.arange(self.page_size, device=self.device)).flatten()


class TokenAllocator:
    def __init__(self, physical):
        self.hisparse_attn_allocator = physical
        self._kvcache = SimpleNamespace()

    def free_hisparse_indices(self, slots):
        pages = sorted({int(s) // self.hisparse_attn_allocator.page_size for s in slots.tolist()})
        self.hisparse_attn_allocator.tracker.release(set(pages))
        self.hisparse_attn_allocator.free_pages.extend(pages)


def migration_world(device, *, layers, heads, head_dim, page_size, pages, rows=4, hot_capacity=64,
                    host_rows=8192, table_width=8192, spare_chunks=0):
    """Backing + tracker + host pool + coordinator for ``rows`` request rows.

    Returns a namespace with ``coordinator``, ``pool`` (the device pool view the
    transactions use), ``views`` (one [slots, heads, head_dim] bf16 tensor per
    plane, K and V of each layer), ``tracker``, ``backing``, ``physical``,
    ``host`` and ``close()``.
    """
    from .backing import Backing
    from .host_pool import PinnedHostKVPool
    from .physical_pages import PhysicalPages

    dev = torch.device(device)
    size = pages * page_size
    row_bytes = heads * head_dim * 2
    plane_bytes = (size + page_size) * row_bytes
    plane_chunks = -(-plane_bytes // CHUNK)
    backing = Backing(CHUNK * 2 * layers * plane_chunks, CHUNK, device=dev.index, spare_chunks=spare_chunks)
    planes = [(p * plane_chunks, row_bytes) for p in range(2 * layers)]
    tracker = PhysicalPages(backing, page_size, pages, planes, torch.cuda.synchronize)
    raw = backing.raw
    views = [raw.narrow(0, first * CHUNK, (size + page_size) * row_bytes).view(torch.bfloat16)
             .view(size + page_size, heads, head_dim) for first, _ in planes]
    pool = SimpleNamespace(
        page_size=page_size, start_layer=0, end_layer=layers, adaptive_vmm=tracker,
        get_key_buffer=lambda layer: views[2 * layer], get_value_buffer=lambda layer: views[2 * layer + 1],
        full_to_hisparse_device_index_mapping=torch.zeros(rows * table_width * 8, dtype=torch.int64, device=dev))
    pool.translate_loc_from_full_to_hisparse_device = (
        lambda logical: pool.full_to_hisparse_device_index_mapping[logical])
    physical = PagedAllocator(tracker, page_size, pages, dev)
    host = PinnedHostKVPool(host_rows, layers, row_bytes, dev)
    coordinator = SimpleNamespace(
        is_m3_hisparse=True, spec_swap=SimpleNamespace(enabled=False, reset=lambda row: None),
        padded_buffer_size=hot_capacity, device_buffer_size=hot_capacity - page_size, compress_ratio=1,
        req_device_buffer_size=torch.zeros(rows, dtype=torch.int64, device=dev),
        req_to_host_pool=torch.full((rows, table_width), -1, dtype=torch.int64),
        req_to_host_pool_allocated_len=torch.zeros(rows, dtype=torch.int64),
        req_to_token_pool=SimpleNamespace(req_to_token=torch.zeros((rows, table_width), dtype=torch.int64,
                                                                   device=dev)),
        mem_pool_device=pool, mem_pool_host=host, wait_for_pending_backup=lambda: None,
        token_to_kv_pool_allocator=TokenAllocator(physical),
        req_to_device_buffer=torch.zeros((rows, table_width), dtype=torch.int64, device=dev),
        req_device_buffer_tokens=torch.zeros((1, rows, hot_capacity), dtype=torch.int64, device=dev),
        req_device_buffer_token_locs=torch.zeros((1, rows, table_width), dtype=torch.int64, device=dev),
        lru_slots=torch.zeros((1, rows, hot_capacity), dtype=torch.int64, device=dev),
        _lru_init=torch.arange(hot_capacity, device=dev), _skip_first_backup=[False] * rows)

    def cleanup(req):  # promotion releases the host rows and the hot buffer of the row
        row = req.kv.req_pool_idx
        n = int(coordinator.req_to_host_pool_allocated_len[row])
        if n:
            host.free(coordinator.req_to_host_pool[row, :n])
        coordinator.req_to_host_pool[row].fill_(-1)
        coordinator.req_to_host_pool_allocated_len[row] = 0
        coordinator.req_device_buffer_size[row] = 0

    coordinator._ekv_cleanup_promotion_source = cleanup
    world = SimpleNamespace(coordinator=coordinator, pool=pool, views=views, tracker=tracker, backing=backing,
                            physical=physical, host=host, layers=layers, page=page_size, row_bytes=row_bytes)

    def close():
        world.views.clear()
        torch.cuda.synchronize()
        backing.close()

    world.close = close
    del raw
    return world


def install_request(world, row, length, logical_stride=7, seed=3):
    """Give request ``row`` ``length`` committed tokens in fresh pages, with seeded rows.

    Returns ``(req, slots, logical)``: the request object the transactions take,
    its physical slots and its logical token ids.
    """
    c, pool, page = world.coordinator, world.pool, world.page
    dev = pool.full_to_hisparse_device_index_mapping.device
    slots = world.physical.alloc(-(-length // page) * page)[:length]
    logical = torch.arange(1, length + 1, device=dev) * logical_stride + 3
    c.req_to_token_pool.req_to_token[row, :length] = logical
    pool.full_to_hisparse_device_index_mapping[logical] = slots
    gen = torch.Generator(device=dev).manual_seed(seed)
    for view in world.views:
        view[slots] = torch.randn(view[slots].shape, generator=gen, device=dev).to(torch.bfloat16)
    req = SimpleNamespace(kv=SimpleNamespace(req_pool_idx=row, kv_committed_len=length, kv_allocated_len=length),
                          hisparse_staging=False)
    return req, slots, logical
