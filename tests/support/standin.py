"""A minimal stand-in for the SGLang objects the migration transactions touch.

adaptive_sparse/migration.py:27-288 reads and writes a HiSparse coordinator
(request -> token / host / hot-buffer tables, the device and host KV pools, the
token allocator) that lives in SGLang.  This module builds the smallest
coordinator those transactions accept, in two flavours with identical state
and allocation order:

* ``migration_world(device)`` on a GPU: this package's VMM ``Backing``, its
  ``PhysicalPages`` tracker over chunk-aligned K/V planes
  (adaptive_sparse/minimax_vmm.py:210-243 is the plane layout) and its
  ``PinnedHostKVPool`` -- used by the GPU tests and bench.py's round-trip leg;
* ``migration_world("cpu", tracker_cls=..., host_pool_cls=CpuHostPool)`` on
  CPU tensors with a set-based fake backing -- used by the golden generator to
  run the REFERENCE's transactions and PhysicalPages.

It is test infrastructure: it moves no KV data of its own except the seeded
payload it writes when a request is installed (the "prefill").
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

CHUNK = 2 << 20


def payload(plane, slots, width):
    """Seeded int16 payload of rows ``slots`` of plane ``plane``: [n, width] int16.

    The same formula on CPU and GPU, so either world can check any moved row.
    """
    slots = slots.to(torch.int64)
    cols = torch.arange(width, device=slots.device, dtype=torch.int64)
    mixed = slots[:, None] * 2654435761 + plane * 40503 + cols[None, :] * 97
    return ((mixed >> 7) & 0x7FFF).to(torch.int16)


class FakeBacking:
    """Set-based stand-in of ``Backing`` for the CPU world (ensure / reclaim / counts)."""

    def __init__(self, chunk_bytes):
        self.chunk_bytes = chunk_bytes
        self.mapped_chunks = set()

    @property
    def backed_bytes(self):
        return len(self.mapped_chunks) * self.chunk_bytes

    def ensure(self, indices):
        self.mapped_chunks.update(int(i) for i in indices)

    def reclaim(self, indices, *, synchronize=True):
        gone = self.mapped_chunks & {int(i) for i in indices}
        self.mapped_chunks -= gone
        return len(gone)


class CpuHostPool:
    """Host KV pool on plain CPU tensors with ``PinnedHostKVPool``'s allocation order
    (lowest free rows first) and SGLang HostKVCache's migration methods."""

    def __init__(self, capacity, layer_num, row_bytes, device, dtype=torch.bfloat16):
        self.capacity, self.layer_num, self.row_bytes = capacity, layer_num, row_bytes
        self.planes = torch.zeros((2 * layer_num, capacity, row_bytes), dtype=torch.uint8)
        self._free = torch.ones(capacity, dtype=torch.bool)

    def available_size(self):
        return int(self._free.sum())

    def alloc(self, need):
        free = torch.nonzero(self._free).flatten()
        if free.numel() < need:
            return None
        chosen = free[:need]
        self._free[chosen] = False
        return chosen

    def free(self, indices):
        indices = indices.to("cpu", torch.int64)
        if (~self._free[indices]).sum() != indices.numel():
            raise RuntimeError("double free of host KV rows")
        self._free[indices] = True
        return indices.numel()

    def alloc_paged_token_slots(self, req_to_host_pool, allocated_len, row, start, length):
        indices = self.alloc(length - start)
        if indices is None:
            raise MemoryError("host KV pool exhausted")
        req_to_host_pool[row, start:length] = indices.to(req_to_host_pool.dtype)
        allocated_len[row] = length
        return req_to_host_pool[row, :length]

    def allocated_host_indices(self, req_to_host_pool, row, length):
        return req_to_host_pool[row, :int(length)]

    def plane_view(self, plane):
        return self.planes[plane]

    @staticmethod
    def _bytes(view):
        return view.reshape(view.shape[0], -1).view(torch.uint8)

    def backup_from_device_all_layer(self, device_pool, host_indices, device_indices, io_backend="kernel"):
        for layer in range(device_pool.start_layer, device_pool.end_layer):
            for which, view in enumerate((device_pool.get_key_buffer(layer), device_pool.get_value_buffer(layer))):
                self.planes[2 * layer + which][host_indices.long()] = self._bytes(view)[device_indices.long()]

    def load_to_device_per_layer(self, device_pool, host_indices, device_indices, layer_id, io_backend="kernel"):
        for which, view in enumerate((device_pool.get_key_buffer(layer_id), device_pool.get_value_buffer(layer_id))):
            self._bytes(view)[device_indices.long()] = self.planes[2 * layer_id + which][host_indices.long()]


class PagedAllocator:
    """Page-granular physical allocator (lowest free pages first, freed pages go to the
    back of the list) that acquires and releases pages through the tracker."""

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
        self.freed = []  # pages of every free call, in call order

    def free_hisparse_indices(self, slots):
        pages = sorted({int(s) // self.hisparse_attn_allocator.page_size for s in slots.tolist()})
        self.hisparse_attn_allocator.tracker.release(set(pages))
        self.hisparse_attn_allocator.free_pages.extend(pages)
        self.freed.append(pages)


def migration_world(device, *, layers, heads, head_dim, page_size, pages, rows=4, hot_capacity=64,
                    host_rows=8192, table_width=8192, spare_chunks=0, tracker_cls=None,
                    host_pool_cls=None):
    """Backing + tracker + host pool + coordinator for ``rows`` request rows.

    ``device`` "cpu" builds the CPU world (``FakeBacking``, CPU planes); a CUDA
    device builds this package's world.  ``tracker_cls`` / ``host_pool_cls``
    default to this package's ``PhysicalPages`` / ``PinnedHostKVPool``.

    Returns a namespace with ``coordinator``, ``pool`` (the device pool view the
    transactions use), ``views`` (one [slots, heads, head_dim] bf16 tensor per
    plane, K and V of each layer), ``tracker``, ``backing``, ``physical``,
    ``host``, ``width`` and ``close()``.
    """
    dev = torch.device(device)
    size = pages * page_size
    row_bytes = heads * head_dim * 2
    plane_rows = size + page_size
    plane_chunks = -(-(plane_rows * row_bytes) // CHUNK)
    planes = [(p * plane_chunks, row_bytes) for p in range(2 * layers)]
    if dev.type == "cpu":
        backing = FakeBacking(CHUNK)
        views = [torch.zeros((plane_rows, heads, head_dim), dtype=torch.bfloat16) for _ in planes]
        sync = (lambda: None)
    else:
        from ekv_b200.backing import Backing

        backing = Backing(CHUNK * 2 * layers * plane_chunks, CHUNK, device=dev.index, spare_chunks=spare_chunks)
        sync = torch.cuda.synchronize
        views = None
    if tracker_cls is None:
        from ekv_b200.physical_pages import PhysicalPages as tracker_cls
    if host_pool_cls is None:
        from ekv_b200.host_pool import PinnedHostKVPool as host_pool_cls
    tracker = tracker_cls(backing, page_size, pages, planes, sync)
    if views is None:
        raw = backing.raw
        views = [raw.narrow(0, first * CHUNK, plane_rows * row_bytes).view(torch.bfloat16)
                 .view(plane_rows, heads, head_dim) for first, _ in planes]
        del raw
    pool = SimpleNamespace(
        page_size=page_size, start_layer=0, end_layer=layers, adaptive_vmm=tracker,
        get_key_buffer=lambda layer: views[2 * layer], get_value_buffer=lambda layer: views[2 * layer + 1],
        full_to_hisparse_device_index_mapping=torch.zeros(rows * table_width * 8, dtype=torch.int64, device=dev))
    pool.translate_loc_from_full_to_hisparse_device = (
        lambda logical: pool.full_to_hisparse_device_index_mapping[logical])
    physical = PagedAllocator(tracker, page_size, pages, dev)
    host = host_pool_cls(host_rows, layers, row_bytes, dev)
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
                            physical=physical, host=host, layers=layers, page=page_size, row_bytes=row_bytes,
                            width=heads * head_dim, device=dev, sync=sync)

    def close():
        world.views.clear()
        if dev.type == "cuda":
            torch.cuda.synchronize()
            backing.close()

    world.close = close
    return world


def install_request(world, row, length, logical_stride=7, seed=3):
    """Give request ``row`` ``length`` committed tokens in fresh pages and write their
    K/V rows ("prefill") with the seeded ``payload``.

    Returns ``(req, slots, logical)``: the request object the transactions take,
    its physical slots and its logical token ids.
    """
    c, pool, page = world.coordinator, world.pool, world.page
    dev = pool.full_to_hisparse_device_index_mapping.device
    slots = world.physical.alloc(-(-length // page) * page)[:length]
    logical = torch.arange(1, length + 1, device=dev) * logical_stride + 3
    c.req_to_token_pool.req_to_token[row, :length] = logical
    pool.full_to_hisparse_device_index_mapping[logical] = slots
    for p, view in enumerate(world.views):
        view.view(view.shape[0], -1).view(torch.int16)[slots] = payload(p + 100 * seed, slots, world.width)
    req = SimpleNamespace(kv=SimpleNamespace(req_pool_idx=row, kv_committed_len=length, kv_allocated_len=length),
                          hisparse_staging=False)
    return req, slots, logical
