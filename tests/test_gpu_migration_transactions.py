"""The reference's migration transactions, driven end to end on a B200.

prepare_demote -> commit_demote -> prepare_promote -> commit_promote
(adaptive_sparse/migration.py:67-288) run over a VMM-backed device pool laid out
like the MiniMax planes (adaptive_sparse/minimax_vmm.py:210-243: chunk-aligned
K/V planes of one reservation), a PhysicalPages tracker, the pinned host pool
and a minimal stand-in for SGLang's coordinator.  Every committed row must come
back bit for bit, released pages' chunks must be unmapped, and the promotion's
fresh pages must be committed before they are written.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

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


@pytest.fixture()
def world(cuda_device):
    from ekv_b200.backing import Backing
    from ekv_b200.host_pool import PinnedHostKVPool
    from ekv_b200.physical_pages import PhysicalPages

    dev = cuda_device
    layers, heads, dim, page, pages = 3, 2, 128, 8, 2048
    size = pages * page
    row_bytes = heads * dim * 2
    plane_bytes = (size + page) * row_bytes
    plane_chunks = -(-plane_bytes // CHUNK)
    backing = Backing(CHUNK * 2 * layers * plane_chunks, CHUNK, device=dev.index)
    planes = [(p * plane_chunks, row_bytes) for p in range(2 * layers)]
    tracker = PhysicalPages(backing, page, pages, planes, torch.cuda.synchronize)
    raw = backing.raw
    views = [raw.narrow(0, first * CHUNK, (size + page) * row_bytes).view(torch.bfloat16).view(size + page, heads, dim)
             for first, _ in planes]
    pool = SimpleNamespace(
        page_size=page, start_layer=0, end_layer=layers, adaptive_vmm=tracker,
        get_key_buffer=lambda l: views[2 * l], get_value_buffer=lambda l: views[2 * l + 1],
        full_to_hisparse_device_index_mapping=torch.zeros(1 << 16, dtype=torch.int64, device=dev))
    pool.translate_loc_from_full_to_hisparse_device = lambda logical: pool.full_to_hisparse_device_index_mapping[logical]
    physical = PagedAllocator(tracker, page, pages, dev)
    rows, capacity = 4, 64
    host = PinnedHostKVPool(8192, layers, row_bytes, dev)
    coordinator = SimpleNamespace(
        is_m3_hisparse=True, spec_swap=SimpleNamespace(enabled=False, reset=lambda row: None),
        padded_buffer_size=capacity, device_buffer_size=capacity - page, compress_ratio=1,
        req_device_buffer_size=torch.zeros(rows, dtype=torch.int64, device=dev),
        req_to_host_pool=torch.full((rows, 8192), -1, dtype=torch.int64),
        req_to_host_pool_allocated_len=torch.zeros(rows, dtype=torch.int64),
        req_to_token_pool=SimpleNamespace(req_to_token=torch.zeros((rows, 8192), dtype=torch.int64, device=dev)),
        mem_pool_device=pool, mem_pool_host=host, wait_for_pending_backup=lambda: None,
        token_to_kv_pool_allocator=TokenAllocator(physical),
        req_to_device_buffer=torch.zeros((rows, 4096), dtype=torch.int64, device=dev),
        req_device_buffer_tokens=torch.zeros((1, rows, capacity), dtype=torch.int64, device=dev),
        req_device_buffer_token_locs=torch.zeros((1, rows, 4096), dtype=torch.int64, device=dev),
        lru_slots=torch.zeros((1, rows, capacity), dtype=torch.int64, device=dev),
        _lru_init=torch.arange(capacity, device=dev), _skip_first_backup=[False] * rows)

    def cleanup(req):  # promotion releases the host rows and the hot buffer of the row
        row = req.kv.req_pool_idx
        n = int(coordinator.req_to_host_pool_allocated_len[row])
        if n:
            host.free(coordinator.req_to_host_pool[row, :n])
        coordinator.req_to_host_pool[row].fill_(-1)
        coordinator.req_to_host_pool_allocated_len[row] = 0
        coordinator.req_device_buffer_size[row] = 0

    coordinator._ekv_cleanup_promotion_source = cleanup
    yield SimpleNamespace(coordinator=coordinator, pool=pool, views=views, tracker=tracker, backing=backing,
                          physical=physical, host=host, layers=layers, page=page)
    del raw, views
    torch.cuda.synchronize()
    backing.close()


def test_demote_then_promote_round_trip(world, monkeypatch):
    from ekv_b200 import migration

    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
    c, pool, page = world.coordinator, world.pool, world.page
    dev = pool.full_to_hisparse_device_index_mapping.device
    # Pages 1..511 belong to other requests (they share chunk 0 of every plane
    # with the sink page); this request's 625 pages fill chunk 1 and part of
    # chunk 2 of every plane, so a demotion can release a whole chunk per plane.
    world.physical.alloc(511 * page)
    row, length = 1, 5000
    slots = world.physical.alloc(-(-length // page) * page)[:length]
    logical = torch.arange(1, length + 1, device=dev) * 7 + 3
    c.req_to_token_pool.req_to_token[row, :length] = logical
    pool.full_to_hisparse_device_index_mapping[logical] = slots
    gen = torch.Generator(device=dev).manual_seed(3)
    for view in world.views:
        view[slots] = torch.randn(view[slots].shape, generator=gen, device=dev).to(torch.bfloat16)
    original = [view[slots].clone() for view in world.views]
    req = SimpleNamespace(kv=SimpleNamespace(req_pool_idx=row, kv_committed_len=length, kv_allocated_len=length),
                          hisparse_staging=False)
    mapped_before = len(world.backing.mapped_chunks)

    prepared = migration.prepare_demote(c, req, torch.cuda.synchronize)
    host_rows = c.req_to_host_pool[row, :length]
    for p, want in enumerate(original):
        got = world.host.plane_view(p)[host_rows].view(torch.bfloat16).view(want.shape)
        assert torch.equal(got.to(dev), want)
    published = []
    released = migration.commit_demote(prepared, published.append, torch.cuda.synchronize,
                                       trim_quiescent=world.tracker.trim_quiescent)
    assert published == [row] and prepared.status == "committed"
    assert released > 0 and len(world.backing.mapped_chunks) < mapped_before
    assert (pool.full_to_hisparse_device_index_mapping[logical] == 0).all()
    kept = c.req_to_device_buffer[row, :c.padded_buffer_size]
    assert torch.equal(torch.sort(kept).values, torch.sort(slots[torch.isin(slots, kept)]).values)

    promoted = migration.prepare_promote(c, req, torch.cuda.synchronize)
    destination = promoted.destination[:length]
    for p, want in enumerate(original):
        assert torch.equal(world.views[p][destination], want)
    grown = migration.commit_promote(promoted, published.append, torch.cuda.synchronize)
    assert published == [row, row] and promoted.status == "committed" and grown >= 0
    assert torch.equal(pool.full_to_hisparse_device_index_mapping[logical], destination)
    assert int(c.req_to_host_pool_allocated_len[row]) == 0
    with pytest.raises(RuntimeError):
        migration.abort_promote(promoted)
