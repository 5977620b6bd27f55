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

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture()
def world(cuda_device):
    from ekv_b200.standin import migration_world

    world = migration_world(cuda_device, layers=3, heads=2, head_dim=128, page_size=8, pages=2048)
    yield world
    world.close()


def test_demote_then_promote_round_trip(world, monkeypatch):
    from ekv_b200 import migration
    from ekv_b200.standin import install_request

    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
    c, pool, page = world.coordinator, world.pool, world.page
    dev = pool.full_to_hisparse_device_index_mapping.device
    # Pages 1..511 belong to other requests (they share chunk 0 of every plane
    # with the sink page); this request's 625 pages fill chunk 1 and part of
    # chunk 2 of every plane, so a demotion can release a whole chunk per plane.
    world.physical.alloc(511 * page)
    row, length = 1, 5000
    req, slots, logical = install_request(world, row, length)
    original = [view[slots].clone() for view in world.views]
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
