"""Migration transactions on a B200, state for state against the reference's.

tests/golden/migration_trace.json was recorded by running the REFERENCE's
prepare_demote / commit_demote / prepare_promote / commit_promote / abort_*
(adaptive_sparse/migration.py:67-288) and its PhysicalPages
(adaptive_sparse/minimax_vmm.py:20-98) over the CPU stand-in world
(tests/golden/make_golden.py).  Here the same scenarios run through this
package's transactions, page tracker, VMM ``Backing`` and pinned host pool on
the GPU -- demotion packs rows with the staged copy-engine path, promotion
restores all layers in one transfer and copies the newest token with the
row-copy kernel -- and every recorded field must be equal: retained and
released page rows, host rows, hot-buffer hand-off, published mapping, owned
pages, per-chunk references, mapped chunks, pages freed, bytes released and
grown, rejected calls' exception types and messages, and that every moved row
holds the bytes it should.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_json

pytestmark = pytest.mark.gpu


def _gpu_world(cuda_device):
    from tests.support.standin import migration_world

    def make_world(**geometry):
        return migration_world(cuda_device, **geometry)

    return make_world


@pytest.mark.parametrize("scenario", ["plain", "chunk_aware", "newest_on_device", "aborts"])
def test_transactions_match_the_reference_trace(scenario, cuda_device):
    from ekv_b200 import migration
    from tests.support import migration_scenarios as ms

    want = load_json("migration_trace.json")[scenario]
    runner = {"plain": lambda mw: ms.round_trip(mw, migration, aware=False),
              "chunk_aware": lambda mw: ms.round_trip(mw, migration, aware=True),
              "newest_on_device": lambda mw: ms.round_trip(mw, migration, aware=True, newest_on_device=True),
              "aborts": lambda mw: ms.aborts(mw, migration)}[scenario]
    got = runner(_gpu_world(cuda_device))
    assert len(got) == len(want)
    for step_got, step_want in zip(got, want):
        for key in step_want:
            assert step_got[key] == step_want[key], f"{scenario} / {step_want.get('step')} / {key}"


def test_rejections_match_the_reference_trace(cuda_device):
    from ekv_b200 import migration
    from tests.support import migration_scenarios as ms

    want = load_json("migration_trace.json")["rejections"]
    got = ms.rejections(_gpu_world(cuda_device), migration)
    assert got == want


def test_demote_then_promote_moves_every_row(cuda_device, monkeypatch):
    """A larger round trip (3 layers, 5000 tokens) with chunk-aware retention: every
    committed row comes back bit for bit, released pages' chunks are unmapped, and the
    promotion's fresh pages are committed before they are written."""
    from ekv_b200 import migration
    from tests.support.standin import install_request, migration_world

    world = migration_world(cuda_device, layers=3, heads=2, head_dim=128, page_size=8, pages=2048)
    try:
        monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
        c, pool = world.coordinator, world.pool
        # Pages 1..511 belong to other requests (they share chunk 0 of every plane with
        # the sink page); this request's 625 pages fill chunk 1 and part of chunk 2 of
        # every plane, so a demotion can release a whole chunk per plane.
        world.physical.alloc(511 * world.page)
        row, length = 1, 5000
        req, slots, logical = install_request(world, row, length)
        original = [view[slots].clone() for view in world.views]
        mapped_before = len(world.backing.mapped_chunks)
        prepared = migration.prepare_demote(c, req, torch.cuda.synchronize)
        published = []
        released = migration.commit_demote(prepared, published.append, torch.cuda.synchronize,
                                           trim_quiescent=world.tracker.trim_quiescent)
        assert published == [row] and released > 0 and len(world.backing.mapped_chunks) < mapped_before
        assert (pool.full_to_hisparse_device_index_mapping[logical] == 0).all()
        promoted = migration.prepare_promote(c, req, torch.cuda.synchronize)
        destination = promoted.destination[:length]
        for p, want in enumerate(original):  # bit patterns: the seeded payload includes NaN encodings
            assert torch.equal(world.views[p][destination].view(torch.int16), want.view(torch.int16))
        grown = migration.commit_promote(promoted, published.append, torch.cuda.synchronize)
        assert published == [row, row] and grown >= 0
        assert torch.equal(pool.full_to_hisparse_device_index_mapping[logical], destination)
        with pytest.raises(RuntimeError):
            migration.abort_promote(promoted)
    finally:
        world.close()
