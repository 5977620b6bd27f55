"""GPU parity of the page -> chunk counts, the freeable bitmap and the AND combine (R4, R6)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from oracle import releasable as orl

pytestmark = pytest.mark.gpu


def _refs_array(refs, n):
    arr = torch.zeros(n, dtype=torch.int32)
    for k, v in refs.items():
        arr[int(k)] = v
    return arr


@pytest.mark.parametrize("index", range(40))
def test_counts_and_bitmap_match_reference(index, cuda_device):
    from ekv_b200.releasable import ChunkProjection, bitmap_to_chunks, chunks_to_bitmap, freeable_bitmap

    case = load_json("host_golden.json")["releasable"][index]
    n = case["n_chunks"]
    projection = ChunkProjection(case["planes"], case["page_size"], case["chunk_bytes"], n, cuda_device)
    refs = _refs_array(case["refs"], n).to(cuda_device)
    mapped = chunks_to_bitmap(case["mapped"], n, cuda_device)
    # refs themselves are the histogram of all owned pages plus the sink page 0.
    owned = torch.tensor([0, *case["owned"]], dtype=torch.int64, device=cuda_device)
    assert torch.equal(projection.counts(owned), refs)
    for pages, expected in zip(case["candidates"], case["releasable"]):
        page_t = torch.tensor(sorted(set(pages)), dtype=torch.int32, device=cuda_device)
        counts = projection.counts(page_t)
        want = orl.chunk_counts_np(sorted(set(pages)), case["planes"], case["page_size"],
                                   case["chunk_bytes"], n)
        np.testing.assert_array_equal(counts.cpu().numpy(), want)
        assert sorted(bitmap_to_chunks(freeable_bitmap(counts, refs, mapped))) == expected
    assert int(projection.overflow.item()) == 0


def test_plans_fixture_joint_chunks(cuda_device):
    """The captured TP4 state: per-rank bitmaps of the pair [1, 2] AND to the 120 chunks."""
    from ekv_b200.releasable import (ChunkProjection, bitmap_and, bitmap_to_chunks, chunks_to_bitmap,
                                     freeable_bitmap)

    plan = load_json("plans_pair12k.json")
    n = max(plan["mapped_chunks"]) + 1
    projection = ChunkProjection(plan["planes"], plan["page_size"], plan["chunk_bytes"], n, cuda_device)
    refs = _refs_array(plan["refs"], n).to(cuda_device)
    mapped = chunks_to_bitmap(plan["mapped_chunks"], n, cuda_device)
    for request in plan["requests"].values():
        counts = projection.counts(torch.tensor(request["released"], device=cuda_device))
        assert bitmap_to_chunks(freeable_bitmap(counts, refs, mapped)) == set(request["predicted_chunks"])
    pair = plan["pairs"][0]
    union = sorted({p for row in pair["rows"] for p in plan["requests"][str(row)]["released"]})
    local = freeable_bitmap(projection.counts(torch.tensor(union, device=cuda_device)), refs, mapped)
    gathered = local.repeat(plan["ranks"], 1).contiguous()
    joint = bitmap_and(gathered)
    assert sorted(bitmap_to_chunks(joint)) == pair["predicted_chunks"]


@pytest.mark.parametrize("n_chunks", [4096, 100_003])
def test_counts_shared_and_global_paths(n_chunks, cuda_device):
    """Small tables use the shared-memory histogram, large ones global atomics."""
    from ekv_b200.releasable import ChunkProjection

    gen = torch.Generator().manual_seed(n_chunks)
    chunk_bytes, page_size = 4096, 4
    planes = []
    per_plane = n_chunks // 8
    for p in range(8):
        planes.append((p * per_plane, int(torch.randint(1, 600, (1,), generator=gen)) * 2))
    max_page = min(per_plane * chunk_bytes // (page_size * max(r for _, r in planes)), 1 << 20) - 1
    pages = torch.randperm(max_page, generator=gen)[: max_page // 2] + 1
    projection = ChunkProjection(planes, page_size, chunk_bytes, n_chunks, cuda_device)
    got = projection.counts(pages.to(cuda_device))
    want = orl.chunk_counts_np(pages.numpy(), planes, page_size, chunk_bytes, n_chunks)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    assert int(projection.overflow.item()) == 0
    again = projection.counts(pages.to(cuda_device), out=got, accumulate=True)
    np.testing.assert_array_equal(again.cpu().numpy(), 2 * want)


def test_bitmap_and_random(cuda_device):
    from ekv_b200.releasable import bitmap_and

    gen = torch.Generator().manual_seed(4)
    gathered = torch.randint(-(1 << 62), 1 << 62, (8, 64), generator=gen)
    got = bitmap_and(gathered.to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(got, orl.bitmap_and_np(gathered.numpy()))


def test_freeable_chunks_tracker_view(cuda_device):
    """FreeableChunks over a PhysicalPages tracker answers like the reference's set helpers."""
    from ekv_b200.physical_pages import PhysicalPages
    from ekv_b200.releasable import FreeableChunks

    class Backing:
        def __init__(self):
            self.mapped_chunks = set()
            self.backed_bytes = 0

        def ensure(self, indices):
            self.mapped_chunks.update(indices)

        def reclaim(self, indices, *, synchronize):
            self.mapped_chunks.difference_update(indices)
            return len(indices)

    case = load_json("host_golden.json")["releasable"][7]
    tracker = PhysicalPages(Backing(), case["page_size"], case["page_count"],
                            [tuple(p) for p in case["planes"]], lambda: None, chunk_bytes=case["chunk_bytes"])
    tracker.acquire(case["owned"])
    tracker.backing.mapped_chunks.intersection_update(case["mapped"])
    freeable = FreeableChunks(tracker, cuda_device)
    for pages, expected in zip(case["candidates"], case["releasable"]):
        assert sorted(freeable.releasable(pages)) == expected
    c = case["candidates"]
    assert sorted(freeable.releasable_group([c[0], c[1]])) == case["pair"]
    assert sorted(freeable.releasable_group(c)) == case["group"]
