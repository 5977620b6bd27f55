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


@pytest.mark.parametrize("owners", [2, 3])
def test_shared_chunk_is_freeable_only_with_every_owner(owners, cuda_device):
    """tests/test_scheduler_budget.py:414-426 and :769-775 on the device: a chunk owned by
    ``owners`` pages is in the freeable bitmap only for a candidate set holding all of them."""
    import itertools

    from ekv_b200.releasable import ChunkProjection, bitmap_to_chunks, chunks_to_bitmap, freeable_bitmap

    planes, page_size, chunk_bytes, n = [(9, 16)], 4, 256, 64  # pages 0-3 all lie in chunk 9
    projection = ChunkProjection(planes, page_size, chunk_bytes, n, cuda_device)
    refs = torch.zeros(n, dtype=torch.int32, device=cuda_device)
    refs[9] = owners
    pages = list(range(1, owners + 1))
    for mapped_chunks in ({9}, set()):
        mapped = chunks_to_bitmap(mapped_chunks, n, cuda_device)
        for size in range(1, owners + 1):
            for subset in itertools.combinations(pages, size):
                counts = projection.counts(torch.tensor(subset, dtype=torch.int64, device=cuda_device))
                want = {9} if size == owners and mapped_chunks else set()
                assert bitmap_to_chunks(freeable_bitmap(counts, refs, mapped)) == want


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


def _peer_inputs(gen, n_chunks, device):
    refs = torch.randint(0, 4, (n_chunks,), generator=gen).to(torch.int32)
    counts = torch.where(torch.rand(n_chunks, generator=gen) < 0.6, refs,
                         torch.randint(0, 4, (n_chunks,), generator=gen).to(torch.int32))
    mapped = torch.randint(-(1 << 62), 1 << 62, ((n_chunks + 63) // 64,), generator=gen)
    return counts.to(device), refs.to(device), mapped.to(device)


def test_peer_combine_single_rank_equals_freeable_bitmap(cuda_device):
    from ekv_b200.releasable import PEER_FLAG_BYTES, PeerFreeableCombiner, freeable_bitmap

    gen = torch.Generator().manual_seed(21)
    n = 4099
    buf = torch.zeros(PEER_FLAG_BYTES + 2 * 8 * ((n + 63) // 64), dtype=torch.uint8, device=cuda_device)
    combiner = PeerFreeableCombiner(n, cuda_device, buffers=[buf.data_ptr()], rank=0, max_polls=1000)
    for _ in range(3):
        counts, refs, mapped = _peer_inputs(gen, n, cuda_device)
        assert torch.equal(combiner.combine(counts, refs, mapped), freeable_bitmap(counts, refs, mapped))
    assert not combiner.failed()
    # Tensors of the wrong size or type are refused before the launch.
    for bad in (dict(counts=counts[:-1]), dict(refs=refs.long()), dict(mapped_bits=mapped[:-1])):
        args = dict(counts=counts, refs=refs, mapped_bits=mapped) | bad
        with pytest.raises(ValueError, match="contiguous"):
            combiner.combine(**args)


def test_peer_combine_two_ranks_with_the_peer_already_arrived(cuda_device):
    """Rank 0 of two, the peer's flag and bitmap already in place (written from the host):
    one kernel, nothing to wait for but the flag, result = AND of both bitmaps."""
    from ekv_b200.releasable import PEER_FLAG_BYTES, PeerFreeableCombiner, freeable_bitmap

    gen = torch.Generator().manual_seed(22)
    n = 3000
    words = (n + 63) // 64
    size = PEER_FLAG_BYTES + 2 * 8 * words
    mine = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    peer = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    combiner = PeerFreeableCombiner(n, cuda_device, buffers=[mine.data_ptr(), peer.data_ptr()], rank=0,
                                    max_polls=100000)
    for epoch in (1, 2, 3):
        peer_bits = torch.randint(-(1 << 62), 1 << 62, (words,), generator=gen).to(cuda_device)
        slot = (epoch & 1) * words
        peer.view(torch.int64)[PEER_FLAG_BYTES // 8 + slot: PEER_FLAG_BYTES // 8 + slot + words] = peer_bits
        mine.view(torch.int32)[1] = epoch  # the peer (rank 1) has published this epoch
        torch.cuda.synchronize()
        counts, refs, mapped = _peer_inputs(gen, n, cuda_device)
        local = torch.empty(words, dtype=torch.int64, device=cuda_device)
        out = combiner.combine(counts, refs, mapped, local_out=local)
        torch.cuda.synchronize()
        assert torch.equal(local, freeable_bitmap(counts, refs, mapped))
        assert torch.equal(out, local & peer_bits)
        assert int(peer.view(torch.int32)[0]) == epoch  # our arrival flag landed in the peer's buffer
    assert not combiner.failed()


def test_peer_combine_wait_gives_up_with_a_status(cuda_device):
    """A peer that never arrives: the bounded wait runs out, the status word is set and
    the output is left untouched -- no hang, the context stays usable."""
    from ekv_b200.releasable import PEER_FLAG_BYTES, PeerFreeableCombiner

    n = 640
    size = PEER_FLAG_BYTES + 2 * 8 * 10
    mine = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    absent = torch.zeros(size, dtype=torch.uint8, device=cuda_device)
    combiner = PeerFreeableCombiner(n, cuda_device, buffers=[mine.data_ptr(), absent.data_ptr()], rank=0,
                                    max_polls=2000)
    out = torch.full((10,), 12345, dtype=torch.int64, device=cuda_device)
    bits = torch.full((10,), -1, dtype=torch.int64, device=cuda_device)
    combiner.combine(local_bits=bits, out=out)
    assert combiner.failed()
    assert (out == 12345).all()
    # The context is still usable: the next launch (the single-rank form) completes.
    alone = PeerFreeableCombiner(n, cuda_device, buffers=[mine.data_ptr()], rank=0, max_polls=10)
    assert torch.equal(alone.combine(local_bits=bits), bits)
    assert not alone.failed()


def _overflow_np(pages, planes, page_size, chunk_bytes, n_chunks):
    """(page, plane, chunk) hits outside [0, n_chunks) for non-negative pages."""
    total = 0
    pages = np.asarray(pages, dtype=np.int64)
    for first_chunk, row_bytes in planes:
        span = page_size * row_bytes
        lo = first_chunk + pages * span // chunk_bytes
        hi = first_chunk + (pages * span + span - 1) // chunk_bytes
        for page_lo, page_hi in zip(lo, hi):
            c = np.arange(page_lo, page_hi + 1)
            total += int(((c < 0) | (c >= n_chunks)).sum())
    return total


@pytest.mark.parametrize("n_chunks", [700, 70_000])
def test_counts_with_plane_groups_straddles_and_overflow(n_chunks, cuda_device):
    """Planes sharing a row size go through one grouped histogram (shared-memory tables),
    lone planes through the per-plane kernel; pages that straddle chunk boundaries and
    chunks past the table (counted in ``overflow``) give the same answers either way."""
    from ekv_b200.releasable import ChunkProjection

    gen = torch.Generator().manual_seed(n_chunks)
    chunk_bytes, page_size = 512, 3
    rows = [96] * 6 + [40, 40] + [1000]  # a group of 6, a group of 2, a lone plane
    planes = [(i * (n_chunks // 12), r) for i, r in enumerate(rows)]
    pages = torch.randperm(4000, generator=gen)[:1500] + 1
    projection = ChunkProjection(planes, page_size, chunk_bytes, n_chunks, cuda_device)
    got = projection.counts(pages.to(cuda_device))
    want = orl.chunk_counts_np(pages.numpy(), planes, page_size, chunk_bytes, n_chunks)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    want_overflow = _overflow_np(pages.numpy(), planes, page_size, chunk_bytes, n_chunks)
    assert int(projection.overflow.item()) == want_overflow
    if n_chunks == 700:
        assert want_overflow > 0  # the last planes run past the table


def test_grouped_counts_equal_the_sum_of_single_planes(cuda_device):
    """A group of planes (one shared histogram) counts exactly what its planes count one at
    a time through the per-plane kernel, overflow included -- also for negative page ids,
    which the grouped kernel hands to its inline per-plane path."""
    from ekv_b200.releasable import ChunkProjection

    gen = torch.Generator().manual_seed(8)
    n_chunks, chunk_bytes, page_size = 3000, 1024, 5
    planes = [(0, 200), (700, 200), (1500, 200), (2900, 200)]
    pages = torch.cat([torch.randint(-3000, 0, (200,), generator=gen), torch.randperm(6000, generator=gen)[:2000]])
    pages_dev = pages.to(cuda_device)
    joint = ChunkProjection(planes, page_size, chunk_bytes, n_chunks, cuda_device)
    got = joint.counts(pages_dev)
    total = torch.zeros(n_chunks, dtype=torch.int32, device=cuda_device)
    overflow = 0
    for plane in planes:
        single = ChunkProjection([plane], page_size, chunk_bytes, n_chunks, cuda_device)
        total += single.counts(pages_dev)
        overflow += int(single.overflow.item())
    assert torch.equal(got, total)
    assert int(joint.overflow.item()) == overflow and overflow > 0
