"""Freeable-chunk bitmaps and their cross-rank AND (R6).

The reference decides which chunks a demotion would release with Python sets
(_chunk_release_counts / _releasable_counts / _releasable_pair /
_releasable_group, adaptive_sparse/scheduler_budget.py:151-189) and agrees
across tensor-parallel ranks by pickling per-rank candidate maps through
``all_gather_object`` and intersecting them (exchange(),
scheduler_budget.py:1447-1452; rank_demotions, runtime_value.py:180-185).

Here the same decision is a bitmap on the device: chunk c is freeable by a
set of candidate pages iff every page reference to c belongs to the set
(count == refs[c] > 0) and c is mapped.  The per-rank bitmaps (one bit per
chunk, 512 B for 4096 chunks) are combined with one NCCL all-gather and an AND
kernel, giving the chunks freeable on EVERY rank.  NCCL has no bitwise-AND
reduction, hence all-gather + AND rather than all-reduce.
"""

from __future__ import annotations

from typing import Callable, Iterable

import torch

from ._lib import MAX_PLANES, call, i64_array, index_esize, require_cuda, stream_handle, u64_array


def words_for(n_chunks: int) -> int:
    return (n_chunks + 63) // 64


def chunks_to_bitmap(chunks: Iterable[int], n_chunks: int, device) -> torch.Tensor:
    """Bitmap (int64 words, chunk c at word c // 64 bit c % 64) of ``chunks``."""
    words = torch.zeros(words_for(n_chunks), dtype=torch.int64)
    ids = sorted(int(c) for c in chunks)
    if ids:
        if ids[0] < 0 or ids[-1] >= n_chunks:
            raise ValueError("chunk id outside the bitmap")
        ids_t = torch.tensor(ids, dtype=torch.int64)
        bits = torch.ones(len(ids), dtype=torch.int64) << (ids_t % 64)
        words.index_put_((ids_t // 64,), bits, accumulate=True)
    return words.to(device)


def bitmap_to_chunks(bitmap: torch.Tensor) -> frozenset:
    """Set of chunk ids whose bit is set."""
    words = bitmap.detach().to("cpu", torch.int64)
    shifts = torch.arange(64, dtype=torch.int64)
    bits = ((words[:, None] >> shifts) & 1).bool()
    return frozenset(torch.nonzero(bits.flatten()).flatten().tolist())


class ChunkProjection:
    """Plane geometry for the page -> chunk histogram kernel.

    ``planes`` is ``[(first_chunk, row_bytes), ...]`` as in PhysicalPages.
    """

    def __init__(self, planes, page_size: int, chunk_bytes: int, n_chunks: int, device):
        planes = [(int(c), int(r)) for c, r in planes]
        if not 1 <= len(planes) <= MAX_PLANES:
            raise ValueError("plane count outside [1, EKV_MAX_PLANES]")
        self.planes = planes
        self.page_size = int(page_size)
        self.chunk_bytes = int(chunk_bytes)
        self.n_chunks = int(n_chunks)
        self.device = torch.device(device)
        self._first = i64_array(c for c, _ in planes)
        self._rows = i64_array(r for _, r in planes)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=self.device)

    @classmethod
    def of(cls, tracker, device, n_chunks=None):
        return cls(tracker.planes, tracker.page_size, tracker.chunk_bytes,
                   n_chunks or tracker.n_chunks, device)

    def counts(self, pages: torch.Tensor, *, out: torch.Tensor | None = None,
               accumulate: bool = False) -> torch.Tensor:
        """int32 [n_chunks]: how many of ``pages`` (distinct) cover each chunk."""
        require_cuda(dict(pages=pages), self.device)
        if pages.dim() != 1 or not pages.is_contiguous():
            raise ValueError("pages must be a contiguous 1-D tensor")
        if out is None:
            out = torch.empty(self.n_chunks, dtype=torch.int32, device=self.device)
            accumulate = False
        elif out.dtype != torch.int32 or out.numel() != self.n_chunks or not out.is_contiguous():
            raise ValueError("out must be a contiguous int32 tensor of n_chunks entries")
        call("ekv_chunk_counts", pages.data_ptr(), index_esize(pages, "pages"), pages.numel(),
             self._first, self._rows, len(self.planes), self.page_size, self.chunk_bytes,
             out.data_ptr(), self.n_chunks, int(accumulate), self.overflow.data_ptr(),
             self.device.index, stream_handle(self.device))
        return out


def freeable_bitmap(counts: torch.Tensor, refs: torch.Tensor, mapped_bits: torch.Tensor, *,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Bitmap of chunks with ``counts == refs > 0`` that are mapped."""
    device = require_cuda(dict(counts=counts, refs=refs, mapped_bits=mapped_bits))
    n_chunks = counts.numel()
    if counts.dtype != torch.int32 or refs.dtype != torch.int32 or refs.numel() != n_chunks:
        raise ValueError("counts and refs must be int32 tensors of equal length")
    if mapped_bits.dtype != torch.int64 or mapped_bits.numel() != words_for(n_chunks):
        raise ValueError("mapped_bits must hold ceil(n_chunks / 64) int64 words")
    if out is None:
        out = torch.empty(words_for(n_chunks), dtype=torch.int64, device=device)
    call("ekv_freeable_bitmap", counts.data_ptr(), refs.data_ptr(), mapped_bits.data_ptr(),
         n_chunks, out.data_ptr(), device.index, stream_handle(device))
    return out


def bitmap_and(gathered: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """AND over the rows of ``gathered`` [ranks, words] (int64 words)."""
    device = require_cuda(dict(gathered=gathered))
    if gathered.dim() != 2 or gathered.dtype != torch.int64 or not gathered.is_contiguous():
        raise ValueError("gathered must be a contiguous [ranks, words] int64 tensor")
    ranks, words = gathered.shape
    if out is None:
        out = torch.empty(words, dtype=torch.int64, device=device)
    call("ekv_bitmap_and", gathered.data_ptr(), ranks, words, out.data_ptr(), device.index,
         stream_handle(device))
    return out


def combine_freeable(bitmap: torch.Tensor, group=None, *,
                     and_fn: Callable[[torch.Tensor], torch.Tensor] | None = None) -> torch.Tensor:
    """Chunks freeable on every rank of ``group``: all-gather + AND.

    The all-gather goes through torch.distributed (NCCL over NVLink for CUDA
    tensors).  ``and_fn`` replaces the AND kernel; it exists so the exchange
    logic can be exercised on CPU process groups in tests.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return bitmap.clone()
    flat = torch.empty(world * bitmap.numel(), dtype=bitmap.dtype, device=bitmap.device)
    dist.all_gather_into_tensor(flat, bitmap.contiguous().view(-1), group=group)
    gathered = flat.view(world, bitmap.numel())
    if and_fn is not None:
        return and_fn(gathered)
    return bitmap_and(gathered)


PEER_FLAG_BYTES = 256  # 64 uint32 arrival flags at the head of each rank's buffer


class PeerFreeableCombiner:
    """Freeable bitmap + cross-rank AND in one kernel over peer (symmetric) memory.

    Every rank of ``group`` builds one combiner (a collective: it allocates and
    exchanges the peer buffers) and then calls ``combine`` in the same order.
    ``buffers`` may instead be given directly as a list of peer-visible device
    addresses (rank order) with ``rank``; that form serves tests.
    ``max_polls`` bounds each wait for a peer (~64 ns per poll).
    """

    def __init__(self, n_chunks: int, device, group=None, *, buffers=None, rank=None,
                 max_polls: int = 1 << 24):
        self.n_chunks = int(n_chunks)
        self.n_words = words_for(self.n_chunks)
        self.device = torch.device(device)
        self.max_polls = int(max_polls)
        self.epoch = 0
        self._keep = None
        if buffers is None:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm_mem

            nbytes = PEER_FLAG_BYTES + 2 * 8 * self.n_words
            local = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            local.zero_()
            handle = symm_mem.rendezvous(local, group if group is not None else dist.group.WORLD)
            handle.barrier()
            buffers = list(handle.buffer_ptrs)
            rank = handle.rank
            self._keep = (local, handle)
        if rank is None:
            raise ValueError("rank is required with explicit buffers")
        self.rank = int(rank)
        self.n_ranks = len(buffers)
        self._buffers = u64_array(buffers)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def combine(self, counts=None, refs=None, mapped_bits=None, *, local_bits=None, out=None, local_out=None):
        """AND over the ranks of every rank's freeable bitmap; returns ``out`` (int64 words).

        The local bitmap is built from ``counts`` / ``refs`` (int32, n_chunks) and
        ``mapped_bits`` (int64 words), or taken from ``local_bits`` (int64 words).
        """
        if local_bits is None and (counts is None or refs is None or mapped_bits is None):
            raise ValueError("give counts, refs and mapped_bits, or local_bits")
        if out is None:
            out = torch.empty(self.n_words, dtype=torch.int64, device=self.device)
        expected = dict(counts=(torch.int32, self.n_chunks), refs=(torch.int32, self.n_chunks),
                        mapped_bits=(torch.int64, self.n_words), local_bits=(torch.int64, self.n_words),
                        out=(torch.int64, self.n_words), local_out=(torch.int64, self.n_words))
        given = dict(counts=counts, refs=refs, mapped_bits=mapped_bits, local_bits=local_bits, out=out,
                     local_out=local_out)
        require_cuda(given, self.device)
        for name, tensor in given.items():
            if tensor is None:
                continue
            dtype, numel = expected[name]
            if tensor.dtype != dtype or tensor.numel() != numel or not tensor.is_contiguous():
                raise ValueError(f"{name} must be a contiguous {dtype} tensor of {numel} elements")
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        call("ekv_freeable_and_peers",
             None if counts is None else counts.data_ptr(), None if refs is None else refs.data_ptr(),
             None if mapped_bits is None else mapped_bits.data_ptr(),
             None if local_bits is None else local_bits.data_ptr(), self.n_chunks, self._buffers,
             self.n_ranks, self.rank, self.epoch, self.max_polls, out.data_ptr(),
             None if local_out is None else local_out.data_ptr(), self.status.data_ptr(),
             self.device.index, stream_handle(self.device))
        return out

    def failed(self) -> bool:
        """True once a wait for a peer ran out (synchronizes with the device)."""
        return bool(self.status.item())


class FreeableChunks:
    """Device-side releasable-chunk queries for one PhysicalPages tracker.

    Mirrors what the planner asks of the reference's set helpers: the chunks a
    candidate page set (or the union of several candidates' pages) would free,
    optionally agreed across tensor-parallel ranks.
    """

    def __init__(self, tracker, device, group=None):
        self.tracker = tracker
        self.device = torch.device(device)
        self.group = group
        self.projection = ChunkProjection.of(tracker, self.device)
        self.refresh()

    def refresh(self):
        """Re-export refs and the mapped bitmap after acquire/release/trim."""
        n = self.projection.n_chunks
        self.refs = self.tracker.device_refs(self.device, n)
        self.mapped = self.tracker.device_mapped_bits(self.device, n)

    def _pages(self, pages) -> torch.Tensor:
        if isinstance(pages, torch.Tensor):
            tensor = pages.to(self.device, torch.int64)
        else:
            tensor = torch.tensor(sorted({int(p) for p in pages}), dtype=torch.int64,
                                  device=self.device)
        return torch.unique(tensor)  # union semantics for shared pages

    def bitmap(self, pages, *, joint: bool = False) -> torch.Tensor:
        counts = self.projection.counts(self._pages(pages))
        local = freeable_bitmap(counts, self.refs, self.mapped)
        return combine_freeable(local, self.group) if joint else local

    def releasable(self, pages, *, joint: bool = False) -> frozenset:
        """Chunks released by demoting ``pages`` (on every rank if ``joint``)."""
        return bitmap_to_chunks(self.bitmap(pages, joint=joint))

    def releasable_group(self, candidates, *, joint: bool = False) -> frozenset:
        """Chunks released by demoting several candidates' page sets together."""
        union = set()
        for pages in candidates:
            union.update(int(p) for p in pages)
        return self.releasable(union, joint=joint)
