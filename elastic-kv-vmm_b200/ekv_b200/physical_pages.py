"""Physical page ownership projected onto chunk-aligned K/V planes (R4).

``PhysicalPages`` keeps the API and bookkeeping of the reference's
adaptive_sparse/minimax_vmm.py:20-98 (page -> chunk projection, chunk
reference counts, trim of mapped-but-unreferenced chunks) so the allocator
hook and the demotion planner can use it unchanged.  On top of that it exports
its state as device arrays -- per-chunk reference counts and the mapped-chunk
bitmap -- which are the inputs of the freeable-bitmap kernel.
"""

from __future__ import annotations

from time import perf_counter_ns

import torch

CHUNK_BYTES = 2 << 20


class PhysicalPages:
    """Pages of ``page_size`` token slots living in every plane.

    ``planes`` lists ``(first_chunk, row_bytes)`` per plane (K and V of every
    layer, each plane starting on a chunk boundary).  Page 0 is the sink: it
    is owned from the start and its chunks are mapped at construction.
    """

    def __init__(self, backing, page_size, page_count, planes, synchronize,
                 chunk_bytes=CHUNK_BYTES, fast_decode=False):
        self.backing = backing
        self.page_size = page_size
        self.page_count = page_count
        self.planes = planes
        self.synchronize = synchronize
        self.chunk_bytes = chunk_bytes
        self.fast_decode = fast_decode
        self.trim_sync_ns = 0
        self.fast_no_new_page = 0
        self.decode_new_page = 0
        self._projection_cache = {} if fast_decode else None
        self.pages = {0}
        self.refs = dict.fromkeys(self.chunks(0), 1)
        self.backing.ensure(self.refs)

    def chunks(self, page):
        """Every chunk holding a byte of ``page`` in any plane."""
        cache = self._projection_cache
        if cache is not None and page in cache:
            return cache[page]
        span_start = page * self.page_size
        found = set()
        for first_chunk, row_bytes in self.planes:
            begin = span_start * row_bytes
            last = begin + self.page_size * row_bytes - 1
            found.update(range(first_chunk + begin // self.chunk_bytes,
                               first_chunk + last // self.chunk_bytes + 1))
        result = frozenset(found)
        if cache is not None:
            cache[page] = result
        return result

    def acquire(self, pages):
        """Own ``pages``; map the chunks of pages not owned yet first."""
        pages = set(pages)
        if any(page <= 0 or page > self.page_count for page in pages):
            raise ValueError("invalid physical page")
        new = pages - self.pages
        projected = [self.chunks(page) for page in new]
        if projected:
            self.backing.ensure(set().union(*projected))
        for chunks in projected:
            for chunk in chunks:
                self.refs[chunk] = self.refs.get(chunk, 0) + 1
        self.pages.update(new)

    def validate_release(self, pages):
        if 0 in pages or not pages <= self.pages:
            raise RuntimeError("invalid or duplicate physical free")

    def release(self, pages):
        self.validate_release(pages)
        for page in pages:
            for chunk in self.chunks(page):
                left = self.refs[chunk] - 1
                if left:
                    self.refs[chunk] = left
                else:
                    del self.refs[chunk]
        self.pages.difference_update(pages)

    def clear(self):
        self.release(self.pages - {0})

    def stats(self):
        idle = self.backing.mapped_chunks - self.refs.keys()
        return {"backed_bytes": self.backing.backed_bytes,
                "reclaimable_bytes": len(idle) * self.chunk_bytes,
                "owned_pages": len(self.pages) - 1,
                "trim_sync_ns": self.trim_sync_ns,
                "fast_no_new_page": self.fast_no_new_page,
                "decode_new_page": self.decode_new_page}

    def trim_quiescent(self):
        """Unmap chunks no page references.  Call only with scheduling paused."""
        idle = self.backing.mapped_chunks - self.refs.keys()
        if not idle:
            return 0
        started = perf_counter_ns()
        self.synchronize()
        self.trim_sync_ns += perf_counter_ns() - started
        return self.backing.reclaim(idle, synchronize=False) * self.chunk_bytes

    # ------------------------------------------------------------ device export

    @property
    def n_chunks(self):
        """Chunks spanned by the planes (one past the last chunk of the last plane)."""
        last_page = self.page_count
        return 1 + max(first + ((last_page + 1) * self.page_size * row - 1) // self.chunk_bytes
                       for first, row in self.planes)

    def device_refs(self, device, n_chunks=None):
        """int32 [n_chunks] reference counts on ``device`` (0 = unreferenced)."""
        n_chunks = n_chunks or self.n_chunks
        refs = torch.zeros(n_chunks, dtype=torch.int32)
        if self.refs:
            ids = torch.tensor(list(self.refs.keys()), dtype=torch.int64)
            refs[ids] = torch.tensor(list(self.refs.values()), dtype=torch.int32)
        return refs.to(device)

    def device_mapped_bits(self, device, n_chunks=None):
        """Mapped-chunk bitmap as int64 words on ``device``."""
        from .releasable import chunks_to_bitmap

        n_chunks = n_chunks or self.n_chunks
        return chunks_to_bitmap(self.backing.mapped_chunks, n_chunks, device)
