"""Physical page ownership projected onto chunk-aligned K/V planes (R4).

The reference tracks which 2 MiB chunks of the VMM pool hold a byte of some
owned physical page with Python sets and a ``{chunk: refs}`` dict
(adaptive_sparse/minimax_vmm.py:20-98).  Its callers -- the allocator hook, the
demotion planner (adaptive_sparse/migration.py:36-39), the releasable-chunk
math (adaptive_sparse/scheduler_budget.py:151-189) and the logical-shadow page
mask (adaptive_sparse/logical_shadow.py:235) -- read ``chunks(page)``,
``refs`` as a mapping, ``pages`` as a set, ``acquire`` / ``release`` /
``trim_quiescent`` / ``stats`` and a few counters; this class keeps exactly that
surface.

The state underneath is laid out for the device kernels instead:

* ``_count``: one int32 reference count per chunk of the pool, a dense array
  (a 180 GB pool is ~90k chunks), so the freeable-bitmap kernel's input is a
  single host-to-device copy of it, not a dict conversion;
* ``_owned``: one bool per physical page;
* the projection page -> chunks is computed for a whole batch of pages at once
  with numpy, per group of planes that share a row size (every K and V plane of
  a model), instead of a Python loop over planes per page.

``refs`` and ``pages`` are read-only views over those arrays.
"""

from __future__ import annotations

import operator
from collections.abc import Mapping, Set
from time import perf_counter_ns

import numpy as np
import torch

CHUNK_BYTES = 2 << 20


class _ChunkRefs(Mapping):
    """``{chunk: references}`` over the dense count array (only referenced chunks)."""

    __slots__ = ("_owner",)

    def __init__(self, owner):
        self._owner = owner

    def __getitem__(self, chunk):
        count = self._owner._count
        try:
            index = operator.index(chunk)
        except TypeError:
            raise KeyError(chunk) from None
        if 0 <= index < count.shape[0] and count[index]:
            return int(count[index])
        raise KeyError(chunk)

    def __contains__(self, chunk):
        try:
            self[chunk]
        except KeyError:
            return False
        return True

    def __iter__(self):
        return iter(np.flatnonzero(self._owner._count).tolist())

    def __len__(self):
        return self._owner._live

    def __repr__(self):
        return repr(dict(self))


class _OwnedPages(Set):
    """The set of owned physical pages, a view over the ownership bitmap."""

    __slots__ = ("_owner",)

    def __init__(self, owner):
        self._owner = owner

    @classmethod
    def _from_iterable(cls, values):
        return set(values)

    def __contains__(self, page):
        owned = self._owner._owned
        return isinstance(page, (int, np.integer)) and 0 <= page < owned.shape[0] and bool(owned[page])

    def __iter__(self):
        return iter(np.flatnonzero(self._owner._owned).tolist())

    def __len__(self):
        return self._owner._n_owned

    def __repr__(self):
        return repr(set(self))


class PhysicalPages:
    """Pages of ``page_size`` token slots living in every plane.

    ``planes`` lists ``(first_chunk, row_bytes)`` per plane (K and V of every
    layer, each plane starting on a chunk boundary).  Page 0 is the sink: owned
    from the start, its chunks mapped at construction.  Page ids run from 1 to
    ``page_count``.
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
        self._cache = {} if fast_decode else None
        groups = {}
        for first, row_bytes in planes:
            groups.setdefault(int(row_bytes), []).append(int(first))
        # (bytes of one page in a plane of the group, first chunk of each plane)
        self._groups = [(page_size * row_bytes, np.asarray(firsts, dtype=np.int64))
                        for row_bytes, firsts in groups.items()]
        self._count = np.zeros(self.n_chunks, dtype=np.int32)
        self._owned = np.zeros(page_count + 1, dtype=bool)
        self._n_owned = 0
        self._live = 0
        self.refs = _ChunkRefs(self)
        self.pages = _OwnedPages(self)
        sink = np.zeros(1, dtype=np.int64)
        self._add(sink, +1)
        self.backing.ensure(set(self.refs))

    # ------------------------------------------------------------ projection

    @property
    def n_chunks(self):
        """Chunks spanned by the planes (one past the last chunk of the last plane)."""
        last_page = self.page_count
        return 1 + max(first + ((last_page + 1) * self.page_size * row - 1) // self.chunk_bytes
                       for first, row in self.planes)

    def _project(self, pages):
        """Distinct (page index, chunk) pairs of ``pages`` (int64 array) over all planes.

        Returns two int64 arrays of equal length: the position of the page in
        ``pages`` and one chunk it touches, every pair once.
        """
        owners, chunks = [], []
        for span, firsts in self._groups:
            begin = pages * span
            lo = begin // self.chunk_bytes
            hi = (begin + span - 1) // self.chunk_bytes
            width = int((hi - lo).max()) + 1 if pages.size else 0
            for step in range(width):
                inside = lo + step <= hi                               # [pages]
                idx = np.flatnonzero(inside)
                ids = (firsts[None, :] + (lo[idx] + step)[:, None])    # [pages', planes]
                owners.append(np.repeat(idx, firsts.size))
                chunks.append(ids.reshape(-1))
        if not owners:
            empty = np.zeros(0, dtype=np.int64)
            return empty, empty
        owner = np.concatenate(owners)
        chunk = np.concatenate(chunks)
        # A chunk reached twice by one page (overlapping planes) counts once.
        stride = int(chunk.max()) + 1
        key = np.unique(owner * stride + chunk)
        return key // stride, key % stride

    def chunks(self, page):
        """Every chunk holding a byte of ``page`` in any plane."""
        cache = self._cache
        if cache is not None:
            hit = cache.get(page)
            if hit is not None:
                return hit
        _, chunk = self._project(np.asarray([page], dtype=np.int64))
        result = frozenset(chunk.tolist())
        if cache is not None:
            cache[page] = result
        return result

    def _add(self, pages, sign):
        """Add ``sign`` to the count of every chunk of every page; mark ownership."""
        _, chunk = self._project(pages)
        if chunk.size:
            touched, times = np.unique(chunk, return_counts=True)
            before = self._count[touched] != 0
            self._count[touched] += (sign * times).astype(np.int32)
            after = self._count[touched] != 0
            self._live += int(after.sum()) - int(before.sum())
        self._owned[pages] = sign > 0
        self._n_owned += sign * int(pages.size)

    # ------------------------------------------------------------ ownership

    def acquire(self, pages):
        """Own ``pages``; map the chunks of pages not owned yet first."""
        wanted = np.unique(np.fromiter((int(p) for p in pages), dtype=np.int64))
        if wanted.size and (wanted[0] <= 0 or wanted[-1] > self.page_count):
            raise ValueError("invalid physical page")
        fresh = wanted[~self._owned[wanted]]
        if not fresh.size:
            return
        _, chunk = self._project(fresh)
        self.backing.ensure(set(np.unique(chunk).tolist()))
        self._add(fresh, +1)

    def _owned_array(self, pages):
        """``pages`` as a sorted int64 array; RuntimeError unless every page is owned and not the sink."""
        array = np.unique(np.fromiter((int(p) for p in pages), dtype=np.int64))
        if array.size and (array[0] <= 0 or array[-1] > self.page_count or not self._owned[array].all()):
            raise RuntimeError("invalid or duplicate physical free")
        return array

    def validate_release(self, pages):
        self._owned_array(pages)

    def release(self, pages):
        array = self._owned_array(pages)
        if array.size:
            self._add(array, -1)

    def clear(self):
        owned = np.flatnonzero(self._owned)
        owned = owned[owned != 0]
        if owned.size:
            self._add(owned, -1)

    # ------------------------------------------------------------ reclaim

    def _idle(self):
        """Mapped chunks that no owned page references."""
        mapped = np.fromiter(self.backing.mapped_chunks, dtype=np.int64)
        if not mapped.size:
            return set()
        inside = mapped < self._count.shape[0]
        idle = mapped[~inside]
        idle = np.concatenate([idle, mapped[inside][self._count[mapped[inside]] == 0]])
        return set(idle.tolist())

    def stats(self):
        return {"backed_bytes": self.backing.backed_bytes,
                "reclaimable_bytes": len(self._idle()) * self.chunk_bytes,
                "owned_pages": self._n_owned - 1,
                "trim_sync_ns": self.trim_sync_ns,
                "fast_no_new_page": self.fast_no_new_page,
                "decode_new_page": self.decode_new_page}

    def trim_quiescent(self):
        """Unmap chunks no page references.  Call only with scheduling paused."""
        idle = self._idle()
        if not idle:
            return 0
        started = perf_counter_ns()
        self.synchronize()
        self.trim_sync_ns += perf_counter_ns() - started
        return self.backing.reclaim(idle, synchronize=False) * self.chunk_bytes

    # ------------------------------------------------------------ device export

    def device_refs(self, device, n_chunks=None):
        """int32 [n_chunks] reference counts on ``device`` (0 = unreferenced)."""
        n_chunks = n_chunks or self._count.shape[0]
        refs = np.zeros(n_chunks, dtype=np.int32)
        n = min(n_chunks, self._count.shape[0])
        refs[:n] = self._count[:n]
        return torch.from_numpy(refs).to(device)

    def device_mapped_bits(self, device, n_chunks=None):
        """Mapped-chunk bitmap as int64 words on ``device``."""
        from .releasable import chunks_to_bitmap

        n_chunks = n_chunks or self.n_chunks
        return chunks_to_bitmap(self.backing.mapped_chunks, n_chunks, device)
