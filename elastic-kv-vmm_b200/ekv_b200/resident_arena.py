"""VMM arena of fixed-position request regions (the pool under the direct gather).

Interface of the reference's experimental/resident_arena.py:4-92
(``VmmResidentArena(layout, device, backing_factory, synchronize=...)``,
``reserve``, ``resize_quiescent``, ``row_view``, ``close``) and its contract:
the sink chunk is committed at construction, a growing prefix keeps its rows,
a shrinking one is reclaimed only after a device synchronize, and any backing
failure stops the arena for good.  The backing sees the same calls in the same
order, so code written against the reference's arena (and its mock-based test,
tests/test_virtual_layout.py:41-88) behaves the same.

Bookkeeping here is extent arithmetic rather than set algebra: every request
region of a ``VirtualKVLayout`` starts on a chunk boundary, so the mapped part
of a request is always the contiguous chunk range
``[first_chunk(r), first_chunk(r) + ceil(rows * row_bytes / chunk_bytes))``.
The arena keeps one committed row count per request and derives the chunks to
map or unmap from the old and new extents.
"""

from __future__ import annotations

from contextlib import contextmanager

_OPEN, _FAILED, _CLOSED = "open", "failed", "closed"


class VmmResidentArena:
    """Views are borrowed: drop tail views before shrinking and all views
    before closing.  Rows exposed by growing must be written before they are
    read: a chunk kept across a shrink can still hold bytes of the old tail.
    Single-threaded, like the backing it owns.
    """

    def __init__(self, layout, device=0, backing_factory=None, *, synchronize=None):
        if layout.chunk_bytes % layout.itemsize:
            raise ValueError("chunk size must align to the element size")
        if backing_factory is None:
            from .backing import Backing as backing_factory
        self.layout = layout
        self.backing = backing_factory(layout.capacity_bytes, chunk_bytes=layout.chunk_bytes, device=device)
        self._synchronize = synchronize or self._device_synchronize
        self._rows = [0] * layout.max_requests   # committed rows per request
        self._state = _OPEN
        self.backing.ensure({0})

    def _device_synchronize(self):
        import torch

        torch.cuda.synchronize(self.backing.device)

    # ------------------------------------------------------------ helpers

    @property
    def _lengths(self):
        """Committed rows per request (read-only copy)."""
        return list(self._rows)

    def _require_open(self):
        if self._state != _OPEN:
            raise RuntimeError("arena is closed or has encountered a backing error")

    @contextmanager
    def _fail_stop(self):
        """Any exception from the backing leaves the arena unusable."""
        try:
            yield
        except BaseException:
            self._state = _FAILED
            raise

    def _extent_chunks(self, req, rows):
        """Chunk range holding the first ``rows`` rows of request ``req`` (validates both)."""
        layout = self.layout
        if type(rows) is not int:
            raise TypeError("prefix length must be an integer")
        if not 0 <= rows <= layout.max_tokens:
            raise ValueError("prefix length outside supported range")
        first = layout.request_offset(req) // layout.chunk_bytes
        return range(first, first + -(-rows * layout.row_bytes // layout.chunk_bytes))

    # ------------------------------------------------------------ extent changes

    def reserve(self, req, length):
        """Grow the mapped prefix of ``req`` to ``length`` rows, keeping its rows."""
        self._require_open()
        wanted = self._extent_chunks(req, length)
        held = self._rows[req]
        if length <= held:
            return
        have = self._extent_chunks(req, held)
        grow = frozenset(range(have.stop, wanted.stop))
        if grow:
            with self._fail_stop():
                self.backing.ensure(grow)
        self._rows[req] = length

    def resize_quiescent(self, req, length):
        """Set the prefix of ``req`` to ``length`` rows; shrinking discards the tail."""
        self._require_open()
        wanted = self._extent_chunks(req, length)
        held = self._rows[req]
        if length >= held:
            self.reserve(req, length)
            return
        have = self._extent_chunks(req, held)
        shrink = frozenset(range(wanted.stop, have.stop))
        with self._fail_stop():
            self._synchronize()
            if shrink:
                self.backing.reclaim(shrink, synchronize=False)
        self._rows[req] = length

    # ------------------------------------------------------------ access

    def row_view(self, req, length, dtype):
        """Borrow a (length, row_elements) tensor over the committed prefix."""
        self._require_open()
        self._extent_chunks(req, length)
        if length > self._rows[req]:
            raise ValueError("requested view exceeds the committed prefix")
        layout = self.layout
        if dtype.itemsize != layout.itemsize:
            raise ValueError("dtype item size does not match the layout")
        return (self.backing.raw.narrow(0, layout.request_offset(req), length * layout.row_bytes)
                .view(dtype).reshape(length, layout.row_elements))

    def close(self):
        """Synchronize and release the reservation once every view is gone."""
        if self._state == _CLOSED:
            return
        with self._fail_stop():
            self._synchronize()
            self.backing.close()
        self._state = _CLOSED
