"""Single-threaded VMM arena of fixed-position request regions.

Same call sequence and failure behaviour as the reference's
experimental/resident_arena.py:4-92: the sink chunk is committed at
construction, ``reserve`` grows a request's mapped prefix, ``resize_quiescent``
shrinks it (device sync, then reclaim of the dropped tail chunks), and any
backing failure makes the arena refuse further use.
"""

from __future__ import annotations


class VmmResidentArena:
    """Views are borrowed: drop tail views before shrinking and all views
    before closing.  Newly exposed rows must be written before use, since a
    retained chunk can still hold bytes of a discarded tail.
    """

    def __init__(self, layout, device=0, backing_factory=None, *, synchronize=None):
        if layout.chunk_bytes % layout.itemsize:
            raise ValueError("chunk size must align to the element size")
        if backing_factory is None:
            from .backing import Backing

            backing_factory = Backing
        self.layout = layout
        self.backing = backing_factory(layout.capacity_bytes, chunk_bytes=layout.chunk_bytes,
                                       device=device)
        if synchronize is None:
            def synchronize():
                import torch

                torch.cuda.synchronize(self.backing.device)
        self._synchronize = synchronize
        self._lengths = [0] * layout.max_requests
        self._closed = False
        self._failed = False
        self.backing.ensure({0})

    def _usable(self):
        if self._closed or self._failed:
            raise RuntimeError("arena is closed or has encountered a backing error")

    def reserve(self, req, length):
        """Grow the mapped prefix of ``req`` to ``length`` rows, keeping its rows."""
        self._usable()
        wanted = self.layout.prefix_chunks(req, length)
        current = self._lengths[req]
        if length <= current:
            return
        missing = wanted - self.layout.prefix_chunks(req, current)
        if missing:
            try:
                self.backing.ensure(missing)
            except Exception:
                self._failed = True
                raise
        self._lengths[req] = length

    def resize_quiescent(self, req, length):
        """Resize a prefix; shrinking discards the tail rows."""
        self._usable()
        wanted = self.layout.prefix_chunks(req, length)
        current = self._lengths[req]
        if length >= current:
            self.reserve(req, length)
            return
        dropped = self.layout.prefix_chunks(req, current) - wanted
        try:
            self._synchronize()
            if dropped:
                self.backing.reclaim(dropped, synchronize=False)
        except Exception:
            self._failed = True
            raise
        self._lengths[req] = length

    def row_view(self, req, length, dtype):
        """Borrow a (length, row_elements) tensor over the mapped prefix."""
        self._usable()
        self.layout.prefix_chunks(req, length)
        if length > self._lengths[req]:
            raise ValueError("requested view exceeds the committed prefix")
        if dtype.itemsize != self.layout.itemsize:
            raise ValueError("dtype item size does not match the layout")
        start = self.layout.request_offset(req)
        return (self.backing.raw.narrow(0, start, length * self.layout.row_bytes)
                .view(dtype).reshape(length, self.layout.row_elements))

    def close(self):
        """Synchronize and release the reservation once every view is gone."""
        if self._closed:
            return
        try:
            self._synchronize()
            self.backing.close()
        except Exception:
            self._failed = True
            raise
        self._closed = True
