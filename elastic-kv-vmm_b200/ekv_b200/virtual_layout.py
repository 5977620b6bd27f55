"""Fixed-position, chunk-aligned per-request KV layout.

Same field names, validation and byte arithmetic as the reference's
experimental/virtual_layout.py:13-61 (the gather kernel derives its direct-mode
strides from it): chunk 0 is the always-mapped sink, request ``r`` owns the
chunk-aligned region starting at ``chunk_bytes + r * request_bytes``, and token
``t`` of request ``r`` sits ``t * row_bytes`` into that region.
"""

from __future__ import annotations

from dataclasses import dataclass


def _check_int(name, value, low, high=None):
    # bool is an int subclass; the layout accepts only genuine ints.
    if type(value) is not int:
        raise TypeError(f"{name} must be an integer")
    if value < low or (high is not None and value > high):
        raise ValueError(f"{name} outside supported range")


@dataclass(frozen=True)
class VirtualKVLayout:
    max_requests: int
    max_tokens: int
    row_elements: int
    itemsize: int = 2
    chunk_bytes: int = 2 << 20

    def __post_init__(self):
        for field in ("max_requests", "max_tokens", "row_elements", "itemsize", "chunk_bytes"):
            _check_int(field, getattr(self, field), 1)

    @property
    def row_bytes(self):
        return self.row_elements * self.itemsize

    @property
    def request_bytes(self):
        """Bytes of one request region, rounded up to whole chunks."""
        chunks = -(-(self.max_tokens * self.row_bytes) // self.chunk_bytes)
        return chunks * self.chunk_bytes

    @property
    def capacity_bytes(self):
        return self.chunk_bytes + self.max_requests * self.request_bytes

    def request_offset(self, req):
        _check_int("request index", req, 0, self.max_requests - 1)
        return self.chunk_bytes + req * self.request_bytes

    def token_offset(self, req, token):
        _check_int("token position", token, 0, self.max_tokens - 1)
        return self.request_offset(req) + token * self.row_bytes

    def _chunks_of(self, start, size):
        if not size:
            return range(0)
        return range(start // self.chunk_bytes, (start + size - 1) // self.chunk_bytes + 1)

    def prefix_chunks(self, req, length):
        """Chunks under the first ``length`` rows of request ``req``."""
        _check_int("prefix length", length, 0, self.max_tokens)
        return frozenset(self._chunks_of(self.request_offset(req), length * self.row_bytes))

    def selected_chunks(self, req, positions):
        """Chunks touched by the rows at ``positions`` of request ``req``."""
        self.request_offset(req)
        chunks = set()
        for token in positions:
            chunks.update(self._chunks_of(self.token_offset(req, token), self.row_bytes))
        return frozenset(chunks)
