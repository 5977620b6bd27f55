"""Chunked CUDA VMM backing with a stable tensor view (the pool under the gather).

``Backing`` keeps the constructor, methods and error behaviour the data path
relies on from the reference's elastic_kv/backing.py:114-545 (``ensure``,
``precommit``, ``reclaim``, ``close``, ``raw``, ``mapped_chunks``,
``backed_bytes``, ``metrics``), over the ev_* entry points of libekv_b200.so.
The multi-tenant admission broker of the reference is not part of this data
path and is not implemented.  ``raw`` is built through
``__cuda_array_interface__`` instead of CuPy/DLPack.
"""

from __future__ import annotations

import ctypes as ct
import operator
import os
import time
import weakref

import torch

from ._lib import library as load_library

DEFAULT_CHUNK_BYTES = 2 << 20
_INVALID = (1 << 64) - 1


class _DeviceBytes:
    """Minimal CUDA array interface over an externally owned byte range."""

    def __init__(self, address: int, nbytes: int, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (address, False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


def _close_handle(lib, handle_box):
    handle = handle_box[0]
    if handle:
        handle_box[0] = None
        lib.ev_close(handle)


class Backing:
    """Single-thread owner of one CUDA virtual reservation.

    A tensor from ``raw`` spans unmapped addresses: before touching a range the
    caller must ``ensure`` every chunk under it.  ``reclaim`` waits on the
    device by default; the caller must also keep future work away from a
    chunk until it is ensured again.
    """

    def __init__(self, capacity_bytes, chunk_bytes=DEFAULT_CHUNK_BYTES, device=0, library=None, *,
                 spare_chunks=0):
        self.capacity_bytes = operator.index(capacity_bytes)
        self.chunk_bytes = operator.index(chunk_bytes)
        if not (0 < self.capacity_bytes < _INVALID and 0 < self.chunk_bytes < _INVALID):
            raise ValueError("capacity_bytes and chunk_bytes must be positive uint64 values")
        device = torch.device(f"cuda:{device}" if isinstance(device, int) else device)
        if device.type != "cuda":
            raise ValueError("VMM backing requires a CUDA device")
        self.device = torch.cuda.current_device() if device.index is None else device.index
        # ``library``: None (the in-tree libekv_b200.so), a path, or an object
        # exposing the ev_* functions (tests inject failures through one).
        if library is None or isinstance(library, (str, os.PathLike)):
            self._lib = load_library(None if library is None else str(library))
        else:
            self._lib = library
        handle = self._lib.ev_create(self.device, self.capacity_bytes, self.chunk_bytes)
        if not handle:
            raise RuntimeError(self._error())
        self._handle_box = [handle]
        self._finalizer = weakref.finalize(self, _close_handle, self._lib, self._handle_box)
        self._finalizer.atexit = False
        self.base = self._number("ev_base")
        self.reserved_bytes = self._number("ev_reserved")
        self.granularity = self._number("ev_granularity")
        self._mapped = set()
        self._precommitted = set()
        self._raw_ref = None
        self._poisoned = False
        self._metrics = dict.fromkeys(
            ("ensure_calls", "ensure_chunks", "ensure_ns", "precommit_calls", "precommit_chunks",
             "precommit_ns", "reclaim_calls", "reclaim_chunks", "reclaim_ns", "reclaim_sync_ns",
             "peak_backed_bytes"), 0)
        if spare_chunks:
            self.set_spare_chunks(spare_chunks)

    @property
    def _handle(self):
        return self._handle_box[0]

    def _error(self):
        return self._lib.ev_error().decode("utf-8", errors="replace")

    def _number(self, name):
        if not self._handle:
            raise RuntimeError("VMM backing is closed")
        value = getattr(self._lib, name)(self._handle)
        if value == _INVALID:
            raise RuntimeError(self._error())
        return value

    def _check(self):
        if not self._handle or self._poisoned:
            raise RuntimeError("VMM backing is closed or has encountered a CUDA error")

    def _ids(self, indices):
        ids = {operator.index(i) for i in indices}
        limit = self.reserved_bytes // self.chunk_bytes
        if any(i < 0 or i >= limit for i in ids):
            raise ValueError("chunk index outside reserved range")
        return ids

    def _batch(self, name, indices):
        ids = sorted(indices)
        array = (ct.c_uint64 * max(1, len(ids)))(*ids)
        if getattr(self._lib, name)(self._handle, array, len(ids)):
            error = self._error()
            if self._lib.ev_poisoned(self._handle) != 0:
                self._poisoned = True
            raise RuntimeError(error)

    @property
    def mapped_chunks(self):
        return frozenset(self._mapped - self._precommitted)

    @property
    def backed_bytes(self):
        return self._number("ev_backed")

    @property
    def spare_bytes(self):
        """Device memory held by unmapped physical handles kept for reuse."""
        return self._number("ev_spare")

    def set_spare_chunks(self, chunks):
        """Keep up to ``chunks`` physical handles that ``reclaim`` unmaps, so a later
        ``ensure`` maps them again instead of creating new ones (skips cuMemRelease +
        cuMemCreate, ~300 us per 2 MiB chunk on B200).  0 (the default, the
        reference's behaviour) releases every reclaimed chunk at once; lowering
        the limit releases the surplus now.  Kept handles are device memory that
        ``backed_bytes`` does not count."""
        self._check()
        chunks = operator.index(chunks)
        if chunks < 0:
            raise ValueError("spare chunk limit must be non-negative")
        if self._lib.ev_set_spare(self._handle, chunks):
            error = self._error()
            if self._lib.ev_poisoned(self._handle) != 0:
                self._poisoned = True
            raise RuntimeError(error)

    @property
    def metrics(self):
        return {**self._metrics, "backed_bytes": self.backed_bytes,
                "reserved_bytes": self.reserved_bytes, "spare_bytes": self.spare_bytes}

    @property
    def raw(self):
        """Borrow a contiguous uint8 tensor spanning the logical reservation."""
        self._check()
        if 0 not in self.mapped_chunks:
            raise RuntimeError("commit the sink chunk before building the tensor view")
        cached = self._raw_ref() if self._raw_ref else None
        if cached is not None:
            return cached
        with torch.cuda.device(self.device):
            raw = torch.as_tensor(_DeviceBytes(self.base, self.capacity_bytes, self),
                                  device=f"cuda:{self.device}")
        if raw.data_ptr() != self.base:
            raise RuntimeError("tensor view did not preserve the reserved address")
        self._raw_ref = weakref.ref(raw)
        return raw

    def ensure(self, indices):
        """Commit and zero missing chunks, returning their count."""
        self._check()
        ids = self._ids(indices)
        pending = ids - self._mapped
        if not pending and not ids & self._precommitted:
            return 0
        start = time.perf_counter_ns()
        self._batch("ev_ensure", pending)
        self._mapped.update(pending)
        self._precommitted.clear()
        self._metrics["ensure_ns"] += time.perf_counter_ns() - start
        self._metrics["ensure_calls"] += 1
        self._metrics["ensure_chunks"] += len(pending)
        self._metrics["peak_backed_bytes"] = max(self._metrics["peak_backed_bytes"],
                                                 len(self._mapped) * self.chunk_bytes)
        return len(pending)

    def precommit(self, indices):
        """Map missing chunks and start their zero fill without waiting for it."""
        self._check()
        pending = self._ids(indices) - self._mapped
        if not pending:
            return 0
        start = time.perf_counter_ns()
        self._batch("ev_precommit", pending)
        self._mapped.update(pending)
        self._precommitted.update(pending)
        self._metrics["precommit_ns"] += time.perf_counter_ns() - start
        self._metrics["precommit_calls"] += 1
        self._metrics["precommit_chunks"] += len(pending)
        self._metrics["peak_backed_bytes"] = max(self._metrics["peak_backed_bytes"],
                                                 len(self._mapped) * self.chunk_bytes)
        return len(pending)

    def reclaim(self, indices, *, synchronize=True):
        """Release idle chunks, returning their count."""
        self._check()
        pending = self._ids(indices) & self._mapped
        if not pending:
            return 0
        start = time.perf_counter_ns()
        if synchronize:
            torch.cuda.synchronize(self.device)
            self._metrics["reclaim_sync_ns"] += time.perf_counter_ns() - start
        self._batch("ev_drop", pending)
        self._mapped.difference_update(pending)
        self._precommitted.difference_update(pending)
        self._metrics["reclaim_ns"] += time.perf_counter_ns() - start
        self._metrics["reclaim_calls"] += 1
        self._metrics["reclaim_chunks"] += len(pending)
        return len(pending)

    def close(self):
        """Close once no tensor view, kernel or transfer can touch the backing.

        ``ev_close`` frees the native handle even when the teardown fails, so a
        failed close raises once and leaves the backing poisoned without a handle;
        a later ``close`` (or the finalizer) does not call ``ev_close`` again.
        """
        handle = self._handle
        if handle:
            if self._lib.ev_close(handle):
                self._poisoned = True
                self._handle_box[0] = None
                raise RuntimeError(f"native VMM teardown failed: {self._error()}")
            self._handle_box[0] = None
        self._finalizer.detach()
        self._mapped.clear()
        self._precommitted.clear()
