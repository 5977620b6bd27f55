"""Demote/promote data movement (R5): row pack/unpack and a pinned host KV pool.

The reference's migration transactions (adaptive_sparse/migration.py) move
rows through SGLang's host KV pool: ``alloc_paged_token_slots``,
``backup_from_device_all_layer`` (migration.py:105-111), ``load_to_device_per_layer``
(migration.py:231-234), ``allocated_host_indices`` and ``free``
(migration.py:58-63).  ``PinnedHostKVPool`` implements those methods on top
of the pack/unpack kernels, plus ``load_to_device_all_layer`` (every layer in
one staged transfer), which this package's promotion uses when present.

Host layout: plane-major ("layer first"): plane p (K of layer l at p = 2l,
V at p = 2l + 1) is a region of ``capacity`` rows starting on a 2 MiB
boundary, so a device chunk's worth of rows maps onto a chunk-aligned host
range.  Two ways across the host link: "staged" (default) packs rows densely
into a device scratch ring and moves each run of consecutive host rows with
the copy engines, overlapped on a side stream; "zero_copy" has the row-copy
kernel store to / load from the pinned buffer directly through unified
addressing (used when host rows are too fragmented for per-run copies).
"""

from __future__ import annotations

import ctypes as ct

import torch

from ._lib import MAX_PLANES, call, index_esize, require_cuda, stream_handle, u64_array

CHUNK_BYTES = 2 << 20


def _plane_rows(planes):
    planes = list(planes)
    if not planes:
        raise ValueError("need at least one plane")
    row_bytes = planes[0][0].numel() * planes[0].element_size()
    for plane in planes:
        if not plane.is_contiguous():
            raise ValueError("planes must be contiguous")
        if plane[0].numel() * plane.element_size() != row_bytes:
            raise ValueError("all planes must share one row size")
    return planes, row_bytes


def _row_copy(kind, planes, slots, staging, *, plane_index=None, stage_rows=None,
              stage_plane_stride=0, device=None, stream=None):
    planes, row_bytes = _plane_rows(planes)
    if len(planes) > MAX_PLANES:
        raise ValueError("more planes than EKV_MAX_PLANES in one call")
    device = require_cuda(dict(slots=slots, plane_index=plane_index, stage_rows=stage_rows,
                               **{f"plane{i}": p for i, p in enumerate(planes)}), device)
    if not slots.is_contiguous() or slots.dim() != 1:
        raise ValueError("slots must be a contiguous 1-D tensor")
    if plane_index is not None:
        if plane_index.dtype != torch.int32 or plane_index.numel() != slots.numel():
            raise ValueError("plane_index must be int32 with one entry per slot")
        n_tasks = slots.numel()
    else:
        n_tasks = len(planes) * slots.numel()
    if stage_rows is not None and stage_rows.numel() != slots.numel():
        raise ValueError("stage_rows must have one entry per slot")
    if not staging.is_contiguous():
        raise ValueError("staging must be contiguous")
    if staging.device.type == "cpu" and not staging.is_pinned():
        raise ValueError("host staging must be pinned memory")
    call(
        kind,
        u64_array(p.data_ptr() for p in planes), len(planes), row_bytes,
        None if plane_index is None else plane_index.data_ptr(),
        slots.data_ptr(), index_esize(slots, "slots"), slots.numel(),
        None if stage_rows is None else stage_rows.data_ptr(),
        8 if stage_rows is None else index_esize(stage_rows, "stage_rows"),
        staging.data_ptr(), int(stage_plane_stride), n_tasks,
        device.index, stream if stream is not None else stream_handle(device),
    )


def pack_rows(planes, slots, staging, **kwargs):
    """Copy rows ``planes[p][slots[j]]`` into ``staging`` (device or pinned host).

    Cross form (``plane_index`` None): plane p's row j lands at byte
    ``p * stage_plane_stride + (stage_rows[j] if given else j) * row_bytes``.
    List form: task t copies ``planes[plane_index[t]][slots[t]]`` to row
    ``stage_rows[t]`` (or t) of ``staging``.
    """
    _row_copy("ekv_pack_rows", planes, slots, staging, **kwargs)


def unpack_rows(planes, slots, staging, **kwargs):
    """Inverse of ``pack_rows``: staging rows back into ``planes`` at ``slots``."""
    _row_copy("ekv_unpack_rows", planes, slots, staging, **kwargs)


SCRATCH_BYTES = 64 << 20  # default device ring for staged transfers (4 slots x 16 MiB)
_scratch_cache: dict = {}


def scratch_buffer(device, nbytes: int = SCRATCH_BYTES) -> torch.Tensor:
    """Per-device scratch ring for staged transfers, allocated once and reused."""
    device = torch.device(device)
    buf = _scratch_cache.get(device)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _scratch_cache[device] = buf
    return buf


def segments_tensor(segments) -> torch.Tensor:
    """(first_task, count, host_byte_offset) triples as a contiguous CPU int64 [n, 3] tensor."""
    seg = torch.as_tensor(segments, dtype=torch.int64).reshape(-1, 3).contiguous()
    if seg.device.type != "cpu":
        seg = seg.cpu()
    return seg


def row_runs(host_rows: torch.Tensor):
    """Maximal runs of consecutive values: [(start_index, length, first_value), ...]."""
    rows = host_rows.to("cpu", torch.int64).flatten()
    if not rows.numel():
        return []
    breaks = torch.nonzero(rows[1:] - rows[:-1] != 1).flatten() + 1
    starts = torch.cat([torch.zeros(1, dtype=torch.int64), breaks])
    ends = torch.cat([breaks, torch.tensor([rows.numel()])])
    return [(int(s), int(e - s), int(rows[s])) for s, e in zip(starts.tolist(), ends.tolist())]


def _staged(kind, planes, slots, host, segments, *, plane_index=None, scratch=None, copy_stream=None,
            device=None, stream=None):
    planes, row_bytes = _plane_rows(planes)
    if len(planes) > MAX_PLANES:
        raise ValueError("more planes than EKV_MAX_PLANES in one call")
    device = require_cuda(dict(slots=slots, plane_index=plane_index,
                               **{f"plane{i}": p for i, p in enumerate(planes)}), device)
    if not slots.is_contiguous() or slots.dim() != 1:
        raise ValueError("slots must be a contiguous 1-D tensor")
    if plane_index is not None:
        if plane_index.dtype != torch.int32 or plane_index.numel() != slots.numel():
            raise ValueError("plane_index must be int32 with one entry per slot")
        n_tasks = slots.numel()
    else:
        n_tasks = len(planes) * slots.numel()
    if host.device.type != "cpu" or not host.is_pinned() or not host.is_contiguous():
        raise ValueError("host staging must be contiguous pinned memory")
    seg = segments_tensor(segments)
    if seg.numel():
        last = seg[:, 2] + seg[:, 1] * row_bytes
        if int(last.max()) > host.numel() * host.element_size():
            raise ValueError("a segment runs past the end of the host staging buffer")
    if scratch is None:
        scratch = scratch_buffer(device)
    require_cuda(dict(scratch=scratch), device)
    call(
        kind,
        u64_array(p.data_ptr() for p in planes), len(planes), row_bytes,
        None if plane_index is None else plane_index.data_ptr(),
        slots.data_ptr(), index_esize(slots, "slots"), slots.numel(),
        ct.cast(seg.data_ptr(), ct.POINTER(ct.c_int64)), seg.shape[0],
        host.data_ptr(), n_tasks,
        scratch.data_ptr(), scratch.numel() * scratch.element_size(),
        device.index, stream if stream is not None else stream_handle(device),
        None if copy_stream is None else copy_stream.cuda_stream,
    )


def pack_rows_staged(planes, slots, host, segments, **kwargs):
    """``pack_rows`` into PINNED host memory through the copy engines.

    Tasks as in ``pack_rows`` (cross or list form, no ``stage_rows``);
    ``segments`` lists (first_task, count, host_byte_offset) runs of tasks that
    are consecutive rows of ``host``.  Complete when the current stream is.
    """
    _staged("ekv_pack_rows_staged", planes, slots, host, segments, **kwargs)


def unpack_rows_staged(planes, slots, host, segments, **kwargs):
    """Inverse of ``pack_rows_staged``."""
    _staged("ekv_unpack_rows_staged", planes, slots, host, segments, **kwargs)


def pinned_buffer(nbytes: int) -> torch.Tensor:
    """Pinned host bytes, rounded up to whole 2 MiB chunks."""
    rounded = -(-nbytes // CHUNK_BYTES) * CHUNK_BYTES
    return torch.empty(rounded, dtype=torch.uint8, pin_memory=True)


class PinnedHostKVPool:
    """Host KV pool with SGLang HostKVCache's migration methods.

    ``capacity`` token rows per plane, ``layer_num`` layers of K and V, rows of
    ``row_bytes`` bytes.  Host slots are handed out one token at a time (page
    size 1 on the host; device page structure is preserved by the indices the
    caller passes).
    """

    def __init__(self, capacity: int, layer_num: int, row_bytes: int, device, dtype=torch.bfloat16,
                 transfer: str = "staged"):
        if transfer not in ("staged", "zero_copy"):
            raise ValueError("transfer must be 'staged' or 'zero_copy'")
        self.capacity = int(capacity)
        self.layer_num = int(layer_num)
        self.row_bytes = int(row_bytes)
        self.device = torch.device(device)
        self.dtype = dtype
        self.transfer = transfer
        plane_bytes = self.capacity * self.row_bytes
        self.plane_stride = -(-plane_bytes // CHUNK_BYTES) * CHUNK_BYTES
        self.buffer = pinned_buffer(self.plane_stride * 2 * self.layer_num)
        self._free = torch.ones(self.capacity, dtype=torch.bool)

    # --- allocation (host indices are int64 row numbers) ---------------------

    def available_size(self) -> int:
        return int(self._free.sum())

    def alloc(self, need: int) -> torch.Tensor | None:
        free = torch.nonzero(self._free).flatten()
        if free.numel() < need:
            return None
        chosen = free[:need]
        self._free[chosen] = False
        return chosen

    def free(self, indices: torch.Tensor) -> int:
        indices = indices.to("cpu", torch.int64)
        if (~self._free[indices]).sum() != indices.numel():
            raise RuntimeError("double free of host KV rows")
        self._free[indices] = True
        return indices.numel()

    def alloc_paged_token_slots(self, req_to_host_pool, allocated_len, row, start, length):
        """Allocate host rows for tokens [start, length) of request row ``row``."""
        need = length - start
        indices = self.alloc(need)
        if indices is None:
            raise MemoryError("host KV pool exhausted")
        req_to_host_pool[row, start:length] = indices.to(req_to_host_pool.device, req_to_host_pool.dtype)
        allocated_len[row] = length
        return req_to_host_pool[row, :length]

    def allocated_host_indices(self, req_to_host_pool, row, length):
        return req_to_host_pool[row, :int(length)]

    # --- data movement --------------------------------------------------------

    def plane_view(self, plane: int) -> torch.Tensor:
        """Host rows of plane ``plane`` as [capacity, row_bytes] uint8."""
        start = plane * self.plane_stride
        return self.buffer[start:start + self.capacity * self.row_bytes].view(self.capacity, self.row_bytes)

    @staticmethod
    def _device_planes(device_pool, layers):
        planes = []
        for layer in layers:
            planes.append(device_pool.get_key_buffer(layer))
            planes.append(device_pool.get_value_buffer(layer))
        return planes

    MAX_STAGED_RUNS = 256  # more host-row runs than this: move rows with the zero-copy kernel

    def _segments(self, host_indices, first_plane, n_planes):
        """Staged-transfer segments for planes [first_plane, first_plane + n_planes), or
        None when the host rows are too fragmented for per-run copies."""
        if self.transfer != "staged":
            return None
        runs = row_runs(host_indices)
        if len(runs) > self.MAX_STAGED_RUNS:
            return None
        n = int(host_indices.numel())
        return [(p * n + start, length, (first_plane + p) * self.plane_stride + first_row * self.row_bytes)
                for p in range(n_planes) for start, length, first_row in runs]

    def backup_from_device_all_layer(self, device_pool, host_indices, device_indices,
                                     io_backend="kernel"):
        """Copy rows ``device_indices`` of every layer's K and V to host rows ``host_indices``."""
        layers = range(getattr(device_pool, "start_layer", 0),
                       getattr(device_pool, "end_layer", self.layer_num))
        planes = self._device_planes(device_pool, layers)
        slots = device_indices.to(self.device, torch.int64).contiguous()
        for start in range(0, len(planes), MAX_PLANES):
            chunk = planes[start:start + MAX_PLANES]
            first_plane = 2 * layers.start + start
            segments = self._segments(host_indices, first_plane, len(chunk))
            if segments is not None:
                pack_rows_staged(chunk, slots, self.buffer, segments)
            else:
                rows = host_indices.to(self.device, torch.int64).contiguous()
                pack_rows(chunk, slots, self.buffer[first_plane * self.plane_stride:], stage_rows=rows,
                          stage_plane_stride=self.plane_stride)

    def load_to_device_all_layer(self, device_pool, host_indices, device_indices, io_backend="kernel"):
        """Copy host rows ``host_indices`` of every layer's K and V into rows ``device_indices``:
        the inverse of ``backup_from_device_all_layer``, one staged transfer over all
        planes instead of one per layer."""
        layers = range(getattr(device_pool, "start_layer", 0),
                       getattr(device_pool, "end_layer", self.layer_num))
        planes = self._device_planes(device_pool, layers)
        slots = device_indices.to(self.device, torch.int64).contiguous()
        for start in range(0, len(planes), MAX_PLANES):
            chunk = planes[start:start + MAX_PLANES]
            first_plane = 2 * layers.start + start
            segments = self._segments(host_indices, first_plane, len(chunk))
            if segments is not None:
                unpack_rows_staged(chunk, slots, self.buffer, segments)
            else:
                rows = host_indices.to(self.device, torch.int64).contiguous()
                unpack_rows(chunk, slots, self.buffer[first_plane * self.plane_stride:], stage_rows=rows,
                            stage_plane_stride=self.plane_stride)

    def load_to_device_per_layer(self, device_pool, host_indices, device_indices, layer_id,
                                 io_backend="kernel"):
        """Copy host rows ``host_indices`` of layer ``layer_id`` into K/V rows ``device_indices``."""
        planes = self._device_planes(device_pool, [layer_id])
        slots = device_indices.to(self.device, torch.int64).contiguous()
        segments = self._segments(host_indices, 2 * layer_id, 2)
        if segments is not None:
            unpack_rows_staged(planes, slots, self.buffer, segments)
        else:
            rows = host_indices.to(self.device, torch.int64).contiguous()
            unpack_rows(planes, slots, self.buffer[2 * layer_id * self.plane_stride:], stage_rows=rows,
                        stage_plane_stride=self.plane_stride)
