"""Top-K K/V row gather on sm_100a (R3).

``gather_rows`` keeps the signature, checks and zero-fill of the reference's
experimental/sparse_read.py:33-51.  ``gather_rows_planes`` applies one row
selection to many planes (every layer's K and V) in a single launch, resolving
the index chain once per row; it is the form the decode path and the benchmark
use.  ``PlaneGather`` pre-binds it for a decode loop, ``LookupGather`` runs a
layer's residency lookup inside its mapped gather, and ``LayerGather`` gathers
every layer's own selection in one launch.
"""

from __future__ import annotations

from ._lib import MAX_LAYERS, MAX_PLANES, call, index_esize, last_error, require_cuda, stream_handle, torch_binding, u64_array

INDICES_READY = 16  # EKV_GATHER_INDICES_READY of include/ekv_kernels.h
DISJOINT = 32  # EKV_GATHER_DISJOINT of include/ekv_kernels.h


def _mode(indirect, mapped):
    """Addressing mode of the C ABI: 0 direct, 1 indirect (software table), 2 mapped."""
    if mapped and indirect:
        raise ValueError("choose indirect or mapped addressing, not both")
    return 2 if mapped else int(bool(indirect))


def _index_args(positions, request_ids, lengths, request_table, slot_offsets, mode):
    if mode == 1 and (request_table is None or slot_offsets is None):
        raise ValueError("indirect gather needs request_table and slot_offsets")
    if mode == 2 and request_table is None:
        raise ValueError("mapped gather needs request_table (the residency map)")
    table = request_table if mode else None
    offsets = slot_offsets if mode == 1 else None
    return (
        positions.data_ptr(), index_esize(positions, "positions"),
        request_ids.data_ptr(), index_esize(request_ids, "request_ids"),
        lengths.data_ptr(), index_esize(lengths, "lengths"),
        None if table is None else table.data_ptr(),
        8 if table is None else index_esize(table, "request_table"),
        None if offsets is None else offsets.data_ptr(),
        8 if offsets is None else index_esize(offsets, "slot_offsets"),
    )


def _check_contiguous(tensors):
    for name, tensor in tensors.items():
        if tensor is not None and not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")


def gather_rows(raw, positions, request_ids, lengths, request_table, slot_offsets,
                output, layout, *, indirect):
    """All tensors must be contiguous CUDA tensors on the same device.

    ``output[b, i, :]`` is the ``layout.row_elements``-element row of ``raw``
    at element offset ``slot_offsets[request_table[request_ids[b], pos]]``
    (indirect) or ``sink + request_ids[b] * request_stride + pos * width``
    (direct, strides from ``layout``), with ``pos = positions[b, i]``; rows
    with ``pos`` outside ``[0, lengths[b])`` are zero.  Table values are
    ELEMENT offsets into ``raw``.  ``raw`` and ``output`` share a dtype: the
    payload is copied bit for bit.
    """
    fast = torch_binding()
    if fast is not None:
        try:
            rc = fast.gather_rows(raw, positions, request_ids, lengths, request_table, slot_offsets, output,
                                  layout.row_elements, layout.max_tokens, layout.request_bytes // layout.itemsize,
                                  layout.chunk_bytes // layout.itemsize, bool(indirect))
        except TypeError:  # not tensors: the checked path below reports it
            rc = fast.NOT_HANDLED
        if rc == 0:
            return
        if rc == fast.KERNEL_ERROR:
            raise last_error("ekv_gather_rows")
    batch, selected = positions.shape
    if output.shape != (batch, selected, layout.row_elements):
        raise ValueError("output shape does not match positions and row width")
    if not batch or not selected:
        return
    tensors = dict(raw=raw, positions=positions, request_ids=request_ids, lengths=lengths,
                   request_table=request_table, slot_offsets=slot_offsets, output=output)
    device = require_cuda(tensors)
    _check_contiguous(tensors)
    if raw.dtype != output.dtype:
        raise TypeError("raw and output must have the same dtype (bitwise row copy)")
    call(
        "ekv_gather_rows",
        raw.data_ptr(), output.data_ptr(), raw.element_size(),
        *_index_args(positions, request_ids, lengths, request_table, slot_offsets, int(bool(indirect))),
        batch, selected, layout.row_elements,
        layout.max_tokens, layout.request_bytes // layout.itemsize,
        layout.chunk_bytes // layout.itemsize,
        int(bool(indirect)), device.index, stream_handle(device),
    )


def gather_rows_planes(planes, positions, request_ids, lengths, request_table, slot_offsets,
                       outputs, layout, *, indirect, mapped=False, indices_ready=False):
    """``gather_rows`` over every plane in ``planes`` with one row selection.

    ``planes[p]`` and ``outputs[p]`` play the roles of ``raw`` and ``output``
    for plane p (e.g. layer l's K at p = 2l and V at p = 2l + 1).  Element
    offsets are relative to each plane's start.  Planes are processed
    EKV_MAX_PLANES per launch.

    ``mapped=True`` (new, beside the reference's two modes) reads
    ``request_table`` as a residency map: ``s = request_table[req, pos]`` is the
    row's slot in the request's fixed region (``sink + req * request_stride +
    s * width``), and ``s < 0`` reads as a zero row -- a lookup and its gather
    in one launch.

    ``indices_ready=True`` promises that the kernel launched just before this
    call on the current stream writes none of the index tensors; the gather
    then resolves its first index batch while that kernel finishes (see
    ``EKV_GATHER_INDICES_READY``).  The bytes written are the same either way.
    """
    fast = None if indices_ready else torch_binding()
    if fast is not None:
        try:
            rc = fast.gather_rows_planes(planes, outputs, positions, request_ids, lengths, request_table,
                                         slot_offsets, layout.row_elements, layout.max_tokens,
                                         layout.request_bytes // layout.itemsize,
                                         layout.chunk_bytes // layout.itemsize, bool(indirect), bool(mapped))
        except TypeError:  # not tensors: the checked path below reports it
            rc = fast.NOT_HANDLED
        if rc == 0:
            return
        if rc == fast.KERNEL_ERROR:
            raise last_error("ekv_gather_rows_planes")
    planes = list(planes)
    outputs = list(outputs)
    if len(planes) != len(outputs):
        raise ValueError("planes and outputs differ in length")
    batch, selected = positions.shape
    for output in outputs:
        if output.shape != (batch, selected, layout.row_elements):
            raise ValueError("output shape does not match positions and row width")
    if not planes or not batch or not selected:
        return
    index = dict(positions=positions, request_ids=request_ids, lengths=lengths,
                 request_table=request_table, slot_offsets=slot_offsets)
    device = require_cuda(index)
    _check_contiguous(index)
    itemsize = planes[0].element_size()
    for plane, output in zip(planes, outputs):
        require_cuda(dict(plane=plane, output=output), device)
        if not plane.is_contiguous() or not output.is_contiguous():
            raise ValueError("planes and outputs must be contiguous")
        if plane.dtype != output.dtype or plane.element_size() != itemsize:
            raise TypeError("all planes and outputs must share one dtype")
    mode = _mode(indirect, mapped)
    args = _index_args(positions, request_ids, lengths, request_table, slot_offsets, mode)
    # A residency map is indexed by token: its row width is the map's, not the layout's.
    table_width = request_table.shape[-1] if mode == 2 else layout.max_tokens
    stream = stream_handle(device)
    for start in range(0, len(planes), MAX_PLANES):
        src = planes[start:start + MAX_PLANES]
        dst = outputs[start:start + MAX_PLANES]
        call(
            "ekv_gather_rows_planes",
            u64_array(t.data_ptr() for t in src), u64_array(t.data_ptr() for t in dst), len(src),
            itemsize, *args, batch, selected, layout.row_elements,
            table_width, layout.request_bytes // layout.itemsize,
            layout.chunk_bytes // layout.itemsize,
            mode | (INDICES_READY if indices_ready else 0), device.index, stream,
        )


class PlaneGather:
    """Pre-bound plane gather for a hot loop: plane/output pointer tables and
    the index tensors are fixed at construction, so each call only launches.

    The tensors passed here must outlive the object and keep their storage.
    ``indices_ready`` as in ``gather_rows_planes``; ``disjoint`` as in
    ``LookupGather``.
    """

    def __init__(self, planes, positions, request_ids, lengths, request_table, slot_offsets,
                 outputs, layout, *, indirect, mapped=False, indices_ready=False, disjoint=False):
        planes = list(planes)
        outputs = list(outputs)
        if not planes or len(planes) != len(outputs) or len(planes) > MAX_PLANES:
            raise ValueError("need 1..EKV_MAX_PLANES planes with one output each")
        batch, selected = positions.shape
        for output in outputs:
            if output.shape != (batch, selected, layout.row_elements):
                raise ValueError("output shape does not match positions and row width")
        index = dict(positions=positions, request_ids=request_ids, lengths=lengths,
                     request_table=request_table, slot_offsets=slot_offsets)
        self.device = require_cuda(index)
        _check_contiguous(index)
        for plane, output in zip(planes, outputs):
            require_cuda(dict(plane=plane, output=output), self.device)
            if not plane.is_contiguous() or not output.is_contiguous():
                raise ValueError("planes and outputs must be contiguous")
            if plane.dtype != output.dtype or plane.dtype != planes[0].dtype:
                raise TypeError("all planes and outputs must share one dtype")
        self._keep = (planes, outputs, index)
        self._src = u64_array(t.data_ptr() for t in planes)
        self._dst = u64_array(t.data_ptr() for t in outputs)
        mode = _mode(indirect, mapped)
        # A residency map is indexed by token: its row width is the map's, not the layout's.
        table_width = request_table.shape[-1] if mode == 2 else layout.max_tokens
        self._args = (
            self._src, self._dst, len(planes), planes[0].element_size(),
            *_index_args(positions, request_ids, lengths, request_table, slot_offsets, mode),
            batch, selected, layout.row_elements,
            table_width, layout.request_bytes // layout.itemsize,
            layout.chunk_bytes // layout.itemsize,
            mode | (INDICES_READY if indices_ready else 0) | (DISJOINT if disjoint else 0), self.device.index,
        )
        self.empty = not batch or not selected

    def __call__(self, stream: int | None = None) -> None:
        if self.empty:
            return
        if stream is None:
            stream = stream_handle(self.device)
        call("ekv_gather_rows_planes", *self._args, stream)


class LookupGather:
    """One layer's residency lookup and its mapped gather in one launch
    (``ekv_lookup_gather_planes``); the miss list on request (``compact``).

    ``residency_map`` [R, T] maps token t of request r to its slot in the
    request's fixed region of every plane (-1: not resident); ``topk`` [B, K]
    holds token ids, ``request_ids`` [B] the map row / region of each row and
    ``lengths`` [B] bounds the valid tokens (a token is valid when
    ``0 <= t < min(lengths[b], T)``).  A call writes ``outputs[p][b, i]`` --
    plane p's row of the token's slot, zeros for an invalid token, a miss or a
    slot past the region, as ``gather_rows_planes(..., mapped=True)`` -- and
    ``slots`` (int32 [B, K]) and ``miss`` (bool [B, K]) as
    ``lookup_slots(residency_map[request_ids], topk, lengths)`` gives them;
    ``compact(stream)`` then writes that call's ``miss_list`` and
    ``miss_count`` from the mask.  Each map entry is read once, where a lookup
    followed by a gather reads it twice.  Pointer tables and outputs are bound
    at construction (the tensors passed here must outlive the object);
    ``indices_ready`` as in ``gather_rows_planes``.  ``disjoint=True`` promises
    that no kernel still running when this launch starts (the launches before
    it on the stream back to the last one without the promise) writes what it
    reads or touches what it writes -- true of a decode step's back-to-back
    per-layer launches -- so it copies at once and waits for them only before
    completing (``EKV_GATHER_DISJOINT``); the bytes are the same either way.
    """

    def __init__(self, planes, residency_map, topk, request_ids, lengths, outputs, layout, *,
                 indices_ready=False, disjoint=False):
        planes, outputs = list(planes), list(outputs)
        if not planes or len(planes) != len(outputs) or len(planes) > MAX_PLANES:
            raise ValueError("need 1..EKV_MAX_PLANES planes with one output each")
        if residency_map.dim() != 2 or topk.dim() != 2:
            raise ValueError("expected residency_map [R, T] and topk [B, K]")
        batch, k = topk.shape
        if request_ids.shape != (batch,) or lengths.shape != (batch,):
            raise ValueError("request_ids and lengths need one entry per Top-K row")
        for output in outputs:
            if output.shape != (batch, k, layout.row_elements):
                raise ValueError("output shape does not match topk and row width")
        index = dict(residency_map=residency_map, topk=topk, request_ids=request_ids, lengths=lengths)
        self.device = require_cuda(index)
        _check_contiguous(index)
        for plane, output in zip(planes, outputs):
            require_cuda(dict(plane=plane, output=output), self.device)
            if not plane.is_contiguous() or not output.is_contiguous():
                raise ValueError("planes and outputs must be contiguous")
            if plane.dtype != output.dtype or plane.dtype != planes[0].dtype:
                raise TypeError("all planes and outputs must share one dtype")
        import torch

        self.slots = torch.empty((batch, k), dtype=torch.int32, device=self.device)
        self.miss = torch.empty((batch, k), dtype=torch.bool, device=self.device)
        self.miss_list = torch.empty((batch, k), dtype=torch.int32, device=self.device)
        self.miss_count = torch.empty((batch,), dtype=torch.int32, device=self.device)
        self._keep = (planes, outputs, index)
        self._src = u64_array(t.data_ptr() for t in planes)
        self._dst = u64_array(t.data_ptr() for t in outputs)
        self._args = (
            self._src, self._dst, len(planes), planes[0].element_size(),
            topk.data_ptr(), index_esize(topk, "topk"),
            request_ids.data_ptr(), index_esize(request_ids, "request_ids"),
            lengths.data_ptr(), index_esize(lengths, "lengths"),
            residency_map.data_ptr(), index_esize(residency_map, "residency_map"), residency_map.shape[1],
            batch, k, layout.row_elements,
            layout.request_bytes // layout.itemsize, layout.chunk_bytes // layout.itemsize,
            self.slots.data_ptr(), self.miss.data_ptr(),
            (INDICES_READY if indices_ready else 0) | (DISJOINT if disjoint else 0), self.device.index,
        )
        self._compact_args = (
            self.miss.data_ptr(), k, topk.data_ptr(), index_esize(topk, "topk"), k,
            batch, k, self.miss_list.data_ptr(), k, self.miss_count.data_ptr(), self.device.index,
        )
        self.empty = not batch or not k
        self._rows = batch

    def __call__(self, stream: int | None = None) -> None:
        if self.empty:
            return
        call("ekv_lookup_gather_planes", *self._args, stream_handle(self.device) if stream is None else stream)

    def compact(self, stream: int | None = None) -> None:
        """``miss_list`` / ``miss_count`` from the last call's miss mask (launch after it)."""
        if not self._rows:
            return
        call("ekv_compact_misses", *self._compact_args, stream_handle(self.device) if stream is None else stream)


__all__ = ["gather_rows", "gather_rows_planes", "PlaneGather", "LookupGather", "LayerGather"]


class LayerGather:
    """Every layer's own Top-K gather in one launch (``ekv_gather_layers``).

    ``planes`` / ``outputs`` list every layer's planes layer-major
    (``planes_per_layer`` each, e.g. K and V); ``positions[l]`` and, in indirect
    or mapped mode, ``request_tables[l]`` are layer l's.  Layer l's result is
    that of ``gather_rows_planes`` over its planes with its positions and
    table; request ids, lengths, slot offsets and ``layout`` are shared.  For a
    decode step whose every layer's Top-K is known when the step starts; a
    step that learns layer l's Top-K only after layer l-1 calls the per-layer
    ``PlaneGather`` instead.  Pointer tables are bound at construction, so the
    tensors passed here must outlive the object and keep their storage.
    """

    def __init__(self, planes, positions, request_ids, lengths, request_tables, slot_offsets,
                 outputs, layout, *, planes_per_layer, indirect, mapped=False):
        planes, outputs, positions = list(planes), list(outputs), list(positions)
        n_layers = len(positions)
        if not 1 <= n_layers <= MAX_LAYERS:
            raise ValueError("need 1..EKV_MAX_LAYERS layers")
        if planes_per_layer < 1 or len(planes) != n_layers * planes_per_layer or len(outputs) != len(planes):
            raise ValueError("need planes_per_layer planes and outputs per layer")
        if len(planes) > MAX_PLANES:
            raise ValueError("more than EKV_MAX_PLANES planes")
        mode = _mode(indirect, mapped)
        tables = list(request_tables) if mode else [None] * n_layers
        if len(tables) != n_layers or (mode and any(t is None for t in tables)):
            raise ValueError("indirect and mapped gathers need one request table per layer")
        if mode == 1 and slot_offsets is None:
            raise ValueError("indirect gather needs request_table and slot_offsets")
        batch, selected = positions[0].shape
        for pos, table in zip(positions, tables):
            if pos.shape != (batch, selected) or pos.dtype != positions[0].dtype:
                raise ValueError("every layer's positions must share one shape and dtype")
            if table is not None and (table.shape != tables[0].shape or table.dtype != tables[0].dtype):
                raise ValueError("every layer's request table must share one shape and dtype")
        for output in outputs:
            if output.shape != (batch, selected, layout.row_elements):
                raise ValueError("output shape does not match positions and row width")
        index = dict(request_ids=request_ids, lengths=lengths, slot_offsets=slot_offsets if mode == 1 else None)
        index.update({f"positions[{i}]": t for i, t in enumerate(positions)})
        index.update({f"request_tables[{i}]": t for i, t in enumerate(tables) if t is not None})
        self.device = require_cuda(index)
        _check_contiguous(index)
        for plane, output in zip(planes, outputs):
            require_cuda(dict(plane=plane, output=output), self.device)
            if not plane.is_contiguous() or not output.is_contiguous():
                raise ValueError("planes and outputs must be contiguous")
            if plane.dtype != output.dtype or plane.dtype != planes[0].dtype:
                raise TypeError("all planes and outputs must share one dtype")
        self._keep = (planes, outputs, positions, tables, index)
        self._src = u64_array(t.data_ptr() for t in planes)
        self._dst = u64_array(t.data_ptr() for t in outputs)
        self._positions = u64_array(t.data_ptr() for t in positions)
        self._tables = u64_array(t.data_ptr() for t in tables) if mode else None
        table_width = tables[0].shape[-1] if mode == 2 else layout.max_tokens
        offsets = slot_offsets if mode == 1 else None
        self._args = (
            self._src, self._dst, n_layers, planes_per_layer, planes[0].element_size(),
            self._positions, index_esize(positions[0], "positions"),
            request_ids.data_ptr(), index_esize(request_ids, "request_ids"),
            lengths.data_ptr(), index_esize(lengths, "lengths"),
            self._tables, index_esize(tables[0], "request_table") if mode else 8,
            None if offsets is None else offsets.data_ptr(),
            8 if offsets is None else index_esize(offsets, "slot_offsets"),
            batch, selected, layout.row_elements,
            table_width, layout.request_bytes // layout.itemsize,
            layout.chunk_bytes // layout.itemsize,
            mode, self.device.index,
        )
        self.empty = not batch or not selected

    def __call__(self, stream: int | None = None) -> None:
        if self.empty:
            return
        if stream is None:
            stream = stream_handle(self.device)
        call("ekv_gather_layers", *self._args, stream)

