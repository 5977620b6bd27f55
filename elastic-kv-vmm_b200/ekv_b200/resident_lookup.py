"""Residency lookups on sm_100a (R1, R2).

``resolve_resident`` keeps the signature, in-place output and sentinel of the
reference's adaptive_sparse/resident_lookup.py:29-40 so the request-residency
swap hook (adaptive_sparse/request_residency.py:810-818) can import it
unchanged.  ``lookup_slots`` is the batched token -> hot-slot lookup with miss
detection and per-request miss compaction that the reference delegates to
SGLang's swap kernel.
"""

from __future__ import annotations

import torch

from ._lib import call, index_esize, last_error, require_cuda, stream_handle, torch_binding


def resolve_resident(topk, table, mapping, rows, lengths, selected, output, block_size):
    """Write only selected rows into an existing [1, B, K * block_size] tensor.

    For every row listed in ``selected`` and column j::

        block = topk[0, row, j // block_size]
        pos = block * block_size + j % block_size
        output[0, row, j] = mapping[table[rows[row], pos]]   if block >= 0 and pos < lengths[row]
                            -1                               otherwise

    Other rows of ``output`` are left untouched.  Every tensor may be strided;
    index tensors are int32 or int64; ``output`` is int32 (a wider mapping value
    is truncated on store, as in the reference).  No-op when ``selected`` is
    empty or the width is zero (resident_lookup.py:31-33).
    """
    fast = torch_binding()
    if fast is not None and type(block_size) is int:
        try:
            rc = fast.resolve_resident(topk, table, mapping, rows, lengths, selected, output, block_size)
        except TypeError:  # not tensors: the checked path below reports it
            rc = fast.NOT_HANDLED
        if rc == 0:
            return
        if rc == fast.KERNEL_ERROR:
            raise last_error("ekv_resolve_resident")
    width = topk.shape[2] * block_size
    if not selected.numel() or not width:
        return
    device = require_cuda(dict(topk=topk, table=table, mapping=mapping, rows=rows,
                               lengths=lengths, selected=selected, output=output))
    if output.dtype != torch.int32:
        raise TypeError("output must be an int32 tensor")
    if topk.dim() != 3 or table.dim() != 2 or output.dim() != 3:
        raise ValueError("expected topk [1, B, K], table [R, T] and output [1, B, K * block_size]")
    call(
        "ekv_resolve_resident",
        topk.data_ptr(), index_esize(topk, "topk"), topk.stride(1), topk.stride(2), topk.shape[2],
        table.data_ptr(), index_esize(table, "table"), table.stride(0), table.stride(1),
        mapping.data_ptr(), index_esize(mapping, "mapping"), mapping.stride(0),
        rows.data_ptr(), index_esize(rows, "rows"), rows.stride(0),
        lengths.data_ptr(), index_esize(lengths, "lengths"), lengths.stride(0),
        selected.data_ptr(), index_esize(selected, "selected"), selected.stride(0), selected.numel(),
        output.data_ptr(), output.stride(1), output.stride(2),
        int(block_size), device.index, stream_handle(device),
    )


class LookupPlan:
    """``lookup_slots`` pre-bound to fixed tensors for a hot loop (or a CUDA graph).

    Each call only launches; the tensors must outlive the plan and keep their
    storage.  ``slots``, ``miss``, ``miss_list`` and ``miss_count`` hold the
    results after every call.
    """

    def __init__(self, residency_map, topk, lengths=None, *, slots=None, miss=None, miss_list=None,
                 miss_count=None):
        device = require_cuda(dict(residency_map=residency_map, topk=topk, lengths=lengths))
        batch, k = topk.shape
        self.slots = slots if slots is not None else torch.empty((batch, k), dtype=torch.int32, device=device)
        self.miss = miss if miss is not None else torch.empty((batch, k), dtype=torch.bool, device=device)
        self.miss_list = (miss_list if miss_list is not None
                          else torch.empty((batch, k), dtype=torch.int32, device=device))
        self.miss_count = (miss_count if miss_count is not None
                           else torch.empty((batch,), dtype=torch.int32, device=device))
        # Validate once through the public function (this also runs the lookup).
        lookup_slots(residency_map, topk, lengths, slots=self.slots, miss=self.miss,
                     miss_list=self.miss_list, miss_count=self.miss_count)
        self.device = device
        self._keep = (residency_map, topk, lengths)
        self._args = (
            residency_map.data_ptr(), index_esize(residency_map, "residency_map"),
            residency_map.stride(0), residency_map.shape[1],
            topk.data_ptr(), index_esize(topk, "topk"), topk.stride(0),
            None if lengths is None else lengths.data_ptr(),
            4 if lengths is None else index_esize(lengths, "lengths"),
            batch, k, self.slots.data_ptr(), self.slots.stride(0), self.miss.data_ptr(), self.miss.stride(0),
            self.miss_list.data_ptr(), self.miss_list.stride(0), self.miss_count.data_ptr(), device.index,
        )

    def __call__(self, stream: int | None = None) -> None:
        call("ekv_lookup_slots", *self._args, stream_handle(self.device) if stream is None else stream)


def lookup_slots(residency_map, topk, lengths=None, *, slots=None, miss=None, miss_list=None,
                 miss_count=None, compact=True):
    """Token ids -> hot slots through a per-request residency map.

    ``residency_map`` is [B, T] (int32/int64, -1 = token not resident, else its
    hot slot); ``topk`` is [B, K] token ids; ``lengths`` [B] optionally bounds
    the valid token range of each row (tokens outside [0, min(length, T)) get
    slot -1 and are not misses).  Returns ``(slots, miss, miss_list,
    miss_count)``: int32 [B, K] slots, bool [B, K] miss mask, int32 [B, K] miss
    token ids of each row compacted in column order then padded with -1, and
    int32 [B] miss counts.  Output tensors may be passed in to avoid
    allocation.  With ``compact=False`` only ``slots`` and ``miss`` are
    produced.
    """
    fast = torch_binding()
    if fast is not None:
        try:
            rc, *results = fast.lookup_slots(residency_map, topk, lengths, slots, miss, miss_list, miss_count,
                                             bool(compact))
        except TypeError:  # not tensors: the checked path below reports it
            rc = fast.NOT_HANDLED
        if rc == 0:
            return tuple(results)
        if rc == fast.KERNEL_ERROR:
            raise last_error("ekv_lookup_slots")
    device = require_cuda(dict(residency_map=residency_map, topk=topk, lengths=lengths))
    if residency_map.dim() != 2 or topk.dim() != 2 or residency_map.shape[0] != topk.shape[0]:
        raise ValueError("expected residency_map [B, T] and topk [B, K]")
    if residency_map.stride(1) != 1 or topk.stride(1) != 1:
        raise ValueError("residency_map and topk rows must be contiguous")
    batch, k = topk.shape
    if lengths is not None and (lengths.dim() != 1 or lengths.shape[0] != batch or lengths.stride(0) != 1):
        raise ValueError("lengths must be a contiguous [B] tensor")
    if slots is None:
        slots = torch.empty((batch, k), dtype=torch.int32, device=device)
    if miss is None:
        miss = torch.empty((batch, k), dtype=torch.bool, device=device)
    if compact:
        if miss_list is None:
            miss_list = torch.empty((batch, k), dtype=torch.int32, device=device)
        if miss_count is None:
            miss_count = torch.empty((batch,), dtype=torch.int32, device=device)
    outputs = dict(slots=(slots, torch.int32), miss=(miss, torch.bool),
                   miss_list=(miss_list, torch.int32), miss_count=(miss_count, torch.int32))
    for name, (tensor, dtype) in outputs.items():
        if tensor is None:
            continue
        require_cuda({name: tensor}, device)
        if tensor.dtype != dtype:
            raise TypeError(f"{name} must be {dtype}")
        if tensor.shape[0] != batch or tensor.stride(-1) != 1:
            raise ValueError(f"{name} must have {batch} rows with contiguous columns")
    if miss_count is not None and miss_count.numel() != batch:
        raise ValueError("miss_count must have one entry per row")
    call(
        "ekv_lookup_slots",
        residency_map.data_ptr(), index_esize(residency_map, "residency_map"),
        residency_map.stride(0), residency_map.shape[1],
        topk.data_ptr(), index_esize(topk, "topk"), topk.stride(0),
        None if lengths is None else lengths.data_ptr(),
        4 if lengths is None else index_esize(lengths, "lengths"),
        batch, k,
        slots.data_ptr(), slots.stride(0),
        miss.data_ptr(), miss.stride(0),
        None if miss_list is None else miss_list.data_ptr(),
        0 if miss_list is None else miss_list.stride(0),
        None if miss_count is None else miss_count.data_ptr(),
        device.index, stream_handle(device),
    )
    return slots, miss, miss_list, miss_count
