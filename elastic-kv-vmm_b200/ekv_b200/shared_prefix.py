"""Shared-prefix direct resolution on the device (the donor-slot variant of R1).

Mirrors the resolvers of adaptive_sparse/shared_prefix.py: a host-backed
consumer request whose prompt shares a prefix with a live, fully resident
SOURCE request reads the complete shared blocks straight from the source's
device slots.  Same names, keyword arguments, validation messages and outputs
(valid bool [.., blocks], physical int32 [.., blocks, block_size]) as the
reference; the address arithmetic of all consumers runs in ONE kernel
(``ekv_resolve_shared_blocks``) instead of a dozen torch ops.

The prefix registry and claims of the same module (fingerprints of token ids)
are control-plane metadata and are not part of this package.
"""

from __future__ import annotations

from typing import Iterable

import torch

import numpy as np

from ._lib import SHARED_INLINE_MAX, call, index_esize, last_error, stream_handle, torch_binding


def _is_int(value) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def complete_shared_blocks(block_ids: Iterable[int], *, seq_len: int, shared_tokens: int,
                           block_size: int) -> tuple[bool, ...]:
    """Whether each selected block lies wholly in the shared prefix (shared_prefix.py:36-67).

    Pure host logic (a handful of block ids): identical checks and result.
    """
    for value, name, minimum in ((seq_len, "seq_len", 1), (shared_tokens, "shared_tokens", 0),
                                 (block_size, "block_size", 1)):
        if not _is_int(value) or value < minimum:
            raise ValueError(f"{name} is outside the supported range")
    result = []
    for block in block_ids:
        if not _is_int(block):
            raise ValueError("block ids must be integers")
        end = block * block_size + block_size
        result.append(block >= 0 and end <= shared_tokens and end <= seq_len)
    return tuple(result)


def _checked_lists(source_rows, shared_tokens, table_rows: int) -> tuple[list, list]:
    """The per-request lists, validated as shared_prefix.py:150-165 does (same messages)."""
    rows, prefixes = list(source_rows), list(shared_tokens)
    # Fast path for plain ints (min / max over the lists); anything else takes the
    # element-wise checks, which raise exactly where the reference does.
    if set(map(type, rows)) <= {int} and set(map(type, prefixes)) <= {int}:
        if rows and (min(rows) < 0 or max(rows) >= table_rows):
            raise ValueError("source row is outside the request table")
        if prefixes and min(prefixes) < 0:
            raise ValueError("invalid shared prefix geometry")
        return rows, prefixes
    for row in rows:
        if not _is_int(row) or row < 0 or row >= table_rows:
            raise ValueError("source row is outside the request table")
    for tokens in prefixes:
        if not _is_int(tokens) or tokens < 0:
            raise ValueError("invalid shared prefix geometry")
    return rows, prefixes


def _index_tensor(tensor: torch.Tensor, device: torch.device) -> torch.Tensor:
    """int32 / int64 view of an index tensor on ``device`` (other integer types widen)."""
    if tensor.device != device:
        tensor = tensor.to(device)
    if tensor.dtype not in (torch.int32, torch.int64):
        tensor = tensor.to(torch.int64)
    return tensor


def _geometry(request_table: torch.Tensor, device_mapping: torch.Tensor, device: torch.device):
    if device.type != "cuda":
        raise ValueError("block ids must be a CUDA tensor (the resolver runs only on the device)")
    table = _index_tensor(request_table, device)
    mapping = _index_tensor(device_mapping, device).reshape(-1)
    return table, mapping


def _launch(blocks, requests, per_request, block_row, block_col, rows, row, prefixes, prefix,
            lengths, len_stride, block_size, table, mapping, valid, physical, masked, exclude_newest,
            on_host=False):
    """``rows`` / ``prefixes``: device int64 tensors, host addresses of int64
    arrays (``on_host``), or None for the scalar ``row`` / ``prefix``."""
    device = blocks.device

    def address(meta):
        if meta is None:
            return None
        return meta if on_host else meta.data_ptr()

    call("ekv_resolve_shared_blocks",
         blocks.data_ptr(), index_esize(blocks, "block_ids"), requests, per_request, block_row, block_col,
         address(rows), row, address(prefixes), prefix,
         lengths.data_ptr(), index_esize(lengths, "seq_len"), len_stride, block_size,
         table.data_ptr(), index_esize(table, "request_table"), table.shape[0], table.shape[1],
         table.stride(0), table.stride(1),
         mapping.data_ptr(), index_esize(mapping, "device_mapping"), mapping.numel(), mapping.stride(0),
         int(on_host), valid.data_ptr(), physical.data_ptr(), None if masked is None else masked.data_ptr(),
         int(exclude_newest), device.index, stream_handle(device))


def resolve_shared_block_locations(block_ids: torch.Tensor, *, source_row: int, seq_len: torch.Tensor,
                                   shared_tokens: int, block_size: int, request_table: torch.Tensor,
                                   device_mapping: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Complete shared blocks -> the source request's device slots (shared_prefix.py:70-119).

    Returns ``(valid [blocks] bool, physical [blocks, block_size] int32)``.
    """
    if block_ids.ndim != 1:
        raise ValueError("block ids must be one-dimensional")
    if not _is_int(source_row) or source_row < 0 or source_row >= request_table.shape[0]:
        raise ValueError("source row is outside the request table")
    if request_table.ndim != 2 or not request_table.shape[1] or not device_mapping.numel():
        raise ValueError("shared prefix address geometry is empty")
    if not _is_int(block_size) or block_size < 1 or not _is_int(shared_tokens) or shared_tokens < 0:
        raise ValueError("invalid shared block geometry")
    device = block_ids.device
    table, mapping = _geometry(request_table, device_mapping, device)
    blocks = _index_tensor(block_ids, device)
    lengths = _index_tensor(torch.as_tensor(seq_len).reshape(-1)[:1], device)
    count = blocks.shape[0]
    valid = torch.empty(count, dtype=torch.bool, device=device)
    physical = torch.empty((count, block_size), dtype=torch.int32, device=device)
    if count:
        _launch(blocks, 1, count, 0, blocks.stride(0), None, source_row, None, shared_tokens, lengths, 0,
                block_size, table, mapping, valid, physical, None, False)
    return valid, physical


def resolve_shared_block_locations_batched(
        block_ids: torch.Tensor, *, source_rows: Iterable[int], seq_len: torch.Tensor,
        shared_tokens: Iterable[int], block_size: int, request_table: torch.Tensor,
        device_mapping: torch.Tensor, exclude_newest: bool = False,
        masked_block_ids: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Many consumers in one kernel (shared_prefix.py:122-204).

    ``block_ids`` [requests, blocks]; ``source_rows`` and ``shared_tokens`` one
    entry per request.  Returns ``(valid [requests, blocks] bool, physical
    [requests, blocks, block_size] int32)``.

    Extensions (off by default, so the reference's call is unchanged):
    ``exclude_newest`` folds in the caller's rule that the block holding the
    consumer's newest token stays on its own path (request_residency.py:220);
    ``masked_block_ids`` (same shape and dtype as ``block_ids``, may be
    ``block_ids`` itself) receives the block ids with valid blocks set to -1
    (request_residency.py:231).
    """
    fast = torch_binding()
    if fast is not None and type(block_size) is int:
        try:
            rc, valid, physical = fast.shared_blocks(block_ids, source_rows, seq_len, shared_tokens, block_size,
                                                     request_table, device_mapping, bool(exclude_newest),
                                                     masked_block_ids)
        except TypeError:  # not tensors / not sequences: the checked path below reports it
            rc = fast.NOT_HANDLED
        if rc == 0:
            return valid, physical
        if rc == fast.KERNEL_ERROR:
            raise last_error("ekv_resolve_shared_blocks")
    if block_ids.ndim != 2:
        raise ValueError("block ids must be two-dimensional")
    request_count, blocks_per_request = block_ids.shape
    if block_ids.dtype == torch.bool:
        raise ValueError("block ids must be integers")
    if block_size < 1:
        raise ValueError("invalid shared block geometry")
    if request_table.ndim != 2 or not request_table.shape[1] or not device_mapping.numel():
        raise ValueError("shared prefix address geometry is empty")
    rows, prefixes = _checked_lists(source_rows, shared_tokens, request_table.shape[0])
    device = block_ids.device
    lengths = torch.as_tensor(seq_len, device=device).reshape(-1)
    if len(rows) != request_count or len(prefixes) != request_count:
        raise ValueError("shared prefix metadata dimensions differ")
    if lengths.numel() != request_count:
        raise ValueError("sequence length dimensions differ")
    valid = torch.empty((request_count, blocks_per_request), dtype=torch.bool, device=device)
    physical = torch.empty((request_count, blocks_per_request, block_size), dtype=torch.int32, device=device)
    if request_count == 0 or blocks_per_request == 0:
        return valid, physical
    table, mapping = _geometry(request_table, device_mapping, device)
    blocks = _index_tensor(block_ids, device)
    lengths = _index_tensor(lengths, device)
    if masked_block_ids is not None and (masked_block_ids.shape != block_ids.shape
                                         or masked_block_ids.dtype != blocks.dtype
                                         or masked_block_ids.stride() != blocks.stride()
                                         or masked_block_ids.device != device):
        raise ValueError("masked_block_ids must match block_ids in shape, dtype, strides and device")
    if request_count <= SHARED_INLINE_MAX:
        # The per-request lists ride in the launch parameters: no device copy.
        meta = np.array(rows + prefixes, dtype=np.int64)
        address = meta.ctypes.data
        _launch(blocks, request_count, blocks_per_request, blocks.stride(0), blocks.stride(1),
                address, 0, address + 8 * request_count, 0, lengths, lengths.stride(0), block_size,
                table, mapping, valid, physical, masked_block_ids, exclude_newest, on_host=True)
    else:
        # One host -> device copy carries both per-request vectors.
        meta = torch.tensor(rows + prefixes, dtype=torch.int64).to(device, non_blocking=True)
        _launch(blocks, request_count, blocks_per_request, blocks.stride(0), blocks.stride(1),
                meta[:request_count], 0, meta[request_count:], 0, lengths, lengths.stride(0), block_size,
                table, mapping, valid, physical, masked_block_ids, exclude_newest)
    return valid, physical
