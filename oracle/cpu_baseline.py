"""Timed CPU baseline of the data path -- test / benchmark infrastructure only.

Multi-threaded torch-CPU restatements of the reference's CPU-capable path,
run on the host cores for the ``cpu_baseline`` leg and the ``--impl reference``
arm of bench.py:

* gather: the row selection of experimental/sparse_read.py:18-30 (indirect:
  positions -> request_table -> slot_offsets; invalid rows zero) as
  ``index_select`` over every plane;
* lookup: the reference's own torch resolver expression
  (adaptive_sparse/request_residency.py:819-826) on CPU tensors.

The reference has no CPU implementation of its Triton gather; this
restatement is the "port" baseline and is checked against the numpy oracle
in tests.
"""

from __future__ import annotations

import torch


def gather_planes(planes, positions, request_ids, lengths, request_table, slot_offsets, width, outputs):
    """``outputs[p][b, i] = planes[p][slot_offsets[table[req, pos]] // width]`` or 0.

    ``planes[p]`` is [slots, width] (any dtype), ``outputs[p]`` [B, S, width].
    Offsets must be whole rows (multiples of ``width``), as in the benchmark layout.
    """
    pos = positions.to(torch.int64)
    valid = (pos >= 0) & (pos < lengths.to(torch.int64)[:, None])
    safe = torch.where(valid, pos, torch.zeros_like(pos))
    logical = request_table[request_ids.to(torch.int64)[:, None], safe]
    rows = torch.div(slot_offsets[logical], width, rounding_mode="floor")
    rows = torch.where(valid, rows, torch.zeros_like(rows)).reshape(-1)
    invalid = ~valid.reshape(-1)
    any_invalid = bool(invalid.any())
    for plane, out in zip(planes, outputs):
        flat = out.view(-1, width)
        torch.index_select(plane, 0, rows, out=flat)
        if any_invalid:
            flat[invalid] = 0


def torch_resolver(topk, table, mapping, rows, lengths, selected, result, block_size):
    """The reference's torch resolver (request_residency.py:819-826) on any device."""
    blocks = topk[0, selected].long()
    positions = blocks.unsqueeze(-1) * block_size + torch.arange(block_size, device=rows.device)
    positions = positions.flatten(1)
    valid = (positions >= 0) & (positions < lengths[selected, None])
    logical = table[rows[selected, None], positions.masked_fill(~valid, 0)]
    result[0, selected] = mapping[logical].masked_fill(~valid, -1).to(torch.int32)


def torch_shared_resolver(block_ids, rows, prefixes, seq_len, block_size, request_table, device_mapping):
    """The reference's batched shared-prefix resolver expression
    (adaptive_sparse/shared_prefix.py:188-204) on any device; rows / prefixes are
    int64 tensors."""
    blocks = block_ids.to(torch.long)
    starts = blocks * block_size
    ends = starts + block_size
    valid = (blocks >= 0) & (ends <= prefixes.reshape(-1, 1)) & (ends <= seq_len.reshape(-1, 1))
    positions = starts.unsqueeze(2) + torch.arange(block_size, device=blocks.device, dtype=torch.long)
    safe_positions = positions.clamp(0, request_table.shape[1] - 1)
    logical = request_table[rows.reshape(-1, 1, 1), safe_positions]
    safe_logical = logical.clamp(0, device_mapping.numel() - 1)
    physical = device_mapping[safe_logical]
    valid = valid & (logical >= 0).all(dim=2) & (physical > 0).all(dim=2)
    return valid, physical.to(torch.int32)


def torch_shadow_check(k, v, initialized, k_cache, v_cache, table, lengths, rows, block_size, blocks, physical,
                       live_pages, page_size):
    """The reference's LogicalShadow.check body (adaptive_sparse/logical_shadow.py:50-86) as
    plain torch ops on any device; returns (counts [7], clean_blocks, physical_out)."""
    capacity = k.shape[0]
    block_limit = (lengths[:, None] + block_size - 1) // block_size
    valid_blocks = (blocks >= 0) & (blocks < block_limit)
    prefix = valid_blocks.to(torch.int32).cumprod(-1).bool()
    malformed = ((blocks != -1) & ~valid_blocks) | (valid_blocks & ~prefix)
    clean_blocks = blocks.masked_fill(~prefix, -1)
    ids = clean_blocks[0].long()
    positions = (ids[..., None] * block_size + torch.arange(block_size, device=ids.device)).flatten(1)
    selected = (positions >= 0) & (positions < lengths[:, None])
    bounded = selected & (positions < table.shape[1])
    logical = table[rows[:, None], positions.masked_fill(~bounded, 0)].long()
    logical_valid = bounded & (logical >= page_size) & (logical < capacity)
    logical = logical.masked_fill(~logical_valid, 0)
    source_valid = logical_valid & initialized[logical]
    physical = logical if physical is None else physical[0].long()
    in_range = (physical >= page_size) & (physical < k_cache.shape[0])
    safe = physical.masked_fill(~in_range, 0)
    backed = in_range if live_pages is None else in_range & live_pages[safe // page_size]
    safe = safe.masked_fill(~backed, 0)
    same_k = (k_cache[safe].reshape(*safe.shape, -1).view(torch.int16)
              == k[logical].reshape(*safe.shape, -1).view(torch.int16)).all(-1)
    same_v = (v_cache[safe].reshape(*safe.shape, -1).view(torch.int16)
              == v[logical].reshape(*safe.shape, -1).view(torch.int16)).all(-1)
    checked = selected & source_valid & backed
    tokens = checked.sum()
    bytes_per_token = (k[0].numel() + v[0].numel()) * 2
    counts = torch.stack((tokens, tokens * bytes_per_token, (selected & ~source_valid).sum(),
                          (selected & ~backed).sum(), (checked & ~(same_k & same_v)).sum(),
                          tokens.new_ones(()), malformed.sum()))
    return counts, clean_blocks, physical.masked_fill(selected & ~backed, 0).to(torch.int32).unsqueeze(0)
