"""Oracle for the shared-prefix donor-slot resolution -- test infrastructure only.

Restates adaptive_sparse/shared_prefix.py of the reference:

* ``complete_shared_blocks`` (:36-67): which Top-K blocks lie wholly inside
  the shared prefix and the consumer's sequence;
* ``resolve_shared_block_locations`` (:70-119) and its batched form
  (:122-204): complete shared blocks -> the SOURCE request's logical slots
  (request_table[source_row, position]) -> device slots (device_mapping),
  valid only when every position of the block is mapped to a live slot
  (logical >= 0 and physical > 0 for the whole block).

Positions and logical ids are clamped before they index (:114-116, :199-201),
so ``physical`` holds a value for every block, valid or not; the int64 ->
int32 cast wraps (two's complement).  The caller at
adaptive_sparse/request_residency.py:210-220 further drops the block holding
the consumer's newest token (``exclude_newest`` here).
"""

from __future__ import annotations

import numpy as np


def complete_shared_blocks(block_ids, seq_len, shared_tokens, block_size):
    """Tuple of bools, shared_prefix.py:59-67 (argument checks are the host mirror's)."""
    out = []
    for block in block_ids:
        start = block * block_size
        out.append(block >= 0 and start + block_size <= shared_tokens and start + block_size <= seq_len)
    return tuple(out)


def _wrap_i64(values):
    return np.asarray(values).astype(np.int64)


def resolve_batched(block_ids, source_rows, seq_len, shared_tokens, block_size, request_table,
                    device_mapping, exclude_newest=False):
    """Batched resolution, shared_prefix.py:188-204.

    block_ids [R, B] (int), source_rows [R], seq_len [R], shared_tokens [R];
    request_table [rows, T]; device_mapping [N].  Returns (valid bool [R, B],
    physical int32 [R, B, block_size]).
    """
    blocks = _wrap_i64(block_ids)
    requests, per_request = blocks.shape
    if requests == 0:
        return (np.zeros((0, per_request), dtype=bool),
                np.zeros((0, per_request, block_size), dtype=np.int32))
    rows = _wrap_i64(source_rows).reshape(-1, 1)
    prefixes = _wrap_i64(shared_tokens).reshape(-1, 1)
    lengths = _wrap_i64(seq_len).reshape(-1, 1)
    with np.errstate(over="ignore"):
        starts = blocks * np.int64(block_size)                                    # :189
        ends = starts + np.int64(block_size)                                      # :190
        valid = (blocks >= 0) & (ends <= prefixes) & (ends <= lengths)            # :191-195
        positions = starts[:, :, None] + np.arange(block_size, dtype=np.int64)    # :196-198
    table = np.asarray(request_table)
    mapping = np.asarray(device_mapping)
    safe_positions = np.clip(positions, 0, table.shape[1] - 1)                     # :199
    logical = table[rows[:, :, None], safe_positions].astype(np.int64)            # :200
    safe_logical = np.clip(logical, 0, mapping.size - 1)
    physical = mapping[safe_logical].astype(np.int64)
    valid &= (logical >= 0).all(axis=2) & (physical > 0).all(axis=2)
    if exclude_newest:
        # request_residency.py:220 -- the consumer's newest token stays on its own path.
        with np.errstate(over="ignore"):
            valid &= (blocks + 1) * np.int64(block_size) < lengths
    return valid, physical.astype(np.int32)


def resolve_scalar(block_ids, source_row, seq_len, shared_tokens, block_size, request_table,
                   device_mapping):
    """Single-consumer resolution, shared_prefix.py:107-119 (one row of the batched form)."""
    valid, physical = resolve_batched(np.asarray(block_ids).reshape(1, -1), [source_row],
                                      [int(seq_len)], [shared_tokens], block_size, request_table,
                                      device_mapping)
    return valid[0], physical[0]
