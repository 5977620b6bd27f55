"""Oracle for the residency lookups (R1, R1', R2) -- test infrastructure only."""

from __future__ import annotations

import numpy as np


def resolve_resident(topk, table, mapping, rows, lengths, selected, output, block_size):
    """Restates the Triton ``_resolve`` kernel, adaptive_sparse/resident_lookup.py:6-40.

    Arrays are numpy (any strides): topk [1, B, K], table [R, T], mapping [N],
    rows [B], lengths [B], selected [n], output [1, B, K * block_size] int32,
    modified in place.  Only rows listed in ``selected`` are written
    (resident_lookup.py:14, :26); an empty selection or zero width is a no-op
    (:31-33).
    """
    width = topk.shape[2] * block_size
    if not selected.size or not width:
        return
    sel = selected.astype(np.int64)
    j = np.arange(width, dtype=np.int64)
    block = topk[0][sel[:, None], j[None, :] // block_size].astype(np.int64)      # :17-18
    position = block * block_size + j[None, :] % block_size                      # :19
    length = lengths[sel].astype(np.int64)[:, None]                               # :20
    req = rows[sel].astype(np.int64)[:, None]                                     # :21
    valid = (block >= 0) & (position < length)                                    # :22
    safe_pos = np.where(valid, position, 0)
    logical = np.where(valid, table[np.broadcast_to(req, safe_pos.shape), safe_pos], 0)  # :23-24
    physical = np.where(valid, mapping[logical.astype(np.int64)].astype(np.int64), -1)   # :25
    output[0, sel, :] = physical.astype(np.int64).astype(np.int32)               # :26 (int32 store)


def torch_resolver_numpy(topk, table, mapping, rows, lengths, selected, block_size):
    """Restates the reference's torch resolver, adaptive_sparse/request_residency.py:819-826.

    Returns the [n, K * block_size] int32 rows it assigns to ``result[resident]``.
    """
    blocks = topk[0, selected].astype(np.int64)
    positions = (blocks[..., None] * block_size + np.arange(block_size)).reshape(len(selected), -1)
    valid = (positions >= 0) & (positions < lengths[selected].astype(np.int64)[:, None])
    logical = table[rows[selected].astype(np.int64)[:, None], np.where(valid, positions, 0)]
    return np.where(valid, mapping[logical.astype(np.int64)], -1).astype(np.int64).astype(np.int32)


def lookup_slots(res_map, topk, lengths=None):
    """R2: token ids -> hot slots with miss mask and per-row compacted miss list.

    No single reference symbol: R1 with ``mapping`` replaced by a per-request
    residency map (-1 = not resident), plus the hit/miss contract of the swap
    kernel exercised in tests/smoke_minimax_swap.py:28-62.  Compaction order
    (ascending Top-K column) and the -1 padding are defined by this build.
    Returns (slots int32 [B,K], miss bool [B,K], miss_list int32 [B,K], miss_count int32 [B]).
    """
    batch, k = topk.shape
    width = res_map.shape[1]
    limit = np.full(batch, width, dtype=np.int64)
    if lengths is not None:
        limit = np.minimum(limit, lengths.astype(np.int64))
    token = topk.astype(np.int64)
    valid = (token >= 0) & (token < limit[:, None])
    rows = np.broadcast_to(np.arange(batch)[:, None], token.shape)
    slot64 = np.where(valid, res_map[rows, np.where(valid, token, 0)].astype(np.int64), -1)
    miss = valid & (slot64 < 0)
    miss_list = np.full((batch, k), -1, dtype=np.int32)
    miss_count = miss.sum(axis=1).astype(np.int32)
    for b in range(batch):
        found = token[b][miss[b]]
        miss_list[b, :found.size] = found
    return slot64.astype(np.int32), miss, miss_list, miss_count
