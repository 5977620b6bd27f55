"""Oracle for the hot-buffer swap-in (victim selection, promotion, mapped gather) -- test infrastructure only.

The reference leaves this to SGLang's block swap kernel (called from
adaptive_sparse/request_residency.py:805-809, :829-832; exercised in
tests/smoke_minimax_swap.py:28-67): hot-buffer hit test, eviction of slots not
used by the current request step, host -> device load of the missing rows.
Its eviction order (LRU) is third-party and not pinned by the reference; this
restatement defines the order the B200 kernels implement: misses in
miss-list order take the unreferenced slots in ring order from a per-row hand.
"""

from __future__ import annotations

import numpy as np


def swap_select(res_map, slot_token, hand, slots, miss_list, miss_count):
    """In-place update of res_map / slot_token / hand; returns promo_slot [B, K]."""
    batch, k = slots.shape
    hot = slot_token.shape[1]
    promo = np.full((batch, k), -1, dtype=np.int32)
    for b in range(batch):
        referenced = np.zeros(hot, dtype=bool)
        hit = slots[b][(slots[b] >= 0) & (slots[b] < hot)]
        referenced[hit] = True
        n = int(miss_count[b])
        if n == 0:
            continue
        ring = (int(hand[b]) % hot + np.arange(hot)) % hot
        free = ring[~referenced[ring]]
        victims = free[:n]
        promo[b, :victims.size] = victims
        for r, v in enumerate(victims):
            token = int(miss_list[b, r])
            old = int(slot_token[b, v])
            if 0 <= old < res_map.shape[1]:
                res_map[b, old] = -1
            if 0 <= token < res_map.shape[1]:
                res_map[b, token] = v
            slot_token[b, v] = token
        if victims.size == n:
            hand[b] = (int(victims[-1]) + 1) % hot
    return promo


def promote_rows(history, hot_rows, miss_list, miss_count, promo, context):
    """hot_rows[b, slot] <- history[b * context + token] for every assigned miss.

    ``history`` is [B * context, row] and ``hot_rows`` [B, hot, row] (one plane).
    """
    for b in range(miss_list.shape[0]):
        for r in range(int(miss_count[b])):
            slot = int(promo[b, r])
            token = int(miss_list[b, r])
            if slot >= 0 and 0 <= token < context:
                hot_rows[b, slot] = history[b * context + token]


def mapped_gather(hot_rows, res_map, topk, lengths):
    """out[b, i] = hot_rows[b, res_map[b, t]] for t = topk[b, i] valid and resident, else 0.

    A slot outside the request's hot region (< 0 or >= its capacity) reads as absent."""
    batch, k = topk.shape
    out = np.zeros((batch, k, hot_rows.shape[2]), dtype=hot_rows.dtype)
    for b in range(batch):
        for i in range(k):
            t = int(topk[b, i])
            if 0 <= t < lengths[b]:
                s = int(res_map[b, t])
                if 0 <= s < hot_rows.shape[1]:
                    out[b, i] = hot_rows[b, s]
    return out
