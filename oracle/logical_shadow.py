"""Oracle for the logical-shadow checks -- test infrastructure only.

Restates the two comparisons of LogicalShadow (adaptive_sparse/logical_shadow.py):

* ``check`` (:45-86): the Top-K blocks of one decode step are cleaned (the
  valid prefix of each row is kept, the rest becomes -1, malformed ids are
  counted), their positions resolve through the request table to logical
  slots, and every selected token whose logical slot holds a recorded shadow
  write and whose physical slot is backed has its K and V rows compared
  bit for bit with the shadow;
* ``check_complete`` (:88-123): after a migration, every (logical, physical)
  slot pair of every layer of the pool compares the pool's rows with the shadow.

Rows are int16 views of the bf16 data (the reference compares ``view(torch.int16)``).
"""

from __future__ import annotations

import numpy as np


def check(k_shadow, v_shadow, initialized, k_cache, v_cache, table, lengths, rows, block_size,
          blocks, physical, live_pages, page_size):
    """Returns (counts int64 [7], clean_blocks [1,B,K], physical_out int32 [1,B,K*bs]).

    counts = checked_tokens, checked_bytes, uninitialized_logical_tokens,
    invalid_physical_tokens, mismatched_tokens, checked_calls (1),
    malformed_topk_blocks (logical_shadow.py:79-83).
    """
    capacity = k_shadow.shape[0]
    lengths = np.asarray(lengths).astype(np.int64)
    blocks_in = np.asarray(blocks)
    b64 = blocks_in.astype(np.int64)
    block_limit = (lengths[:, None] + block_size - 1) // block_size                  # :50
    valid_blocks = (b64 >= 0) & (b64 < block_limit)                                  # :51
    prefix = np.cumprod(valid_blocks.astype(np.int32), axis=-1).astype(bool)          # :52
    malformed = ((b64 != -1) & ~valid_blocks) | (valid_blocks & ~prefix)             # :53
    clean_blocks = np.where(prefix, blocks_in, np.asarray(-1, dtype=blocks_in.dtype))  # :54
    cb = clean_blocks[0].astype(np.int64)                                            # :55
    with np.errstate(over="ignore"):
        positions = (cb[..., None] * block_size + np.arange(block_size)).reshape(cb.shape[0], -1)  # :56-57
    selected = (positions >= 0) & (positions < lengths[:, None])                     # :58
    table = np.asarray(table)
    bounded = selected & (positions < table.shape[1])                                 # :59
    rows64 = np.asarray(rows).astype(np.int64)
    logical = table[rows64[:, None], np.where(bounded, positions, 0)].astype(np.int64)  # :60
    logical_valid = bounded & (logical >= page_size) & (logical < capacity)          # :61
    logical = np.where(logical_valid, logical, 0)                                    # :62
    source_valid = logical_valid & np.asarray(initialized)[logical]                  # :63

    phys = logical if physical is None else np.asarray(physical)[0].astype(np.int64)  # :65
    in_range = (phys >= page_size) & (phys < k_cache.shape[0])                       # :66
    safe = np.where(in_range, phys, 0)                                               # :67
    backed = in_range if live_pages is None else in_range & np.asarray(live_pages)[safe // page_size]  # :68
    safe = np.where(backed, safe, 0)                                                 # :69
    flat = lambda a, idx: a[idx].reshape(*idx.shape, -1)                            # noqa: E731
    same_k = (flat(k_cache, safe) == flat(k_shadow, logical)).all(-1)                # :72-73
    same_v = (flat(v_cache, safe) == flat(v_shadow, logical)).all(-1)                # :74-75
    checked = selected & source_valid & backed                                       # :76
    tokens = int(checked.sum())
    bytes_per_token = (k_shadow[0].size + v_shadow[0].size) * 2                      # :78
    counts = np.array([tokens, tokens * bytes_per_token, int((selected & ~source_valid).sum()),
                       int((selected & ~backed).sum()), int((checked & ~(same_k & same_v)).sum()), 1,
                       int(malformed.sum())], dtype=np.int64)                        # :79-83
    physical_out = np.where(selected & ~backed, 0, phys).astype(np.int32)[None]      # :85-86
    return counts, clean_blocks, physical_out


def check_complete(layers, pool_keys, pool_values, logical, physical, page_size, pool_size, live_pages,
                   capacity):
    """Migration check (logical_shadow.py:88-123) over the pool's layers.

    ``layers`` = [(k_shadow, v_shadow, initialized), ...] in the pool's layer
    order, ``pool_keys`` / ``pool_values`` the pool buffers of the same layers,
    ``live_pages`` bool [pool_size // page_size + 1].  Returns int64 [4] =
    checked tokens, checked bytes, invalid tokens, mismatched tokens.
    """
    logical = np.asarray(logical).astype(np.int64)
    physical = np.asarray(physical).astype(np.int64)
    logical_valid = (logical >= page_size) & (logical < capacity)                    # :96
    physical_valid = (physical >= page_size) & (physical < pool_size + page_size)    # :97
    safe_logical = np.where(logical_valid, logical, 0)
    safe_physical = np.where(physical_valid, physical, 0)
    physical_valid &= np.asarray(live_pages)[safe_physical // page_size]             # :100
    safe_physical = np.where(physical_valid, safe_physical, 0)
    counts = np.zeros(4, dtype=np.int64)
    for (key, value, initialized), pool_k, pool_v in zip(layers, pool_keys, pool_values):
        valid = logical_valid & physical_valid & np.asarray(initialized)[safe_logical]  # :107
        actual_k = pool_k[safe_physical].reshape(len(logical), -1)
        actual_v = pool_v[safe_physical].reshape(len(logical), -1)
        expected_k = key[safe_logical].reshape(len(logical), -1)
        expected_v = value[safe_logical].reshape(len(logical), -1)
        equal = (actual_k == expected_k).all(1) & (actual_v == expected_v).all(1)     # :112
        checked = int(valid.sum())
        counts += np.array([checked, checked * 2 * (expected_k.shape[1] + expected_v.shape[1]),
                            int((~valid).sum()), int((valid & ~equal).sum())], dtype=np.int64)  # :114-117
    return counts
