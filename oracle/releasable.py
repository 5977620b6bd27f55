"""Oracle for page -> chunk projection and releasable chunks (R4, R6) -- test infrastructure only."""

from __future__ import annotations

from collections import Counter

import numpy as np


def page_chunks(page, planes, page_size, chunk_bytes):
    """PhysicalPages.chunks, adaptive_sparse/minimax_vmm.py:40-52."""
    found = set()
    for first_chunk, row_bytes in planes:
        begin = page * page_size * row_bytes
        end = begin + page_size * row_bytes - 1
        found.update(range(first_chunk + begin // chunk_bytes, first_chunk + end // chunk_bytes + 1))
    return frozenset(found)


def chunk_release_counts(chunks_of, pages):
    """_chunk_release_counts, adaptive_sparse/scheduler_budget.py:155-156 (pages as a set)."""
    return Counter(chunk for page in set(pages) for chunk in chunks_of(page))


def releasable_counts(refs, mapped, counts):
    """_releasable_counts, adaptive_sparse/scheduler_budget.py:159-162."""
    return {chunk for chunk, count in counts.items() if count == refs.get(chunk) and chunk in mapped}


def releasable(chunks_of, refs, mapped, pages):
    """_releasable, adaptive_sparse/scheduler_budget.py:151-152."""
    return releasable_counts(refs, mapped, chunk_release_counts(chunks_of, pages))


def releasable_group(chunks_of, refs, mapped, candidates):
    """_releasable_group, adaptive_sparse/scheduler_budget.py:172-189: union of page sets."""
    union = set()
    for pages in candidates:
        union.update(pages)
    return releasable(chunks_of, refs, mapped, union)


def joint_releasable(per_rank):
    """Chunks releasable on every rank: the intersection the reference's
    cross-rank agreement applies to candidate keys (runtime_value.py:180-185)."""
    ranks = [set(r) for r in per_rank]
    return set.intersection(*ranks) if ranks else set()


# ---- vectorised forms (device-kernel restatements) ---------------------------

def chunk_counts_np(pages, planes, page_size, chunk_bytes, n_chunks):
    """Histogram of chunks over (distinct) pages x planes; int32 [n_chunks]."""
    counts = np.zeros(n_chunks, dtype=np.int64)
    pages = np.asarray(pages, dtype=np.int64)
    for first_chunk, row_bytes in planes:
        span = page_size * row_bytes
        begin = pages * span
        lo = first_chunk + begin // chunk_bytes
        hi = first_chunk + (begin + span - 1) // chunk_bytes
        for step in range(int((hi - lo).max(initial=0)) + 1):
            c = lo + step
            c = c[c <= hi]
            c = c[(c >= 0) & (c < n_chunks)]
            np.add.at(counts, c, 1)
    return counts.astype(np.int32)


def bits_of(chunks, n_chunks):
    """uint64 words (as int64) with the bits of ``chunks`` set."""
    words = np.zeros((n_chunks + 63) // 64, dtype=np.uint64)
    for c in chunks:
        words[c // 64] |= np.uint64(1) << np.uint64(c % 64)
    return words.view(np.int64)


def chunks_of_bits(words):
    words = np.asarray(words).view(np.uint64)
    out = set()
    for w, value in enumerate(words.tolist()):
        while value:
            low = value & -value
            out.add(w * 64 + low.bit_length() - 1)
            value ^= low
    return out


def freeable_bitmap_np(counts, refs, mapped_words):
    """Bit c = counts[c] > 0 and counts[c] == refs[c] and c mapped."""
    n = counts.size
    hit = (counts > 0) & (counts == refs)
    return bits_of(np.nonzero(hit)[0].tolist(), n) & np.asarray(mapped_words, dtype=np.int64)


def bitmap_and_np(gathered):
    out = np.bitwise_and.reduce(np.asarray(gathered, dtype=np.int64), axis=0)
    return out
