"""Oracle for the Top-K row gather (R3) -- test infrastructure only."""

from __future__ import annotations

import numpy as np


def row_offsets(positions, request_ids, lengths, request_table, slot_offsets, *, width,
                table_width, request_stride, sink_elements, indirect, mapped=False):
    """Element offset of every (b, i) row and its validity.

    Restates experimental/sparse_read.py:18-30: valid iff 0 <= pos < lengths[b]
    (:22); indirect offset = slot_offsets[request_table[req * table_width + pos]]
    (:24-26); direct offset = sink + req * request_stride + pos * width (:28).
    ``mapped`` is this build's third mode (no reference counterpart): the table
    holds the row's slot s in the request's fixed region, valid only when
    pos < table_width (the map's row width), 0 <= s and (s + 1) * width <=
    request_stride; offset = sink + req * request_stride + s * width.
    """
    pos = positions.astype(np.int64)
    req = request_ids.astype(np.int64)[:, None]
    valid = (pos >= 0) & (pos < lengths.astype(np.int64)[:, None])
    if mapped:
        valid &= pos < table_width
        flat = request_table.reshape(-1).astype(np.int64)
        slot = np.where(valid, flat[np.where(valid, req * table_width + pos, 0)], -1)
        valid &= (slot >= 0) & ((slot + 1) * width <= request_stride)
        offset = np.where(valid, sink_elements + req * request_stride + slot * width, 0)
    elif indirect:
        flat = request_table.reshape(-1)
        logical = np.where(valid, flat[np.where(valid, req * table_width + pos, 0)], 0)
        offset = np.where(valid, slot_offsets.reshape(-1)[logical.astype(np.int64)].astype(np.int64), 0)
    else:
        offset = np.where(valid, sink_elements + req * request_stride + pos * width, 0)
    return offset, valid


def gather_rows(raw, positions, request_ids, lengths, request_table, slot_offsets, *, width,
                table_width, request_stride, sink_elements, indirect, mapped=False):
    """``out[b, i, :] = raw[off : off + width]`` for valid rows, else 0 (sparse_read.py:29-30).

    ``raw`` is a 1-D numpy array in the payload's element type (bf16 payloads
    are handled as uint16 bit patterns).
    """
    offset, valid = row_offsets(positions, request_ids, lengths, request_table, slot_offsets,
                                width=width, table_width=table_width,
                                request_stride=request_stride, sink_elements=sink_elements,
                                indirect=indirect, mapped=mapped)
    batch, selected = positions.shape
    out = np.zeros((batch, selected, width), dtype=raw.dtype)
    vb, vi = np.nonzero(valid)
    if vb.size:
        starts = offset[vb, vi]
        if raw.size % width == 0 and not np.any(starts % width):
            out[vb, vi] = raw.reshape(-1, width)[starts // width]
        else:
            out[vb, vi] = raw[starts[:, None] + np.arange(width)]
    return out


def gather_rows_planes(planes, positions, request_ids, lengths, request_table, slot_offsets, **kw):
    """``gather_rows`` applied to each plane with the same row selection."""
    return [gather_rows(plane, positions, request_ids, lengths, request_table, slot_offsets, **kw)
            for plane in planes]
