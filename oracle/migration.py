"""Oracle for demote/promote row movement (R5) -- test infrastructure only.

The reference delegates the bytes to SGLang's host pool
(backup_from_device_all_layer at adaptive_sparse/migration.py:109-111: every
layer, K and V, rows ``physical[:len]`` -> host rows; load_to_device_per_layer
at :231-234: host rows -> ``destination[:host_len]`` per layer).  The
restatement is a row copy by slot index.  Migration parity is bitwise equality
of every moved row at source and destination, the comparison the reference's
logical-shadow checker makes (adaptive_sparse/logical_shadow.py:88-123).
Planes and staging are numpy uint8 arrays of shape [rows, row_bytes].
"""

from __future__ import annotations

import numpy as np


def _tasks(n_planes, slots, plane_index, stage_rows):
    slots = np.asarray(slots, dtype=np.int64)
    if plane_index is None:
        planes = np.repeat(np.arange(n_planes), slots.size)
        task_slots = np.tile(slots, n_planes)
        rows = (np.tile(np.asarray(stage_rows, np.int64), n_planes) if stage_rows is not None
                else np.tile(np.arange(slots.size), n_planes))
        return planes, task_slots, rows, True
    rows = np.asarray(stage_rows, np.int64) if stage_rows is not None else np.arange(slots.size)
    return np.asarray(plane_index, np.int64), slots, rows, False


def pack_rows(planes, slots, staging, *, plane_index=None, stage_rows=None, stage_plane_rows=0):
    """Rows of ``planes`` at ``slots`` -> ``staging`` (rows of the same width).

    Cross form: plane p, slot j -> staging row ``p * stage_plane_rows + stage_rows[j]``.
    List form: task t -> staging row ``stage_rows[t]`` (or t).
    """
    p, s, r, cross = _tasks(len(planes), slots, plane_index, stage_rows)
    dest = p * stage_plane_rows + r if cross else r
    for plane in range(len(planes)):
        pick = p == plane
        staging[dest[pick]] = planes[plane][s[pick]]


def unpack_rows(planes, slots, staging, *, plane_index=None, stage_rows=None, stage_plane_rows=0):
    """Inverse of ``pack_rows``."""
    p, s, r, cross = _tasks(len(planes), slots, plane_index, stage_rows)
    src = p * stage_plane_rows + r if cross else r
    for plane in range(len(planes)):
        pick = p == plane
        planes[plane][s[pick]] = staging[src[pick]]
