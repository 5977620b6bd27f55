"""B200-native sparse-KV residency data path.

Drop-in replacements for the data path of elastic-kv-vmm:

* ``resident_lookup.resolve_resident`` / ``lookup_slots`` -- residency lookups;
* ``sparse_read.gather_rows`` / ``gather_rows_planes`` -- Top-K K/V row gather;
* ``migration`` -- demote/promote transactions over ``host_pool.PinnedHostKVPool``;
* ``releasable`` -- per-chunk freeable bitmaps and their cross-rank AND;
* ``backing.Backing`` -- chunked CUDA VMM reservation (ev_* ABI).

All compute runs in libekv_b200.so (hand-written sm_100a kernels); build it
with ``python -m ekv_b200.build``.
"""

from ._lib import KernelError, LIBRARY_PATH, library

__all__ = ["KernelError", "LIBRARY_PATH", "library"]
