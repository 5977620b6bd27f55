"""The chunked VMM backing on a real device: commit, zero fill, view, reclaim, recommit, ABI."""

from __future__ import annotations

import ctypes as ct

import pytest
import torch

pytestmark = pytest.mark.gpu

CHUNK = 2 << 20


def test_backing_lifecycle(cuda_device):
    from ekv_b200.backing import Backing

    backing = Backing(10 * CHUNK + 123, CHUNK, device=cuda_device.index)
    try:
        assert backing.reserved_bytes == 11 * CHUNK and backing.granularity <= CHUNK
        assert backing.base % CHUNK == 0 and backing.backed_bytes == 0
        with pytest.raises(RuntimeError, match="sink"):
            backing.raw
        assert backing.ensure({0, 3, 4}) == 3
        assert backing.backed_bytes == 3 * CHUNK
        raw = backing.raw
        assert raw.data_ptr() == backing.base and raw.numel() == backing.capacity_bytes
        assert raw.device == cuda_device
        assert not raw[3 * CHUNK:5 * CHUNK].any()  # zero-filled on commit
        raw[3 * CHUNK:5 * CHUNK].fill_(0xAB)
        torch.cuda.synchronize()
        assert backing.reclaim({4}) == 1 and backing.backed_bytes == 2 * CHUNK
        assert int(raw[3 * CHUNK]) == 0xAB
        assert backing.ensure({4}) == 1
        assert not raw[4 * CHUNK:5 * CHUNK].any()  # a recommitted chunk is fresh memory
        assert backing.precommit({7, 8}) == 2
        assert backing.mapped_chunks == {0, 3, 4}
        assert backing.ensure({7}) == 0 and backing.mapped_chunks == {0, 3, 4, 7, 8}
        assert not raw[7 * CHUNK:9 * CHUNK].any()
        with pytest.raises(ValueError):
            backing.ensure({11})
        del raw
    finally:
        torch.cuda.synchronize()
        backing.close()
    with pytest.raises(RuntimeError):
        backing.ensure({1})


def test_backing_rejects_unaligned_chunk(cuda_device):
    from ekv_b200.backing import Backing

    with pytest.raises(RuntimeError, match="granularity"):
        Backing(8 * CHUNK, CHUNK + 4096, device=cuda_device.index)


def test_reference_ctypes_binding_loads_this_library(cuda_device, library_path):
    """Bind the ev_* ABI with the argument types of elastic_kv/backing.py:19-52."""
    lib = ct.CDLL(str(library_path))
    lib.ev_create.argtypes = [ct.c_int, ct.c_uint64, ct.c_uint64]
    lib.ev_create.restype = ct.c_void_p
    for name in ("ev_ensure", "ev_precommit", "ev_drop"):
        fn = getattr(lib, name)
        fn.argtypes = [ct.c_void_p, ct.POINTER(ct.c_uint64), ct.c_size_t]
        fn.restype = ct.c_int
    for name in ("ev_base", "ev_backed", "ev_reserved", "ev_granularity"):
        fn = getattr(lib, name)
        fn.argtypes = [ct.c_void_p]
        fn.restype = ct.c_uint64
    lib.ev_poisoned.argtypes = [ct.c_void_p]
    lib.ev_poisoned.restype = ct.c_int
    lib.ev_close.argtypes = [ct.c_void_p]
    lib.ev_close.restype = ct.c_int
    lib.ev_error.restype = ct.c_char_p
    handle = lib.ev_create(cuda_device.index, 4 * CHUNK, CHUNK)
    assert handle, lib.ev_error()
    ids = (ct.c_uint64 * 2)(2, 1)
    assert lib.ev_ensure(handle, ids, 2) == 0
    assert lib.ev_backed(handle) == 2 * CHUNK
    bad = (ct.c_uint64 * 1)(9)
    assert lib.ev_ensure(handle, bad, 1) == -1 and b"outside" in lib.ev_error()
    assert lib.ev_poisoned(handle) == 0
    assert lib.ev_drop(handle, ids, 2) == 0 and lib.ev_backed(handle) == 0
    assert lib.ev_close(handle) == 0


def test_spare_handles_are_reused_and_zeroed(cuda_device):
    """Reclaimed physical handles kept under the spare limit come back through the next
    ensure: the chunk reads as zeros again (the zero fill runs for reused handles too),
    spare memory is reported apart from the backed bytes, and lowering the limit or
    closing releases it."""
    from ekv_b200.backing import Backing

    backing = Backing(16 * CHUNK, CHUNK, device=cuda_device.index, spare_chunks=3)
    try:
        assert backing.ensure({0, 1, 2, 3, 4}) == 5
        raw = backing.raw
        raw[CHUNK:5 * CHUNK].fill_(0x5A)
        torch.cuda.synchronize()
        assert backing.reclaim({1, 2, 3, 4}) == 4
        assert backing.spare_bytes == 3 * CHUNK and backing.backed_bytes == CHUNK
        assert backing.ensure({9, 10}) == 2
        assert backing.spare_bytes == CHUNK and backing.backed_bytes == 3 * CHUNK
        assert not raw[9 * CHUNK:11 * CHUNK].any()  # reused handles are zero-filled
        raw[9 * CHUNK:11 * CHUNK].fill_(7)
        torch.cuda.synchronize()
        assert int(raw[10 * CHUNK + 5]) == 7
        assert backing.metrics["spare_bytes"] == CHUNK
        backing.set_spare_chunks(0)
        assert backing.spare_bytes == 0
        assert backing.ensure({12}) == 1 and not raw[12 * CHUNK:13 * CHUNK].any()
        backing.set_spare_chunks(8)
        assert backing.reclaim({9, 10, 12}) == 3 and backing.spare_bytes == 3 * CHUNK
        del raw
    finally:
        torch.cuda.synchronize()
        backing.close()  # releases the kept handles too


def test_captured_gather_survives_reclaim_and_recommit(cuda_device):
    """A CUDA graph captured over the VMM-backed pool keeps working across a reclaim and a
    recommit of one chunk: the virtual addresses it captured stay valid, rows that avoid
    the reclaimed chunk still gather, and after the recommit the chunk reads as its new
    contents (as tests/test_graph_backing.py:9-51 of the reference checks for index_select)."""
    from ekv_b200.backing import Backing
    from ekv_b200.sparse_read import PlaneGather
    from ekv_b200.virtual_layout import VirtualKVLayout

    layout = VirtualKVLayout(2, 2048, 512, itemsize=2, chunk_bytes=CHUNK)  # one chunk per request region
    backing = Backing(layout.capacity_bytes, CHUNK, device=cuda_device.index)
    try:
        backing.ensure({0, 1, 2})
        plane = backing.raw.view(torch.int16)
        base = backing.raw.data_ptr()
        rows = plane[CHUNK // 2:].view(2, 2048, 512)
        rows[0] = torch.arange(2048, device=cuda_device, dtype=torch.int16)[:, None]
        rows[1] = -torch.arange(2048, device=cuda_device, dtype=torch.int16)[:, None]
        positions = torch.tensor([[5, 9, 2047, 0], [7, 1, 100, 3]], dtype=torch.int64, device=cuda_device)
        request_ids = torch.tensor([0, 1], dtype=torch.int64, device=cuda_device)
        lengths = torch.tensor([2048, 2048], dtype=torch.int64, device=cuda_device)
        out = torch.empty((2, 4, 512), dtype=torch.int16, device=cuda_device)
        gather = PlaneGather([plane], positions, request_ids, lengths, None, None, [out], layout, indirect=False)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gather()

        def replay(pos, want_first):
            positions.copy_(torch.tensor(pos, dtype=torch.int64, device=cuda_device))
            graph.replay()
            torch.cuda.synchronize()
            assert out[:, :, 0].tolist() == want_first
            assert backing.raw.data_ptr() == base

        replay([[5, 9, 2047, 0], [7, 1, 100, 3]], [[5, 9, 2047, 0], [-7, -1, -100, -3]])
        assert backing.reclaim({2}) == 1 and backing.mapped_chunks == {0, 1}
        # Request 1's rows are invalid (-1): they read as zeros without touching its chunk.
        replay([[4, 3, 2, 1], [-1, -1, -1, -1]], [[4, 3, 2, 1], [0, 0, 0, 0]])
        assert backing.ensure({2}) == 1
        rows = backing.raw.view(torch.int16)[CHUNK // 2:].view(2, 2048, 512)
        assert not rows[1].any()  # recommitted memory is zero-filled
        rows[1] = 3000
        replay([[1, 1, 1, 1], [0, 5, 2047, 9]], [[1, 1, 1, 1], [3000, 3000, 3000, 3000]])
        del graph, plane, rows
    finally:
        torch.cuda.synchronize()
        backing.close()
