"""The staged demotion entry point that allocates nothing (ekv_pack_rows_staged_noalloc).

Callers that cannot allocate device memory when they demote -- an engine whose
KV pool reserved all of HBM up front, so the pressure that triggers the
demotion leaves nothing to allocate from, or a host with no device allocator of
its own -- use this entry point: it stages rows through a ring built into the
library instead of a scratch buffer the caller passes in.  This file is named
to be collected last; it checks the new entry point, called through the C ABI,
against the existing ekv_pack_rows_staged on two calls in a row (bit exact).
"""

from __future__ import annotations

import ctypes as ct

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bind(library_path):
    lib = ct.CDLL(str(library_path))
    fn = lib.ekv_pack_rows_staged_noalloc
    p, i32, i64 = ct.c_void_p, ct.c_int, ct.c_int64
    fn.argtypes = [ct.POINTER(ct.c_uint64), i32, i64, p, p, i32, i64,
                   ct.POINTER(ct.c_int64), i64, p, i64, i32, p, p]
    fn.restype = ct.c_int
    lib.ekv_error.restype = ct.c_char_p
    return lib, fn


def _case(gen, device, n_planes, rows, row_bytes, count):
    planes = [torch.randint(0, 256, (rows, row_bytes), generator=gen, dtype=torch.int32)
              .to(torch.uint8).to(device) for _ in range(n_planes)]
    plane_index = torch.randint(0, n_planes, (count,), generator=gen).to(torch.int32).to(device)
    slots = torch.randint(0, rows, (count,), generator=gen).to(device)
    # Two host runs, the second starting on the first 2 MiB boundary after the first.
    split = count // 3
    second = -(-(split * row_bytes) // (2 << 20)) * (2 << 20)
    segments = torch.tensor([[0, split, 0], [split, count - split, second]], dtype=torch.int64)
    return planes, plane_index, slots, segments, second + (count - split) * row_bytes


def test_noalloc_staged_demotion_matches_the_allocating_entry_point(cuda_device, library_path):
    from ekv_b200.host_pool import pack_rows_staged, pinned_buffer

    lib, fn = _bind(library_path)
    gen = torch.Generator().manual_seed(2026)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    # Two calls in a row with different rows: the ring keeps the first call's
    # bytes, which must not leak into the second call's result.
    for n_planes, rows, row_bytes, count in ((4, 6000, 2048, 5000), (3, 3000, 1024, 2500)):
        planes, plane_index, slots, segments, host_size = _case(gen, cuda_device, n_planes, rows, row_bytes,
                                                                count)
        expected = pinned_buffer(host_size)
        expected.fill_(0)
        got = pinned_buffer(host_size)
        got.fill_(0)
        pack_rows_staged(planes, slots, expected, segments, plane_index=plane_index)
        addresses = (ct.c_uint64 * n_planes)(*[p.data_ptr() for p in planes])
        rc = fn(addresses, n_planes, row_bytes, plane_index.data_ptr(), slots.data_ptr(), 8, slots.numel(),
                ct.cast(segments.data_ptr(), ct.POINTER(ct.c_int64)), segments.shape[0],
                got.data_ptr(), count, cuda_device.index, stream, None)
        assert rc == 0, lib.ekv_error()
        torch.cuda.synchronize()
        assert torch.equal(got, expected)


def test_noalloc_staged_demotion_at_the_row_limit_and_on_a_caller_copy_stream(cuda_device, library_path):
    """Rows of exactly 2 MiB (one row per ring slot, more rows than ring slots, so the
    ring wraps) and a caller-supplied copy stream, each bit exact against the allocating
    entry point."""
    from ekv_b200.host_pool import pack_rows_staged, pinned_buffer

    lib, fn = _bind(library_path)
    gen = torch.Generator().manual_seed(77)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for n_planes, rows, row_bytes, count, own_stream in ((2, 6, 2 << 20, 7, False), (3, 900, 4096, 700, True)):
        planes, plane_index, slots, segments, host_size = _case(gen, cuda_device, n_planes, rows, row_bytes,
                                                                count)
        expected = pinned_buffer(host_size)
        expected.fill_(0)
        got = pinned_buffer(host_size)
        got.fill_(0)
        copy_stream = torch.cuda.Stream(cuda_device) if own_stream else None
        pack_rows_staged(planes, slots, expected, segments, plane_index=plane_index, copy_stream=copy_stream)
        addresses = (ct.c_uint64 * n_planes)(*[p.data_ptr() for p in planes])
        rc = fn(addresses, n_planes, row_bytes, plane_index.data_ptr(), slots.data_ptr(), 8, slots.numel(),
                ct.cast(segments.data_ptr(), ct.POINTER(ct.c_int64)), segments.shape[0],
                got.data_ptr(), count, cuda_device.index, stream,
                None if copy_stream is None else copy_stream.cuda_stream)
        assert rc == 0, lib.ekv_error()
        torch.cuda.synchronize()
        assert torch.equal(got, expected)


def test_noalloc_staged_demotion_rejects_rows_larger_than_a_ring_slot(cuda_device, library_path):
    lib, fn = _bind(library_path)
    plane = torch.zeros(4 << 20, dtype=torch.uint8, device=cuda_device)
    slots = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    segments = torch.tensor([[0, 1, 0]], dtype=torch.int64)
    addresses = (ct.c_uint64 * 1)(plane.data_ptr())
    rc = fn(addresses, 1, 4 << 20, None, slots.data_ptr(), 8, 1,
            ct.cast(segments.data_ptr(), ct.POINTER(ct.c_int64)), 1, None, 1, cuda_device.index, None, None)
    assert rc == -1 and b"2 MiB" in lib.ekv_error()
