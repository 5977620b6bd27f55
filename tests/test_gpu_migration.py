"""GPU parity of demote/promote row movement (R5) and the VMM-backed round trip (config 3)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import migration as om

pytestmark = pytest.mark.gpu


def _planes(gen, n, rows, row_bytes, device):
    return [torch.randint(0, 256, (rows, row_bytes), generator=gen, dtype=torch.int32).to(torch.uint8).to(device)
            for _ in range(n)]


@pytest.mark.parametrize("row_bytes", [2048, 256, 48, 10])
def test_pack_unpack_cross_form(row_bytes, cuda_device):
    from ekv_b200.host_pool import pack_rows, unpack_rows

    gen = torch.Generator().manual_seed(row_bytes)
    n, rows, count, plane_rows = 4, 1000, 300, 320
    planes = _planes(gen, n, rows, row_bytes, cuda_device)
    slots = torch.randperm(rows, generator=gen)[:count]
    staging = torch.zeros((n * plane_rows, row_bytes), dtype=torch.uint8, device=cuda_device)
    pack_rows(planes, slots.to(cuda_device), staging, stage_plane_stride=plane_rows * row_bytes)
    torch.cuda.synchronize()
    expected = np.zeros((n * plane_rows, row_bytes), dtype=np.uint8)
    om.pack_rows([p.cpu().numpy() for p in planes], slots.numpy(), expected, stage_plane_rows=plane_rows)
    np.testing.assert_array_equal(staging.cpu().numpy(), expected)
    fresh = [torch.zeros_like(p) for p in planes]
    dest = torch.randperm(rows, generator=gen)[:count].to(torch.int32)
    unpack_rows(fresh, dest.to(cuda_device), staging, stage_plane_stride=plane_rows * row_bytes)
    torch.cuda.synchronize()
    want = [np.zeros((rows, row_bytes), dtype=np.uint8) for _ in range(n)]
    om.unpack_rows(want, dest.numpy(), expected, stage_plane_rows=plane_rows)
    for f, w in zip(fresh, want):
        np.testing.assert_array_equal(f.cpu().numpy(), w)


def test_pack_list_form_to_pinned_host(cuda_device):
    from ekv_b200.host_pool import pack_rows, pinned_buffer, unpack_rows

    gen = torch.Generator().manual_seed(11)
    n, rows, count, row_bytes = 6, 2048, 1500, 2048
    planes = _planes(gen, n, rows, row_bytes, cuda_device)
    plane_index = torch.randint(0, n, (count,), generator=gen).to(torch.int32)
    slots = torch.randint(0, rows, (count,), generator=gen)
    stage_rows = torch.randperm(2 * count, generator=gen)[:count]
    host = pinned_buffer(2 * count * row_bytes)
    staging = host[: 2 * count * row_bytes].view(2 * count, row_bytes)
    staging.zero_()
    pack_rows(planes, slots.to(cuda_device), staging, plane_index=plane_index.to(cuda_device),
              stage_rows=stage_rows.to(cuda_device))
    torch.cuda.synchronize()
    expected = np.zeros((2 * count, row_bytes), dtype=np.uint8)
    om.pack_rows([p.cpu().numpy() for p in planes], slots.numpy(), expected,
                 plane_index=plane_index.numpy(), stage_rows=stage_rows.numpy())
    np.testing.assert_array_equal(staging.numpy(), expected)
    # Promote straight from pinned host memory into fresh planes (unique destinations).
    fresh = [torch.zeros_like(p) for p in planes]
    dest = torch.randperm(rows * n, generator=gen)[:count]
    unpack_rows(fresh, (dest % rows).to(cuda_device), staging, plane_index=(dest // rows).to(torch.int32).to(cuda_device),
                stage_rows=stage_rows.to(cuda_device))
    torch.cuda.synchronize()
    for t in range(0, count, 97):
        p, s = int(dest[t]) // rows, int(dest[t]) % rows
        np.testing.assert_array_equal(fresh[p][s].cpu().numpy(), expected[int(stage_rows[t])])


def test_config3_round_trip_through_fresh_vmm_chunks(cuda_device):
    """Config 3 at reduced size: victim chunks with 50-100% occupancy are packed
    into 2 MiB-aligned pinned staging, unmapped, re-mapped fresh (zeroed) and
    restored with a permuted slot assignment; the round trip is bit-exact."""
    from ekv_b200.backing import Backing
    from ekv_b200.host_pool import CHUNK_BYTES, pack_rows, pinned_buffer, unpack_rows

    gen = torch.Generator().manual_seed(3)
    layers, slots, row_bytes = 4, 8192, 2048
    n_planes = 2 * layers
    rows_per_chunk = CHUNK_BYTES // row_bytes
    chunks_per_plane = slots * row_bytes // CHUNK_BYTES
    capacity = CHUNK_BYTES * (1 + n_planes * chunks_per_plane)
    backing = Backing(capacity, CHUNK_BYTES, device=cuda_device.index)
    try:
        backing.ensure(range(1 + n_planes * chunks_per_plane))
        raw = backing.raw
        planes = [raw[CHUNK_BYTES * (1 + p * chunks_per_plane):][: slots * row_bytes].view(slots, row_bytes)
                  for p in range(n_planes)]
        for plane in planes:
            plane.copy_(torch.randint(0, 256, (slots, row_bytes), generator=gen, dtype=torch.int32)
                        .to(torch.uint8))
        original = [plane.clone() for plane in planes]
        victims = torch.randperm(n_planes * chunks_per_plane, generator=gen)[:10]
        plane_index, src_slots, dst_slots, stage_rows = [], [], [], []
        for v, victim in enumerate(victims.tolist()):
            plane, chunk = divmod(victim, chunks_per_plane)
            density = 0.5 + 0.5 * torch.rand((), generator=gen).item()
            occupied = torch.nonzero(torch.rand(rows_per_chunk, generator=gen) < density).flatten()
            perm = torch.randperm(rows_per_chunk, generator=gen)
            first = chunk * rows_per_chunk
            plane_index.append(torch.full((occupied.numel(),), plane, dtype=torch.int32))
            src_slots.append(first + occupied)
            dst_slots.append(first + perm[occupied])
            stage_rows.append(v * rows_per_chunk + torch.arange(occupied.numel()))
        plane_index = torch.cat(plane_index)
        src_slots, dst_slots, stage_rows = torch.cat(src_slots), torch.cat(dst_slots), torch.cat(stage_rows)
        staging = pinned_buffer(len(victims) * CHUNK_BYTES).view(-1, row_bytes)
        pack_rows(planes, src_slots.to(cuda_device), staging, plane_index=plane_index.to(cuda_device),
                  stage_rows=stage_rows.to(cuda_device))
        torch.cuda.synchronize()
        victim_chunks = {1 + int(v) for v in victims}
        assert backing.reclaim(victim_chunks) == len(victim_chunks)
        assert backing.ensure(victim_chunks) == len(victim_chunks)
        for victim in victims.tolist():
            plane, chunk = divmod(victim, chunks_per_plane)
            assert not planes[plane][chunk * rows_per_chunk:(chunk + 1) * rows_per_chunk].any()
        unpack_rows(planes, dst_slots.to(cuda_device), staging, plane_index=plane_index.to(cuda_device),
                    stage_rows=stage_rows.to(cuda_device))
        torch.cuda.synchronize()
        for t in range(src_slots.numel()):
            if t % 53:
                continue
            p = int(plane_index[t])
            assert torch.equal(planes[p][int(dst_slots[t])], original[p][int(src_slots[t])])
        # Whole-chunk check: restored rows at their new slots, zeros elsewhere.
        for v, victim in enumerate(victims.tolist()):
            plane, chunk = divmod(victim, chunks_per_plane)
            pick = plane_index == plane
            pick &= (src_slots // rows_per_chunk) == chunk
            want = torch.zeros((rows_per_chunk, row_bytes), dtype=torch.uint8, device=cuda_device)
            want[(dst_slots[pick] % rows_per_chunk).to(cuda_device)] = original[plane][src_slots[pick].to(cuda_device)]
            got = planes[plane][chunk * rows_per_chunk:(chunk + 1) * rows_per_chunk]
            assert torch.equal(got, want)
        del raw, planes, original
    finally:
        torch.cuda.synchronize()
        backing.close()


def test_pinned_host_pool_backup_and_load(cuda_device):
    from ekv_b200.host_pool import PinnedHostKVPool

    gen = torch.Generator().manual_seed(5)
    layers, slots, row_elems = 3, 512, 256
    keys = [torch.randn((slots, 2, 128), generator=gen).to(torch.bfloat16).to(cuda_device) for _ in range(layers)]
    vals = [torch.randn((slots, 2, 128), generator=gen).to(torch.bfloat16).to(cuda_device) for _ in range(layers)]
    device_pool = SimpleNamespace(get_key_buffer=lambda l: keys[l], get_value_buffer=lambda l: vals[l],
                                  start_layer=0, end_layer=layers)
    pool = PinnedHostKVPool(1000, layers, row_elems * 2, cuda_device)
    table = torch.full((2, 400), -1, dtype=torch.int64)
    allocated = torch.zeros(2, dtype=torch.int64)
    host = pool.alloc_paged_token_slots(table, allocated, 1, 0, 300)
    physical = torch.randperm(slots, generator=gen)[:300].to(cuda_device)
    pool.backup_from_device_all_layer(device_pool, host, physical)
    torch.cuda.synchronize()
    for layer in range(layers):
        k_host = pool.plane_view(2 * layer)[host].view(torch.bfloat16).view(300, 2, 128)
        assert torch.equal(k_host.to(cuda_device), keys[layer][physical])
    dest = torch.randperm(slots, generator=gen)[:300].to(cuda_device)
    for layer in range(layers):
        pool.load_to_device_per_layer(device_pool, host, dest, layer)
    torch.cuda.synchronize()
    for layer in range(layers):
        for plane, device_plane in ((2 * layer, keys[layer]), (2 * layer + 1, vals[layer])):
            host_rows = pool.plane_view(plane)[host].view(torch.bfloat16).view(300, 2, 128)
            assert torch.equal(device_plane[dest], host_rows.to(cuda_device))
    assert pool.available_size() == 700
    assert pool.free(host) == 300 and pool.available_size() == 1000


@pytest.mark.parametrize("row_bytes,scratch_bytes", [(2048, 64 << 20), (2048, 40 << 10), (48, 8 << 10),
                                                     (256, 1 << 20)])
def test_staged_cross_form_round_trip(row_bytes, scratch_bytes, cuda_device):
    """Copy-engine transfers through a scratch ring (small rings force many wraps)."""
    from ekv_b200.host_pool import pack_rows_staged, pinned_buffer, unpack_rows_staged

    gen = torch.Generator().manual_seed(row_bytes + scratch_bytes)
    n, rows, count = 3, 4000, 2500
    planes = _planes(gen, n, rows, row_bytes, cuda_device)
    slots = torch.randperm(rows, generator=gen)[:count].to(cuda_device)
    plane_stride = 3000 * row_bytes
    host = pinned_buffer(n * plane_stride)
    host.fill_(0)
    # Host rows of each plane: two runs (rows 10.. and 1500..), like a fragmented host pool.
    segments = []
    for p in range(n):
        segments.append((p * count, 1200, p * plane_stride + 10 * row_bytes))
        segments.append((p * count + 1200, count - 1200, p * plane_stride + 1500 * row_bytes))
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=cuda_device)
    pack_rows_staged(planes, slots, host, segments, scratch=scratch)
    torch.cuda.synchronize()
    host_rows = torch.cat([torch.arange(10, 1210), torch.arange(1500, 1500 + count - 1200)])
    for p in range(n):
        view = host[p * plane_stride:(p + 1) * plane_stride].view(3000, row_bytes)
        assert torch.equal(view[host_rows], planes[p][slots].cpu())
    fresh = [torch.zeros_like(pl) for pl in planes]
    dest = torch.randperm(rows, generator=gen)[:count].to(cuda_device)
    unpack_rows_staged(fresh, dest, host, segments, scratch=scratch)
    torch.cuda.synchronize()
    for p in range(n):
        assert torch.equal(fresh[p][dest], planes[p][slots])
        untouched = torch.ones(rows, dtype=torch.bool, device=cuda_device)
        untouched[dest] = False
        assert not fresh[p][untouched].any()


def test_staged_list_form_chunk_aligned(cuda_device):
    """Victim-chunk staging: each chunk's rows start on a 2 MiB boundary of pinned memory."""
    from ekv_b200.host_pool import CHUNK_BYTES, pack_rows_staged, pinned_buffer, unpack_rows_staged

    gen = torch.Generator().manual_seed(8)
    n, rows, row_bytes = 4, 4096, 2048
    per_chunk = CHUNK_BYTES // row_bytes
    planes = _planes(gen, n, rows, row_bytes, cuda_device)
    victims = [(0, 1), (2, 3), (3, 0), (1, 2)]  # (plane, chunk)
    plane_index, src, segments, t = [], [], [], 0
    for v, (plane, chunk) in enumerate(victims):
        occupied = torch.nonzero(torch.rand(per_chunk, generator=gen) < 0.7).flatten()
        plane_index.append(torch.full((occupied.numel(),), plane, dtype=torch.int32))
        src.append(chunk * per_chunk + occupied)
        segments.append((t, occupied.numel(), v * CHUNK_BYTES))
        t += occupied.numel()
    plane_index = torch.cat(plane_index).to(cuda_device)
    src = torch.cat(src).to(cuda_device)
    host = pinned_buffer(len(victims) * CHUNK_BYTES)
    pack_rows_staged(planes, src, host, segments, plane_index=plane_index,
                     scratch=torch.empty(1 << 20, dtype=torch.uint8, device=cuda_device))
    torch.cuda.synchronize()
    for (first, count, offset) in segments:
        got = host[offset:offset + count * row_bytes].view(count, row_bytes)
        idx = slice(first, first + count)
        want = torch.stack([planes[int(p)][int(s)] for p, s in zip(plane_index[idx].tolist(), src[idx].tolist())])
        assert torch.equal(got.to(cuda_device), want)
    fresh = [torch.zeros_like(pl) for pl in planes]
    unpack_rows_staged(fresh, src, host, segments, plane_index=plane_index)
    torch.cuda.synchronize()
    for p in range(n):
        pick = plane_index == p
        assert torch.equal(fresh[p][src[pick]], planes[p][src[pick]])


def test_staged_rejects_bad_segments(cuda_device):
    from ekv_b200._lib import KernelError
    from ekv_b200.host_pool import pack_rows_staged, pinned_buffer

    planes = [torch.zeros((64, 32), dtype=torch.uint8, device=cuda_device)]
    slots = torch.arange(10, device=cuda_device)
    host = pinned_buffer(1 << 20)
    with pytest.raises(KernelError, match="cover"):
        pack_rows_staged(planes, slots, host, [(0, 5, 0)])
    with pytest.raises(KernelError, match="task order"):
        pack_rows_staged(planes, slots, host, [(0, 5, 0), (6, 4, 4096)])
    with pytest.raises(ValueError, match="pinned"):
        pack_rows_staged(planes, slots, torch.zeros(1 << 20, dtype=torch.uint8), [(0, 10, 0)])


def test_pinned_host_pool_fragmented_rows_use_zero_copy(cuda_device):
    from ekv_b200.host_pool import PinnedHostKVPool

    gen = torch.Generator().manual_seed(9)
    slots, layers = 1024, 2
    keys = [torch.randn((slots, 256), generator=gen).to(torch.bfloat16).to(cuda_device) for _ in range(layers)]
    vals = [torch.randn((slots, 256), generator=gen).to(torch.bfloat16).to(cuda_device) for _ in range(layers)]
    device_pool = SimpleNamespace(get_key_buffer=lambda l: keys[l], get_value_buffer=lambda l: vals[l],
                                  start_layer=0, end_layer=layers)
    pool = PinnedHostKVPool(2000, layers, 512, cuda_device)
    host = torch.arange(0, 1200, 2)  # 600 runs of one row: more than MAX_STAGED_RUNS
    physical = torch.randperm(slots, generator=gen)[:600].to(cuda_device)
    pool.backup_from_device_all_layer(device_pool, host, physical)
    torch.cuda.synchronize()
    for layer in range(layers):
        got = pool.plane_view(2 * layer + 1)[host].view(torch.bfloat16).view(600, 256)
        assert torch.equal(got.to(cuda_device), vals[layer][physical])
