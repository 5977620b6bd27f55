"""GPU parity of the fused lookup + mapped gather (ekv_lookup_gather_planes) and the
miss-list compaction (ekv_compact_misses) against the oracle's lookup_slots and mapped
gather, and against the separate lookup + gather launches they replace."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gather as og
from oracle import lookup as ol

pytestmark = pytest.mark.gpu


def _case(row_bytes, n_planes, map_dtype, seed):
    from ekv_b200.virtual_layout import VirtualKVLayout

    gen = torch.Generator().manual_seed(seed)
    width = row_bytes // 2
    n_map_rows, tokens, context, batch, k = 8, 40, 300, 6, 97
    layout = VirtualKVLayout(n_map_rows, tokens, width, itemsize=2, chunk_bytes=4096)
    region = layout.request_bytes // row_bytes  # slots per request region
    elems = layout.capacity_bytes // 2
    planes = [torch.randint(-30000, 30000, (elems,), generator=gen, dtype=torch.int16) for _ in range(n_planes)]
    # Residency map: ~30 % absent (-1, or another negative value), a few slots just
    # past the region (absent to the gather, a hit to the lookup).
    res_map = torch.randint(0, region, (n_map_rows, context), generator=gen)
    res_map[torch.rand((n_map_rows, context), generator=gen) < 0.3] = -1
    res_map[torch.rand((n_map_rows, context), generator=gen) < 0.02] = -7
    res_map[torch.rand((n_map_rows, context), generator=gen) < 0.02] = region
    res_map = res_map.to(map_dtype)
    # Token ids: negative, past the length, past the map width, and valid ones.
    topk = torch.randint(-3, context + 20, (batch, k), generator=gen).to(torch.int32)
    ids = torch.randperm(n_map_rows, generator=gen)[:batch]
    lengths = torch.randint(0, context + 50, (batch,), generator=gen)
    lengths[1] = 0
    lengths[2] = context + 40  # longer than the map row: the map width bounds it
    return layout, width, planes, res_map, topk, ids, lengths


@pytest.mark.parametrize("row_bytes", [6, 256, 512, 2048])
@pytest.mark.parametrize("n_planes", [1, 2, 5])
@pytest.mark.parametrize("map_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("flags", ["none", "ready", "disjoint"])
def test_lookup_gather_matches_the_oracle(row_bytes, n_planes, map_dtype, flags, cuda_device):
    """Slots, miss mask, miss list, count and every plane's rows bit-equal to the oracle's
    lookup_slots over the selected map rows and its mapped gather, for ragged Top-K rows,
    invalid tokens, an empty request, lengths past the map width and misaligned rows
    (6-byte rows take the element copy); with no flag, the indices-ready flag and the
    disjoint flag (which every instance either serves or runs as an ordinary launch)."""
    from ekv_b200.sparse_read import LookupGather

    seed = row_bytes * 10 + n_planes + 7 * ["none", "ready", "disjoint"].index(flags)
    layout, width, planes, res_map, topk, ids, lengths = _case(row_bytes, n_planes, map_dtype, seed)
    dev = cuda_device
    outs = [torch.full((topk.shape[0], topk.shape[1], width), 9, dtype=torch.int16, device=dev) for _ in planes]
    fused = LookupGather([p.to(dev) for p in planes], res_map.to(dev), topk.to(dev), ids.to(dev), lengths.to(dev),
                         outs, layout, indices_ready=flags == "ready", disjoint=flags == "disjoint")
    fused.miss_list.fill_(123)
    fused()
    fused.compact()
    torch.cuda.synchronize()
    slots, miss, miss_list, miss_count = ol.lookup_slots(res_map[ids].numpy(), topk.numpy(), lengths.numpy())
    np.testing.assert_array_equal(fused.slots.cpu().numpy(), slots)
    np.testing.assert_array_equal(fused.miss.cpu().numpy(), miss)
    np.testing.assert_array_equal(fused.miss_list.cpu().numpy(), miss_list)
    np.testing.assert_array_equal(fused.miss_count.cpu().numpy(), miss_count)
    want = og.gather_rows_planes([p.numpy() for p in planes], topk.numpy(), ids.numpy(), lengths.numpy(),
                                 res_map.numpy(), None, width=width, table_width=res_map.shape[1],
                                 request_stride=layout.request_bytes // 2, sink_elements=layout.chunk_bytes // 2,
                                 indirect=False, mapped=True)
    for out, exp in zip(outs, want):
        np.testing.assert_array_equal(out.cpu().numpy(), exp)


@pytest.mark.parametrize("disjoint", [False, True])
def test_lookup_gather_equals_the_separate_launches(disjoint, cuda_device):
    """At a config-4 layer shape (32 requests x 2048 Top-K, 90 % hits, 256 B rows): the fused
    launch leaves the slots, mask, miss list, count and K/V rows that lookup_slots followed
    by the mapped gather leave, eagerly and replayed from a CUDA graph with the compaction
    on a second stream (LayerPipeline: fused launch, then the compaction beside the next
    layer); also with every launch marked disjoint from the ones before it."""
    from ekv_b200.pipeline import LayerPipeline
    from ekv_b200.resident_lookup import lookup_slots
    from ekv_b200.sparse_read import LookupGather, gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    dev = cuda_device
    gen = torch.Generator(device=dev).manual_seed(11)
    reqs, context, hot, k, width, layers = 32, 16384, 4096, 2048, 128, 3
    layout = VirtualKVLayout(reqs, hot, width, itemsize=2, chunk_bytes=1 << 21)
    n_hits = int(0.9 * k)
    fused, maps, topks, planes, outs = [], [], [], [], []
    ids = torch.arange(reqs, device=dev)
    lengths = torch.full((reqs,), context, dtype=torch.int64, device=dev)
    for _ in range(layers):
        res_map = torch.full((reqs, context), -1, dtype=torch.int32, device=dev)
        topk = torch.empty((reqs, k), dtype=torch.int32, device=dev)
        for r in range(reqs):
            perm = torch.randperm(context, generator=gen, device=dev)
            res_map[r, perm[:hot]] = torch.randperm(hot, generator=gen, device=dev).to(torch.int32)
            pick = torch.cat([perm[:n_hits], perm[hot:hot + k - n_hits]])
            topk[r] = pick[torch.randperm(k, generator=gen, device=dev)].to(torch.int32)
        kv = [torch.randint(-30000, 30000, (layout.capacity_bytes // 2,), generator=gen, device=dev,
                            dtype=torch.int16) for _ in range(2)]
        out = [torch.empty((reqs, k, width), dtype=torch.int16, device=dev) for _ in range(2)]
        maps.append(res_map)
        topks.append(topk)
        planes.append(kv)
        outs.append(out)
        fused.append(LookupGather(kv, res_map, topk, ids, lengths, out, layout, indices_ready=True,
                                  disjoint=disjoint))
    expected = []
    for layer in range(layers):
        found = lookup_slots(maps[layer], topks[layer], lengths)
        rows = [torch.empty_like(o) for o in outs[layer]]
        gather_rows_planes(planes[layer], topks[layer], ids, lengths, maps[layer], None, rows, layout,
                           indirect=False, mapped=True)
        expected.append((found, rows))
    step = LayerPipeline([f for f in fused], [f.compact for f in fused], dev)
    for use_graph in (False, True):
        for f in fused:
            for t in (f.slots, f.miss, f.miss_list, f.miss_count):
                t.zero_()
        for layer_outs in outs:
            for o in layer_outs:
                o.fill_(3)
        if use_graph:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                step()
            torch.cuda.current_stream(dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            for f in fused:
                f.miss_list.fill_(-5)
            graph.replay()
        else:
            step()
        torch.cuda.synchronize()
        for layer, ((slots, miss, miss_list, miss_count), rows) in enumerate(expected):
            f = fused[layer]
            assert torch.equal(f.slots, slots) and torch.equal(f.miss, miss)
            assert torch.equal(f.miss_list, miss_list) and torch.equal(f.miss_count, miss_count)
            assert int(f.miss_count.sum()) == reqs * (k - n_hits)
            for got, want in zip(outs[layer], rows):
                assert torch.equal(got, want)
        if use_graph:
            del graph


def test_lookup_gather_checks_its_arguments(cuda_device):
    from ekv_b200.sparse_read import LookupGather
    from ekv_b200.virtual_layout import VirtualKVLayout

    dev = cuda_device
    layout = VirtualKVLayout(2, 8, 16, itemsize=2, chunk_bytes=4096)
    plane = torch.zeros(layout.capacity_bytes // 2, dtype=torch.int16, device=dev)
    res_map = torch.full((2, 20), -1, dtype=torch.int32, device=dev)
    topk = torch.zeros((2, 5), dtype=torch.int32, device=dev)
    ids = torch.arange(2, device=dev)
    lengths = torch.full((2,), 20, device=dev)
    out = torch.empty((2, 5, 16), dtype=torch.int16, device=dev)
    with pytest.raises(ValueError):
        LookupGather([plane], res_map, topk, ids, lengths, [out[:, :4]], layout)
    with pytest.raises(ValueError):
        LookupGather([plane], res_map, topk, ids[:1], lengths, [out], layout)
    with pytest.raises(TypeError):
        LookupGather([plane], res_map, topk, ids, lengths, [out.view(torch.bfloat16).float()], layout)
    with pytest.raises(ValueError):
        LookupGather([plane], res_map.cpu(), topk, ids, lengths, [out], layout)
    empty = LookupGather([plane], res_map, topk[:, :0], ids, lengths, [out[:, :0]], layout)
    empty.miss_count.fill_(7)
    empty()
    empty.compact()
    torch.cuda.synchronize()
    assert not empty.miss_count.any()
