"""GPU parity of the Top-K row gather (R3) against the reference's golden vectors and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_npz_cases
from oracle import gather as og

pytestmark = pytest.mark.gpu


def _layout_of(c):
    from ekv_b200.virtual_layout import VirtualKVLayout

    reqs, tokens, width, itemsize, chunk = (int(v) for v in c["layout"])
    return VirtualKVLayout(reqs, tokens, width, itemsize=itemsize, chunk_bytes=chunk)


def _to(a, device, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("case", sorted(load_npz_cases("gather_golden.npz")))
@pytest.mark.parametrize("indirect", [False, True])
def test_gather_rows_matches_reference(case, indirect, cuda_device):
    from ekv_b200.sparse_read import gather_rows

    c = load_npz_cases("gather_golden.npz")[case]
    layout = _layout_of(c)
    raw = _to(c["raw"].view(np.int16), cuda_device).view(torch.bfloat16)
    positions = _to(c["positions"], cuda_device)
    output = torch.full((*positions.shape, layout.row_elements), 7.0, dtype=torch.bfloat16,
                        device=cuda_device)
    gather_rows(raw, positions, _to(c["request_ids"], cuda_device), _to(c["lengths"], cuda_device),
                _to(c["request_table"], cuda_device), _to(c["slot_offsets"], cuda_device), output,
                layout, indirect=indirect)
    torch.cuda.synchronize()
    got = output.view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, c["expected_indirect" if indirect else "expected_direct"])


def test_gather_rows_contract(cuda_device):
    from ekv_b200.sparse_read import gather_rows
    from ekv_b200.virtual_layout import VirtualKVLayout

    layout = VirtualKVLayout(1, 4, 8)
    dev = cuda_device
    raw = torch.zeros(layout.capacity_bytes // 2, dtype=torch.bfloat16, device=dev)
    idx = torch.zeros((1, 2), dtype=torch.int64, device=dev)
    one = torch.ones(1, dtype=torch.int64, device=dev)
    with pytest.raises(ValueError, match="output shape"):
        gather_rows(raw, idx, one, one, idx, one, torch.empty((1, 2, 7), dtype=torch.bfloat16, device=dev),
                    layout, indirect=False)
    # Empty selection returns without touching the output.
    empty = torch.zeros((1, 0), dtype=torch.int64, device=dev)
    gather_rows(raw, empty, one, one, idx, one, torch.empty((1, 0, 8), dtype=torch.bfloat16, device=dev),
                layout, indirect=False)
    with pytest.raises(TypeError):
        gather_rows(raw, idx, one, one, idx, one, torch.empty((1, 2, 8), dtype=torch.float32, device=dev),
                    layout, indirect=False)


@pytest.mark.parametrize("width,itemsize_dtype", [(1024, torch.bfloat16), (128, torch.bfloat16),
                                                  (3, torch.bfloat16), (64, torch.float32),
                                                  (17, torch.uint8)])
def test_gather_rows_planes_matches_oracle(width, itemsize_dtype, cuda_device):
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    gen = torch.Generator().manual_seed(width)
    slots, batch, selected, n_planes, tokens = 4096, 6, 300, 5, 512
    esize = torch.empty((), dtype=itemsize_dtype).element_size()
    layout = VirtualKVLayout(batch, tokens, width, itemsize=esize)
    planes_cpu = [torch.randint(0, 256, (slots * width * esize,), generator=gen, dtype=torch.int32)
                  .to(torch.uint8).view(itemsize_dtype) for _ in range(n_planes)]
    table = torch.randint(0, slots, (batch, tokens), generator=gen)
    slot_offsets = torch.arange(slots, dtype=torch.int64) * width
    positions = torch.randint(-2, tokens + 2, (batch, selected), generator=gen)
    lengths = torch.randint(tokens // 2, tokens + 1, (batch,), generator=gen)
    request_ids = torch.randperm(batch, generator=gen)
    planes = [p.to(cuda_device) for p in planes_cpu]
    outputs = [torch.full((batch, selected, width), 3, dtype=itemsize_dtype, device=cuda_device)
               for _ in range(n_planes)]
    gather_rows_planes(planes, positions.to(cuda_device), request_ids.to(cuda_device),
                       lengths.to(cuda_device), table.to(cuda_device), slot_offsets.to(cuda_device),
                       outputs, layout, indirect=True)
    torch.cuda.synchronize()
    raw_views = [p.view(torch.uint8).numpy().view({1: np.uint8, 2: np.uint16, 4: np.uint32}[esize])
                 for p in planes_cpu]
    expected = og.gather_rows_planes(raw_views, positions.numpy(), request_ids.numpy(), lengths.numpy(),
                                     table.numpy(), slot_offsets.numpy(), width=width,
                                     table_width=tokens, request_stride=0, sink_elements=0,
                                     indirect=True)
    for out, exp in zip(outputs, expected):
        np.testing.assert_array_equal(out.cpu().view(torch.uint8).numpy().view(exp.dtype), exp)


def test_gather_rows_planes_more_planes_than_one_launch(cuda_device):
    """300 planes: split into EKV_MAX_PLANES-sized launches."""
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    n_planes, slots, width = 300, 64, 8
    layout = VirtualKVLayout(1, slots, width)
    planes = [torch.full((slots * width,), p, dtype=torch.int16, device=cuda_device).view(torch.bfloat16)
              for p in range(n_planes)]
    outputs = [torch.zeros((1, 4, width), dtype=torch.bfloat16, device=cuda_device) for _ in range(n_planes)]
    positions = torch.tensor([[0, 5, 63, 64]], device=cuda_device)
    one = torch.ones(1, dtype=torch.int64, device=cuda_device)
    lengths = torch.full((1,), slots, dtype=torch.int64, device=cuda_device)
    table = torch.arange(slots, device=cuda_device).view(1, slots)
    offsets = torch.arange(slots, device=cuda_device) * width
    gather_rows_planes(planes, positions, one * 0, lengths, table, offsets, outputs, layout, indirect=True)
    torch.cuda.synchronize()
    for p, out in enumerate(outputs):
        vals = out.view(torch.int16)
        assert (vals[0, :3] == p).all() and (vals[0, 3] == 0).all()


def test_gather_full_config2_property(cuda_device):
    """Config 2 at full size (36 layers x K,V pools [262144, 8, 128] bf16, 64 requests x
    2048 Top-K slots): every gathered word identifies its plane, slot and column."""
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    slots, width, layers, batch, topk = 262144, 1024, 36, 64, 2048
    n_planes = 2 * layers
    words = width // 2  # int32 words per row
    layout = VirtualKVLayout(batch, topk, width)
    base = torch.arange(slots * words, dtype=torch.int32, device=cuda_device).view(slots, words)
    keys = [(p * 0x9E3779B1) & 0x7FFFFFFF for p in range(n_planes)]
    planes = [torch.bitwise_xor(base, key) for key in keys]
    del base
    gen = torch.Generator(device=cuda_device).manual_seed(2)
    table = torch.stack([torch.randperm(slots, generator=gen, device=cuda_device)[:topk]
                         for _ in range(batch)])
    positions = torch.stack([torch.randperm(topk, generator=gen, device=cuda_device)
                             for _ in range(batch)])
    request_ids = torch.arange(batch, device=cuda_device)
    lengths = torch.full((batch,), topk, dtype=torch.int64, device=cuda_device)
    positions[3, 7] = -1
    positions[5, 9] = topk
    offsets = torch.arange(slots, dtype=torch.int64, device=cuda_device) * width
    outputs = [torch.empty((batch, topk, width), dtype=torch.bfloat16, device=cuda_device)
               for _ in range(n_planes)]
    gather_rows_planes([p.view(torch.bfloat16) for p in planes], positions, request_ids, lengths, table,
                       offsets, outputs, layout, indirect=True)
    torch.cuda.synchronize()
    valid = (positions >= 0) & (positions < topk)
    slot = torch.gather(table, 1, positions.clamp(0, topk - 1))
    expect_words = slot[..., None].to(torch.int32) * words + torch.arange(words, device=cuda_device,
                                                                           dtype=torch.int32)
    for p, out in enumerate(outputs):
        got = out.view(torch.int32)
        ok = torch.where(valid[..., None], (got ^ keys[p]) == expect_words, got == 0)
        assert bool(ok.all()), f"plane {p} mismatch"


def test_gather_falls_back_for_misaligned_rows(cuda_device):
    """16-byte aligned planes and row size, but some slot offsets land on odd elements:
    those 32-row batches are copied with element loads, the rest with 16-byte vectors."""
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    gen = torch.Generator().manual_seed(77)
    slots, width, batch, selected, tokens = 2048, 64, 4, 700, 1024
    layout = VirtualKVLayout(batch, tokens, width)
    planes_cpu = [torch.randint(-32768, 32767, (slots * width + 8,), generator=gen, dtype=torch.int16)
                  for _ in range(3)]
    offsets = torch.arange(slots, dtype=torch.int64) * width
    offsets[torch.randperm(slots, generator=gen)[:20]] += 3  # a few rows start mid-vector
    table = torch.randint(0, slots, (batch, tokens), generator=gen)
    positions = torch.randint(-1, tokens, (batch, selected), generator=gen)
    lengths = torch.full((batch,), tokens, dtype=torch.int64)
    request_ids = torch.arange(batch)
    outputs = [torch.empty((batch, selected, width), dtype=torch.bfloat16, device=cuda_device) for _ in planes_cpu]
    gather_rows_planes([p.to(cuda_device).view(torch.bfloat16) for p in planes_cpu], positions.to(cuda_device),
                       request_ids.to(cuda_device), lengths.to(cuda_device), table.to(cuda_device),
                       offsets.to(cuda_device), outputs, layout, indirect=True)
    torch.cuda.synchronize()
    expected = og.gather_rows_planes([p.numpy() for p in planes_cpu], positions.numpy(), request_ids.numpy(),
                                     lengths.numpy(), table.numpy(), offsets.numpy(), width=width,
                                     table_width=tokens, request_stride=0, sink_elements=0, indirect=True)
    for out, exp in zip(outputs, expected):
        np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy(), exp)


def test_mapped_gather_reads_slots_outside_the_region_as_absent(cuda_device):
    """Mapped mode (residency map -> slot in the request's fixed hot region): slots < 0 or
    past the region's capacity give zero rows, never bytes from outside the region."""
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout
    from oracle import swap as osw

    gen = torch.Generator().manual_seed(17)
    batch, hot, width, context, k = 3, 64, 128, 500, 40
    layout = VirtualKVLayout(batch, hot, width, itemsize=2, chunk_bytes=1 << 16)
    region = layout.request_bytes // 2 // width  # slots per request region (>= hot)
    planes = [torch.randint(-30000, 30000, (layout.capacity_bytes // 2,), generator=gen, dtype=torch.int16)
              for _ in range(2)]
    res_map = torch.full((batch, context), -1, dtype=torch.int32)
    topk = torch.stack([torch.randperm(context, generator=gen)[:k] for _ in range(batch)]).to(torch.int32)
    for b in range(batch):
        res_map[b, topk[b, :20]] = torch.randperm(region, generator=gen)[:20].to(torch.int32)
        res_map[b, topk[b, 20]] = region          # just past the region
        res_map[b, topk[b, 21]] = region + 1000   # far past it
    lengths = torch.full((batch,), context, dtype=torch.int64)
    outs = [torch.empty((batch, k, width), dtype=torch.int16, device=cuda_device) for _ in range(2)]
    gather_rows_planes([p.to(cuda_device) for p in planes], topk.to(cuda_device),
                       torch.arange(batch, device=cuda_device), lengths.to(cuda_device),
                       res_map.to(cuda_device), None, outs, layout, indirect=False, mapped=True)
    sink = layout.chunk_bytes // 2
    for plane, out in zip(planes, outs):
        hot_rows = plane[sink:].view(batch, region, width).numpy()
        want = osw.mapped_gather(hot_rows, res_map.numpy(), topk.numpy(), lengths.numpy())
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        assert not out[:, 20:22].any()  # the out-of-region slots read as zero rows


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("form", ["pipelined", "concurrent"])
def test_layer_pipeline_lookup_then_gather(form, graph, cuda_device):
    """LayerPipeline over per-layer (lookup, gather) pairs -- the config-4 decode step --
    gives every layer's slots and rows exactly as the oracle's lookup + gather.
    ``pipelined``: direct gathers of the lookup's slots, layer i's gather beside layer
    i+1's lookup.  ``concurrent`` (wait=False): mapped gathers that read the residency
    map themselves, beside their own layer's lookup.  With ``graph`` the step is
    captured once and replayed."""
    from ekv_b200.pipeline import LayerPipeline
    from ekv_b200.resident_lookup import LookupPlan
    from ekv_b200.sparse_read import PlaneGather
    from ekv_b200.virtual_layout import VirtualKVLayout
    from oracle import lookup as ol

    dev = cuda_device
    gen = torch.Generator().manual_seed(29)
    layers, batch, context, hot, k, width = 5, 6, 3000, 256, 200, 128
    layout = VirtualKVLayout(batch, hot, width, itemsize=2, chunk_bytes=1 << 16)
    req_ids = torch.arange(batch, device=dev)
    lengths = torch.full((batch,), hot, dtype=torch.int64, device=dev)
    ctx_lengths = torch.full((batch,), context, dtype=torch.int64, device=dev)
    maps, topks, planes, outs, lookups, gathers = [], [], [], [], [], []
    for _ in range(layers):
        res_map = torch.full((batch, context), -1, dtype=torch.int32)
        topk = torch.empty((batch, k), dtype=torch.int32)
        for b in range(batch):
            perm = torch.randperm(context, generator=gen)
            res_map[b, perm[:hot]] = torch.randperm(hot, generator=gen).to(torch.int32)
            topk[b] = torch.cat([perm[:150], perm[hot:hot + k - 150]])[torch.randperm(k, generator=gen)].to(torch.int32)
        maps.append(res_map)
        topks.append(topk)
        layer_planes = [torch.randint(-30000, 30000, (layout.capacity_bytes // 2,), generator=gen,
                                      dtype=torch.int16) for _ in range(2)]
        planes.append(layer_planes)
        layer_outs = [torch.full((batch, k, width), 7, dtype=torch.int16, device=dev) for _ in range(2)]
        outs.append(layer_outs)
        dmap, dtopk = res_map.to(dev), topk.to(dev)
        plan = LookupPlan(dmap, dtopk)
        lookups.append(plan)
        dev_planes = [p.to(dev).view(torch.bfloat16) for p in layer_planes]
        if form == "pipelined":
            gathers.append(PlaneGather(dev_planes, plan.slots, req_ids, lengths, None, None,
                                       [o.view(torch.bfloat16) for o in layer_outs], layout, indirect=False))
        else:
            gathers.append(PlaneGather(dev_planes, dtopk, req_ids, ctx_lengths, dmap, None,
                                       [o.view(torch.bfloat16) for o in layer_outs], layout, indirect=False,
                                       mapped=True))
    pipeline = LayerPipeline(lookups, gathers, dev, wait=form == "pipelined")

    def poison():  # the plans ran their lookup once when built: make the step's own run visible
        for plan in lookups:
            for t in (plan.slots, plan.miss_list, plan.miss_count):
                t.fill_(-5)
        for layer_outs in outs:
            for o in layer_outs:
                o.fill_(7)

    if graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            pipeline()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        replay = torch.cuda.CUDAGraph()
        with torch.cuda.graph(replay):
            pipeline()
        poison()
        replay.replay()
    else:
        poison()
        pipeline()
    torch.cuda.synchronize()
    for layer in range(layers):
        slots, _, miss_list, miss_count = ol.lookup_slots(maps[layer].numpy(), topks[layer].numpy())
        np.testing.assert_array_equal(lookups[layer].slots.cpu().numpy(), slots)
        np.testing.assert_array_equal(lookups[layer].miss_list.cpu().numpy(), miss_list)
        np.testing.assert_array_equal(lookups[layer].miss_count.cpu().numpy(), miss_count)
        want = og.gather_rows_planes([p.numpy() for p in planes[layer]], slots, req_ids.cpu().numpy(),
                                     lengths.cpu().numpy(), None, None, width=width, table_width=hot,
                                     request_stride=layout.request_bytes // 2,
                                     sink_elements=layout.chunk_bytes // 2, indirect=False)
        for out, exp in zip(outs[layer], want):
            np.testing.assert_array_equal(out.cpu().numpy(), exp)
    if graph:
        del replay



def test_compiled_binding_serves_gathers_like_the_ctypes_path(cuda_device, monkeypatch):
    """gather_rows and gather_rows_planes (direct, indirect, mapped; more planes than one
    launch takes) give the same bytes through the compiled binding as through the checked
    ctypes path (forced by hiding the binding), and the same errors for malformed calls."""
    from ekv_b200 import _lib, sparse_read
    from ekv_b200.virtual_layout import VirtualKVLayout

    assert _lib.torch_binding() is not None, "lib/_ekv_torch.so was not built"
    dev = cuda_device
    gen = torch.Generator().manual_seed(41)
    batch, tokens, width, selected = 3, 96, 64, 50
    layout = VirtualKVLayout(batch, tokens, width, itemsize=2, chunk_bytes=1 << 16)
    n_planes = _lib.MAX_PLANES + 7
    planes = [torch.randint(-30000, 30000, (layout.capacity_bytes // 2,), generator=gen, dtype=torch.int16)
              .to(dev).view(torch.bfloat16) for _ in range(n_planes)]
    positions = torch.randint(-3, tokens + 3, (batch, selected), generator=gen).to(dev)
    ids = torch.tensor([2, 0, 1], device=dev)
    lengths = torch.tensor([tokens, tokens // 2, 7], device=dev)
    slots = layout.capacity_bytes // 2 // width
    offsets = (torch.randperm(slots, generator=gen)[:tokens * batch] * width).to(dev)
    table = torch.arange(tokens * batch, device=dev).view(batch, tokens)
    res_map = torch.randint(-1, tokens + 4, (batch, tokens), generator=gen, dtype=torch.int32).to(dev)

    def run():
        outs = {}
        for indirect in (False, True):
            out = torch.full((batch, selected, width), 3.0, dtype=torch.bfloat16, device=dev)
            sparse_read.gather_rows(planes[0], positions, ids, lengths, table, offsets, out, layout,
                                    indirect=indirect)
            outs[("rows", indirect)] = out
        for mode in ("direct", "indirect", "mapped"):
            many = [torch.full((batch, selected, width), 3.0, dtype=torch.bfloat16, device=dev)
                    for _ in range(n_planes)]
            sparse_read.gather_rows_planes(planes, positions, ids, lengths,
                                           res_map if mode == "mapped" else table, offsets, many, layout,
                                           indirect=mode == "indirect", mapped=mode == "mapped")
            outs[("planes", mode)] = many
        torch.cuda.synchronize()
        return outs

    def errors():
        out = torch.empty((batch, selected, width), dtype=torch.bfloat16, device=dev)
        found = []
        for call in (
            lambda: sparse_read.gather_rows(planes[0], positions, ids, lengths, table, offsets, out[:, 1:], layout,
                                            indirect=True),
            lambda: sparse_read.gather_rows(planes[0], positions, ids, lengths, None, offsets, out, layout,
                                            indirect=True),
            lambda: sparse_read.gather_rows(planes[0].float(), positions, ids, lengths, table, offsets, out,
                                            layout, indirect=True),
            lambda: sparse_read.gather_rows_planes(planes[:2], positions, ids, lengths, table, offsets, [out],
                                                   layout, indirect=True),
            lambda: sparse_read.gather_rows_planes(planes[:1], positions, ids, lengths, table, offsets, [out],
                                                   layout, indirect=True, mapped=True),
            lambda: sparse_read.gather_rows_planes(planes[:1], positions.cpu(), ids, lengths, table, offsets, [out],
                                                   layout, indirect=True),
        ):
            with pytest.raises((ValueError, TypeError)) as info:
                call()
            found.append((info.type, str(info.value)))
        return found

    fast, fast_errors = run(), errors()
    monkeypatch.setattr(sparse_read, "torch_binding", lambda: None)
    slow, slow_errors = run(), errors()
    assert fast_errors == slow_errors
    for key, value in fast.items():
        values = value if isinstance(value, list) else [value]
        others = slow[key] if isinstance(slow[key], list) else [slow[key]]
        for a, b in zip(values, others):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16)), key
    # Direct mode against the oracle, so the shared result is also the right one.
    want = og.gather_rows(planes[0].view(torch.int16).cpu().numpy(), positions.cpu().numpy(), ids.cpu().numpy(),
                          lengths.cpu().numpy(), None, None, width=width, table_width=tokens,
                          request_stride=layout.request_bytes // 2, sink_elements=layout.chunk_bytes // 2,
                          indirect=False)
    np.testing.assert_array_equal(fast[("rows", False)].view(torch.int16).cpu().numpy(), want)


@pytest.mark.parametrize("indirect", [False, True])
def test_small_rows_over_many_planes_match_the_oracle(indirect, cuda_device):
    """256 B rows over more planes than the default kernel instance flattens (the TP8
    shard of every layer in one launch) take the small-row instance; its bytes equal the
    oracle's, invalid positions give zero rows, and a batch holding a row that is not
    16-byte aligned falls back to element copies."""
    from ekv_b200.sparse_read import gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    gen = torch.Generator().manual_seed(43)
    batch, tokens, width, selected, n_planes = 5, 300, 128, 180, 20
    layout = VirtualKVLayout(batch, tokens, width, itemsize=2, chunk_bytes=1 << 16)
    elems = layout.capacity_bytes // 2
    planes = [torch.randint(-30000, 30000, (elems,), generator=gen, dtype=torch.int16) for _ in range(n_planes)]
    positions = torch.randint(-4, tokens + 4, (batch, selected), generator=gen)
    ids = torch.tensor([3, 1, 4, 0, 2])
    lengths = torch.tensor([tokens, 250, 17, tokens, 0])
    n_logical = batch * tokens
    table = torch.randperm(n_logical, generator=gen).view(batch, tokens)
    offsets = layout.chunk_bytes // 2 + torch.randperm(elems // width - layout.chunk_bytes // 2 // width,
                                                      generator=gen)[:n_logical] * width
    offsets[table[0, 5]] = layout.chunk_bytes // 2 + 3  # one row not 16-byte aligned (request 0, token 5)
    positions[3, 0] = 5  # batch row 3 is request 0: the unaligned row is selected
    outs = [torch.full((batch, selected, width), 9, dtype=torch.int16, device=cuda_device) for _ in planes]
    gather_rows_planes([p.to(cuda_device).view(torch.bfloat16) for p in planes], positions.to(cuda_device),
                       ids.to(cuda_device), lengths.to(cuda_device), table.to(cuda_device),
                       offsets.to(cuda_device), [o.view(torch.bfloat16) for o in outs], layout, indirect=indirect)
    torch.cuda.synchronize()
    want = og.gather_rows_planes([p.numpy() for p in planes], positions.numpy(), ids.numpy(), lengths.numpy(),
                                 table.numpy(), offsets.numpy(), width=width, table_width=tokens,
                                 request_stride=layout.request_bytes // 2, sink_elements=layout.chunk_bytes // 2,
                                 indirect=indirect)
    for out, exp in zip(outs, want):
        np.testing.assert_array_equal(out.cpu().numpy(), exp)


@pytest.mark.parametrize("row_bytes", [16, 32, 64, 128, 256, 512])
@pytest.mark.parametrize("n_planes", [1, 2, 3, 7, 40])
@pytest.mark.parametrize("mode", ["indirect", "mapped_ready"])
def test_grouped_small_rows_match_the_oracle(row_bytes, n_planes, mode, cuda_device):
    """Rows of 16 to 512 B (a power-of-two number of 16-byte vectors) take the grouped
    copy, one instance per plane-count class: every byte equals the oracle's for ragged
    batches (rows not a multiple of 32), invalid positions, empty requests and, in the
    indirect case, a batch holding a row that starts off a 16-byte boundary (element
    copy fallback).  The mapped case also sets the indices-ready flag, whose only
    effect is when the index chain is walked; the second launch is marked disjoint
    (two-plane launches take the disjoint instance, the others run it as an ordinary
    launch)."""
    from ekv_b200.sparse_read import PlaneGather, gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    width = row_bytes // 2
    gen = torch.Generator().manual_seed(row_bytes * 100 + n_planes)
    batch, tokens, selected = 7, 96, 173
    layout = VirtualKVLayout(batch, tokens, width, itemsize=2, chunk_bytes=4096)
    elems = layout.capacity_bytes // 2
    planes = [torch.randint(-30000, 30000, (elems,), generator=gen, dtype=torch.int16) for _ in range(n_planes)]
    positions = torch.randint(-3, tokens + 3, (batch, selected), generator=gen)
    ids = torch.randperm(batch, generator=gen)
    lengths = torch.randint(0, tokens + 1, (batch,), generator=gen)
    lengths[2] = 0
    if mode == "indirect":
        n_logical = batch * tokens
        table = torch.randperm(n_logical, generator=gen).view(batch, tokens)
        first = layout.chunk_bytes // 2
        offsets = first + torch.randperm((elems - first) // width, generator=gen)[:n_logical] * width
        offsets[table[int(ids[4]), 7]] = first + 1  # an odd element offset: off the 16-byte grid
        positions[4, 3] = 7
        lengths[4] = tokens
        table_arg, indirect, mapped, ready = table, True, False, False
    else:
        # Residency map: token -> slot in the request's fixed region, -1 absent, some slots
        # past the region (read as absent too).
        rows_per_request = layout.request_bytes // row_bytes
        table = torch.randint(-1, rows_per_request + 2, (batch, tokens), generator=gen)
        offsets, table_arg, indirect, mapped, ready = None, table, False, True, True
    outs = [torch.full((batch, selected, width), 9, dtype=torch.int16, device=cuda_device) for _ in planes]
    dev_planes = [p.to(cuda_device).view(torch.bfloat16) for p in planes]
    args = (positions.to(cuda_device), ids.to(cuda_device), lengths.to(cuda_device),
            table_arg.to(cuda_device), None if offsets is None else offsets.to(cuda_device))
    gather_rows_planes(dev_planes, *args, [o.view(torch.bfloat16) for o in outs], layout,
                       indirect=indirect, mapped=mapped, indices_ready=ready)
    again = [torch.full_like(o, 5) for o in outs]
    PlaneGather(dev_planes, *args, [o.view(torch.bfloat16) for o in again], layout,
                indirect=indirect, mapped=mapped, indices_ready=not ready, disjoint=True)()
    torch.cuda.synchronize()
    if mapped:
        want = og.gather_rows_planes([p.numpy() for p in planes], positions.numpy(), ids.numpy(),
                                     lengths.numpy(), table.numpy(), None, width=width, table_width=tokens,
                                     request_stride=layout.request_bytes // 2,
                                     sink_elements=layout.chunk_bytes // 2, indirect=False, mapped=True)
    else:
        want = og.gather_rows_planes([p.numpy() for p in planes], positions.numpy(), ids.numpy(),
                                     lengths.numpy(), table.numpy(), offsets.numpy(), width=width,
                                     table_width=tokens, request_stride=layout.request_bytes // 2,
                                     sink_elements=layout.chunk_bytes // 2, indirect=True)
    for out, other, exp in zip(outs, again, want):
        np.testing.assert_array_equal(out.cpu().numpy(), exp)
        np.testing.assert_array_equal(other.cpu().numpy(), exp)


@pytest.mark.parametrize("row_bytes", [6, 16, 48, 256, 512, 1024, 2048])
@pytest.mark.parametrize("planes_per_layer", [1, 2, 3])
@pytest.mark.parametrize("mode", ["direct", "indirect", "mapped"])
@pytest.mark.parametrize("layers", [1, 5])
def test_layer_gather_matches_the_oracle_per_layer(row_bytes, planes_per_layer, mode, layers, cuda_device):
    """One ekv_gather_layers launch writes, for every layer, what the oracle's
    gather of that layer's planes with that layer's positions and table gives:
    every copy instance (grouped, flattened, per-row off the 16-byte grid), every
    addressing mode, zero rows for positions outside [0, length)."""
    from ekv_b200.sparse_read import LayerGather
    from ekv_b200.virtual_layout import VirtualKVLayout

    width = row_bytes // 2
    gen = torch.Generator().manual_seed(row_bytes * 1000 + planes_per_layer * 10 + layers)
    batch, tokens, selected = 5, 64, 97
    layout = VirtualKVLayout(batch, tokens, width, itemsize=2, chunk_bytes=4096)
    elems = layout.capacity_bytes // 2
    ids = torch.randperm(batch, generator=gen)
    lengths = torch.randint(0, tokens + 1, (batch,), generator=gen)
    lengths[1] = tokens
    n_logical = batch * tokens
    first = layout.chunk_bytes // 2
    offsets = first + torch.randperm((elems - first) // width, generator=gen)[:n_logical] * width
    rows_per_request = layout.request_bytes // row_bytes
    planes, outs, positions, tables = [], [], [], []
    for layer in range(layers):
        planes += [torch.randint(-30000, 30000, (elems,), generator=gen, dtype=torch.int16)
                   for _ in range(planes_per_layer)]
        outs += [torch.full((batch, selected, width), 9, dtype=torch.int16, device=cuda_device)
                 for _ in range(planes_per_layer)]
        pos = torch.randint(-3, tokens + 3, (batch, selected), generator=gen)
        if mode == "indirect":
            table = torch.randperm(n_logical, generator=gen).view(batch, tokens)
            if layer == layers - 1:
                # an odd element offset: this batch leaves the 16-byte grid
                offsets[table[int(ids[1]), 5]] = first + 1
                pos[1, 2] = 5
        else:
            table = torch.randint(-1, rows_per_request + 2, (batch, tokens), generator=gen)
        positions.append(pos)
        tables.append(table)
    dev = lambda t: t.to(cuda_device)  # noqa: E731
    indirect, mapped = mode == "indirect", mode == "mapped"
    gather = LayerGather([dev(p).view(torch.bfloat16) for p in planes], [dev(p) for p in positions], dev(ids),
                         dev(lengths), [dev(t) for t in tables] if mode != "direct" else None,
                         dev(offsets) if indirect else None, [o.view(torch.bfloat16) for o in outs], layout,
                         planes_per_layer=planes_per_layer, indirect=indirect, mapped=mapped)
    gather()
    torch.cuda.synchronize()
    for layer in range(layers):
        sl = slice(layer * planes_per_layer, (layer + 1) * planes_per_layer)
        want = og.gather_rows_planes([p.numpy() for p in planes[sl]], positions[layer].numpy(), ids.numpy(),
                                     lengths.numpy(), tables[layer].numpy() if mode != "direct" else None,
                                     offsets.numpy() if indirect else None, width=width, table_width=tokens,
                                     request_stride=layout.request_bytes // 2,
                                     sink_elements=layout.chunk_bytes // 2, indirect=indirect, mapped=mapped)
        for out, exp in zip(outs[sl], want):
            np.testing.assert_array_equal(out.cpu().numpy(), exp)


def test_layer_gather_checks_its_arguments(cuda_device):
    from ekv_b200.sparse_read import LayerGather
    from ekv_b200.virtual_layout import VirtualKVLayout

    layout = VirtualKVLayout(2, 16, 128, itemsize=2, chunk_bytes=4096)
    plane = torch.zeros(layout.capacity_bytes // 2, dtype=torch.bfloat16, device=cuda_device)
    out = torch.zeros((2, 4, 128), dtype=torch.bfloat16, device=cuda_device)
    pos = torch.zeros((2, 4), dtype=torch.int32, device=cuda_device)
    ids = torch.arange(2, device=cuda_device)
    lengths = torch.full((2,), 16, device=cuda_device)
    with pytest.raises(ValueError, match="planes_per_layer"):
        LayerGather([plane] * 3, [pos, pos], ids, lengths, None, None, [out] * 3, layout, planes_per_layer=2,
                    indirect=False)
    with pytest.raises(ValueError, match="one request table per layer"):
        LayerGather([plane] * 4, [pos, pos], ids, lengths, [pos], None, [out] * 4, layout, planes_per_layer=2,
                    indirect=False, mapped=True)
    with pytest.raises(ValueError, match="EKV_MAX_LAYERS"):
        LayerGather([plane] * 129, [pos] * 129, ids, lengths, None, None, [out] * 129, layout,
                    planes_per_layer=1, indirect=False)
