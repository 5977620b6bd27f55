"""GPU parity of the hot-buffer swap-in (victim selection, promotion, mapped gather) and a
multi-step sparse decode loop against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import lookup as ol
from oracle import swap as osw

pytestmark = pytest.mark.gpu


def _state(rng, batch, context, hot, fill):
    """A consistent residency state: `fill` resident tokens per row in random slots."""
    res_map = np.full((batch, context), -1, dtype=np.int32)
    slot_token = np.full((batch, hot), -1, dtype=np.int32)
    for b in range(batch):
        tokens = rng.choice(context, fill, replace=False)
        slots = rng.choice(hot, fill, replace=False)
        res_map[b, tokens] = slots
        slot_token[b, slots] = tokens
    hand = rng.integers(0, hot, batch).astype(np.int32)
    return res_map, slot_token, hand


def _topk(rng, res_map, k, hit_fraction):
    batch, context = res_map.shape
    out = np.empty((batch, k), dtype=np.int32)
    for b in range(batch):
        resident = np.nonzero(res_map[b] >= 0)[0]
        absent = np.nonzero(res_map[b] < 0)[0]
        hits = min(int(k * hit_fraction), resident.size)
        pick = np.concatenate([rng.choice(resident, hits, replace=False),
                               rng.choice(absent, k - hits, replace=False)])
        out[b] = rng.permutation(pick)
    return out


@pytest.mark.parametrize("batch,context,hot,k,fill,hit", [
    (6, 3000, 256, 64, 200, 0.7),     # ring smaller than one tile
    (3, 20000, 8192, 2048, 6000, 0.9),  # several tiles, hand anywhere
    (4, 500, 64, 48, 64, 0.5),        # full buffer, evictions wrap the ring
    (2, 800, 100, 30, 0, 0.0),        # cold: every Top-K token misses
])
def test_swap_select_matches_oracle(batch, context, hot, k, fill, hit, cuda_device):
    from ekv_b200.resident_lookup import lookup_slots
    from ekv_b200.swap import swap_select

    rng = np.random.default_rng(batch * 1000 + hot)
    res_map, slot_token, hand = _state(rng, batch, context, hot, fill)
    topk = _topk(rng, res_map, k, hit)
    dev = cuda_device
    g_map, g_tok, g_hand = (torch.from_numpy(a.copy()).to(dev) for a in (res_map, slot_token, hand))
    slots, _, miss_list, miss_count = lookup_slots(g_map, torch.from_numpy(topk).to(dev))
    promo = torch.empty((batch, k), dtype=torch.int32, device=dev)
    swap_select(g_map, g_tok, g_hand, slots, miss_list, miss_count, promo)
    torch.cuda.synchronize()
    o_slots, _, o_list, o_count = ol.lookup_slots(res_map, topk)
    o_promo = osw.swap_select(res_map, slot_token, hand, o_slots, o_list, o_count)
    np.testing.assert_array_equal(promo.cpu().numpy(), o_promo)
    np.testing.assert_array_equal(g_map.cpu().numpy(), res_map)
    np.testing.assert_array_equal(g_tok.cpu().numpy(), slot_token)
    np.testing.assert_array_equal(g_hand.cpu().numpy(), hand)
    # Every Top-K token is resident afterwards, in a distinct slot.
    for b in range(batch):
        s = res_map[b, topk[b]]
        assert (s >= 0).all() and np.unique(s).size == k


def test_promote_rows_matches_oracle(cuda_device):
    from ekv_b200.host_pool import pinned_buffer
    from ekv_b200.swap import promote_rows
    from ekv_b200.virtual_layout import VirtualKVLayout

    rng = np.random.default_rng(5)
    batch, context, hot, k, row_bytes = 3, 700, 96, 40, 256
    layout = VirtualKVLayout(batch, hot, row_bytes // 2, chunk_bytes=1 << 16)
    histories = []
    for _ in range(2):
        h = pinned_buffer(batch * context * row_bytes)[: batch * context * row_bytes].view(batch * context, row_bytes)
        h.copy_(torch.from_numpy(rng.integers(0, 256, (batch * context, row_bytes), dtype=np.uint8)))
        histories.append(h)
    hot_planes = [torch.zeros(layout.capacity_bytes, dtype=torch.uint8, device=cuda_device) for _ in range(2)]
    miss_count = np.array([40, 0, 17], dtype=np.int32)
    miss_list = np.full((batch, k), -1, dtype=np.int32)
    promo = np.full((batch, k), -1, dtype=np.int32)
    for b in range(batch):
        n = miss_count[b]
        miss_list[b, :n] = rng.choice(context, n, replace=False)
        promo[b, :n] = rng.choice(hot, n, replace=False)
    promote_rows(histories, hot_planes, layout, context, *(torch.from_numpy(a).to(cuda_device)
                                                            for a in (miss_list, miss_count, promo)))
    torch.cuda.synchronize()
    for h, plane in zip(histories, hot_planes):
        want = np.zeros((batch, hot, row_bytes), dtype=np.uint8)
        osw.promote_rows(h.numpy(), want, miss_list, miss_count, promo, context)
        got = plane.cpu().numpy()[layout.chunk_bytes:].reshape(batch, -1)[:, : hot * row_bytes]
        np.testing.assert_array_equal(got.reshape(batch, hot, row_bytes), want)


def _evolve(rng, previous, context, keep, new_dist):
    """Keep `keep` of the previous ids, draw the rest from `new_dist` (distinct)."""
    batch, k = previous.shape
    out = np.empty_like(previous)
    for b in range(batch):
        kept = previous[b, :keep]
        chosen = set(kept.tolist())
        fresh = []
        while len(fresh) < k - keep:
            t = int(new_dist(rng))
            if t not in chosen:
                chosen.add(t)
                fresh.append(t)
        out[b] = rng.permutation(np.concatenate([kept, np.array(fresh, dtype=np.int32)]))
    return out


def test_multi_step_decode_matches_oracle(cuda_device):
    """Several layers, several decode steps: lookup -> swap -> promote -> mapped gather,
    outputs and residency state bit-exact against the oracle at every step."""
    from ekv_b200.host_pool import pinned_buffer
    from ekv_b200.swap import HotLayer, SwapStep

    rng = np.random.default_rng(11)
    batch, context, hot, k, width, layers, steps = 4, 1024, 128, 48, 64, 2, 8
    row_bytes = width * 2
    histories = []
    for _ in range(2):  # K and V history, shared by the layers
        h = pinned_buffer(batch * context * row_bytes)[: batch * context * row_bytes].view(batch * context, row_bytes)
        h.copy_(torch.from_numpy(rng.integers(0, 256, (batch * context, row_bytes), dtype=np.uint8)))
        histories.append(h)
    hist_np = [h.numpy() for h in histories]
    dev = cuda_device
    gpu_layers = [HotLayer(batch, context, hot, width, dev, chunk_bytes=1 << 16) for _ in range(layers)]
    oracle_state = [dict(res_map=np.full((batch, context), -1, np.int32),
                         slot_token=np.full((batch, hot), -1, np.int32), hand=np.zeros(batch, np.int32),
                         hot_rows=[np.zeros((batch, hot, row_bytes), np.uint8) for _ in range(2)])
                    for _ in range(layers)]
    topk = np.stack([rng.choice(context, k, replace=False) for _ in range(batch)]).astype(np.int32)
    topk_dev = torch.from_numpy(topk).to(dev)
    outputs = [[torch.empty((batch, k, width), dtype=torch.bfloat16, device=dev) for _ in range(2)]
               for _ in range(layers)]
    plans = [SwapStep(layer, topk_dev, [h.view(torch.bfloat16) for h in histories], outputs[i])
             for i, layer in enumerate(gpu_layers)]
    zipf = lambda r: context - 1 - min(int(r.zipf(1.1)) - 1, context - 1)  # noqa: E731
    lengths = np.full(batch, context)
    for step in range(steps):
        if step:
            topk = _evolve(rng, topk, context, int(0.9 * k), zipf)
            topk_dev.copy_(torch.from_numpy(topk))
        for layer in range(layers):
            plans[layer]()
            st = oracle_state[layer]
            slots, _, miss_list, miss_count = ol.lookup_slots(st["res_map"], topk)
            promo = osw.swap_select(st["res_map"], st["slot_token"], st["hand"], slots, miss_list, miss_count)
            for plane in range(2):
                osw.promote_rows(hist_np[plane], st["hot_rows"][plane], miss_list, miss_count, promo, context)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(plans[layer].lookup.miss_list.cpu().numpy(), miss_list)
            np.testing.assert_array_equal(plans[layer].promo_slot.cpu().numpy(), promo)
            np.testing.assert_array_equal(gpu_layers[layer].res_map.cpu().numpy(), st["res_map"])
            for plane in range(2):
                want = osw.mapped_gather(st["hot_rows"][plane], st["res_map"], topk, lengths)
                got = outputs[layer][plane].view(torch.uint8).cpu().numpy().reshape(batch, k, row_bytes)
                np.testing.assert_array_equal(got, want)
                # Size-independent property: every gathered row is the token's history row.
                rows = np.arange(batch)[:, None] * context + topk
                np.testing.assert_array_equal(got, hist_np[plane][rows])


@pytest.mark.parametrize("graph", [False, True])
def test_pipeline_equals_layer_order(graph, cuda_device):
    """SwapPipeline (layer i's gather on a second stream during layer i+1's promotion)
    leaves exactly the state and outputs of running the layers in order, step after
    step; with ``graph`` the pipelined step is captured once and replayed.  Layers share
    one output pair, as a decode step does."""
    from ekv_b200.host_pool import pinned_buffer
    from ekv_b200.swap import HotLayer, SwapPipeline, SwapStep

    rng = np.random.default_rng(21)
    batch, context, hot, k, width, layers, steps = 16, 4096, 512, 256, 256, 6, 6
    row_bytes = width * 2
    histories = []
    for _ in range(2):
        h = pinned_buffer(batch * context * row_bytes)[: batch * context * row_bytes].view(batch * context, row_bytes)
        h.copy_(torch.from_numpy(rng.integers(0, 256, (batch * context, row_bytes), dtype=np.uint8)))
        histories.append(h)
    hist_views = [h.view(torch.bfloat16) for h in histories]
    dev = cuda_device
    topk = np.stack([rng.choice(context, k, replace=False) for _ in range(batch)]).astype(np.int32)
    topk_dev = torch.from_numpy(topk).to(dev)
    runs = {}
    for mode in ("ordered", "pipelined"):
        topk_dev.copy_(torch.from_numpy(topk))  # each mode starts from the same step-0 Top-K
        hot_layers = [HotLayer(batch, context, hot, width, dev, chunk_bytes=1 << 16) for _ in range(layers)]
        shared = [torch.empty((batch, k, width), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        plans = [SwapStep(layer, topk_dev, hist_views, shared) for layer in hot_layers]
        pipeline = SwapPipeline(plans)
        replay = None
        if graph and mode == "pipelined":
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                pipeline()  # warm-up outside capture: counts as step 0
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize()
            replay = torch.cuda.CUDAGraph()
            with torch.cuda.graph(replay):
                pipeline()
        local = np.random.default_rng(5)
        ids = topk.copy()
        outs, states = [], []
        zipf = lambda r: context - 1 - min(int(r.zipf(1.1)) - 1, context - 1)  # noqa: E731
        for step in range(steps):
            if step:
                ids = _evolve(local, ids, context, int(0.9 * k), zipf)
            topk_dev.copy_(torch.from_numpy(ids))
            if mode == "ordered":
                if graph and step == 0:
                    for plan in plans:
                        plan()  # the pipelined run's warm-up step
                for plan in plans:
                    plan()
            elif replay is not None:
                replay.replay()
            else:
                pipeline()
            torch.cuda.synchronize()
            outs.append([o.view(torch.uint8).cpu().numpy().copy() for o in shared])
            states.append([(l.res_map.cpu().numpy().copy(), l.slot_token.cpu().numpy().copy()) for l in hot_layers])
            rows = np.arange(batch)[:, None] * context + ids
            for plane in range(2):  # the last layer's rows are the tokens' history rows
                np.testing.assert_array_equal(outs[-1][plane].reshape(batch, k, row_bytes),
                                              histories[plane].numpy()[rows])
        runs[mode] = (outs, states)
        del replay
    for step in range(steps):
        for a, b in zip(runs["ordered"][0][step], runs["pipelined"][0][step]):
            np.testing.assert_array_equal(a, b)
        for (ma, ta), (mb, tb) in zip(runs["ordered"][1][step], runs["pipelined"][1][step]):
            np.testing.assert_array_equal(ma, mb)
            np.testing.assert_array_equal(ta, tb)
