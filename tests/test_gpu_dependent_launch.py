"""Dependent launch is a scheduling switch only: a decode step of lookups and gathers gives
the same bytes, equal to the oracle's, with EKV_B200_PDL=0 (ordinary launches) as with
the default (programmatic dependent launches), including the fused lookup + gather whose
launches are marked disjoint (they copy before the previous layer completes).  The switch is read once per process, so
each setting runs in its own child process."""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import PACKAGE_ROOT, ROOT

pytestmark = pytest.mark.gpu

STEP = textwrap.dedent('''
    import sys

    import numpy as np
    import torch

    from ekv_b200.pipeline import LayerPipeline
    from ekv_b200.resident_lookup import LookupPlan
    from ekv_b200.sparse_read import LookupGather, PlaneGather
    from ekv_b200.virtual_layout import VirtualKVLayout
    from oracle import gather as og
    from oracle import lookup as ol

    dev = torch.device("cuda:0")
    gen = torch.Generator().manual_seed(5)
    layers, batch, context, hot, k, width = 4, 4, 2000, 128, 96, 64
    layout = VirtualKVLayout(batch, hot, width, itemsize=2, chunk_bytes=1 << 16)
    req_ids = torch.arange(batch, device=dev)
    hot_lengths = torch.full((batch,), hot, dtype=torch.int64, device=dev)
    ctx_lengths = torch.full((batch,), context, dtype=torch.int64, device=dev)
    saved, keep, lookups, mapped, direct, fused = {}, [], [], [], [], []
    for layer in range(layers):
        res_map = torch.full((batch, context), -1, dtype=torch.int32)
        topk = torch.empty((batch, k), dtype=torch.int32)
        for b in range(batch):
            perm = torch.randperm(context, generator=gen)
            res_map[b, perm[:hot]] = torch.randperm(hot, generator=gen).to(torch.int32)
            topk[b] = torch.cat([perm[:70], perm[hot:hot + k - 70]])[torch.randperm(k, generator=gen)].to(torch.int32)
        planes = [torch.randint(-30000, 30000, (layout.capacity_bytes // 2,), generator=gen, dtype=torch.int16)
                  for _ in range(2)]
        dmap, dtopk = res_map.to(dev), topk.to(dev)
        dplanes = [p.to(dev).view(torch.bfloat16) for p in planes]
        outs = {form: [torch.full((batch, k, width), 7, dtype=torch.int16, device=dev) for _ in range(2)]
                for form in ("mapped", "direct", "fused")}
        plan = LookupPlan(dmap, dtopk)
        lookups.append(plan)
        mapped.append(PlaneGather(dplanes, dtopk, req_ids, ctx_lengths, dmap, None,
                                  [o.view(torch.bfloat16) for o in outs["mapped"]], layout, indirect=False,
                                  mapped=True))
        direct.append(PlaneGather(dplanes, plan.slots, req_ids, hot_lengths, None, None,
                                  [o.view(torch.bfloat16) for o in outs["direct"]], layout, indirect=False))
        # The fused lookup + gather with every launch disjoint from the ones before it.
        fused.append(LookupGather(dplanes, dmap, dtopk, req_ids, ctx_lengths,
                                  [o.view(torch.bfloat16) for o in outs["fused"]], layout, indices_ready=True,
                                  disjoint=True))
        keep.append((dmap, dtopk, dplanes, outs))
        slots = ol.lookup_slots(res_map.numpy(), topk.numpy())[0]
        want = og.gather_rows_planes([p.numpy() for p in planes], slots, req_ids.cpu().numpy(),
                                     hot_lengths.cpu().numpy(), None, None, width=width, table_width=hot,
                                     request_stride=layout.request_bytes // 2,
                                     sink_elements=layout.chunk_bytes // 2, indirect=False)
        saved[f"want{layer}"] = np.stack(want)

    # The concurrent form from one CUDA graph, then the plain layer order eagerly.
    step = LayerPipeline(lookups, mapped, dev, wait=False)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for plan in lookups:
        plan.slots.fill_(-5)
    for _, _, _, outs in keep:
        for o in outs["mapped"]:
            o.fill_(7)
    graph.replay()
    torch.cuda.synchronize()
    saved.update({f"mapped{i}": np.stack([o.cpu().numpy() for o in keep[i][3]["mapped"]]) for i in range(layers)})
    for plan, gather in zip(lookups, direct):
        plan()
        gather()
    torch.cuda.synchronize()
    saved.update({f"direct{i}": np.stack([o.cpu().numpy() for o in keep[i][3]["direct"]]) for i in range(layers)})
    saved.update({f"slots{i}": lookups[i].slots.cpu().numpy() for i in range(layers)})
    saved.update({f"misses{i}": lookups[i].miss_list.cpu().numpy() for i in range(layers)})
    # The fused disjoint form from one CUDA graph (compaction beside the next layer).
    fused_step = LayerPipeline(fused, [f.compact for f in fused], dev)
    with torch.cuda.stream(side):
        fused_step()
    torch.cuda.current_stream(dev).wait_stream(side)
    fused_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(fused_graph):
        fused_step()
    for i, f in enumerate(fused):
        f.slots.fill_(-5)
        f.miss_list.fill_(-5)
        for o in keep[i][3]["fused"]:
            o.fill_(7)
    fused_graph.replay()
    torch.cuda.synchronize()
    saved.update({f"fused{i}": np.stack([o.cpu().numpy() for o in keep[i][3]["fused"]]) for i in range(layers)})
    saved.update({f"fused_slots{i}": fused[i].slots.cpu().numpy() for i in range(layers)})
    saved.update({f"fused_misses{i}": fused[i].miss_list.cpu().numpy() for i in range(layers)})
    del graph, fused_graph
    np.savez(sys.argv[1], **saved)
''')


def _run(tmp_path, pdl):
    out = tmp_path / f"pdl{pdl}.npz"
    paths = [str(PACKAGE_ROOT), str(ROOT), os.environ.get("PYTHONPATH", "")]
    env = dict(os.environ, EKV_B200_PDL=pdl, PYTHONPATH=os.pathsep.join(p for p in paths if p))
    subprocess.run([sys.executable, "-c", STEP, str(out)], env=env, check=True, timeout=300)
    return dict(np.load(out))


def test_dependent_launch_switch_changes_no_bytes(tmp_path):
    on, off = _run(tmp_path, "1"), _run(tmp_path, "0")
    assert sorted(on) == sorted(off)
    for key in on:
        np.testing.assert_array_equal(on[key], off[key], err_msg=key)
    for layer in range(4):
        np.testing.assert_array_equal(on[f"mapped{layer}"], on[f"want{layer}"])
        np.testing.assert_array_equal(on[f"direct{layer}"], on[f"want{layer}"])
        np.testing.assert_array_equal(on[f"fused{layer}"], on[f"want{layer}"])
        np.testing.assert_array_equal(on[f"fused_slots{layer}"], on[f"slots{layer}"])
        np.testing.assert_array_equal(on[f"fused_misses{layer}"], on[f"misses{layer}"])
