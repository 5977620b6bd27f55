"""GPU parity of the residency lookups (R1, R2) against the oracle and the reference's golden vectors."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_npz_cases
from oracle import lookup as ol

pytestmark = pytest.mark.gpu


def _strided_cuda(values: np.ndarray, device) -> torch.Tensor:
    """Stride-2 CUDA view of ``values`` (tests/smoke_resident_lookup.py:28-33)."""
    source = torch.from_numpy(np.ascontiguousarray(values)).to(device)
    backing = torch.zeros((*source.shape, 2), dtype=source.dtype, device=device)
    view = backing[..., 1]
    view.copy_(source)
    return view


@pytest.mark.parametrize("case", sorted(load_npz_cases("lookup_golden.npz")))
@pytest.mark.parametrize("strided", [False, True])
def test_resolve_resident_matches_reference(case, strided, cuda_device):
    from ekv_b200.resident_lookup import resolve_resident

    c = load_npz_cases("lookup_golden.npz")[case]
    if strided:
        prep = lambda a: _strided_cuda(a, cuda_device)  # noqa: E731
        shape = c["expected"].shape
        output = torch.full((shape[0], shape[1], shape[2] * 2), int(c["init"]), dtype=torch.int32,
                            device=cuda_device)[..., ::2]
    else:
        prep = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
        output = torch.full(c["expected"].shape, int(c["init"]), dtype=torch.int32, device=cuda_device)
    resolve_resident(prep(c["topk"]), prep(c["table"]), prep(c["mapping"]), prep(c["rows"]),
                     prep(c["lengths"]), prep(c["selected"]), output, int(c["block_size"]))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(output.cpu().numpy(), c["expected"])


def test_resolve_resident_empty_selection_is_noop(cuda_device):
    from ekv_b200.resident_lookup import resolve_resident

    dev = cuda_device
    out = torch.full((1, 2, 4), -77, dtype=torch.int32, device=dev)
    resolve_resident(torch.zeros((1, 2, 4), dtype=torch.int32, device=dev),
                     torch.zeros((2, 4), dtype=torch.int64, device=dev),
                     torch.zeros(4, dtype=torch.int64, device=dev), torch.zeros(2, dtype=torch.int64, device=dev),
                     torch.ones(2, dtype=torch.int32, device=dev), torch.zeros(0, dtype=torch.int64, device=dev),
                     out, 1)
    torch.cuda.synchronize()
    assert (out == -77).all()


def _resident_map(gen, batch, ctx, resident, device):
    """cfg1 residency map: -1, with `resident` random tokens per row holding a
    permutation of hot slots [0, resident)."""
    res_map = torch.full((batch, ctx), -1, dtype=torch.int32)
    resident_tokens = []
    for b in range(batch):
        tokens = torch.randperm(ctx, generator=gen)[:resident]
        res_map[b, tokens] = torch.randperm(resident, generator=gen).to(torch.int32)
        resident_tokens.append(tokens)
    return res_map, resident_tokens


def _topk(gen, res_map, resident_tokens, k, hits):
    batch, ctx = res_map.shape
    rows = []
    for b in range(batch):
        hit = resident_tokens[b][torch.randperm(resident_tokens[b].numel(), generator=gen)[:hits]]
        non = torch.nonzero(res_map[b] < 0).flatten()
        miss = non[torch.randperm(non.numel(), generator=gen)[:k - hits]]
        row = torch.cat([hit, miss])[torch.randperm(k, generator=gen)]
        rows.append(row)
    return torch.stack(rows).to(torch.int32)


@pytest.mark.parametrize("with_lengths", [False, True])
def test_lookup_slots_config1_bit_exact(with_lengths, cuda_device):
    """Config 1 at full size: 32 x 16384 map, 2048 resident, Top-K 512 (~75% hits)."""
    from ekv_b200.resident_lookup import lookup_slots

    gen = torch.Generator().manual_seed(1)
    res_map, resident_tokens = _resident_map(gen, 32, 16384, 2048, cuda_device)
    topk = _topk(gen, res_map, resident_tokens, 512, 384)
    lengths = torch.randint(8000, 16385, (32,), generator=gen).to(torch.int32) if with_lengths else None
    expected = ol.lookup_slots(res_map.numpy(), topk.numpy(), None if lengths is None else lengths.numpy())
    got = lookup_slots(res_map.to(cuda_device), topk.to(cuda_device),
                       None if lengths is None else lengths.to(cuda_device))
    torch.cuda.synchronize()
    for g, e in zip(got, expected):
        np.testing.assert_array_equal(g.cpu().numpy(), e)
    if not with_lengths:
        assert int(got[3].sum()) == 32 * 128


@pytest.mark.parametrize("k,map_dtype,topk_dtype", [(700, torch.int64, torch.int32), (1, torch.int32, torch.int64),
                                                   (2048, torch.int32, torch.int32), (0, torch.int32, torch.int32)])
def test_lookup_slots_ragged_shapes(k, map_dtype, topk_dtype, cuda_device):
    from ekv_b200.resident_lookup import lookup_slots

    gen = torch.Generator().manual_seed(k + 5)
    batch, ctx = 7, 3000
    res_map = torch.where(torch.rand((batch, ctx), generator=gen) < 0.4,
                          torch.randint(0, 1 << 20, (batch, ctx), generator=gen), -1).to(map_dtype)
    topk = torch.randint(-3, ctx + 50, (batch, k), generator=gen).to(topk_dtype)
    lengths = torch.randint(0, ctx + 1, (batch,), generator=gen).to(torch.int64)
    expected = ol.lookup_slots(res_map.numpy(), topk.numpy(), lengths.numpy())
    got = lookup_slots(res_map.to(cuda_device), topk.to(cuda_device), lengths.to(cuda_device))
    torch.cuda.synchronize()
    for g, e in zip(got, expected):
        np.testing.assert_array_equal(g.cpu().numpy(), e)


def test_resolve_resident_config_scale_matches_torch_resolver(cuda_device):
    """cfg5-sized lookup (B=128, Top-K 2048, page size 1) against the reference's torch
    resolver restated in numpy (request_residency.py:819-826)."""
    from ekv_b200.resident_lookup import resolve_resident

    gen = torch.Generator().manual_seed(9)
    batch, ctx, k = 128, 65536, 2048
    table = torch.randperm(batch * ctx, generator=gen).reshape(batch, ctx).to(torch.int32)
    mapping = torch.randint(0, 1 << 30, (batch * ctx,), generator=gen)
    rows = torch.randperm(batch, generator=gen)
    lengths = torch.randint(ctx // 2, ctx + 1, (batch,), generator=gen).to(torch.int32)
    topk = torch.randint(-1, ctx, (1, batch, k), generator=gen).to(torch.int32)
    selected = torch.randperm(batch, generator=gen)[:100]
    out = torch.full((1, batch, k), -77, dtype=torch.int32, device=cuda_device)
    resolve_resident(topk.to(cuda_device), table.to(cuda_device), mapping.to(cuda_device),
                     rows.to(cuda_device), lengths.to(cuda_device), selected.to(cuda_device), out, 1)
    torch.cuda.synchronize()
    expected = ol.torch_resolver_numpy(topk.numpy(), table.numpy(), mapping.numpy(), rows.numpy(),
                                       lengths.numpy(), selected.numpy(), 1)
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got[0, selected.numpy()], expected)
    untouched = np.setdiff1d(np.arange(batch), selected.numpy())
    assert (got[0, untouched] == -77).all()


def test_compiled_binding_is_loaded_and_matches_the_ctypes_path(cuda_device, monkeypatch):
    """The pybind11 binding serves resolve_resident / lookup_slots when it is built, and
    gives the same results as the ctypes path (forced by hiding the binding)."""
    from ekv_b200 import _lib, resident_lookup

    assert _lib.torch_binding() is not None, "lib/_ekv_torch.so was not built"
    gen = torch.Generator().manual_seed(31)
    batch, ctx, k = 8, 4096, 300
    res_map = torch.full((batch, ctx), -1, dtype=torch.int32)
    for b in range(batch):
        tokens = torch.randperm(ctx, generator=gen)[:1000]
        res_map[b, tokens] = torch.randperm(1000, generator=gen).to(torch.int32)
    topk = torch.randint(-5, ctx + 5, (batch, k), generator=gen, dtype=torch.int32)
    lengths = torch.randint(ctx // 2, ctx + 1, (batch,), generator=gen, dtype=torch.int64)
    args = (res_map.to(cuda_device), topk.to(cuda_device), lengths.to(cuda_device))
    fast = [t.cpu() for t in resident_lookup.lookup_slots(*args)]
    table = torch.randint(0, 5000, (6, 512), generator=gen, dtype=torch.int64)
    mapping = torch.randint(-2, 1 << 20, (5001,), generator=gen, dtype=torch.int64)
    blocks = torch.randint(-1, 40, (1, 6, 16), generator=gen, dtype=torch.int32)
    rows, lens, sel = torch.tensor([5, 4, 3, 2, 1, 0]), torch.randint(1, 512, (6,), generator=gen), torch.tensor([0, 2, 5])
    res_args = [t.to(cuda_device) for t in (blocks, table, mapping, rows, lens, sel)]
    out_fast = torch.full((1, 6, 16 * 8), -77, dtype=torch.int32, device=cuda_device)
    resident_lookup.resolve_resident(*res_args, out_fast, 8)
    monkeypatch.setattr(resident_lookup, "torch_binding", lambda: None)
    slow = [t.cpu() for t in resident_lookup.lookup_slots(*args)]
    out_slow = torch.full((1, 6, 16 * 8), -77, dtype=torch.int32, device=cuda_device)
    resident_lookup.resolve_resident(*res_args, out_slow, 8)
    for a, b in zip(fast, slow):
        assert torch.equal(a, b)
    assert torch.equal(out_fast, out_slow)
    assert (out_fast[0, 1] == -77).all()  # rows not selected stay untouched
