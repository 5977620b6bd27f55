"""GPU parity of the logical-shadow checker (ekv_shadow_*) against the reference's
LogicalShadow outputs (golden fixtures) and the CPU oracle."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import load_npz_cases
from oracle import logical_shadow as osh

pytestmark = pytest.mark.gpu

CASES = load_npz_cases("shadow_golden.npz")


def _bf16(array, device):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device).view(torch.bfloat16)


def _t(array, device):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)


@pytest.mark.parametrize("case", sorted(c for c in CASES if c.startswith("check_")))
def test_check_matches_reference(case, cuda_device):
    from ekv_b200.logical_shadow import LogicalShadow

    c = CASES[case]
    shadow = LogicalShadow(c["k_shadow"].shape[0], cuda_device)
    shadow.layers[3] = (_bf16(c["k_shadow"], cuda_device), _bf16(c["v_shadow"], cuda_device),
                        _t(c["initialized"], cuda_device))
    physical = _t(c["physical"], cuda_device) if "physical" in c else None
    live = _t(c["live_pages"], cuda_device) if "live_pages" in c else None
    clean, phys_out = shadow.check(3, _bf16(c["k_cache"], cuda_device), _bf16(c["v_cache"], cuda_device),
                                   _t(c["table"], cuda_device), _t(c["lengths"], cuda_device),
                                   _t(c["rows"], cuda_device), int(c["block_size"]), _t(c["blocks"], cuda_device),
                                   physical, live, int(c["page_size"]))
    np.testing.assert_array_equal(shadow.counts.cpu().numpy(), c["counts"])
    np.testing.assert_array_equal(clean.cpu().numpy(), c["clean_blocks"])
    assert clean.dtype == torch.from_numpy(c["clean_blocks"]).dtype
    np.testing.assert_array_equal(phys_out.cpu().numpy(), c["physical_out"])
    assert shadow.dirty
    # Counters accumulate across calls, as the reference's add_ does.
    shadow.check(3, _bf16(c["k_cache"], cuda_device), _bf16(c["v_cache"], cuda_device),
                 _t(c["table"], cuda_device), _t(c["lengths"], cuda_device), _t(c["rows"], cuda_device),
                 int(c["block_size"]), _t(c["blocks"], cuda_device), physical, live, int(c["page_size"]))
    np.testing.assert_array_equal(shadow.counts.cpu().numpy(), 2 * c["counts"])


def _pool_of(c, device):
    n_layers = sum(1 for k in c if k.startswith("pool_k"))
    pool_k = [_bf16(c[f"pool_k{i}"], device) for i in range(n_layers)]
    pool_v = [_bf16(c[f"pool_v{i}"], device) for i in range(n_layers)]
    return SimpleNamespace(page_size=int(c["page_size"]), size=int(c["size"]),
                           adaptive_vmm=SimpleNamespace(pages=set(c["pages"].tolist())),
                           start_layer=10, end_layer=10 + n_layers,
                           get_key_buffer=lambda layer: pool_k[layer - 10],
                           get_value_buffer=lambda layer: pool_v[layer - 10]), n_layers


@pytest.mark.parametrize("case", sorted(c for c in CASES if c.startswith("complete_")))
def test_check_complete_matches_reference(case, cuda_device):
    from ekv_b200.logical_shadow import LogicalShadow

    c = CASES[case]
    shadow = LogicalShadow(int(c["capacity"]), cuda_device)
    pool, n_layers = _pool_of(c, cuda_device)
    for i in range(n_layers):
        shadow.layers[10 + i] = (_bf16(c[f"k_shadow{i}"], cuda_device), _bf16(c[f"v_shadow{i}"], cuda_device),
                                 _t(c[f"initialized{i}"], cuda_device))
    logical, physical = _t(c["logical"], cuda_device), _t(c["physical"], cuda_device)
    if bool(c["raised"]):
        with pytest.raises(RuntimeError, match="migration shadow mismatch at test"):
            shadow.check_complete(pool, logical, physical, "test")
    else:
        shadow.check_complete(pool, logical, physical, "test")
    assert list(shadow.migration_counts.values()) == c["counts"].tolist()


def test_write_and_reset_match_index_assignment(cuda_device):
    """write = k[locations] = key, valid[locations] = True; reset clears the flags on
    every layer (logical_shadow.py:26-43), for 2 KiB, 24 B and unaligned key rows."""
    from ekv_b200.logical_shadow import LogicalShadow

    gen = torch.Generator().manual_seed(3)
    capacity = 5000
    shadow = LogicalShadow(capacity, cuda_device)
    expected = {}
    for layer, shape in ((0, (8, 128)), (1, (1, 12)), (2, (3, 5))):
        k_ref = None
        for round_ in range(3):
            n = 700
            loc = torch.randperm(capacity, generator=gen)[:n]
            key = torch.randn((n, *shape), generator=gen).to(torch.bfloat16)
            value = torch.randn((n, *shape), generator=gen).to(torch.bfloat16)
            if round_ == 2:
                # A strided producer: every second row of a larger buffer.
                key = torch.randn((2 * n, *shape), generator=gen).to(torch.bfloat16)[::2]
                value = torch.randn((2 * n, *shape), generator=gen).to(torch.bfloat16)[::2]
            shadow.write(layer, loc.to(cuda_device), key.to(cuda_device), value.to(cuda_device), (None, 1.0))
            if k_ref is None:
                k_ref = torch.zeros((capacity, *shape), dtype=torch.bfloat16)
                v_ref = torch.zeros((capacity, *shape), dtype=torch.bfloat16)
                valid_ref = torch.zeros(capacity, dtype=torch.bool)
            k_ref[loc], v_ref[loc], valid_ref[loc] = key, value, True
        expected[layer] = (k_ref, v_ref, valid_ref)
    for layer, (k_ref, v_ref, valid_ref) in expected.items():
        k, v, valid = shadow.layers[layer]
        assert torch.equal(valid.cpu(), valid_ref)
        mask = valid_ref
        assert torch.equal(k.cpu()[mask].view(torch.int16), k_ref[mask].view(torch.int16))
        assert torch.equal(v.cpu()[mask].view(torch.int16), v_ref[mask].view(torch.int16))
    forget = torch.randperm(capacity, generator=gen)[:1000]
    shadow.reset(forget.to(cuda_device))
    for layer, (_, _, valid_ref) in expected.items():
        valid_ref[forget] = False
        assert torch.equal(shadow.layers[layer][2].cpu(), valid_ref)
    with pytest.raises(RuntimeError, match="unit-scale BF16"):
        shadow.write(0, loc, key.float(), value, (None, None))


def test_check_at_decode_scale_against_oracle(cuda_device):
    """32 requests x 2048 Top-K tokens of 2 KiB rows, shadow written through the kernel,
    a cache holding the rows at permuted physical slots with planted corruptions."""
    from ekv_b200.logical_shadow import LogicalShadow

    gen = torch.Generator().manual_seed(9)
    capacity, slots, batch, topk, ctx, page = 40000, 50000, 32, 2048, 8192, 16
    heads, dim = 8, 128
    shadow = LogicalShadow(capacity, cuda_device)
    written = torch.randperm(capacity, generator=gen)[:36000]
    key = torch.randn((len(written), heads, dim), generator=gen).to(torch.bfloat16)
    value = torch.randn((len(written), heads, dim), generator=gen).to(torch.bfloat16)
    shadow.write(0, written.to(cuda_device), key.to(cuda_device), value.to(cuda_device), (None, None))
    k_shadow, v_shadow, initialized = (t.cpu() for t in shadow.layers[0])
    phys_of = torch.randperm(slots - page, generator=gen)[:capacity] + page
    k_cache = torch.randn((slots, heads, dim), generator=gen).to(torch.bfloat16)
    v_cache = torch.randn((slots, heads, dim), generator=gen).to(torch.bfloat16)
    k_cache[phys_of], v_cache[phys_of] = k_shadow, v_shadow
    bad = torch.randperm(capacity, generator=gen)[:300]
    k_cache[phys_of[bad[:150]], 3, 7] = torch.tensor(99.0, dtype=torch.bfloat16)
    v_cache[phys_of[bad[150:]], 7, 127] = torch.tensor(-99.0, dtype=torch.bfloat16)
    table = torch.randint(0, capacity, (batch, ctx), generator=gen, dtype=torch.int32)
    lengths = torch.randint(ctx // 2, ctx + 1, (batch,), generator=gen, dtype=torch.int64)
    rows = torch.randperm(batch, generator=gen)
    blocks = torch.stack([torch.randperm(int(lengths[b]), generator=gen)[:topk] for b in range(batch)])
    blocks = blocks.to(torch.int32)[None]
    blocks[0, 3, 100:] = -1
    blocks[0, 5, 10] = ctx + 50  # malformed: ends the prefix
    logical = table[rows[:, None], blocks[0].clamp(0, ctx - 1).long()]
    physical = phys_of[logical.long()].to(torch.int32)[None]
    live = torch.rand(slots // page + 1, generator=gen) < 0.97
    want = osh.check(k_shadow.view(torch.int16).numpy(), v_shadow.view(torch.int16).numpy(), initialized.numpy(),
                     k_cache.view(torch.int16).numpy(), v_cache.view(torch.int16).numpy(), table.numpy(),
                     lengths.numpy(), rows.numpy(), 1, blocks.numpy(), physical.numpy(), live.numpy(), page)
    clean, phys_out = shadow.check(0, k_cache.to(cuda_device), v_cache.to(cuda_device), table.to(cuda_device),
                                   lengths.to(cuda_device), rows.to(cuda_device), 1, blocks.to(cuda_device),
                                   physical.to(cuda_device), live.to(cuda_device), page)
    np.testing.assert_array_equal(shadow.counts.cpu().numpy(), want[0])
    np.testing.assert_array_equal(clean.cpu().numpy(), want[1])
    np.testing.assert_array_equal(phys_out.cpu().numpy(), want[2])
    assert want[0][4] > 0 and want[0][0] > 50000


def test_check_complete_multi_layer_against_oracle(cuda_device):
    """A migration of 20000 slot pairs over 12 layers of 1 KiB rows."""
    from ekv_b200.logical_shadow import LogicalShadow

    gen = torch.Generator().manual_seed(12)
    capacity, size, page, n, layers = 30000, 32768, 16, 20000, 12
    shadow = LogicalShadow(capacity, cuda_device)
    logical = torch.randperm(capacity - page, generator=gen)[:n] + page
    physical = torch.randperm(size, generator=gen)[:n] + page
    pool_k, pool_v, oracle_layers = [], [], []
    for layer in range(layers):
        written = torch.randperm(capacity, generator=gen)[:28000]
        key = torch.randn((len(written), 4, 128), generator=gen).to(torch.bfloat16)
        value = torch.randn((len(written), 4, 128), generator=gen).to(torch.bfloat16)
        shadow.write(layer, written.to(cuda_device), key.to(cuda_device), value.to(cuda_device), (None, None))
        k, v, valid = (t.cpu() for t in shadow.layers[layer])
        pk = torch.randn((size + page, 4, 128), generator=gen).to(torch.bfloat16)
        pv = torch.randn((size + page, 4, 128), generator=gen).to(torch.bfloat16)
        pk[physical], pv[physical] = k[logical], v[logical]
        pk[physical[layer::997], 0, 0] = torch.tensor(5.5, dtype=torch.bfloat16)
        pool_k.append(pk.to(cuda_device))
        pool_v.append(pv.to(cuda_device))
        oracle_layers.append((k.view(torch.int16).numpy(), v.view(torch.int16).numpy(), valid.numpy()))
    pages = set(range(1, size // page + 1)) - {int(physical[0]) // page}
    pool = SimpleNamespace(page_size=page, size=size, adaptive_vmm=SimpleNamespace(pages=pages), start_layer=0,
                           end_layer=layers, get_key_buffer=lambda layer: pool_k[layer],
                           get_value_buffer=lambda layer: pool_v[layer])
    live = np.zeros(size // page + 1, dtype=bool)
    live[sorted(pages)] = True
    want = osh.check_complete(oracle_layers, [p.cpu().view(torch.int16).numpy() for p in pool_k],
                              [p.cpu().view(torch.int16).numpy() for p in pool_v], logical.numpy(),
                              physical.numpy(), page, size, live, capacity)
    with pytest.raises(RuntimeError, match="mismatch at migration"):
        shadow.check_complete(pool, logical.to(cuda_device), physical.to(cuda_device), "migration")
    assert list(shadow.migration_counts.values()) == want.tolist()
    assert want[3] > 0 and want[0] > 100000
