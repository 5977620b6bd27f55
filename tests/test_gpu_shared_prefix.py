"""GPU parity of the shared-prefix donor-slot resolver (ekv_resolve_shared_blocks)
against the reference's outputs (golden fixtures) and the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_npz_cases
from oracle import shared_prefix as osp

pytestmark = pytest.mark.gpu

CASES = load_npz_cases("shared_prefix_golden.npz")


def _t(array, device):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)


@pytest.mark.parametrize("case", sorted(CASES))
def test_matches_reference_outputs(case, cuda_device):
    from ekv_b200.shared_prefix import resolve_shared_block_locations, resolve_shared_block_locations_batched

    c = CASES[case]
    table, mapping = _t(c["request_table"], cuda_device), _t(c["device_mapping"], cuda_device)
    if "source_row" in c:
        valid, physical = resolve_shared_block_locations(
            _t(c["block_ids"], cuda_device), source_row=int(c["source_row"]),
            seq_len=torch.tensor(int(c["seq_len"]), device=cuda_device), shared_tokens=int(c["shared_tokens"]),
            block_size=int(c["block_size"]), request_table=table, device_mapping=mapping)
    else:
        valid, physical = resolve_shared_block_locations_batched(
            _t(c["block_ids"], cuda_device), source_rows=c["source_rows"].tolist(),
            seq_len=_t(c["seq_len"], cuda_device), shared_tokens=c["shared_tokens"].tolist(),
            block_size=int(c["block_size"]), request_table=table, device_mapping=mapping)
    assert valid.dtype == torch.bool and physical.dtype == torch.int32
    np.testing.assert_array_equal(valid.cpu().numpy(), c["valid"])
    np.testing.assert_array_equal(physical.cpu().numpy(), c["physical"])


def _random_case(seed, requests, per_request, block_size, table_rows, width, slots, table_dtype):
    gen = torch.Generator().manual_seed(seed)
    table = torch.randint(-2, slots, (table_rows, width), generator=gen, dtype=torch.int64)
    table[table < 0] = -1
    mapping = torch.randint(1, 1 << 24, (slots,), generator=gen, dtype=torch.int64)
    mapping[torch.rand(slots, generator=gen) < 0.05 / block_size] = 0
    blocks = torch.randint(-1, width // block_size + 4, (requests, per_request), generator=gen, dtype=torch.int64)
    rows = torch.randint(0, table_rows, (requests,), generator=gen).tolist()
    lengths = torch.randint(1, width + 8, (requests,), generator=gen, dtype=torch.int64)
    prefixes = torch.randint(0, width + 8, (requests,), generator=gen).tolist()
    return blocks, rows, lengths, prefixes, table.to(table_dtype), mapping


@pytest.mark.parametrize("block_size", [1, 4, 7, 32, 64, 128])
@pytest.mark.parametrize("extensions", [False, True])
def test_random_batches_with_strides_and_extensions(block_size, extensions, cuda_device):
    """Strided (transposed) block ids and table, int32 everywhere, plus the fused caller
    rule (exclude_newest) and the in-place masked block ids, against the oracle."""
    from ekv_b200.shared_prefix import resolve_shared_block_locations_batched

    blocks, rows, lengths, prefixes, table, mapping = _random_case(
        block_size, 9, 37, block_size, 6, 24 * block_size + 5, 5000, torch.int32)
    want_valid, want_physical = osp.resolve_batched(blocks.numpy(), rows, lengths.numpy(), prefixes, block_size,
                                                    table.numpy(), mapping.numpy(), exclude_newest=extensions)
    # Transposed storage: strides (1, requests) for the block ids, (1, rows) for the table.
    blocks_dev = blocks.to(torch.int32).t().contiguous().to(cuda_device).t()
    table_dev = table.t().contiguous().to(cuda_device).t()
    assert not blocks_dev.is_contiguous() and not table_dev.is_contiguous()
    masked = blocks_dev.clone().t().contiguous().t() if extensions else None
    valid, physical = resolve_shared_block_locations_batched(
        blocks_dev, source_rows=rows, seq_len=lengths.to(torch.int32).to(cuda_device), shared_tokens=prefixes,
        block_size=block_size, request_table=table_dev, device_mapping=mapping.to(cuda_device),
        exclude_newest=extensions, masked_block_ids=masked)
    np.testing.assert_array_equal(valid.cpu().numpy(), want_valid)
    np.testing.assert_array_equal(physical.cpu().numpy(), want_physical)
    if extensions:
        want_masked = np.where(want_valid, -1, blocks.numpy())
        np.testing.assert_array_equal(masked.cpu().numpy(), want_masked)
        assert want_valid.any() and not want_valid.all()


def test_in_place_masking_of_the_block_ids(cuda_device):
    """masked_block_ids may be block_ids itself (the caller's private Top-K tensor)."""
    from ekv_b200.shared_prefix import resolve_shared_block_locations_batched

    blocks, rows, lengths, prefixes, table, mapping = _random_case(5, 4, 64, 1, 4, 300, 1000, torch.int64)
    want_valid, _ = osp.resolve_batched(blocks.numpy(), rows, lengths.numpy(), prefixes, 1, table.numpy(),
                                        mapping.numpy(), exclude_newest=True)
    dev_blocks = blocks.to(cuda_device)
    valid, _ = resolve_shared_block_locations_batched(
        dev_blocks, source_rows=rows, seq_len=lengths.to(cuda_device), shared_tokens=prefixes, block_size=1,
        request_table=table.to(cuda_device), device_mapping=mapping.to(cuda_device), exclude_newest=True,
        masked_block_ids=dev_blocks)
    np.testing.assert_array_equal(valid.cpu().numpy(), want_valid)
    np.testing.assert_array_equal(dev_blocks.cpu().numpy(), np.where(want_valid, -1, blocks.numpy()))


def test_config5_scale(cuda_device):
    """The config-5 shape (128 consumers x 2048 Top-K, page size 1, 65536-token table):
    bit-exact against the oracle."""
    from ekv_b200.shared_prefix import resolve_shared_block_locations_batched

    requests, topk, ctx, slots = 128, 2048, 65536, 1 << 20
    gen = torch.Generator().manual_seed(55)
    table = torch.randint(0, slots, (requests, ctx), generator=gen, dtype=torch.int32)
    mapping = torch.randint(0, 1 << 22, (slots,), generator=gen, dtype=torch.int64)
    blocks = torch.stack([torch.randperm(ctx, generator=gen)[:topk] for _ in range(requests)]).to(torch.int32)
    rows = torch.randint(0, requests, (requests,), generator=gen).tolist()
    lengths = torch.full((requests,), ctx, dtype=torch.int64)
    prefixes = torch.randint(0, ctx, (requests,), generator=gen).tolist()
    want_valid, want_physical = osp.resolve_batched(blocks.numpy(), rows, lengths.numpy(), prefixes, 1,
                                                    table.numpy(), mapping.numpy())
    valid, physical = resolve_shared_block_locations_batched(
        blocks.to(cuda_device), source_rows=rows, seq_len=lengths.to(cuda_device), shared_tokens=prefixes,
        block_size=1, request_table=table.to(cuda_device), device_mapping=mapping.to(cuda_device))
    np.testing.assert_array_equal(valid.cpu().numpy(), want_valid)
    np.testing.assert_array_equal(physical.cpu().numpy(), want_physical)


def test_empty_and_single_block(cuda_device):
    from ekv_b200.shared_prefix import resolve_shared_block_locations, resolve_shared_block_locations_batched

    table = torch.arange(1, 13, device=cuda_device).reshape(2, 6)
    mapping = torch.arange(20, device=cuda_device)
    valid, physical = resolve_shared_block_locations(
        torch.empty(0, dtype=torch.long, device=cuda_device), source_row=0, seq_len=torch.tensor(6),
        shared_tokens=4, block_size=2, request_table=table, device_mapping=mapping)
    assert valid.shape == (0,) and physical.shape == (0, 2)
    valid, physical = resolve_shared_block_locations_batched(
        torch.empty(3, 0, dtype=torch.long, device=cuda_device), source_rows=[0, 1, 0], shared_tokens=[1, 2, 3],
        seq_len=torch.tensor([6, 6, 6]), block_size=2, request_table=table, device_mapping=mapping)
    assert valid.shape == (3, 0) and physical.shape == (3, 0, 2)
    valid, physical = resolve_shared_block_locations(
        torch.tensor([1], device=cuda_device), source_row=1, seq_len=6, shared_tokens=4, block_size=2,
        request_table=table, device_mapping=mapping)
    assert valid.tolist() == [True] and physical.tolist() == [[9, 10]]


@pytest.mark.parametrize("requests", [512, 513, 700])
def test_metadata_in_launch_parameters_and_on_the_device(requests, cuda_device):
    """Up to EKV_SHARED_INLINE_MAX requests the per-request lists ride in the launch
    parameters; above it they are copied to the device.  Same answers either way."""
    from ekv_b200.shared_prefix import resolve_shared_block_locations_batched

    blocks, rows, lengths, prefixes, table, mapping = _random_case(requests, requests, 5, 2, 40, 120, 500,
                                                                   torch.int64)
    want_valid, want_physical = osp.resolve_batched(blocks.numpy(), rows, lengths.numpy(), prefixes, 2,
                                                    table.numpy(), mapping.numpy())
    valid, physical = resolve_shared_block_locations_batched(
        blocks.to(cuda_device), source_rows=rows, seq_len=lengths.to(cuda_device), shared_tokens=prefixes,
        block_size=2, request_table=table.to(cuda_device), device_mapping=mapping.to(cuda_device))
    np.testing.assert_array_equal(valid.cpu().numpy(), want_valid)
    np.testing.assert_array_equal(physical.cpu().numpy(), want_physical)


def test_compiled_binding_matches_the_ctypes_path(cuda_device, monkeypatch):
    """The pybind11 binding serves the batched resolver (lists checked in C++) and gives
    the results of the ctypes path; lists it does not take (bools, numpy ints) go to the
    checked path, which answers as the reference does."""
    from ekv_b200 import _lib, shared_prefix as sp

    assert _lib.torch_binding() is not None, "lib/_ekv_torch.so was not built"
    blocks, rows, lengths, prefixes, table, mapping = _random_case(77, 12, 40, 4, 6, 200, 900, torch.int32)
    args = dict(source_rows=rows, seq_len=lengths.to(cuda_device), shared_tokens=prefixes, block_size=4,
                request_table=table.to(cuda_device), device_mapping=mapping.to(cuda_device), exclude_newest=True)
    dev_blocks = blocks.to(cuda_device)
    masked_fast = dev_blocks.clone()
    fast = sp.resolve_shared_block_locations_batched(dev_blocks, **args, masked_block_ids=masked_fast)
    tuple_rows = sp.resolve_shared_block_locations_batched(dev_blocks, **{**args, "source_rows": tuple(rows)})
    # The reference accepts only Python ints (shared_prefix.py:150-160): numpy ints and
    # bools are refused with its message, through the checked path.
    for bad in (np.array(rows), [True] * 12):
        with pytest.raises(ValueError, match="source row is outside"):
            sp.resolve_shared_block_locations_batched(dev_blocks, **{**args, "source_rows": bad})
    monkeypatch.setattr(sp, "torch_binding", lambda: None)
    masked_slow = dev_blocks.clone()
    slow = sp.resolve_shared_block_locations_batched(dev_blocks, **args, masked_block_ids=masked_slow)
    for a, b, c in zip(fast, slow, tuple_rows):
        assert torch.equal(a, b) and torch.equal(a, c)
    assert torch.equal(masked_fast, masked_slow)
