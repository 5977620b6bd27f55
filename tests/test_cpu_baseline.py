"""The timed CPU baseline computes what the oracle computes.

bench.py times ``oracle/cpu_baseline.py`` on the host cores (the ``cpu_baseline``
leg and the ``--impl reference`` arm).  These checks pin each of its torch
restatements to the numpy oracle or to the reference's golden vectors, so the
baseline is the same work as the GPU path, not a cheaper approximation.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_npz_cases
from oracle import cpu_baseline as cb
from oracle import gather as og
from oracle import logical_shadow as osh
from oracle import shared_prefix as osp


def test_gather_planes_matches_the_oracle():
    gen = torch.Generator().manual_seed(51)
    slots, width, batch, selected, tokens, n_planes = 700, 24, 4, 90, 120, 3
    planes = [torch.randint(-30000, 30000, (slots, width), generator=gen, dtype=torch.int16) for _ in range(n_planes)]
    positions = torch.randint(-3, tokens + 3, (batch, selected), generator=gen)
    request_ids = torch.tensor([2, 0, 3, 1])
    lengths = torch.tensor([tokens, 60, 0, 7])
    table = torch.randperm(batch * tokens, generator=gen).view(batch, tokens)
    offsets = torch.randperm(slots, generator=gen)[:batch * tokens] * width
    outputs = [torch.full((batch, selected, width), 5, dtype=torch.int16) for _ in planes]
    cb.gather_planes(planes, positions, request_ids, lengths, table, offsets, width, outputs)
    want = og.gather_rows_planes([p.reshape(-1).numpy() for p in planes], positions.numpy(), request_ids.numpy(),
                                 lengths.numpy(), table.numpy(), offsets.numpy(), width=width, table_width=tokens,
                                 request_stride=0, sink_elements=0, indirect=True)
    for out, exp in zip(outputs, want):
        np.testing.assert_array_equal(out.numpy(), exp)


@pytest.mark.parametrize("case", sorted(load_npz_cases("lookup_golden.npz")))
def test_torch_resolver_matches_the_reference_vectors(case):
    c = {k: v for k, v in load_npz_cases("lookup_golden.npz")[case].items()}
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in c.items() if np.ndim(v)}
    result = torch.full(c["expected"].shape, int(c["init"]), dtype=torch.int32)
    cb.torch_resolver(t["topk"], t["table"], t["mapping"], t["rows"], t["lengths"], t["selected"], result,
                      int(c["block_size"]))
    np.testing.assert_array_equal(result.numpy(), c["expected"])


SHARED = load_npz_cases("shared_prefix_golden.npz")


@pytest.mark.parametrize("case", sorted(c for c in SHARED if "source_row" not in SHARED[c]))
def test_torch_shared_resolver_matches_the_reference_vectors(case):
    c = SHARED[case]
    valid, physical = cb.torch_shared_resolver(
        torch.from_numpy(c["block_ids"]), torch.as_tensor(c["source_rows"], dtype=torch.int64),
        torch.as_tensor(c["shared_tokens"], dtype=torch.int64), torch.from_numpy(c["seq_len"]),
        int(c["block_size"]), torch.from_numpy(c["request_table"]), torch.from_numpy(c["device_mapping"]))
    np.testing.assert_array_equal(valid.numpy(), c["valid"])
    # Slots of invalid blocks are unspecified; the valid ones are the resolved slots.
    np.testing.assert_array_equal(physical.numpy()[c["valid"]], c["physical"][c["valid"]])
    want_valid, _ = osp.resolve_batched(c["block_ids"], c["source_rows"], c["seq_len"], c["shared_tokens"],
                                        int(c["block_size"]), c["request_table"], c["device_mapping"])
    np.testing.assert_array_equal(valid.numpy(), want_valid)


SHADOW = load_npz_cases("shadow_golden.npz")


@pytest.mark.parametrize("case", sorted(c for c in SHADOW if c.startswith("check_")))
def test_torch_shadow_check_matches_the_reference_vectors(case):
    c = SHADOW[case]
    t = lambda name: None if name not in c else torch.from_numpy(np.ascontiguousarray(c[name]))  # noqa: E731
    live = t("live_pages")
    counts, clean, physical = cb.torch_shadow_check(
        t("k_shadow"), t("v_shadow"), t("initialized").bool(), t("k_cache"), t("v_cache"), t("table"),
        t("lengths"), t("rows"), int(c["block_size"]), t("blocks"), t("physical"),
        None if live is None else live.bool(), int(c["page_size"]))
    np.testing.assert_array_equal(counts.numpy(), c["counts"])
    np.testing.assert_array_equal(clean.numpy(), c["clean_blocks"])
    np.testing.assert_array_equal(physical.numpy(), c["physical_out"])
    want = osh.check(c["k_shadow"], c["v_shadow"], c["initialized"], c["k_cache"], c["v_cache"], c["table"],
                     c["lengths"], c["rows"], int(c["block_size"]), c["blocks"], c.get("physical"),
                     c.get("live_pages"), int(c["page_size"]))
    np.testing.assert_array_equal(counts.numpy(), want[0])
