"""Pin the CPU oracle to the reference: golden vectors and the reference tests' known answers."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_json, load_npz_cases
from oracle import gather as og
from oracle import lookup as ol
from oracle import migration as om
from oracle import releasable as orl


def _strided(values):
    """A stride-2 view holding ``values`` (tests/smoke_resident_lookup.py:28-33)."""
    backing = np.zeros((*values.shape, 2), dtype=values.dtype)
    view = backing[..., 1]
    view[...] = values
    return view


@pytest.mark.parametrize("case", sorted(load_npz_cases("lookup_golden.npz")))
@pytest.mark.parametrize("strided", [False, True])
def test_resolve_oracle_matches_reference_kernel(case, strided):
    c = load_npz_cases("lookup_golden.npz")[case]
    prep = _strided if strided else (lambda a: a)
    out = np.full(c["expected"].shape, int(c["init"]), dtype=np.int32)
    ol.resolve_resident(prep(c["topk"]), prep(c["table"]), prep(c["mapping"]), prep(c["rows"]),
                        prep(c["lengths"]), prep(c["selected"]), out, int(c["block_size"]))
    np.testing.assert_array_equal(out, c["expected"])


def test_smoke_known_answers():
    """tests/smoke_resident_lookup.py:21-23."""
    expected = load_npz_cases("lookup_golden.npz")["smoke"]["expected"][0]
    assert expected[0, :3].tolist() == [3089, 3092, -1]
    assert expected[0, -1] == -1 and (expected[2] == -1).all()
    assert (expected[1] == -77).all()


@pytest.mark.parametrize("case", sorted(load_npz_cases("lookup_golden.npz")))
def test_torch_resolver_restatement_agrees(case):
    c = load_npz_cases("lookup_golden.npz")[case]
    sel = c["selected"]
    got = ol.torch_resolver_numpy(c["topk"], c["table"], c["mapping"], c["rows"], c["lengths"], sel,
                                  int(c["block_size"]))
    np.testing.assert_array_equal(got, c["expected"][0, sel])


@pytest.mark.parametrize("batch", [1, 2, 4])
def test_resolve_closed_form(batch):
    """tests/bench_resident_lookup.py:38-42, 83-87."""
    selected = np.arange(batch)
    rows = selected[::-1].copy()
    lengths = np.full(batch, 8192, dtype=np.int32)
    table = np.arange(batch * 8192).reshape(batch, 8192) + 1
    mapping = np.arange(batch * 8192 + 1) * 3 + 5
    topk = np.broadcast_to((np.arange(16) * 4).astype(np.int32), (1, batch, 16)).copy()
    out = np.empty((1, batch, 2048), dtype=np.int32)
    ol.resolve_resident(topk, table, mapping, rows, lengths, selected, out, 128)
    expected = np.array([[((batch - 1 - row) * 8192 + block * 512 + offset + 1) * 3 + 5
                          for block in range(16) for offset in range(128)] for row in range(batch)])
    np.testing.assert_array_equal(out[0], expected)


def test_lookup_slots_oracle_small():
    res_map = np.array([[-1, 5, 7, -1, 2], [0, -1, -1, 3, 1]], dtype=np.int32)
    topk = np.array([[0, 1, 3, 4, -1, 9], [4, 3, 2, 1, 0, 1]], dtype=np.int32)
    lengths = np.array([5, 3])
    slots, miss, miss_list, count = ol.lookup_slots(res_map, topk, lengths)
    assert slots.tolist() == [[-1, 5, -1, 2, -1, -1], [-1, -1, -1, -1, 0, -1]]
    assert miss.tolist() == [[True, False, True, False, False, False],
                             [False, False, True, True, False, True]]
    assert miss_list.tolist() == [[0, 3, -1, -1, -1, -1], [2, 1, 1, -1, -1, -1]]
    assert count.tolist() == [2, 3]


@pytest.mark.parametrize("case", sorted(load_npz_cases("gather_golden.npz")))
@pytest.mark.parametrize("indirect", [False, True])
def test_gather_oracle_matches_reference_kernel(case, indirect):
    c = load_npz_cases("gather_golden.npz")[case]
    reqs, tokens, width, itemsize, chunk = (int(v) for v in c["layout"])
    request_bytes = -(-(tokens * width * itemsize) // chunk) * chunk
    out = og.gather_rows(c["raw"], c["positions"], c["request_ids"], c["lengths"], c["request_table"],
                         c["slot_offsets"], width=width, table_width=tokens,
                         request_stride=request_bytes // itemsize, sink_elements=chunk // itemsize,
                         indirect=indirect)
    np.testing.assert_array_equal(out, c["expected_indirect" if indirect else "expected_direct"])


def test_gather_payload_pattern_known_answer():
    """scripts/bench_virtual_addressing.py:47-48, 69-88: payload (pos*width+col+req*17) % 97,
    reversed logical ids, invalid lanes (-1 and length) read as a zero row."""
    batch, length, width, chunk = 3, 40, 8, 256
    itemsize = 2
    request_bytes = -(-(length * width * itemsize) // chunk) * chunk
    raw = np.zeros((chunk + batch * request_bytes) // itemsize, dtype=np.float32)
    for req in range(batch):
        start = (chunk + req * request_bytes) // itemsize
        values = (np.arange(length * width) + req * 17) % 97
        raw[start:start + length * width] = values
    request_ids = np.arange(batch)[::-1].copy()
    lengths = np.full(batch, length)
    count = batch * length
    table = np.arange(count, 0, -1).reshape(batch, length)
    flat = np.arange(count)
    addresses = chunk // itemsize + (flat // length) * (request_bytes // itemsize) + (flat % length) * width
    offsets = np.zeros(count + 1, dtype=np.int64)
    offsets[table.flatten()] = addresses
    positions = np.tile(np.arange(0, length, 3), (batch, 1))
    positions[:, 0] = -1
    positions[:, 1] = length
    expected = ((positions.clip(min=0)[..., None] * width + np.arange(width)
                 + request_ids[:, None, None] * 17) % 97).astype(np.float32)
    expected[:, :2, :] = 0
    for indirect in (False, True):
        got = og.gather_rows(raw, positions, request_ids, lengths, table, offsets, width=width,
                             table_width=length, request_stride=request_bytes // itemsize,
                             sink_elements=chunk // itemsize, indirect=indirect)
        np.testing.assert_array_equal(got, expected)


def _chunks_fn(case):
    return lambda page: orl.page_chunks(page, case["planes"], case["page_size"], case["chunk_bytes"])


@pytest.mark.parametrize("index", range(40))
def test_releasable_oracle_matches_reference(index):
    case = load_json("host_golden.json")["releasable"][index]
    chunks_of = _chunks_fn(case)
    refs = {int(k): v for k, v in case["refs"].items()}
    mapped = set(case["mapped"])
    for page, chunks in case["page_chunks"].items():
        assert sorted(chunks_of(int(page))) == chunks
    for pages, expected in zip(case["candidates"], case["releasable"]):
        assert sorted(orl.releasable(chunks_of, refs, mapped, pages)) == expected
    c = case["candidates"]
    assert sorted(orl.releasable_group(chunks_of, refs, mapped, [c[0], c[1]])) == case["pair"]
    assert sorted(orl.releasable_group(chunks_of, refs, mapped, c)) == case["group"]
    # Vectorised restatement (what the kernels compute) agrees with the set form.
    n = case["n_chunks"]
    refs_arr = np.zeros(n, dtype=np.int32)
    for k, v in refs.items():
        refs_arr[k] = v
    mapped_bits = orl.bits_of(mapped, n)
    for pages, expected in zip(c, case["releasable"]):
        counts = orl.chunk_counts_np(sorted(set(pages)), case["planes"], case["page_size"],
                                     case["chunk_bytes"], n)
        bits = orl.freeable_bitmap_np(counts, refs_arr, mapped_bits)
        assert sorted(orl.chunks_of_bits(bits)) == expected


SHARED_CHUNK = dict(planes=[(9, 16)], page_size=4, chunk_bytes=256, n_chunks=64)  # pages 0-3 all in chunk 9


@pytest.mark.parametrize("owners", [2, 3])
def test_shared_chunk_is_freeable_only_with_every_owner(owners):
    """Known answers of tests/test_scheduler_budget.py:414-426 (a chunk with three owning
    candidates: no two of them free it, all three do) and :769-775 (two owners: neither
    alone, the pair does), through the set form and the bitmap form the kernels restate."""
    import itertools

    g = SHARED_CHUNK
    chunks_of = lambda page: orl.page_chunks(page, g["planes"], g["page_size"], g["chunk_bytes"])  # noqa: E731
    pages = list(range(1, owners + 1))
    assert all(chunks_of(p) == {9} for p in pages)
    refs, mapped = {9: owners}, {9}
    refs_arr = np.zeros(g["n_chunks"], dtype=np.int32)
    refs_arr[9] = owners
    mapped_bits = orl.bits_of(mapped, g["n_chunks"])
    for size in range(1, owners + 1):
        for subset in itertools.combinations(pages, size):
            want = {9} if size == owners else set()
            assert orl.releasable(chunks_of, refs, mapped, subset) == want
            assert orl.releasable_group(chunks_of, refs, mapped, [[p] for p in subset]) == want
            counts = orl.chunk_counts_np(sorted(subset), g["planes"], g["page_size"], g["chunk_bytes"],
                                         g["n_chunks"])
            assert orl.chunks_of_bits(orl.freeable_bitmap_np(counts, refs_arr, mapped_bits)) == want
    assert orl.releasable(chunks_of, refs, set(), pages) == set()  # an unmapped chunk is never freeable


def test_plans_fixture_pair_frees_120_chunks_on_every_rank():
    """README.md:30 / results/vmm-pair12k-shadow: neither request alone frees a
    chunk; the pair frees 120 chunks (240 MiB) on each of the 4 TP ranks."""
    plan = load_json("plans_pair12k.json")
    assert plan["all_ranks_identical"] and plan["ranks"] == 4
    chunks_of = lambda page: orl.page_chunks(page, plan["planes"], plan["page_size"], plan["chunk_bytes"])
    refs = {int(k): v for k, v in plan["refs"].items()}
    mapped = set(plan["mapped_chunks"])
    owned = set(plan["other_live_pages"])
    for request in plan["requests"].values():
        owned.update(request["page_ids"])
        assert sorted(orl.releasable(chunks_of, refs, mapped, request["released"])) == \
            request["predicted_chunks"] == []
    # refs are exactly the page -> chunk histogram of every owned page.
    assert orl.chunk_release_counts(chunks_of, owned) == refs
    pair = plan["pairs"][0]
    union = [p for row in pair["rows"] for p in plan["requests"][str(row)]["released"]]
    per_rank = [orl.releasable(chunks_of, refs, mapped, union) for _ in range(plan["ranks"])]
    joint = orl.joint_releasable(per_rank)
    assert sorted(joint) == pair["predicted_chunks"] and len(joint) == 120
    assert len(joint) * plan["chunk_bytes"] == 240 << 20
    n = max(mapped) + 1
    gathered = [orl.bits_of(r, n) for r in per_rank]
    assert orl.chunks_of_bits(orl.bitmap_and_np(gathered)) == joint


def test_migration_oracle_round_trip():
    rng = np.random.default_rng(3)
    planes = [rng.integers(0, 255, (64, 48), dtype=np.uint8) for _ in range(3)]
    slots = rng.permutation(64)[:20]
    staging = np.zeros((3 * 32, 48), dtype=np.uint8)
    om.pack_rows(planes, slots, staging, stage_plane_rows=32)
    fresh = [np.zeros_like(p) for p in planes]
    dest = rng.permutation(64)[:20]
    om.unpack_rows(fresh, dest, staging, stage_plane_rows=32)
    for p in range(3):
        np.testing.assert_array_equal(fresh[p][dest], planes[p][slots])
    # list form
    plane_index = rng.integers(0, 3, 20)
    staging2 = np.zeros((20, 48), dtype=np.uint8)
    om.pack_rows(planes, slots, staging2, plane_index=plane_index)
    for t in range(20):
        np.testing.assert_array_equal(staging2[t], planes[plane_index[t]][slots[t]])


# --------------------------------------------------------------------------- shared prefix

from oracle import shared_prefix as osp  # noqa: E402

SHARED_CASES = load_npz_cases("shared_prefix_golden.npz")


@pytest.mark.parametrize("case", sorted(SHARED_CASES))
def test_shared_prefix_oracle_matches_reference(case):
    c = SHARED_CASES[case]
    if "source_row" in c:
        valid, physical = osp.resolve_scalar(c["block_ids"], int(c["source_row"]), int(c["seq_len"]),
                                             int(c["shared_tokens"]), int(c["block_size"]),
                                             c["request_table"], c["device_mapping"])
    else:
        valid, physical = osp.resolve_batched(c["block_ids"], c["source_rows"], c["seq_len"],
                                              c["shared_tokens"], int(c["block_size"]), c["request_table"],
                                              c["device_mapping"])
    np.testing.assert_array_equal(valid, c["valid"])
    np.testing.assert_array_equal(physical, c["physical"])


def test_shared_prefix_known_answers():
    """tests/test_shared_prefix.py:138-186 of the reference, as literal answers."""
    assert osp.complete_shared_blocks([0, 1, 2, -1], 300, 256, 128) == (True, True, False, False)
    a = SHARED_CASES["scalar_a"]
    assert a["valid"].tolist() == [True, True, False]
    assert a["physical"][a["valid"]].tolist() == [[10, 11], [12, 13]]
    assert SHARED_CASES["scalar_b"]["valid"].tolist() == [False, True]
    assert SHARED_CASES["scalar_c"]["valid"].tolist() == [True, False]
    # The batched case equals the stacked scalar resolutions (test_shared_prefix.py:188-228).
    b = SHARED_CASES["batched_test"]
    for r in range(3):
        valid, physical = osp.resolve_scalar(b["block_ids"][r], int(b["source_rows"][r]), int(b["seq_len"][r]),
                                             int(b["shared_tokens"][r]), 2, b["request_table"],
                                             b["device_mapping"])
        np.testing.assert_array_equal(valid, b["valid"][r])
        np.testing.assert_array_equal(physical, b["physical"][r])


def test_shared_prefix_fixture_covers_the_edges():
    """The seeded cases reach every branch: partial blocks, unmapped slots, int32 wrap."""
    wrapped = SHARED_CASES["wrapping_blocks"]
    # (2^62 + k) * 4 wraps to 4k: blocks 2^62 and 2^62 + 1 read positions 0-3 and 4-7.
    assert wrapped["valid"].tolist() == [[True, True, False, True]]
    assert wrapped["physical"][0, 1].tolist() == [5, 6, 7, 8]
    total_valid = sum(int(SHARED_CASES[c]["valid"].sum()) for c in SHARED_CASES if c.startswith("random"))
    total_invalid = sum(int((~SHARED_CASES[c]["valid"]).sum()) for c in SHARED_CASES if c.startswith("random"))
    assert total_valid > 100 and total_invalid > 100
    assert any((SHARED_CASES[c]["physical"] == 77).any() for c in SHARED_CASES if c.startswith("random"))


# --------------------------------------------------------------------------- logical shadow

from oracle import logical_shadow as osh  # noqa: E402

SHADOW_CASES = load_npz_cases("shadow_golden.npz")


@pytest.mark.parametrize("case", sorted(c for c in SHADOW_CASES if c.startswith("check_")))
def test_shadow_check_oracle_matches_reference(case):
    c = SHADOW_CASES[case]
    counts, clean, physical = osh.check(c["k_shadow"], c["v_shadow"], c["initialized"], c["k_cache"], c["v_cache"],
                                        c["table"], c["lengths"], c["rows"], int(c["block_size"]), c["blocks"],
                                        c.get("physical"), c.get("live_pages"), int(c["page_size"]))
    np.testing.assert_array_equal(counts, c["counts"])
    np.testing.assert_array_equal(clean, c["clean_blocks"])
    assert clean.dtype == c["clean_blocks"].dtype
    np.testing.assert_array_equal(physical, c["physical_out"])


@pytest.mark.parametrize("case", sorted(c for c in SHADOW_CASES if c.startswith("complete_")))
def test_shadow_check_complete_oracle_matches_reference(case):
    c = SHADOW_CASES[case]
    n_layers = sum(1 for k in c if k.startswith("pool_k"))
    page, size = int(c["page_size"]), int(c["size"])
    live = np.zeros(size // page + 1, dtype=bool)
    live[c["pages"]] = True
    counts = osh.check_complete([(c[f"k_shadow{i}"], c[f"v_shadow{i}"], c[f"initialized{i}"]) for i in range(n_layers)],
                                [c[f"pool_k{i}"] for i in range(n_layers)], [c[f"pool_v{i}"] for i in range(n_layers)],
                                c["logical"], c["physical"], page, size, live, int(c["capacity"]))
    np.testing.assert_array_equal(counts, c["counts"])
    assert bool(c["raised"]) == bool(counts[2] or counts[3])


# --------------------------------------------------------------------------- swap-in (this build's policy)

from oracle import swap as osw  # noqa: E402


def _inverse(res_map, slot_token):
    for b in range(res_map.shape[0]):
        tokens = np.nonzero(res_map[b] >= 0)[0]
        assert (slot_token[b, res_map[b, tokens]] == tokens).all()
        slots = np.nonzero(slot_token[b] >= 0)[0]
        assert (res_map[b, slot_token[b, slots]] == slots).all()


def test_swap_oracle_invariants_over_decode_steps():
    """The clock victim policy the swap kernels implement, over 8 decode steps: the map
    and the slot table stay inverse, hits keep their slots, victims come in ring order
    from the hand, and after promotion every Top-K row reads its history row."""
    rng = np.random.default_rng(61)
    batch, context, hot, k, width = 3, 400, 48, 32, 4
    res_map = np.full((batch, context), -1, dtype=np.int32)
    slot_token = np.full((batch, hot), -1, dtype=np.int32)
    hand = np.zeros(batch, dtype=np.int32)
    history = rng.integers(-30000, 30000, (batch * context, width)).astype(np.int16)
    hot_rows = np.zeros((batch, hot, width), dtype=np.int16)
    lengths = np.full(batch, context)
    topk = np.stack([rng.choice(context, k, replace=False) for _ in range(batch)]).astype(np.int32)
    for _ in range(8):
        slots, miss, miss_list, miss_count = ol.lookup_slots(res_map, topk)
        before_hand = hand.copy()
        hits = {(b, int(t)): int(s) for b in range(batch) for t, s in zip(topk[b], slots[b]) if s >= 0}
        promo = osw.swap_select(res_map, slot_token, hand, slots, miss_list, miss_count)
        _inverse(res_map, slot_token)
        for (b, t), s in hits.items():
            assert res_map[b, t] == s  # a hit is never evicted in its own step
        for b in range(batch):
            n = int(miss_count[b])
            got = promo[b, :n]
            assert (got >= 0).all() and len(set(got.tolist())) == n
            ring = (before_hand[b] + np.arange(hot)) % hot
            free = [s for s in ring if s not in set(slots[b][slots[b] >= 0].tolist())]
            assert got.tolist() == free[:n]  # ring order from the hand, referenced slots skipped
        osw.promote_rows(history, hot_rows, miss_list, miss_count, promo, context)
        out = osw.mapped_gather(hot_rows, res_map, topk, lengths)
        rows = np.arange(batch)[:, None] * context + topk
        np.testing.assert_array_equal(out, history[rows])
        keep = topk[:, : k * 3 // 4]  # 75 % of the ids stay, the rest are new
        fresh = [rng.choice(np.setdiff1d(np.arange(context), keep[b]), k - keep.shape[1], replace=False)
                 for b in range(batch)]
        topk = np.concatenate([keep, np.stack(fresh)], axis=1).astype(np.int32)


def test_swap_oracle_assigns_only_free_slots():
    """More misses than unreferenced slots: the free slots are assigned in ring order,
    the rest of promo_slot stays -1 and the hand does not move."""
    res_map = np.full((1, 20), -1, dtype=np.int32)
    slot_token = np.full((1, 4), -1, dtype=np.int32)
    res_map[0, [3, 5]] = [0, 2]
    slot_token[0, [0, 2]] = [3, 5]
    hand = np.array([1], dtype=np.int32)
    topk = np.array([[3, 5, 7, 8, 9]], dtype=np.int32)
    slots, _, miss_list, miss_count = ol.lookup_slots(res_map, topk)
    assert miss_count.tolist() == [3]
    promo = osw.swap_select(res_map, slot_token, hand, slots, miss_list, miss_count)
    assert promo[0].tolist() == [1, 3, -1, -1, -1]
    assert hand.tolist() == [1]
    assert res_map[0, [3, 5, 7, 8, 9]].tolist() == [0, 2, 1, 3, -1]
    _inverse(res_map, slot_token)
