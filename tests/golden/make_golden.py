"""Generate the golden fixtures in this directory by running the REFERENCE code.

Run in a container where the reference checkout is importable:

    EKV_REFERENCE=/path/to/elastic-kv-vmm TRITON_INTERPRET=1 python tests/golden/make_golden.py [fixture ...]

(with fixture names -- ``migration``, ``plan_demote_large`` -- only those are rewritten).

The reference's Triton kernels (adaptive_sparse/resident_lookup.py,
experimental/sparse_read.py) run on CPU tensors under the Triton interpreter;
its Python helpers (VirtualKVLayout, PhysicalPages.chunks, _releasable*,
plan_demote_pages) run as they are.  Inputs are seeded; every fixture stores
inputs and the reference's outputs.  The captured TP4 plan state
results/vmm-pair12k-shadow/adaptive_stats/plans-rank0{0..3}.json is reduced to
the fields the freeable-bitmap test needs.  Nothing in the test suite reads
the reference at run time: only these files.
"""

from __future__ import annotations

import json
import os
import random
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("EKV_REFERENCE", ""))


def _import_reference():
    if not os.environ.get("EKV_REFERENCE"):
        raise SystemExit("set EKV_REFERENCE to the reference checkout")
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 so the reference Triton kernels run on CPU")
    sys.path.insert(0, str(REFERENCE))
    import torch  # noqa: F401

    from adaptive_sparse import logical_shadow, minimax_vmm, migration, scheduler_budget, shared_prefix
    from adaptive_sparse.resident_lookup import resolve_resident
    from experimental.sparse_read import gather_rows
    from experimental.virtual_layout import VirtualKVLayout

    return dict(resolve_resident=resolve_resident, gather_rows=gather_rows,
                VirtualKVLayout=VirtualKVLayout, PhysicalPages=minimax_vmm.PhysicalPages,
                scheduler_budget=scheduler_budget, migration=migration, shared_prefix=shared_prefix,
                logical_shadow=logical_shadow)


def lookup_cases(ref):
    import torch

    cases = {}

    def run(name, topk, table, mapping, rows, lengths, selected, width_out, block_size, init=-77):
        out = torch.full((1, topk.shape[1], width_out), init, dtype=torch.int32)
        ref["resolve_resident"](topk, table, mapping, rows, lengths, selected, out, block_size)
        cases[name] = dict(topk=topk.numpy(), table=table.numpy(), mapping=mapping.numpy(),
                           rows=rows.numpy(), lengths=lengths.numpy(), selected=selected.numpy(),
                           block_size=np.int64(block_size), init=np.int32(init), expected=out.numpy())

    # The vectors of tests/smoke_resident_lookup.py:8-13.
    run("smoke",
        torch.tensor([[[1, -1, 2] + [-1] * 13, [0] * 16, [0, 2, -1] + [-1] * 13]], dtype=torch.int32),
        torch.tensor([[i * 300 + j for j in range(300)] for i in range(4)], dtype=torch.int64),
        torch.tensor([i * 3 + 5 for i in range(1200)], dtype=torch.int64),
        torch.tensor([3, 0, 1], dtype=torch.int64), torch.tensor([130, 0, 0], dtype=torch.int32),
        torch.tensor([2, 0], dtype=torch.int64), 2048, 128)

    gen = torch.Generator().manual_seed(20261201)
    for name, (batch, k, bs, width, tdtype, mdtype) in {
        "random_bs4": (6, 7, 4, 40, torch.int32, torch.int64),
        "random_bs1": (9, 300, 1, 512, torch.int64, torch.int32),
        "random_bs16_big": (4, 40, 16, 1024, torch.int32, torch.int64),
    }.items():
        reqs = batch + 3
        table = torch.randint(0, 5000, (reqs, width), generator=gen).to(tdtype)
        mapping = (torch.randint(-(1 << 33), 1 << 33, (5000,), generator=gen)
                   if mdtype == torch.int64 else torch.randint(-9, 1 << 20, (5000,), generator=gen)).to(mdtype)
        n_blocks = width // bs
        topk = torch.randint(-1, n_blocks + 2, (1, batch, k), generator=gen).to(torch.int32)
        lengths = torch.randint(0, width + 1, (batch,), generator=gen).to(torch.int32)
        rows = torch.randint(0, reqs, (batch,), generator=gen).to(torch.int64)
        selected = torch.randperm(batch, generator=gen)[: max(1, batch - 2)].to(torch.int64)
        run(name, topk, table, mapping, rows, lengths, selected, k * bs, bs)
    return cases


def gather_cases(ref):
    import torch

    cases = {}
    gen = torch.Generator().manual_seed(97)
    for name, (reqs, tokens, width, chunk, batch, selected) in {
        "small_w24": (3, 37, 24, 512, 3, 10),
        "w1024": (2, 16, 1024, 1 << 15, 2, 19),
        "odd_w5": (2, 21, 5, 256, 2, 7),
    }.items():
        layout = ref["VirtualKVLayout"](reqs, tokens, width, chunk_bytes=chunk)
        n_elem = layout.capacity_bytes // layout.itemsize
        raw_bits = torch.randint(0, 1 << 16, (n_elem,), generator=gen, dtype=torch.int32).to(torch.int16)
        raw = raw_bits.view(torch.bfloat16)
        request_ids = torch.randperm(reqs, generator=gen)[:batch].to(torch.int64)
        lengths = torch.randint(1, tokens + 1, (batch,), generator=gen).to(torch.int64)
        positions = torch.randint(-2, tokens + 2, (batch, selected), generator=gen).to(torch.int64)
        count = reqs * tokens
        table = torch.randperm(count, generator=gen).reshape(reqs, tokens).to(torch.int64) + 1
        flat = torch.arange(count, dtype=torch.int64)
        addresses = (layout.chunk_bytes // layout.itemsize
                     + (flat // tokens) * (layout.request_bytes // layout.itemsize)
                     + (flat % tokens) * width)
        offsets = torch.zeros(count + 1, dtype=torch.int64)
        offsets[table.flatten()] = addresses
        record = dict(raw=raw_bits.numpy().view(np.uint16), positions=positions.numpy(),
                      request_ids=request_ids.numpy(), lengths=lengths.numpy(),
                      request_table=table.numpy(), slot_offsets=offsets.numpy(),
                      layout=np.array([reqs, tokens, width, layout.itemsize, chunk], dtype=np.int64))
        for indirect in (False, True):
            out = torch.full((batch, selected, width), 7.0, dtype=torch.bfloat16)
            ref["gather_rows"](raw, positions, request_ids, lengths, table, offsets, out, layout,
                               indirect=indirect)
            record["expected_indirect" if indirect else "expected_direct"] = (
                out.view(torch.int16).numpy().view(np.uint16))
        cases[name] = record
    return cases


def layout_cases(ref):
    out = []
    rng = random.Random(5)
    for _ in range(12):
        fields = dict(max_requests=rng.randint(1, 5), max_tokens=rng.randint(1, 40),
                      row_elements=rng.randint(1, 9), itemsize=rng.choice([1, 2, 4]),
                      chunk_bytes=rng.choice([8, 16, 64, 256]))
        layout = ref["VirtualKVLayout"](**fields)
        req = rng.randrange(fields["max_requests"])
        length = rng.randint(0, fields["max_tokens"])
        positions = [rng.randrange(fields["max_tokens"]) for _ in range(rng.randint(0, 5))]
        out.append(dict(fields=fields, row_bytes=layout.row_bytes, request_bytes=layout.request_bytes,
                        capacity_bytes=layout.capacity_bytes, req=req, length=length,
                        request_offset=layout.request_offset(req),
                        token_offsets=[layout.token_offset(req, p) for p in positions],
                        positions=positions,
                        prefix_chunks=sorted(layout.prefix_chunks(req, length)),
                        selected_chunks=sorted(layout.selected_chunks(req, positions))))
    return out


class _FakeBacking:
    def __init__(self):
        self.mapped_chunks = set()
        self.backed_bytes = 0

    def ensure(self, indices):
        self.mapped_chunks.update(indices)

    def reclaim(self, indices, *, synchronize):
        self.mapped_chunks.difference_update(indices)
        return len(indices)


def releasable_cases(ref):
    sb = ref["scheduler_budget"]
    rng = random.Random(137)
    cases = []
    for trial in range(40):
        chunk_bytes = rng.choice([64, 256, 1024])
        page_size = rng.choice([1, 2, 4])
        row_choices = [8, 24, 40, 96, 128]
        n_planes = rng.randint(1, 6)
        page_count = rng.randint(4, 40)
        planes = []
        offset = 0
        for _ in range(n_planes):
            row = rng.choice(row_choices)
            planes.append((offset // chunk_bytes, row))
            length = (page_count + 1) * page_size * row
            offset += -(-length // chunk_bytes) * chunk_bytes
        n_chunks = offset // chunk_bytes
        backing = _FakeBacking()
        tracker = ref["PhysicalPages"](backing, page_size, page_count, planes, lambda: None,
                                       chunk_bytes=chunk_bytes)
        owned = rng.sample(range(1, page_count + 1), rng.randint(1, page_count))
        tracker.acquire(owned)
        if trial % 3 == 0:
            # Some mapped chunks stop being mapped (partially reclaimed state).
            drop = rng.sample(sorted(backing.mapped_chunks), len(backing.mapped_chunks) // 5)
            backing.mapped_chunks.difference_update(drop)
        candidates = [sorted(rng.sample(owned, rng.randint(1, len(owned)))) for _ in range(3)]
        single = [sorted(sb._releasable(tracker, c)) for c in candidates]
        counts = [sb._chunk_release_counts(tracker, set(c)) for c in candidates]
        pair = sorted(sb._releasable_pair(tracker, set(candidates[0]), counts[0],
                                          set(candidates[1]), counts[1]))
        group = sorted(sb._releasable_group(tracker, [(set(c), k) for c, k in zip(candidates, counts)]))
        cases.append(dict(chunk_bytes=chunk_bytes, page_size=page_size, page_count=page_count,
                          planes=planes, n_chunks=n_chunks, owned=sorted(owned),
                          refs={str(k): v for k, v in tracker.refs.items()},
                          mapped=sorted(backing.mapped_chunks), candidates=candidates,
                          page_chunks={str(p): sorted(tracker.chunks(p)) for p in [0, *owned]},
                          releasable=single, pair=pair, group=group))
    return cases


def plans_fixture():
    states = []
    for rank in range(4):
        path = REFERENCE / f"results/vmm-pair12k-shadow/adaptive_stats/plans-rank{rank:02d}.json"
        states.append(json.loads(path.read_text())[0])
    first = states[0]
    identical = all(s == first for s in states[1:])
    reduced = {key: first[key] for key in ("chunk_bytes", "page_size", "planes", "refs",
                                           "mapped_chunks", "other_live_pages", "requests", "pairs")}
    reduced["all_ranks_identical"] = identical
    reduced["ranks"] = len(states)
    return reduced


def plan_demote_cases(ref):
    migration = ref["migration"]
    rng = random.Random(7)
    cases = []
    for trial in range(12):
        chunk_bytes = rng.choice([64, 256])
        page_size = rng.choice([1, 2])
        planes = [(0, 40), (8, 24)] if trial % 2 else [(0, 96)]
        backing = _FakeBacking()
        tracker = ref["PhysicalPages"](backing, page_size, 60, planes, lambda: None, chunk_bytes=chunk_bytes)
        pages = rng.sample(range(1, 61), rng.randint(2, 20))
        others = [p for p in range(1, 61) if p not in pages]
        tracker.acquire(pages + rng.sample(others, rng.randint(0, 10)))
        keep = rng.randint(1, len(pages))
        result = {}
        for aware in ("0", "1"):
            os.environ["EKV_CHUNK_AWARE_RETENTION"] = aware
            retained, released = migration.plan_demote_pages(tracker, pages, keep)
            result[aware] = [list(retained), list(released)]
        os.environ.pop("EKV_CHUNK_AWARE_RETENTION", None)
        cases.append(dict(chunk_bytes=chunk_bytes, page_size=page_size, planes=planes,
                          owned=sorted(tracker.pages - {0}), pages=pages, keep=keep,
                          plain=result["0"], aware=result["1"]))
    return cases


def shared_prefix_cases(ref):
    """resolve_shared_block_locations[_batched] (adaptive_sparse/shared_prefix.py:70-204).

    The vectors of tests/test_shared_prefix.py:146-228 plus seeded batches over
    block sizes 1..100, int32 / int64 tables, unmapped and negative slots,
    out-of-range and wrapping block ids, and slots above 2^31 (int32 wrap).
    """
    import torch

    sp = ref["shared_prefix"]
    cases = {}

    def batched(name, blocks, rows, lengths, prefixes, block_size, table, mapping):
        valid, physical = sp.resolve_shared_block_locations_batched(
            blocks, source_rows=rows, seq_len=lengths, shared_tokens=prefixes, block_size=block_size,
            request_table=table, device_mapping=mapping)
        cases[name] = dict(block_ids=blocks.numpy(), source_rows=np.asarray(rows, dtype=np.int64),
                           seq_len=lengths.numpy(), shared_tokens=np.asarray(prefixes, dtype=np.int64),
                           block_size=np.int64(block_size), request_table=table.numpy(),
                           device_mapping=mapping.numpy(), valid=valid.numpy(), physical=physical.numpy())

    # tests/test_shared_prefix.py:146-152 and :188-196.
    table2 = torch.tensor([[10, 11, 12, 13, 14, 15], [20, 21, 22, 23, 24, 25]])
    mapping30 = torch.arange(30, dtype=torch.long)
    mapping30[21] = 0
    for name, blocks, row in (("scalar_a", [0, 1, 2], 0), ("scalar_b", [0, 1], 1), ("scalar_c", [0, 99], 0)):
        valid, physical = sp.resolve_shared_block_locations(
            torch.tensor(blocks), source_row=row, seq_len=torch.tensor(6), shared_tokens=4, block_size=2,
            request_table=table2, device_mapping=mapping30)
        cases[name] = dict(block_ids=np.asarray(blocks, dtype=np.int64), source_row=np.int64(row),
                           seq_len=np.int64(6), shared_tokens=np.int64(4), block_size=np.int64(2),
                           request_table=table2.numpy(), device_mapping=mapping30.numpy(),
                           valid=valid.numpy(), physical=physical.numpy())
    table3 = torch.tensor([[10, 11, 12, 13, 14, 15], [20, 21, 22, 23, 24, 25], [30, 31, 32, 33, 34, 35]])
    mapping40 = torch.arange(40, dtype=torch.long)
    mapping40[21] = 0
    batched("batched_test", torch.tensor([[0, 1, 2], [1, 2, 3], [0, 1, 9]]), [0, 1, 2],
            torch.tensor([6, 4, 6]), [4, 4, 2], 2, table3, mapping40)

    gen = torch.Generator().manual_seed(2024)
    for i, block_size in enumerate((1, 2, 3, 8, 16, 32, 64, 100)):
        requests, per_request, table_rows, width = 7, 33, 5, 40 * block_size + 7
        slots = 4096
        dtype = torch.int32 if i % 2 else torch.int64
        table = torch.randint(-3, slots, (table_rows, width), generator=gen, dtype=torch.int64)
        table[table < 0] = -1
        table = table.to(dtype)
        mapping = torch.randint(1, 1 << 20, (slots,), generator=gen, dtype=torch.int64)
        # Unmapped (0) and negative slots, rarer for wide blocks so some of those stay valid.
        mapping[torch.rand(slots, generator=gen) < 0.1 / block_size] = 0
        mapping[torch.rand(slots, generator=gen) < 0.05 / block_size] = -5
        mapping[:8] = (1 << 32) + 77  # slots above 2^31: the int32 result wraps
        blocks = torch.randint(-2, 48, (requests, per_request), generator=gen, dtype=torch.int64)
        rows = torch.randint(0, table_rows, (requests,), generator=gen).tolist()
        lengths = torch.randint(1, width + 64, (requests,), generator=gen, dtype=torch.int64)
        prefixes = torch.randint(0, width + 64, (requests,), generator=gen).tolist()
        prefixes[0] = width + 1000
        batched(f"random_bs{block_size}", blocks.to(torch.int32 if i % 3 == 0 else torch.int64), rows,
                lengths, prefixes, block_size, table, mapping)
    # Block ids whose start wraps int64 (2^62 * 4 = 2^64 -> 0), as torch's int64 arithmetic does.
    huge = torch.tensor([[1 << 62, (1 << 62) + 1, -(1 << 62), 3]], dtype=torch.int64)
    batched("wrapping_blocks", huge, [0], torch.tensor([100]), [100], 4,
            torch.arange(64, dtype=torch.int64).reshape(2, 32) + 1, torch.arange(200, dtype=torch.int64))
    return cases


def _i16(tensor):
    return tensor.contiguous().view(torch_module().int16).numpy()


def torch_module():
    import torch

    return torch


def _seed_shadow_layer(shadow, layer, key, value, gen):
    """Create the layer with an empty write (the reference allocates it with
    new_empty) and give its never-written rows seeded contents, so the fixture
    does not depend on what the allocator returned."""
    import torch

    shadow.write(layer, torch.empty(0, dtype=torch.long), key[:0], value[:0], (None, None))
    k, v, _ = shadow.layers[layer]
    k.copy_(torch.randn(k.shape, generator=gen).to(k.dtype))
    v.copy_(torch.randn(v.shape, generator=gen).to(v.dtype))


def shadow_cases(ref):
    """LogicalShadow.check / check_complete (adaptive_sparse/logical_shadow.py:45-123).

    The reference class runs on CPU tensors: producer writes recorded with
    ``write``, a cache holding those rows with a few corrupted ones, Top-K block
    ids with clean prefixes, padding, malformed ids and blocks past the length,
    request-table entries below the page size and above the capacity, physical
    slots out of range or on dead pages.  Rows of 32 B, 24 B (not a multiple of
    16) and 2 KiB.
    """
    import torch

    LogicalShadow = ref["logical_shadow"].LogicalShadow
    cases = {}
    gen = torch.Generator().manual_seed(77)
    configs = [  # (name, heads, dim, block_size, page_size, use_physical, use_live)
        ("bs1_phys_live", 2, 8, 1, 4, True, True),
        ("bs4_logical", 1, 12, 4, 2, False, False),
        ("bs2_phys", 4, 64, 2, 8, True, False),
        ("bs1_logical_live", 1, 12, 1, 4, False, True),
    ]
    for name, heads, dim, block_size, page_size, use_physical, use_live in configs:
        capacity, slots, batch, k_blocks, table_rows, width = 160, 200, 5, 12, 6, 64
        shadow = LogicalShadow(capacity, "cpu")
        written = torch.randperm(capacity, generator=gen)[:120]
        key = torch.randn((120, heads, dim), generator=gen).to(torch.bfloat16)
        value = torch.randn((120, heads, dim), generator=gen).to(torch.bfloat16)
        _seed_shadow_layer(shadow, 3, key, value, gen)
        shadow.write(3, written, key, value, (None, 1.0))
        k_shadow, v_shadow, initialized = shadow.layers[3]
        # The cache mirrors the shadow through a permutation; a few rows are corrupted.
        # With explicit physical slots the cache holds logical slot l at phys_of[l];
        # without, physical == logical.
        perm = torch.randperm(slots, generator=gen)
        k_cache = torch.randn((slots, heads, dim), generator=gen).to(torch.bfloat16)
        v_cache = torch.randn((slots, heads, dim), generator=gen).to(torch.bfloat16)
        phys_of = perm[:capacity] if use_physical else torch.arange(capacity)
        k_cache[phys_of] = k_shadow
        v_cache[phys_of] = v_shadow
        for bad in torch.randperm(capacity, generator=gen)[:12].tolist():
            target = k_cache if bad % 2 else v_cache
            target[phys_of[bad], 0, bad % dim] = torch.tensor(123.5, dtype=torch.bfloat16)
        table = torch.randint(0, capacity + 20, (table_rows, width), generator=gen, dtype=torch.int32)
        lengths = torch.randint(1, width + 4, (batch,), generator=gen, dtype=torch.int64)
        rows = torch.randint(0, table_rows, (batch,), generator=gen, dtype=torch.int64)
        limit = (lengths + block_size - 1) // block_size
        blocks = torch.full((1, batch, k_blocks), -1, dtype=torch.int32)
        for b in range(batch):
            n_valid = int(torch.randint(0, k_blocks + 1, (1,), generator=gen))
            ids = torch.randint(0, int(limit[b]), (n_valid,), generator=gen)
            blocks[0, b, :n_valid] = ids.to(torch.int32)
            if b == 1 and n_valid < k_blocks - 2:   # valid id after padding: malformed
                blocks[0, b, n_valid + 1] = 0
            if b == 2:                              # id past the length: malformed, ends the prefix
                blocks[0, b, min(n_valid, k_blocks - 1)] = int(limit[b]) + 3
        physical = None
        if use_physical:
            positions = (blocks[0].long().clamp(min=0)[..., None] * block_size
                         + torch.arange(block_size)).flatten(1).clamp(max=width - 1)
            logical_guess = table[rows[:, None], positions]
            physical = phys_of[logical_guess.clamp(max=capacity - 1).long()].to(torch.int32)[None]
            physical[0, 0, :3] = torch.tensor([slots + 5, 1, -4], dtype=torch.int32)  # out of range
        live = None
        if use_live:
            live = torch.rand(slots // page_size + 1, generator=gen) < 0.85
        clean, phys_out = shadow.check(3, k_cache, v_cache, table, lengths, rows, block_size, blocks,
                                       physical, live, page_size)
        case = dict(k_shadow=_i16(k_shadow), v_shadow=_i16(v_shadow), initialized=initialized.numpy(),
                    k_cache=_i16(k_cache), v_cache=_i16(v_cache), table=table.numpy(), lengths=lengths.numpy(),
                    rows=rows.numpy(), block_size=np.int64(block_size), blocks=blocks.numpy(),
                    page_size=np.int64(page_size), counts=shadow.counts.numpy().copy(),
                    clean_blocks=clean.numpy(), physical_out=phys_out.numpy())
        if physical is not None:
            case["physical"] = physical.numpy()
        if live is not None:
            case["live_pages"] = live.numpy()
        cases["check_" + name] = case

    # check_complete over a 3-layer pool.
    for name, heads, dim, page_size in (("complete_small", 2, 8, 4), ("complete_odd", 1, 12, 2)):
        capacity, size, n_layers = 96, 128, 3
        shadow = LogicalShadow(capacity, "cpu")
        pool_k, pool_v = [], []
        logical = torch.randperm(capacity - page_size, generator=gen)[:60] + page_size
        physical = torch.randperm(size, generator=gen)[:60] + page_size
        for layer in range(n_layers):
            written = torch.randperm(capacity, generator=gen)[:80]
            key = torch.randn((80, heads, dim), generator=gen).to(torch.bfloat16)
            value = torch.randn((80, heads, dim), generator=gen).to(torch.bfloat16)
            _seed_shadow_layer(shadow, 10 + layer, key, value, gen)
            shadow.write(10 + layer, written, key, value, (None, None))
            k, v, _ = shadow.layers[10 + layer]
            pk = torch.randn((size + page_size, heads, dim), generator=gen).to(torch.bfloat16)
            pv = torch.randn((size + page_size, heads, dim), generator=gen).to(torch.bfloat16)
            pk[physical] = k[logical]
            pv[physical] = v[logical]
            for bad in range(layer, 60, 17):
                (pk if bad % 2 else pv)[physical[bad], 0, 0] = torch.tensor(-7.25, dtype=torch.bfloat16)
            pool_k.append(pk)
            pool_v.append(pv)
        logical[5] = 1            # below the page size
        logical[6] = capacity + 3  # past the capacity
        physical[7] = size + page_size + 1  # past the pool
        pages = sorted(set(range(1, size // page_size + 1)) - {int(physical[9]) // page_size})
        pool = SimpleNamespace(page_size=page_size, size=size, adaptive_vmm=SimpleNamespace(pages=set(pages)),
                               start_layer=10, end_layer=10 + n_layers,
                               get_key_buffer=lambda layer, pk=pool_k: pk[layer - 10],
                               get_value_buffer=lambda layer, pv=pool_v: pv[layer - 10])
        try:
            shadow.check_complete(pool, logical, physical, "test")
            raised = False
        except RuntimeError:
            raised = True
        case = dict(logical=logical.numpy(), physical=physical.numpy(), page_size=np.int64(page_size),
                    size=np.int64(size), capacity=np.int64(capacity), pages=np.asarray(pages, dtype=np.int64),
                    raised=np.bool_(raised),
                    counts=np.asarray(list(shadow.migration_counts.values()), dtype=np.int64))
        for layer in range(n_layers):
            k, v, initialized = shadow.layers[10 + layer]
            case[f"k_shadow{layer}"] = _i16(k)
            case[f"v_shadow{layer}"] = _i16(v)
            case[f"initialized{layer}"] = initialized.numpy()
            case[f"pool_k{layer}"] = _i16(pool_k[layer])
            case[f"pool_v{layer}"] = _i16(pool_v[layer])
        cases[name] = case
    return cases


def plan_demote_large_cases(ref):
    """The chunk-aware retention planner on larger, denser ownership patterns than
    ``plan_demote_cases``: many pages per chunk, several owners per chunk, long keeps."""
    migration = ref["migration"]
    rng = random.Random(2027)
    cases = []
    for trial in range(60):
        chunk_bytes = rng.choice([128, 256, 512])
        page_size = rng.choice([1, 2, 4])
        row_sizes = rng.choice([[32], [32, 16], [48, 24, 24]])
        first, planes = 0, []
        page_count = 120
        for plane in range(rng.randint(1, 4)):
            row = row_sizes[plane % len(row_sizes)]
            planes.append((first, row))
            first += -(-((page_count + 1) * page_size * row) // chunk_bytes)
        tracker = ref["PhysicalPages"](_FakeBacking(), page_size, page_count, planes, lambda: None,
                                       chunk_bytes=chunk_bytes)
        pages = rng.sample(range(1, page_count + 1), rng.randint(5, 60))
        others = [q for q in range(1, page_count + 1) if q not in pages]
        tracker.acquire(pages + rng.sample(others, rng.randint(0, 40)))
        keep = rng.randint(1, len(pages))
        os.environ["EKV_CHUNK_AWARE_RETENTION"] = "1"
        retained, released = migration.plan_demote_pages(tracker, pages, keep)
        os.environ.pop("EKV_CHUNK_AWARE_RETENTION", None)
        cases.append(dict(chunk_bytes=chunk_bytes, page_size=page_size, page_count=page_count,
                          planes=planes, owned=sorted(tracker.pages - {0}), pages=pages, keep=keep,
                          aware=[list(retained), list(released)]))
    return cases


def migration_trace(ref):
    """The reference's demote / promote transactions (adaptive_sparse/migration.py:67-288)
    and its PhysicalPages, run over the CPU stand-in world of tests/support/standin.py:
    every scenario of tests/support/migration_scenarios.py, recorded as a state trace."""
    sys.path.insert(0, str(HERE.parents[1]))
    from tests.support import migration_scenarios, standin

    def make_world(**geometry):
        return standin.migration_world("cpu", tracker_cls=ref["PhysicalPages"],
                                       host_pool_cls=standin.CpuHostPool, **geometry)

    return migration_scenarios.run_all(make_world, ref["migration"])


def main():
    ref = _import_reference()
    only = sys.argv[1:]
    if only:  # e.g. `make_golden.py migration plan_demote_large`: rewrite just those fixtures
        if "migration" in only:
            (HERE / "migration_trace.json").write_text(json.dumps(migration_trace(ref), sort_keys=True))
        if "plan_demote_large" in only:
            (HERE / "plan_demote_large.json").write_text(json.dumps(plan_demote_large_cases(ref), sort_keys=True))
        print("golden fixtures written to", HERE, only)
        return
    np.savez_compressed(HERE / "lookup_golden.npz",
                        **{f"{case}__{key}": value for case, arrays in lookup_cases(ref).items()
                           for key, value in arrays.items()})
    np.savez_compressed(HERE / "gather_golden.npz",
                        **{f"{case}__{key}": value for case, arrays in gather_cases(ref).items()
                           for key, value in arrays.items()})
    np.savez_compressed(HERE / "shared_prefix_golden.npz",
                        **{f"{case}__{key}": value for case, arrays in shared_prefix_cases(ref).items()
                           for key, value in arrays.items()})
    np.savez_compressed(HERE / "shadow_golden.npz",
                        **{f"{case}__{key}": value for case, arrays in shadow_cases(ref).items()
                           for key, value in arrays.items()})
    (HERE / "host_golden.json").write_text(json.dumps(
        dict(layouts=layout_cases(ref), releasable=releasable_cases(ref),
             plan_demote=plan_demote_cases(ref)), sort_keys=True))
    (HERE / "plans_pair12k.json").write_text(json.dumps(plans_fixture(), sort_keys=True))
    (HERE / "plan_demote_large.json").write_text(json.dumps(plan_demote_large_cases(ref), sort_keys=True))
    (HERE / "migration_trace.json").write_text(json.dumps(migration_trace(ref), sort_keys=True))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
