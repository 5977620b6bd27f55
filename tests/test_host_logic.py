"""Host-side logic of the package, on CPU: layout, arena, page tracker, demotion
planning, bitmap helpers, Backing error handling and the migration state machine."""

from __future__ import annotations

import ctypes as ct
import os
from types import SimpleNamespace
from unittest.mock import Mock, call

import pytest
import torch

from conftest import load_json
from ekv_b200 import migration
from ekv_b200.backing import Backing
from ekv_b200.physical_pages import PhysicalPages
from ekv_b200.releasable import bitmap_to_chunks, chunks_to_bitmap
from ekv_b200.resident_arena import VmmResidentArena
from ekv_b200.virtual_layout import VirtualKVLayout


# ---------------------------------------------------------------- layout / arena

@pytest.mark.parametrize("index", range(12))
def test_layout_matches_reference(index):
    case = load_json("host_golden.json")["layouts"][index]
    layout = VirtualKVLayout(**case["fields"])
    assert layout.row_bytes == case["row_bytes"]
    assert layout.request_bytes == case["request_bytes"]
    assert layout.capacity_bytes == case["capacity_bytes"]
    assert layout.request_offset(case["req"]) == case["request_offset"]
    assert [layout.token_offset(case["req"], p) for p in case["positions"]] == case["token_offsets"]
    assert sorted(layout.prefix_chunks(case["req"], case["length"])) == case["prefix_chunks"]
    assert sorted(layout.selected_chunks(case["req"], case["positions"])) == case["selected_chunks"]


def test_layout_alignment_and_validation():
    """Known answers of tests/test_virtual_layout.py:10-37."""
    layout = VirtualKVLayout(2, 3, 3, chunk_bytes=8)
    assert layout.capacity_bytes == 56 and layout.request_offset(1) == 32
    assert layout.token_offset(0, 1) == 14
    assert layout.prefix_chunks(0, 0) == set() and layout.selected_chunks(0, []) == set()
    assert layout.selected_chunks(0, [1, 1]) == {1, 2}
    assert layout.prefix_chunks(0, 3) == {1, 2, 3} and layout.prefix_chunks(1, 3) == {4, 5, 6}
    fields = dict(max_requests=2, max_tokens=3, row_elements=3, itemsize=2, chunk_bytes=8)
    for field in fields:
        with pytest.raises(ValueError):
            VirtualKVLayout(**(fields | {field: 0}))
        with pytest.raises(TypeError):
            VirtualKVLayout(**(fields | {field: True}))
    layout = VirtualKVLayout(**fields)
    for bad in (-1, 2):
        with pytest.raises(ValueError):
            layout.selected_chunks(bad, [])
    for bad in (-1, 3):
        with pytest.raises(ValueError):
            layout.selected_chunks(0, [bad])
    for bad in (-1, 4):
        with pytest.raises(ValueError):
            layout.prefix_chunks(0, bad)


def test_arena_call_sequence():
    """Same backing call sequence as tests/test_virtual_layout.py:49-65."""
    calls = Mock()
    layout = VirtualKVLayout(2, 5, 3, chunk_bytes=8)
    arena = VmmResidentArena(layout, backing_factory=calls.factory, synchronize=calls.sync)
    arena.reserve(0, 3)
    arena.reserve(0, 1)
    arena.reserve(1, 1)
    arena.resize_quiescent(0, 2)
    arena.close()
    arena.close()
    assert calls.mock_calls == [
        call.factory(72, chunk_bytes=8, device=0), call.factory().ensure({0}),
        call.factory().ensure({1, 2, 3}), call.factory().ensure({5}),
        call.sync(), call.factory().reclaim({3}, synchronize=False),
        call.sync(), call.factory().close(),
    ]
    with pytest.raises(RuntimeError):
        arena.reserve(0, 1)


def test_arena_failure_stops_use():
    calls = Mock()
    layout = VirtualKVLayout(2, 5, 3, chunk_bytes=8)
    arena = VmmResidentArena(layout, backing_factory=calls.factory, synchronize=calls.sync)
    calls.factory.return_value.ensure.side_effect = RuntimeError("allocation failed")
    with pytest.raises(RuntimeError, match="allocation failed"):
        arena.reserve(0, 2)
    with pytest.raises(RuntimeError):
        arena.row_view(0, 0, SimpleNamespace(itemsize=2))
    arena.close()
    calls.sync.assert_called_once()


# ---------------------------------------------------------------- page tracker

class FakeBacking:
    def __init__(self):
        self.mapped_chunks = set()
        self.fail = False

    @property
    def backed_bytes(self):
        return len(self.mapped_chunks) * 8

    def ensure(self, indices):
        if self.fail:
            raise RuntimeError("map failed")
        self.mapped_chunks.update(indices)

    def reclaim(self, indices, *, synchronize):
        assert not synchronize
        self.mapped_chunks.difference_update(indices)
        return len(indices)


def test_physical_pages_known_answers():
    """tests/test_minimax_vmm.py:27-51."""
    backing = FakeBacking()
    syncs = []
    pages = PhysicalPages(backing, 2, 4, [(0, 3), (8, 2)], lambda: syncs.append(True), chunk_bytes=8)
    assert pages.chunks(1) == {0, 1, 8}
    pages.acquire([1, 2, 2])
    pages.acquire([2])
    pages.release({1})
    assert pages.stats()["reclaimable_bytes"] == 0
    pages.release({2})
    assert pages.trim_quiescent() == 24
    assert backing.mapped_chunks == {0, 8} and syncs == [True]
    with pytest.raises(RuntimeError):
        pages.release({0})
    failing = FakeBacking()
    tracker = PhysicalPages(failing, 1, 3, [(0, 8)], lambda: None, chunk_bytes=8)
    failing.fail = True
    with pytest.raises(RuntimeError, match="map failed"):
        tracker.acquire([1])
    assert tracker.pages == {0} and tracker.refs == {0: 1}


@pytest.mark.parametrize("index", range(40))
def test_physical_pages_projection_matches_reference(index):
    case = load_json("host_golden.json")["releasable"][index]
    tracker = PhysicalPages(FakeBacking(), case["page_size"], case["page_count"],
                            [tuple(p) for p in case["planes"]], lambda: None,
                            chunk_bytes=case["chunk_bytes"])
    for page, chunks in case["page_chunks"].items():
        assert sorted(tracker.chunks(int(page))) == chunks
    tracker.acquire(case["owned"])
    assert {str(k): v for k, v in tracker.refs.items()} == case["refs"]
    assert tracker.n_chunks == case["n_chunks"]


@pytest.mark.parametrize("index", range(12))
def test_plan_demote_pages_matches_reference(index, monkeypatch):
    case = load_json("host_golden.json")["plan_demote"][index]
    tracker = PhysicalPages(FakeBacking(), case["page_size"], 60, [tuple(p) for p in case["planes"]],
                            lambda: None, chunk_bytes=case["chunk_bytes"])
    tracker.acquire(case["owned"])
    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "0")
    kept, released = migration.plan_demote_pages(tracker, case["pages"], case["keep"])
    assert [list(kept), list(released)] == case["plain"]
    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
    kept, released = migration.plan_demote_pages(tracker, case["pages"], case["keep"])
    assert [list(kept), list(released)] == case["aware"]


def test_plan_demote_pages_rejects_bad_input(monkeypatch):
    monkeypatch.delenv("EKV_CHUNK_AWARE_RETENTION", raising=False)
    for pages, keep in (([1, 2], 0), ([1, 2], 3), ([1, 1], 1)):
        with pytest.raises(ValueError):
            migration.plan_demote_pages(None, pages, keep)
    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
    with pytest.raises(RuntimeError):
        migration.plan_demote_pages(None, [1, 2], 1)


def test_bitmap_helpers_round_trip():
    chunks = {0, 1, 63, 64, 127, 200, 4095}
    bits = chunks_to_bitmap(chunks, 4096, "cpu")
    assert bits.dtype == torch.int64 and bits.numel() == 64
    assert bitmap_to_chunks(bits) == chunks
    with pytest.raises(ValueError):
        chunks_to_bitmap({4096}, 4096, "cpu")


# ---------------------------------------------------------------- Backing with a fake ABI

class FakeLibrary:
    """Stands in for the ev_* ABI; can fail a call and report poisoning."""

    def __init__(self):
        self.calls = []
        self.fail = None
        self.poisoned = 0
        self.error = b""
        self.mapped = set()
        self.spare_limit = 0
        self.spare = 0

    def ev_create(self, device, capacity, chunk):
        self.chunk = chunk
        self.capacity = -(-capacity // chunk) * chunk
        return 1234

    def _ids(self, array, count):
        return [array[i] for i in range(count)]

    def _op(self, name, handle, array, count):
        ids = self._ids(array, count)
        self.calls.append((name, ids))
        if self.fail == name:
            self.error = f"{name} failed".encode()
            return -1
        if name == "ev_drop":
            dropped = len(self.mapped & set(ids))
            self.mapped.difference_update(ids)
            self.spare = min(self.spare_limit, self.spare + dropped)
        else:
            fresh = len(set(ids) - self.mapped)
            self.spare -= min(self.spare, fresh)
            self.mapped.update(ids)
        return 0

    def ev_set_spare(self, handle, chunks):
        self.calls.append(("ev_set_spare", [chunks]))
        if self.fail == "ev_set_spare":
            self.error = b"ev_set_spare failed"
            return -1
        self.spare_limit = chunks
        self.spare = min(self.spare, chunks)
        return 0

    def ev_spare(self, handle):
        return self.spare * self.chunk

    def ev_ensure(self, handle, array, count):
        return self._op("ev_ensure", handle, array, count)

    def ev_precommit(self, handle, array, count):
        return self._op("ev_precommit", handle, array, count)

    def ev_drop(self, handle, array, count):
        return self._op("ev_drop", handle, array, count)

    def ev_base(self, handle):
        return 1 << 40

    def ev_reserved(self, handle):
        return self.capacity

    def ev_granularity(self, handle):
        return self.chunk

    def ev_backed(self, handle):
        return len(self.mapped) * self.chunk

    def ev_poisoned(self, handle):
        return self.poisoned

    def ev_error(self):
        return self.error

    def ev_close(self, handle):
        self.calls.append(("ev_close", []))
        if self.fail == "ev_close":
            self.error = b"ev_close failed"
            return -1
        return 0


def test_backing_batches_and_metrics():
    lib = FakeLibrary()
    backing = Backing(10 << 20, 2 << 20, device=0, library=lib)
    assert backing.reserved_bytes == 10 << 20
    assert backing.ensure({3, 1, 1}) == 2
    assert backing.ensure({1}) == 0
    assert backing.precommit({4}) == 1
    assert backing.mapped_chunks == {1, 3}
    assert backing.ensure({4}) == 0 and backing.mapped_chunks == {1, 3, 4}
    assert backing.reclaim({3, 2}, synchronize=False) == 1
    assert lib.calls == [("ev_ensure", [1, 3]), ("ev_precommit", [4]), ("ev_ensure", []),
                         ("ev_drop", [3])]
    assert backing.metrics["ensure_chunks"] == 2 and backing.metrics["reclaim_chunks"] == 1
    with pytest.raises(ValueError):
        backing.ensure({5})
    backing.close()
    assert lib.calls[-1] == ("ev_close", [])
    with pytest.raises(RuntimeError):
        backing.ensure({1})


def test_backing_clean_failure_stays_usable_and_poison_stops_it():
    lib = FakeLibrary()
    backing = Backing(8 << 20, 2 << 20, device=0, library=lib)
    lib.fail = "ev_ensure"
    with pytest.raises(RuntimeError, match="ev_ensure failed"):
        backing.ensure({1})
    assert backing.mapped_chunks == set()
    lib.fail = None
    assert backing.ensure({1}) == 1
    lib.fail, lib.poisoned = "ev_drop", 1
    with pytest.raises(RuntimeError, match="ev_drop failed"):
        backing.reclaim({1}, synchronize=False)
    with pytest.raises(RuntimeError, match="closed or has encountered"):
        backing.ensure({2})


def test_backing_failed_close_is_final():
    """ev_close frees its handle even when the teardown fails, so a failed close leaves
    the backing poisoned with no handle: it raises once, and neither a second close nor
    the garbage-collection finalizer calls ev_close on the freed handle again."""
    import gc

    lib = FakeLibrary()
    backing = Backing(8 << 20, 2 << 20, device=0, library=lib)
    backing.ensure({1})
    lib.fail = "ev_close"
    with pytest.raises(RuntimeError, match="teardown failed: ev_close failed"):
        backing.close()
    with pytest.raises(RuntimeError, match="closed or has encountered"):
        backing.ensure({2})
    backing.close()
    del backing
    gc.collect()
    assert [c for c in lib.calls if c[0] == "ev_close"] == [("ev_close", [])]
    # A backing dropped without close is closed once by its finalizer.
    lib2 = FakeLibrary()
    dropped = Backing(8 << 20, 2 << 20, device=0, library=lib2)
    del dropped
    gc.collect()
    assert [c for c in lib2.calls if c[0] == "ev_close"] == [("ev_close", [])]


def test_backing_spare_handles():
    """Reclaimed handles are kept up to the spare limit and reused by the next ensure;
    the metrics report them apart from the backed bytes."""
    lib = FakeLibrary()
    backing = Backing(16 << 20, 2 << 20, device=0, library=lib, spare_chunks=2)
    assert lib.calls[0] == ("ev_set_spare", [2])
    backing.ensure({1, 2, 3})
    backing.reclaim({1, 2, 3}, synchronize=False)
    assert backing.spare_bytes == 2 * (2 << 20) and backing.backed_bytes == 0
    backing.ensure({4})
    assert backing.metrics["spare_bytes"] == 2 << 20 and backing.metrics["backed_bytes"] == 2 << 20
    backing.set_spare_chunks(0)
    assert backing.spare_bytes == 0
    with pytest.raises(ValueError):
        backing.set_spare_chunks(-1)
    lib.fail = "ev_set_spare"
    with pytest.raises(RuntimeError, match="ev_set_spare failed"):
        backing.set_spare_chunks(3)


def test_backing_rejects_bad_arguments():
    lib = FakeLibrary()
    with pytest.raises(ValueError):
        Backing(0, 2 << 20, library=lib)
    with pytest.raises(ValueError):
        Backing(1 << 20, 2 << 20, device="cpu", library=lib)


# ---------------------------------------------------------------- migration state machine

def _coordinator(length=8, capacity=4, page_size=2):
    rows = 3
    host_calls = []

    class HostPool:
        def alloc_paged_token_slots(self, table, allocated, row, start, end):
            table[row, start:end] = torch.arange(start, end)
            allocated[row] = end
            return table[row, :end]

        def backup_from_device_all_layer(self, pool, host, physical, io_backend):
            host_calls.append(("backup", host.tolist(), physical.tolist(), io_backend))

        def allocated_host_indices(self, table, row, n):
            return table[row, :int(n)]

        def free(self, indices):
            host_calls.append(("free", indices.tolist()))

    physical = torch.arange(2, 2 + length, dtype=torch.int64)  # page-aligned, pages 1..4
    device_pool = SimpleNamespace(
        page_size=page_size,
        translate_loc_from_full_to_hisparse_device=lambda logical: physical.clone(),
        full_to_hisparse_device_index_mapping=torch.arange(64, dtype=torch.int64),
        start_layer=0, end_layer=1)
    coordinator = SimpleNamespace(
        is_m3_hisparse=True, spec_swap=SimpleNamespace(enabled=False, reset=lambda row: None),
        padded_buffer_size=capacity, device_buffer_size=capacity,
        req_device_buffer_size=torch.zeros(rows, dtype=torch.int64),
        req_to_host_pool=torch.full((rows, 16), -1, dtype=torch.int64),
        req_to_host_pool_allocated_len=torch.zeros(rows, dtype=torch.int64),
        req_to_token_pool=SimpleNamespace(req_to_token=torch.arange(rows * 16).reshape(rows, 16)),
        mem_pool_device=device_pool, mem_pool_host=HostPool(),
        wait_for_pending_backup=lambda: None,
        token_to_kv_pool_allocator=SimpleNamespace(_kvcache=SimpleNamespace(),
                                                   free_hisparse_indices=Mock()),
        req_to_device_buffer=torch.zeros((rows, 16), dtype=torch.int64),
        req_device_buffer_tokens=torch.zeros((1, rows, 16), dtype=torch.int64),
        req_device_buffer_token_locs=torch.zeros((1, rows, 16), dtype=torch.int64),
        lru_slots=torch.zeros((1, rows, 4), dtype=torch.int64), _lru_init=torch.arange(4),
        _skip_first_backup=[False] * rows)
    request = SimpleNamespace(kv=SimpleNamespace(req_pool_idx=1, kv_committed_len=length,
                                                 kv_allocated_len=length),
                              hisparse_staging=False)
    return coordinator, request, host_calls


def test_demotion_transaction_state_machine(monkeypatch):
    monkeypatch.delenv("EKV_CHUNK_AWARE_RETENTION", raising=False)
    coordinator, request, host_calls = _coordinator()
    syncs = []
    prepared = migration.prepare_demote(coordinator, request, lambda: syncs.append(1))
    assert prepared.status == "prepared"
    assert prepared.retained_rows == (0, 1) and prepared.released_rows == (2, 3)
    assert host_calls[0][0] == "backup" and host_calls[0][2] == list(range(2, 10))
    published = []
    released = migration.commit_demote(prepared, published.append, lambda: None)
    assert released == 0 and published == [1] and prepared.status == "committed"
    assert coordinator.req_to_device_buffer[1, :4].tolist() == [2, 3, 4, 5]
    assert coordinator._skip_first_backup[1] is True
    freed = coordinator.token_to_kv_pool_allocator.free_hisparse_indices.call_args[0][0]
    assert freed.tolist() == [6, 8]
    with pytest.raises(RuntimeError):
        migration.commit_demote(prepared, published.append, lambda: None)
    with pytest.raises(RuntimeError):
        migration.abort_demote(prepared)


def test_demotion_abort_and_rejections(monkeypatch):
    monkeypatch.delenv("EKV_CHUNK_AWARE_RETENTION", raising=False)
    coordinator, request, host_calls = _coordinator()
    prepared = migration.prepare_demote(coordinator, request, lambda: None)
    migration.abort_demote(prepared)
    assert prepared.status == "aborted" and host_calls[-1][0] == "free"
    assert int(coordinator.req_to_host_pool_allocated_len[1]) == 0
    short, short_request, _ = _coordinator(length=2, capacity=4)
    with pytest.raises(ValueError):
        migration.prepare_demote(short, short_request, lambda: None)
    coordinator, request, _ = _coordinator()
    coordinator.spec_swap.enabled = True
    with pytest.raises(RuntimeError):
        migration.prepare_demote(coordinator, request, lambda: None)


def test_profile_ranges_env_is_read_at_decoration(monkeypatch):
    from ekv_b200.profile_ranges import profile_range

    def fn():
        return 3

    monkeypatch.delenv("EKV_PROFILE_RANGES", raising=False)
    assert profile_range("x")(fn) is fn
    monkeypatch.setenv("EKV_PROFILE_RANGES", "1")
    wrapped = profile_range("x")(fn)
    assert wrapped is not fn and wrapped() == 3


def test_profile_ranges_nest_and_let_exceptions_through(monkeypatch):
    """Enabled ranges enter and exit in nesting order around each call, an exception
    raised inside propagates unchanged through both ranges, and the wrapper keeps the
    function's name (the behaviour tests/test_profile_ranges.py:24-50 of the reference
    pins)."""
    import contextlib

    import torch

    from ekv_b200.profile_ranges import profile_range

    events = []

    @contextlib.contextmanager
    def record_function(name):
        events.append(("enter", name))
        try:
            yield
        finally:
            events.append(("exit", name))

    monkeypatch.setenv("EKV_PROFILE_RANGES", "1")
    monkeypatch.setattr(torch.profiler, "record_function", record_function)
    expected = ValueError("bad input")

    @profile_range("test/inner")
    def inner(*, fail):
        if fail:
            raise expected
        return 7

    @profile_range("test/outer")
    def outer(fail):
        return inner(fail=fail)

    assert outer(False) == 7
    with pytest.raises(ValueError) as caught:
        outer(True)
    assert caught.value is expected and inner.__name__ == "inner"
    assert events == [("enter", "ekv/test/outer"), ("enter", "ekv/test/inner"),
                      ("exit", "ekv/test/inner"), ("exit", "ekv/test/outer")] * 2


def test_no_cpu_fallback_without_cuda_tensors():
    from ekv_b200.resident_lookup import lookup_slots, resolve_resident

    x = torch.zeros((1, 2, 3), dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        resolve_resident(x, torch.zeros((2, 3), dtype=torch.int32), torch.zeros(3, dtype=torch.int64),
                         torch.zeros(2, dtype=torch.int64), torch.zeros(2, dtype=torch.int32),
                         torch.zeros(1, dtype=torch.int64), torch.zeros((1, 2, 3), dtype=torch.int32), 1)
    with pytest.raises(ValueError, match="CUDA"):
        lookup_slots(torch.zeros((2, 4), dtype=torch.int32), torch.zeros((2, 3), dtype=torch.int32))


def test_lookup_gather_has_no_cpu_fallback():
    """The fused lookup + gather rejects host tensors before any launch, and rejects
    mismatched shapes first."""
    from ekv_b200.sparse_read import LookupGather
    from ekv_b200.virtual_layout import VirtualKVLayout

    layout = VirtualKVLayout(2, 8, 16, itemsize=2, chunk_bytes=4096)
    plane = torch.zeros(layout.capacity_bytes // 2, dtype=torch.int16)
    res_map = torch.full((2, 20), -1, dtype=torch.int32)
    topk = torch.zeros((2, 5), dtype=torch.int32)
    ids, lengths = torch.arange(2), torch.full((2,), 20)
    out = torch.empty((2, 5, 16), dtype=torch.int16)
    with pytest.raises(ValueError, match="CUDA"):
        LookupGather([plane], res_map, topk, ids, lengths, [out], layout, disjoint=True)
    with pytest.raises(ValueError, match="output shape"):
        LookupGather([plane], res_map, topk, ids, lengths, [out[:, :4]], layout)
    with pytest.raises(ValueError, match="one entry per Top-K row"):
        LookupGather([plane], res_map, topk, ids[:1], lengths, [out], layout)
    with pytest.raises(ValueError, match="EKV_MAX_PLANES"):
        LookupGather([], res_map, topk, ids, lengths, [], layout)


def test_library_missing_fails_loudly(tmp_path):
    from ekv_b200 import _lib

    with pytest.raises(RuntimeError, match="no fallback"):
        _lib.library(str(tmp_path / "missing.so"))


def test_library_without_the_entry_points_asks_for_a_rebuild(tmp_path):
    """A shared library that loads but lacks this package's entry points (an older build)
    is refused with a rebuild instruction, not an AttributeError from ctypes."""
    import shutil
    import subprocess

    from ekv_b200 import _lib

    compiler = shutil.which("gcc") or shutil.which("cc")
    if compiler is None:
        pytest.skip("no C compiler")
    source = tmp_path / "old.c"
    source.write_text("int ekv_unrelated(void) { return 0; }\n")
    stale = tmp_path / "libold.so"
    subprocess.run([compiler, "-shared", "-fPIC", "-o", str(stale), str(source)], check=True)
    with pytest.raises(RuntimeError, match="ABI is outdated"):
        _lib.library(str(stale))


def test_ctypes_arrays():
    from ekv_b200._lib import i64_array, u64_array

    assert list(u64_array([1, 2])) == [1, 2]
    assert isinstance(i64_array([]), ct.Array)
    assert os.path.basename(str(__file__)).startswith("test_")


# ---------------------------------------------------------------- shared prefix (host checks)

def test_complete_shared_blocks_matches_reference_answers():
    from ekv_b200.shared_prefix import complete_shared_blocks

    # tests/test_shared_prefix.py:138-144 of the reference.
    assert complete_shared_blocks([0, 1, 2, -1], seq_len=300, shared_tokens=256, block_size=128) == (
        True, True, False, False)
    for kwargs in (dict(seq_len=0, shared_tokens=1, block_size=1), dict(seq_len=1, shared_tokens=-1, block_size=1),
                   dict(seq_len=1, shared_tokens=1, block_size=True)):
        with pytest.raises(ValueError, match="outside the supported range"):
            complete_shared_blocks([0], **kwargs)
    with pytest.raises(ValueError, match="block ids must be integers"):
        complete_shared_blocks([True], seq_len=4, shared_tokens=4, block_size=1)


def test_shared_resolvers_reject_like_the_reference():
    """Validation runs before any device work, with the reference's messages
    (shared_prefix.py:86-106, :137-178)."""
    from ekv_b200.shared_prefix import resolve_shared_block_locations, resolve_shared_block_locations_batched

    table = torch.arange(12).reshape(2, 6)
    mapping = torch.arange(12)
    scalar = dict(seq_len=torch.tensor(6), shared_tokens=4, block_size=2, request_table=table,
                  device_mapping=mapping)
    with pytest.raises(ValueError, match="one-dimensional"):
        resolve_shared_block_locations(torch.zeros(2, 2, dtype=torch.long), source_row=0, **scalar)
    with pytest.raises(ValueError, match="source row is outside"):
        resolve_shared_block_locations(torch.tensor([0]), source_row=2, **scalar)
    with pytest.raises(ValueError, match="geometry is empty"):
        resolve_shared_block_locations(torch.tensor([0]), source_row=0,
                                       **{**scalar, "device_mapping": torch.empty(0, dtype=torch.long)})
    with pytest.raises(ValueError, match="invalid shared block geometry"):
        resolve_shared_block_locations(torch.tensor([0]), source_row=0, **{**scalar, "shared_tokens": -1})
    batched = dict(seq_len=torch.tensor([6]), block_size=2, request_table=table, device_mapping=mapping)
    # tests/test_shared_prefix.py:230-242 of the reference.
    with pytest.raises(ValueError, match="dimensions differ"):
        resolve_shared_block_locations_batched(torch.tensor([[0, 1]]), source_rows=[0], shared_tokens=[2, 4],
                                               **batched)
    with pytest.raises(ValueError, match="sequence length dimensions differ"):
        resolve_shared_block_locations_batched(torch.tensor([[0, 1]]), source_rows=[0], shared_tokens=[2],
                                               **{**batched, "seq_len": torch.tensor([6, 6])})
    with pytest.raises(ValueError, match="two-dimensional"):
        resolve_shared_block_locations_batched(torch.tensor([0, 1]), source_rows=[0], shared_tokens=[2], **batched)
    with pytest.raises(ValueError, match="must be integers"):
        resolve_shared_block_locations_batched(torch.ones(1, 2, dtype=torch.bool), source_rows=[0],
                                               shared_tokens=[2], **batched)
    with pytest.raises(ValueError, match="source row is outside"):
        resolve_shared_block_locations_batched(torch.tensor([[0]]), source_rows=[5], shared_tokens=[2], **batched)
    with pytest.raises(ValueError, match="invalid shared prefix geometry"):
        resolve_shared_block_locations_batched(torch.tensor([[0]]), source_rows=[0], shared_tokens=[-2], **batched)
    # Empty batches return empty results without touching a device (shared_prefix.py:167-181).
    valid, physical = resolve_shared_block_locations_batched(
        torch.empty(0, 3, dtype=torch.long), source_rows=[], shared_tokens=[],
        **{**batched, "seq_len": torch.empty(0, dtype=torch.long)})
    assert valid.shape == (0, 3) and physical.shape == (0, 3, 2) and physical.dtype == torch.int32
    # A CPU tensor reaching the kernel path is refused: there is no CPU fallback.
    with pytest.raises(ValueError, match="CUDA tensor"):
        resolve_shared_block_locations_batched(torch.tensor([[0]]), source_rows=[0], shared_tokens=[2], **batched)


# ---------------------------------------------------------------- logical shadow (host side)

def test_logical_shadow_host_contract(tmp_path):
    """Errors raised before any device work and the publish record
    (adaptive_sparse/logical_shadow.py:30-48, :88-105, :125-140)."""
    from ekv_b200.logical_shadow import LogicalShadow

    shadow = LogicalShadow(16, "cpu")
    key = torch.zeros((2, 1, 4), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="unit-scale BF16"):
        shadow.write(0, torch.tensor([1, 2]), key.float(), key, (None, None))
    with pytest.raises(RuntimeError, match="unit-scale BF16"):
        shadow.write(0, torch.tensor([1, 2]), key, key, (None, 0.5))
    with pytest.raises(RuntimeError, match="recorded producer writes"):
        shadow.check(5, key, key, None, None, None, 1, torch.zeros((1, 1, 1), dtype=torch.int32), None, None, 1)
    with pytest.raises(ValueError, match="Invalid migration shadow slot vectors"):
        shadow.check_complete(None, torch.zeros((2, 2)), torch.zeros((2, 2)), "b")
    with pytest.raises(ValueError, match="Invalid migration shadow slot vectors"):
        shadow.check_complete(None, torch.zeros(0), torch.zeros(0), "b")
    pool = SimpleNamespace(page_size=4, size=64, start_layer=3, end_layer=5)
    with pytest.raises(RuntimeError, match="Missing migration shadow writes for layer 3"):
        shadow.check_complete(pool, torch.arange(4, 8), torch.arange(4, 8), "b")
    shadow.reset(torch.tensor([1, 2]))  # no layers yet: nothing to do

    shadow.publish(tmp_path, 0)  # not dirty: no file
    assert not list(tmp_path.iterdir())
    shadow.counts += torch.tensor([5, 40, 0, 0, 0, 1, 0])
    shadow.migration_counts["migration_checked_tokens"] = 9
    shadow.dirty = True
    shadow.publish(tmp_path, 2)
    stats = __import__("json").loads((tmp_path / "shadow-tp-2.json").read_text())
    assert stats["checked_tokens"] == 5 and stats["checked_bytes"] == 40 and stats["checked_calls"] == 1
    assert stats["migration_checked_tokens"] == 9 and stats["tp_rank"] == 2 and stats["logical_capacity"] == 16
    assert stats["boundary"] == "scheduler_idle" and not shadow.dirty
    shadow.counts[6] += 1  # a malformed Top-K block is a failure
    shadow.dirty = True
    with pytest.raises(RuntimeError, match="Logical KV shadow mismatch"):
        shadow.publish(tmp_path, 2)


def test_layer_pipeline_contract():
    from ekv_b200.pipeline import LayerPipeline

    with pytest.raises(ValueError, match="one producer and one consumer"):
        LayerPipeline([], [], "cpu")
    with pytest.raises(ValueError, match="one producer and one consumer"):
        LayerPipeline([lambda s: None], [], "cpu")


def test_peer_combiner_checks_its_arguments():
    """PeerFreeableCombiner.combine refuses a call without a local bitmap source and
    tensors that are not CUDA tensors of the combiner's sizes, before any launch."""
    import torch

    from ekv_b200.releasable import PeerFreeableCombiner

    combiner = PeerFreeableCombiner(100, "cpu", buffers=[0x1000], rank=0)
    assert combiner.n_words == 2
    with pytest.raises(ValueError, match="counts, refs and mapped_bits, or local_bits"):
        combiner.combine()
    with pytest.raises(ValueError, match="counts, refs and mapped_bits, or local_bits"):
        combiner.combine(torch.zeros(100, dtype=torch.int32), torch.zeros(100, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA tensor"):
        combiner.combine(local_bits=torch.zeros(2, dtype=torch.int64), out=torch.zeros(2, dtype=torch.int64))
    with pytest.raises(ValueError, match="rank is required"):
        PeerFreeableCombiner(100, "cpu", buffers=[0x1000])


def _fake_pipeline_torch(log):
    """A stand-in for the torch.cuda calls LayerPipeline makes, recording each one."""
    import types

    import torch

    class Stream:
        def __init__(self, name="side"):
            self.name = self.cuda_stream = name

        def wait_stream(self, other):
            log.append(("wait_stream", self.name, other.name))

        def wait_event(self, event):
            log.append(("wait_event", self.name, event.id))

    class Event:
        made = 0

        def __init__(self):
            Event.made += 1
            self.id = Event.made

        def record(self, stream):
            log.append(("record", self.id, stream.name))

    main = Stream("main")
    cuda = types.SimpleNamespace(Stream=lambda device: Stream("side"), Event=Event,
                                 current_stream=lambda device: main)
    return types.SimpleNamespace(cuda=cuda, device=torch.device)


@pytest.mark.parametrize("wait", [True, False])
def test_layer_pipeline_stream_order(wait, monkeypatch):
    """LayerPipeline's schedule, recorded through fake streams and events.  wait=True:
    producers on the caller's stream, consumer i on the second stream after an event
    recorded behind producer i.  wait=False: consumers on the caller's stream, producer i
    forked onto the second stream behind everything issued before layer i (so after
    consumer i-1, not after consumer i).  Both fork first and join once at the end."""
    from ekv_b200 import pipeline

    log = []
    monkeypatch.setattr(pipeline, "torch", _fake_pipeline_torch(log))
    layers = 3
    produce = [lambda s, i=i: log.append(("produce", i, s)) for i in range(layers)]
    consume = [lambda s, i=i: log.append(("consume", i, s)) for i in range(layers)]
    step = pipeline.LayerPipeline(produce, consume, "cpu", wait=wait)
    event = {i: step.ready[i].id for i in range(layers)}
    step()
    want = [("wait_stream", "side", "main")]
    for i in range(layers):
        if wait:
            want += [("produce", i, "main"), ("record", event[i], "main"), ("wait_event", "side", event[i]),
                     ("consume", i, "side")]
        else:
            want += [("record", event[i], "main"), ("wait_event", "side", event[i]), ("produce", i, "side"),
                     ("consume", i, "main")]
    want.append(("wait_stream", "main", "side"))
    assert log == want


def test_swap_pipeline_is_the_waiting_layer_pipeline(monkeypatch):
    """SwapPipeline runs each plan's swap-in as the producer and its gather as the
    consumer, in the waiting form (the gather reads the rows the swap-in promoted)."""
    import types

    from ekv_b200 import pipeline, swap

    log = []
    monkeypatch.setattr(pipeline, "torch", _fake_pipeline_torch(log))

    def plan(i):
        return types.SimpleNamespace(device="cpu", swap_in=lambda s: log.append(("swap_in", i, s)),
                                     gather=lambda s: log.append(("gather", i, s)))

    step = swap.SwapPipeline([plan(0), plan(1)])
    assert step.wait
    step()
    calls = [entry for entry in log if entry[0] in ("swap_in", "gather")]
    assert calls == [("swap_in", 0, "main"), ("gather", 0, "side"), ("swap_in", 1, "main"), ("gather", 1, "side")]
    with pytest.raises(ValueError, match="at least one layer"):
        swap.SwapPipeline([])


# ---------------------------------------------------------------- migration transactions vs the reference

def _cpu_world(**geometry):
    from tests.support.standin import CpuHostPool, migration_world

    return migration_world("cpu", tracker_cls=PhysicalPages, host_pool_cls=CpuHostPool, **geometry)


@pytest.mark.parametrize("scenario", ["plain", "chunk_aware", "aborts"])
def test_transaction_logic_matches_the_reference_trace(scenario):
    """This package's transactions and page tracker over the CPU stand-in world (host
    rows moved by the stand-in's CPU host pool) leave the state the reference's left in
    tests/golden/migration_trace.json, step for step.  The GPU test runs the same
    scenarios, plus the newest-token copy, through the device data path."""
    from tests.support import migration_scenarios as ms

    want = load_json("migration_trace.json")[scenario]
    got = (ms.aborts(_cpu_world, migration) if scenario == "aborts"
           else ms.round_trip(_cpu_world, migration, aware=scenario == "chunk_aware"))
    assert got == want


def test_transaction_rejections_match_the_reference_trace():
    from tests.support import migration_scenarios as ms

    assert ms.rejections(_cpu_world, migration) == load_json("migration_trace.json")["rejections"]


def test_newest_token_copy_needs_the_device_path():
    """The newest token's rows are copied by the row-copy kernel: on CPU tensors the
    promotion refuses instead of falling back to host copies."""
    from tests.support import migration_scenarios as ms

    with pytest.raises(ValueError, match="CUDA"):
        ms.round_trip(_cpu_world, migration, aware=True, newest_on_device=True)


@pytest.mark.parametrize("index", range(60))
def test_plan_demote_pages_large_matches_reference(index, monkeypatch):
    """The incremental retention planner against the reference's greedy planner on
    denser ownership patterns (tests/golden/plan_demote_large.json)."""
    case = load_json("plan_demote_large.json")[index]
    tracker = PhysicalPages(FakeBacking(), case["page_size"], case["page_count"],
                            [tuple(p) for p in case["planes"]], lambda: None, chunk_bytes=case["chunk_bytes"])
    tracker.acquire(case["owned"])
    monkeypatch.setenv("EKV_CHUNK_AWARE_RETENTION", "1")
    kept, released = migration.plan_demote_pages(tracker, case["pages"], case["keep"])
    assert [list(kept), list(released)] == case["aware"]
