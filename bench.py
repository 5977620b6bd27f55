#!/usr/bin/env python
"""Benchmark of the B200 sparse-KV residency data path.

Headline: Top-K K/V row gather from a VMM-backed
pool of 36 layers x K,V planes [262144, 8, 128] bf16 (36 GiB), 64 requests x
2048 Top-K slots, all 72 planes in one launch of the sm_100a gather kernel
(index chain positions -> request_table -> slot_offsets resolved per row).
Under ``--gpus N`` (torchrun) the KV heads are sharded across ranks
(tensor-parallel layout: 8/N heads per rank, same slots), so the total work is
fixed: ``scaling = strong``.  One step = one launch over the whole batch.

Extra keys: ``e2e`` (public Python API per step, positions copied from pinned
host memory -- one step ahead, on a second stream -- and one result row read back), ``roofline`` (gather kernel vs the
measured HBM copy peak), ``cpu_baseline`` (torch-CPU restatement on the host
cores, bounded sample), ``migration`` (config 3: 256 victim chunks packed into
pinned host staging through the copy-engine ring and restored into fresh VMM
chunks with permuted slots; host-link GB/s per direction; plus the commit path and a
forced demote + promote round trip through the transaction API at the size of the
reference's published case), ``lookup``
(config 1 lookups, resolve_resident at the reference's microbenchmark shape,
shared-prefix donor resolution at the config-5 shape, the reference's single-plane
gather_rows at one TP8 layer plane), ``shadow`` (logical-shadow
bitwise check of one decode step at the config-2 batch, vs the reference's torch body
on the same GPU), ``bitmap`` (config 4
geometry: freeable bitmap build, the NCCL AND-combine latency and, for N > 1,
the fused peer-memory combine), ``clocks`` (NVML samples during the timed
region).

``config4``: config 4 (BASELINE.json's 2/4/8-GPU configuration) measured in the
same run after the config-2 pool is released: 48 layers of lookup + K,V gather per
decode step and the freeable bitmap with its cross-rank AND-combine (for N > 1 one
kernel over NVLink peer memory beside the layers; NCCL all-gather + AND after them
timed beside it), all inside the timed step (``--skip-config4`` leaves it out).  ``config5``, on one GPU:
config 5's 64 decode steps (lookup -> victim selection -> promotion from pinned host
history -> gather per layer), as ``--config 5`` reports them (``--skip-config5``).

``--config 4`` / ``--config 5`` time the decode-step configurations instead (one
JSON line each): config 4 reports its fused form (each layer's lookup and mapped
gather in one launch, the miss-list compaction beside the next layer) with the
concurrent form (the lookup beside the mapped gather), the plain layer order, and
the two forms that need every layer's Top-K up front (pipelined, multi-layer) in
``step_forms``; config 5 reports the swap-in pipeline with the plain layer
order as ``sequential_ms_per_step``.

``--impl reference`` times the reference's CPU path (torch-CPU restatement,
all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _path in (str(ROOT / "elastic-kv-vmm_b200"), str(ROOT)):
    if _path not in sys.path:
        sys.path.insert(0, _path)

# The fused bitmap combine reads peers through plain peer mappings; torch's symmetric
# memory need not bind an NVSwitch multicast object for it.
os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")

import torch  # noqa: E402

CHUNK = 2 << 20
CFG2 = dict(layers=36, kv_heads=8, head_dim=128, slots=262144, requests=64, topk=2048)
INDEX_BYTES_PER_ROW_PAIR = 4  # per-unit index bytes of the algorithmic byte count
METRIC = "Top-K KV rows/s (gather, row-pairs/s)"
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", type=int, choices=(2, 4, 5), default=2,
                   help="2 = headline gather (default); 4 = TP-sharded lookup + gather + bitmap combine; "
                        "5 = multi-step decode with swap-in from host history")
    p.add_argument("--layers", type=int, default=None,
                   help="layers (default: 36 for config 2, 48 for config 4; fewer only for profiling captures)")
    p.add_argument("--skip-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--skip-migration", action="store_true")
    p.add_argument("--skip-e2e", action="store_true")
    p.add_argument("--skip-config4", action="store_true", help="skip the config-4 decode-step leg")
    p.add_argument("--skip-config5", action="store_true", help="skip the config-5 decode leg (1 GPU runs)")
    p.add_argument("--skip-legs", action="store_true",
                   help="measurement aid: skip the bitmap, lookup and shadow side legs (profiling captures)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline time budget")
    p.add_argument("--only", choices=("lookup", "shadow", "bitmap", "roundtrip"), default=None,
                   help="measurement aid: run one side leg alone (no config-2 pool) and print its JSON")
    p.add_argument("--tp-shard", type=int, default=0,
                   help="measurement aid: gather one rank's head shard of TP=N on this GPU "
                        "(default: the launch's world size)")
    return p.parse_args(argv)


# --------------------------------------------------------------------------- plumbing

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1
        if self.enabled:
            import datetime

            import torch.distributed as dist

            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local_rank))
        self.device = torch.device("cuda", self.local_rank)
        torch.cuda.set_device(self.device)

    def barrier(self):
        if self.enabled:
            import torch.distributed as dist

            dist.barrier(device_ids=[self.local_rank])

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        import torch.distributed as dist

        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.enabled:
            import torch.distributed as dist

            dist.destroy_process_group()


def measured_hbm_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback (profiling recipe 6.65 TB/s)"


class ClockSampler:
    """NVML samples of SM clock and clock-event reasons while the region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks",
               0x10: "sync_boost", 0x100: "display_clocks"}

    def __init__(self, index: int, period: float = 0.02):
        self.samples = []
        self.reasons = set()
        self.period = period
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report no clocks rather than guess
            self._nvml = None

    def _reasons_now(self):
        nvml = self._nvml
        getter = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(getter(self._handle))

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM))
                bits = self._reasons_now()
                for bit, name in self.REASONS.items():
                    if bits & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def timed(fn, steps, warmup, dist: Dist):
    """Device time (ms, max over ranks) of `steps` calls after `warmup` calls."""
    for _ in range(warmup):
        fn()
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(start.elapsed_time(end))


# --------------------------------------------------------------------------- workload

class Workload:
    """Config-2 pool (VMM-backed) and Top-K indices for this rank's head shard."""

    def __init__(self, dist: Dist, layers: int, shard: int = 0):
        from ekv_b200.backing import Backing
        from ekv_b200.virtual_layout import VirtualKVLayout

        shard = shard or dist.world
        if CFG2["kv_heads"] % shard:
            raise SystemExit("--gpus / --tp-shard must divide the 8 KV heads")
        self.dist = dist
        dev = dist.device
        self.layers = layers
        self.heads = CFG2["kv_heads"] // shard
        self.width = self.heads * CFG2["head_dim"]             # elements per row (this rank)
        self.row_bytes = self.width * 2
        self.slots = CFG2["slots"]
        self.n_planes = 2 * layers
        self.plane_bytes = self.slots * self.row_bytes
        self.plane_chunks = -(-self.plane_bytes // CHUNK)
        capacity = CHUNK * (1 + self.n_planes * self.plane_chunks)
        started = time.perf_counter()
        self.backing = Backing(capacity, CHUNK, device=dev.index)
        self.backing.ensure(range(1 + self.n_planes * self.plane_chunks))
        self.map_seconds = time.perf_counter() - started
        raw = self.backing.raw
        gen = torch.Generator(device=dev).manual_seed(1234 + dist.rank)
        self.planes = []
        for p in range(self.n_planes):
            start = CHUNK * (1 + p * self.plane_chunks)
            plane = raw[start:start + self.plane_bytes].view(torch.bfloat16).view(
                self.slots, self.heads, CFG2["head_dim"])
            torch.randn(plane.shape, generator=gen, dtype=torch.bfloat16, device=dev, out=plane)
            self.planes.append(plane)
        del raw
        b, k = CFG2["requests"], CFG2["topk"]
        igen = torch.Generator(device=dev).manual_seed(42)  # same indices on every rank
        self.request_table = torch.stack([torch.randperm(self.slots, generator=igen, device=dev)[:k]
                                          for _ in range(b)])
        # Top-K ids as int32, the dtype an indexer emits (4 B per id, as the byte count has it).
        self.positions = torch.stack([torch.randperm(k, generator=igen, device=dev) for _ in range(b)]).to(torch.int32)
        self.request_ids = torch.arange(b, device=dev)
        self.lengths = torch.full((b,), k, dtype=torch.int64, device=dev)
        self.slot_offsets = torch.arange(self.slots, dtype=torch.int64, device=dev) * self.width
        self.layout = VirtualKVLayout(b, k, self.width)
        self.outputs = [torch.empty((b, k, self.heads, CFG2["head_dim"]), dtype=torch.bfloat16, device=dev)
                        for _ in range(self.n_planes)]
        self.rows = b * k                                  # row-pairs per layer
        self.units = self.rows * layers                    # row-pairs per step (whole job)
        torch.cuda.synchronize()

    def plane_gather(self):
        from ekv_b200.sparse_read import PlaneGather

        return PlaneGather([p.view(self.slots, self.width) for p in self.planes], self.positions,
                           self.request_ids, self.lengths, self.request_table, self.slot_offsets,
                           [o.view(o.shape[0], o.shape[1], self.width) for o in self.outputs],
                           self.layout, indirect=True)

    def close(self):
        self.planes = self.outputs = None
        torch.cuda.synchronize()
        self.backing.close()


def algorithmic_bytes_per_row_pair(row_bytes: int) -> int:
    """Read K and V rows, write K and V rows, plus the per-unit index bytes."""
    return 4 * row_bytes + INDEX_BYTES_PER_ROW_PAIR


def traffic_per_launch(units: int, row_bytes: int):
    """DRAM bytes per launch from the committed ncu summary (scaled per row-pair)."""
    path = ROOT / "profiles" / "gather_kernel_cfg2.md"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("dram_bytes_per_row_pair_2048B:"):
                per_unit = float(line.split(":", 1)[1])
                return per_unit * units * (row_bytes / 2048.0)
    except OSError:
        pass
    return None


# --------------------------------------------------------------------------- CPU legs

def cpu_sample(work: Workload, layers: int):
    """Host copies of `layers` layers of the pool plus the indices (the bounded sample)."""
    planes = [work.planes[p].view(work.slots, work.width).view(torch.int16).cpu()
              for p in range(2 * layers)]
    idx = dict(positions=work.positions.cpu(), request_ids=work.request_ids.cpu(),
               lengths=work.lengths.cpu(), request_table=work.request_table.cpu(),
               slot_offsets=work.slot_offsets.cpu())
    outputs = [torch.empty((work.rows // CFG2["topk"], CFG2["topk"], work.width), dtype=torch.int16)
               for _ in planes]
    return planes, idx, outputs


def run_cpu_gather(planes, idx, outputs, width):
    from oracle.cpu_baseline import gather_planes

    gather_planes(planes, idx["positions"], idx["request_ids"], idx["lengths"], idx["request_table"],
                  idx["slot_offsets"], width, outputs)


def cpu_baseline(work: Workload, seconds: float, sample_layers: int = 1):
    """Time the torch-CPU restatement on all host threads for ~`seconds`; check parity."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    planes, idx, outputs = cpu_sample(work, sample_layers)
    run_cpu_gather(planes, idx, outputs, work.width)  # warm-up + parity sample
    parity = all(torch.equal(out, work.outputs[p].view(out.shape).view(torch.int16).cpu())
                 for p, out in enumerate(outputs))
    reps, started = 0, time.perf_counter()
    while reps < 2 or time.perf_counter() - started < seconds:
        run_cpu_gather(planes, idx, outputs, work.width)
        reps += 1
    elapsed = time.perf_counter() - started
    units = reps * work.rows * sample_layers
    return {"value": units / elapsed, "unit": "row-pairs/s", "cores": threads, "kind": "port",
            "sample": f"{sample_layers} of {work.layers} layers (K and V), all {work.rows} Top-K "
                      f"row-pairs per layer, {reps} repetitions in {elapsed:.1f} s",
            "cpu": platform.processor() or platform.machine(), "parity_with_gpu": parity}


# --------------------------------------------------------------------------- migration (config 3)

def migration_bench(work: Workload, victims_n: int = 256, reps: int = 3):
    """Config 3: demote 256 victim chunks to 2 MiB-aligned pinned staging, re-commit
    them fresh, promote the rows back to permuted slots; host-link GB/s each way."""
    from ekv_b200.host_pool import pack_rows, pack_rows_staged, pinned_buffer, unpack_rows, unpack_rows_staged

    dev = work.dist.device
    gen = torch.Generator().manual_seed(7)
    rows_per_chunk = CHUNK // work.row_bytes
    victims = torch.randperm(work.n_planes * work.plane_chunks, generator=gen)[:victims_n]
    plane_index, src, dst, stage, segments = [], [], [], [], []
    first = 0
    for v, victim in enumerate(victims.tolist()):
        plane, chunk = divmod(victim, work.plane_chunks)
        density = 0.5 + 0.5 * torch.rand((), generator=gen).item()
        occupied = torch.nonzero(torch.rand(rows_per_chunk, generator=gen) < density).flatten()
        perm = torch.randperm(rows_per_chunk, generator=gen)
        plane_index.append(torch.full((occupied.numel(),), plane, dtype=torch.int32))
        src.append(chunk * rows_per_chunk + occupied)
        dst.append(chunk * rows_per_chunk + perm[occupied])
        stage.append(v * rows_per_chunk + torch.arange(occupied.numel()))
        segments.append((first, occupied.numel(), v * CHUNK))  # victim v starts on a 2 MiB boundary
        first += occupied.numel()
    plane_index = torch.cat(plane_index).to(dev)
    src, dst, stage = torch.cat(src).to(dev), torch.cat(dst).to(dev), torch.cat(stage).to(dev)
    n_rows = src.numel()
    moved = n_rows * work.row_bytes
    planes = [p.view(work.slots, work.row_bytes // 2).view(torch.uint8).view(work.slots, work.row_bytes)
              for p in work.planes]
    host = pinned_buffer(victims_n * CHUNK)
    staging = host.view(-1, work.row_bytes)
    shadow = torch.empty((n_rows, work.row_bytes), dtype=torch.uint8, device=dev)
    dense = torch.arange(n_rows, device=dev)
    pack_rows(planes, src, shadow, plane_index=plane_index, stage_rows=dense)  # device copy for checking

    def event_time(fn):
        times = []
        for _ in range(reps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record()
            fn()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end) / 1e3)
        return min(times), statistics.median(times)

    # Dense host layout: victim v's rows follow victim v-1's (its start row is kept
    # in `segments`), so each 16 MiB ring slot crosses the link in one copy.
    dense_segments = [(0, n_rows, 0)]
    zc_d2h, _ = event_time(lambda: pack_rows(planes, src, staging, plane_index=plane_index, stage_rows=stage))
    aligned_d2h, _ = event_time(lambda: pack_rows_staged(planes, src, host, segments, plane_index=plane_index))
    d2h_best, d2h_med = event_time(lambda: pack_rows_staged(planes, src, host, dense_segments,
                                                            plane_index=plane_index))
    chunk_ids = sorted({1 + int(v) for v in victims})
    vmm = vmm_phases(work.backing, chunk_ids)
    h2d_best, h2d_med = event_time(lambda: unpack_rows_staged(planes, dst, host, dense_segments,
                                                              plane_index=plane_index))
    # The alternative layouts restore the same rows (the host image above is the
    # dense one; write the chunk-aligned image first so both promote the same bytes).
    pack_rows_staged(planes, dst, host, segments, plane_index=plane_index)
    aligned_h2d, _ = event_time(lambda: unpack_rows_staged(planes, dst, host, segments, plane_index=plane_index))
    zc_h2d, _ = event_time(lambda: unpack_rows(planes, dst, staging, plane_index=plane_index, stage_rows=stage))
    restored = torch.empty_like(shadow)
    pack_rows(planes, dst, restored, plane_index=plane_index, stage_rows=dense)
    torch.cuda.synchronize()
    exact = bool(torch.equal(restored, shadow))
    commit = commit_path_bench(work, victims, segments, planes, dst, host, plane_index, shadow, dense)
    # Copy-engine reference on the same link: one contiguous pinned <-> device copy.
    flat_host = host[:moved]
    flat_dev = torch.empty(moved, dtype=torch.uint8, device=dev)
    ce_h2d, _ = event_time(lambda: flat_dev.copy_(flat_host, non_blocking=True))
    ce_d2h, _ = event_time(lambda: flat_host.copy_(flat_dev, non_blocking=True))
    gbs = lambda seconds: moved / seconds / 1e9  # noqa: E731
    first, median = vmm["first"], vmm["median"]
    vmm_s = (median["unmap_ms"] + median["release_ms"] + median["ensure_ms"]) / 1e3
    first_s = (first["unmap_ms"] + first["release_ms"] + first["ensure_ms"]) / 1e3
    return {"victim_chunks": victims_n, "rows": n_rows, "bytes_per_direction": moved,
            "config3_end_to_end_gbs": 2 * moved / (d2h_best + vmm_s + h2d_best) / 1e9,
            "config3_end_to_end_gbs_first_round": 2 * moved / (d2h_best + first_s + h2d_best) / 1e9,
            "config3_end_to_end": "bytes moved both ways / (staged demotion + unmap + release of the victim "
                                  "chunks + commit of fresh chunks (create, map, access, zero) + staged "
                                  "promotion), with each VMM phase's median over the rounds of vmm; "
                                  "_first_round: the same with the first round's VMM calls",
            "vmm": vmm,
            "d2h_gbs": gbs(d2h_best), "h2d_gbs": gbs(h2d_best),
            "d2h_gbs_median": gbs(d2h_med), "h2d_gbs_median": gbs(h2d_med),
            "zero_copy_d2h_gbs": gbs(zc_d2h), "zero_copy_h2d_gbs": gbs(zc_h2d),
            "staged_chunk_aligned_d2h_gbs": gbs(aligned_d2h), "staged_chunk_aligned_h2d_gbs": gbs(aligned_h2d),
            "copy_engine_contiguous_d2h_gbs": gbs(ce_d2h), "copy_engine_contiguous_h2d_gbs": gbs(ce_h2d),
            "host_link_nominal_gbs": 64.0, "frac_of_nominal_d2h": gbs(d2h_best) / 64.0,
            "frac_of_nominal_h2d": gbs(h2d_best) / 64.0,
            "reclaim_ms": median["unmap_ms"] + median["release_ms"], "ensure_ms": median["ensure_ms"],
            "round_trip_bit_exact": exact, "commit_path": commit,
            "path": "staged: pack/unpack kernel into a 64 MiB device ring + copy-engine transfers on a side "
                    "stream, dense host layout (2 MiB pinned chunks, victim start rows recorded); "
                    "alternatives: per-victim 2 MiB-aligned host layout, zero-copy kernel stores/loads"}


def vmm_phases(backing, chunk_ids, singles=8, rounds=5):
    """Driver time of reclaiming and re-committing ``chunk_ids`` on a live pool, by phase.

    ``single_drop_ms``: ``singles`` chunks unmapped and released one call each (the
    latency distribution of individual drops); then ``rounds`` rounds over all victims,
    each split into ``unmap_ms`` (reclaim while spare handles are kept, so only
    cuMemUnmap runs), ``release_ms`` (cuMemRelease of the kept handles) and
    ``ensure_ms`` (cuMemCreate, cuMemMap, cuMemSetAccess, zero fill).  ``first`` is the
    first round on the pool as the run left it; ``median`` takes each phase's median
    over the rounds.  A round now and then stalls for 0.3-1 s inside the driver, at any
    position in the sequence (probed in fresh processes: the slow round was the fourth
    as often as the first), so the median is the pool's cost and ``rounds_ms`` shows
    every round's total.
    """
    out = {"single_drop_ms": [], "rounds_ms": []}
    for chunk in chunk_ids[:singles]:
        started = time.perf_counter()
        backing.reclaim({chunk}, synchronize=False)
        out["single_drop_ms"].append((time.perf_counter() - started) * 1e3)
    backing.ensure(chunk_ids[:singles])
    torch.cuda.synchronize()
    per_round = []
    for _ in range(rounds):
        backing.set_spare_chunks(len(chunk_ids))
        started = time.perf_counter()
        backing.reclaim(chunk_ids, synchronize=False)
        unmap = time.perf_counter() - started
        started = time.perf_counter()
        backing.set_spare_chunks(0)
        release = time.perf_counter() - started
        started = time.perf_counter()
        backing.ensure(chunk_ids)
        ensure = time.perf_counter() - started
        per_round.append({"unmap_ms": unmap * 1e3, "release_ms": release * 1e3, "ensure_ms": ensure * 1e3,
                          "chunks": len(chunk_ids)})
        out["rounds_ms"].append((unmap + release + ensure) * 1e3)
    out["first"] = per_round[0]
    out["median"] = {phase: statistics.median(r[phase] for r in per_round)
                     for phase in ("unmap_ms", "release_ms", "ensure_ms")}
    out["median"]["chunks"] = len(chunk_ids)
    return out


# --------------------------------------------------------------------------- lookups (config 1, R1)

REFERENCE_ROUND_TRIP = dict(bytes=503_347_200, seconds=0.1314, gbs=3.8,
                            source="results/vmm-roundtrip-shadow/results.json:699-700 (4x A100, TP4, per rank)")


def round_trip_bench(dev, reps=5, spare_chunks=0):
    """A forced demote + promote round trip through the reference's transaction API
    (prepare_demote -> commit_demote -> prepare_promote -> commit_promote,
    adaptive_sparse/migration.py:67-288) on one TP4 rank's shard: 48 layers x K,V of
    2 KV heads x 128 (512 B rows), page size 64, one request of 5120 committed tokens
    = 503 MB moved per round trip (the reference's published case moved 503,347,200 B).
    Wall time includes every sync, the chunk reclaim of the demotion and the chunk
    commit of the promotion, as the reference's figure does.  The SGLang objects are
    the test stand-in (tests/support/standin.py); rows are checked bit for bit."""
    from ekv_b200 import migration
    from tests.support.standin import install_request, migration_world

    world = migration_world(dev, layers=48, heads=2, head_dim=128, page_size=64, pages=2048, host_rows=8192,
                            spare_chunks=spare_chunks)
    try:
        c = world.coordinator
        length = 5120
        req, slots, logical = install_request(world, 1, length)
        original = [view[slots].clone() for view in world.views]
        moved = length * 2 * world.layers * world.row_bytes  # per direction
        samples = []
        metric_keys = ("ensure_ns", "reclaim_ns", "reclaim_sync_ns", "ensure_chunks", "reclaim_chunks")
        for _ in range(reps):
            before = {k: world.backing.metrics[k] for k in metric_keys}
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            prepared = migration.prepare_demote(c, req, torch.cuda.synchronize)
            released = migration.commit_demote(prepared, lambda row: None, torch.cuda.synchronize,
                                               trim_quiescent=world.tracker.trim_quiescent)
            t1 = time.perf_counter()
            promoted = migration.prepare_promote(c, req, torch.cuda.synchronize)
            migration.commit_promote(promoted, lambda row: None, torch.cuda.synchronize)
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            after = world.backing.metrics
            samples.append((t1 - t0, t2 - t1, t2 - t0, released, {k: after[k] - before[k] for k in metric_keys}))
        destination = world.pool.full_to_hisparse_device_index_mapping[logical]
        # Bit patterns: the stand-in's seeded payload includes bf16 NaN encodings.
        exact = all(bool(torch.equal(view[destination].view(torch.int16), want.view(torch.int16)))
                    for view, want in zip(world.views, original))
        demote_s, promote_s, total_s, released, vmm = min(samples, key=lambda x: x[2])
        ref = REFERENCE_ROUND_TRIP
        return {"tokens": length, "layers": world.layers, "row_bytes": world.row_bytes,
                "bytes_round_trip": 2 * moved, "demote_ms": demote_s * 1e3, "promote_ms": promote_s * 1e3,
                "round_trip_ms": total_s * 1e3, "gbs_combined": 2 * moved / total_s / 1e9,
                "round_trip_ms_median": statistics.median(x[2] for x in samples) * 1e3,
                "released_bytes_per_demotion": released, "bit_exact": exact, "spare_chunks": spare_chunks,
                "vmm": {"commit_ms": vmm["ensure_ns"] / 1e6, "reclaim_ms": vmm["reclaim_ns"] / 1e6,
                        "reclaim_sync_ms": vmm["reclaim_sync_ns"] / 1e6, "chunks_committed": vmm["ensure_chunks"],
                        "chunks_reclaimed": vmm["reclaim_chunks"]},
                "reference_published": ref, "vs_reference_published": (2 * moved / total_s / 1e9) / ref["gbs"]}
    finally:
        world.close()


def commit_path_bench(work, victims, segments, planes, dst, host, plane_index, shadow, dense, batch=32,
                      rounds=3):
    """Promotion into freshly committed chunks (config 3): the 256 victim chunks are
    reclaimed, then committed again and their rows restored from pinned host memory.

    * sequential: commit every chunk, then restore every row (the reference's order:
      the allocator maps, then load_to_device_per_layer copies);
    * pipelined: commit 32 victims' chunks, launch their rows' restore (asynchronous:
      copy engine + unpack kernel), commit the next 32 while it runs;
    * *_spare_handles: the same after a reclaim that kept the physical handles (no
      cuMemRelease / cuMemCreate).
    Wall time from the first commit to the restored rows on the device, min and median
    of 3 interleaved rounds; every run is checked bit for bit against the rows before
    demotion."""
    from ekv_b200.host_pool import pack_rows, pack_rows_staged, unpack_rows_staged

    chunk_of = [1 + int(v) for v in victims]
    firsts = [first for first, _, _ in segments] + [dst.numel()]
    row_bytes = work.row_bytes
    # The dense host image of the restored rows (victim v's rows from row firsts[v]).
    pack_rows_staged(planes, dst, host, [(0, dst.numel(), 0)], plane_index=plane_index)

    def restore(a, b):
        first, last = firsts[a], firsts[b]
        unpack_rows_staged(planes, dst[first:last], host, [(0, last - first, first * row_bytes)],
                           plane_index=plane_index[first:last])

    def exact():
        restored = torch.empty_like(shadow)
        pack_rows(planes, dst, restored, plane_index=plane_index, stage_rows=dense)
        torch.cuda.synchronize()
        return bool(torch.equal(restored, shadow))

    def run(pipelined):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if pipelined:
            for a in range(0, len(chunk_of), batch):
                b = min(len(chunk_of), a + batch)
                work.backing.ensure(chunk_of[a:b])
                restore(a, b)
        else:
            work.backing.ensure(chunk_of)
            restore(0, len(chunk_of))
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e3

    variants = (("sequential", False, 0), ("pipelined", True, 0),
                ("sequential_spare_handles", False, len(chunk_of)),
                ("pipelined_spare_handles", True, len(chunk_of)))
    samples = {name: {"reclaim_ms": [], "commit_and_restore_ms": [], "bit_exact": True} for name, _, _ in variants}
    for _ in range(rounds):  # interleaved: the driver's cost drifts between calls
        for name, pipelined, spare in variants:
            work.backing.set_spare_chunks(spare)
            t0 = time.perf_counter()
            work.backing.reclaim(chunk_of)
            samples[name]["reclaim_ms"].append((time.perf_counter() - t0) * 1e3)
            samples[name]["commit_and_restore_ms"].append(run(pipelined))
            samples[name]["bit_exact"] &= exact()
    work.backing.set_spare_chunks(0)
    out = {name: {"reclaim_ms_min": min(v["reclaim_ms"]), "reclaim_ms_median": statistics.median(v["reclaim_ms"]),
                  "commit_and_restore_ms_min": min(v["commit_and_restore_ms"]),
                  "commit_and_restore_ms_median": statistics.median(v["commit_and_restore_ms"]),
                  "bit_exact": v["bit_exact"]} for name, v in samples.items()}
    restore_only = []
    for _ in range(2):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        restore(0, len(chunk_of))
        torch.cuda.synchronize()
        restore_only.append((time.perf_counter() - t0) * 1e3)
    out["restore_only_ms"] = min(restore_only)
    out["chunks"] = len(chunk_of)
    return out


def lookup_bench(dist: Dist, rounds: int = 20, calls: int = 100):
    """R2 at config 1 and R1 at the reference's own microbenchmark shape.

    Methodology of tests/bench_resident_lookup.py:94-107: CUDA events around
    `calls` back-to-back calls per round, p50 over rounds (launch-bound sizes).
    """
    from ekv_b200.resident_lookup import lookup_slots, resolve_resident

    dev = dist.device
    gen = torch.Generator().manual_seed(1)
    batch, ctx, resident, k = 32, 16384, 2048, 512
    res_map = torch.full((batch, ctx), -1, dtype=torch.int32)
    topk = torch.empty((batch, k), dtype=torch.int32)
    for b in range(batch):
        tokens = torch.randperm(ctx, generator=gen)
        res_map[b, tokens[:resident]] = torch.randperm(resident, generator=gen).to(torch.int32)
        pick = torch.cat([tokens[:resident][torch.randperm(resident, generator=gen)[:384]],
                          tokens[resident:][torch.randperm(ctx - resident, generator=gen)[:128]]])
        topk[b] = pick[torch.randperm(k, generator=gen)].to(torch.int32)
    res_map, topk = res_map.to(dev), topk.to(dev)
    outs = lookup_slots(res_map, topk)

    def p50(fn):
        for _ in range(calls):
            fn()
        torch.cuda.synchronize()
        samples = []
        for _ in range(rounds):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(calls):
                fn()
            end.record()
            end.synchronize()
            samples.append(start.elapsed_time(end) * 1e3 / calls)
        return statistics.median(samples)

    def graph_us(fn):
        """Device time per call: `calls` calls captured in one CUDA graph, replayed."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(calls):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        samples = []
        for _ in range(rounds):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            graph.replay()
            end.record()
            end.synchronize()
            samples.append(start.elapsed_time(end) * 1e3 / calls)
        del graph
        return statistics.median(samples)

    def cfg1_call():
        lookup_slots(res_map, topk, slots=outs[0], miss=outs[1], miss_list=outs[2], miss_count=outs[3])

    cfg1_us = p50(cfg1_call)
    cfg1_graph_us = graph_us(cfg1_call)
    # tests/bench_resident_lookup.py:61-66 shapes at batch 4.
    rb = 4
    selected = torch.arange(rb, device=dev)
    rows = selected.flip(0)
    lengths = torch.full((rb,), 8192, dtype=torch.int32, device=dev)
    table = torch.arange(rb * 8192, device=dev).reshape(rb, 8192) + 1
    mapping = torch.arange(rb * 8192 + 1, device=dev) * 3 + 5
    blocks = (torch.arange(16, device=dev) * 4).int().expand(1, rb, 16).contiguous()
    result = torch.empty((1, rb, 2048), dtype=torch.int32, device=dev)
    def resolve_call():
        resolve_resident(blocks, table, mapping, rows, lengths, selected, result, 128)

    resolve_us = p50(resolve_call)
    resolve_graph_us = graph_us(resolve_call)
    shared = shared_prefix_bench(dev, p50, graph_us)
    gather_api = gather_api_bench(dev, p50, graph_us)
    expected = torch.tensor([[((rb - 1 - r) * 8192 + blk * 512 + off + 1) * 3 + 5
                              for blk in range(16) for off in range(128)] for r in range(rb)],
                            dtype=torch.int32, device=dev)
    return {"config1_lookup_slots_us": cfg1_us, "config1_lookups_per_s": batch * k / (cfg1_us * 1e-6),
            "config1_device_us": cfg1_graph_us,
            "config1_device_lookups_per_s": batch * k / (cfg1_graph_us * 1e-6),
            "config1_misses": int(outs[3].sum()),
            "resolve_resident_batch4_us": resolve_us,
            "resolve_resident_batch4_lookups_per_s": rb * 2048 / (resolve_us * 1e-6),
            "resolve_resident_batch4_device_us": resolve_graph_us,
            "resolve_resident_published_a100_triton_us": 30.08,
            "resolve_resident_correct": bool(torch.equal(result[0], expected)),
            "shared_prefix": shared, "gather_rows_api": gather_api,
            "timing": "p50 of per-call CUDA-event time, 100 calls per round (reference methodology, "
                      "includes host dispatch); *_device_us: the same 100 calls replayed from one CUDA graph"}


def gather_api_bench(dev, p50, graph_us):
    """The reference's single-plane ``gather_rows`` call (indirect addressing) at one
    layer's K plane of config 2 under TP8 (64 requests x 2048 rows of 256 B): time per
    call through the public API (compiled binding, and the ctypes path with the binding
    hidden) against the kernel's device time (CUDA graph)."""
    from ekv_b200 import sparse_read
    from ekv_b200.virtual_layout import VirtualKVLayout

    batch, rows, width = 64, 2048, 128
    layout = VirtualKVLayout(batch, rows, width, itemsize=2, chunk_bytes=CHUNK)
    gen = torch.Generator(device=dev).manual_seed(12)
    raw = torch.empty(layout.capacity_bytes // 2, dtype=torch.bfloat16, device=dev)
    torch.randn(raw.shape, generator=gen, dtype=torch.bfloat16, device=dev, out=raw)
    slots = (layout.capacity_bytes // 2 - layout.chunk_bytes // 2) // width
    positions = torch.stack([torch.randperm(rows, generator=gen, device=dev) for _ in range(batch)])
    request_ids = torch.arange(batch, device=dev)
    lengths = torch.full((batch,), rows, dtype=torch.int64, device=dev)
    table = torch.arange(batch * rows, device=dev).view(batch, rows)
    offsets = layout.chunk_bytes // 2 + torch.randperm(slots, generator=gen, device=dev)[:batch * rows] * width
    out = torch.empty((batch, rows, width), dtype=torch.bfloat16, device=dev)

    def call():
        sparse_read.gather_rows(raw, positions, request_ids, lengths, table, offsets, out, layout, indirect=True)

    def host_us(calls=50, rounds=10):
        """Host time per call (the launches queue up; the device is not waited for)."""
        samples = []
        for _ in range(rounds):
            torch.cuda.synchronize()
            start = time.perf_counter()
            for _ in range(calls):
                call()
            samples.append((time.perf_counter() - start) * 1e6 / calls)
        torch.cuda.synchronize()
        return statistics.median(samples)

    api_us, api_host_us = p50(call), host_us()
    device_us = graph_us(call)
    binding = sparse_read.torch_binding
    sparse_read.torch_binding = lambda: None
    try:
        ctypes_us, ctypes_host_us = p50(call), host_us()
    finally:
        sparse_read.torch_binding = binding
    return {"api_us": api_us, "host_us": api_host_us, "ctypes_api_us": ctypes_us, "ctypes_host_us": ctypes_host_us,
            "device_us": device_us, "binding": binding() is not None, "rows": batch * rows,
            "row_bytes": width * 2,
            "timing": "api_us: p50 CUDA-event time per call of 100 back-to-back calls (the slower of host "
                      "and device); host_us: host time per call; device_us: CUDA-graph replay"}


def shared_prefix_bench(dev, p50, graph_us):
    """Shared-prefix donor-slot resolution at the config-5 shape: 128 consumers x
    2048 Top-K blocks of one token, 65536-token request table, 1 Mi-slot mapping.
    Public API per call (includes the host -> device copy of the per-request
    lists), device time of the kernel alone (CUDA graph), and the reference's torch
    expression on the host cores for the same inputs."""
    from ekv_b200 import shared_prefix as sp
    from oracle.cpu_baseline import torch_shared_resolver

    requests, topk, ctx, slots = 128, 2048, 65536, 1 << 20
    gen = torch.Generator().manual_seed(8)
    table = torch.randint(0, slots, (requests, ctx), generator=gen, dtype=torch.int32)
    mapping = torch.randint(0, 1 << 22, (slots,), generator=gen, dtype=torch.int64)
    blocks = torch.randint(0, ctx, (requests, topk), generator=gen, dtype=torch.int32)
    rows = torch.randint(0, requests, (requests,), generator=gen)
    prefixes = torch.randint(0, ctx, (requests,), generator=gen)
    lengths = torch.full((requests,), ctx, dtype=torch.int64)
    d_table, d_mapping, d_blocks, d_lengths = (t.to(dev) for t in (table, mapping, blocks, lengths))
    rows_l, prefixes_l = rows.tolist(), prefixes.tolist()

    def api_call():
        return sp.resolve_shared_block_locations_batched(
            d_blocks, source_rows=rows_l, seq_len=d_lengths, shared_tokens=prefixes_l, block_size=1,
            request_table=d_table, device_mapping=d_mapping)

    valid, physical = api_call()
    meta = torch.cat([rows, prefixes]).to(dev)

    def kernel_call():
        sp._launch(d_blocks, requests, topk, d_blocks.stride(0), d_blocks.stride(1), meta[:requests], 0,
                   meta[requests:], 0, d_lengths, 1, 1, d_table, d_mapping, valid, physical, None, False)

    api_us = p50(api_call)
    device_us = graph_us(kernel_call)
    want_valid, want_physical = torch_shared_resolver(blocks, rows, prefixes, lengths, 1, table, mapping)
    correct = bool(torch.equal(valid.cpu(), want_valid)) and bool(torch.equal(physical.cpu(), want_physical))
    torch.set_num_threads(os.cpu_count() or 1)
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        torch_shared_resolver(blocks, rows, prefixes, lengths, 1, table, mapping)
    cpu_us = (time.perf_counter() - t0) / reps * 1e6
    return {"shape": "128 x 2048 blocks, block_size 1, table 128 x 65536 int32, mapping 1Mi int64",
            "api_us": api_us, "device_us": device_us, "blocks_per_s_device": requests * topk / (device_us * 1e-6),
            "reference_torch_cpu_us": cpu_us, "cpu_threads": torch.get_num_threads(), "correct": correct,
            "shared_blocks": int(want_valid.sum())}


def shadow_bench(dist: Dist, reps: int = 10):
    """Logical-shadow check of one decode step at the config-2 batch: 64 requests x
    2048 Top-K tokens, 2 KiB K and V rows, a 262144-slot shadow and cache (1 GiB
    each), every token checked.  Algorithmic bytes per checked token: K and V row
    of the cache and of the shadow (4 x 2048 B) + 17 B of indices, flags and
    output.  The reference's torch body of the same check runs on the same GPU
    beside it."""
    from ekv_b200.logical_shadow import LogicalShadow
    from oracle.cpu_baseline import torch_shadow_check

    dev = dist.device
    batch, topk, ctx, heads, dim, capacity = 64, 2048, 16384, 8 // dist.world or 1, 128, 262144
    gen = torch.Generator(device=dev).manual_seed(5)
    shadow = LogicalShadow(capacity, dev)
    key = torch.randn((capacity, heads, dim), device=dev, generator=gen).to(torch.bfloat16)
    value = torch.randn((capacity, heads, dim), device=dev, generator=gen).to(torch.bfloat16)
    shadow.write(0, torch.arange(capacity, device=dev), key, value, (None, None))
    phys_of = torch.randperm(capacity, device=dev, generator=gen)
    k_cache, v_cache = torch.empty_like(key), torch.empty_like(value)
    k_cache[phys_of], v_cache[phys_of] = key, value
    del key, value
    table = torch.randint(1, capacity, (batch, ctx), device=dev, generator=gen, dtype=torch.int32)
    lengths = torch.full((batch,), ctx, device=dev, dtype=torch.int64)
    rows = torch.arange(batch, device=dev)
    blocks = torch.argsort(torch.rand((batch, ctx), device=dev, generator=gen), dim=1)[:, :topk]
    blocks = blocks.to(torch.int32)[None].contiguous()
    physical = phys_of[table[rows[:, None], blocks[0].long()].long()].to(torch.int32)[None].contiguous()
    args = (k_cache, v_cache, table, lengths, rows, 1, blocks, physical, None, 1)

    def ours():
        return shadow.check(0, *args)

    k_shadow, v_shadow, initialized = shadow.layers[0]

    def reference():
        return torch_shadow_check(k_shadow, v_shadow, initialized, *args)

    def per_call_ms(fn):
        for _ in range(2):
            fn()
        stream = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(reps):
            fn()
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / reps

    shadow.counts.zero_()
    ours_ms = per_call_ms(ours)
    counts = shadow.counts.tolist()
    ref_ms = per_call_ms(reference)
    ref_counts, ref_clean, ref_phys = reference()
    clean, phys_out = ours()
    calls = counts[5]
    agree = (bool(torch.equal(ref_clean, clean)) and bool(torch.equal(ref_phys, phys_out))
             and calls > 0 and ref_counts.tolist()[0] == counts[0] / calls)
    row_bytes = heads * dim * 2
    per_token = 4 * row_bytes + 17
    achieved = batch * topk * per_token / (ours_ms * 1e-3) / 1e9
    peak, source = measured_hbm_peak()
    del k_cache, v_cache, table, physical, blocks, args, ref_counts, ref_clean, ref_phys
    result = {"shape": f"{batch} x {topk} tokens, {row_bytes} B rows, {capacity}-slot shadow and cache",
              "check_ms": ours_ms, "tokens_per_s": batch * topk / (ours_ms * 1e-3),
              "achieved_gbs": achieved, "peak_gbs": peak, "frac": achieved / peak, "peak_source": source,
              "reference_torch_same_gpu_ms": ref_ms, "speedup_vs_reference_torch": ref_ms / ours_ms,
              "checked_per_call": counts[0] / calls if calls else 0, "mismatched": counts[4],
              "agrees_with_reference_torch": agree}
    result["migration_check"] = shadow_complete_bench(shadow, dev, heads, dim, capacity, reps)
    return result


def shadow_complete_bench(shadow, dev, heads, dim, capacity, reps, layers=4, pairs=196608):
    """check_complete after a config-3-sized migration (196608 slot pairs) over 4
    layers, each with its own shadow and pool buffers (1 GiB each): per pair and
    layer the pool's K and V rows and the shadow's (4 x 2 KiB) + 16 B of slot ids."""
    from types import SimpleNamespace

    gen = torch.Generator(device=dev).manual_seed(6)
    page = 1
    key0, value0, init0 = shadow.layers[0]
    for layer in range(1, layers):  # the same recorded writes, in each layer's own buffers
        shadow.layers[layer] = (key0.clone(), value0.clone(), init0.clone())
    logical = torch.randperm(capacity - page, device=dev, generator=gen)[:pairs] + page
    physical = torch.randperm(capacity, device=dev, generator=gen)[:pairs] + page
    pool_k, pool_v = [], []
    for layer in range(layers):
        pk = torch.empty((capacity + page, heads, dim), device=dev, dtype=torch.bfloat16)
        pv = torch.empty_like(pk)
        pk[physical], pv[physical] = key0[logical], value0[logical]
        pool_k.append(pk)
        pool_v.append(pv)
    pool = SimpleNamespace(page_size=page, size=capacity, adaptive_vmm=SimpleNamespace(pages=set(range(capacity + 1))),
                           start_layer=0, end_layer=layers, get_key_buffer=lambda layer: pool_k[layer],
                           get_value_buffer=lambda layer: pool_v[layer])
    shadow.check_complete(pool, logical, physical, "bench")
    torch.cuda.synchronize()
    api = []
    for _ in range(reps):
        t0 = time.perf_counter()
        shadow.check_complete(pool, logical, physical, "bench")  # ends with the counters' host read
        api.append((time.perf_counter() - t0) * 1e3)
    live = torch.ones(capacity // page + 1, dtype=torch.uint8, device=dev)
    counts = torch.zeros(4, dtype=torch.int64, device=dev)
    layer_ids = list(range(layers))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        shadow.launch_complete(pool, layer_ids, logical, physical, live, counts)
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end) / reps
    row_bytes = heads * dim * 2
    moved = pairs * layers * (4 * row_bytes + 16)
    peak, _ = measured_hbm_peak()
    checked = shadow.migration_counts["migration_checked_tokens"]
    return {"pairs": pairs, "layers": layers, "kernel_ms": ms, "achieved_gbs": moved / (ms * 1e-3) / 1e9,
            "frac": moved / (ms * 1e-3) / 1e9 / peak, "api_ms_p50": statistics.median(api),
            "checked_all": checked == pairs * layers * (reps + 1) and int(counts[0]) == pairs * layers * reps,
            "mismatched": shadow.migration_counts["migration_mismatched_tokens"] + int(counts[3]),
            "timing": "kernel_ms: CUDA events around the launches alone; api_ms_p50: wall time of the public "
                      "call (live-page mask from the page set, launch, counter read)"}



# --------------------------------------------------------------------------- bitmap (config 4 geometry)

def freeable_world(dist: Dist, shard: int = 0):
    """Config-4 geometry of the freeable-bitmap step: 48 layers x K,V planes over 4096
    chunks, rows of 2048 / TP bytes, 32 requests owning the pages (page size 1), request
    0 the demotion candidate; each rank leaves a few rank-specific chunks unmapped so
    the cross-rank AND is not trivial.  Returns the projection, refs, mapped bitmap,
    candidate pages and the expected joint chunk set."""
    from ekv_b200.releasable import ChunkProjection, chunks_to_bitmap

    dev = dist.device
    layers, n_chunks = 48, 4096
    row_bytes = 2048 // (shard or dist.world)
    planes_n = 2 * layers
    per_plane = n_chunks // planes_n
    slots = per_plane * CHUNK // row_bytes
    planes = [(p * per_plane, row_bytes) for p in range(planes_n)]
    # Every page (slot, page size 1) belongs to one of 32 requests; request 0
    # owns the first eighth of the slots, so its pages hold whole chunks.
    gen = torch.Generator().manual_seed(11)
    owner = torch.randint(1, 32, (slots,), generator=gen)
    owner[: slots // 8] = 0
    projection = ChunkProjection(planes, 1, CHUNK, n_chunks, dev)
    refs = projection.counts(torch.arange(slots, device=dev))
    unmapped = {r: {(r * 37 + 5 * i) % n_chunks for i in range(8)} for r in range(dist.world)}
    mapped = chunks_to_bitmap(set(range(n_chunks)) - unmapped[dist.rank], n_chunks, dev)
    candidate = torch.nonzero(owner == 0).flatten().to(dev)
    return projection, refs, mapped, candidate, unmapped, n_chunks, planes_n


def bitmap_bench(dist: Dist, reps: int = 50, shard: int = 0):
    from ekv_b200.releasable import bitmap_to_chunks, combine_freeable, freeable_bitmap

    dev = dist.device
    projection, refs, mapped, candidate, unmapped, n_chunks, planes_n = freeable_world(dist, shard)

    def build():
        return freeable_bitmap(projection.counts(candidate), refs, mapped)

    local = build()
    joint = combine_freeable(local)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        build()
    end.record(stream)
    torch.cuda.synchronize()
    build_ms = start.elapsed_time(end) / reps
    # Device time of the build alone: `reps` builds into fixed buffers captured in
    # one CUDA graph and replayed (the loop above is bound by host dispatch).
    counts_buf = projection.counts(candidate)
    bits_buf = freeable_bitmap(counts_buf, refs, mapped)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        freeable_bitmap(projection.counts(candidate, out=counts_buf), refs, mapped, out=bits_buf)
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            freeable_bitmap(projection.counts(candidate, out=counts_buf), refs, mapped, out=bits_buf)
    graph.replay()
    torch.cuda.synchronize()
    start.record(stream)
    graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    build_device_ms = start.elapsed_time(end) / reps
    del graph
    dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        combine_freeable(local)
    end.record(stream)
    torch.cuda.synchronize()
    combine_ms = dist.max(start.elapsed_time(end) / reps)
    fused = {}
    if dist.world > 1:
        # One kernel builds this rank's bitmap, publishes it in symmetric memory and ANDs
        # the peers' words over NVLink; timed with the counts kernel in front, like
        # build + combine above.
        from ekv_b200.releasable import PeerFreeableCombiner

        try:
            combiner = PeerFreeableCombiner(n_chunks, dev)
        except Exception as exc:  # symmetric memory unavailable: report, keep the bench line
            combiner, fused = None, {"fused_unavailable": f"{type(exc).__name__}: {exc}"[:200]}
        if combiner is not None:
            fused_joint = combiner.combine(projection.counts(candidate), refs, mapped)
            dist.barrier()
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(reps):
                combiner.combine(projection.counts(candidate), refs, mapped, out=fused_joint)
            end.record(stream)
            torch.cuda.synchronize()
            fused_ms = dist.max(start.elapsed_time(end) / reps)
            fused = {"fused_build_combine_us": fused_ms * 1e3,
                     "unfused_build_combine_us": (build_ms + combine_ms) * 1e3,
                     "fused_matches_nccl": bool(torch.equal(fused_joint, joint)) and not combiner.failed()}
            dist.barrier()
            del combiner
    local_set = bitmap_to_chunks(local)
    expected_joint = set(local_set)
    for r in range(dist.world):
        expected_joint -= unmapped[r]
    return {"chunks": n_chunks, "words": n_chunks // 64, "ranks": dist.world,
            "freeable_local": len(local_set), "freeable_joint": len(bitmap_to_chunks(joint)),
            "joint_matches_intersection": bitmap_to_chunks(joint) == expected_joint,
            "build_us": build_ms * 1e3, "build_device_us": build_device_ms * 1e3,
            "pages": int(candidate.numel()), "planes": planes_n, "combine_us": combine_ms * 1e3,
            "combine": "NCCL all_gather_into_tensor + AND kernel" if dist.world > 1 else "single rank",
            **fused}


# --------------------------------------------------------------------------- arms

def run_ours(args, dist: Dist):
    from ekv_b200._lib import torch_binding
    from ekv_b200.sparse_read import gather_rows_planes

    work = Workload(dist, args.layers or CFG2["layers"], args.tp_shard)
    gather = work.plane_gather()
    with ClockSampler(dist.local_rank) as clocks:
        ms = timed(gather, args.steps, args.warmup, dist)
    ms_per_step = ms / args.steps
    value = work.units / (ms_per_step / 1e3)
    peak, peak_source = measured_hbm_peak()
    bytes_per_launch = work.units * algorithmic_bytes_per_row_pair(work.row_bytes)
    achieved = bytes_per_launch / (ms_per_step / 1e3) / 1e9
    rank_achieved = achieved  # per-GPU: every rank moves its own head shard
    traffic = traffic_per_launch(work.units, work.row_bytes)

    result = {
        "metric": METRIC, "value": value, "unit": "row-pairs/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 pool, seeded Top-K slots)",
        "config": {"workload": f"config 2: sparse Top-K KV gather, {work.layers} layers x K,V, "
                               f"pool [262144, 8, 128] bf16 per plane (VMM-backed), 64 requests x 2048 "
                               f"Top-K, heads sharded {work.heads}/rank",
                   "layers": work.layers, "requests": CFG2["requests"], "topk": CFG2["topk"],
                   "slots": CFG2["slots"], "kv_heads_per_rank": work.heads, "row_bytes": work.row_bytes,
                   "parallelism": f"tp{dist.world} (KV-head sharding, no data-path collective)",
                   "l2": f"no flush: each step moves {bytes_per_launch / 1e9:.1f} GB per GPU (> 126 MB L2)"},
        "hbm_gbs_per_gpu": achieved,
        "roofline": {"bound": "hbm", "achieved": rank_achieved, "peak": peak, "unit": "GB/s",
                     "frac": rank_achieved / peak, "traffic": traffic, "peak_source": peak_source,
                     "kernel": "gather_kernel (ekv_gather_rows_planes)",
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "frac_of_nominal_8tbs": rank_achieved / 8000.0},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "vmm_map_seconds": work.map_seconds,
    }

    if not args.skip_e2e:
        # End to end through the public API: every step's Top-K positions cross the host
        # link from pinned memory, gather_rows_planes runs (pointer tables rebuilt per
        # call) and one gathered row is read back.  The positions are double-buffered:
        # step t+1's copy runs on a second stream while step t gathers, as a serving loop
        # that receives its Top-K from the host would overlap them.
        dev = dist.device
        pos_host = work.positions.cpu().pin_memory()
        result_host = torch.empty(work.outputs[0][0, 0].shape, dtype=torch.bfloat16).pin_memory()
        planes = [p.view(work.slots, work.width) for p in work.planes]
        outs = [o.view(o.shape[0], o.shape[1], work.width) for o in work.outputs]
        main = torch.cuda.current_stream(dev)
        copy_stream = torch.cuda.Stream(dev)
        pos_dev = [work.positions, torch.empty_like(work.positions)]
        landed = [torch.cuda.Event(), torch.cuda.Event()]    # buffer i holds its step's positions
        released = [torch.cuda.Event(), torch.cuda.Event()]  # the gather reading buffer i is done
        for event in released:
            event.record(main)
        e2e_state = {"step": 0}

        def load(i):
            copy_stream.wait_event(released[i])
            with torch.cuda.stream(copy_stream):
                pos_dev[i].copy_(pos_host, non_blocking=True)
            landed[i].record(copy_stream)

        load(0)

        def e2e_step():
            i = e2e_state["step"] % 2
            e2e_state["step"] += 1
            load(1 - i)  # the next step's positions cross the link during this step's gather
            main.wait_event(landed[i])
            gather_rows_planes(planes, pos_dev[i], work.request_ids, work.lengths, work.request_table,
                               work.slot_offsets, outs, work.layout, indirect=True)
            released[i].record(main)
            result_host.copy_(work.outputs[0][0, 0], non_blocking=True)

        e2e_steps = max(3, args.steps // 2)
        ms_e2e = timed(e2e_step, e2e_steps, max(3, args.warmup), dist)
        result["e2e"] = {"value": work.units / (ms_e2e / e2e_steps / 1e3), "unit": "row-pairs/s",
                         "h2d_bytes_per_step": pos_host.numel() * pos_host.element_size(),
                         "d2h_bytes_per_step": result_host.numel() * result_host.element_size(),
                         "steps": e2e_steps, "ms_per_step": ms_e2e / e2e_steps,
                         "overlap": "step t+1's positions copied H2D on a second stream during step t's "
                                    "gather (double-buffered); one copy per step inside the timed region",
                         "api": "ekv_b200.sparse_read.gather_rows_planes ("
                                + ("compiled binding" if torch_binding() is not None else "ctypes")
                                + " -> ekv_gather_rows_planes)"}
        result["gpu_launches"] = args.steps  # the e2e loop is timed separately

    if not args.skip_legs:
        result["bitmap"] = bitmap_bench(dist)
        result["lookup"] = lookup_bench(dist)
        result["shadow"] = shadow_bench(dist)

    if dist.rank == 0 and dist.world == 1 and not args.skip_cpu:
        result["cpu_baseline"] = cpu_baseline(work, args.cpu_seconds)
    if dist.world == 1 and not args.skip_migration:
        result["migration"] = migration_bench(work)
        result["migration"]["round_trip"] = round_trip_bench(dist.device)
        result["migration"]["round_trip_spare_handles"] = round_trip_bench(dist.device, spare_chunks=256)
    work.close()
    return result


def run_default(args, dist: Dist):
    """The driver's default line: config 2 (``run_ours``), then -- with the config-2 pool
    released -- config 4, BASELINE.json's multi-GPU configuration, as the ``config4``
    object (every rank takes part), and on a single GPU config 5's multi-step decode as
    the ``config5`` object."""
    result = run_ours(args, dist)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if not args.skip_config4:
        config4 = config4_leg(args, dist, args.steps, args.warmup)
        result["config4"] = {key: value for key, value in config4.items()
                             if key not in ("metric", "higher_is_better", "vs_baseline", "dtype", "n_gpus")}
    if dist.world == 1 and not args.skip_config5:
        # Config 5's 64 decode steps on this GPU (24 layers without head sharding), after
        # config 4's buffers are released.
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        config5 = config5_leg(args, dist, CFG5["steps"])
        result["config5"] = {key: value for key, value in config5.items()
                             if key not in ("metric", "higher_is_better", "vs_baseline", "dtype", "n_gpus")}
    return result


CFG4 = dict(layers=48, kv_heads=8, head_dim=128, requests=32, context=131072, hot=4096, topk=2048,
            hit_fraction=0.9)
# The two config-4 step forms that hold when layer i's Top-K is known only after layer
# i-1; the reported one is timed with the combine variants too.
CFG4_FORMS = {
    "fused": "each layer's lookup and mapped K,V gather in ONE launch (ekv_lookup_gather_planes: the slot "
             "read once from the residency map, slots and miss mask written beside the rows), back to back "
             "on the step's stream, each marked disjoint from the layers before it (EKV_GATHER_DISJOINT: a "
             "one-block-per-SM grid that copies while the previous layer drains and waits for it only "
             "before completing), and layer i's miss-list compaction from the mask (ekv_compact_misses) on "
             "a second stream beside layer i+1 (LayerPipeline)",
    "concurrent": "the mapped K,V gathers (slot read from the residency map) back to back on the step's "
                  "stream, each layer's lookup (slots, miss mask, miss list) forked onto a second stream at "
                  "the start of its layer and joined at the end of the step (LayerPipeline wait=False); the "
                  "map is read twice per layer",
}
CFG4_REPORTED = "fused"


def config4_leg(args, dist: Dist, steps: int, warmup: int):
    """Config 4: TP-sharded sparse residency.  One decode step = for each of 48 layers a
    hot-slot lookup (R2) of that layer's Top-K and the gather of its K and V rows from
    the layer's fixed-position hot pool (misses read as zero rows) into the layer's own
    output buffers; then this rank's freeable bitmap over the config-4 chunk geometry
    (counts + bitmap kernels) and its AND-combine across the ranks (NCCL all-gather +
    AND kernel) -- the combine that replaces the reference's pickled all_gather_object
    and rank_demotions intersection (scheduler_budget.py:1447-1452,
    runtime_value.py:167-214).  The layers' launches are replayed from one CUDA
    graph; the bitmap build runs eagerly on a second stream beside them and the
    exchange + AND after them, inside the timed step (build and exchange after the
    layers, and both beside them, are timed too).  Reported: CFG4_REPORTED, the fused
    form (each layer's lookup and mapped gather in one launch, its miss list compacted
    beside the next layer), which holds when layer i's Top-K is known only after layer
    i-1; timed beside it: the concurrent form (each layer's lookup beside its mapped
    gather), the plain layer order (lookup, then the direct gather of its slots), and
    two forms that need every layer's Top-K up front -- the pipelined order (layer i's
    gather beside layer i+1's lookup) and the multi-layer form (one lookup launch over
    all layers, then one ekv_gather_layers launch)."""
    import numpy as np

    from ekv_b200.pipeline import LayerPipeline
    from ekv_b200.releasable import bitmap_to_chunks, combine_freeable, freeable_bitmap
    from ekv_b200.resident_lookup import LookupPlan
    from ekv_b200.sparse_read import LayerGather, LookupGather, PlaneGather
    from ekv_b200.virtual_layout import VirtualKVLayout
    from oracle import gather as og
    from oracle import lookup as ol

    c = CFG4
    dev = dist.device
    shard = args.tp_shard or dist.world
    heads = c["kv_heads"] // shard
    width = heads * c["head_dim"]
    row_bytes = width * 2
    layers, reqs, ctx, hot, k = args.layers or c["layers"], c["requests"], c["context"], c["hot"], c["topk"]
    layout = VirtualKVLayout(reqs, hot, width, chunk_bytes=CHUNK)
    plane_elems = layout.capacity_bytes // 2
    gen = torch.Generator(device=dev).manual_seed(4)
    n_hits = int(k * c["hit_fraction"])
    # Every layer's residency map and Top-K are slices of one stacked tensor, so the
    # multi-layer form can look all layers up in one launch over layers x requests rows.
    maps_all = torch.full((layers, reqs, ctx), -1, dtype=torch.int32, device=dev)
    topks_all = torch.empty((layers, reqs, k), dtype=torch.int32, device=dev)
    maps, topks, planes, outs = [], [], [], []
    for layer in range(layers):
        res_map = maps_all[layer]
        topk = topks_all[layer]
        for r in range(reqs):
            perm = torch.randperm(ctx, generator=gen, device=dev)
            res_map[r, perm[:hot]] = torch.randperm(hot, generator=gen, device=dev).to(torch.int32)
            pick = torch.cat([perm[:n_hits], perm[hot:hot + k - n_hits]])
            topk[r] = pick[torch.randperm(k, generator=gen, device=dev)].to(torch.int32)
        maps.append(res_map)
        topks.append(topk)
        for _ in range(2):
            plane = torch.empty(plane_elems, dtype=torch.bfloat16, device=dev)
            torch.randn(plane.shape, generator=gen, dtype=torch.bfloat16, device=dev, out=plane)
            planes.append(plane)
            # Each layer gathers into its own K / V buffers, so the written rows reach
            # DRAM instead of being overwritten in L2 by the next layer.
            outs.append(torch.empty((reqs, k, width), dtype=torch.bfloat16, device=dev))
    req_ids = torch.arange(reqs, device=dev)
    lengths = torch.full((reqs,), hot, dtype=torch.int64, device=dev)
    lookups, gathers = [], []
    for layer in range(layers):
        plan = LookupPlan(maps[layer], topks[layer])
        lookups.append(plan)
        gathers.append(PlaneGather(planes[2 * layer:2 * layer + 2], plan.slots, req_ids, lengths, None, None,
                                   outs[2 * layer:2 * layer + 2], layout, indirect=False))
    # Mapped gathers read each token's slot from the residency map themselves, so they
    # need none of the lookup's output and run beside it (slots and miss list are still
    # produced for the swap-in); same rows as the direct gather of the lookup's slots.
    # The kernel before each one on the step's stream is the previous layer's gather,
    # which writes only K/V outputs: the index inputs are ready, so every gather walks
    # its first index chain while the previous one drains.
    ctx_lengths = torch.full((reqs,), ctx, dtype=torch.int64, device=dev)
    mapped = [PlaneGather(planes[2 * layer:2 * layer + 2], topks[layer], req_ids, ctx_lengths, maps[layer], None,
                          outs[2 * layer:2 * layer + 2], layout, indirect=False, mapped=True, indices_ready=True)
              for layer in range(layers)]
    pipelines = {"concurrent": LayerPipeline(lookups, mapped, dev, wait=False),
                 "pipelined": LayerPipeline(lookups, gathers, dev)}
    # Fused: each layer's lookup and mapped gather in ONE launch (the map read once),
    # back to back on the step's stream, and the miss-list compaction of layer i from
    # the miss mask on a second stream beside layer i+1; valid for per-layer Top-K.
    # The layers' launches touch disjoint memory, so each is marked disjoint from the
    # ones before it: it copies while they drain and waits for them only at its end.
    fused = [LookupGather(planes[2 * layer:2 * layer + 2], maps[layer], topks[layer], req_ids, ctx_lengths,
                          outs[2 * layer:2 * layer + 2], layout, indices_ready=True, disjoint=True)
             for layer in range(layers)]
    pipelines["fused"] = LayerPipeline(fused, [f.compact for f in fused], dev)
    # Every layer's Top-K known when the step starts: one lookup launch over all layers'
    # rows (the stacked maps and Top-K as layers x requests rows), then every layer's
    # direct K,V gather of its slots in one ekv_gather_layers launch.  Each residency-map
    # entry is read once per step (the mapped forms read it in the lookup and again in the
    # gather), and no launch boundary separates the layers.
    all_lookup = LookupPlan(maps_all.view(layers * reqs, ctx), topks_all.view(layers * reqs, k))
    all_slots = all_lookup.slots.view(layers, reqs, k)
    layer_gather = LayerGather(planes, [all_slots[layer] for layer in range(layers)], req_ids, lengths, None, None,
                               outs, layout, planes_per_layer=2, indirect=False)

    def multi_layer_step():
        all_lookup()
        layer_gather()

    pipelines["multi_layer"] = multi_layer_step
    pipelines["multi_layer_gather"] = layer_gather  # the gather launch alone: its kernel's roofline
    modes = ("order", "fused", "concurrent", "pipelined", "multi_layer")
    projection, refs, mapped_bits, candidate, unmapped, n_chunks, _ = freeable_world(dist, shard)
    counts_buf = projection.counts(candidate)
    bits_buf = freeable_bitmap(counts_buf, refs, mapped_bits)
    # Across ranks, the alternative to NCCL: one kernel builds this rank's bitmap and ANDs
    # the peers' over NVLink (symmetric memory, bounded polls), launched beside the layers.
    peer, peer_error = None, None
    if dist.world > 1:
        from ekv_b200.releasable import PeerFreeableCombiner

        try:
            peer = PeerFreeableCombiner(n_chunks, dev)
        except Exception as exc:  # every rank meets the same failure (same setup)
            peer_error = f"{type(exc).__name__}: {exc}"[:200]
        peer_counts = torch.empty_like(counts_buf)
        peer_bits = torch.empty_like(bits_buf)

    def layers_step(mode="order"):
        if mode in pipelines:
            pipelines[mode]()
        else:
            for layer in range(layers):
                lookups[layer]()
                gathers[layer]()

    def build_bitmap():
        freeable_bitmap(projection.counts(candidate, out=counts_buf), refs, mapped_bits, out=bits_buf)

    layers_step()
    torch.cuda.synchronize()
    # Parity on layer 0 and the last layer against the oracle, on this rank's head shard.
    parity = True
    for layer in sorted({0, layers - 1}):
        slots, miss, miss_list, miss_count = ol.lookup_slots(maps[layer].cpu().numpy(), topks[layer].cpu().numpy())
        parity &= np.array_equal(lookups[layer].slots.cpu().numpy(), slots)
        parity &= np.array_equal(lookups[layer].miss_list.cpu().numpy(), miss_list)
        for which in range(2):
            want = og.gather_rows(planes[2 * layer + which].view(torch.int16).cpu().numpy(), slots,
                                  req_ids.cpu().numpy(), lengths.cpu().numpy(), None, None, width=width,
                                  table_width=hot, request_stride=layout.request_bytes // 2,
                                  sink_elements=CHUNK // 2, indirect=False)
            parity &= np.array_equal(outs[2 * layer + which].view(torch.int16).cpu().numpy(), want)
    # Every form of the step leaves the rows and lookup outputs of the plain one.
    check = sorted({0, layers // 2, layers - 1})
    plain_out = [outs[2 * layer + w].clone() for layer in check for w in range(2)]
    plain_lookup = [t.clone() for t in (lookups[-1].slots, lookups[-1].miss_list, lookups[-1].miss_count)]
    last_of_all = (all_slots[-1], all_lookup.miss_list.view(layers, reqs, k)[-1],
                   all_lookup.miss_count.view(layers, reqs)[-1])
    for mode in modes[1:]:
        last_lookup = last_of_all if mode == "multi_layer" else \
            (fused[-1].slots, fused[-1].miss_list, fused[-1].miss_count) if mode == "fused" else \
            (lookups[-1].slots, lookups[-1].miss_list, lookups[-1].miss_count)
        for t in (*outs, *last_lookup):
            t.zero_()
        layers_step(mode)
        torch.cuda.synchronize()
        parity &= all(torch.equal(outs[2 * layer + w], plain_out[2 * i + w])
                      for i, layer in enumerate(check) for w in range(2))
        parity &= all(torch.equal(a, b) for a, b in zip(last_lookup, plain_lookup))
    del plain_out, plain_lookup
    graphs = {}
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for mode in (*modes, "multi_layer_gather"):
                layers_step(mode)
        torch.cuda.current_stream(dev).wait_stream(side)
        for mode in (*modes, "multi_layer_gather"):
            graphs[mode] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphs[mode]):
                layers_step(mode)
    except Exception as exc:  # capture unsupported: time eager launches instead
        graphs = {}
        capture_error = str(exc)
    else:
        capture_error = None

    def replay(mode):
        if graphs:
            graphs[mode].replay()
        else:
            layers_step(mode)

    joint = {}
    main_stream = torch.cuda.current_stream(dev)
    bitmap_stream = torch.cuda.Stream(dev)

    def bitmap_and_combine():
        build_bitmap()
        joint["bits"] = combine_freeable(bits_buf)

    def step(mode, combine="beside"):
        # The freeable bitmap depends only on chunk ownership.  "peer" (reported across
        # ranks): counts + the fused build/exchange/AND kernel over peer memory on a second
        # stream beside the layers.  "beside" (reported on one rank): the build on a second
        # stream beside the layers and the NCCL exchange + AND after them.  "after": build
        # and NCCL exchange after the layers.  "second_stream": build and NCCL exchange
        # beside the layers -- measured slower across ranks: the gathers' persistent grids
        # hold every SM, so the NCCL kernels, which wait for the peer rank's, start late
        # (2 GPUs: +334 us per step against +30 us after the layers).
        if combine == "after":
            replay(mode)
            bitmap_and_combine()
            return
        bitmap_stream.wait_stream(main_stream)
        with torch.cuda.stream(bitmap_stream):
            if combine == "second_stream":
                bitmap_and_combine()
            elif combine == "peer":
                peer.combine(projection.counts(candidate, out=peer_counts), refs, mapped_bits, out=peer_bits)
            else:
                build_bitmap()
        replay(mode)
        main_stream.wait_stream(bitmap_stream)
        if combine == "beside":
            joint["bits"] = combine_freeable(bits_buf)

    mode_ms = {}
    reported = CFG4_REPORTED
    # Across ranks the reported exchange is the fused peer-memory kernel beside the layers
    # (build, exchange and AND in one launch over NVLink); NCCL (all-gather + AND kernel
    # after the layers) is timed beside it.  One rank, or no symmetric memory: NCCL form.
    exchange = "peer" if peer is not None else "beside"

    def peer_alone():
        peer.combine(projection.counts(candidate, out=peer_counts), refs, mapped_bits, out=peer_bits)

    with ClockSampler(dist.local_rank) as clocks:
        for mode in modes:
            mode_ms[mode] = timed(lambda: step(mode, combine=exchange), steps, warmup, dist) / steps
        after_ms = timed(lambda: step(reported, combine="after"), steps, warmup, dist) / steps
        second_stream_ms = timed(lambda: step(reported, combine="second_stream"), steps, warmup, dist) / steps
        without_combine_ms = timed(lambda: replay(reported), steps, warmup, dist) / steps
        combine_alone_ms = timed(bitmap_and_combine, steps, warmup, dist) / steps
        layer_gather_ms = timed(lambda: replay("multi_layer_gather"), steps, warmup, dist) / steps
        nccl_ms = timed(lambda: step(reported, combine="beside"), steps, warmup, dist) / steps
        peer_alone_ms = timed(peer_alone, steps, warmup, dist) / steps if peer is not None else None
    torch.cuda.synchronize()
    expected_joint = bitmap_to_chunks(bits_buf)
    for r in range(dist.world):
        expected_joint -= unmapped[r]
    joint_ok = bitmap_to_chunks(joint["bits"]) == expected_joint
    peer_record = {}
    if peer is not None:
        peer_ok = bitmap_to_chunks(peer_bits) == expected_joint and not peer.failed()
        joint_ok = joint_ok and peer_ok
        peer_record = {"peer_alone_us": peer_alone_ms * 1e3, "peer_combine_matches_intersection": peer_ok}
    elif peer_error:
        peer_record = {"peer_combine_unavailable": peer_error}
    ms_per_step = mode_ms[reported]
    units = reqs * k * layers
    hits = reqs * n_hits * layers
    misses = units - hits
    # K and V: a hit row is read and written, a miss row written as zeros; lookup: 13 B per
    # Top-K id (index, map entry, slot, mask) + 4 B per miss-list entry.
    gather_bytes = hits * 4 * row_bytes + misses * 2 * row_bytes
    bytes_per_step = gather_bytes + units * (4 + 4 + 4 + 1) + misses * 4
    peak, peak_source = measured_hbm_peak()
    achieved = bytes_per_step / (ms_per_step / 1e3) / 1e9
    result = {
        "metric": METRIC, "value": units / (ms_per_step / 1e3), "unit": "row-pairs/s",
        "n_gpus": dist.world, "steps": steps, "warmup": warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded residency maps, Top-K with 90% hits, N(0,1) bf16 hot pools)",
        "config": {"workload": f"config 4: TP-sharded sparse residency, {layers} layers x (lookup + K,V gather), "
                               f"{reqs} requests x {ctx} context, hot {hot}/request, Top-K {k}, "
                               f"heads {heads}/rank, freeable bitmap + AND-combine per step",
                   "parallelism": f"tp{dist.world} (KV-head sharding; lookup replicated; NCCL AND-combine)",
                   "cuda_graph": bool(graphs), "capture_error": capture_error,
                   "l2": "no flush: each layer gathers into its own output buffers; a step touches "
                         f"{bytes_per_step / 1e9:.2f} GB per GPU (> 126 MB L2)"},
        "step_forms": {
            "reported": f"{reported}: {CFG4_FORMS[reported]}",
            **{mode: {"ms_per_step": mode_ms[mode], "value": units / (mode_ms[mode] / 1e3),
                      "frac": bytes_per_step / (mode_ms[mode] / 1e3) / 1e9 / peak, "what": CFG4_FORMS[mode]}
               for mode in ("fused", "concurrent") if mode != reported},
            "layer_order": {"ms_per_step": mode_ms["order"], "value": units / (mode_ms["order"] / 1e3),
                            "what": "lookup, then the direct gather of its slots, layer after layer (the "
                                    "reference's order)"},
            "pipelined": {"ms_per_step": mode_ms["pipelined"], "value": units / (mode_ms["pipelined"] / 1e3),
                          "what": "layer i's direct gather on a second stream while layer i+1's lookup runs; "
                                  "valid only when every layer's Top-K is known when the step starts"},
            "multi_layer": {"ms_per_step": mode_ms["multi_layer"],
                            "value": units / (mode_ms["multi_layer"] / 1e3),
                            "frac": bytes_per_step / (mode_ms["multi_layer"] / 1e3) / 1e9 / peak,
                            "gather_launch_us": layer_gather_ms * 1e3,
                            "gather_launch_frac": gather_bytes / (layer_gather_ms / 1e3) / 1e9 / peak,
                            "what": "one lookup launch over every layer's rows, then every layer's direct K,V "
                                    "gather of its slots in one ekv_gather_layers launch (no launch boundary "
                                    "between layers, each residency-map entry read once); valid only when "
                                    "every layer's Top-K is known when the step starts.  gather_launch_*: "
                                    "that gather launch alone against its own bytes"}},
        "hbm_gbs_per_gpu": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_source,
                     "note": f"step = {layers} lookups + {layers} two-plane gathers + bitmap build + combine; "
                             "bytes = hit rows x 4 x row_bytes (K and V read and written) + miss rows x 2 x "
                             "row_bytes (zero rows written) + 13 B per lookup + 4 B per miss-list entry"},
        "combine": {"what": ("counts kernel + ekv_freeable_and_peers (this rank's bitmap built, published "
                             "to every peer and ANDed with theirs over NVLink peer memory in one single-block "
                             "kernel, bounded polls) on a second stream beside the layers"
                             if exchange == "peer" else
                             "freeable-bitmap build (counts + bitmap kernels) on a second stream beside the "
                             "layers, then NCCL all_gather_into_tensor of each rank's 512 B bitmap + AND kernel "
                             "after them"
                             if dist.world > 1 else "freeable-bitmap build (counts + bitmap kernels) on a second "
                                                    "stream beside the layers, single rank (no exchange)"),
                    "alone_us": (peer_alone_ms if exchange == "peer" else combine_alone_ms) * 1e3,
                    "us_added_to_step": (ms_per_step - without_combine_ms) * 1e3,
                    "step_without_combine_ms": without_combine_ms,
                    "step_with_nccl_exchange_after_the_layers_ms": nccl_ms,
                    "nccl_alone_us": combine_alone_ms * 1e3,
                    "step_with_build_and_nccl_exchange_after_the_layers_ms": after_ms,
                    "step_with_nccl_combine_on_second_stream_ms": second_stream_ms,
                    "freeable_joint": len(bitmap_to_chunks(joint["bits"])),
                    "joint_matches_intersection": bool(joint_ok), **peer_record},
        "parity_layer0_and_last": bool(parity),
        # per step: 48 fused launches + 48 compactions + counts + (bitmap, or the fused
        # exchange kernel); the NCCL form adds the AND kernel across ranks
        "gpu_launches": (2 * layers + 2) * steps + steps * (dist.world > 1 and exchange != "peer"),
        "clocks": clocks.summary(),
    }
    graphs.clear()
    del peer
    return result


def run_config4(args, dist: Dist):
    return config4_leg(args, dist, args.steps, args.warmup)


CFG5 = dict(layers=48, kv_heads=8, head_dim=128, requests=128, context=65536, hot=8192, topk=2048, steps=64,
            keep=0.9, zipf_s=1.1)


def zipf_topk_schedule(steps, batch, context, k, keep, s, seed):
    """Top-K token ids per decode step [steps, batch, k] (int32, distinct per row).

    Step 0 draws k distinct ids; every later step keeps ``keep`` of the previous
    step's ids and draws the rest from Zipf(s) over the distance from the newest
    token (distance d -> position context - 1 - d, truncated to the context).
    """
    import numpy as np

    rng = np.random.default_rng(seed)

    def fresh(row_exclude, n):
        out = []
        seen = set(row_exclude)
        while len(out) < n:
            d = rng.zipf(s, 4 * (n - len(out)) + 16) - 1
            for pos in (context - 1 - d[d < context]).tolist():
                if pos not in seen:
                    seen.add(pos)
                    out.append(pos)
                    if len(out) == n:
                        break
        return out

    sched = np.empty((steps, batch, k), dtype=np.int32)
    n_keep = int(k * keep)
    for b in range(batch):
        sched[0, b] = rng.permutation(fresh((), k))
    for t in range(1, steps):
        for b in range(batch):
            kept = sched[t - 1, b, :n_keep].tolist()
            sched[t, b] = rng.permutation(np.array(kept + fresh(kept, k - n_keep), dtype=np.int32))
    return sched


def run_config5(args, dist: Dist):
    return config5_leg(args, dist, args.steps if args.steps != 100 else CFG5["steps"])


def config5_leg(args, dist: Dist, steps: int):
    """Config 5: multi-step sparse decode with host-backed history.  Each step, for every
    layer: lookup of the step's Top-K in the layer's hot buffer, clock victim selection for
    the misses, promotion of the missed rows from pinned host history, mapped gather of all
    Top-K rows -- four launches per layer, replayed from one CUDA graph; the step's Top-K
    ids are copied from pinned host memory first."""
    from ekv_b200.host_pool import pinned_buffer
    from ekv_b200.swap import HotLayer, SwapPipeline, SwapStep

    c = CFG5
    dev = dist.device
    shard = args.tp_shard or dist.world
    heads = c["kv_heads"] // shard
    width = heads * c["head_dim"]
    row_bytes = width * 2
    batch, ctx, hot, k = c["requests"], c["context"], c["hot"], c["topk"]
    # 1 GPU without head sharding cannot hold 48 layers of hot buffers (4 GiB per layer).
    layers = args.layers or (c["layers"] if shard > 1 else 24)
    # Host history shared by every layer (per-layer history would be 1.5 TiB):
    # word w of token t of request b, plane p = ((b*ctx + t) * words + w) XOR key[p].
    words = row_bytes // 4
    keys = [0x5BD1E995, 0x27D4EB2F]
    history = []
    rows_total = batch * ctx
    chunk_rows = max(1, (1 << 30) // row_bytes)
    for key in keys:
        host = pinned_buffer(rows_total * row_bytes)[: rows_total * row_bytes].view(rows_total, row_bytes)
        for r0 in range(0, rows_total, chunk_rows):
            r1 = min(rows_total, r0 + chunk_rows)
            vals = (torch.arange(r0 * words, r1 * words, dtype=torch.int64, device=dev) ^ key).to(torch.int32)
            host[r0:r1].copy_(vals.view(torch.uint8).view(r1 - r0, row_bytes), non_blocking=True)
        history.append(host)
    torch.cuda.synchronize()
    sched = zipf_topk_schedule(steps + 1, batch, ctx, k, c["keep"], c["zipf_s"], seed=55)
    sched_pinned = torch.from_numpy(sched).pin_memory()
    topk_dev = torch.empty((batch, k), dtype=torch.int32, device=dev)
    topk_dev.copy_(sched_pinned[0])
    hot_layers = [HotLayer(batch, ctx, hot, width, dev) for _ in range(layers)]
    # One K/V output pair reused by every layer, as a decode step consumes each
    # layer's rows before the next layer runs.
    shared_out = [torch.empty((batch, k, width), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    outputs = [shared_out for _ in range(layers)]
    plans = [SwapStep(layer, topk_dev, [h.view(torch.bfloat16) for h in history], outputs[i])
             for i, layer in enumerate(hot_layers)]
    promoted = torch.zeros((), dtype=torch.int64, device=dev)
    pipeline = SwapPipeline(plans)

    def layers_step(overlap=True):
        if overlap:
            pipeline()  # layer i's gather overlaps layer i+1's promotion
        else:
            for plan in plans:
                plan()
        for plan in plans:
            promoted.add_(plan.lookup.miss_count.sum())

    def check(step_ids):
        """Every gathered row is its token's history row (last layer, both planes)."""
        ok = True
        rows = (torch.arange(batch, device=dev)[:, None] * ctx + step_ids.to(torch.int64))
        w = torch.arange(words, device=dev, dtype=torch.int64)
        for p, key in enumerate(keys):
            want = ((rows[..., None] * words + w) ^ key).to(torch.int32)
            ok &= bool(torch.equal(outputs[-1][p].view(torch.int32).view(batch, k, words), want))
        return ok

    # Step 0 (cold: every Top-K id misses), timed on its own.
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    layers_step()
    end.record()
    end.synchronize()
    cold_ms = start.elapsed_time(end)
    cold_promoted = int(promoted.item())
    parity = check(topk_dev)
    graphs = {}
    capture_error = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            topk_dev.copy_(sched_pinned[1], non_blocking=True)
            layers_step()  # step 1 eagerly (also warms every launch path)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        parity &= check(topk_dev)
        for overlap in (True, False):
            graphs[overlap] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphs[overlap]):
                layers_step(overlap)
    except Exception as exc:
        graphs, capture_error = {}, str(exc)
    promoted.zero_()
    first = 2

    def step(t, overlap):
        topk_dev.copy_(sched_pinned[t], non_blocking=True)
        if graphs:
            graphs[overlap].replay()
        else:
            layers_step(overlap)

    # Even steps overlapped (the product path), odd steps in plain layer order, so
    # both see the same miss distribution; each step timed with its own events.
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(first, steps + 1)]
    promoted_by_mode = {True: 0, False: 0}
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dist.local_rank) as clocks:
        start.record()
        for i, t in enumerate(range(first, steps + 1)):
            overlap = t % 2 == 0
            marks[i][0].record()
            step(t, overlap)
            marks[i][1].record()
        end.record()
        end.synchronize()
    per_step = {True: [], False: []}
    for i, t in enumerate(range(first, steps + 1)):
        per_step[t % 2 == 0].append(marks[i][0].elapsed_time(marks[i][1]))
    parity &= check(topk_dev)
    timed_steps = len(per_step[True])
    promoted_rows = int(promoted.item())
    ms_per_step = dist.max(sum(per_step[True]) / timed_steps)
    sequential_ms_per_step = dist.max(sum(per_step[False]) / max(1, len(per_step[False])))
    all_steps = len(per_step[True]) + len(per_step[False])
    units = batch * k * layers
    promoted_bytes_step = promoted_rows * 2 * row_bytes / all_steps
    gather_bytes_step = units * 4 * row_bytes
    peak, peak_source = measured_hbm_peak()
    used_graph = bool(graphs)
    graphs.clear()
    return {
        "metric": METRIC, "value": units / (ms_per_step / 1e3), "unit": "row-pairs/s", "n_gpus": dist.world,
        "steps": timed_steps, "warmup": first, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf(1.1) Top-K schedule, 90% kept per step; host history pattern)",
        "config": {"workload": f"config 5: multi-step sparse decode, {batch} requests x {ctx} context, "
                               f"{layers} layers, hot {hot}/request, Top-K {k}, lookup -> swap-in -> "
                               f"promotion from pinned host -> mapped gather per layer",
                   "layers": layers, "heads_per_rank": heads, "cuda_graph": used_graph,
                   "capture_error": capture_error,
                   "cuts": ("host history shared by all layers (per-layer history would be 1.5 TiB); "
                            + ("24 of 48 layers at 1 GPU (hot buffers are 4 GiB per layer)" if layers < 48 else
                               "none"))},
        "cold_step": {"ms": cold_ms, "promoted_rows": cold_promoted,
                      "promoted_bytes": cold_promoted * 2 * row_bytes},
        "sequential_ms_per_step": sequential_ms_per_step,
        "overlap_speedup": sequential_ms_per_step / ms_per_step,
        "timing": "even steps overlapped (SwapPipeline: layer i's gather on a second stream during layer "
                  "i+1's promotion) = the reported value; odd steps in plain layer order = sequential_ms_per_step; "
                  "the overlap is valid because a step's one Top-K set (copied in before the layers) serves "
                  "every layer, so no layer's swap-in waits on an earlier layer",
        "promoted_rows_per_step": promoted_rows / all_steps,
        "promoted_bytes_per_step": promoted_bytes_step,
        "host_link_gbs": promoted_bytes_step / (ms_per_step / 1e3) / 1e9,
        "hbm_gbs_per_gpu": (gather_bytes_step + 2 * promoted_bytes_step) / (ms_per_step / 1e3) / 1e9,
        "hbm_peak": peak, "peak_source": peak_source,
        "parity_rows_equal_history": bool(parity),
        "gpu_launches": 4 * layers * all_steps,
        "clocks": clocks.summary(),
    }


def run_reference(args, dist: Dist):
    """Reference arm: the torch-CPU restatement on the host cores, rank 0 only."""
    if dist.rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # The host has no head sharding: it gathers whole rows (all 8 heads) of the job.
    width = CFG2["kv_heads"] * CFG2["head_dim"]
    slots, b, k = CFG2["slots"], CFG2["requests"], CFG2["topk"]
    layers = args.layers or CFG2["layers"]
    # The whole configuration: every layer's K and V plane in host memory (36 GiB + 18 GiB
    # of outputs at config 2), unless the host lacks the memory -- then as many layers as
    # fit, said in the line.  A bit copy's time does not depend on the bytes, so the
    # planes get one fast fill instead of random draws.
    per_layer = 2 * (slots + b * k) * width * 2
    try:
        import psutil

        available = psutil.virtual_memory().available
    except Exception:  # no psutil: assume the configuration fits
        available = per_layer * layers * 2
    sample_layers = max(1, min(layers, int(available * 0.6) // per_layer))
    planes = []
    for p in range(2 * sample_layers):
        plane = torch.empty((slots, width), dtype=torch.int16)
        plane.view(torch.int64).fill_(0x0123456789ABCDEF + p)
        planes.append(plane)
    igen = torch.Generator().manual_seed(42)
    idx = dict(request_table=torch.stack([torch.randperm(slots, generator=igen)[:k] for _ in range(b)]),
               positions=torch.stack([torch.randperm(k, generator=igen) for _ in range(b)]),
               request_ids=torch.arange(b), lengths=torch.full((b,), k, dtype=torch.int64),
               slot_offsets=torch.arange(slots, dtype=torch.int64) * width)
    outputs = [torch.empty((b, k, width), dtype=torch.int16) for _ in planes]
    for _ in range(args.warmup):
        run_cpu_gather(planes, idx, outputs, width)
    started = time.perf_counter()
    for _ in range(args.steps):
        run_cpu_gather(planes, idx, outputs, width)
    elapsed = time.perf_counter() - started
    units = b * k * sample_layers
    value = units * args.steps / elapsed
    sample = (f"{sample_layers} of {layers} layers (K and V planes [262144, {width}] bf16 bits), "
              f"all {b * k} Top-K row-pairs per layer per step")
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "row-pairs/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": (f"config 2: sparse Top-K KV gather on the host cores, {sample_layers} of "
                                f"{layers} layers x K,V, 64 requests x 2048 Top-K"),
                   "layers_sampled": sample_layers, "layers": layers, "requests": b, "topk": k,
                   "parallelism": "cpu (all host threads)"},
        "cpu_baseline": {"value": value, "unit": "row-pairs/s", "cores": threads, "kind": "port",
                         "sample": sample, "cpu": platform.processor() or platform.machine()},
        "e2e": {"value": value, "unit": "row-pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _result_stream():
    """Keep stdout for the one JSON line: send everything else written to fd 1
    (NCCL's version banner, library prints) to stderr."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(saved, "w")


def main(argv=None):
    args = parse_args(argv)
    out = _result_stream()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        from types import SimpleNamespace

        world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
        result = run_reference(args, SimpleNamespace(rank=0, world=world))
        print(json.dumps(result), file=out, flush=True)
        return 0
    dist = Dist()
    try:
        if args.only:
            if args.only == "bitmap":
                leg_result = bitmap_bench(dist, shard=args.tp_shard)
            elif args.only == "roundtrip":
                leg_result = {"plain": round_trip_bench(dist.device),
                              "spare_handles": round_trip_bench(dist.device, spare_chunks=256)}
            else:
                leg_result = {"lookup": lookup_bench, "shadow": shadow_bench}[args.only](dist)
            result = {"leg": args.only, **leg_result}
        else:
            runner = {4: run_config4, 5: run_config5}.get(args.config, run_default)
            result = runner(args, dist)
        if dist.rank == 0:
            print(json.dumps(result), file=out, flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
