"""Cross-rank AND of freeable bitmaps: gloo ranks on CPU, NCCL ranks on GPUs.

The CPU test runs the exchange logic of ``combine_freeable`` on two gloo
processes with the oracle's AND standing in for the kernel.  The GPU test runs
the real path (NCCL all-gather over NVLink + the AND kernel) when two or more
GPUs are visible, with NVLS off.
"""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PACKAGE_ROOT, ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_bitmap(rank, n_chunks):
    """Deterministic per-rank freeable set: common chunks plus rank-private ones."""
    rng = np.random.default_rng(100 + rank)
    common = set(range(0, n_chunks, 7))
    private = set(rng.choice(n_chunks, 40, replace=False).tolist())
    return common | private


def _worker(rank, world, port, backend, n_chunks, results):
    sys.path[:0] = [str(PACKAGE_ROOT), str(ROOT)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from ekv_b200.releasable import bitmap_to_chunks, chunks_to_bitmap, combine_freeable
    from oracle.releasable import bitmap_and_np

    if backend == "nccl":
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
    else:
        device = torch.device("cpu")
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        local = chunks_to_bitmap(_rank_bitmap(rank, n_chunks), n_chunks, device)
        if backend == "nccl":
            joint = combine_freeable(local)
            torch.cuda.synchronize()
            # The fused peer-memory combine agrees with the NCCL path, epoch after epoch.
            from ekv_b200.releasable import PeerFreeableCombiner

            combiner = PeerFreeableCombiner(n_chunks, device)
            for epoch in range(6):
                bits = chunks_to_bitmap(_rank_bitmap(rank + 10 * epoch, n_chunks), n_chunks, device)
                fused = combiner.combine(local_bits=bits)
                reference = combine_freeable(bits)
                torch.cuda.synchronize()
                assert torch.equal(fused, reference), f"epoch {epoch}"
            assert not combiner.failed()
            del combiner
        else:
            joint = combine_freeable(local, and_fn=lambda g: torch.from_numpy(bitmap_and_np(g.numpy())))
        results[rank] = sorted(bitmap_to_chunks(joint))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, backend, n_chunks=4096):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, backend, n_chunks, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    expected = sorted(set.intersection(*[_rank_bitmap(r, n_chunks) for r in range(world)]))
    for r in range(world):
        assert results[r] == expected
    return expected


def test_combine_freeable_gloo_two_ranks():
    joint = _run(2, "gloo")
    assert set(range(0, 4096, 7)) <= set(joint)


@pytest.mark.gpu
def test_combine_freeable_nccl(cuda_device):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    # The peer combine reads plain peer mappings; keep torch's symmetric memory unbound
    # from any NVSwitch multicast object.
    os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"
    _run(min(world, 8), "nccl")


def test_single_rank_combine_is_identity():
    from ekv_b200.releasable import chunks_to_bitmap, combine_freeable

    bits = chunks_to_bitmap({1, 2, 900}, 1000, "cpu")
    assert torch.equal(combine_freeable(bits), bits)
