"""Host-side multi-GPU logic on CPU: window ranges, the shared-memory host
gather and the max-over-ranks timing, run as world_size-2 `gloo` ranks.
The decode itself is replaced by a host function (no GPU); a failing rank is
made on the host (an exception), never by a GPU fault."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__ as entry


def test_shard_range_covers_every_window_once():
    sh = entry.load_package().sharding
    for n in range(0, 20):
        for world in (1, 2, 3, 4, 8):
            got = [sh.shard_range(n, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sh.shard_range(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def fake_decode(window: int, shape) -> np.ndarray:
    return np.full(shape, float(window + 1), np.float32) * np.arange(shape[-1], dtype=np.float32)


def _worker(rank, world, port, tag, windows, fail_rank, force_file, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    sh = entry.load_package().sharding
    if force_file and rank == 0:
        sh._free_bytes = lambda _path: 0  # rank 0 alone sees a full /dev/shm: the others must follow it
    try:
        shape = (windows, 2, 50)
        g = sh.HostGather(tag, shape, rank, dist.barrier)
        start, stop = sh.shard_range(windows, rank, world)
        ok = 1
        try:
            if rank == fail_rank:
                raise RuntimeError("injected decode failure")
            for w in range(start, stop):
                g.view(start, stop)[w - start] = fake_decode(w, shape[1:])
        except RuntimeError:
            ok = 0
        # every rank takes the same collective steps, failure or not
        import torch

        flag = torch.tensor([ok], dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        elapsed = torch.tensor([0.5 + rank], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        assert (g.shm is None) == force_file
        if rank == 0:
            complete = bool(flag.item())
            good = complete and all(np.array_equal(g.array[w], fake_decode(w, shape[1:])) for w in range(windows))
            q.put((complete, good, float(elapsed.item())))
        g.close(dist.barrier)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank,force_file", [(-1, False), (1, False), (-1, True)])
def test_two_rank_gather(fail_rank, force_file):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    tag = f"test_{port}"
    mp.start_processes(_worker, args=(2, port, tag, 7, fail_rank, force_file, q), nprocs=2, join=True,
                       start_method="spawn")
    complete, good, elapsed = q.get(timeout=10)
    assert elapsed == 1.5  # max over ranks
    if fail_rank < 0:
        assert complete and good
    else:
        assert not complete  # rank 0 learns of the failure on the host, no partial result is accepted


def test_bind_to_gpu_local_cpus_with_a_fake_nvml(pkg, monkeypatch):
    """The rank is restricted to the CPUs NVML lists for its GPU (intersected with those it may use);
    without NVML the affinity is left alone."""
    import os
    import sys
    import types

    sh = pkg.sharding
    allowed = sorted(os.sched_getaffinity(0))
    want = allowed[: max(1, len(allowed) // 2)]
    mask = [0] * ((os.cpu_count() + 63) // 64)
    for c in want:
        mask[c // 64] |= 1 << (c % 64)
    calls = {}
    fake = types.SimpleNamespace(
        nvmlInit=lambda: None, nvmlShutdown=lambda: None,
        nvmlDeviceGetHandleByIndex=lambda i: calls.setdefault("device", i),
        nvmlDeviceGetCpuAffinity=lambda h, n: mask[:n])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    set_to = {}
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, cpus: set_to.setdefault("cpus", list(cpus)))
    assert sh.bind_to_gpu_local_cpus(3) == want
    assert calls["device"] == 3 and set_to["cpus"] == want

    def broken():
        raise RuntimeError("NVML Shared Library Not Found")

    monkeypatch.setitem(sys.modules, "pynvml", types.SimpleNamespace(nvmlInit=broken))
    set_to.clear()
    assert sh.bind_to_gpu_local_cpus(0) is None and not set_to
