"""Reentrancy of the C ABI: host threads driving their own streams at once get
the same results as serial calls, and each thread sees only its own last error
(the reference's thread-local error model, src/cantor-abi.cpp:55-66)."""
from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


def test_threads_on_separate_streams(ops, orc, dev):
    rng = np.random.default_rng(5)
    jobs = []
    for i in range(6):
        x = rng.standard_normal((32, 20000 + 8 * i)).astype(np.float32)
        a = (0.1 * rng.standard_normal(32)).astype(np.float32)
        b = (0.1 * rng.standard_normal(32)).astype(np.float32)
        jobs.append((x, a, b))
    results = [None] * len(jobs)
    errors = []

    def work(i):
        try:
            stream = torch.cuda.Stream(device=dev)
            with torch.cuda.stream(stream):
                x, a, b = (torch.from_numpy(t).to(dev, non_blocking=False) for t in jobs[i])
                for _ in range(20):
                    y = ops.snakebeta_t(x, a, b)
                stream.synchronize()
                results[i] = y.cpu().numpy()
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(jobs))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for (x, a, b), y in zip(jobs, results):
        assert_close(y, orc.snakebeta(x, a, b), 1e-5)


def test_last_error_is_thread_local(ops, dev):
    lib = ops.lib()
    barrier = threading.Barrier(2)
    seen = {}

    def fail_then_read():
        assert lib.levo_weightnorm_f32(None, None, None, None, 1, 1, None) == ops.EINVAL
        barrier.wait()  # the other thread now succeeds, clearing only its own message
        barrier.wait()
        seen["failing"] = ops.last_error()

    def succeed():
        barrier.wait()
        v = torch.ones((2, 8), device=dev)
        ops.weightnorm_t(v, torch.ones(2, device=dev))
        seen["succeeding"] = ops.last_error()
        barrier.wait()

    t1, t2 = threading.Thread(target=fail_then_read), threading.Thread(target=succeed)
    t1.start()
    t2.start()
    t1.join()
    t2.join()
    assert "null" in seen["failing"] and seen["succeeding"] == ""
