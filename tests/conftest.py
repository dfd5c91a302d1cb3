"""Shared fixtures.  Tests marked `gpu` need a CUDA device and the built
liblevo_b200.so; everything else runs on the CPU (oracle, host logic, ABI
surface)."""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as entry  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and liblevo_b200.so")


def pytest_sessionstart(session):
    """A fresh checkout has neither liblevo_b200.so nor the oracle library: build them once
    (nvcc and gcc).  Existing builds are used as they are."""
    lib = ROOT / "levo2.cpp_b200" / "liblevo_b200.so"
    oracle_lib = ROOT / "oracle" / "liblevo_oracle.so"
    if not lib.exists() or not oracle_lib.exists():
        entry.build()


@pytest.fixture(scope="session")
def pkg():
    return entry.load_package()


@pytest.fixture(scope="session")
def ops(pkg):
    return pkg.ops


@pytest.fixture(scope="session")
def orc():
    return entry.load_oracle()


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def scaled_error(got, want) -> float:
    """max |got - want| / max(|want|, 1): relative for large values, absolute near zero."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want) / np.maximum(np.abs(want), 1.0)))


def assert_close(got, want, tol: float, what: str = "") -> None:
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.array_equal(np.isfinite(got), np.isfinite(want)), f"{what}: finiteness differs"
    m = np.isfinite(want)
    err = scaled_error(got[m], want[m])
    assert err <= tol, f"{what}: max scaled error {err:.3g} > {tol:g}"
