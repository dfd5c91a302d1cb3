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


# --------------------------------------------------------------------------- upstream norm fixtures

UPSTREAM_NORM_CASES = ("rms_f32", "rms_f16", "ln_f32", "ln_f16")


def upstream_norm_case(name: str) -> dict:
    """One case of tests/golden/norms_upstream.npz (tests/golden/make_norm_golden.py): inputs x, r,
    weight w (and bias b for LayerNorm) in the activation dtype, the upstream module's output y,
    and h = x + r rounded to the activation dtype."""
    z = np.load(GOLDEN / "norms_upstream.npz")
    case = {k[len(name) + 1:]: z[k] for k in z.files if k.startswith(name + "_")}
    case["h"] = case["x"] + case["r"]
    case["layer"] = name.startswith("ln")
    case["half"] = case["x"].dtype == np.float16
    return case


def assert_upstream_gates(got, want, what: str) -> None:
    """The reference's own parity gates against the upstream modules (docs/parity.md:16-18):
    F32 atol = rtol = 1e-4; F16 cosine similarity >= 0.9999 and normalised RMSE <= 1e-2.  F16
    results must also stay within one F16 ulp of the upstream value on every element (the two
    differ only in the F32 rounding of the statistics before the final F16 rounding), the ulp taken
    at max(|ref|, 0.05 RMS(ref)) like the relative bar of assert_close: a LayerNorm output that is
    small only because + beta cancels the normalised term carries the error of that term."""
    g = np.asarray(got).astype(np.float64)
    w = np.asarray(want).astype(np.float64)
    if np.asarray(want).dtype == np.float16:
        cos = float(np.sum(g * w) / np.sqrt(np.sum(g * g) * np.sum(w * w)))
        nrmse = float(np.sqrt(np.mean((g - w) ** 2)) / np.sqrt(np.mean(w * w)))
        floor = REL_FLOOR_RMS * float(np.sqrt(np.mean(w * w)))
        ulp = np.spacing(np.maximum(np.abs(np.asarray(want)), np.float16(floor))).astype(np.float64)
        assert cos >= 0.9999, f"{what}: cosine {cos}"
        assert nrmse <= 1e-2, f"{what}: normalised RMSE {nrmse}"
        assert np.all(np.abs(g - w) <= ulp), f"{what}: {int(np.sum(np.abs(g - w) > ulp))} values beyond 1 F16 ulp"
    else:
        assert np.allclose(g, w, rtol=1e-4, atol=1e-4), f"{what}: beyond atol = rtol = 1e-4"
