"""Generates the golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree exists (its path in LEVO_REFERENCE_ROOT, or the
reference_path of BASELINE.json) after `make -C oracle REF_ROOT=...` has built
oracle/_ref/libref_levo.so:

    python tests/golden/make_golden.py

Fixtures (all small):
  snakebeta_kat.npz   the SnakeBeta known-answer case of tests/test-audio-ops.cpp:163-215,
                      expected values computed as that test does (float sinf/expf via libm)
  weightnorm_ref.npz  outputs of the reference converters' _fold_weight_norm
                      (convert/convert_vae.py:187-199) and _materialize_weight_norm
                      (convert/convert_flow.py:288-293) on seeded inputs
  flow_ref.npz        outputs of the reference's own solve_flow_euler / combine_renderer_cfg /
                      make_renderer_schedule (src/levo-flow-renderer.cpp, src/levo-renderer-pattern.cpp)
                      compiled from the reference sources (oracle/_ref)
"""
from __future__ import annotations

import ctypes
import ctypes.util
import importlib.util
import os
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
import __graft_entry__ as _entry  # noqa: E402

REF = _entry.reference_root()
if REF is None:
    raise SystemExit("make_golden: the reference tree was not found (set LEVO_REFERENCE_ROOT)")


def _libm():
    m = ctypes.CDLL(ctypes.util.find_library("m"))
    for name in ("sinf", "expf"):
        getattr(m, name).restype = ctypes.c_float
        getattr(m, name).argtypes = [ctypes.c_float]
    return m


def snakebeta_kat() -> None:
    m = _libm()
    x = np.array([[-1.0, 0.0, 1.0], [-0.5, 0.5, 1.5]], np.float32)
    alpha_log = np.array([np.log(np.float32(2.0)), np.log(np.float32(0.5))], np.float32)
    beta_log = np.array([np.log(np.float32(1.5)), np.log(np.float32(0.75))], np.float32)
    y = np.empty_like(x)
    for c in range(2):
        alpha = np.float32(m.expf(float(alpha_log[c])))
        beta = np.float32(np.float32(m.expf(float(beta_log[c]))) + np.float32(1e-9))
        for t in range(3):
            v = x[c, t]
            s = np.float32(m.sinf(float(np.float32(v * alpha))))
            y[c, t] = np.float32(v + np.float32(np.float32(s * s) / beta))
    np.savez(HERE / "snakebeta_kat.npz", x=x, alpha_log=alpha_log, beta_log=beta_log, y=y)


def weightnorm_ref() -> None:
    sys.path.insert(0, str(REF / "convert"))
    import convert_flow as cflow
    import convert_vae as cvae

    rng = np.random.default_rng(1234)
    out = {}
    for name, shape, transpose in (("conv", (96, 48, 7), False), ("transpose", (24, 12, 8), True),
                                   ("wide", (8, 1024, 7), False)):
        v = (0.02 * rng.standard_normal(shape)).astype(np.float32)
        g = rng.uniform(0.5, 1.5, (shape[0], 1, 1)).astype(np.float32)
        spec = cvae.ConvSpec("example", "weight", None, shape, transpose=transpose)
        out[f"{name}_v"] = v
        out[f"{name}_g"] = g
        out[f"{name}_w"] = cvae._fold_weight_norm(v, g, spec)
    g = rng.uniform(0.5, 1.5, (cflow.CONDITION_DIM, 1, 1)).astype(np.float32)
    v = (0.02 * rng.standard_normal((cflow.CONDITION_DIM, cflow.CODEBOOK_DIM, 1))).astype(np.float32)
    out["flow_v"], out["flow_g"], out["flow_w"] = v, g, cflow._materialize_weight_norm(g, v)
    np.savez_compressed(HERE / "weightnorm_ref.npz", **out)


def flow_ref() -> None:
    spec = importlib.util.spec_from_file_location("levo_oracle", ROOT / "oracle" / "oracle.py")
    orc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(orc)
    if not orc.ref_available():
        raise SystemExit("oracle/_ref/libref_levo.so is missing: run `make -C oracle` first")
    rng = np.random.default_rng(4321)
    frames, dim, inc, steps, g, smin = 25, 64, 3, 8, 1.5, 1e-4
    n = frames * dim
    noise = rng.standard_normal(n).astype(np.float32)
    ctx = rng.standard_normal(n).astype(np.float32)
    ctx[inc * dim:] = 0.0
    vu = rng.standard_normal((steps, n)).astype(np.float32)
    vc = rng.standard_normal((steps, n)).astype(np.float32)
    _, solved, done, seen = orc.ref_solve_flow_euler(noise, ctx, frames, dim, inc, smin, steps, vu, vc, True, g,
                                                     want_seen=True)
    assert done == steps
    st, paused, done3, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, inc, smin, steps, vu, vc, True, g,
                                                    pause_after=3)
    assert st == 1 and done3 == 3
    cu = rng.standard_normal(1000).astype(np.float32)
    cc = rng.standard_normal(1000).astype(np.float32)
    cfg = orc.ref_combine_renderer_cfg(cu, cc, 1.5)
    sched_frames = np.array([1, 252, 750, 1000, 1001, 1751, 3000], np.int64)
    sched = [orc.ref_make_renderer_schedule(int(f)) for f in sched_frames]
    np.savez_compressed(
        HERE / "flow_ref.npz", frames=frames, dim=dim, incontext=inc, steps=steps, guidance=g, sigma_min=smin,
        noise=noise, context=ctx, uncond=vu, cond=vc, solved=solved, seen=seen, paused_state=paused,
        paused_steps=done3, cfg_u=cu, cfg_c=cc, cfg_out=cfg, sched_frames=sched_frames,
        sched_padded=np.array([s["padded_frames"] for s in sched], np.int64),
        sched_target=np.array([s["target_samples"] for s in sched], np.int64),
        sched_windows=np.concatenate([np.concatenate([np.full((len(s["windows"]), 1), i), s["windows"]], axis=1)
                                      for i, s in enumerate(sched)]).astype(np.int64))


if __name__ == "__main__":
    snakebeta_kat()
    weightnorm_ref()
    flow_ref()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
