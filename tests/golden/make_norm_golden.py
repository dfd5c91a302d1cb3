"""Generates tests/golden/norms_upstream.npz: the norms of the path run through the
upstream PyTorch modules that the reference's own parity policy gates its norms
against (docs/parity.md:5-6, 16-18: the pinned official LeVo source on PyTorch
and Transformers; python/export_layer0_operators.py:59,81 captures the LM's
`input_layernorm` / `post_attention_layernorm` outputs, Transformers' Llama
RMSNorm).

The reference's own norms are GGML graph nodes (`rms_norm_weighted`,
src/levo-lm.cpp:131-138; `layer_norm`, src/levo-flow-estimator.cpp:106-109),
and GGML is an absent submodule, so these modules are the nearest executable
definition of what the reference is held to.  Run in an environment with torch
and transformers (no reference tree needed):

    python tests/golden/make_norm_golden.py

Versions used are stored in the file; the reference pins Transformers 4.37.2 and
PyTorch 2.6, whose RMSNorm / LayerNorm forward passes compute the same
expressions (F32 statistics; for F16 models, the normalised value is cast to
F16 before the F16 weight multiplies it).

Cases (seeded, small; h = x + r is not stored, numpy's x + r gives it):
  rms_f32   LM RMSNorm, F32: h = x + r [8, 1536], eps 1e-5 (src/levo-model.h:106)
  rms_f16   the same in F16 (x, r, weight F16; h = x + r rounded to F16)
  ln_f32    Flow estimator LayerNorm, F32: h = x + r [4, 2200], eps 1e-5
            (src/levo-flow-estimator.cpp:20; hidden 2200, src/levo-flow-model.h:15),
            x offset by +3 so mean >> stddev
  ln_f16    the same in F16 (weights F16)
"""
from __future__ import annotations

import pathlib

import numpy as np
import torch
import transformers
from transformers.models.llama.modeling_llama import LlamaRMSNorm

HERE = pathlib.Path(__file__).resolve().parent


def _rms(rng, rows, dim, dt):
    x = rng.standard_normal((rows, dim)).astype(dt)
    r = rng.standard_normal((rows, dim)).astype(dt)
    w = (1 + 0.02 * rng.standard_normal(dim)).astype(dt)
    mod = LlamaRMSNorm(dim, eps=1e-5)
    with torch.no_grad():
        mod.weight.copy_(torch.from_numpy(w.astype(np.float32)))
        if dt == np.float16:
            mod = mod.half()
        h = torch.from_numpy(x) + torch.from_numpy(r)  # rounded to the activation dtype
        y = mod(h)
    return x, r, w, h.numpy(), y.numpy()


def _ln(rng, rows, dim, dt):
    x = (3 + rng.standard_normal((rows, dim))).astype(dt)
    r = rng.standard_normal((rows, dim)).astype(dt)
    w = (1 + 0.02 * rng.standard_normal(dim)).astype(dt)
    b = (0.02 * rng.standard_normal(dim)).astype(dt)
    mod = torch.nn.LayerNorm(dim, eps=1e-5)
    with torch.no_grad():
        mod.weight.copy_(torch.from_numpy(w.astype(np.float32)))
        mod.bias.copy_(torch.from_numpy(b.astype(np.float32)))
        if dt == np.float16:
            mod = mod.half()
        h = torch.from_numpy(x) + torch.from_numpy(r)
        y = mod(h)
    return x, r, w, b, h.numpy(), y.numpy()


def main() -> None:
    torch.manual_seed(0)
    out = {"versions": np.array(f"torch {torch.__version__}; transformers {transformers.__version__}")}
    for name, dt, seed in (("rms_f32", np.float32, 11), ("rms_f16", np.float16, 12)):
        x, r, w, h, y = _rms(np.random.default_rng(seed), 8, 1536, dt)
        assert np.array_equal(h, x + r)  # numpy rounds the sum to the activation dtype the same way
        out.update({f"{name}_x": x, f"{name}_r": r, f"{name}_w": w, f"{name}_y": y})
    for name, dt, seed in (("ln_f32", np.float32, 13), ("ln_f16", np.float16, 14)):
        x, r, w, b, h, y = _ln(np.random.default_rng(seed), 4, 2200, dt)
        assert np.array_equal(h, x + r)
        out.update({f"{name}_x": x, f"{name}_r": r, f"{name}_w": w, f"{name}_b": b, f"{name}_y": y})
    np.savez_compressed(HERE / "norms_upstream.npz", **out)
    print("wrote", HERE / "norms_upstream.npz", out["versions"])


if __name__ == "__main__":
    main()
