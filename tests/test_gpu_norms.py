"""GPU parity of residual add + RMSNorm / LayerNorm (a5, a6) and the weight-norm
fold (a9) against the oracle, through the C ABI.

Tolerances: F16-boundary norms 2e-3 scaled error (north_star), F32 norms and
weight norm 1e-5.  h = x + r is rounded identically on both sides: bit-exact.
RMSNorm / LayerNorm parity is unpinned against the reference itself (its tests
only check shapes and finiteness; its norms are GGML nodes and GGML is absent):
they are anchored on the upstream modules the reference's parity policy holds
them to (Transformers' Llama RMSNorm, torch's LayerNorm; fixtures from
tests/golden/make_norm_golden.py).  Weight norm is pinned by the fixtures of
the reference converters."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, UPSTREAM_NORM_CASES, assert_close, assert_upstream_gates, upstream_norm_case

pytestmark = pytest.mark.gpu


def _inputs(rng, rows, dim, dt):
    x = rng.standard_normal((rows, dim)).astype(dt)
    r = rng.standard_normal((rows, dim)).astype(dt)
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    return x, r, g, b


@pytest.mark.parametrize("layer", [False, True])
@pytest.mark.parametrize("dt", [np.float16, np.float32])
@pytest.mark.parametrize("dim", [1, 7, 16, 100, 512, 768, 1024, 1280, 1536, 2048, 2200, 4096])
def test_add_norm_matches_oracle(ops, orc, dev, layer, dt, dim):
    rng = np.random.default_rng(dim * 3 + layer)
    rows = 37
    x, r, g, b = _inputs(rng, rows, dim, dt)
    eps = 1e-5 if layer else 1e-6
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    if layer:
        h, y = ops.add_layernorm_t(T(x), T(r), T(g), T(b), eps)
        hw, yw = orc.add_layernorm(x, r, g, b, eps)
    else:
        h, y = ops.add_rmsnorm_t(T(x), T(r), T(g), eps)
        hw, yw = orc.add_rmsnorm(x, r, g, eps)
    assert np.array_equal(h.cpu().numpy(), hw)
    assert_close(y.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3 if dt == np.float16 else 1e-5)


@pytest.mark.parametrize("name", UPSTREAM_NORM_CASES)
def test_add_norm_matches_upstream_modules(ops, dev, name):
    """The CUDA norms against the upstream modules the reference's parity policy holds its norms to
    (tests/golden/norms_upstream.npz): the reference's own gates and north_star's bars.  dim 1536
    (F16 and F32) runs the register form, dim 2200 the staged form."""
    c = upstream_norm_case(name)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    w = T(c["w"].astype(np.float32))
    if c["layer"]:
        h, y = ops.add_layernorm_t(T(c["x"]), T(c["r"]), w, T(c["b"].astype(np.float32)), 1e-5)
    else:
        h, y = ops.add_rmsnorm_t(T(c["x"]), T(c["r"]), w, 1e-5, f16_boundary=c["half"])
    y = y.cpu().numpy()
    assert np.array_equal(h.cpu().numpy(), c["h"])
    assert_upstream_gates(y, c["y"], name)
    if not c["half"]:
        assert_close(y.astype(np.float64), c["y"].astype(np.float64), 1e-5, name)


@pytest.mark.parametrize("layer", [False, True])
def test_config1_full_size(ops, orc, dev, layer):
    # F16 [4096, 1536], gamma ~ N(1, 0.02), beta ~ N(0, 0.02), seed 1234.
    rng = np.random.default_rng(1234)
    x, r, g, b = _inputs(rng, 4096, 1536, np.float16)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    if layer:
        h, y = ops.add_layernorm_t(T(x), T(r), T(g), T(b), 1e-5)
        hw, yw = orc.add_layernorm(x, r, g, b, 1e-5)
    else:
        h, y = ops.add_rmsnorm_t(T(x), T(r), T(g), 1e-6)
        hw, yw = orc.add_rmsnorm(x, r, g, 1e-6)
    assert np.array_equal(h.cpu().numpy(), hw)
    assert_close(y.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3)
    # size-independent property of the RMS / LN output before the affine
    yf = y.float()
    if not layer:
        n = yf / torch.from_numpy(g).to(dev)
        assert torch.allclose(n.pow(2).mean(1), torch.ones(4096, device=dev), atol=2e-2)


@pytest.mark.parametrize("layer", [False, True])
def test_f16_boundary_flag(ops, orc, dev, layer):
    rng = np.random.default_rng(77)
    x, r, g, b = _inputs(rng, 64, 1536, np.float16)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    if layer:
        _, y = ops.add_layernorm_t(T(x), T(r), T(g), T(b), 1e-5, f16_boundary=True)
        _, yw = orc.add_layernorm(x, r, g, b, 1e-5, f16_boundary=True)
    else:
        _, y = ops.add_rmsnorm_t(T(x), T(r), T(g), 1e-5, f16_boundary=True)
        _, yw = orc.add_rmsnorm(x, r, g, 1e-5, f16_boundary=True)
    assert_close(y.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3)


def test_norm_without_residual_and_unaligned(ops, orc, dev):
    rng = np.random.default_rng(78)
    x, _, g, b = _inputs(rng, 10, 1536, np.float16)
    buf = torch.empty(10 * 1536 + 8, dtype=torch.float16, device=dev)
    xt = buf[1:1 + 10 * 1536].view(10, 1536)  # 2-byte offset: scalar path
    xt.copy_(torch.from_numpy(x))
    _, y = ops.add_layernorm_t(xt, None, torch.from_numpy(g).to(dev), torch.from_numpy(b).to(dev), 1e-5)
    _, yw = orc.add_layernorm(x, None, g, b, 1e-5)
    assert_close(y.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3)


def test_norm_single_row_and_large_offset_rows(ops, orc, dev):
    rng = np.random.default_rng(79)
    x, r, g, _ = _inputs(rng, 1, 8192, np.float16)
    x = x + np.float16(30)  # large mean: tests the two-pass variance path for LN too
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    h, y = ops.add_rmsnorm_t(T(x), T(r), T(g), 1e-6)
    hw, yw = orc.add_rmsnorm(x, r, g, 1e-6)
    assert np.array_equal(h.cpu().numpy(), hw)
    assert_close(y.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3)


def test_norm_empty_is_noop(ops, dev):
    x = torch.empty((0, 1536), dtype=torch.float16, device=dev)
    g = torch.ones(1536, device=dev)
    ops.add_rmsnorm_t(x, x, g, 1e-6)


# --------------------------------------------------------------------------- weight norm

@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (64, 448), (1024, 7168), (16, 8 * 1024 + 8), (4, 20000), (5, 333)])
def test_weightnorm_matches_oracle(ops, orc, dev, shape):
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    v = (0.02 * rng.standard_normal(shape)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, shape[0]).astype(np.float32)
    norms = torch.empty(shape[0], device=dev)
    w = ops.weightnorm_t(torch.from_numpy(v).to(dev), torch.from_numpy(g).to(dev), norms=norms)
    ww, nw, ok = orc.weightnorm(v, g)
    assert ok
    assert_close(w.cpu().numpy(), ww, 1e-5, f"w {shape}")
    assert_close(norms.cpu().numpy(), nw, 1e-5, f"norms {shape}")


def test_weightnorm_matches_reference_converter_fixtures(ops, dev):
    d = np.load(GOLDEN / "weightnorm_ref.npz")
    for name in ("conv", "transpose", "wide", "flow"):
        v = torch.from_numpy(d[f"{name}_v"]).to(dev)
        g = torch.from_numpy(d[f"{name}_g"].reshape(-1)).to(dev)
        w = ops.fold_weight_norm_t(v, g).cpu().numpy().reshape(d[f"{name}_w"].shape)
        assert_close(w, d[f"{name}_w"], 1e-5, name)


def test_weightnorm_known_answers(ops, dev):
    v = torch.tensor([[[3, 4], [0, 0], [0, 0]], [[0, 0], [5, 12], [0, 0]]], dtype=torch.float32, device=dev)
    g = torch.tensor([10.0, 26.0], device=dev)
    w = ops.fold_weight_norm_t(v, g)
    assert torch.allclose(w, v * 2.0)


def test_weightnorm_zero_norm_raises_like_the_reference(ops, dev):
    v = torch.ones((3, 8), device=dev)
    v[2] = 0
    with pytest.raises(ValueError, match="zero weight-norm"):
        ops.fold_weight_norm_t(v, torch.ones(3, device=dev))


# --------------------------------------------------------------------------- Flow block tail (next item)

@pytest.mark.parametrize("dim", [2200, 64, 13])
@pytest.mark.parametrize("parts", ["all", "no_gate", "no_residual", "no_mod"])
def test_gated_layernorm_modulate_matches_oracle(ops, orc, dev, dim, parts):
    # Flow estimator block: [batch=2, frames, 2200] F32 (src/levo-flow-estimator.cpp:89-93,106-109,221-227)
    rng = np.random.default_rng(dim + len(parts))
    batch, frames = 2, 50
    rows = batch * frames
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    r = None if parts == "no_residual" else rng.standard_normal((rows, dim)).astype(np.float32)
    gate = None if parts == "no_gate" else rng.standard_normal((batch, dim)).astype(np.float32)
    gamma = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    scale = None if parts == "no_mod" else (0.1 * rng.standard_normal((batch, dim))).astype(np.float32)
    shift = None if parts == "no_mod" else (0.1 * rng.standard_normal((batch, dim))).astype(np.float32)
    T = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    h, y = ops.gated_layernorm_modulate_t(T(x), T(gate), T(r), T(gamma), T(beta), T(scale), T(shift), frames)
    hw, yw = orc.gated_layernorm_modulate(x, gate, r, gamma, beta, scale, shift, frames)
    assert np.array_equal(h.cpu().numpy(), hw)  # products and sums only: bit-exact
    assert_close(y.cpu().numpy(), yw, 1e-5, parts)


def test_gated_layernorm_modulate_flow_full_size(ops, orc, dev):
    # The Flow estimator's real block size: [batch = 2 (CFG rows)][1000 frames][2200] F32.
    rng = np.random.default_rng(2200)
    batch, frames, dim = 2, 1000, 2200
    rows = batch * frames
    x, r = rng.standard_normal((2, rows, dim)).astype(np.float32)
    gate, scale, shift = (0.5 * rng.standard_normal((3, batch, dim))).astype(np.float32)
    gamma = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    h, y = ops.gated_layernorm_modulate_t(T(x), T(gate), T(r), T(gamma), T(beta), T(scale), T(shift), frames)
    hw, yw = orc.gated_layernorm_modulate(x, gate, r, gamma, beta, scale, shift, frames)
    assert np.array_equal(h.cpu().numpy(), hw)
    assert_close(y.cpu().numpy(), yw, 1e-5, "flow full size")


def test_gated_layernorm_modulate_rejects_bad_batch(ops, dev):
    x = torch.zeros((10, 64), device=dev)
    g = torch.ones(64, device=dev)
    with pytest.raises(ValueError, match="batch_rows"):
        ops.gated_layernorm_modulate_t(x, None, None, g, g, None, None, 3)
