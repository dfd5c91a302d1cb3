"""GPU parity of the streaming kernels (SnakeBeta a1, bias add a2, fused decoder
unit a3) against the CPU oracle, through the C ABI.

Tolerance (F32 ops): |gpu - oracle| <= 1e-5 * max(|oracle|, 1) per element.
The reference's own CUDA SnakeBeta test uses 2e-5 absolute
(tests/test-audio-ops.cpp:214-215); the known-answer case is checked at that.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_close

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _params(rng, c, scale=0.1):
    return (scale * rng.standard_normal(c)).astype(np.float32), (scale * rng.standard_normal(c)).astype(np.float32)


def test_snakebeta_known_answer(ops, dev):
    d = np.load(GOLDEN / "snakebeta_kat.npz")
    x = torch.from_numpy(d["x"]).to(dev)
    for dt, tol in ((torch.float32, 2e-5), (torch.float16, 2e-3)):
        a = torch.from_numpy(d["alpha_log"]).to(dev, dt)
        b = torch.from_numpy(d["beta_log"]).to(dev, dt)
        y = ops.snakebeta_t(x, a, b).cpu().numpy()
        assert np.max(np.abs(y - d["y"])) <= tol


@pytest.mark.parametrize("shape", [(1, 1), (1, 7), (3, 5), (2, 8), (5, 13), (16, 1001), (128, 4837), (3000, 9),
                                   (7, 65536 + 3)])
def test_snakebeta_matches_oracle(ops, orc, dev, shape):
    rng = np.random.default_rng(hash(shape) % 2**32)
    x = rng.standard_normal(shape).astype(np.float32)
    a, b = _params(rng, shape[0])
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    assert_close(y.cpu().numpy(), orc.snakebeta(x, a, b), TOL, f"snake {shape}")


def test_snakebeta_f16_parameters(ops, orc, dev):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((9, 3001)).astype(np.float32)
    a, b = [p.astype(np.float16) for p in _params(rng, 9)]
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    assert_close(y.cpu().numpy(), orc.snakebeta(x, a, b), TOL, "f16 params")


def test_snakebeta_large_arguments(ops, orc, dev):
    # sin() argument reduction far from the origin (|x*alpha| up to ~1e6).
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((4, 4096)) * np.array([[1], [1e2], [1e4], [1e6]])).astype(np.float32)
    a, b = _params(rng, 4)
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    assert_close(y.cpu().numpy(), orc.snakebeta(x, a, b), TOL, "large |x|")


@pytest.mark.parametrize("offset", [1, 3, 5, 7])
def test_snakebeta_unaligned_views(ops, orc, dev, offset):
    # Tensors starting at a non-32-byte boundary: ragged head + vector body + tail.
    rng = np.random.default_rng(offset)
    c, t = 6, 2053
    base = torch.from_numpy(rng.standard_normal(c * t + 16).astype(np.float32)).to(dev)
    x = base[offset:offset + c * t].view(c, t)
    out = torch.empty(c * t + 16, device=dev)[offset:offset + c * t].view(c, t)
    a, b = _params(rng, c)
    ops.snakebeta_t(x, torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), out=out)
    assert_close(out.cpu().numpy(), orc.snakebeta(x.cpu().numpy(), a, b), TOL, f"offset {offset}")


def test_snakebeta_mismatched_phases_use_scalar_path(ops, orc, dev):
    rng = np.random.default_rng(21)
    c, t = 5, 999
    xs = torch.from_numpy(rng.standard_normal(c * t + 8).astype(np.float32)).to(dev)
    x = xs[1:1 + c * t].view(c, t)
    out = torch.empty(c * t + 8, device=dev)[2:2 + c * t].view(c, t)
    a, b = _params(rng, c)
    ops.snakebeta_t(x, torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), out=out)
    assert_close(out.cpu().numpy(), orc.snakebeta(x.cpu().numpy(), a, b), TOL)


def test_snakebeta_strided_rows(ops, orc, dev):
    rng = np.random.default_rng(22)
    big = torch.from_numpy(rng.standard_normal((10, 700)).astype(np.float32)).to(dev)
    x = big[:, 13:13 + 600]  # row stride 700
    a, b = _params(rng, 10)
    y = ops.snakebeta_t(x, torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    assert_close(y.cpu().numpy(), orc.snakebeta(x.cpu().numpy(), a, b), TOL)


def test_snakebeta_in_place(ops, orc, dev):
    rng = np.random.default_rng(23)
    x = rng.standard_normal((8, 5000)).astype(np.float32)
    a, b = _params(rng, 8)
    t = torch.from_numpy(x).to(dev)
    ops.snakebeta_t(t, torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), out=t)
    assert_close(t.cpu().numpy(), orc.snakebeta(x, a, b), TOL)


def test_snakebeta_many_channels_unstaged_params(ops, orc, dev):
    # > 4096 channels: parameters are read from global memory instead of shared memory.
    rng = np.random.default_rng(24)
    x = rng.standard_normal((5000, 40)).astype(np.float32)
    a, b = _params(rng, 5000)
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    assert_close(y.cpu().numpy(), orc.snakebeta(x, a, b), TOL)


def test_snakebeta_empty_is_noop(ops, dev):
    x = torch.empty((0, 10), device=dev)
    a = torch.zeros(0, device=dev)
    assert ops.snakebeta_t(x, a, a).shape == (0, 10)


def test_snakebeta_config0_full_size(ops, orc, dev):
    # [128, 483840] ~ N(0,1), params ~ N(0, 0.1), seed 1234.
    rng = np.random.default_rng(1234)
    x = rng.standard_normal((128, 483840), dtype=np.float32)
    a, b = _params(rng, 128)
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev))
    y = y.cpu().numpy()
    want = orc.snakebeta(x, a, b)
    assert_close(y, want, TOL, "config 0")
    # size-independent property: 0 <= y - x <= 1/beta
    d = y.astype(np.float64) - x
    inv_beta = 1.0 / (np.exp(b.astype(np.float64)) + 1e-9)
    assert np.all(d >= -1e-6) and np.all(d <= inv_beta[:, None] * (1 + 1e-5) + 1e-6)


def test_channel_bias_add(ops, orc, dev):
    rng = np.random.default_rng(25)
    for shape in [(3, 17), (64, 4096), (1, 1)]:
        x = rng.standard_normal(shape).astype(np.float32)
        bias = rng.standard_normal(shape[0]).astype(np.float32)
        y = ops.channel_bias_add_t(torch.from_numpy(x).to(dev), torch.from_numpy(bias).to(dev))
        assert np.array_equal(y.cpu().numpy(), orc.channel_bias_add(x, bias))
        y16 = ops.channel_bias_add_t(torch.from_numpy(x).to(dev), torch.from_numpy(bias).to(dev, torch.float16))
        want16 = orc.channel_bias_add(x, bias.astype(np.float16).astype(np.float32))
        assert np.array_equal(y16.cpu().numpy(), want16)


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("res", [False, True])
@pytest.mark.parametrize("snake", [False, True])
@pytest.mark.parametrize("write_x", [False, True])
@pytest.mark.parametrize("tanh", [False, True])
def test_fused_unit_variants(ops, orc, dev, bias, res, snake, write_x, tanh):
    rng = np.random.default_rng(7 * bias + 5 * res + 3 * snake + 2 * write_x + tanh)
    c, t = 12, 3333
    u = rng.standard_normal((c, t)).astype(np.float32)
    r = rng.standard_normal((c, t)).astype(np.float32) if res else None
    b = (0.02 * rng.standard_normal(c)).astype(np.float32) if bias else None
    a, bl = _params(rng, c) if snake else (None, None)
    g = lambda v: None if v is None else torch.from_numpy(v).to(dev)  # noqa: E731
    x_out = torch.full((c, t), np.nan, device=dev) if write_x else None
    y_out = torch.full((c, t), np.nan, device=dev)
    ops.fused_unit_t(g(u), g(b), g(r), g(a), g(bl), x_out, y_out, tanh=tanh)
    xw, yw = orc.fused_unit(u, b, r, a, bl, tanh=tanh)
    assert_close(y_out.cpu().numpy(), yw, TOL, "y")
    if write_x:
        assert np.array_equal(x_out.cpu().numpy(), xw)  # additions only: bit-exact


def test_fused_unit_in_place_like_the_chain(ops, orc, dev):
    # The chain writes x over the residual and y over the conv output.
    rng = np.random.default_rng(31)
    c, t = 32, 10007
    u, r = rng.standard_normal((2, c, t)).astype(np.float32)
    b = (0.02 * rng.standard_normal(c)).astype(np.float32)
    a, bl = _params(rng, c)
    tu, tr = torch.from_numpy(u).to(dev), torch.from_numpy(r).to(dev)
    ops.fused_unit_t(tu, torch.from_numpy(b).to(dev), tr, torch.from_numpy(a).to(dev), torch.from_numpy(bl).to(dev),
                     x_out=tr, y_out=tu)
    xw, yw = orc.fused_unit(u, b, r, a, bl)
    assert np.array_equal(tr.cpu().numpy(), xw)
    assert_close(tu.cpu().numpy(), yw, TOL)


@pytest.mark.parametrize("pdt", [torch.float32, torch.float16])
def test_snake_params_prepare(ops, dev, pdt):
    rng = np.random.default_rng(41)
    a, b = _params(rng, 5000, scale=2.0)
    ta, tb = torch.from_numpy(a).to(dev, pdt), torch.from_numpy(b).to(dev, pdt)
    alpha, inv_beta = ops.snake_params_prepare_t(ta, tb)
    a64, b64 = ta.double().cpu().numpy(), tb.double().cpu().numpy()
    # expf is within 2 ulp; the reciprocal is IEEE-rounded
    np.testing.assert_allclose(alpha.cpu().numpy(), np.exp(a64), rtol=3e-7, atol=0)
    np.testing.assert_allclose(inv_beta.cpu().numpy(), 1.0 / (np.exp(b64) + 1e-9), rtol=5e-7, atol=0)


@pytest.mark.parametrize("shape", [(1, 7), (16, 1001), (128, 4096), (3000, 9), (64, 20008), (5000, 8)])
@pytest.mark.parametrize("pdt", [torch.float32, torch.float16])
def test_snakebeta_prepared_equals_log_form(ops, dev, shape, pdt):
    """Every dispatch form (rows, flat vectors, scalar, staged or not) gives the same bits."""
    rng = np.random.default_rng(sum(shape))
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dev)
    a, b = [torch.from_numpy(p).to(dev, pdt) for p in _params(rng, shape[0])]
    alpha, inv_beta = ops.snake_params_prepare_t(a, b)
    want = ops.snakebeta_t(x, a, b)
    got = ops.snakebeta_t(x, alpha, inv_beta, prepared=True)
    assert torch.equal(got, want)
    xs = x[:, 1:]  # strided view: scalar path
    assert torch.equal(ops.snakebeta_t(xs, alpha, inv_beta, prepared=True), ops.snakebeta_t(xs, a, b))


def test_fused_unit_prepared_params(ops, dev):
    rng = np.random.default_rng(43)
    c, t = 40, 8008
    u, r = (torch.from_numpy(v).to(dev) for v in rng.standard_normal((2, c, t)).astype(np.float32))
    bias = torch.from_numpy((0.02 * rng.standard_normal(c)).astype(np.float32)).to(dev)
    a, b = (torch.from_numpy(p).to(dev) for p in _params(rng, c))
    alpha, inv_beta = ops.snake_params_prepare_t(a, b)
    out = [torch.empty_like(u) for _ in range(4)]
    ops.fused_unit_t(u, bias, r, a, b, out[0], out[1])
    ops.fused_unit_t(u, bias, r, alpha, inv_beta, out[2], out[3], param_dtype=ops.DTYPE_SNAKE_PREPARED)
    assert torch.equal(out[0], out[2]) and torch.equal(out[1], out[3])


@pytest.mark.parametrize("scale", [1.0, 3e4])
def test_snakebeta_vector_and_scalar_paths_agree_bitwise(ops, dev, scale):
    """The paired-F32 vector path and the scalar path round every step alike: same bits,
    on the fast range and past the sinf fallback limit (|x*alpha| > 65536)."""
    rng = np.random.default_rng(61)
    c, t = 24, 4096
    x = torch.from_numpy((scale * rng.standard_normal((c, t))).astype(np.float32)).to(dev)
    a, b = (torch.from_numpy(p).to(dev) for p in _params(rng, c, scale=1.0))
    dense = ops.snakebeta_t(x, a, b)
    wide = torch.empty((c, t + 3), device=dev)
    wide[:, :t] = x
    strided = ops.snakebeta_t(wide[:, :t], a, b)  # row stride t + 3: scalar path
    assert torch.equal(dense, strided)


def test_sin_squared_accuracy_against_float64(ops, dev):
    """This library's sin^2 (Cody-Waite reduction + fitted polynomial, |t| <= 65536; CUDA sinf
    beyond) against float64 sin^2 of the same F32 argument t = fl(x * alpha).  With |x| <= 1
    and 1/beta = 1, y - x recovers sin^2(t) to within one rounding of y; the bound below is
    4 F32 ulp at 1 (CUDA's sinf is specified to 2 ulp, so its square to about 2.4e-7)."""
    rng = np.random.default_rng(71)
    alphas = np.array([2.0 ** k for k in range(0, 21)] + [3.7, 1234.5, 65535.0, 70000.0], np.float32)
    c, t = alphas.size, 65536
    x = rng.uniform(-1, 1, (c, t)).astype(np.float32)
    alpha = torch.from_numpy(alphas).to(dev)
    inv_beta = torch.ones(c, device=dev)
    y = ops.snakebeta_t(torch.from_numpy(x).to(dev), alpha, inv_beta, prepared=True).cpu().numpy()
    targ = (x * alphas[:, None]).astype(np.float32).astype(np.float64)  # the F32 product the kernel forms
    want = np.sin(targ) ** 2
    got = y.astype(np.float64) - x.astype(np.float64)
    err = np.abs(got - want)
    assert err.max() <= 4 * 2.0 ** -23, f"max |sin^2 error| {err.max():.3g}"
    assert (np.abs(targ) > 65536).any() and (np.abs(targ) < 65536).any()  # both paths exercised
