"""GPU parity of the Flow CFG combine and Euler update (a7, a8): bit-exact
against the oracle and against the reference's own solve_flow_euler /
combine_renderer_cfg (compiled from the reference sources; fixtures in
tests/golden/flow_ref.npz)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_cfg_known_answer(ops, dev):
    out = ops.cfg_combine_t(T(np.array([1, 2], np.float32), dev), T(np.array([3, 6], np.float32), dev), 1.5)
    assert out.cpu().tolist() == [4.0, 8.0]


@pytest.mark.parametrize("n", [1, 7, 8, 1000, 32256, 1 << 20])
def test_cfg_combine_bit_exact(ops, orc, dev, n):
    rng = np.random.default_rng(n)
    u, c = rng.standard_normal((2, n)).astype(np.float32)
    out = ops.cfg_combine_t(T(u, dev), T(c, dev), 1.5).cpu().numpy()
    assert np.array_equal(out, orc.cfg_combine(u, c, 1.5))


def test_cfg_matches_reference_fixture(ops, dev):
    d = np.load(GOLDEN / "flow_ref.npz")
    out = ops.cfg_combine_t(T(d["cfg_u"], dev), T(d["cfg_c"], dev), 1.5).cpu().numpy()
    assert np.array_equal(out, d["cfg_out"])


def test_multi_step_matches_reference_solver(ops, dev):
    d = np.load(GOLDEN / "flow_ref.npz")
    dim, inc, steps = int(d["dim"]), int(d["incontext"]), int(d["steps"])
    st = T(d["noise"], dev)
    ops.cfg_euler_multi_t(st, T(d["noise"], dev), T(d["context"], dev), T(d["uncond"], dev), T(d["cond"], dev),
                          batch=1, prefix=inc * dim, first_step=0, count=steps, steps=steps,
                          guidance=float(d["guidance"]), sigma_min=float(d["sigma_min"]))
    assert np.array_equal(st.cpu().numpy(), d["solved"])
    # pause at step 3, resume: the durable boundary is bit-exact
    st = T(d["noise"], dev)
    ops.cfg_euler_multi_t(st, T(d["noise"], dev), T(d["context"], dev), T(d["uncond"], dev), T(d["cond"], dev),
                          batch=1, prefix=inc * dim, first_step=0, count=3, steps=steps,
                          guidance=float(d["guidance"]), sigma_min=float(d["sigma_min"]))
    assert np.array_equal(st.cpu().numpy(), d["paused_state"])
    ops.cfg_euler_multi_t(st, T(d["noise"], dev), T(d["context"], dev), T(d["uncond"][3:], dev),
                          T(d["cond"][3:], dev), batch=1, prefix=inc * dim, first_step=3, count=steps - 3,
                          steps=steps, guidance=float(d["guidance"]), sigma_min=float(d["sigma_min"]))
    assert np.array_equal(st.cpu().numpy(), d["solved"])


def test_single_step_kernels_reproduce_reference_solver(ops, dev):
    """The per-step form of the real renderer: prefix interpolation, then the
    estimator (here the recorded velocities), then the fused CFG + Euler step."""
    d = np.load(GOLDEN / "flow_ref.npz")
    dim, inc, steps = int(d["dim"]), int(d["incontext"]), int(d["steps"])
    noise, ctx = T(d["noise"], dev), T(d["context"], dev)
    st = noise.clone()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for k in range(steps):
        ops.flow_incontext_t(st, noise, ctx, inc * dim, k, steps, float(d["sigma_min"]))
        assert np.array_equal(st.cpu().numpy(), d["seen"][k])  # the state the estimator sees
        ops.euler_cfg_step_t(st, T(d["uncond"][k], dev), T(d["cond"][k], dev), float(d["guidance"]), steps,
                             status=status)
    st[: inc * dim] = ctx[: inc * dim]  # final context restore (src/levo-flow-renderer.cpp:113-114)
    assert status.item() == 0
    assert np.array_equal(st.cpu().numpy(), d["solved"])


def test_euler_known_answer(ops, dev):
    # tests/test-flow-renderer.cpp:33-65
    noise = np.array([1, 2, 10, 20, 30, 40], np.float32)
    ctx = np.array([4, 8, 0, 0, 0, 0], np.float32)
    st = T(noise, dev)
    ones = T(np.ones((2, 6), np.float32), dev)
    ops.cfg_euler_multi_t(st, T(noise, dev), T(ctx, dev), ones, None, batch=1, prefix=2, first_step=0, count=2,
                          steps=2, cfg=False, sigma_min=0.1)
    assert np.allclose(st.cpu().numpy(), [4, 8, 11, 21, 31, 41], atol=1e-6, rtol=0)


@pytest.mark.parametrize("prefix_frames", [0, 1, 40])
def test_config2_full_size_bit_exact(ops, orc, dev, prefix_frames):
    # 2 windows x [64, 252] F32, 50 steps, dt 1/50, g 1.5.
    rng = np.random.default_rng(1234)
    batch, row, steps = 2, 64 * 252, 50
    x = rng.standard_normal(batch * row).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, batch * row)).astype(np.float32)
    noise = x.copy()
    ctx = rng.standard_normal(batch * row).astype(np.float32)
    st = T(x, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.cfg_euler_multi_t(st, T(noise, dev), T(ctx, dev), T(vu, dev), T(vc, dev), batch=batch,
                          prefix=prefix_frames * 64, first_step=0, count=steps, steps=steps, guidance=1.5,
                          sigma_min=1e-4, status=status)
    want, ok = orc.cfg_euler(x, noise, ctx, vu, vc, batch=batch, prefix=prefix_frames * 64, first_step=0,
                             count=steps, steps=steps, guidance=1.5, sigma_min=1e-4)
    assert ok and status.item() == 0
    assert np.array_equal(st.cpu().numpy(), want)


def test_no_cfg_path(ops, orc, dev):
    rng = np.random.default_rng(3)
    n, steps = 5000, 4
    x = rng.standard_normal(n).astype(np.float32)
    vu = rng.standard_normal((steps, n)).astype(np.float32)
    st = T(x, dev)
    ops.cfg_euler_multi_t(st, None, None, T(vu, dev), None, batch=1, prefix=0, first_step=0, count=steps,
                          steps=steps, cfg=False)
    want, _ = orc.cfg_euler(x, None, None, vu, None, batch=1, prefix=0, first_step=0, count=steps, steps=steps,
                            cfg=False)
    assert np.array_equal(st.cpu().numpy(), want)
    st2 = T(x, dev)
    for k in range(steps):
        ops.euler_cfg_step_t(st2, T(vu[k], dev), None, 1.0, steps, cfg=False)
    assert np.array_equal(st2.cpu().numpy(), want)


def test_nonfinite_velocity_sets_status(ops, dev):
    # The reference throws on a non-finite velocity / state (src/levo-flow-renderer.cpp:104,106).
    n = 64
    st = torch.zeros(n, device=dev)
    vu = torch.ones((3, n), device=dev)
    vu[1, 5] = float("inf")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.cfg_euler_multi_t(st, None, None, vu, vu, batch=1, prefix=0, first_step=0, count=3, steps=3,
                          status=status)
    assert status.item() & 1
    status.zero_()
    ops.euler_cfg_step_t(torch.full((n,), 3e38, device=dev), torch.full((n,), 3e38, device=dev), None, 1.0, 1,
                         cfg=False, status=status)
    assert status.item() == 2  # finite velocity, overflowing state
