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


def _failing_case(case, frames, dim, steps, prefix_frames, fail_step, element, seed=11):
    """Seeded inputs whose `element` fails at `fail_step`: a NaN conditional velocity, or a finite
    velocity that pushes a near-maximal state past FLT_MAX."""
    rng = np.random.default_rng(seed)
    n = frames * dim
    noise = rng.standard_normal(n).astype(np.float32)
    ctx = rng.standard_normal(n).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    if case == "velocity":
        vc[fail_step, element] = np.nan
    else:
        noise[element] = np.float32(3.39e38)
        if element >= prefix_frames * dim:  # outside the prefix the state itself starts near FLT_MAX
            vu[:fail_step, element] = 0.0
            vc[:fail_step, element] = 0.0
        vu[fail_step, element] = np.float32(3.4e38)
        vc[fail_step, element] = np.float32(3.4e38)
    return noise, ctx, vu, vc


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
@pytest.mark.parametrize("case", ["velocity", "state"])
@pytest.mark.parametrize("layout", [(252, 64, 70), (7, 5, 9)])  # staged kernel (n % 4 == 0), register kernel
@pytest.mark.parametrize("where", ["body", "prefix"])
def test_solve_stops_at_the_reference_checkpoint(ops, orc, dev, case, layout, where):
    """The first non-finite velocity or state ends the solve where the reference's solve_flow_euler throws
    (src/levo-flow-renderer.cpp:104,106): state = its checkpoint of the completed steps, bit for bit."""
    frames, dim, steps = layout
    prefix_frames = 2
    fail_step = steps - 4 if steps > 64 else 5  # past the first 64-step staging round when there is one
    element = 3 if where == "prefix" else prefix_frames * dim + 7
    if case == "state" and where == "prefix":
        fail_step = 0  # the interpolated prefix value is near FLT_MAX at step 0 only
    noise, ctx, vu, vc = _failing_case(case, frames, dim, steps, prefix_frames, fail_step, element)
    status, want, done, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc,
                                                     guidance=1.5)
    assert status == 2 and done == fail_step
    message = orc.ref_last_message()
    assert ("velocity" if case == "velocity" else "state") in message
    # the oracle restatement stops at the same checkpoint
    st_o, failure, k = orc.cfg_euler_checked(noise, noise, ctx, vu, vc, batch=1, prefix=prefix_frames * dim,
                                             first_step=0, count=steps, steps=steps)
    assert failure == case and k == fail_step and np.array_equal(st_o, want)
    st = T(noise, dev)
    with pytest.raises(ops.LevoNonFinite) as err:
        ops.cfg_euler_solve_t(st, T(noise, dev), T(ctx, dev), T(vu, dev), T(vc, dev), batch=1,
                              prefix=prefix_frames * dim, first_step=0, count=steps, steps=steps)
    assert err.value.completed_steps == fail_step
    assert f"Euler {case} contains a non-finite value (step {fail_step})" in str(err.value)
    assert np.array_equal(st.cpu().numpy(), want)


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
@pytest.mark.parametrize("which", ["noise", "in-context latent", "resume state"])
@pytest.mark.parametrize("solve", ["fused", "per-step"])
def test_solve_rejects_nonfinite_inputs_before_any_step(ops, orc, dev, which, solve):
    """solve_flow_euler checks its noise, in-context latent and resume state before the first step
    (src/levo-flow-renderer.cpp:71-72,81) and throws without stepping.  Both solve entry points do the
    same: the reference's message, completed_steps at the start, the state untouched.  The non-finite
    context value sits outside the in-context prefix, which the steps never read: only the up-front
    check sees it."""
    frames, dim, steps, pf = 7, 5, 9, 2
    n = frames * dim
    rng = np.random.default_rng(23)
    noise, ctx = rng.standard_normal((2, n)).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    first = 3 if which == "resume state" else 0
    start = noise.copy()
    if which == "noise":
        noise[n - 2] = np.nan
        start = noise.copy()
    elif which == "in-context latent":
        ctx[n - 2] = np.inf
    else:
        start = rng.standard_normal(n).astype(np.float32)
        start[n - 2] = np.nan
    message = f"Euler {which} contains a non-finite value"
    with pytest.raises(ValueError, match=message):
        orc.ref_solve_flow_euler(noise, ctx, frames, dim, pf, 1e-4, steps, vu, vc, guidance=1.5,
                                 resume_step=first if first else -1, resume_state=start if first else None)
    st = T(start, dev)
    with pytest.raises(ops.LevoNonFinite, match=message) as err:
        if solve == "fused":
            ops.cfg_euler_solve_t(st, T(noise, dev), T(ctx, dev), T(vu[first:], dev), T(vc[first:], dev), batch=1,
                                  prefix=pf * dim, first_step=first, count=steps - first, steps=steps)
        else:
            vel = T(np.stack([vu, vc], axis=1), dev)  # [steps][2][n]
            ops.flow_euler_solve_t(st, T(noise, dev), T(ctx, dev), frames=frames, latent_dim=dim,
                                   incontext_frames=pf, steps=steps, first_step=first,
                                   velocity=lambda _s, k, _t: vel[k])
    assert err.value.completed_steps == first
    assert np.array_equal(st.cpu().numpy(), start, equal_nan=True)


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
@pytest.mark.parametrize("layout", [(252, 64, 70), (7, 5, 9)])
def test_solve_velocity_failure_wins_a_tie_with_a_state_failure(ops, orc, dev, layout):
    """At one step, a non-finite velocity in one element and a state overflow in another: the reference
    checks the whole velocity first (src/levo-flow-renderer.cpp:104), so the velocity failure is the one
    reported."""
    frames, dim, steps = layout
    prefix_frames = 1
    fail_step = steps - 3
    state_element, velocity_element = prefix_frames * dim + 5, prefix_frames * dim + 11
    noise, ctx, vu, vc = _failing_case("state", frames, dim, steps, prefix_frames, fail_step, state_element)
    vc[fail_step, velocity_element] = np.nan
    status, want, done, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc,
                                                     guidance=1.5)
    assert status == 2 and done == fail_step and "velocity" in orc.ref_last_message()
    st = T(noise, dev)
    with pytest.raises(ops.LevoNonFinite) as err:
        ops.cfg_euler_solve_t(st, T(noise, dev), T(ctx, dev), T(vu, dev), T(vc, dev), batch=1,
                              prefix=prefix_frames * dim, first_step=0, count=steps, steps=steps)
    assert err.value.completed_steps == fail_step
    assert f"Euler velocity contains a non-finite value (step {fail_step})" in str(err.value)
    assert np.array_equal(st.cpu().numpy(), want)


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
def test_solve_resumed_after_a_pause_stops_at_the_same_checkpoint(ops, orc, dev):
    frames, dim, steps, prefix_frames, fail_step = 252, 64, 12, 1, 9
    noise, ctx, vu, vc = _failing_case("velocity", frames, dim, steps, prefix_frames, fail_step, 100)
    _, want, done, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc)
    assert done == fail_step
    st = T(noise, dev)
    assert ops.cfg_euler_solve_t(st, T(noise, dev), T(ctx, dev), T(vu, dev), T(vc, dev), batch=1,
                                 prefix=prefix_frames * dim, first_step=0, count=4, steps=steps) == 4
    with pytest.raises(ops.LevoNonFinite) as err:
        ops.cfg_euler_solve_t(st, T(noise, dev), T(ctx, dev), T(vu[4:], dev), T(vc[4:], dev), batch=1,
                              prefix=prefix_frames * dim, first_step=4, count=steps - 4, steps=steps)
    assert err.value.completed_steps == fail_step
    assert np.array_equal(st.cpu().numpy(), want)


def test_solve_without_failure_equals_the_fused_kernel(ops, orc, dev):
    rng = np.random.default_rng(5)
    batch, row, steps = 2, 64 * 252, 50
    x = rng.standard_normal(batch * row).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, batch * row)).astype(np.float32)
    ctx = rng.standard_normal(batch * row).astype(np.float32)
    st = T(x, dev)
    assert ops.cfg_euler_solve_t(st, T(x, dev), T(ctx, dev), T(vu, dev), T(vc, dev), batch=batch, prefix=64,
                                 first_step=0, count=steps, steps=steps) == steps
    want, ok = orc.cfg_euler(x, x, ctx, vu, vc, batch=batch, prefix=64, first_step=0, count=steps, steps=steps)
    assert ok and np.array_equal(st.cpu().numpy(), want)


@pytest.mark.parametrize("layout", [(252, 64, 70), (7, 5, 9)])
def test_multi_step_status_records_the_first_failing_step(ops, orc, dev, layout):
    """levo_cfg_euler_multi_f32 alone: the status word holds the earliest failing step (velocity kind on a
    tie), and each failing element keeps its state after the last step it completed."""
    frames, dim, steps = layout
    n = frames * dim
    fail_step = steps - 2
    noise, ctx, vu, vc = _failing_case("velocity", frames, dim, steps, 0, fail_step, 9)
    vu[fail_step - 1, 20] = np.float32(3.4e38)  # element 20: state overflow one step earlier
    vc[fail_step - 1, 20] = np.float32(3.4e38)
    noise[20] = np.float32(3.39e38)
    vu[: fail_step - 1, 20] = 0.0
    vc[: fail_step - 1, 20] = 0.0
    st = T(noise, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.cfg_euler_multi_t(st, None, None, T(vu, dev), T(vc, dev), batch=1, prefix=0, first_step=0, count=steps,
                          steps=steps, status=status)
    word = int(status.item())
    assert ops.euler_status_step(word) == fail_step - 1 and word & 3 == ops.EULER_FAIL_STATE
    got = st.cpu().numpy()
    for e, k in ((9, fail_step), (20, fail_step - 1)):
        one, _, _ = orc.cfg_euler_checked(noise[e:e + 1], None, None, vu[:, e:e + 1], vc[:, e:e + 1], batch=1,
                                          prefix=0, first_step=0, count=k, steps=steps)
        assert got[e] == one[0]
    # every other element ran all steps
    others = np.setdiff1d(np.arange(n), [9, 20])
    full, ok = orc.cfg_euler(noise[others], None, None, vu[:, others], vc[:, others], batch=1, prefix=0,
                             first_step=0, count=steps, steps=steps)
    assert ok and np.array_equal(got[others], full)


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
@pytest.mark.parametrize("case", ["none", "velocity", "state"])
def test_per_step_solve_matches_the_reference(ops, orc, dev, case):
    """levo_flow_euler_solve_f32 with a velocity callback (the estimator's place) against the reference's
    solve_flow_euler: the states the estimator sees, the solved state, and on a non-finite velocity or
    state the reference's checkpoint and step, all bit for bit."""
    frames, dim, steps, prefix_frames, fail = 252, 64, 12, 2, 7
    if case == "none":
        rng = np.random.default_rng(21)
        n = frames * dim
        noise, ctx = rng.standard_normal((2, n)).astype(np.float32)
        vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    else:
        noise, ctx, vu, vc = _failing_case(case, frames, dim, steps, prefix_frames, fail, prefix_frames * dim + 5)
    status, want, done, seen = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc,
                                                        want_seen=True)
    VU, VC = T(vu, dev), T(vc, dev)
    got_seen = []

    def velocity(state, step, time):
        got_seen.append(state.cpu().numpy().copy())
        return torch.stack([VU[step], VC[step]])

    st = T(noise, dev)
    kw = dict(frames=frames, latent_dim=dim, incontext_frames=prefix_frames, steps=steps, velocity=velocity)
    if case == "none":
        assert status == 0
        assert ops.flow_euler_solve_t(st, T(noise, dev), T(ctx, dev), **kw) == steps
    else:
        assert status == 2 and done == fail
        with pytest.raises(ops.LevoNonFinite) as err:
            ops.flow_euler_solve_t(st, T(noise, dev), T(ctx, dev), **kw)
        assert err.value.completed_steps == fail and f"Euler {case} contains" in str(err.value)
    assert np.array_equal(st.cpu().numpy(), want)
    ran = steps if case == "none" else fail + 1
    assert len(got_seen) == ran
    for k in range(ran):
        assert np.array_equal(got_seen[k], seen[k]), k


@pytest.mark.skipif("not __import__('levo_oracle').ref_available()")
def test_per_step_solve_cancel_and_resume(ops, orc, dev):
    """A cancellation before step 4 leaves the reference's pause checkpoint; resuming from it finishes
    with the reference's solved state."""
    frames, dim, steps, prefix_frames = 100, 64, 9, 3
    rng = np.random.default_rng(8)
    n = frames * dim
    noise, ctx = rng.standard_normal((2, n)).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    status, paused, done, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc,
                                                       pause_after=4)
    assert status == 1 and done == 4
    _, solved, _, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, prefix_frames, 1e-4, steps, vu, vc)
    VU, VC = T(vu, dev), T(vc, dev)
    polls = []

    def cancel():
        polls.append(1)
        return len(polls) > 4

    st = T(noise, dev)
    kw = dict(frames=frames, latent_dim=dim, incontext_frames=prefix_frames, steps=steps,
              velocity=lambda s, k, t: torch.stack([VU[k], VC[k]]))
    with pytest.raises(ops.LevoCancelled) as err:
        ops.flow_euler_solve_t(st, T(noise, dev), T(ctx, dev), cancel=cancel, **kw)
    assert err.value.completed_steps == 4
    assert np.array_equal(st.cpu().numpy(), paused)
    assert ops.flow_euler_solve_t(st, T(noise, dev), T(ctx, dev), first_step=4, **kw) == steps
    assert np.array_equal(st.cpu().numpy(), solved)
