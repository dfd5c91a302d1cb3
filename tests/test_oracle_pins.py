"""Pins the CPU oracle (oracle/levo_oracle.c) against the reference.

Sources of truth, in order of strength:
  * the reference's own code compiled from its sources (oracle/_ref: the CFG
    combine, the Euler solver and the window schedule);
  * fixtures produced by the reference's Python converters (weight norm);
  * the reference's known-answer tests, restated here value for value.
RMSNorm / LayerNorm have no reference numeric test (parity unpinned); they are
checked against their defining formulas in float64.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, UPSTREAM_NORM_CASES, assert_close, assert_upstream_gates, upstream_norm_case


# --------------------------------------------------------------------------- SnakeBeta

def test_snakebeta_known_answer(orc):
    # tests/test-audio-ops.cpp:163-215 (CPU tolerance 1e-6, F16 parameters 2e-3)
    d = np.load(GOLDEN / "snakebeta_kat.npz")
    y = orc.snakebeta(d["x"], d["alpha_log"], d["beta_log"], threads=1)
    assert np.max(np.abs(y - d["y"])) <= 1e-6
    y16 = orc.snakebeta(d["x"], d["alpha_log"].astype(np.float16), d["beta_log"].astype(np.float16), threads=1)
    assert np.max(np.abs(y16 - d["y"])) <= 2e-3


def test_snakebeta_matches_definition(orc):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 333)).astype(np.float32) * 3
    a = (0.1 * rng.standard_normal(5)).astype(np.float32)
    b = (0.1 * rng.standard_normal(5)).astype(np.float32)
    y = orc.snakebeta(x, a, b, threads=3)
    xd = x.astype(np.float64)
    want = xd + np.sin(xd * np.exp(a.astype(np.float64))[:, None]) ** 2 / (np.exp(b.astype(np.float64)) + 1e-9)[:, None]
    assert_close(y, want, 1e-6, "snake vs float64 definition")


def test_snakebeta_threads_do_not_change_values(orc):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((7, 1001)).astype(np.float32)
    a = (0.1 * rng.standard_normal(7)).astype(np.float32)
    b = (0.1 * rng.standard_normal(7)).astype(np.float32)
    assert np.array_equal(orc.snakebeta(x, a, b, threads=1), orc.snakebeta(x, a, b, threads=4))


def test_fused_unit_is_the_node_sequence(orc):
    rng = np.random.default_rng(3)
    u, r = rng.standard_normal((2, 4, 50)).astype(np.float32)
    b = rng.standard_normal(4).astype(np.float32)
    a = (0.1 * rng.standard_normal(4)).astype(np.float32)
    bl = (0.1 * rng.standard_normal(4)).astype(np.float32)
    x, y = orc.fused_unit(u, b, r, a, bl)
    xx = r + (u + b[:, None])  # residual + (conv + bias), src/levo-vae.cpp:100
    assert np.array_equal(x, xx)
    assert np.array_equal(y, orc.snakebeta(xx, a, bl))
    _, yt = orc.fused_unit(u, b, r, a, bl, tanh=True)
    assert_close(yt, np.tanh(y.astype(np.float64)), 1e-6)


# --------------------------------------------------------------------------- weight norm

def test_weightnorm_known_answers(orc):
    # tests/python/test_vae_converter.py:44-52 (transpose layout, norm 5 and 13 -> scale 2)
    v = np.asarray([[[3, 4], [0, 0], [0, 0]], [[0, 0], [5, 12], [0, 0]]], dtype=np.float32)
    g = np.asarray([[[10]], [[26]]], dtype=np.float32)
    w, norms, ok = orc.weightnorm(v, g)
    assert ok and np.allclose(norms, [5, 13])
    assert np.allclose(w[0], v[0] * 2.0) and np.allclose(w[1], v[1] * 2.0)
    # tests/python/test_flow_converter.py:53-60
    g = np.full((1024, 1, 1), 2.0, np.float32)
    v = np.zeros((1024, 32, 1), np.float32)
    v[:, 0, 0] = 3.0
    w, _, ok = orc.weightnorm(v, g)
    assert ok and np.all(w[:, 0, 0] == 2.0) and np.count_nonzero(w[:, 1:]) == 0


def test_weightnorm_matches_reference_converters(orc):
    d = np.load(GOLDEN / "weightnorm_ref.npz")
    for name in ("conv", "transpose", "wide", "flow"):
        w, _, ok = orc.weightnorm(d[f"{name}_v"], d[f"{name}_g"])
        assert ok
        assert_close(w.reshape(d[f"{name}_w"].shape), d[f"{name}_w"], 1e-6, name)


def test_weightnorm_zero_norm_is_an_error(orc):
    v = np.ones((3, 4, 2), np.float32)
    v[1] = 0
    _, norms, ok = orc.weightnorm(v, np.ones(3, np.float32))
    assert not ok and norms[1] == 0


# --------------------------------------------------------------------------- norms (unpinned against the reference itself; anchored on the upstream modules below)

@pytest.mark.parametrize("half", [False, True])
def test_rmsnorm_matches_definition(orc, half):
    rng = np.random.default_rng(4)
    dt = np.float16 if half else np.float32
    x = rng.standard_normal((9, 300)).astype(dt)
    r = rng.standard_normal((9, 300)).astype(dt)
    g = (1 + 0.02 * rng.standard_normal(300)).astype(np.float32)
    h, y = orc.add_rmsnorm(x, r, g, 1e-6)
    hh = (x.astype(np.float32) + r.astype(np.float32)).astype(dt).astype(np.float64)
    want = hh / np.sqrt(np.mean(hh * hh, axis=1, keepdims=True) + 1e-6) * g
    assert np.array_equal(h, hh.astype(dt))
    assert_close(y.astype(np.float64), want, 2e-3 if half else 1e-5)


@pytest.mark.parametrize("half", [False, True])
def test_layernorm_matches_definition(orc, half):
    rng = np.random.default_rng(5)
    dt = np.float16 if half else np.float32
    x = (3 + rng.standard_normal((6, 2200))).astype(dt)
    r = rng.standard_normal((6, 2200)).astype(dt)
    g = (1 + 0.02 * rng.standard_normal(2200)).astype(np.float32)
    b = (0.02 * rng.standard_normal(2200)).astype(np.float32)
    _, y = orc.add_layernorm(x, r, g, b, 1e-5)
    hh = (x.astype(np.float32) + r.astype(np.float32)).astype(dt).astype(np.float64)
    mu = hh.mean(axis=1, keepdims=True)
    want = (hh - mu) / np.sqrt(((hh - mu) ** 2).mean(axis=1, keepdims=True) + 1e-5) * g + b
    assert_close(y.astype(np.float64), want, 2e-3 if half else 1e-5)


@pytest.mark.parametrize("name", UPSTREAM_NORM_CASES)
def test_norms_match_upstream_modules(orc, name):
    """The oracle against the upstream modules the reference's parity policy holds its norms to
    (Transformers' Llama RMSNorm for the LM, torch's LayerNorm for the Flow estimator;
    tests/golden/make_norm_golden.py): the reference's gates, and north_star's relative bars
    (1e-5 F32; F16 within one F16 ulp).  F16 RMSNorm is the F16-boundary form, which casts the
    normalised value to F16 before the weight multiplies it, as the upstream module does."""
    c = upstream_norm_case(name)
    w = c["w"].astype(np.float32)
    if c["layer"]:
        h, y = orc.add_layernorm(c["x"], c["r"], w, c["b"].astype(np.float32), 1e-5)
    else:
        h, y = orc.add_rmsnorm(c["x"], c["r"], w, 1e-5, f16_boundary=c["half"])
    assert np.array_equal(h, c["h"])
    assert_upstream_gates(y, c["y"], name)
    if not c["half"]:
        assert_close(y.astype(np.float64), c["y"].astype(np.float64), 1e-5, name)
    if name == "rms_f16":
        assert np.array_equal(y, c["y"])  # every value bit-identical to the upstream module's


# --------------------------------------------------------------------------- CFG + Euler

def test_cfg_known_answer(orc):
    # tests/test-renderer-pattern.cpp:88-90
    assert np.array_equal(orc.cfg_combine([1, 2], [3, 6], 1.5), np.array([4, 8], np.float32))


def test_euler_known_answer(orc):
    # tests/test-flow-renderer.cpp:33-65: 3 frames x 2 dims, 1 in-context frame,
    # sigma_min 0.1, 2 steps of constant velocity 1.
    noise = np.array([1, 2, 10, 20, 30, 40], np.float32)
    ctx = np.array([4, 8, 0, 0, 0, 0], np.float32)
    ones = np.ones((2, 6), np.float32)
    out, ok = orc.cfg_euler(noise, noise, ctx, ones, None, batch=1, prefix=2, first_step=0, count=2, steps=2,
                            cfg=False, sigma_min=0.1)
    assert ok
    assert np.allclose(out, [4, 8, 11, 21, 31, 41], atol=1e-6, rtol=0)


def test_euler_resume_is_bit_exact(orc):
    # tests/test-flow-renderer.cpp:67-93: every step is a durable restart boundary.
    rng = np.random.default_rng(6)
    n, steps = 40, 5
    noise, ctx = rng.standard_normal((2, n)).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    full, _ = orc.cfg_euler(noise, noise, ctx, vu, vc, batch=1, prefix=8, first_step=0, count=steps, steps=steps)
    for k in range(steps + 1):
        part, _ = orc.cfg_euler(noise, noise, ctx, vu[:k], vc[:k], batch=1, prefix=8, first_step=0, count=k,
                                steps=steps)
        rest, _ = orc.cfg_euler(part, noise, ctx, vu[k:], vc[k:], batch=1, prefix=8, first_step=k,
                                count=steps - k, steps=steps)
        assert np.array_equal(rest, full)


def test_euler_nonfinite_is_an_error(orc):
    n = 10
    vu = np.ones((3, n), np.float32)
    vu[1, 4] = np.nan
    _, ok = orc.cfg_euler(np.zeros(n, np.float32), None, None, vu, vu, batch=1, prefix=0, first_step=0, count=3,
                          steps=3)
    assert not ok


# --------------------------------------------------------------------------- against the compiled reference

needs_ref = pytest.mark.skipif("not __import__('__graft_entry__').load_oracle().ref_available()",
                               reason="oracle/_ref not built (reference tree absent)")


def test_oracle_euler_matches_fixture_of_reference(orc):
    d = np.load(GOLDEN / "flow_ref.npz")
    frames, dim, inc, steps = int(d["frames"]), int(d["dim"]), int(d["incontext"]), int(d["steps"])
    out, ok = orc.cfg_euler(d["noise"], d["noise"], d["context"], d["uncond"], d["cond"], batch=1, prefix=inc * dim,
                            first_step=0, count=steps, steps=steps, guidance=float(d["guidance"]),
                            sigma_min=float(d["sigma_min"]))
    assert ok and np.array_equal(out, d["solved"])
    part, _ = orc.cfg_euler(d["noise"], d["noise"], d["context"], d["uncond"], d["cond"], batch=1, prefix=inc * dim,
                            first_step=0, count=3, steps=steps, guidance=float(d["guidance"]),
                            sigma_min=float(d["sigma_min"]))
    assert np.array_equal(part, d["paused_state"])
    assert np.array_equal(orc.cfg_combine(d["cfg_u"], d["cfg_c"], 1.5), d["cfg_out"])


@needs_ref
def test_reference_euler_known_answer_states():
    import __graft_entry__ as entry

    orc = entry.load_oracle()
    noise = np.array([1, 2, 10, 20, 30, 40], np.float32)
    ctx = np.array([4, 8, 0, 0, 0, 0], np.float32)
    ones = np.ones((2, 6), np.float32)
    st, out, done, seen = orc.ref_solve_flow_euler(noise, ctx, 3, 2, 1, 0.1, 2, ones, None, cfg=False, want_seen=True)
    assert st == 0 and done == 2
    assert np.allclose(seen[0, :2], [1, 2]) and np.allclose(seen[1, :2], [2.55, 5.10], atol=1e-6)
    assert np.allclose(out, [4, 8, 11, 21, 31, 41])


@needs_ref
@pytest.mark.parametrize("inc", [0, 1, 7])
def test_oracle_euler_bit_exact_vs_reference_code(inc):
    import __graft_entry__ as entry

    orc = entry.load_oracle()
    rng = np.random.default_rng(7 + inc)
    frames, dim, steps = 12, 64, 9
    n = frames * dim
    noise, ctx = rng.standard_normal((2, n)).astype(np.float32)
    vu, vc = rng.standard_normal((2, steps, n)).astype(np.float32)
    _, want, _, _ = orc.ref_solve_flow_euler(noise, ctx, frames, dim, inc, 1e-4, steps, vu, vc, True, 1.5)
    got, ok = orc.cfg_euler(noise, noise, ctx, vu, vc, batch=1, prefix=inc * dim, first_step=0, count=steps,
                            steps=steps, guidance=1.5, sigma_min=1e-4)
    assert ok and np.array_equal(got, want)


@needs_ref
def test_reference_schedule_fixture_matches_compiled_reference():
    import __graft_entry__ as entry

    orc = entry.load_oracle()
    d = np.load(GOLDEN / "flow_ref.npz")
    for i, f in enumerate(d["sched_frames"]):
        s = orc.ref_make_renderer_schedule(int(f))
        assert s["padded_frames"] == d["sched_padded"][i]
        rows = d["sched_windows"][d["sched_windows"][:, 0] == i][:, 1:]
        assert np.array_equal(s["windows"], rows)


# --------------------------------------------------------------------------- chain oracle

def test_chain_oracle_stage_shapes_and_determinism(orc, ops):
    t = ops.Topology()
    t.latent_dim, t.audio_channels, t.entry_width, t.n_stages = 4, 2, 16, 2
    t.stage_width[0], t.stage_stride[0], t.stage_width[1], t.stage_stride[1] = 8, 3, 4, 2
    t.n_residual = 2
    n = 16 + (2 * 16 + 8 + 2 * 6 * 8) + (2 * 8 + 4 + 2 * 6 * 4) + 2 * 4
    rng = np.random.default_rng(8)
    p = (0.1 * rng.standard_normal(n)).astype(np.float32)
    lat = rng.standard_normal((4, 5)).astype(np.float32)
    a1 = orc.vae_chain(t.as_list(), p, lat, 5, 2, 30, threads=1)
    a2 = orc.vae_chain(t.as_list(), p, lat, 5, 2, 30, threads=4)
    assert a1.shape == (2, 30) and np.all(np.isfinite(a1)) and np.array_equal(a1, a2)


# --------------------------------------------------------------------------- window assembly (next item)

def test_assembly_known_answer(orc):
    # tests/test-renderer-pattern.cpp:93-108: two windows of constant 1/3 (left) and 2/4 (right)
    win, hop, ov = 1000 * 1920, 750 * 1920, 250 * 1920
    target = 1001 * 1920
    w = np.empty((2, 2, win), np.float32)
    w[0, 0], w[0, 1], w[1, 0], w[1, 1] = 1.0, 2.0, 3.0, 4.0
    out = orc.assemble_windows(w, hop, ov, target)
    assert out.shape == (2, target)
    assert abs(out[0, hop] - 1.0) < 1e-6 and abs(out[0, hop + ov - 1] - 3.0) < 1e-6
    assert abs(out[0, hop + ov] - 3.0) < 1e-6
    assert abs(out[1, 0] - 2.0) < 1e-6 and abs(out[1, -1] - 4.0) < 1e-6


@needs_ref
@pytest.mark.parametrize("source_frames", [1001, 1751])
def test_assembly_oracle_bit_exact_vs_reference_code(source_frames):
    import __graft_entry__ as entry

    orc = entry.load_oracle()
    sched = orc.ref_make_renderer_schedule(source_frames)
    n = len(sched["windows"])
    win = int(sched["windows"][0][2])
    rng = np.random.default_rng(source_frames)
    w = rng.standard_normal((n, 2, win)).astype(np.float32)
    ref_l, ref_r = orc.ref_assemble_renderer_audio(source_frames, w[:, 0], w[:, 1])
    got = orc.assemble_windows(w, 750 * 1920, 250 * 1920, sched["target_samples"])
    assert np.array_equal(got[0], ref_l) and np.array_equal(got[1], ref_r)


def test_gated_layernorm_modulate_matches_definition(orc):
    rng = np.random.default_rng(9)
    batch, frames, dim = 2, 7, 300
    x, r = rng.standard_normal((2, batch * frames, dim)).astype(np.float32)
    gate, scale, shift = rng.standard_normal((3, batch, dim)).astype(np.float32)
    gamma = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    h, y = orc.gated_layernorm_modulate(x, gate, r, gamma, beta, scale, shift, frames)
    b = np.repeat(np.arange(batch), frames)
    hh = x.astype(np.float64) * gate[b] + r
    mu = hh.mean(1, keepdims=True)
    n = (hh - mu) / np.sqrt(((hh - mu) ** 2).mean(1, keepdims=True) + 1e-5)
    want = (n * gamma + beta) * (1 + scale[b]) + shift[b]
    assert_close(h, hh, 1e-6)
    assert_close(y, want, 1e-5)


# --------------------------------------------------------------------------- greedy token selection (next item)

def test_greedy_known_answers(orc):
    # tests/test-sampling.cpp:12-15: token 2 is penalised, the EOS (last) logit is exempt
    tok, ok = orc.greedy_tokens(np.array([[9, 8, 10, 7]], np.float32), recent=np.array([[2, 3]]), penalty=2.0,
                                penalty_limit=3)
    assert ok and tok.tolist() == [0]
    # tests/test-sampling.cpp:36: greedy streams pick the first maximum per stream
    tok, ok = orc.greedy_tokens(np.array([[0, 2, 1], [1, 4, 0]], np.float32))
    assert ok and tok.tolist() == [1, 1]
    # tests/test-sampling.cpp:8: LM-side CFG uses the same combine as the renderer
    assert np.array_equal(orc.cfg_combine([1, 1], [2, 4], 1.5), np.array([2.5, 5.5], np.float32))


@needs_ref
def test_greedy_oracle_matches_reference_code():
    import __graft_entry__ as entry

    orc = entry.load_oracle()
    rng = np.random.default_rng(11)
    vocab = 16385
    for trial in range(6):
        x = rng.standard_normal((3, vocab)).astype(np.float32)
        x[:, rng.integers(0, vocab, 40)] = x.max() + 1.0  # ties at the maximum
        if trial == 3:
            x[1] = -np.inf
        recent = rng.integers(-1, vocab, (3, 50))
        ignore = rng.integers(0, vocab, 8)
        want = orc.ref_sample_streams_greedy(x, recent, 1.1, ignore)
        got, ok = orc.greedy_tokens(x, recent, 1.1, vocab - 1, ignore)
        assert ok and np.array_equal(got, want)
    u, c = rng.standard_normal((2, 999)).astype(np.float32)
    assert np.array_equal(orc.ref_apply_cfg(c, u, 1.5), orc.cfg_combine(u, c, 1.5))


def test_latent_layout_and_normalisation_definitions(orc):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((25, 64)).astype(np.float32)
    mean = rng.standard_normal(64).astype(np.float32)
    std = rng.uniform(0.5, 2.0, 64).astype(np.float32)
    assert np.array_equal(orc.latent_to_vae(x), x.T)
    den = orc.latent_to_vae(x, mean, std)
    assert np.array_equal(den, ((x * std).astype(np.float32) + mean).astype(np.float32).T)
    assert np.array_equal(orc.latent_normalize(x, mean, std), ((x - mean).astype(np.float32) / std).astype(np.float32))


def test_upstream_norm_fixture_is_what_its_generator_makes():
    """tests/golden/norms_upstream.npz holds exactly what tests/golden/make_norm_golden.py computes from the
    upstream modules (skipped where torch or transformers is missing)."""
    pytest.importorskip("transformers")
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_norm_golden", GOLDEN / "make_norm_golden.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    z = np.load(GOLDEN / "norms_upstream.npz")
    for name, dt, seed in (("rms_f32", np.float32, 11), ("rms_f16", np.float16, 12)):
        x, r, w, _, y = gen._rms(np.random.default_rng(seed), 8, 1536, dt)
        for key, val in (("x", x), ("r", r), ("w", w), ("y", y)):
            assert np.array_equal(z[f"{name}_{key}"], val), (name, key)
    for name, dt, seed in (("ln_f32", np.float32, 13), ("ln_f16", np.float16, 14)):
        x, r, w, b, _, y = gen._ln(np.random.default_rng(seed), 4, 2200, dt)
        for key, val in (("x", x), ("r", r), ("w", w), ("b", b), ("y", y)):
            assert np.array_equal(z[f"{name}_{key}"], val), (name, key)
