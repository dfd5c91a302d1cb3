"""ctypes wrapper of the parity oracle (TEST INFRASTRUCTURE ONLY).

liblevo_oracle.so is the C restatement (levo_oracle.c); _ref/libref_levo.so is
the reference's own GGML-free renderer code (built only where the reference
tree exists).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline use this module, and only as the checker / the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import pathlib
from typing import Optional

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liblevo_oracle.so"
REF_LIB = HERE / "_ref" / "libref_levo.so"

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_INT = ctypes.c_int

_SIGS = {
    "oracle_snakebeta_f32": [_P, _P, _P, _P, _I64, _I64, _INT],
    "oracle_snakebeta_f16params": [_P, _P, _P, _P, _I64, _I64, _INT],
    "oracle_channel_bias_add_f32": [_P, _P, _P, _I64, _I64, _INT],
    "oracle_fused_unit_f32": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _INT, _INT],
    "oracle_conv_standin_f32": [_P, _I64, _I64, _P, _I64, _I64, _INT],
    "oracle_vae_chain_f32": [_P, _P, _P, _I64, _P, _INT, _INT],
    "oracle_vae_chain_stages_f32": [_P, _P, _P, _I64, _P, _INT, _INT, _P],
    "oracle_add_rmsnorm_f16": [_P, _P, _P, _P, _P, _I64, _I64, _F, _INT, _INT],
    "oracle_add_rmsnorm_f32": [_P, _P, _P, _P, _P, _I64, _I64, _F, _INT],
    "oracle_add_layernorm_f16": [_P, _P, _P, _P, _P, _P, _I64, _I64, _F, _INT, _INT],
    "oracle_add_layernorm_f32": [_P, _P, _P, _P, _P, _P, _I64, _I64, _F, _INT],
    "oracle_weightnorm_f32": [_P, _P, _P, _P, _I64, _I64, _INT],
    "oracle_cfg_combine_f32": [_P, _P, _P, _I64, _F],
    "oracle_gated_layernorm_modulate_f32": [_P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _F],
    "oracle_assemble_windows_f32": [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P],
    "oracle_greedy_tokens_f32": [_P, _I64, _I64, _P, _I64, _F, _I64, _P, _I64, _P],
    "oracle_latent_to_vae_f32": [_P, _P, _P, _I64, _I64, _P],
    "oracle_latent_normalize_f32": [_P, _P, _P, _I64, _I64, _P],
    "oracle_cfg_euler_f32": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _INT, _F, _F,
                             ctypes.POINTER(_I64)],
}

_REF_SIGS = {
    "ref_last_error": (ctypes.c_char_p, []),
    "ref_sample_streams_greedy": (_INT, [_P, _I64, _I64, _P, _I64, _F, _P, _I64, _P]),
    "ref_apply_cfg": (_INT, [_P, _P, _I64, _F, _P]),
    "ref_combine_renderer_cfg": (_INT, [_P, _P, _I64, _F, _P]),
    "ref_solve_flow_euler": (_INT, [_P, _P, _I64, _I64, _I64, _F, _I64, _P, _P, _INT, _F, _I64, _P, _I64, _P, _P,
                                    ctypes.POINTER(_I64)]),
    "ref_make_renderer_schedule": (_INT, [_I64, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                                          _P, _I64]),
    "ref_assemble_renderer_audio": (_INT, [_I64, _P, _P, _P, _P]),
    "ref_make_renderer_euler_schedule": (_INT, [_I64, _P, ctypes.POINTER(_F)]),
}

_lib = None
_ref = None

# --------------------------------------------------------------------------- reference decoder topology
# The reference's Oobleck decoder, restated on the test side (independent of liblevo_b200):
#   input conv latent_dim -> 2048 with bias        src/levo-vae-model.cpp:172
#   stage output widths 1024, 512, 256, 128, 128   src/levo-vae-model.cpp:174
#   strides 10, 6, 4, 4, 2                         src/levo-vae-model.cpp:175, src/levo-vae.cpp:215
#   3 residual units per stage, dilations 1, 3, 9  src/levo-vae-model.cpp:181, src/levo-vae.cpp:216
#   output snake on 128 channels, conv to 2 audio channels without bias   src/levo-vae-model.cpp:190-191
# latent_dim 64 and 2 audio channels are the VAE hyper-parameters the reference validates.
# Flat form, as vae_chain takes it: latent_dim, audio_channels, entry_width, S, widths[S], strides[S], R.
REFERENCE_TOPOLOGY = (64, 2, 2048, 5, 1024, 512, 256, 128, 128, 10, 6, 4, 4, 2, 3)
REFERENCE_DILATIONS = (1, 3, 9)


def topology_fields(topology) -> dict:
    t = [int(v) for v in topology]
    s = t[3]
    return {"latent_dim": t[0], "audio_channels": t[1], "entry_width": t[2], "n_stages": s,
            "widths": t[4:4 + s], "strides": t[4 + s:4 + 2 * s], "n_residual": t[4 + 2 * s]}


def param_count(topology) -> int:
    """Elementwise parameters of the decoder in the reference's tensor-inventory order
    (src/levo-vae-model.cpp:172-191): input bias; per stage the upsample snake (2 x Cin),
    upsample bias, and per residual unit pre snake, conv.0 bias, post snake, conv.1 bias;
    the output snake."""
    f = topology_fields(topology)
    n, cin = f["entry_width"], f["entry_width"]
    for c in f["widths"]:
        n += 2 * cin + c + 6 * c * f["n_residual"]
        cin = c
    return n + 2 * cin


def upsampling(topology) -> int:
    out = 1
    for s in topology_fields(topology)["strides"]:
        out *= s
    return out


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            raise RuntimeError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        h = ctypes.CDLL(str(ORACLE_LIB))
        for name, args in _SIGS.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = None if name in ("oracle_conv_standin_f32", "oracle_latent_to_vae_f32",
                                          "oracle_latent_normalize_f32") else _INT
        _lib = h
    return _lib


def ref_available() -> bool:
    return REF_LIB.exists()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"{REF_LIB} missing: the reference tree was not present at build time")
        h = ctypes.CDLL(str(REF_LIB))
        for name, (res, args) in _REF_SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _ref = h
    return _ref


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------- oracle (C restatement)

def snakebeta(x, alpha_log, beta_log, threads: int = 0) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    if np.asarray(alpha_log).dtype == np.float16:
        a = np.ascontiguousarray(alpha_log, dtype=np.float16).view(np.uint16)
        b = np.ascontiguousarray(beta_log, dtype=np.float16).view(np.uint16)
        rc = lib().oracle_snakebeta_f16params(_p(x), _p(a), _p(b), _p(y), x.shape[0], x.shape[1], threads)
    else:
        a, b = _f32(alpha_log), _f32(beta_log)
        rc = lib().oracle_snakebeta_f32(_p(x), _p(a), _p(b), _p(y), x.shape[0], x.shape[1], threads)
    assert rc == 0
    return y


def channel_bias_add(x, bias, threads: int = 0) -> np.ndarray:
    x, bias = _f32(x), _f32(bias)
    y = np.empty_like(x)
    assert lib().oracle_channel_bias_add_f32(_p(x), _p(bias), _p(y), x.shape[0], x.shape[1], threads) == 0
    return y


def fused_unit(u, bias=None, residual=None, alpha_log=None, beta_log=None, tanh=False, threads: int = 0):
    """Returns (x, y) of the fused decoder unit expressed as separate reference nodes."""
    u = _f32(u)
    args = [None if a is None else _f32(a) for a in (bias, residual, alpha_log, beta_log)]
    x = np.empty_like(u)
    y = np.empty_like(u)
    rc = lib().oracle_fused_unit_f32(_p(u), *[_p(a) for a in args], _p(x), _p(y), u.shape[0], u.shape[1],
                                     1 if tanh else 0, threads)
    assert rc == 0
    return x, y


def conv_standin(x, cout: int, lout: int, stride: int) -> np.ndarray:
    x = _f32(x)
    out = np.empty((cout, lout), dtype=np.float32)
    lib().oracle_conv_standin_f32(_p(x), x.shape[0], x.shape[1], _p(out), cout, lout, stride)
    return out


def vae_chain(topology_list, params, latent, frames: int, audio_channels: int, samples: int, tanh=False,
              threads: int = 0, stages: bool = False):
    """Audio [audio_channels][samples]; with stages=True also the list of stage outputs."""
    topo = np.ascontiguousarray(topology_list, dtype=np.int32)
    params, latent = _f32(params), _f32(latent)
    audio = np.empty((audio_channels, samples), dtype=np.float32)
    if not stages:
        rc = lib().oracle_vae_chain_f32(_p(topo), _p(params), _p(latent), frames, _p(audio), 1 if tanh else 0,
                                        threads)
        assert rc == 0
        return audio
    n_stages = int(topo[3])
    widths, strides = topo[4:4 + n_stages], topo[4 + n_stages:4 + 2 * n_stages]
    outs, length = [], frames
    for w, s in zip(widths, strides):
        length *= int(s)
        outs.append(np.empty((int(w), length), dtype=np.float32))
    ptrs = (ctypes.c_void_p * n_stages)(*[o.ctypes.data for o in outs])
    rc = lib().oracle_vae_chain_stages_f32(_p(topo), _p(params), _p(latent), frames, _p(audio), 1 if tanh else 0,
                                           threads, ctypes.cast(ptrs, ctypes.c_void_p))
    assert rc == 0
    return audio, outs


def _norm(layer: bool, x, r, gamma, beta, eps, f16_boundary, threads):
    half = x.dtype == np.float16
    rows, dim = x.shape
    gamma = _f32(gamma)
    beta = _f32(beta) if beta is not None else None
    if half:
        xb = np.ascontiguousarray(x).view(np.uint16)
        rb = None if r is None else np.ascontiguousarray(r, dtype=np.float16).view(np.uint16)
        h = np.empty((rows, dim), np.uint16)
        y = np.empty((rows, dim), np.uint16)
        if layer:
            rc = lib().oracle_add_layernorm_f16(_p(xb), _p(rb), _p(gamma), _p(beta), _p(h), _p(y), rows, dim, eps,
                                                1 if f16_boundary else 0, threads)
        else:
            rc = lib().oracle_add_rmsnorm_f16(_p(xb), _p(rb), _p(gamma), _p(h), _p(y), rows, dim, eps,
                                              1 if f16_boundary else 0, threads)
        assert rc == 0
        return h.view(np.float16), y.view(np.float16)
    xf = _f32(x)
    rf = None if r is None else _f32(r)
    h = np.empty_like(xf)
    y = np.empty_like(xf)
    if layer:
        rc = lib().oracle_add_layernorm_f32(_p(xf), _p(rf), _p(gamma), _p(beta), _p(h), _p(y), rows, dim, eps, threads)
    else:
        rc = lib().oracle_add_rmsnorm_f32(_p(xf), _p(rf), _p(gamma), _p(h), _p(y), rows, dim, eps, threads)
    assert rc == 0
    return h, y


def add_rmsnorm(x, r, gamma, eps, f16_boundary=False, threads: int = 0):
    return _norm(False, x, r, gamma, None, eps, f16_boundary, threads)


def add_layernorm(x, r, gamma, beta, eps, f16_boundary=False, threads: int = 0):
    return _norm(True, x, r, gamma, beta, eps, f16_boundary, threads)


def gated_layernorm_modulate(x, gate, r, gamma, beta, scale, shift, batch_rows, eps=1e-5):
    x = _f32(x)
    f = lambda a: None if a is None else _f32(a)  # noqa: E731
    gate, r, gamma, beta, scale, shift = map(f, (gate, r, gamma, beta, scale, shift))
    h = np.empty_like(x)
    y = np.empty_like(x)
    rc = lib().oracle_gated_layernorm_modulate_f32(_p(x), _p(gate), _p(r), _p(gamma), _p(beta), _p(scale), _p(shift),
                                                   batch_rows, _p(h), _p(y), x.shape[0], x.shape[1], eps)
    assert rc == 0
    return h, y


def weightnorm(v, g, threads: int = 0):
    """Returns (w, norms, ok) where ok is False when a row norm is zero."""
    v = _f32(v)
    rows = v.shape[0]
    cols = v.size // max(rows, 1)
    g = _f32(g).reshape(-1)
    w = np.empty_like(v)
    norms = np.empty(rows, dtype=np.float32)
    rc = lib().oracle_weightnorm_f32(_p(v), _p(g), _p(w), _p(norms), rows, cols, threads)
    assert rc in (0, -1)
    return w, norms, rc == 0


def cfg_combine(u, c, g) -> np.ndarray:
    u, c = _f32(u), _f32(c)
    out = np.empty_like(u)
    assert lib().oracle_cfg_combine_f32(_p(u), _p(c), _p(out), u.size, g) == 0
    return out


def cfg_euler_checked(state, noise, context, uncond, cond, *, batch, prefix, first_step, count, steps, cfg=True,
                      guidance=1.5, sigma_min=1e-4):
    """Returns (state_after, failure, failed_step): failure is None, "velocity" or "state"; on a
    failure state_after is the checkpoint of the steps completed before failed_step."""
    st = _f32(state).copy()
    n = st.size
    nz = _f32(noise) if noise is not None else np.zeros(n, np.float32)
    cx = _f32(context) if context is not None else np.zeros(n, np.float32)
    u = _f32(uncond) if uncond is not None else np.zeros(1, np.float32)
    c = _f32(cond) if (cond is not None and cfg) else None
    failed = _I64(-1)
    rc = lib().oracle_cfg_euler_f32(_p(st), _p(nz), _p(cx), _p(u), _p(c), batch, n // batch, prefix, first_step,
                                    count, steps, 1 if cfg else 0, guidance, sigma_min, ctypes.byref(failed))
    assert rc in (0, -1, -3)
    return st, {0: None, -1: "velocity", -3: "state"}[rc], failed.value


def cfg_euler(state, noise, context, uncond, cond, *, batch, prefix, first_step, count, steps, cfg=True,
              guidance=1.5, sigma_min=1e-4):
    """Returns (state_after, ok)."""
    st, failure, _ = cfg_euler_checked(state, noise, context, uncond, cond, batch=batch, prefix=prefix,
                                       first_step=first_step, count=count, steps=steps, cfg=cfg,
                                       guidance=guidance, sigma_min=sigma_min)
    return st, failure is None


def assemble_windows(windows, hop, overlap, target) -> np.ndarray:
    w = _f32(windows)
    n, c, s = w.shape
    out = np.empty((c, target), np.float32)
    assert lib().oracle_assemble_windows_f32(_p(w), n, c, s, hop, overlap, target, _p(out)) == 0
    return out


def greedy_tokens(logits, recent=None, penalty=1.0, penalty_limit=0, ignore=None):
    """Returns (tokens, ok); ok is False when a logit is NaN."""
    x = _f32(logits)
    rows, vocab = x.shape
    rec = None if recent is None else np.ascontiguousarray(recent, dtype=np.int64)
    ign = None if ignore is None else np.ascontiguousarray(ignore, dtype=np.int64)
    out = np.empty(rows, np.int64)
    rc = lib().oracle_greedy_tokens_f32(_p(x), rows, vocab, _p(rec), 0 if rec is None else rec.shape[1], penalty,
                                        penalty_limit, _p(ign), 0 if ign is None else ign.size, _p(out))
    assert rc in (0, -1)
    return out, rc == 0


def latent_to_vae(frame_major, mean=None, stddev=None) -> np.ndarray:
    x = _f32(frame_major)
    frames, dim = x.shape
    out = np.empty((dim, frames), np.float32)
    m = None if mean is None else _f32(mean)
    s = None if stddev is None else _f32(stddev)
    lib().oracle_latent_to_vae_f32(_p(x), _p(m), _p(s), frames, dim, _p(out))
    return out


def latent_normalize(raw, mean, stddev) -> np.ndarray:
    x = _f32(raw)
    out = np.empty_like(x)
    lib().oracle_latent_normalize_f32(_p(x), _p(_f32(mean)), _p(_f32(stddev)), x.shape[0], x.shape[1], _p(out))
    return out


# --------------------------------------------------------------------------- reference (compiled sources)

def _ref_err() -> str:
    m = ref().ref_last_error()
    return m.decode() if m else ""


def ref_combine_renderer_cfg(u, c, g) -> np.ndarray:
    u, c = _f32(u), _f32(c)
    out = np.empty_like(u)
    if ref().ref_combine_renderer_cfg(_p(u), _p(c), u.size, g, _p(out)) != 0:
        raise ValueError(_ref_err())
    return out


def ref_solve_flow_euler(noise, context, frames, latent_dim, incontext_frames, sigma_min, steps, uncond, cond,
                         cfg=True, guidance=1.5, resume_step=-1, resume_state=None, pause_after=-1,
                         want_seen=False):
    """Returns (status, state, completed_steps, seen) — status 0 solved, 1 paused, 2 stopped by a
    non-finite velocity or state (state = the reference's checkpoint, message in ref_last_message())."""
    n = frames * latent_dim
    noise, context, uncond = _f32(noise), _f32(context), _f32(uncond)
    cond = _f32(cond) if cond is not None else uncond
    rs = _f32(resume_state) if resume_state is not None else None
    seen = np.zeros((steps, n), np.float32) if want_seen else None
    out = np.empty(n, np.float32)
    done = _I64(0)
    rc = ref().ref_solve_flow_euler(_p(noise), _p(context), frames, latent_dim, incontext_frames, sigma_min, steps,
                                    _p(uncond), _p(cond), 1 if cfg else 0, guidance, resume_step, _p(rs),
                                    pause_after, _p(seen), _p(out), ctypes.byref(done))
    if rc == -2:
        return 2, out, done.value, seen
    if rc < 0:
        raise ValueError(_ref_err())
    return rc, out, done.value, seen


def ref_last_message() -> str:
    return _ref_err()


def ref_make_renderer_schedule(source_frames: int, max_windows: int = 4096):
    pf, ts, nw = _I64(), _I64(), _I64()
    desc = np.zeros((max_windows, 5), np.int64)
    if ref().ref_make_renderer_schedule(source_frames, ctypes.byref(pf), ctypes.byref(ts), ctypes.byref(nw),
                                        _p(desc), max_windows) != 0:
        raise ValueError(_ref_err())
    return {"padded_frames": pf.value, "target_samples": ts.value, "windows": desc[: nw.value].copy()}


def ref_assemble_renderer_audio(source_frames: int, left, right):
    sched = ref_make_renderer_schedule(source_frames)
    left, right = _f32(left), _f32(right)
    ol = np.empty(sched["target_samples"], np.float32)
    orr = np.empty(sched["target_samples"], np.float32)
    if ref().ref_assemble_renderer_audio(source_frames, _p(left), _p(right), _p(ol), _p(orr)) != 0:
        raise ValueError(_ref_err())
    return ol, orr


def ref_make_renderer_euler_schedule(steps: int):
    times = np.empty(steps + 1, np.float32)
    dt = _F()
    if ref().ref_make_renderer_euler_schedule(steps, _p(times), ctypes.byref(dt)) != 0:
        raise ValueError(_ref_err())
    return times, dt.value


def ref_sample_streams_greedy(logits, recent=None, penalty=1.0, ignore=None):
    """The reference's Sampler::sample_streams(use_sampling=False): penalty over each full
    recent row (window = its length), ignore list on stream 0, vocabulary limit = vocab - 1."""
    x = _f32(logits)
    rows, vocab = x.shape
    rec = None if recent is None else np.ascontiguousarray(recent, dtype=np.int64)
    ign = None if ignore is None else np.ascontiguousarray(ignore, dtype=np.int64)
    out = np.empty(rows, np.int64)
    if ref().ref_sample_streams_greedy(_p(x), rows, vocab, _p(rec), 0 if rec is None else rec.shape[1], penalty,
                                       _p(ign), 0 if ign is None else ign.size, _p(out)) != 0:
        raise ValueError(_ref_err())
    return out


def ref_apply_cfg(cond, uncond, scale):
    c, u = _f32(cond), _f32(uncond)
    out = np.empty_like(c)
    if ref().ref_apply_cfg(_p(c), _p(u), c.size, scale, _p(out)) != 0:
        raise ValueError(_ref_err())
    return out
