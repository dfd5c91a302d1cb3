"""ctypes binding of liblevo_b200.so (the C ABI of include/levo_ops.h).

The library is loaded from this package directory; there is no fallback: when
it is missing every call raises, so nothing silently runs on the CPU.  The
`*_t` helpers take torch CUDA tensors (torch is only the device-memory and
stream plumbing here) and pass raw pointers plus the current stream.

Error behaviour mirrors the reference: invalid arguments raise ValueError
(the reference throws std::invalid_argument, src/levo-audio-ops.cpp:10-12),
everything else raises LevoOpsError with the library's thread-local message.
"""
from __future__ import annotations

import ctypes
import pathlib
from typing import Optional

LIB_PATH = pathlib.Path(__file__).resolve().parent / "liblevo_b200.so"

OK, EINVAL, ELAUNCH, EUNSUPPORTED, ENONFINITE, ECANCELLED, ENOMEM, ECUDA = 0, -1, -2, -3, -4, -5, -6, -7
DTYPE_F32, DTYPE_F16, DTYPE_SNAKE_PREPARED = 0, 1, 2
FUSED_TANH = 1
NORM_F16_BOUNDARY = 1
CHAIN_TANH, CHAIN_TIMING = 1, 2
KCLASS_NAMES = ("entry", "upsample", "post", "residual", "epilogue", "conv")
CONV_INPUT, CONV_UPSAMPLE, CONV_RES0, CONV_RES1, CONV_OUTPUT = range(5)
MAX_STAGES, MAX_RESIDUALS = 8, 4


class LevoOpsError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[levo_ops {code}] {message}")
        self.code = code


class LevoCancelled(LevoOpsError):
    pass


class LevoNonFinite(LevoOpsError):
    """A finiteness check failed (LEVO_OPS_ENONFINITE): the reference throws std::runtime_error.
    For the Euler solve, `completed_steps` is the step the solve stopped at."""

    completed_steps: Optional[int] = None


class LevoNonFiniteAudio(LevoNonFinite, ValueError):
    """A decoded window given to the window assembly holds a non-finite sample: the reference's
    assemble_renderer_audio throws std::invalid_argument (src/levo-renderer-pattern.cpp:25-28,159-160)."""


class Topology(ctypes.Structure):
    _fields_ = [
        ("latent_dim", ctypes.c_int32),
        ("audio_channels", ctypes.c_int32),
        ("entry_width", ctypes.c_int32),
        ("n_stages", ctypes.c_int32),
        ("stage_width", ctypes.c_int32 * MAX_STAGES),
        ("stage_stride", ctypes.c_int32 * MAX_STAGES),
        ("n_residual", ctypes.c_int32),
        ("dilation", ctypes.c_int32 * MAX_RESIDUALS),
    ]

    def as_list(self) -> list[int]:
        """Flat integer form: latent_dim, audio_channels, entry_width, S, widths[S], strides[S], R."""
        s = self.n_stages
        return ([self.latent_dim, self.audio_channels, self.entry_width, s]
                + list(self.stage_width[:s]) + list(self.stage_stride[:s]) + [self.n_residual])

    def upsampling(self) -> int:
        f = 1
        for i in range(self.n_stages):
            f *= self.stage_stride[i]
        return f


class FusedUnit(ctypes.Structure):
    _fields_ = [
        ("u", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("alpha_log", ctypes.c_void_p),
        ("beta_log", ctypes.c_void_p),
        ("x_out", ctypes.c_void_p),
        ("y_out", ctypes.c_void_p),
        ("channels", ctypes.c_int64),
        ("time", ctypes.c_int64),
        ("param_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
    ]


class ConvCall(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("stage", ctypes.c_int32),
        ("unit", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("stride", ctypes.c_int32),
        ("padding", ctypes.c_int32),
        ("dilation", ctypes.c_int32),
        ("input", ctypes.c_void_p),
        ("in_channels", ctypes.c_int64),
        ("in_length", ctypes.c_int64),
        ("output", ctypes.c_void_p),
        ("out_channels", ctypes.c_int64),
        ("out_length", ctypes.c_int64),
        ("result", ctypes.c_void_p),
    ]


class KernelTiming(ctypes.Structure):
    _fields_ = [
        ("launches", ctypes.c_int64),
        ("milliseconds", ctypes.c_double),
        ("algorithmic_bytes", ctypes.c_double),
        ("elements", ctypes.c_double),
    ]


CONV_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ConvCall), ctypes.c_void_p)
VELOCITY_FN = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_float,
                               ctypes.c_void_p)
CANCEL_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_F = ctypes.c_float
_INT = ctypes.c_int

# name -> (restype, argtypes); every symbol include/levo_ops.h declares.
SIGNATURES = {
    "levo_ops_abi_version": (_U32, []),
    "levo_ops_last_error": (ctypes.c_char_p, []),
    "levo_snake_params_prepare": (_INT, [_P, _P, _INT, _I64, _P, _P, _P]),
    "levo_snakebeta_f32": (_INT, [_P, _I64, _P, _P, _INT, _P, _I64, _I64, _I64, _P]),
    "levo_channel_bias_add_f32": (_INT, [_P, _P, _INT, _P, _I64, _I64, _P]),
    "levo_vae_fused_unit_f32": (_INT, [ctypes.POINTER(FusedUnit), _P]),
    "levo_vae_topology_reference": (_INT, [ctypes.POINTER(Topology)]),
    "levo_vae_param_count": (_I64, [ctypes.POINTER(Topology)]),
    "levo_vae_chain_create": (_INT, [ctypes.POINTER(_P), ctypes.POINTER(Topology), _P, _I64, CONV_FN, _P, _INT]),
    "levo_vae_chain_create_f16": (_INT, [ctypes.POINTER(_P), ctypes.POINTER(Topology), _P, _I64, CONV_FN, _P, _INT]),
    "levo_vae_chain_destroy": (None, [_P]),
    "levo_vae_chain_set_stage_capture": (_INT, [_P, _P, _I32]),
    "levo_vae_chain_decode": (_INT, [_P, _P, _I64, _P, _U32, _P]),
    "levo_vae_chain_decode_windows": (_INT, [_P, _P, _I64, _I64, _P, _U32, CANCEL_FN, _P, _P]),
    "levo_vae_chains_decode_windows": (_INT, [_P, _I32, _P, _I64, _I64, _P, _U32, CANCEL_FN, _P]),
    "levo_vae_chain_timing": (_INT, [_P, ctypes.POINTER(KernelTiming), _INT]),
    "levo_conv_standin_f32": (_INT, [_P, _I64, _I64, _P, _I64, _I64, _I32, _P]),
    "levo_add_rmsnorm_f16": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _F, _U32, _P]),
    "levo_add_rmsnorm_f32": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _F, _U32, _P]),
    "levo_add_layernorm_f16": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _F, _U32, _P]),
    "levo_add_layernorm_f32": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _F, _U32, _P]),
    "levo_weightnorm_f32": (_INT, [_P, _P, _P, _P, _I64, _I64, _P]),
    "levo_cfg_combine_f32": (_INT, [_P, _P, _P, _I64, _F, _P]),
    "levo_flow_incontext_f32": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P]),
    "levo_euler_cfg_step_f32": (_INT, [_P, _P, _P, _I64, _I32, _F, _I64, _P, _P]),
    "levo_cfg_euler_multi_f32": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _F, _F, _P, _P]),
    "levo_flow_euler_solve_f32": (_INT, [_P, _P, _P, _I64, _I64, _I64, _F, _I64, _I64, _I32, _F, VELOCITY_FN, _P,
                                         CANCEL_FN, _P, _P, _P, ctypes.POINTER(_I64), _P]),
    "levo_cfg_euler_solve_f32": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _F, _F, _P, _P,
                                        ctypes.POINTER(_I64), _P]),
    "levo_gated_layernorm_modulate_f32": (_INT, [_P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _F, _P]),
    "levo_vae_decode_noalloc_f32": (_INT, [ctypes.POINTER(Topology), _P, _P, _I64, _P, CONV_FN, _P, _U32, _P]),
    "levo_greedy_tokens_f32": (_INT, [_P, _I64, _I64, _I64, _P, _I64, _F, _I64, _P, _I64, _P, _P, _P]),
    "levo_latent_to_vae_f32": (_INT, [_P, _P, _P, _I64, _I64, _P, _P, _P]),
    "levo_latent_normalize_f32": (_INT, [_P, _P, _P, _I64, _I64, _P, _P, _P]),
    "levo_assemble_windows_f32": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I32, _P, _P]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads liblevo_b200.so (raises when it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise LevoOpsError(ECUDA, f"{LIB_PATH} is missing; build it with __graft_entry__.build()")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().levo_ops_last_error()
    return msg.decode() if msg else ""


def check(code: int) -> None:
    if code == OK:
        return
    msg = last_error()
    if code == EINVAL:
        raise ValueError(msg)
    if code == ECANCELLED:
        raise LevoCancelled(code, msg)
    if code == ENONFINITE:
        raise LevoNonFinite(code, msg)
    raise LevoOpsError(code, msg)


# ---------------------------------------------------------------------------
# torch convenience layer (device memory + current stream)
# ---------------------------------------------------------------------------

def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("levo_b200 ops take CUDA tensors")


def _pdtype(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.float16:
        return DTYPE_F16
    raise ValueError("parameters must be float32 or float16")


def snake_params_prepare_t(alpha_log, beta_log):
    """Returns (alpha, inv_beta) F32 [channels]: exp(alpha_log) and 1/(exp(beta_log)+1e-9),
    for snakebeta_t(..., prepared=True) and fused units with DTYPE_SNAKE_PREPARED."""
    import torch

    _require_cuda(alpha_log, beta_log)
    if alpha_log.dtype != beta_log.dtype or alpha_log.numel() != beta_log.numel():
        raise ValueError("alpha_log and beta_log must share a dtype and a channel count")
    alpha = torch.empty(alpha_log.numel(), dtype=torch.float32, device=alpha_log.device)
    inv_beta = torch.empty_like(alpha)
    check(lib().levo_snake_params_prepare(_ptr(alpha_log), _ptr(beta_log), _pdtype(alpha_log), alpha_log.numel(),
                                          _ptr(alpha), _ptr(inv_beta), _stream(alpha_log.device)))
    return alpha, inv_beta


def snakebeta_t(x, alpha_log, beta_log, out=None, prepared=False):
    """y = x + sin(x*exp(alpha_log))^2 / (exp(beta_log)+1e-9) over [C, T] (row stride honoured).
    With prepared=True the parameters are snake_params_prepare_t's (alpha, inv_beta)."""
    import torch

    _require_cuda(x, alpha_log, beta_log)
    if x.dim() != 2 or x.dtype != torch.float32 or x.stride(1) != 1:
        raise ValueError("SnakeBeta input must be F32 [channels, time] with unit time stride")
    if alpha_log.dtype != beta_log.dtype:
        raise ValueError("alpha_log and beta_log must share a dtype")
    if alpha_log.numel() != x.shape[0] or beta_log.numel() != x.shape[0]:
        raise ValueError("SnakeBeta parameters must have shape [1, channels, 1]")
    if prepared and alpha_log.dtype != torch.float32:
        raise ValueError("prepared SnakeBeta parameters are float32")
    y = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    pdtype = DTYPE_SNAKE_PREPARED if prepared else _pdtype(alpha_log)
    check(lib().levo_snakebeta_f32(_ptr(x), x.stride(0), _ptr(alpha_log), _ptr(beta_log), pdtype,
                                   _ptr(y), y.stride(0), x.shape[0], x.shape[1], _stream(x.device)))
    return y


def channel_bias_add_t(x, bias, out=None):
    import torch

    _require_cuda(x, bias)
    y = torch.empty_like(x) if out is None else out
    check(lib().levo_channel_bias_add_f32(_ptr(x), _ptr(bias), _pdtype(bias), _ptr(y), x.shape[0], x.shape[1],
                                          _stream(x.device)))
    return y


def fused_unit_t(u, bias=None, residual=None, alpha_log=None, beta_log=None, x_out=None, y_out=None,
                 tanh=False, param_dtype=None):
    _require_cuda(u, bias, residual, alpha_log, beta_log, x_out, y_out)
    ref = next((t for t in (bias, alpha_log) if t is not None), None)
    unit = FusedUnit(_ptr(u), _ptr(bias), _ptr(residual), _ptr(alpha_log), _ptr(beta_log), _ptr(x_out), _ptr(y_out),
                     u.shape[0], u.shape[1],
                     param_dtype if param_dtype is not None else (_pdtype(ref) if ref is not None else DTYPE_F32),
                     FUSED_TANH if tanh else 0)
    check(lib().levo_vae_fused_unit_f32(ctypes.byref(unit), _stream(u.device)))


def _norm_call(name, x, r, gamma, beta, h_out, y_out, eps, flags):
    _require_cuda(x, r, gamma, beta, h_out, y_out)
    rows, dim = x.shape
    args = [_ptr(x), _ptr(r), _ptr(gamma)]
    if beta is not None or "layernorm" in name:
        args.append(_ptr(beta))
    args += [_ptr(h_out), _ptr(y_out), rows, dim, eps, flags, _stream(x.device)]
    check(getattr(lib(), name)(*args))


def add_rmsnorm_t(x, r, gamma, eps, f16_boundary=False, h_out=None, y_out=None):
    """Returns (h, y): h = x + r, y = RMSNorm(h) * gamma; F16 or F32 activations."""
    import torch

    h = torch.empty_like(x) if (h_out is None and r is not None) else h_out
    y = torch.empty_like(x) if y_out is None else y_out
    name = "levo_add_rmsnorm_f16" if x.dtype == torch.float16 else "levo_add_rmsnorm_f32"
    _norm_call(name, x, r, gamma, None, h, y, eps, NORM_F16_BOUNDARY if f16_boundary else 0)
    return h, y


def add_layernorm_t(x, r, gamma, beta, eps, f16_boundary=False, h_out=None, y_out=None):
    import torch

    h = torch.empty_like(x) if (h_out is None and r is not None) else h_out
    y = torch.empty_like(x) if y_out is None else y_out
    name = "levo_add_layernorm_f16" if x.dtype == torch.float16 else "levo_add_layernorm_f32"
    _norm_call(name, x, r, gamma, beta, h, y, eps, NORM_F16_BOUNDARY if f16_boundary else 0)
    return h, y


def gated_layernorm_modulate_t(x, gate, r, gamma, beta, scale, shift, batch_rows, eps=1e-5, h_out=None,
                               y_out=None):
    """Flow block tail: h = r + x*gate[b]; y = (LN(h)*gamma + beta)*(1 + scale[b]) + shift[b]."""
    import torch

    _require_cuda(x, gate, r, gamma, beta, scale, shift, h_out, y_out)
    h = torch.empty_like(x) if h_out is None else h_out
    y = torch.empty_like(x) if y_out is None else y_out
    rows, dim = x.shape
    check(lib().levo_gated_layernorm_modulate_f32(_ptr(x), _ptr(gate), _ptr(r), _ptr(gamma), _ptr(beta), _ptr(scale),
                                                  _ptr(shift), batch_rows, _ptr(h), _ptr(y), rows, dim, eps,
                                                  _stream(x.device)))
    return h, y


def weightnorm_t(v, g, w=None, norms=None):
    """w = v * (g / ||v||) per dim-0 row; v is [rows, ...] F32, g has one value per row."""
    import torch

    _require_cuda(v, g, w, norms)
    rows = v.shape[0]
    cols = v.numel() // max(rows, 1)
    w = torch.empty_like(v) if w is None else w
    check(lib().levo_weightnorm_f32(_ptr(v), _ptr(g), _ptr(w), _ptr(norms), rows, cols, _stream(v.device)))
    return w


def fold_weight_norm_t(v, g):
    """Reference semantics of _fold_weight_norm (convert/convert_vae.py:187-199): raises on a zero norm."""
    import torch

    norms = torch.empty(v.shape[0], dtype=torch.float32, device=v.device)
    w = weightnorm_t(v, g, norms=norms)
    if bool((norms == 0).any().item()):
        raise ValueError("zero weight-norm magnitude in weight_v")
    return w


def cfg_combine_t(uncond, cond, guidance, out=None):
    import torch

    _require_cuda(uncond, cond, out)
    if uncond.numel() != cond.numel():
        raise ValueError("CFG vectors must have equal non-empty lengths")
    out = torch.empty_like(uncond) if out is None else out
    check(lib().levo_cfg_combine_f32(_ptr(uncond), _ptr(cond), _ptr(out), uncond.numel(), guidance,
                                     _stream(uncond.device)))
    return out


def flow_incontext_t(state, noise, context, prefix, step, steps, sigma_min, batch=1):
    _require_cuda(state, noise, context)
    row = state.numel() // batch
    check(lib().levo_flow_incontext_f32(_ptr(state), _ptr(noise), _ptr(context), batch, row, prefix, step, steps,
                                        sigma_min, _stream(state.device)))


def euler_cfg_step_t(state, uncond, cond, guidance, steps, cfg=True, status=None):
    _require_cuda(state, uncond, cond, status)
    check(lib().levo_euler_cfg_step_f32(_ptr(state), _ptr(uncond), _ptr(cond), state.numel(), 1 if cfg else 0,
                                        guidance, steps, _ptr(status), _stream(state.device)))


def cfg_euler_multi_t(state, noise, context, uncond, cond, *, batch, prefix, first_step, count, steps,
                      cfg=True, guidance=1.5, sigma_min=1e-4, status=None):
    _require_cuda(state, noise, context, uncond, cond, status)
    row = state.numel() // batch
    check(lib().levo_cfg_euler_multi_f32(_ptr(state), _ptr(noise), _ptr(context), _ptr(uncond), _ptr(cond),
                                         batch, row, prefix, first_step, count, steps, 1 if cfg else 0, guidance,
                                         sigma_min, _ptr(status), _stream(state.device)))


EULER_STEP_LIMIT = 1 << 28
EULER_FAIL_STATE, EULER_FAIL_VELOCITY = 2, 3


def euler_status_step(word: int) -> int:
    """First failing step recorded in a multi-step status word (LEVO_EULER_STATUS_STEP), -1 if none."""
    return EULER_STEP_LIMIT - (word >> 2) if word >> 2 else -1


def cfg_euler_solve_t(state, noise, context, uncond, cond, *, batch, prefix, first_step, count, steps,
                      cfg=True, guidance=1.5, sigma_min=1e-4) -> int:
    """solve_flow_euler over precomputed velocities (levo_cfg_euler_solve_f32): returns the completed
    step count; on a non-finite velocity or state raises LevoNonFinite with .completed_steps, leaving
    `state` at the reference's checkpoint of the steps completed before the failing one."""
    import torch

    _require_cuda(state, noise, context, uncond, cond)
    row = state.numel() // batch
    checkpoint = torch.empty_like(state)
    status = torch.zeros(1, dtype=torch.int32, device=state.device)
    done = ctypes.c_int64(0)
    code = lib().levo_cfg_euler_solve_f32(_ptr(state), _ptr(noise), _ptr(context), _ptr(uncond), _ptr(cond), batch,
                                          row, prefix, first_step, count, steps, 1 if cfg else 0, guidance,
                                          sigma_min, _ptr(checkpoint), _ptr(status), ctypes.byref(done),
                                          _stream(state.device))
    try:
        check(code)
    except LevoNonFinite as err:
        err.completed_steps = done.value
        raise
    return done.value


def flow_euler_solve_t(state, noise, context, *, frames, latent_dim, incontext_frames, steps, velocity,
                       first_step=0, cfg=True, guidance=1.5, sigma_min=1e-4, cancel=None, checkpoint=True) -> int:
    """solve_flow_euler on a device state with a per-step velocity callable
    velocity(state, step, time) -> CUDA tensor ([2, n] with cfg, else [n]); returns the completed step
    count.  A non-finite velocity or state raises LevoNonFinite (.completed_steps set; with checkpoint=True
    the state is the reference's checkpoint); cancel() returning True raises LevoCancelled."""
    import torch

    _require_cuda(state, noise, context)
    keep = []  # velocity tensors must outlive their step

    def _velocity(_user, state_ptr, step, time, _stream):
        try:
            v = velocity(state, int(step), float(time))
            keep.append(v)
            return v.data_ptr()
        except Exception:  # noqa: BLE001 - reported through the C ABI as a failed callback
            return None

    vcb = VELOCITY_FN(_velocity)
    ccb = CANCEL_FN(lambda _u: 1 if cancel() else 0) if cancel is not None else CANCEL_FN()
    ckpt = torch.empty_like(state) if checkpoint else None
    status = torch.zeros(1, dtype=torch.int32, device=state.device)
    done = ctypes.c_int64(0)
    code = lib().levo_flow_euler_solve_f32(_ptr(state), _ptr(noise), _ptr(context), frames, latent_dim,
                                           incontext_frames, sigma_min, steps, first_step, 1 if cfg else 0, guidance,
                                           vcb, None, ccb, None, _ptr(ckpt), _ptr(status), ctypes.byref(done),
                                           _stream(state.device))
    try:
        check(code)
    except LevoOpsError as err:
        err.completed_steps = done.value
        raise
    return done.value


ASSEMBLE_STATUS_LIMIT = 1 << 30


def assemble_windows_t(windows, hop_samples: int, overlap_samples: int, target_samples: int, interleaved=False,
                       out=None, check_finite=True, status=None):
    """Crossfade-assemble decoded windows [W, C, S] into [C, target] (or [target, C] interleaved).
    With check_finite (the reference's require_finite_audio) a non-finite sample in any window raises
    LevoNonFinite with the reference's message for the first (window, channel), after a synchronize.
    With a caller-owned status tensor (device int32, zeroed) the check runs but nothing is read back:
    the caller decodes the word (LEVO_ASSEMBLE_STATUS) itself, and the call stays asynchronous."""
    import torch

    _require_cuda(windows, out)
    w, c, s = windows.shape
    if out is None:
        shape = (target_samples, c) if interleaved else (c, target_samples)
        out = torch.empty(shape, dtype=torch.float32, device=windows.device)
    own = status is None and check_finite
    if own:
        status = torch.zeros(1, dtype=torch.int32, device=windows.device)
    check(lib().levo_assemble_windows_f32(_ptr(windows), w, c, s, hop_samples, overlap_samples, target_samples,
                                          _ptr(out), 1 if interleaved else 0, _ptr(status),
                                          _stream(windows.device)))
    word = int(status.item()) if own else 0
    if word:
        pair = ASSEMBLE_STATUS_LIMIT - word
        k, ch = divmod(pair, c)
        name = ("left", "right")[ch] if c == 2 else f"{ch}"
        raise LevoNonFiniteAudio(ENONFINITE, f"levo_assemble_windows_f32: decoded {name} channel contains "
                                             f"non-finite samples (window {k})")
    return out


def greedy_tokens_t(logits, recent=None, penalty=1.0, penalty_limit=0, ignore=None, status=None, out=None):
    """Greedy next token per row of logits [rows, vocab] (reference sample_streams, use_sampling=False)."""
    import torch

    _require_cuda(logits, recent, ignore, status, out)
    rows, vocab = logits.shape
    out = torch.empty(rows, dtype=torch.int64, device=logits.device) if out is None else out
    recent_len = recent.shape[1] if recent is not None else 0
    check(lib().levo_greedy_tokens_f32(_ptr(logits), rows, vocab, logits.stride(0), _ptr(recent), recent_len, penalty,
                                       penalty_limit, _ptr(ignore), ignore.numel() if ignore is not None else 0,
                                       _ptr(out), _ptr(status), _stream(logits.device)))
    return out


def _raise_if_flagged(status, what: str, message: str) -> None:
    """Reads an optional status word (synchronising) and raises LevoNonFinite when bit 0 is set."""
    if status is not None and int(status.item()) & 1:
        raise LevoNonFinite(ENONFINITE, f"{what}: {message}")


def latent_to_vae_t(frame_major, mean=None, stddev=None, out=None, check_finite=True, status=None):
    """[frames, dim] frame-major (normalised) latent -> [dim, frames] de-normalised VAE input.  With
    check_finite a non-finite input raises LevoNonFinite, as denormalize_latents throws; with a
    caller-owned status tensor (device int32, zeroed) the flag is set there and not read back."""
    import torch

    _require_cuda(frame_major, mean, stddev, out)
    frames, dim = frame_major.shape
    out = torch.empty((dim, frames), dtype=torch.float32, device=frame_major.device) if out is None else out
    own = status is None and check_finite
    if own:
        status = torch.zeros(1, dtype=torch.int32, device=frame_major.device)
    check(lib().levo_latent_to_vae_f32(_ptr(frame_major), _ptr(mean), _ptr(stddev), frames, dim, _ptr(out),
                                       _ptr(status), _stream(frame_major.device)))
    if own:
        _raise_if_flagged(status, "levo_latent_to_vae_f32", "normalized latent contains a non-finite value")
    return out


def latent_normalize_t(raw, mean, stddev, out=None, check_finite=True):
    """(raw - mean) / stddev per channel; with check_finite a non-finite raw value raises LevoNonFinite,
    as normalize_latents throws."""
    import torch

    _require_cuda(raw, mean, stddev, out)
    frames, dim = raw.shape
    out = torch.empty_like(raw) if out is None else out
    status = torch.zeros(1, dtype=torch.int32, device=raw.device) if check_finite else None
    check(lib().levo_latent_normalize_f32(_ptr(raw), _ptr(mean), _ptr(stddev), frames, dim, _ptr(out),
                                          _ptr(status), _stream(raw.device)))
    _raise_if_flagged(status, "levo_latent_normalize_f32", "raw latent contains a non-finite value")
    return out


def reference_topology() -> Topology:
    t = Topology()
    check(lib().levo_vae_topology_reference(ctypes.byref(t)))
    return t


def param_count(topology: Topology) -> int:
    n = lib().levo_vae_param_count(ctypes.byref(topology))
    if n < 0:
        check(int(n))
    return int(n)


def _host_window_buffers(topology: Topology, latents_host, audio_host, frames: int):
    """Validates the host buffers of a host-to-host decode and returns (windows, latent ptr, audio ptr).
    The library copies windows * audio_channels * samples floats into audio_host and reads
    windows * latent_dim * frames from latents_host, so both must be float32, C-contiguous CPU
    buffers of at least that size."""
    import numpy as np

    def describe(buf, name):
        if hasattr(buf, "ctypes"):  # numpy
            if buf.dtype != np.float32 or not buf.flags["C_CONTIGUOUS"]:
                raise ValueError(f"{name} must be a C-contiguous float32 array")
            return buf.shape, buf.size, buf.ctypes.data
        import torch

        if not isinstance(buf, torch.Tensor) or buf.is_cuda:
            raise ValueError(f"{name} must be a numpy array or a CPU tensor")
        if buf.dtype != torch.float32 or not buf.is_contiguous():
            raise ValueError(f"{name} must be a contiguous float32 tensor")
        return tuple(buf.shape), buf.numel(), buf.data_ptr()

    lat_shape, _, lat_ptr = describe(latents_host, "latents_host")
    _, audio_size, out_ptr = describe(audio_host, "audio_host")
    if len(lat_shape) != 3 or lat_shape[1] != topology.latent_dim or lat_shape[2] != frames:
        raise ValueError(f"latents_host must have shape (windows, {topology.latent_dim}, {frames}), got {lat_shape}")
    windows = lat_shape[0]
    need = windows * topology.audio_channels * frames * topology.upsampling()
    if audio_size < need:
        raise ValueError(f"audio_host holds {audio_size} floats; {windows} windows need {need}")
    return windows, lat_ptr, out_ptr


def decode_windows_multi(chains, latents_host, audio_host, frames: int, flags: int = 0, cancel=None) -> None:
    """Host-to-host decode of independent windows over several chains (one per GPU) from one
    process: chain i decodes a contiguous block of the windows on its own thread and stream."""
    if not chains:
        raise ValueError("at least one chain is required")
    _, lat_ptr, out_ptr = _host_window_buffers(chains[0].topology, latents_host, audio_host, frames)
    handles = (ctypes.c_void_p * len(chains))(*[c.handle.value for c in chains])
    cb = CANCEL_FN(lambda _u: 1 if cancel() else 0) if cancel is not None else CANCEL_FN()
    check(lib().levo_vae_chains_decode_windows(ctypes.cast(handles, ctypes.c_void_p), len(chains), lat_ptr,
                                               latents_host.shape[0], frames, out_ptr, flags, cb, None))


class VaeChain:
    """Owner of a levo_vae_chain (workspace + parameters on one device)."""

    def __init__(self, topology: Topology, params_host, max_frames: int, device: int = 0, conv=None):
        """params_host: packed parameters as float32, or float16 (kept F16 on the device)."""
        import numpy as np

        self.topology = topology
        half = getattr(params_host, "dtype", None) == np.float16
        self.params = np.ascontiguousarray(params_host, dtype=np.float16 if half else np.float32)
        if self.params.size != param_count(topology):
            raise ValueError("parameter array does not match the topology")
        self._conv = CONV_FN(conv) if conv is not None else CONV_FN()
        handle = ctypes.c_void_p()
        create = lib().levo_vae_chain_create_f16 if half else lib().levo_vae_chain_create
        check(create(ctypes.byref(handle), ctypes.byref(topology), self.params.ctypes.data, max_frames, self._conv,
                     None, device))
        self.handle = handle
        self.device = device
        self.max_frames = max_frames

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().levo_vae_chain_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def samples(self, frames: int) -> int:
        return frames * self.topology.upsampling()

    def decode(self, latent, audio, frames: int, flags: int = 0, stream: Optional[int] = None) -> None:
        """Device-resident decode: latent [latent_dim, frames] -> audio [channels, samples] (CUDA tensors)."""
        check(lib().levo_vae_chain_decode(self.handle, _ptr(latent), frames, _ptr(audio), flags,
                                          _stream(latent.device) if stream is None else stream))

    def decode_windows(self, latents_host, audio_host, frames: int, flags: int = 0, cancel=None,
                       stream: Optional[int] = None) -> None:
        """Host-to-host decode of independent windows: latents_host (windows, latent_dim, frames) and
        audio_host (windows, audio_channels, samples), float32 C-contiguous numpy arrays or CPU tensors."""
        windows, lat_ptr, out_ptr = _host_window_buffers(self.topology, latents_host, audio_host, frames)
        cb = CANCEL_FN(lambda _u: 1 if cancel() else 0) if cancel is not None else CANCEL_FN()
        if stream is None:
            import torch

            stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().levo_vae_chain_decode_windows(self.handle, lat_ptr, windows, frames, out_ptr, flags, cb, None,
                                                  stream))

    def set_stage_capture(self, stage_out) -> None:
        """stage_out: one F32 buffer per stage (CUDA tensors or host arrays, [width_s, L_s] for the
        frames decoded), or None to stop capturing.  The buffers must outlive the decodes."""
        if stage_out is None:
            self._capture = None
            check(lib().levo_vae_chain_set_stage_capture(self.handle, None, 0))
            return
        ptrs = [o.ctypes.data if hasattr(o, "ctypes") else o.data_ptr() for o in stage_out]
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        check(lib().levo_vae_chain_set_stage_capture(self.handle, ctypes.cast(arr, ctypes.c_void_p), len(ptrs)))
        self._capture = list(stage_out)  # keep the buffers alive

    def timing(self, reset: bool = True) -> dict:
        arr = (KernelTiming * len(KCLASS_NAMES))()
        check(lib().levo_vae_chain_timing(self.handle, arr, 1 if reset else 0))
        return {name: {"launches": arr[i].launches, "ms": arr[i].milliseconds,
                       "bytes": arr[i].algorithmic_bytes, "elements": arr[i].elements}
                for i, name in enumerate(KCLASS_NAMES)}
