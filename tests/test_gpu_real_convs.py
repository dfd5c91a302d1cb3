"""The decoder chain with REAL convolutions behind its conv callback, against a plain
PyTorch fp32 Oobleck decoder (src/levo-vae.cpp:80-101,172-276) with the same weights.

The chain runs every bias / SnakeBeta / residual node in its fused units and hands each
convolution (kind, kernel, stride, padding, dilation, shapes) to the callback, which runs
torch conv1d / conv_transpose1d without bias.  The reference side is the whole decoder in
torch ops.  TF32 is off on both sides.  Few-ulp SnakeBeta differences (own sin^2 against
torch.sin, multiply by 1/beta against a divide) pass through up to 36 convolutions, so the
bar is the reference's own frozen F32 waveform gate for its whole decoder against PyTorch
(tests/test-vae.cpp:80-94): relative RMS <= 1e-3, cosine >= 0.99999, and max abs error
<= 3e-3 (scaled here by the waveform's peak, since random weights do not keep it in [-1, 1])."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def unpack_params(topo, params):
    """Splits the packed parameter array in levo_vae_param_count's order."""
    it = iter(np.split(params, np.cumsum(_sizes(topo))[:-1]))
    p = {"in_bias": next(it), "stages": []}
    for _ in range(topo.n_stages):
        st = {"up_alpha": next(it), "up_beta": next(it), "up_bias": next(it), "res": []}
        for _ in range(topo.n_residual):
            st["res"].append({k: next(it) for k in ("pre_alpha", "pre_beta", "b0", "post_alpha", "post_beta", "b1")})
        p["stages"].append(st)
    p["out_alpha"], p["out_beta"] = next(it), next(it)
    return p


def _sizes(topo):
    sizes, cin = [topo.entry_width], topo.entry_width
    for s in range(topo.n_stages):
        cout = topo.stage_width[s]
        sizes += [cin, cin, cout] + [cout] * (6 * topo.n_residual)
        cin = cout
    return sizes + [cin, cin]


def make_weights(topo, rng, dev):
    """Conv weights in torch layouts, scaled by 1/sqrt(fan_in) to keep activations O(1)."""
    def w(shape, fan_in):
        return torch.from_numpy((rng.standard_normal(shape) / np.sqrt(fan_in)).astype(np.float32)).to(dev)

    ws = {("in",): w((topo.entry_width, topo.latent_dim, 7), topo.latent_dim * 7)}
    cin = topo.entry_width
    for s in range(topo.n_stages):
        cout, stride = topo.stage_width[s], topo.stage_stride[s]
        ws[("up", s)] = w((cin, cout, 2 * stride), cin * 2)  # conv_transpose1d: [in, out, k]
        for r in range(topo.n_residual):
            ws[("res0", s, r)] = w((cout, cout, 7), cout * 7)
            ws[("res1", s, r)] = w((cout, cout, 1), cout)
        cin = cout
    ws[("out",)] = w((topo.audio_channels, cin, 7), cin * 7)
    return ws


def snake(x, alpha_log, beta_log):
    a = torch.exp(alpha_log)[:, None]
    b = torch.exp(beta_log)[:, None] + 1e-9
    return x + torch.sin(x * a) ** 2 / b


def torch_decoder(topo, p, ws, latent):
    t = lambda v: torch.from_numpy(v).to(latent.device)  # noqa: E731
    h = F.conv1d(latent[None], ws[("in",)], t(p["in_bias"]), padding=3)[0]
    for s, st in enumerate(p["stages"]):
        stride = topo.stage_stride[s]
        h = snake(h, t(st["up_alpha"]), t(st["up_beta"]))
        h = F.conv_transpose1d(h[None], ws[("up", s)], t(st["up_bias"]), stride=stride,
                               padding=(stride + 1) // 2)[0]
        for r, ru in enumerate(st["res"]):
            d = topo.dilation[r]
            y = snake(h, t(ru["pre_alpha"]), t(ru["pre_beta"]))
            y = F.conv1d(y[None], ws[("res0", s, r)], t(ru["b0"]), padding=3 * d, dilation=d)[0]
            y = snake(y, t(ru["post_alpha"]), t(ru["post_beta"]))
            y = F.conv1d(y[None], ws[("res1", s, r)], t(ru["b1"]))[0]
            h = h + y
    h = snake(h, t(p["out_alpha"]), t(p["out_beta"]))
    return F.conv1d(h[None], ws[("out",)], None, padding=3)[0]


def make_callback(ops, ws, dev):
    def as_tensor(ptr, c, length):
        class Wrap:
            __cuda_array_interface__ = {"shape": (c, length), "typestr": "<f4", "data": (ptr, False), "version": 3}

        return torch.as_tensor(Wrap(), device=dev)

    def conv(_user, call_p, _stream):
        c = call_p.contents
        src = as_tensor(c.input, c.in_channels, c.in_length)
        dst = as_tensor(c.output, c.out_channels, c.out_length)
        if c.kind == ops.CONV_INPUT:
            y = F.conv1d(src[None], ws[("in",)], None, padding=c.padding)
        elif c.kind == ops.CONV_UPSAMPLE:
            y = F.conv_transpose1d(src[None], ws[("up", c.stage)], None, stride=c.stride, padding=c.padding)
        elif c.kind == ops.CONV_RES0:
            y = F.conv1d(src[None], ws[("res0", c.stage, c.unit)], None, padding=c.padding, dilation=c.dilation)
        elif c.kind == ops.CONV_RES1:
            y = F.conv1d(src[None], ws[("res1", c.stage, c.unit)], None, padding=c.padding)
        else:
            y = F.conv1d(src[None], ws[("out",)], None, padding=c.padding)
        if y.shape[1:] != dst.shape:
            return 2
        dst.copy_(y[0])
        return 0

    return conv


def topology(ops, reference):
    if reference:
        return ops.reference_topology()
    t = ops.Topology()
    t.latent_dim, t.audio_channels, t.entry_width, t.n_stages = 16, 2, 64, 3
    for i, (w, s) in enumerate([(48, 4), (32, 6), (16, 2)]):
        t.stage_width[i], t.stage_stride[i] = w, s
    t.n_residual = 3
    for r, d in enumerate((1, 3, 9)):
        t.dilation[r] = d
    return t


@pytest.mark.parametrize("reference,frames", [(False, 23), (False, 64), (True, 3)])
def test_chain_with_real_convolutions_matches_torch_decoder(ops, dev, reference, frames):
    tf32 = torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        topo = topology(ops, reference)
        rng = np.random.default_rng(70 + frames)
        params = (0.1 * rng.standard_normal(ops.param_count(topo))).astype(np.float32)
        ws = make_weights(topo, rng, dev)
        latent = torch.from_numpy(rng.standard_normal((topo.latent_dim, frames)).astype(np.float32)).to(dev)
        chain = ops.VaeChain(topo, params, max_frames=frames, device=0, conv=make_callback(ops, ws, dev))
        audio = torch.full((topo.audio_channels, chain.samples(frames)), np.nan, device=dev)
        chain.decode(latent, audio, frames, stream=torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        want = torch_decoder(topo, unpack_params(topo, params), ws, latent)
        assert want.shape == audio.shape
        got, ref = audio.double().cpu().numpy().ravel(), want.double().cpu().numpy().ravel()
        err = got - ref
        max_error = np.abs(err).max() / max(1.0, np.abs(ref).max())
        relative_rms = np.sqrt((err ** 2).sum() / max((ref ** 2).sum(), 1e-30))
        cosine = (got * ref).sum() / np.sqrt(max((ref ** 2).sum() * (got ** 2).sum(), 1e-30))
        stats = f"max_error={max_error:.3g} relative_rms={relative_rms:.3g} cosine={cosine:.8f} peak={np.abs(ref).max():.3g}"
        assert max_error <= 3e-3 and relative_rms <= 1e-3 and cosine >= 0.99999, stats
        chain.close()
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = tf32
