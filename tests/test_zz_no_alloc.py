"""The allocation-free decode entry point (levo_vae_decode_noalloc_f32).

It serves callers that must not have this library call cudaMalloc: a real-time
render thread, where an allocation can stall the whole device, or a host engine
that owns a fixed device-memory budget and hands the library only its own
buffers.  Its scratch is a static device array, shared by all calls.

Checked here, through the C ABI: two calls in a row give the same audio as the
allocating entry point (levo_vae_chain_create + levo_vae_chain_decode), device
free memory does not change across the second call, and windows too large for
the static array are refused.  This file is named to be collected last and runs
the same alone in a fresh process or after the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu
TOL = 1e-5  # the F32 tolerance of the other chain tests


def _small_topology(ops):
    t = ops.Topology()
    t.latent_dim, t.audio_channels, t.entry_width, t.n_stages = 8, 2, 64, 3
    for i, (w, s) in enumerate([(32, 4), (16, 3), (8, 2)]):
        t.stage_width[i], t.stage_stride[i] = w, s
    t.n_residual = 2
    t.dilation[0], t.dilation[1] = 1, 3
    return t


def _noalloc(ops, topo, params, latent, frames, audio, flags):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return ops.lib().levo_vae_decode_noalloc_f32(ctypes.byref(topo), params.data_ptr(), latent.data_ptr(), frames,
                                                 audio.data_ptr(), ops.CONV_FN(), None, flags, stream)


@pytest.mark.parametrize("which,frames", [("small", 20), ("reference", 8)])
def test_noalloc_decode_matches_chain_decode_twice(ops, dev, which, frames):
    topo = _small_topology(ops) if which == "small" else ops.reference_topology()
    rng = np.random.default_rng(frames)
    params_host = (0.1 * rng.standard_normal(ops.param_count(topo))).astype(np.float32)
    latent = torch.from_numpy(rng.standard_normal((topo.latent_dim, frames)).astype(np.float32)).to(dev)
    samples = frames * topo.upsampling()

    chain = ops.VaeChain(topo, params_host, max_frames=frames, device=0)
    want = torch.empty((topo.audio_channels, samples), device=dev)
    chain.decode(latent, want, frames, flags=ops.CHAIN_TANH)
    torch.cuda.synchronize()
    chain.close()

    params = torch.from_numpy(params_host).to(dev)
    outs = [torch.full((topo.audio_channels, samples), np.nan, device=dev) for _ in range(2)]
    # Call 1 (the first call on this device also resolves the static array's address).
    assert _noalloc(ops, topo, params, latent, frames, outs[0], ops.CHAIN_TANH) == ops.OK, ops.last_error()
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    # Call 2, right after: same result, and device free memory is unchanged.
    assert _noalloc(ops, topo, params, latent, frames, outs[1], ops.CHAIN_TANH) == ops.OK, ops.last_error()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before  # nothing was allocated on the device
    for out in outs:
        assert_close(out.cpu().numpy(), want.cpu().numpy(), TOL, which)


def test_noalloc_decode_rejects_windows_beyond_the_static_scratch(ops, dev):
    topo = ops.reference_topology()
    params = torch.zeros(ops.param_count(topo), device=dev)
    latent = torch.zeros((64, 9), device=dev)
    audio = torch.zeros((2, 9 * 1920), device=dev)
    assert _noalloc(ops, topo, params, latent, 9, audio, 0) == ops.EINVAL
    assert "static scratch limit" in ops.last_error()
