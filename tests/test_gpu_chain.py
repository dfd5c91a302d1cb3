"""GPU parity of the decoder elementwise chain (a4) against the oracle's
node-by-node restatement of src/levo-vae.cpp:212-235, through the C ABI.

Convolutions use the built-in stand-ins on both sides (index-map copies for
the input / upsample / output convs, identities for the residual convs).
Tolerance: 1e-5 scaled error per sample (F32 path)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu
TOL = 1e-5


def small_topology(ops, widths=((32, 4), (16, 3), (8, 2)), entry=64, latent=8, residual=2):
    t = ops.Topology()
    t.latent_dim, t.audio_channels, t.entry_width, t.n_stages = latent, 2, entry, len(widths)
    for i, (w, s) in enumerate(widths):
        t.stage_width[i], t.stage_stride[i] = w, s
    t.n_residual = residual
    for r in range(residual):
        t.dilation[r] = 3 ** r
    return t


def params_for(ops, topo, seed):
    rng = np.random.default_rng(seed)
    return (0.1 * rng.standard_normal(ops.param_count(topo))).astype(np.float32)


def chain_samples(topo, frames):
    return frames * topo.upsampling()


def oracle_audio(orc, topo, params, latent, frames, tanh=False):
    return orc.vae_chain(topo.as_list(), params, latent, frames, topo.audio_channels, frames * topo.upsampling(),
                         tanh=tanh)


@pytest.mark.parametrize("frames", [1, 3, 20, 64])
@pytest.mark.parametrize("tanh", [False, True])
def test_small_chain_matches_oracle(ops, orc, dev, frames, tanh):
    topo = small_topology(ops)
    params = params_for(ops, topo, frames)
    latent = np.random.default_rng(frames + 100).standard_normal((topo.latent_dim, frames)).astype(np.float32)
    chain = ops.VaeChain(topo, params, max_frames=64, device=0)
    audio = torch.full((2, chain.samples(frames)), np.nan, device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames, flags=ops.CHAIN_TANH if tanh else 0)
    assert_close(audio.cpu().numpy(), oracle_audio(orc, topo, params, latent, frames, tanh), TOL)
    chain.close()


@pytest.mark.parametrize("residual", [0, 1, 4])
def test_chain_residual_counts(ops, orc, dev, residual):
    topo = small_topology(ops, residual=residual)
    params = params_for(ops, topo, 40 + residual)
    frames = 9
    latent = np.random.default_rng(residual).standard_normal((topo.latent_dim, frames)).astype(np.float32)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    audio = torch.empty((2, chain.samples(frames)), device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames)
    assert_close(audio.cpu().numpy(), oracle_audio(orc, topo, params, latent, frames), TOL)


@pytest.mark.parametrize("frames", [2, 8])
def test_reference_topology_matches_oracle(ops, orc, dev, frames):
    topo = ops.reference_topology()
    params = params_for(ops, topo, 7)
    latent = np.random.default_rng(8).standard_normal((64, frames)).astype(np.float32)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    audio = torch.empty((2, frames * 1920), device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames)
    assert_close(audio.cpu().numpy(), oracle_audio(orc, topo, params, latent, frames), TOL)


@pytest.mark.parametrize("frames,tanh,f16", [(252, False, False), (750, True, False), (750, True, True)])
def test_reference_topology_full_window_matches_oracle(ops, orc, dev, frames, tanh, f16):
    """BASELINE config 3 (one 10.08 s window, T = 252, final [128][483840] stage) and one
    config-4 window (T = 750 with the tanh epilogue; F32- and F16-stored parameters, the
    latter promoted in-kernel) at full size against the oracle."""
    topo = ops.reference_topology()
    params = params_for(ops, topo, 13)
    if f16:
        params = params.astype(np.float16)
    latent = np.random.default_rng(frames).standard_normal((64, frames)).astype(np.float32)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    params = params.astype(np.float32)  # the oracle takes the promoted values
    audio = torch.empty((2, frames * 1920), device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames, flags=ops.CHAIN_TANH if tanh else 0)
    assert_close(audio.cpu().numpy(), oracle_audio(orc, topo, params, latent, frames, tanh), TOL)
    chain.close()


def test_reference_topology_full_window_properties(ops, dev):
    # A 30 s window (T = 750): finite, tanh-bounded, deterministic across calls.
    topo = ops.reference_topology()
    params = params_for(ops, topo, 9)
    frames = 750
    latent = torch.from_numpy(np.random.default_rng(9).standard_normal((64, frames)).astype(np.float32)).to(dev)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    a1 = torch.empty((2, frames * 1920), device=dev)
    a2 = torch.empty_like(a1)
    chain.decode(latent, a1, frames, flags=ops.CHAIN_TANH)
    chain.decode(latent, a2, frames, flags=ops.CHAIN_TANH)
    assert torch.isfinite(a1).all() and (a1.abs() <= 1).all()
    assert torch.equal(a1, a2)
    chain.close()


def test_conv_callback_is_called_and_may_alias(ops, orc, dev):
    """A user conv callback that reproduces the stand-ins with torch ops must give the same audio."""
    topo = small_topology(ops)
    params = params_for(ops, topo, 3)
    frames = 6
    latent = np.random.default_rng(3).standard_normal((topo.latent_dim, frames)).astype(np.float32)
    seen = []
    storage = {}

    def as_tensor(ptr, c, l):
        # wrap a device pointer as a torch tensor via a tiny cuda array interface
        class Wrap:
            __cuda_array_interface__ = {"shape": (c, l), "typestr": "<f4", "data": (ptr, False), "version": 3}

        return torch.as_tensor(Wrap(), device=dev)

    def conv(_user, call_p, _stream):
        call = call_p.contents
        seen.append(call.kind)
        if call.kind in (ops.CONV_RES0, ops.CONV_RES1):
            call.result = call.input  # identity: alias
            return 0
        src = as_tensor(call.input, call.in_channels, call.in_length)
        dst = as_tensor(call.output, call.out_channels, call.out_length)
        stride = call.stride if call.kind == ops.CONV_UPSAMPLE else 1
        idx_c = torch.arange(call.out_channels, device=dev) % call.in_channels
        idx_t = torch.arange(call.out_length, device=dev) // stride
        dst.copy_(src[idx_c][:, idx_t])
        storage["last"] = dst
        return 0

    chain = ops.VaeChain(topo, params, max_frames=frames, device=0, conv=conv)
    audio = torch.empty((2, chain.samples(frames)), device=dev)
    with torch.cuda.stream(torch.cuda.current_stream()):
        chain.decode(torch.from_numpy(latent).to(dev), audio, frames)
    torch.cuda.synchronize()
    assert seen[0] == ops.CONV_INPUT and seen[-1] == ops.CONV_OUTPUT
    assert seen.count(ops.CONV_UPSAMPLE) == topo.n_stages
    assert seen.count(ops.CONV_RES0) == topo.n_stages * topo.n_residual
    assert_close(audio.cpu().numpy(), oracle_audio(orc, topo, params, latent, frames), TOL)


def test_conv_callback_failure_is_reported(ops, dev):
    topo = small_topology(ops)
    chain = ops.VaeChain(topo, params_for(ops, topo, 4), max_frames=4, device=0, conv=lambda u, c, s: 7)
    audio = torch.empty((2, chain.samples(4)), device=dev)
    with pytest.raises(ops.LevoOpsError, match="callback failed"):
        chain.decode(torch.zeros((topo.latent_dim, 4), device=dev), audio, 4)


def test_decode_windows_host_matches_device_decode(ops, dev):
    topo = small_topology(ops)
    params = params_for(ops, topo, 5)
    frames, windows = 16, 5
    lat = np.random.default_rng(5).standard_normal((windows, topo.latent_dim, frames)).astype(np.float32)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    s = chain.samples(frames)
    host = torch.empty((windows, 2, s), dtype=torch.float32).pin_memory()
    chain.decode_windows(torch.from_numpy(lat).pin_memory(), host, frames, flags=ops.CHAIN_TANH)
    pageable = np.empty((windows, 2, s), np.float32)
    chain.decode_windows(lat, pageable, frames, flags=ops.CHAIN_TANH)
    for w in range(windows):
        d = torch.empty((2, s), device=dev)
        chain.decode(torch.from_numpy(lat[w]).to(dev), d, frames, flags=ops.CHAIN_TANH)
        torch.cuda.synchronize()
        assert torch.equal(host[w], d.cpu())
        assert np.array_equal(pageable[w], d.cpu().numpy())


def test_decode_windows_cancel_between_windows(ops, dev):
    # The reference polls cancellation between windows (src/cantor-abi.cpp:901-913).
    topo = small_topology(ops)
    chain = ops.VaeChain(topo, params_for(ops, topo, 6), max_frames=8, device=0)
    lat = np.random.default_rng(6).standard_normal((4, topo.latent_dim, 8)).astype(np.float32)
    out = np.full((4, 2, chain.samples(8)), np.nan, np.float32)
    polls = []

    def cancel():
        polls.append(1)
        return len(polls) > 2  # allow windows 0 and 1

    with pytest.raises(ops.LevoCancelled, match="before window 2"):
        chain.decode_windows(lat, out, 8, cancel=cancel)
    assert np.all(np.isfinite(out[:2])) and np.all(np.isnan(out[2:]))


def test_chain_timing_reports_every_class(ops, dev):
    topo = ops.reference_topology()
    chain = ops.VaeChain(topo, params_for(ops, topo, 10), max_frames=16, device=0)
    lat = torch.randn((64, 16), device=dev)
    audio = torch.empty((2, 16 * 1920), device=dev)
    chain.decode(lat, audio, 16, flags=ops.CHAIN_TIMING | ops.CHAIN_TANH)
    t = chain.timing()
    assert t["entry"]["launches"] == 1 and t["upsample"]["launches"] == 5
    assert t["post"]["launches"] == 15 and t["residual"]["launches"] == 15 and t["epilogue"]["launches"] == 1
    assert t["conv"]["launches"] == 7  # input + 5 upsample + output stand-ins (residual convs alias)
    assert all(v["ms"] > 0 for k, v in t.items())
    # residual units move 16 B/elem except the last unit of each stage (12 B/elem)
    elems = t["residual"]["elements"]
    assert 12 * elems < t["residual"]["bytes"] < 16 * elems


def test_chain_rejects_too_many_frames(ops, dev):
    topo = small_topology(ops)
    chain = ops.VaeChain(topo, params_for(ops, topo, 11), max_frames=4, device=0)
    with pytest.raises(ValueError, match="max_frames"):
        chain.decode(torch.zeros((topo.latent_dim, 5), device=dev), torch.zeros((2, 1000), device=dev), 5)


def test_conv_standin(ops, orc, dev):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((6, 11)).astype(np.float32)
    out = torch.empty((4, 33), device=dev)
    ops.check(ops.lib().levo_conv_standin_f32(torch.from_numpy(x).to(dev).data_ptr(), 6, 11, out.data_ptr(), 4, 33,
                                              3, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    assert np.array_equal(out.cpu().numpy(), orc.conv_standin(x, 4, 33, 3))


def test_f16_stored_parameters(ops, orc, dev):
    # The F16 VAE artifact keeps parameters in F16; each unit promotes them to F32
    # (src/levo-audio-ops.cpp:32-37): same result as F32 parameters holding the promoted values.
    topo = small_topology(ops)
    params16 = params_for(ops, topo, 21).astype(np.float16)
    frames = 12
    latent = np.random.default_rng(21).standard_normal((topo.latent_dim, frames)).astype(np.float32)
    chain16 = ops.VaeChain(topo, params16, max_frames=frames, device=0)
    chain32 = ops.VaeChain(topo, params16.astype(np.float32), max_frames=frames, device=0)
    a16 = torch.empty((2, chain16.samples(frames)), device=dev)
    a32 = torch.empty_like(a16)
    chain16.decode(torch.from_numpy(latent).to(dev), a16, frames, flags=ops.CHAIN_TANH)
    chain32.decode(torch.from_numpy(latent).to(dev), a32, frames, flags=ops.CHAIN_TANH)
    assert torch.equal(a16, a32)
    assert_close(a16.cpu().numpy(), oracle_audio(orc, topo, params16.astype(np.float32), latent, frames, True), TOL)


@pytest.mark.parametrize("residual", [0, 2])
def test_stage_capture_matches_oracle(ops, orc, dev, residual):
    """capture_stages (src/levo-vae.cpp:230-231,271-274): every stage's output, into device
    tensors (device decode) and host arrays (host decode); audio unchanged by capturing."""
    topo = small_topology(ops, residual=residual)
    params = params_for(ops, topo, 50 + residual)
    frames = 11
    latent = np.random.default_rng(51).standard_normal((topo.latent_dim, frames)).astype(np.float32)
    want_audio, want_stages = orc.vae_chain(topo.as_list(), params, latent, frames, 2, chain_samples(topo, frames),
                                            stages=True)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    dev_stages = [torch.full(w.shape, np.nan, device=dev) for w in want_stages]
    chain.set_stage_capture(dev_stages)
    audio = torch.empty((2, chain.samples(frames)), device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames)
    torch.cuda.synchronize()
    assert_close(audio.cpu().numpy(), want_audio, TOL)
    for got, want in zip(dev_stages, want_stages):
        assert_close(got.cpu().numpy(), want, TOL)
    host_stages = [np.full(w.shape, np.nan, np.float32) for w in want_stages]
    chain.set_stage_capture(host_stages)
    host_audio = np.empty((1, 2, chain.samples(frames)), np.float32)
    chain.decode_windows(latent[None], host_audio, frames)
    for got, want in zip(host_stages, want_stages):
        assert_close(got, want, TOL)
    assert np.array_equal(host_audio[0], audio.cpu().numpy())
    with pytest.raises(ValueError, match="one window"):
        chain.decode_windows(np.stack([latent, latent]), np.empty((2, 2, chain.samples(frames)), np.float32), frames)
    chain.set_stage_capture(None)
    chain.decode_windows(np.stack([latent, latent]), np.empty((2, 2, chain.samples(frames)), np.float32), frames)


def test_decode_windows_rejects_non_finite_latent(ops, dev):
    # vae_decoder::decode: "latent payload contains a non-finite value" (src/levo-vae.cpp:189-191)
    topo = small_topology(ops)
    chain = ops.VaeChain(topo, params_for(ops, topo, 52), max_frames=6, device=0)
    lat = np.random.default_rng(52).standard_normal((3, topo.latent_dim, 6)).astype(np.float32)
    lat[1, 3, 2] = np.inf
    out = np.full((3, 2, chain.samples(6)), np.nan, np.float32)
    with pytest.raises(ops.LevoOpsError, match="non-finite value \\(window 1\\)"):
        chain.decode_windows(lat, out, 6)
    assert np.all(np.isfinite(out[0])) and np.all(np.isnan(out[1:]))


@pytest.mark.parametrize("windows,n_chains", [(5, 2), (7, 3), (2, 3), (0, 2)])
def test_chains_decode_windows_matches_single_chain(ops, dev, windows, n_chains):
    """One-process DECODE over several chains (here all on device 0, as a box with one GPU
    has): each window's audio equals the single-chain host decode."""
    topo = small_topology(ops)
    params = params_for(ops, topo, 60)
    frames = 10
    lat = np.random.default_rng(60).standard_normal((windows, topo.latent_dim, frames)).astype(np.float32)
    chains = [ops.VaeChain(topo, params, max_frames=frames, device=0) for _ in range(n_chains)]
    s = chains[0].samples(frames)
    multi = np.full((windows, 2, s), np.nan, np.float32)
    ops.decode_windows_multi(chains, lat, multi, frames, flags=ops.CHAIN_TANH)
    single = np.empty((windows, 2, s), np.float32)
    chains[0].decode_windows(lat, single, frames, flags=ops.CHAIN_TANH)
    assert np.array_equal(multi, single)


def test_chains_decode_windows_reports_the_failing_chain(ops, dev):
    topo = small_topology(ops)
    params = params_for(ops, topo, 61)
    chains = [ops.VaeChain(topo, params, max_frames=6, device=0) for _ in range(2)]
    lat = np.random.default_rng(61).standard_normal((4, topo.latent_dim, 6)).astype(np.float32)
    lat[3, 0, 0] = np.nan  # window 3 belongs to chain 1 (windows 2..3)
    out = np.empty((4, 2, chains[0].samples(6)), np.float32)
    with pytest.raises(ops.LevoOpsError, match="non-finite.*chain 1"):
        ops.decode_windows_multi(chains, lat, out, 6)
    other = ops.VaeChain(small_topology(ops, residual=1), params_for(ops, small_topology(ops, residual=1), 62),
                         max_frames=6, device=0)
    with pytest.raises(ValueError, match="one topology"):
        ops.decode_windows_multi([chains[0], other], lat, out, 6)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_chains_decode_windows_across_devices(ops):
    """One chain on each of two GPUs, reference topology: same audio as one chain on GPU 0."""
    topo = ops.reference_topology()
    params = params_for(ops, topo, 63)
    frames, windows = 40, 6
    lat = np.random.default_rng(63).standard_normal((windows, 64, frames)).astype(np.float32)
    chains = [ops.VaeChain(topo, params, max_frames=frames, device=d) for d in (0, 1)]
    s = chains[0].samples(frames)
    multi = np.full((windows, 2, s), np.nan, np.float32)
    ops.decode_windows_multi(chains, lat, multi, frames, flags=ops.CHAIN_TANH)
    single = np.empty_like(multi)
    chains[0].decode_windows(lat, single, frames, flags=ops.CHAIN_TANH)
    assert np.array_equal(multi, single)


def test_chain_decode_captures_into_a_cuda_graph(ops, dev):
    """A device-resident decode records into a CUDA graph (programmatic-dependent launches
    included) and its replay gives the eager decode's bits."""
    topo = ops.reference_topology()
    params = params_for(ops, topo, 64)
    frames = 8
    lat = torch.from_numpy(np.random.default_rng(64).standard_normal((64, frames)).astype(np.float32)).to(dev)
    chain = ops.VaeChain(topo, params, max_frames=frames, device=0)
    eager = torch.empty((2, chain.samples(frames)), device=dev)
    chain.decode(lat, eager, frames, flags=ops.CHAIN_TANH)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    graphed = torch.full_like(eager, np.nan)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain.decode(lat, graphed, frames, flags=ops.CHAIN_TANH, stream=stream.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(graphed, eager)
    lat.add_(0.5)  # the graph reads the latent buffer anew on every replay
    chain.decode(lat, eager, frames, flags=ops.CHAIN_TANH)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(graphed, eager)
    del g
    chain.close()


def test_chains_decode_windows_cancellation(ops, dev):
    # The cancel callback is polled by every chain's thread before each of its windows.
    topo = small_topology(ops)
    params = params_for(ops, topo, 65)
    chains = [ops.VaeChain(topo, params, max_frames=6, device=0) for _ in range(2)]
    lat = np.random.default_rng(65).standard_normal((6, topo.latent_dim, 6)).astype(np.float32)
    out = np.empty((6, 2, chains[0].samples(6)), np.float32)
    polls = []

    def cancel():
        polls.append(1)
        return len(polls) > 3

    with pytest.raises(ops.LevoCancelled, match="chain"):
        ops.decode_windows_multi(chains, lat, out, 6, cancel=cancel)
    assert len(polls) >= 4
