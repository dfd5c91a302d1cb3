"""Seeded random sweeps over shapes, memory layouts and options of every kernel family,
against the oracle.  Random element offsets into larger buffers give every streaming
dispatch path: rows form (all tensors 32-byte aligned, rows a multiple of 8 long), ragged
rows (aligned, other lengths), the flat vector form (one common nonzero 32-byte phase) and
the scalar form (mismatched phases, or row strides).  Tolerance 1e-5 scaled (norms in F16:
2e-3); x and h (sums only), the Euler state, the assembled audio, the latent layouts and
the greedy token indices bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close, scaled_error

pytestmark = pytest.mark.gpu
TOL = 1e-5


def placed(dev, arr, offset):
    """A CUDA view of `arr` starting `offset` floats into a fresh 256-byte aligned buffer."""
    buf = torch.empty(arr.size + offset + 8, dtype=torch.float32, device=dev)
    view = buf[offset:offset + arr.size].view(arr.shape)
    view.copy_(torch.from_numpy(arr))
    return view


def empty_placed(dev, shape, offset):
    n = int(np.prod(shape))
    buf = torch.full((n + offset + 8,), np.nan, dtype=torch.float32, device=dev)
    return buf[offset:offset + n].view(shape)


@pytest.mark.parametrize("seed", range(40))
def test_fused_unit_random_layouts(ops, orc, dev, seed):
    rng = np.random.default_rng(1000 + seed)
    c = int(rng.integers(1, 200))
    t = int(rng.choice([int(rng.integers(1, 64)), int(rng.integers(64, 3000)), 8 * int(rng.integers(8, 400))]))
    mode = rng.choice(["aligned", "common_phase", "mixed"])
    if mode == "aligned":
        offs = [0, 0, 0, 0]
    elif mode == "common_phase":
        offs = [int(rng.integers(1, 8))] * 4
    else:
        offs = [int(o) for o in rng.integers(0, 8, 4)]
    has_res, has_bias, snake, write_x, tanh = (bool(b) for b in rng.integers(0, 2, 5))
    u = rng.standard_normal((c, t)).astype(np.float32)
    r = rng.standard_normal((c, t)).astype(np.float32) if has_res else None
    b = (0.05 * rng.standard_normal(c)).astype(np.float32) if has_bias else None
    al, bl = ((0.3 * rng.standard_normal((2, c))).astype(np.float32) if snake else (None, None))
    tu = placed(dev, u, offs[0])
    tr = placed(dev, r, offs[1]) if has_res else None
    x_out = empty_placed(dev, (c, t), offs[2]) if write_x else None
    y_out = empty_placed(dev, (c, t), offs[3])
    g = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    ops.fused_unit_t(tu, g(b), tr, g(al), g(bl), x_out, y_out, tanh=tanh)
    xw, yw = orc.fused_unit(u, b, r, al, bl, tanh=tanh)
    what = f"c={c} t={t} mode={mode} offs={offs} res={has_res} bias={has_bias} snake={snake} tanh={tanh}"
    # The output sums x = r + (u + b) and the snake term, then tanh (slope <= 1): relative error
    # against the size of those terms (log-parameters ~ N(0, 0.3) make the snake term up to ~2.5x
    # larger than a result that cancels towards zero).
    pre = orc.fused_unit(u, b, r, al, bl, tanh=False)[1]
    terms = np.abs(xw) + np.abs(pre - xw)
    assert_close(y_out.cpu().numpy(), yw, TOL, what, terms=terms)
    if write_x:
        assert np.array_equal(x_out.cpu().numpy(), xw), what


@pytest.mark.parametrize("seed", range(20))
def test_snakebeta_random_strides(ops, orc, dev, seed):
    rng = np.random.default_rng(2000 + seed)
    c, t = int(rng.integers(1, 100)), int(rng.integers(1, 4000))
    pad_x, pad_y = (int(p) for p in rng.integers(0, 17, 2))
    x = rng.standard_normal((c, t)).astype(np.float32)
    al, bl = (0.3 * rng.standard_normal((2, c))).astype(np.float32)
    wide_x = torch.empty((c, t + pad_x), device=dev)
    wide_x[:, :t] = torch.from_numpy(x).to(dev)
    wide_y = torch.full((c, t + pad_y), np.nan, device=dev)
    ops.snakebeta_t(wide_x[:, :t], torch.from_numpy(al).to(dev), torch.from_numpy(bl).to(dev), out=wide_y[:, :t])
    assert_close(wide_y[:, :t].cpu().numpy(), orc.snakebeta(x, al, bl), TOL, f"c={c} t={t} pads={pad_x},{pad_y}")
    if pad_y:
        assert torch.isnan(wide_y[:, t:]).all()  # nothing written past each row


def placed_dtype(dev, arr, offset, dtype):
    buf = torch.empty(arr.size + offset + 16, dtype=dtype, device=dev)
    view = buf[offset:offset + arr.size].view(arr.shape)
    view.copy_(torch.from_numpy(arr))
    return view


@pytest.mark.parametrize("seed", range(30))
def test_add_norm_random_layouts(ops, orc, dev, seed):
    """Random dims, row counts, F16 / F32, residual or none, the F16-boundary flag and element
    offsets (16-byte aligned rows take the staged form, others the register or scalar form)."""
    rng = np.random.default_rng(3000 + seed)
    layer = bool(rng.integers(0, 2))
    half = bool(rng.integers(0, 2))
    npdt, tdt = (np.float16, torch.float16) if half else (np.float32, torch.float32)
    dim = int(rng.choice([int(rng.integers(1, 64)), int(rng.integers(64, 5000)), 8 * int(rng.integers(1, 700))]))
    rows = int(rng.integers(1, 300))
    with_r = bool(rng.integers(0, 4))  # mostly with a residual
    boundary = half and bool(rng.integers(0, 2))
    off = 0 if rng.integers(0, 2) else int(rng.integers(1, 8))
    x = rng.standard_normal((rows, dim)).astype(npdt)
    r = rng.standard_normal((rows, dim)).astype(npdt) if with_r else None
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    eps = 1e-5
    tx = placed_dtype(dev, x, off, tdt)
    tr = placed_dtype(dev, r, off, tdt) if with_r else None
    h_out = placed_dtype(dev, np.zeros((rows, dim), npdt), off, tdt) if with_r else None
    y_out = placed_dtype(dev, np.zeros((rows, dim), npdt), off, tdt)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    if layer:
        ops.add_layernorm_t(tx, tr, T(g), T(b), eps, f16_boundary=boundary, h_out=h_out, y_out=y_out)
        hw, yw = orc.add_layernorm(x, r, g, b, eps, f16_boundary=boundary)
    else:
        ops.add_rmsnorm_t(tx, tr, T(g), eps, f16_boundary=boundary, h_out=h_out, y_out=y_out)
        hw, yw = orc.add_rmsnorm(x, r, g, eps, f16_boundary=boundary)
    what = f"layer={layer} half={half} rows={rows} dim={dim} res={with_r} boundary={boundary} off={off}"
    if with_r:
        assert np.array_equal(h_out.cpu().numpy(), hw), what
    assert_close(y_out.cpu().numpy().astype(np.float64), yw.astype(np.float64), 2e-3 if half else 1e-5, what)


@pytest.mark.parametrize("seed", range(20))
def test_weightnorm_random_layouts(ops, orc, dev, seed):
    rng = np.random.default_rng(4000 + seed)
    rows = int(rng.integers(1, 300))
    cols = int(rng.choice([int(rng.integers(1, 40)), int(rng.integers(40, 13000)), 4 * int(rng.integers(1, 4000))]))
    off = 0 if rng.integers(0, 2) else int(rng.integers(1, 8))
    v = (0.02 * rng.standard_normal((rows, cols))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, rows).astype(np.float32)
    tv = placed(dev, v, off)
    w = empty_placed(dev, (rows, cols), off)
    ops.weightnorm_t(tv, torch.from_numpy(g).to(dev), w=w)
    want, _, ok = orc.weightnorm(v, g)
    assert ok
    assert_close(w.cpu().numpy(), want, TOL, f"rows={rows} cols={cols} off={off}")


@pytest.mark.parametrize("seed", range(20))
def test_cfg_euler_random_schedules(ops, orc, dev, seed):
    """Random batch / row / prefix, resume points and step counts (past one 64-step staging
    chunk), with and without CFG: bit-exact with the oracle."""
    rng = np.random.default_rng(5000 + seed)
    batch = int(rng.integers(1, 4))
    row = int(rng.choice([64 * int(rng.integers(1, 40)), int(rng.integers(1, 3000))]))
    steps = int(rng.integers(1, 90))
    first = int(rng.integers(0, steps))
    count = int(rng.integers(1, steps - first + 1))
    prefix = int(rng.integers(0, row + 1)) if rng.integers(0, 2) else 0
    cfg = bool(rng.integers(0, 2))
    guidance = float(rng.uniform(0.5, 3.0))
    n = batch * row
    x = rng.standard_normal(n).astype(np.float32)
    noise = rng.standard_normal(n).astype(np.float32)
    ctx = rng.standard_normal(n).astype(np.float32)
    vu, vc = rng.standard_normal((2, count, n)).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    st = T(x)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.cfg_euler_multi_t(st, T(noise), T(ctx), T(vu), T(vc) if cfg else None, batch=batch, prefix=prefix,
                          first_step=first, count=count, steps=steps, cfg=cfg, guidance=guidance, sigma_min=1e-4,
                          status=status)
    want, ok = orc.cfg_euler(x, noise, ctx, vu, vc if cfg else None, batch=batch, prefix=prefix, first_step=first,
                             count=count, steps=steps, cfg=cfg, guidance=guidance, sigma_min=1e-4)
    what = f"batch={batch} row={row} steps={steps} first={first} count={count} prefix={prefix} cfg={cfg}"
    assert ok and status.item() == 0, what
    assert np.array_equal(st.cpu().numpy(), want), what


@pytest.mark.parametrize("seed", range(20))
def test_assembly_random_schedules(ops, orc, dev, seed):
    """Random valid schedules (0 or 2 <= overlap <= hop, hop + overlap <= window), planar and
    interleaved output: bit-exact with the oracle."""
    rng = np.random.default_rng(6000 + seed)
    n = int(rng.integers(1, 9))
    win = int(rng.integers(3, 400))
    overlap = 0 if (win < 4 or rng.integers(0, 4) == 0) else int(rng.integers(2, win // 2 + 1))
    hop = int(rng.integers(max(overlap, 1), win - overlap + 1))
    target = int(rng.integers(0, (n - 1) * hop + win + 1))
    channels = int(rng.integers(1, 4))
    w = rng.standard_normal((n, channels, win)).astype(np.float32)
    tw = torch.from_numpy(w).to(dev)
    want = orc.assemble_windows(w, hop, overlap, target)
    what = f"n={n} win={win} hop={hop} overlap={overlap} target={target} channels={channels}"
    assert np.array_equal(ops.assemble_windows_t(tw, hop, overlap, target).cpu().numpy(), want), what
    inter = ops.assemble_windows_t(tw, hop, overlap, target, interleaved=True).cpu().numpy()
    assert np.array_equal(inter.reshape(target, channels).T, want), what


@pytest.mark.parametrize("seed", range(20))
def test_greedy_random_rows(ops, orc, dev, seed):
    """Random vocab sizes, row counts, penalties, recent-token lists (with -1 padding and ids
    past the penalty limit) and ignore lists: the same token indices as the oracle."""
    rng = np.random.default_rng(7000 + seed)
    rows = int(rng.integers(1, 40))
    vocab = int(rng.integers(2, 20000))
    x = (rng.standard_normal((rows, vocab)) * rng.uniform(0.1, 20)).astype(np.float32)
    if rng.integers(0, 3) == 0:  # ties at the maximum
        x[:, rng.integers(0, vocab, 8)] = x.max()
    recent = rng.integers(-1, vocab, (rows, int(rng.integers(1, 80))))
    ignore = rng.integers(0, vocab, int(rng.integers(1, 20))) if rng.integers(0, 2) else None
    penalty = float(rng.choice([1.0, rng.uniform(1.0, 2.0)]))
    limit = int(rng.integers(0, vocab + 1))
    T = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    got = ops.greedy_tokens_t(T(x), recent=T(recent), penalty=penalty, penalty_limit=limit, ignore=T(ignore)).cpu()
    want, ok = orc.greedy_tokens(x, recent, penalty, limit, ignore)
    assert ok
    assert np.array_equal(got.numpy(), want), f"rows={rows} vocab={vocab} penalty={penalty} limit={limit}"


@pytest.mark.parametrize("seed", range(10))
def test_latent_random_shapes(ops, orc, dev, seed):
    rng = np.random.default_rng(8000 + seed)
    frames, dim = int(rng.integers(1, 3000)), int(rng.integers(1, 200))
    x = rng.standard_normal((frames, dim)).astype(np.float32)
    mean = rng.standard_normal(dim).astype(np.float32)
    std = rng.uniform(0.5, 2.0, dim).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    assert np.array_equal(ops.latent_to_vae_t(T(x), T(mean), T(std)).cpu().numpy(), orc.latent_to_vae(x, mean, std))
    assert np.array_equal(ops.latent_normalize_t(T(x), T(mean), T(std)).cpu().numpy(),
                          orc.latent_normalize(x, mean, std))


@pytest.mark.parametrize("seed", range(16))
def test_chain_random_topologies(ops, orc, dev, seed):
    """Random decoder topologies (1-8 stages, widths, strides, 0-4 residual units, channel
    counts), frame counts, F32- or F16-stored parameters and the tanh epilogue, through the
    device decode and the stage capture, against the oracle's node-by-node chain.

    With identity stand-ins for the residual convs, every residual unit feeds its SnakeBeta
    output back into the stream and roughly doubles it, so deep random chains are badly
    conditioned: the oracle's own output moves by up to ~2e-4 (scaled) when its input moves
    by one ulp.  Each tensor's bar is therefore max(1e-5, 10 x that measured 1-ulp
    sensitivity of the oracle); the BASELINE-shape chain tests keep a flat 1e-5.  A layout or
    indexing error shows as an O(1) difference."""
    rng = np.random.default_rng(9000 + seed)
    t = ops.Topology()
    t.latent_dim, t.audio_channels = int(rng.integers(1, 17)), int(rng.integers(1, 4))
    t.entry_width, t.n_stages = int(rng.integers(1, 97)), int(rng.integers(1, 9))
    total = 1
    for s in range(t.n_stages):
        t.stage_width[s] = int(rng.integers(1, 65))
        t.stage_stride[s] = int(rng.integers(1, 7)) if total < 2000 else 1
        total *= t.stage_stride[s]
    t.n_residual = int(rng.integers(0, 5))
    for r in range(t.n_residual):
        t.dilation[r] = int(rng.choice([1, 3, 9, 27]))
    frames = int(rng.integers(1, 41))
    tanh = bool(rng.integers(0, 2))
    params = (0.1 * rng.standard_normal(ops.param_count(t))).astype(np.float32)
    if rng.integers(0, 2):
        params = params.astype(np.float16)
    latent = rng.standard_normal((t.latent_dim, frames)).astype(np.float32)
    chain = ops.VaeChain(t, params, max_frames=frames, device=0)
    run = lambda lat: orc.vae_chain(t.as_list(), params.astype(np.float32), lat, frames,  # noqa: E731
                                    t.audio_channels, frames * t.upsampling(), tanh=tanh, stages=True)
    want, want_stages = run(latent)
    nudged, nudged_stages = run(np.nextafter(latent, np.float32(np.inf)))  # the problem's own conditioning
    bar = lambda a, b: max(TOL, 10 * scaled_error(b, a))  # noqa: E731
    stages = [torch.full(w.shape, np.nan, device=dev) for w in want_stages]
    chain.set_stage_capture(stages)
    audio = torch.full((t.audio_channels, chain.samples(frames)), np.nan, device=dev)
    chain.decode(torch.from_numpy(latent).to(dev), audio, frames, flags=ops.CHAIN_TANH if tanh else 0)
    torch.cuda.synchronize()
    what = f"topology={t.as_list()} frames={frames} tanh={tanh} f16={params.dtype == np.float16}"
    assert_close(audio.cpu().numpy(), want, bar(want, nudged), what)
    for s, (got, w, wn) in enumerate(zip(stages, want_stages, nudged_stages)):
        assert_close(got.cpu().numpy(), w, bar(w, wn), f"{what} stage {s}")
    chain.close()
