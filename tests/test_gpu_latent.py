"""GPU parity of the latent path into the VAE (next item f2): de-normalise +
frame-major -> channel-major transpose, and normalise.  Bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("frames,dim", [(1000, 64), (1, 64), (33, 7), (750, 64), (5, 100)])
def test_latent_to_vae_bit_exact(ops, orc, dev, frames, dim):
    rng = np.random.default_rng(frames + dim)
    x = rng.standard_normal((frames, dim)).astype(np.float32)
    mean = rng.standard_normal(dim).astype(np.float32)
    std = rng.uniform(0.5, 2.0, dim).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    got = ops.latent_to_vae_t(T(x), T(mean), T(std)).cpu().numpy()
    assert np.array_equal(got, orc.latent_to_vae(x, mean, std))
    assert np.array_equal(ops.latent_to_vae_t(T(x)).cpu().numpy(), x.T)
    norm = ops.latent_normalize_t(T(x), T(mean), T(std)).cpu().numpy()
    assert np.array_equal(norm, orc.latent_normalize(x, mean, std))


def test_latent_round_trip_into_the_chain(ops, dev):
    # normalise -> de-normalise recovers the raw latent to rounding, in the VAE layout
    rng = np.random.default_rng(3)
    raw = rng.standard_normal((750, 64)).astype(np.float32) * 3 + 1
    mean = rng.standard_normal(64).astype(np.float32)
    std = rng.uniform(0.5, 2.0, 64).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    back = ops.latent_to_vae_t(ops.latent_normalize_t(T(raw), T(mean), T(std)), T(mean), T(std)).cpu().numpy()
    assert np.allclose(back, raw.T, rtol=1e-6, atol=1e-6)


def test_latent_to_vae_rejects_in_place(ops, dev):
    x = torch.zeros((8, 8), device=dev)
    with pytest.raises(ValueError, match="in place"):
        ops.latent_to_vae_t(x, out=x)


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
@pytest.mark.parametrize("where", [(0, 0), (749, 63), (400, 17)])
def test_latent_functions_reject_nonfinite_inputs(ops, dev, bad, where):
    """normalize_latents / denormalize_latents reject a non-finite input before computing
    (require_finite, src/levo-flow-conditioning.cpp:42-44,116,128): the same message here; without the
    check the value just passes through."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((750, 64)).astype(np.float32)
    x[where] = bad
    mean = rng.standard_normal(64).astype(np.float32)
    std = rng.uniform(0.5, 2.0, 64).astype(np.float32)
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    with pytest.raises(ops.LevoNonFinite, match="raw latent contains a non-finite value"):
        ops.latent_normalize_t(T(x), T(mean), T(std))
    with pytest.raises(ops.LevoNonFinite, match="normalized latent contains a non-finite value"):
        ops.latent_to_vae_t(T(x), T(mean), T(std))
    got = ops.latent_to_vae_t(T(x), T(mean), T(std), check_finite=False).cpu().numpy()
    assert not np.isfinite(got[where[1], where[0]])
    finite = ops.latent_to_vae_t(T(np.nan_to_num(x, posinf=0.0, neginf=0.0)), T(mean), T(std))
    assert torch.isfinite(finite).all().item()
