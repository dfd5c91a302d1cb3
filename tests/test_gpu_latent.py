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
