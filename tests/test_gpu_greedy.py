"""GPU parity of greedy next-token selection (next item f3): bit-exact token
indices against the oracle and the reference's own Sampler::sample_streams
(use_sampling = false), compiled from its sources into oracle/_ref."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
VOCAB = 16385  # LeLM codebook 16384 + EOS


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_greedy_known_answers(ops, dev):
    # tests/test-sampling.cpp:12-15 and :36
    out = ops.greedy_tokens_t(T(np.array([[9, 8, 10, 7]], np.float32), dev), recent=T(np.array([[2, 3]]), dev),
                              penalty=2.0, penalty_limit=3)
    assert out.cpu().tolist() == [0]
    out = ops.greedy_tokens_t(T(np.array([[0, 2, 1], [1, 4, 0]], np.float32), dev))
    assert out.cpu().tolist() == [1, 1]


@pytest.mark.parametrize("trial", range(8))
def test_greedy_matches_oracle_and_reference(ops, orc, dev, trial):
    rng = np.random.default_rng(100 + trial)
    rows = 3 if trial < 6 else 17
    x = rng.standard_normal((rows, VOCAB)).astype(np.float32) * (10 if trial % 2 else 1)
    if trial in (2, 3):
        x[:, rng.integers(0, VOCAB, 64)] = x.max() + 0.5  # many ties at the maximum
    if trial == 4:
        x[1] = -np.inf  # all -inf: index 0
    if trial == 5:
        x[:] = 7.0  # all equal: index 0
    recent = rng.integers(-1, VOCAB, (rows, 50))
    ignore = rng.integers(0, VOCAB, 16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    got = ops.greedy_tokens_t(T(x, dev), recent=T(recent, dev), penalty=1.1, penalty_limit=VOCAB - 1,
                              ignore=T(ignore, dev), status=status).cpu().numpy()
    want, ok = orc.greedy_tokens(x, recent, 1.1, VOCAB - 1, ignore)
    assert ok and status.item() == 0
    assert np.array_equal(got, want)
    if orc.ref_available():
        assert np.array_equal(got, orc.ref_sample_streams_greedy(x, recent, 1.1, ignore))


def test_greedy_without_penalty_is_plain_first_argmax(ops, dev):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((5, 1000)).astype(np.float32)
    x[2, [10, 500, 900]] = 99.0
    got = ops.greedy_tokens_t(T(x, dev)).cpu().numpy()
    assert got.tolist() == [int(np.argmax(r)) for r in x]  # numpy argmax is also first-max


def test_greedy_strided_rows(ops, dev):
    rng = np.random.default_rng(8)
    big = rng.standard_normal((4, 3000)).astype(np.float32)
    t = T(big, dev)[:, :2500]
    got = ops.greedy_tokens_t(t).cpu().numpy()
    assert got.tolist() == [int(np.argmax(r[:2500])) for r in big]


def test_greedy_nan_sets_status(ops, dev):
    # The reference throws on a NaN logit (src/levo-sampling.cpp:79).
    x = torch.zeros((2, 100), device=dev)
    x[1, 42] = float("nan")
    x[1, 7] = 3.0
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    got = ops.greedy_tokens_t(x, status=status).cpu().tolist()
    assert status.item() == 1 and got == [0, 7]


def test_greedy_rejects_bad_arguments(ops, dev):
    x = torch.zeros((1, 10), device=dev)
    with pytest.raises(ValueError, match="penalty"):
        ops.greedy_tokens_t(x, recent=torch.zeros((1, 2), dtype=torch.int64, device=dev), penalty=0.0)
