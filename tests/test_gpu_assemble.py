"""GPU parity of the window assembly (crossfade + crop + interleave) against
the oracle and the reference's own assemble_renderer_audio (compiled from its
sources into oracle/_ref): bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WIN, HOP, OV = 1000 * 1920, 750 * 1920, 250 * 1920


def test_assembly_known_answer(ops, dev):
    # tests/test-renderer-pattern.cpp:93-108
    w = torch.empty((2, 2, WIN), device=dev)
    w[0, 0], w[0, 1], w[1, 0], w[1, 1] = 1.0, 2.0, 3.0, 4.0
    out = ops.assemble_windows_t(w, HOP, OV, 1001 * 1920).cpu().numpy()
    assert abs(out[0, HOP] - 1.0) < 1e-6 and abs(out[0, HOP + OV - 1] - 3.0) < 1e-6
    assert abs(out[0, HOP + OV] - 3.0) < 1e-6 and abs(out[1, 0] - 2.0) < 1e-6 and abs(out[1, -1] - 4.0) < 1e-6


@pytest.mark.parametrize("source_frames", [1, 1000, 1001, 1751, 3000])
def test_assembly_bit_exact_vs_reference(ops, orc, dev, source_frames):
    rng = np.random.default_rng(source_frames)
    if orc.ref_available():
        sched = orc.ref_make_renderer_schedule(source_frames)
        n, target = len(sched["windows"]), sched["target_samples"]
    else:  # the same schedule restated: ceil((T - overlap) / hop) windows after the first
        n = 1 if source_frames <= 1000 else -(-(source_frames - 250) // 750)
        target = source_frames * 1920
    w = rng.standard_normal((n, 2, WIN)).astype(np.float32)
    tw = torch.from_numpy(w).to(dev)
    planar = ops.assemble_windows_t(tw, HOP, OV, target).cpu().numpy()
    inter = ops.assemble_windows_t(tw, HOP, OV, target, interleaved=True).cpu().numpy()
    want = orc.assemble_windows(w, HOP, OV, target)
    assert np.array_equal(planar, want)
    assert np.array_equal(inter, want.T)
    if orc.ref_available():
        ref_l, ref_r = orc.ref_assemble_renderer_audio(source_frames, w[:, 0], w[:, 1])
        assert np.array_equal(planar[0], ref_l) and np.array_equal(planar[1], ref_r)


@pytest.mark.parametrize("n,win,hop,ov,target", [(3, 20, 12, 5, 44), (1, 7, 3, 2, 5), (4, 16, 16, 0, 60),
                                                  (5, 33, 20, 13, 113), (2, 10, 5, 5, 15)])
def test_assembly_general_schedules(ops, orc, dev, n, win, hop, ov, target):
    rng = np.random.default_rng(n * 100 + win)
    w = rng.standard_normal((n, 3, win)).astype(np.float32)
    got = ops.assemble_windows_t(torch.from_numpy(w).to(dev), hop, ov, target).cpu().numpy()
    assert np.array_equal(got, orc.assemble_windows(w, hop, ov, target))


def test_assembly_rejects_chained_overlaps(ops, dev):
    w = torch.zeros((2, 2, 10), device=dev)
    with pytest.raises(ValueError, match="overlap descriptor"):
        ops.assemble_windows_t(w, 4, 6, 12)
    with pytest.raises(ValueError, match="target crop"):
        ops.assemble_windows_t(w, 5, 5, 16)


# (window, channel, sample) plants; the reference reports the first window in order, left before right
PLANTS = {
    "window 0 right, start": [(0, 1, 5)],
    "window 1 left, crossfaded head": [(1, 0, 17)],
    "window 0 left, tail read as the next window's overlap": [(0, 0, HOP + 3)],
    "later window listed first": [(2, 0, 0), (1, 1, WIN - 1)],
    "last window, past the crop": [(-1, 0, WIN - 1)],
}


@pytest.mark.parametrize("plant", list(PLANTS))
@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_assembly_rejects_nonfinite_like_the_reference(ops, orc, dev, plant, bad):
    """assemble_renderer_audio rejects a decoded window holding a non-finite sample with
    std::invalid_argument naming the channel of the first failing window (src/levo-renderer-pattern.cpp:
    25-28,159-160); the CUDA path raises a ValueError with the same text for the same window and channel."""
    source_frames = 2300  # 3 windows; the crop ends inside the last one
    n = 3
    target = source_frames * 1920
    rng = np.random.default_rng(7)
    w = rng.standard_normal((n, 2, WIN)).astype(np.float32)
    for k, c, s in PLANTS[plant]:
        w[k, c, s] = bad
    k_first, c_first = min((k % n, c) for k, c, _ in PLANTS[plant])
    side = ("left", "right")[c_first]
    if orc.ref_available():
        assert len(orc.ref_make_renderer_schedule(source_frames)["windows"]) == n
        with pytest.raises(ValueError, match=f"decoded {side} channel contains non-finite samples"):
            orc.ref_assemble_renderer_audio(source_frames, w[:, 0], w[:, 1])
    with pytest.raises(ValueError, match=f"decoded {side} channel contains non-finite samples \\(window {k_first}\\)"):
        ops.assemble_windows_t(torch.from_numpy(w).to(dev), HOP, OV, target)


@pytest.mark.parametrize("k,s", [(0, 18), (1, 17), (2, 19), (2, 5)])
def test_assembly_checks_samples_no_output_reads(ops, dev, k, s):
    """3 windows of 20 samples, hop 12, overlap 5, crop at 43: samples 17..19 of windows 0 and 1 feed no
    output (hop + overlap = 17), nor does sample 19 of the last window (it would land at 43); sample 5
    of the last window is read.  Every sample is still checked, as the reference checks whole windows."""
    w = np.zeros((3, 2, 20), np.float32)
    w[k, 1, s] = np.nan
    with pytest.raises(ValueError, match=f"decoded right channel contains non-finite samples \\(window {k}\\)"):
        ops.assemble_windows_t(torch.from_numpy(w).to(dev), 12, 5, 43)


def test_assembly_without_the_check_runs_through(ops, dev):
    w = torch.zeros((2, 2, 10), device=dev)
    w[1, 0, 9] = float("nan")
    out = ops.assemble_windows_t(w, 5, 5, 15, check_finite=False)
    assert torch.isnan(out[0, 14]).item()


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("k,s", [(0, 17), (1, 19), (2, 18), (2, 3)])
def test_assembly_vector_form_checks_samples_no_output_reads(ops, dev, interleaved, k, s):
    """The same check on the four-samples-at-a-time form (every length a multiple of 4): 3 stereo windows
    of 20 samples, hop 12, overlap 4, crop at 40: samples 16..19 of every window feed no output; sample 3
    of the last one does."""
    w = np.zeros((3, 2, 20), np.float32)
    w[k, 0, s] = np.inf
    with pytest.raises(ValueError, match=f"decoded left channel contains non-finite samples \\(window {k}\\)"):
        ops.assemble_windows_t(torch.from_numpy(w).to(dev), 12, 4, 40, interleaved=interleaved)


def test_assembly_vector_and_scalar_forms_agree(ops, orc, dev):
    """An output tensor one float past a 16-byte boundary takes the scalar form; both forms give the
    oracle's bits."""
    rng = np.random.default_rng(41)
    w = rng.standard_normal((4, 2, 64)).astype(np.float32)
    tw = torch.from_numpy(w).to(dev)
    want = orc.assemble_windows(w, 48, 16, 200)
    vec = ops.assemble_windows_t(tw, 48, 16, 200).cpu().numpy()
    buf = torch.empty(2 * 200 + 1, device=dev)
    scalar = ops.assemble_windows_t(tw, 48, 16, 200, out=buf[1:].view(2, 200)).cpu().numpy()
    assert np.array_equal(vec, want) and np.array_equal(scalar, want)
