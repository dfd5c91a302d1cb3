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
