"""bench.py's arms, checked on the CPU.

The reference arm (`--impl reference`) times the reference's CPU path (its
node-by-node restatement under oracle/) and must not import or load anything
of levo2.cpp_b200; its topology and parameter packing come from the oracle
side and are pinned here against the library's own."""
from __future__ import annotations

import json
import subprocess
import sys

import numpy as np

from conftest import ROOT


def test_oracle_topology_matches_the_library(ops, orc):
    t = ops.reference_topology()
    assert list(orc.REFERENCE_TOPOLOGY) == t.as_list()
    assert list(orc.REFERENCE_DILATIONS) == list(t.dilation[:t.n_residual])
    assert orc.param_count(orc.REFERENCE_TOPOLOGY) == ops.param_count(t)
    assert orc.upsampling(orc.REFERENCE_TOPOLOGY) == t.upsampling() == 1920


def test_both_arms_pack_identical_parameters(ops, orc):
    sys.path.insert(0, str(ROOT))
    import bench

    own = bench.make_params(bench.topology_list(ops.reference_topology()))
    ref = bench.make_params(list(orc.REFERENCE_TOPOLOGY))
    assert own.size == ops.param_count(ops.reference_topology())
    assert np.array_equal(own, ref)


def test_reference_arm_loads_nothing_of_the_product(tmp_path):
    """Runs the reference arm on a tiny window in a fresh process and inspects what it mapped."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '2', '--warmup', '1', '--frames', '3']\n"
        "try:\n"
        "    runpy.run_path(%r, run_name='__main__')\n"
        "except SystemExit as e:\n"
        "    assert not e.code, e.code\n"
        "maps = open('/proc/self/maps').read()\n"
        "sys.stderr.write('MAPS ' + str('liblevo_b200' in maps) + ' ' + str('liblevo_oracle' in maps) + '\\n')\n"
        "sys.stderr.write('MODS ' + str(any(m.startswith('levo2_cpp_b200') for m in sys.modules)) + ' '\n"
        "                 + str('torch' in sys.modules) + '\\n')\n" % str(ROOT / "bench.py")
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=tmp_path, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "MAPS False True" in out.stderr, out.stderr[-2000:]
    assert "MODS False False" in out.stderr, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["unit"] == "audio-s/s"
    assert "one whole window of 3 latent frames" in line["cpu_baseline"]["sample"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
