"""The C ABI surface, checked without a GPU: the library loads, exports every
symbol include/levo_ops.h declares (and the Python binding declares the same
set), and argument validation fails with LEVO_OPS_EINVAL before any CUDA call."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "levo_ops.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"LEVO_OPS_API\s+[\w\s\*]+?\b(levo_\w+)\s*\(", text))


def test_header_and_binding_agree(ops):
    declared = declared_symbols()
    assert len(declared) >= 20
    assert declared == set(ops.SIGNATURES), declared ^ set(ops.SIGNATURES)


def test_library_exports_every_declared_symbol(ops):
    lib = ops.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.levo_ops_abi_version() == 1


def test_only_the_c_abi_is_exported(ops):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(ops.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ours = {s for s in exported if s.startswith("levo_")}
    assert ours == declared_symbols()


def test_reference_topology_and_param_count(ops):
    t = ops.reference_topology()
    assert (t.latent_dim, t.audio_channels, t.entry_width, t.n_stages, t.n_residual) == (64, 2, 2048, 5, 3)
    assert list(t.stage_width[:5]) == [1024, 512, 256, 128, 128]
    assert list(t.stage_stride[:5]) == [10, 6, 4, 4, 2]
    assert list(t.dilation[:3]) == [1, 3, 9]
    assert t.upsampling() == 1920
    # input.bias + per stage (2*Cin + Cout + 6*Cout*R) + output snake
    widths, cin, n = [1024, 512, 256, 128, 128], 2048, 2048
    for c in widths:
        n += 2 * cin + c + 6 * c * 3
        cin = c
    n += 2 * 128
    assert ops.param_count(t) == n


def test_invalid_arguments_are_einval_without_gpu(ops):
    lib = ops.lib()
    assert lib.levo_snakebeta_f32(None, 4, None, None, 0, None, 4, 1, 4, None) == ops.EINVAL
    assert "null" in ops.last_error()
    assert lib.levo_cfg_combine_f32(None, None, None, 0, 1.5, None) == ops.EINVAL
    # non-empty check mirrors combine_renderer_cfg (src/levo-renderer-pattern.cpp:127-128)
    buf = (ctypes.c_float * 8)()
    p = ctypes.addressof(buf)
    assert lib.levo_cfg_combine_f32(p, p, p, 0, 1.5, None) == ops.EINVAL
    assert "non-empty" in ops.last_error()
    assert lib.levo_cfg_combine_f32(p, p, p, 8, float("nan"), None) == ops.EINVAL
    assert lib.levo_euler_cfg_step_f32(p, p, p, 8, 1, 1.5, 0, None, None) == ops.EINVAL
    assert "step count" in ops.last_error()
    assert lib.levo_flow_incontext_f32(p, p, p, 1, 4, 5, 0, 2, 0.1, None) == ops.EINVAL
    assert "exceeds frame count" in ops.last_error()
    assert lib.levo_cfg_euler_multi_f32(p, p, p, p, p, 1, 8, 0, 3, 2, 4, 1, 1.5, 1e-4, None, None) == ops.EINVAL
    assert "resume step" in ops.last_error()
    assert lib.levo_add_rmsnorm_f16(p, None, None, None, p, 1, 8, 1e-6, 0, None) == ops.EINVAL
    assert lib.levo_add_rmsnorm_f32(p, None, p, None, p, 1, 8, -1.0, 0, None) == ops.EINVAL
    assert lib.levo_add_rmsnorm_f32(p, None, p, None, p, 1, 8, 1e-6, 1, None) == ops.EINVAL  # F16 flag on F32
    assert lib.levo_weightnorm_f32(p, None, p, None, 1, 8, None) == ops.EINVAL
    # misaligned pointer
    assert lib.levo_weightnorm_f32(p + 2, p, p, None, 1, 2, None) == ops.EINVAL
    # fused unit: no outputs
    u = ops.FusedUnit(p, None, None, None, None, None, None, 1, 8, 0, 0)
    assert lib.levo_vae_fused_unit_f32(ctypes.byref(u), None) == ops.EINVAL
    assert "no output" in ops.last_error()
    u = ops.FusedUnit(p, None, None, p, None, None, p, 1, 8, 0, 0)
    assert lib.levo_vae_fused_unit_f32(ctypes.byref(u), None) == ops.EINVAL


def test_snake_params_prepare_validation_without_gpu(ops):
    lib = ops.lib()
    buf = (ctypes.c_float * 8)()
    p = ctypes.addressof(buf)
    assert lib.levo_snake_params_prepare(p, p, ops.DTYPE_SNAKE_PREPARED, 4, p, p, None) == ops.EINVAL
    assert lib.levo_snake_params_prepare(p, None, 0, 4, p, p, None) == ops.EINVAL
    assert "null" in ops.last_error()
    assert lib.levo_snake_params_prepare(p, p, 0, -1, p, p, None) == ops.EINVAL
    assert lib.levo_snake_params_prepare(p + 2, p, 0, 4, p, p, None) == ops.EINVAL
    assert lib.levo_snakebeta_f32(p, 4, p, p, 3, p, 4, 1, 4, None) == ops.EINVAL  # unknown dtype


def test_zero_sizes_are_noops_without_gpu(ops):
    lib = ops.lib()
    buf = (ctypes.c_float * 8)()
    p = ctypes.addressof(buf)
    assert lib.levo_snakebeta_f32(p, 0, p, p, 0, p, 0, 0, 0, None) == ops.OK
    assert lib.levo_snakebeta_f32(p, 0, p, p, 0, p, 0, 5, 0, None) == ops.OK
    assert lib.levo_add_layernorm_f32(p, None, p, p, None, p, 0, 16, 1e-5, 0, None) == ops.OK
    assert lib.levo_weightnorm_f32(p, p, p, None, 0, 7, None) == ops.OK
    assert lib.levo_snake_params_prepare(p, p, 0, 0, p, p, None) == ops.OK
    assert lib.levo_vae_chain_set_stage_capture(None, None, 0) == ops.EINVAL  # no chain
    assert lib.levo_vae_chains_decode_windows(None, 0, p, 1, 1, p, 0, ops.CANCEL_FN(), None) == ops.EINVAL
    assert lib.levo_snake_params_prepare(p, p, 0, 0, p, p, None) == ops.OK


def test_chain_rejects_bad_topology_without_gpu(ops):
    lib = ops.lib()
    t = ops.reference_topology()
    t.n_stages = 9
    h = ctypes.c_void_p()
    params = (ctypes.c_float * 4)()
    assert lib.levo_vae_chain_create(ctypes.byref(h), ctypes.byref(t), ctypes.addressof(params), 10, ops.CONV_FN(),
                                     None, 0) == ops.EINVAL
    assert "n_stages" in ops.last_error()
    assert lib.levo_vae_param_count(ctypes.byref(t)) == ops.EINVAL


def test_product_package_does_not_reference_the_oracle():
    pkg = ROOT / "levo2.cpp_b200"
    for path in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh")):
        text = path.read_text()
        assert "oracle" not in text.lower(), f"{path} mentions the oracle"
        assert "_work/" not in text, path


def test_missing_library_fails_loudly(tmp_path):
    """The product path has no fallback: without liblevo_b200.so every call raises."""
    import subprocess
    import sys

    code = (
        "import pathlib, sys; sys.path.insert(0, %r); import __graft_entry__ as e; ops = e.load_package().ops; "
        "ops.LIB_PATH = pathlib.Path(%r); "
        "import numpy as np\n"
        "try:\n    ops.lib()\nexcept ops.LevoOpsError as err:\n    print('raised', err)\n" % (str(ROOT), str(tmp_path / "missing.so"))
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert "raised" in out.stdout and "missing" in out.stdout, out.stdout + out.stderr


@pytest.mark.parametrize("lang,header,std", [("c", "levo_ops.h", "-std=c99"), ("c++", "levo_ops.hpp", "-std=c++17")])
def test_headers_compile_standalone(lang, header, std):
    """levo_ops.h is plain C99 (a cgo / ctypes / JNI binding can include it); levo_ops.hpp is C++17."""
    import shutil
    import subprocess

    compiler = shutil.which("gcc" if lang == "c" else "g++")
    if compiler is None:
        pytest.skip("no host compiler")
    out = subprocess.run([compiler, std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only", "-x", lang,
                          str(ROOT / "include" / header)], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr


def test_multi_chain_decode_rejects_a_chain_passed_twice_without_gpu(ops):
    """Two entries naming one chain would share its workspace and streams across threads: EINVAL,
    checked before any chain is touched."""
    lib = ops.lib()
    dummy = (ctypes.c_float * 8)()
    fake = ctypes.addressof(dummy)  # never dereferenced: the duplicate check comes first
    handles = (ctypes.c_void_p * 2)(fake, fake)
    buf = (ctypes.c_float * 8)()
    p = ctypes.addressof(buf)
    rc = lib.levo_vae_chains_decode_windows(ctypes.cast(handles, ctypes.c_void_p), 2, p, 1, 1, p, 0, ops.CANCEL_FN(),
                                            None)
    assert rc == ops.EINVAL
    assert "passed twice" in ops.last_error()


def test_decode_windows_binding_validates_host_buffers(ops):
    """The binding checks dtype, contiguity and sizes before the C ABI copies into host memory."""
    import numpy as np

    t = ops.reference_topology()
    frames = 4
    lat = np.zeros((2, t.latent_dim, frames), np.float32)
    audio = np.zeros((2, t.audio_channels, frames * t.upsampling()), np.float32)
    assert ops._host_window_buffers(t, lat, audio, frames)[0] == 2
    with pytest.raises(ValueError, match="float32"):
        ops._host_window_buffers(t, lat.astype(np.float64), audio, frames)
    with pytest.raises(ValueError, match="shape"):
        ops._host_window_buffers(t, lat, audio, frames + 1)
    with pytest.raises(ValueError, match="need"):
        ops._host_window_buffers(t, lat, audio[:1], frames)
    with pytest.raises(ValueError, match="C-contiguous"):
        ops._host_window_buffers(t, lat, np.zeros((2, frames * t.upsampling(), 4), np.float32).transpose(0, 2, 1),
                                 frames)
