"""Builds liblevo_b200.so in-tree from csrc/*.cu for sm_100a.

Each translation unit is compiled in parallel with nvcc, then linked into one
shared library exporting only the C ABI of include/levo_ops.h (everything
else has hidden visibility).  The CUDA runtime is linked statically, so the
library needs nothing but the driver at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "liblevo_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblevo_b200.so")
    return path


def _sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def _needs_build() -> bool:
    if not LIB.exists():
        return True
    stamp = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [ROOT / "include" / "levo_ops.h", pathlib.Path(__file__)]
    return any(p.stat().st_mtime > stamp for p in deps if p.is_file())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> pathlib.Path:
    """Compiles every csrc/*.cu and links liblevo_b200.so; returns its path."""
    if not force and not _needs_build():
        return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(src: pathlib.Path) -> tuple[pathlib.Path, str]:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, _sources()))
    if verbose or ptxas_info:
        for obj, log in results:
            if log.strip():
                print(f"--- {obj.name}\n{log}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *[str(o) for o, _ in results]]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv))
