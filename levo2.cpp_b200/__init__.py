"""levo2.cpp_b200 — B200 (sm_100a) kernels for LeVo2.cpp's elementwise, broadcast
and row-reduction layer, behind the C ABI of include/levo_ops.h.

Layout:
  csrc/          CUDA kernels and the extern "C" layer (built into liblevo_b200.so)
  ops.py         ctypes binding of that C ABI + torch convenience wrappers
  sharding.py    one-window-per-GPU host logic (window ranges, host gather)
  build_ext.py   nvcc build of liblevo_b200.so for sm_100a

The directory name is not a Python identifier; load it with
__graft_entry__.load_package(), which registers it as `levo2_cpp_b200`.
"""
from . import ops, sharding  # noqa: F401

__all__ = ["ops", "sharding"]
