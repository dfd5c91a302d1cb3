"""Multi-GPU host logic for independent render windows.

VAE windows are independent (the reference decodes them one after another,
src/levo-render.cpp:442-451, src/cantor-abi.cpp:901-913), so N processes — one
per GPU — each decode a contiguous block of windows with no collective on the
data path.  The audio comes back to the host directly into one shared-memory
buffer laid out [windows][channels][samples] (the host gather); rank 0 owns
and finally unlinks it.  Collectives appear only for timing (a barrier and a
max over ranks), never for data.
"""
from __future__ import annotations

import os
import tempfile
from multiprocessing import shared_memory
from typing import Callable, Optional

import numpy as np


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block [start, stop) of n_items for `rank` out of `world` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world or n_items < 0:
        raise ValueError("invalid shard request")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class HostGather:
    """A [windows, channels, samples] F32 buffer in POSIX shared memory shared by the local ranks.

    Rank 0 creates it before `barrier()`; the others attach after it.  `view(start, stop)` is
    the slice a rank writes its own windows into.  `pin()` registers the mapping with CUDA so
    device-to-host copies land in it by DMA.
    """

    def __init__(self, tag: str, shape: tuple[int, int, int], rank: int, barrier: Callable[[], None]):
        self.shape = tuple(int(s) for s in shape)
        self.nbytes = int(np.prod(self.shape)) * 4
        self.rank = rank
        self.name = f"levo_b200_{tag}"
        self._pinned = False
        self._pinned_base = 0
        self.shm = None
        self.path = None
        # POSIX shared memory when /dev/shm has room, else a file mapping in the temp dir.
        # Rank 0 decides (and clears stale segments or files of the same name); the others
        # attach to whichever it created, so all ranks agree even when /dev/shm is nearly full.
        file_path = os.path.join(tempfile.gettempdir(), self.name + ".f32")
        if rank == 0:
            try:
                stale = shared_memory.SharedMemory(name=self.name)
                stale.close()
                stale.unlink()
            except FileNotFoundError:
                pass
            if os.path.exists(file_path):
                os.unlink(file_path)
            if _free_bytes("/dev/shm") > self.nbytes * 1.1:
                self.shm = shared_memory.SharedMemory(name=self.name, create=True, size=self.nbytes)
            else:
                self.path = file_path
                self.array = np.memmap(self.path, dtype=np.float32, mode="w+", shape=self.shape)
        barrier()
        if rank != 0:
            try:
                self.shm = shared_memory.SharedMemory(name=self.name)
                _untrack(self.shm)
            except FileNotFoundError:
                self.path = file_path
                self.array = np.memmap(self.path, dtype=np.float32, mode="r+", shape=self.shape)
        if self.shm is not None:
            self.array = np.ndarray(self.shape, dtype=np.float32, buffer=self.shm.buf)

    def view(self, start: int, stop: int) -> np.ndarray:
        return self.array[start:stop]

    def pin(self, start: int = 0, stop: Optional[int] = None) -> bool:
        """Page-locks the pages of windows [start, stop) (default: all) for CUDA DMA; returns False
        when registration is refused.  This rank writes those pages first, so that under the kernel's
        first-touch policy they are allocated on the memory node of the CPUs this rank runs on (see
        bind_to_gpu_local_cpus) rather than all on the node of whichever rank touched them first:
        with one GPU per rank, every GPU then copies its audio into memory local to it."""
        import torch

        if self._pinned:
            return True
        stop = self.shape[0] if stop is None else stop
        if stop <= start:
            return True
        per_window = self.nbytes // self.shape[0]
        page = os.sysconf("SC_PAGE_SIZE")
        base = self.array.ctypes.data
        lo = (base + start * per_window) // page * page
        hi = -(-(base + stop * per_window) // page) * page
        lo, hi = max(lo, base // page * page), min(hi, -(-(base + self.nbytes) // page) * page)
        self.array[start:stop] = 0.0  # first touch by this rank
        rc = torch.cuda.cudart().cudaHostRegister(lo, hi - lo, 0)
        self._pinned = int(rc) == 0
        self._pinned_base = lo
        return self._pinned

    def close(self, barrier: Optional[Callable[[], None]] = None) -> None:
        if self._pinned:
            import torch

            torch.cuda.cudart().cudaHostUnregister(self._pinned_base)
            self._pinned = False
        self.array = None
        if barrier is not None:
            barrier()
        if self.shm is not None:
            self.shm.close()
            if self.rank == 0:
                try:
                    self.shm.unlink()
                except FileNotFoundError:
                    pass
        elif self.rank == 0 and self.path and os.path.exists(self.path):
            os.unlink(self.path)


def _untrack(shm: shared_memory.SharedMemory) -> None:
    """Rank 0 owns (and unlinks) the segment; an attaching rank must not have
    Python's resource tracker unlink it again at exit."""
    try:
        from multiprocessing import resource_tracker

        resource_tracker.unregister(shm._name, "shared_memory")  # noqa: SLF001
    except Exception:
        pass


def _free_bytes(path: str) -> int:
    try:
        st = os.statvfs(path)
        return st.f_bavail * st.f_frsize
    except OSError:
        return 0


def bind_to_gpu_local_cpus(device: int) -> Optional[list[int]]:
    """Restricts this process to the CPUs NVML reports as local to GPU `device` (its NUMA node), so
    its pinned host buffers are allocated next to that GPU's PCIe root.  Returns the CPUs, or None
    when NVML is unavailable or reports no affinity (the process is left as it was).  Only this
    process's CPU affinity changes; nothing of the GPU."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByIndex(device)
            n_words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, n_words)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # noqa: BLE001 - NVML missing or refusing: keep the current affinity
        return None
    cpus = [w * 64 + b for w, word in enumerate(mask) for b in range(64) if (int(word) >> b) & 1]
    allowed = os.sched_getaffinity(0)
    cpus = [c for c in cpus if c in allowed]
    if not cpus:
        return None
    os.sched_setaffinity(0, cpus)
    return cpus


def run_tag() -> str:
    """A name shared by the ranks of one torchrun job (MASTER_PORT is common to them)."""
    return f"{os.environ.get('MASTER_PORT', '0')}_{os.getppid() if os.environ.get('LOCAL_RANK') else os.getpid()}"
