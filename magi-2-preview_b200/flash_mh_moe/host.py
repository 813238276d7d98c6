"""Host buffers for feeding the layer from CPU memory.

A serving loop copies each batch from pinned host memory to the GPU and the output back.
On a multi-socket host those copies run at full PCIe speed only when the pinned pages sit
on the NUMA node the GPU is attached to.  ``near_gpu`` runs a block on the CPUs NVML lists
as local to the GPU (the pages a pinned allocation touches there are placed on that node);
``pinned_like`` allocates pinned host buffers that way.
"""
from __future__ import annotations

import contextlib
import os

import torch


def gpu_local_cpus(device) -> set[int] | None:
    """CPUs NVML reports as local to ``device`` (intersected with this process's allowed
    CPUs), or None when NVML or the query is unavailable."""
    try:
        import pynvml
        pynvml.nvmlInit()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
        n = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, (n + 63) // 64)
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


@contextlib.contextmanager
def near_gpu(device):
    """Run the block on the CPUs local to ``device`` (unchanged when they are unknown)."""
    cpus = gpu_local_cpus(device)
    before = os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield cpus
    finally:
        if cpus:
            os.sched_setaffinity(0, before)


def pinned_like(t: torch.Tensor, device, copy: bool = False) -> torch.Tensor:
    """A pinned host tensor shaped like ``t`` (its values when ``copy``), allocated from the
    CPUs local to ``device``."""
    with near_gpu(device):
        return t.pin_memory() if copy else torch.empty_like(t, device="cpu").pin_memory()
