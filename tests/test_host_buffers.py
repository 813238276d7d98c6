"""Host-buffer helpers (flash_mh_moe.host): CPU-side behaviour, no GPU needed."""
import os

import torch

from flash_mh_moe.host import gpu_local_cpus, near_gpu


def test_local_cpus_subset_or_none():
    cpus = gpu_local_cpus(torch.device("cuda", 0))
    assert cpus is None or (cpus and cpus <= os.sched_getaffinity(0))


def test_near_gpu_restores_affinity():
    before = os.sched_getaffinity(0)
    with near_gpu(torch.device("cuda", 0)) as cpus:
        inside = os.sched_getaffinity(0)
        assert inside == (cpus if cpus else before)
    assert os.sched_getaffinity(0) == before
