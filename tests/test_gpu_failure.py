"""GPU: failure detection without a fault.  The library's device waits are bounded; the
self-test entry runs them against a shared-memory barrier nothing arrives on and a
global flag nothing sets.  Each must give up after its limit, leave MHMOE_ERR_TIMEOUT in
the device status word (read on the host), and leave the context usable: a normal
library call afterwards succeeds and matches the oracle."""

import numpy as np
import pytest
import torch

from flash_mh_moe import _lib
from flash_mh_moe.route import flash_mh_moe_global_sort

from oracle import route_ref

pytestmark = pytest.mark.gpu

LIMIT_NS = 2_000_000   # 2 ms per wait


def _selftest(flag, expected, mode, status, elapsed):
    rc = _lib.lib().mhmoe_wait_selftest(flag.data_ptr() if flag is not None else None, expected, mode, LIMIT_NS,
                                        status.data_ptr(), elapsed.data_ptr(), _lib.stream_ptr(status.device))
    _lib.check(rc, "wait_selftest")
    torch.cuda.synchronize()


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_bounded_waits_time_out_and_context_survives(mode):
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    elapsed = torch.zeros(1, dtype=torch.int64, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)           # nothing ever sets it
    _selftest(flag, 1, mode, status, elapsed)
    assert int(status.item()) == _lib.MHMOE_ERR_TIMEOUT
    ns = int(elapsed.item())
    assert LIMIT_NS <= ns < 1_000_000_000, ns
    # the context is still usable: a real call runs and matches the oracle
    g = torch.Generator().manual_seed(3)
    H, S, K, E = 1, 1000, 4, 16
    probs = torch.rand(H, S, K, generator=g)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(H * S)]).view(H, S, K)
    gids, ps, offs = flash_mh_moe_global_sort(probs.to(dev), idx.to(dev), E)
    rg, rp, ro = route_ref.flash_mh_moe_global_sort(probs.numpy(), idx.numpy(), E)
    np.testing.assert_array_equal(gids.cpu().numpy(), rg)
    np.testing.assert_array_equal(offs.cpu().numpy(), ro)
    _lib.check_device_status(dev)


def test_flag_wait_returns_when_set():
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    elapsed = torch.zeros(1, dtype=torch.int64, device=dev)
    flag = torch.full((1,), 5, dtype=torch.int32, device=dev)
    _selftest(flag, 5, 2, status, elapsed)
    assert int(status.item()) == 0
    assert int(elapsed.item()) < LIMIT_NS


def test_selftest_argument_checks():
    dev = torch.device("cuda", 0)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    assert L.mhmoe_wait_selftest(None, 1, 2, LIMIT_NS, status.data_ptr(), None, None) == _lib.MHMOE_ERR_ARGS
    assert L.mhmoe_wait_selftest(None, 1, 1, 10, status.data_ptr(), None, None) == _lib.MHMOE_ERR_ARGS
