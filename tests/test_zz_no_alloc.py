"""GPU: mhmoe_global_sort_noalloc — the stable expert sort for callers that cannot
allocate device memory (an FFI host with no device allocator, or a hot path that must
not call cudaMalloc/cudaFree because they can synchronise the device).

It is called through the C ABI directly and must reproduce mhmoe_global_sort's outputs
bit for bit (integer/permutation outputs: exact equality is this suite's bar), on two
calls in a row with different sizes, so that the shared built-in scratch array carrying
the previous call's contents cannot leak into the next result.  This file is collected
last so that a stop-at-first-failure run has already run every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(H, S, K, E, seed):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((H, S, E)).astype(np.float32)
    logits[..., 1] += 2.5                      # one crowded expert
    idx = np.argsort(-logits, -1, kind="stable")[..., :K].astype(np.int64)
    probs = rng.random((H, S, K)).astype(np.float32)
    return torch.from_numpy(probs).cuda(), torch.from_numpy(idx).cuda()


def _noalloc(L, probs, idx, E):
    from flash_mh_moe import _lib
    H, S, K = idx.shape
    R = H * S * K
    dev = idx.device
    g = torch.full((R,), -7, dtype=torch.int32, device=dev)
    p = torch.full((R,), float("nan"), dtype=torch.float32, device=dev)
    o = torch.full((H * E + 1,), -7, dtype=torch.int64, device=dev)
    inv = torch.full((R,), -7, dtype=torch.int32, device=dev)
    st = _lib.device_status(dev)
    rc = L.mhmoe_global_sort_noalloc(probs.data_ptr(), idx.data_ptr(), H, S, K, E, g.data_ptr(), p.data_ptr(),
                                     o.data_ptr(), inv.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "mhmoe_global_sort_noalloc")
    return g, p, o, inv


def test_noalloc_sort_matches_allocating_sort_twice():
    from flash_mh_moe import _lib
    from flash_mh_moe.route import flash_mh_moe_global_sort_with_inverse
    L = _lib.lib()
    # calls in a row: config-1-sized routing (chunked sort), a smaller multi-head problem,
    # then one small enough for the single-CTA sort (H*S*K <= 8192 rows, H*E <= 256)
    for (H, S, K, E), seed in (((1, 16384, 8, 128), 11), ((3, 1000, 5, 40), 12), ((2, 500, 4, 64), 13)):
        probs, idx = _inputs(H, S, K, E, seed)
        got = _noalloc(L, probs, idx, E)
        want = flash_mh_moe_global_sort_with_inverse(probs, idx, E)
        torch.cuda.synchronize()
        _lib.check_device_status(idx.device)
        for a, b in zip(got, want):
            assert torch.equal(a, b)


def test_noalloc_sort_empty_batch_zeroes_offsets():
    from flash_mh_moe import _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    H, K, E = 2, 4, 64
    dummy = torch.zeros(8, dtype=torch.int64, device=dev)         # R == 0: nothing to write but offsets
    o = torch.full((H * E + 1,), -7, dtype=torch.int64, device=dev)
    rc = L.mhmoe_global_sort_noalloc(dummy.data_ptr(), dummy.data_ptr(), H, 0, K, E, dummy.data_ptr(),
                                     dummy.data_ptr(), o.data_ptr(), None, None, _lib.stream_ptr(dev))
    _lib.check(rc, "mhmoe_global_sort_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(o, torch.zeros_like(o))


def test_noalloc_sort_rejects_oversize():
    from flash_mh_moe import _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    dummy = torch.zeros(8, dtype=torch.int64, device=dev)
    # 1 x 65536 tokens x top-8 = 524288 routed rows > 262144: refused before any launch
    rc = L.mhmoe_global_sort_noalloc(dummy.data_ptr(), dummy.data_ptr(), 1, 65536, 8, 128, dummy.data_ptr(),
                                     dummy.data_ptr(), dummy.data_ptr(), None, None, _lib.stream_ptr(dev))
    assert rc == 7   # MHMOE_ERR_CAPACITY
    assert b"exceed" in L.mhmoe_last_error()
    rc = L.mhmoe_global_sort_noalloc(dummy.data_ptr(), dummy.data_ptr(), 2, 16, 2, 1024, dummy.data_ptr(),
                                     dummy.data_ptr(), dummy.data_ptr(), None, None, _lib.stream_ptr(dev))
    assert rc == 7   # 2048 experts > 1024
