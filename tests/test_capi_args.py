"""CPU: the C ABI rejects bad arguments with MHMOE_ERR_ARGS and names the failed check in
mhmoe_last_error(), before it touches a device.  The pointers passed here are never
dereferenced — argument checks run first, and a call whose arguments pass stops at the
device check (no GPU here) — so placeholder addresses are safe."""
import ctypes

import pytest
import torch

ERR_ARGS, ERR_ARCH = 1, 2
P = 0x10000          # a 16-B aligned placeholder address


@pytest.fixture(scope="module")
def L():
    if torch.cuda.is_available():
        pytest.skip("device present: the valid-argument calls would run")
    from flash_mh_moe import _lib
    return _lib.lib()


def _sort(L, probs=P, idx=P, H=1, S=16, K=2, E=8, ws=P):
    return L.mhmoe_global_sort(probs, idx, H, S, K, E, ws, P, P, P, None, None, None)


def test_global_sort_checks(L):
    assert _sort(L, probs=None) == ERR_ARGS
    assert b"topk_probs" in L.mhmoe_last_error()
    assert _sort(L, K=0) == ERR_ARGS
    assert b"K > 0" in L.mhmoe_last_error()
    assert _sort(L, H=2, E=8192) == ERR_ARGS              # H*E above the compiled-in bound
    assert b"12288" in L.mhmoe_last_error()
    assert _sort(L) == ERR_ARCH                           # valid arguments: stops at the device check


def _quantized(L, xq=P, xq_pitch=1536, xsf_pitch=192, dh=3072, de=1024):
    return L.mhmoe_ffn_nvfp4_quantized(xq, xq_pitch, P, xsf_pitch, P, 4, 64, dh, de, 8, 128, P, P, P, P, P, P,
                                       P, P, P, None, None, 8, P, P, dh, None, 0, None, None)


def test_ffn_quantized_checks(L):
    assert _quantized(L, xq=None) == ERR_ARGS
    assert _quantized(L, xq=P + 8) == ERR_ARGS            # records must be 16-B aligned (TMA / 16-B loads)
    assert b"aligned16" in L.mhmoe_last_error()
    assert _quantized(L, xq_pitch=1544) == ERR_ARGS       # pitch not a multiple of 16
    assert _quantized(L, dh=3000) == ERR_ARGS             # d_head must be a multiple of 256
    assert _quantized(L) == ERR_ARCH
