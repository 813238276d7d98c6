"""Packed-weight cache of flash_mh_moe_fwd: an entry is reused while its source tensors
live and evicted when one of them is freed, so a new tensor that the allocator places at
a freed tensor's address (same version 0, same shape) is packed afresh."""
import gc

import torch

from flash_mh_moe import fwd


def test_reuse_while_alive_and_evict_on_free():
    packs = []

    def pack(*srcs):
        packs.append(srcs)
        return object()

    a, b = torch.zeros(4, 8), torch.ones(4, 8)
    n0 = len(fwd._pack_cache)
    first = fwd._cached_pack("test", (a, b), pack)
    assert fwd._cached_pack("test", (a, b), pack) is first and len(packs) == 1
    for _ in range(3):
        b.add_(1)                               # in-place update: new version, repacked ...
        assert fwd._cached_pack("test", (a, b), pack) is not first and len(packs) >= 2
    assert len(fwd._pack_cache) == n0 + 1       # ... into the same entry
    del b, packs[:]
    gc.collect()
    assert len(fwd._pack_cache) == n0           # the entry named the freed tensor


def test_module_key_is_identity_based():
    from flash_mh_moe.moe import _same_key
    p = torch.nn.Parameter(torch.zeros(2))
    q = torch.nn.Parameter(torch.zeros(2))
    k = ((p, 1, 0),)
    assert _same_key(k, ((p, 1, 0),))
    assert not _same_key(k, ((q, 1, 0),))       # another object at the same address/version
    assert not _same_key(None, k)
