"""CPU: the module registry behind the opaque op (keyed by a stable integer, reference
op ``infra::magi2_mh_moe``) hands out unique keys and does not keep modules alive."""
import gc

import torch


def _cfg():
    from flash_mh_moe.moe import CoreMultiHeadMoEConfig
    return CoreMultiHeadMoEConfig(hidden_size=256, num_heads=1, num_experts=4, top_k=2,
                                  expert_intermediate_size=256, num_layers=1, params_dtype=torch.bfloat16)


def test_keys_unique_and_weak():
    from flash_mh_moe import moe
    a = moe.CoreMultiHeadMoE(_cfg())
    b = moe.CoreMultiHeadMoE(_cfg())
    assert a._moe_key != b._moe_key
    assert moe._magi2_moe_registry[a._moe_key] is a
    ka = a._moe_key
    del a
    gc.collect()
    assert ka not in moe._magi2_moe_registry          # the registry did not keep it alive
    c = moe.CoreMultiHeadMoE(_cfg())
    assert c._moe_key not in (ka, b._moe_key)         # keys are never reused


def _released(m):
    """Release the masters without packing (packing needs the GPU): the packed operands are
    a stand-in, which is all release/load bookkeeping looks at."""
    m.packed_weights = lambda: ("packed-gu", "packed-dn")
    m.release_master_weights()
    assert m._masters_released and all(getattr(m, n).numel() == 0 for n in ("W_gate", "W_up", "W_down"))


def test_release_then_load_restores_masters():
    from flash_mh_moe import moe
    src = moe.CoreMultiHeadMoE(_cfg())
    with torch.no_grad():
        for p in src.parameters():
            p.copy_(torch.randn(p.shape).to(p.dtype))
    sd = src.state_dict()
    m = moe.CoreMultiHeadMoE(_cfg())
    _released(m)
    m.load_state_dict(sd)
    assert not m._masters_released
    for n in ("W_gate", "W_up", "W_down", "gate"):
        assert torch.equal(getattr(m, n), sd[n]), n


def test_release_then_failed_load_stays_released():
    from flash_mh_moe import moe
    m = moe.CoreMultiHeadMoE(_cfg())
    _released(m)
    bad = {k: v.clone() for k, v in moe.CoreMultiHeadMoE(_cfg()).state_dict().items()}
    bad["W_down"] = bad["W_down"][:, :, :128].clone()          # wrong shape
    try:
        m.load_state_dict(bad)
        raise AssertionError("a size mismatch must raise")
    except RuntimeError as e:
        assert "W_down" in str(e)
    # the failed load leaves the module serving its packed weights
    assert m._masters_released
    assert all(getattr(m, n).numel() == 0 for n in ("W_gate", "W_up", "W_down"))


def test_release_then_partial_load_keeps_packed():
    from flash_mh_moe import moe
    m = moe.CoreMultiHeadMoE(_cfg())
    _released(m)
    sd = {k: v for k, v in moe.CoreMultiHeadMoE(_cfg()).state_dict().items() if k != "W_up"}
    try:
        # W_up missing: the masters are not restored, so the other two do not fit
        m.load_state_dict(sd, strict=False)
        raise AssertionError("loading two of three released masters must raise")
    except RuntimeError as e:
        assert "W_gate" in str(e)
    assert m._masters_released


class _FakePsm:
    """Stands in for MAGI-2's inference.infra.distributed.psm (psm.py:94-128)."""

    def __init__(self, size, rank, group):
        self.size, self.rank, self.group = size, rank, group

    def get_world_size(self, dim=""):
        return self.size

    def get_local_rank(self, dim):
        return self.rank

    def get_parallel_group(self, dim):
        return self.group


def _with_psm(monkeypatch, psm):
    import sys
    import types
    for name in ("inference", "inference.infra"):
        monkeypatch.setitem(sys.modules, name, types.ModuleType(name))
    mod = types.ModuleType("inference.infra.distributed")
    mod.psm = psm
    monkeypatch.setitem(sys.modules, "inference.infra.distributed", mod)


def test_ep_group_read_from_psm(monkeypatch):
    """Built as the reference model builds it, CoreMultiHeadMoE(config) with no group
    argument, the module takes its expert-parallel size, rank and group from psm and holds
    this rank's contiguous slice of the flattened experts (the dim-0 rows the reference's
    EP checkpoint reader gives this rank, magi2_checkpointing.py:81-105)."""
    from flash_mh_moe import moe
    group = object()
    _with_psm(monkeypatch, _FakePsm(2, 1, group))
    m = moe.CoreMultiHeadMoE(_cfg())
    assert (m.ep_size, m.ep_rank, m.ep_group) == (2, 1, group)
    assert m.local_flatten_num_experts == 2 and m.expert_lo == 2
    assert m.W_gate.shape[0] == 2 and m.gate.shape[0] == 4      # experts sharded, router replicated


def test_ep_size_without_group_raises_at_forward(monkeypatch):
    """psm reports ep_size > 1 but no EP group: the reference raises this RuntimeError at
    forward (magi2_preview.py:2632-2637); so does the drop-in, before any device work."""
    from flash_mh_moe import moe
    _with_psm(monkeypatch, _FakePsm(2, 0, None))
    m = moe.CoreMultiHeadMoE(_cfg())
    try:
        m._forward_impl(torch.zeros(8, 256, dtype=torch.bfloat16))
        raise AssertionError("expected RuntimeError")
    except RuntimeError as e:
        assert "EP group is not initialized but ep_size=2" in str(e)


def test_single_rank_without_psm():
    from flash_mh_moe import moe
    m = moe.CoreMultiHeadMoE(_cfg())
    assert (m.ep_size, m.ep_rank, m.ep_group) == (1, 0, None)
