"""GPU: NVFP4 quantise-on-load from a safetensors checkpoint.

Loading a MoE layer in chunks of experts straight into its packed operands gives the
same bytes as packing the whole bf16 weights at once (per-expert scales make the chunking
exact), leaves the bf16 masters released, and the module's forward equals the same module
loaded through load_state_dict (bit for bit: same packed operands, same kernels)."""
import pytest
import torch

from test_checkpoint import _write_checkpoint

pytestmark = pytest.mark.gpu


def test_quantise_on_load_matches_state_dict_load(tmp_path):
    from flash_mh_moe import _lib, checkpoint
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig
    from flash_mh_moe.nvfp4 import pack_down, pack_gate_up
    dev = torch.device("cuda", 0)
    prefix = "blocks.2.mlp.moe_mlp."
    full = _write_checkpoint(tmp_path, prefix)
    cfg = CoreMultiHeadMoEConfig(hidden_size=512, num_heads=2, num_experts=4, top_k=2, expert_intermediate_size=256,
                                 num_layers=1, params_dtype=torch.bfloat16, score_func="sigmoid", route_scale=4.9)
    a = CoreMultiHeadMoE(cfg).to(dev)
    checkpoint.load_moe_module(a, str(tmp_path), prefix, quantize=True, release_masters=True, chunk_experts=3)
    assert a._masters_released and a.W_gate.numel() == 0
    gu, dn = a.packed_weights()
    w = {k: v.to(dev) for k, v in full.items()}
    gu_ref, dn_ref = pack_gate_up(w["W_gate"], w["W_up"]), pack_down(w["W_down"])
    for x, y in ((gu.data, gu_ref.data), (gu.sf, gu_ref.sf), (gu.gscale, gu_ref.gscale), (dn.data, dn_ref.data),
                 (dn.sf, dn_ref.sf), (dn.gscale, dn_ref.gscale)):
        assert torch.equal(x, y)

    b = CoreMultiHeadMoE(cfg).to(dev)
    sd = dict(w)
    sd["router.expert_bias"] = w["router.expert_bias_ema"]      # the loader's EMA substitution
    b.load_state_dict(sd)
    x = torch.randn(300, 512, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(dev)
    ya, yb = a(x), b(x)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    assert torch.equal(ya, yb)
