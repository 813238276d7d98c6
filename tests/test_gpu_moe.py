"""GPU parity: the module drop-in (CoreMultiHeadMoE.forward through the custom op) against
the oracle composed from the reference restatements: route.py on the GPU's own fp32
logits, the stable global sort, and the NVFP4 FFN restatement.  Bar: rel L2 <= 1e-2."""
import numpy as np
import pytest
import torch

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

CASES = [
    # S, H, dh, de, E, K, score, route_scale, bias
    (512, 1, 1024, 2048, 8, 2, "softmax", 1.0, False),
    (256, 2, 256, 256, 16, 3, "sigmoid", 4.9, True),       # production-style scoring
    (200, 1, 512, 512, 64, 8, "softmax", 1.0, True),
    (128, 1, 3072, 1024, 16, 8, "softmax", 1.0, False),   # config-1 layer shape, fewer experts
]


@pytest.mark.parametrize("scatter", ["combine", "atomic"])
@pytest.mark.parametrize("S,H,dh,de,E,K,score,scale,use_bias", CASES)
def test_module_forward_matches_oracle(S, H, dh, de, E, K, score, scale, use_bias, scatter, monkeypatch):
    monkeypatch.setenv("MHMOE_SCATTER", scatter)
    from flash_mh_moe import _lib
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    from flash_mh_moe.route import route_fused
    dev = torch.device("cuda", 0)
    cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                 expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                 score_func=score, route_norm=True, route_scale=scale)
    m = CoreMultiHeadMoE(cfg).to(dev)
    init_moe_params_(m, seed=S + E, device=dev)
    if use_bias:
        with torch.no_grad():
            m.router.expert_bias.copy_(torch.randn(H * E, generator=torch.Generator().manual_seed(3)) * 0.01)
    x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(S)).to(torch.bfloat16).to(dev)
    y = m(x)
    y2 = torch.ops.magi2_b200.mh_moe(x, m._moe_key)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    if scatter == "combine":
        assert torch.equal(y, y2)
    else:   # bf16 atomics: the summation order may change the last bits
        assert rel_l2(y.float().cpu().numpy(), y2.float().cpu().numpy()) < 1e-2
    # oracle on the same logits the fused router computes
    planes, nsplit = m.router_planes()
    bias = m.router.expert_bias.view(H, E) if use_bias else None
    _, _, logits = route_fused(x.view(S, H, dh), planes, nsplit, E, K, score, bias, True, 1e-12, scale,
                               return_logits=True)
    lg = logits.cpu().numpy()
    p, i = route_ref.compute_topk_probs_and_indices(lg, K, score, None if bias is None else bias.cpu().numpy())
    p = (p * np.float32(scale)).astype(np.float32)
    g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    Wg, Wu, Wd = (w.detach().float().cpu().numpy() for w in (m.W_gate, m.W_up, m.W_down))
    xh = x.float().cpu().numpy().reshape(S, H, dh)
    ref = ffn_ref.mh_moe_fwd_nvfp4_ref(xh, g, ps, o, nv.pack_gate_up(Wg, Wu), nv.pack_down(Wd))
    got = y.float().cpu().numpy().reshape(S, H, dh)
    err = rel_l2(got, ref)
    assert np.isfinite(got).all() and err < 1e-2, err


def test_module_fake_meta():
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig
    cfg = CoreMultiHeadMoEConfig(hidden_size=256, num_heads=1, num_experts=8, top_k=2, expert_intermediate_size=256,
                                 num_layers=1, params_dtype=torch.bfloat16, score_func="softmax")
    m = CoreMultiHeadMoE(cfg)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        xf = torch.empty(64, 256, dtype=torch.bfloat16, device="cuda")
        yf = torch.ops.magi2_b200.mh_moe(xf, m._moe_key)
        assert yf.shape == xf.shape and yf.dtype == xf.dtype


def test_production_head_split_matches_oracle():
    """MAGI-2's production routing shape (configs/magi2_preview.json: 12 heads of 256,
    top-6 sigmoid with expert bias, route_scale 4.9, expert FFN dim 1280) with 16 experts
    per head instead of 256 so the CPU oracle stays fast.  The oracle runs on the weights
    the GPU packed (the GPU packer is checked byte-exact against the oracle packer in
    test_gpu_nvfp4)."""
    from flash_mh_moe import _lib
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    from flash_mh_moe.route import route_fused
    dev = torch.device("cuda", 0)
    S, H, dh, de, E, K, scale = 128, 12, 256, 1280, 16, 6, 4.9
    cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                 expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                 score_func="sigmoid", route_norm=True, route_scale=scale)
    m = CoreMultiHeadMoE(cfg).to(dev)
    init_moe_params_(m, seed=77, device=dev)
    with torch.no_grad():
        m.router.expert_bias.copy_(torch.randn(H * E, generator=torch.Generator().manual_seed(4)) * 0.01)
    x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(dev)
    y = m(x)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    planes, nsplit = m.router_planes()
    bias = m.router.expert_bias.view(H, E)
    _, _, logits = route_fused(x.view(S, H, dh), planes, nsplit, E, K, "sigmoid", bias, True, 1e-12, scale,
                               return_logits=True)
    p, i = route_ref.compute_topk_probs_and_indices(logits.cpu().numpy(), K, "sigmoid", bias.cpu().numpy())
    p = (p * np.float32(scale)).astype(np.float32)
    g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    gu, dn = m.packed_weights()
    gu_pack = {"data": gu.data.cpu().numpy(), "sf_atoms": gu.sf.cpu().numpy(),
               "gscale_gate": gu.gscale[0].cpu().numpy(), "gscale_up": gu.gscale[1].cpu().numpy(),
               "N": 2 * de, "K": dh, "de": de}
    dn_pack = {"data": dn.data.cpu().numpy(), "sf_atoms": dn.sf.cpu().numpy(), "gscale": dn.gscale.cpu().numpy(),
               "N": dh, "K": de}
    ref = ffn_ref.mh_moe_fwd_nvfp4_ref(x.float().cpu().numpy().reshape(S, H, dh), g, ps, o, gu_pack, dn_pack)
    got = y.float().cpu().numpy().reshape(S, H, dh)
    err = rel_l2(got, ref)
    assert np.isfinite(got).all() and err < 1e-2, err
