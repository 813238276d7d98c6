"""GPU parity: MAGI-2's whole MoE layer (MultiHeadMoELayer, magi2_preview.py:2685-2806) —
multi-modality pre-RMSNorm, split / merge linears, the routed core and the shared plus
modality-specific shared experts — against the oracle (oracle.layer_ref).

* RMSNorm kernel vs the restatement of MultiModalityRMSNorm: within one bf16 ulp.
* Whole layer vs its NVFP4 twin: the routed core's oracle runs on the GPU's own router
  logits (as in test_gpu_moe), the shared experts' oracle on the weights the GPU packed.
  Bar: relative L2 <= 1e-2.  The distance to the bf16 reference layer (shared experts in
  bf16) is printed for information: it is the NVFP4 quantisation of both expert sets.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ffn_ref, layer_ref, nvfp4_ref as nv, route_ref

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

CASES = [
    # S groups, hidden, heads, E, K, de, shared, modality-specific
    ((150, 50, 120), 512, 2, 8, 2, 256, 256, 256),
    ((64, 0, 200), 768, 3, 8, 3, 512, 256, 512),      # an empty modality, unequal shared sizes
]


def _layer(groups, d, H, E, K, de, Is, Im, seed):
    from flash_mh_moe.layer import MLPActivationType, MoEConfig, MultiHeadMoELayer, MultiHeadMoELayerConfig
    from flash_mh_moe.moe import init_moe_params_
    dev = torch.device("cuda", 0)
    mc = MoEConfig(num_experts=E, top_k=K, score_func="sigmoid", route_norm=True, route_scale=4.9,
                   expert_intermediate_size=de, shared_expert_intermediate_size=Is,
                   modality_specific_expert_intermediate_size=Im, num_heads=H)
    cfg = MultiHeadMoELayerConfig(hidden_size=d, num_modality=len(groups), num_layers=1,
                                  activation_type=MLPActivationType.SWIGLU7, params_dtype=torch.bfloat16,
                                  shared_expert_intermediate_sizes=Is,
                                  modality_specific_expert_intermediate_sizes=Im,
                                  shared_expert_params_dtype=torch.bfloat16, split_merge_intermediate_size=None,
                                  moe_config=mc)
    layer = MultiHeadMoELayer(cfg).to(dev)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if name.startswith("moe_mlp."):
                continue
            std = 0.1 if name == "pre_norm.weight" else 0.02
            p.copy_((torch.randn(p.shape, generator=g) * std).to(p.dtype))
    init_moe_params_(layer.moe_mlp, seed=seed, device=dev)
    x = torch.randn(sum(groups), d, generator=g).to(torch.bfloat16).to(dev)
    return layer, x


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("groups,d,H,E,K,de,Is,Im", CASES)
def test_moe_layer_matches_oracle(groups, d, H, E, K, de, Is, Im):
    from flash_mh_moe import _lib
    from flash_mh_moe.route import route_fused
    layer, x = _layer(groups, d, H, E, K, de, Is, Im, seed=sum(groups))
    y = layer(x, list(groups))
    norm = layer.pre_norm(x, list(groups))
    moe_in = F.linear(norm, layer.split_linear.weight)
    torch.cuda.synchronize()
    _lib.check_device_status(x.device)
    S, dh = x.shape[0], d // H

    # the fused RMSNorm against its restatement
    norm_ref = layer_ref.rmsnorm_ref(_np(x), _np(layer.pre_norm.weight), list(groups))
    assert rel_l2(_np(norm), norm_ref) < 2e-3

    # the routed core's oracle on the GPU's own logits for the GPU's moe input
    core = layer.moe_mlp
    planes, nsplit = core.router_planes()
    bias = core.router.expert_bias.view(H, E)
    _, _, logits = route_fused(moe_in.view(S, H, dh), planes, nsplit, E, K, "sigmoid", bias, True, 1e-12, 4.9,
                               return_logits=True)
    p, i = route_ref.compute_topk_probs_and_indices(_np(logits), K, "sigmoid", _np(bias))
    p = (p * np.float32(4.9)).astype(np.float32)
    gg, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    Wg, Wu, Wd = (_np(w) for w in (core.W_gate, core.W_up, core.W_down))
    core_out = ffn_ref.mh_moe_fwd_nvfp4_ref(_np(moe_in).reshape(S, H, dh), gg, ps, o, nv.pack_gate_up(Wg, Wu),
                                            nv.pack_down(Wd)).reshape(S, d)

    gu, dn = layer.shared_packed()
    gu_pack = {"data": gu.data.cpu().numpy(), "sf_atoms": gu.sf.cpu().numpy(),
               "gscale_gate": gu.gscale[0].cpu().numpy(), "gscale_up": gu.gscale[1].cpu().numpy(),
               "N": 2 * gu.d_expert, "K": gu.d_head, "de": gu.d_expert}
    dn_pack = {"data": dn.data.cpu().numpy(), "sf_atoms": dn.sf.cpu().numpy(), "gscale": dn.gscale.cpu().numpy(),
               "N": dn.d_head, "K": dn.d_expert}
    want, _ = layer_ref.layer_nvfp4_ref(_np(x), list(groups), _np(layer.pre_norm.weight),
                                        _np(layer.split_linear.weight), _np(layer.merge_linear.weight),
                                        lambda _m: core_out, gu_pack, dn_pack)
    got = _np(y)
    err = rel_l2(got, want)

    # information: the shared experts on NVFP4 against the bf16 reference's shared experts
    shared_bf16 = layer_ref.shared_experts_ref(norm_ref, list(groups), _np(layer.shared_expert_fc1.weight),
                                               _np(layer.shared_expert_fc2.weight),
                                               _np(layer.modality_specific_shared_expert_fc1.weight),
                                               _np(layer.modality_specific_shared_expert_fc2.weight))
    shared_gpu = _np(layer._shared_expert_forward(norm, list(groups)))
    print(f"layer {groups}: rel L2 vs NVFP4 oracle {err:.2e}; NVFP4 shared experts vs bf16 reference "
          f"{rel_l2(shared_gpu, shared_bf16):.3f}")
    assert np.isfinite(got).all() and err < 1e-2, err


def test_rmsnorm_single_modality_and_strides():
    """One modality (no group table), a strided input view."""
    from flash_mh_moe.layer import MultiModalityRMSNorm
    dev = torch.device("cuda", 0)
    norm = MultiModalityRMSNorm(3072).to(dev)
    with torch.no_grad():
        norm.weight.copy_(torch.randn(3072, generator=torch.Generator().manual_seed(1)) * 0.1)
    big = torch.randn(100, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(dev)
    x = big[:, 512:512 + 3072]
    y = norm(x)
    ref = layer_ref.rmsnorm_ref(_np(x), _np(norm.weight), [100])
    assert rel_l2(_np(y), ref) < 2e-3
