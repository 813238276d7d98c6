"""GPU parity for head and expert sizes the reference accepts (d_head % 64 == 0,
d_expert % 32 == 0: triton/mh_moe_fwd.py:264-265) but the 256-wide tensor-core tiles do
not.  They are packed zero-padded to multiples of 256; the oracle pads the same way
(exact, see flash_mh_moe/nvfp4.py) and crops.  Bar: relative L2 <= 1e-2."""
import numpy as np
import pytest
import torch

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

CASES = [
    # S, H, dh, de, E, K
    (96, 2, 128, 96, 4, 2),
    (64, 1, 192, 160, 8, 3),
    (80, 3, 64, 32, 4, 2),
    (40, 1, 320, 288, 4, 2),
]


def _pad(a, axis, n):
    w = [(0, 0)] * a.ndim
    w[axis] = (0, n - a.shape[axis])
    return np.pad(a, w)


@pytest.mark.parametrize("S,H,dh,de,E,K", CASES)
def test_padded_shapes_match_oracle(S, H, dh, de, E, K):
    from flash_mh_moe import _lib
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    from flash_mh_moe.nvfp4 import padded
    from flash_mh_moe.route import route_fused
    dev = torch.device("cuda", 0)
    cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                 expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                 score_func="softmax", route_norm=True, route_scale=1.0)
    m = CoreMultiHeadMoE(cfg).to(dev)
    init_moe_params_(m, seed=S + dh, device=dev)
    x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(S)).to(torch.bfloat16).to(dev)
    y = m(x)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    assert y.shape == x.shape

    planes, nsplit = m.router_planes()
    _, _, logits = route_fused(x.view(S, H, dh), planes, nsplit, E, K, "softmax", m.router.expert_bias.view(H, E),
                               True, 1e-12, 1.0, return_logits=True)
    p, i = route_ref.compute_topk_probs_and_indices(logits.cpu().numpy(), K, "softmax")
    g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    dhp, dep = padded(dh), padded(de)
    Wg, Wu, Wd = (w.detach().float().cpu().numpy() for w in (m.W_gate, m.W_up, m.W_down))
    Wg, Wu = (_pad(_pad(w, 1, dhp), 2, dep) for w in (Wg, Wu))
    Wd = _pad(_pad(Wd, 1, dep), 2, dhp)
    xh = _pad(x.float().cpu().numpy().reshape(S, H, dh), 2, dhp)
    ref = ffn_ref.mh_moe_fwd_nvfp4_ref(xh, g, ps, o, nv.pack_gate_up(Wg, Wu), nv.pack_down(Wd))[..., :dh]
    got = y.float().cpu().numpy().reshape(S, H, dh)
    err = rel_l2(got, ref)
    assert np.isfinite(got).all() and err < 1e-2, err


def test_reference_shape_contract():
    """Shapes outside the reference's contract raise as the reference does."""
    from flash_mh_moe.nvfp4 import check_dims
    with pytest.raises(AssertionError):
        check_dims(96, 64)
    with pytest.raises(AssertionError):
        check_dims(128, 48)
