"""GPU: the single-GPU MoE layer captured as a CUDA graph (flash_mh_moe.graph) replays to
exactly the eager result (the default combine scatter is deterministic), for new inputs
copied into the captured input too."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_captured_layer_matches_eager():
    from flash_mh_moe import _lib
    from flash_mh_moe.graph import CapturedForward
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    dev = torch.device("cuda", 0)
    S, dh, de, E, K = 256, 512, 256, 16, 4
    cfg = CoreMultiHeadMoEConfig(hidden_size=dh, num_heads=1, num_experts=E, top_k=K, expert_intermediate_size=de,
                                 num_layers=1, params_dtype=torch.bfloat16, score_func="softmax", route_norm=True,
                                 route_scale=1.0)
    layers = []
    for i in range(2):
        m = CoreMultiHeadMoE(cfg).to(dev)
        init_moe_params_(m, seed=11 + i, device=dev)
        layers.append(m)

    def fwd(x):
        for m in layers:
            x = x + m(x)
        return x

    g = torch.Generator().manual_seed(5)
    x1 = torch.randn(S, dh, generator=g).to(torch.bfloat16).to(dev)
    x2 = torch.randn(S, dh, generator=g).to(torch.bfloat16).to(dev)
    cap = CapturedForward(fwd, x1)
    for x in (x1, x2, x1):
        y_graph = cap(x).clone()
        y_eager = fwd(x)
        torch.cuda.synchronize()
        _lib.check_device_status(dev)
        assert torch.equal(y_graph, y_eager)
    with pytest.raises(ValueError):
        cap(x1[: S // 2])
