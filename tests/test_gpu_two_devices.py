"""One process driving two GPUs: every kernel's per-device set-up (shared-memory limits,
cluster occupancy, scratch addresses) must happen on each device, not once per process.
Runs the routed layer on cuda:0, then cuda:1, then cuda:0 again, and requires the three
outputs to be identical.  Skipped on a box with one GPU."""
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs in one process")]


@pytest.mark.parametrize("S,H,dh,de,E,K,score", [(2048, 1, 3072, 1024, 16, 8, "softmax"),   # tensor-core router
                                                 (96, 12, 256, 256, 16, 6, "sigmoid")])     # small-batch router
def test_layer_on_two_devices_in_one_process(S, H, dh, de, E, K, score):
    from flash_mh_moe import _lib
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    from flash_mh_moe.route import flash_mh_moe_global_sort_with_inverse
    cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                 expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                 score_func=score, route_norm=True, route_scale=1.0)
    x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    outs, sorts = [], []
    for d in (0, 1, 0):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            m = CoreMultiHeadMoE(cfg).to(dev)
            init_moe_params_(m, seed=11, device=dev)
            xd = x.to(dev)
            outs.append(m(xd).cpu())
            probs, idx = m._route(xd.view(S, H, dh))
            sorts.append([t.cpu() for t in flash_mh_moe_global_sort_with_inverse(probs, idx, E)])
            torch.cuda.synchronize(dev)
            _lib.check_device_status(dev)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    for a, b in zip(sorts[0], sorts[1]):
        assert torch.equal(a, b)
