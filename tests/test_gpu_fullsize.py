"""GPU: size-independent properties at the benchmark's full size (config 1: 16384 tokens,
d = 3072, 128 experts, top-8, d_expert 1024), where the CPU oracle is too slow.

* Run-to-run: the default (combine) scatter gives bit-identical outputs.
* Two implementations agree: the default path (fused quantise+group, single-CTA GEMMs with
  the scale-factor copier) and the CTA-pair path (per-token quantise, grouping copy,
  cta_group::2 GEMMs; MHMOE_GEMM_PAIR=1) compute the same NVFP4 math with different
  kernels.  Bar: the oracle tests' 1e-2 relative L2 — a last-bit difference in a gate/up
  accumulator can move a hidden value across an E2M1 rounding boundary, so agreement need
  not be bit-exact; a wrong row or tile gives an error of order 1.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_config1_repeatable_and_paths_agree(monkeypatch):
    from flash_mh_moe import _lib
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    dev = torch.device("cuda", 0)
    S, d, E, K, de = 16384, 3072, 128, 8, 1024
    cfg = CoreMultiHeadMoEConfig(hidden_size=d, num_heads=1, num_experts=E, top_k=K, expert_intermediate_size=de,
                                 num_layers=1, params_dtype=torch.bfloat16, score_func="softmax",
                                 route_norm=True, route_scale=1.0)
    m = CoreMultiHeadMoE(cfg).to(dev)
    init_moe_params_(m, seed=1, device=dev)
    x = torch.randn(S, d, generator=torch.Generator(device=dev).manual_seed(11), device=dev).to(torch.bfloat16)
    monkeypatch.setenv("MHMOE_SCATTER", "combine")
    monkeypatch.setenv("MHMOE_GEMM_PAIR", "0")
    y1 = m(x)
    y2 = m(x)
    monkeypatch.setenv("MHMOE_GEMM_PAIR", "1")
    y3 = m(x)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    assert torch.isfinite(y1.float()).all()
    assert float(y1.float().abs().mean()) > 0
    assert torch.equal(y1, y2)
    err = _rel(y3, y1)
    print(f"config 1: pair path vs default path rel L2 {err:.3e}")
    assert err < 1e-2, f"pair path vs default path rel L2 {err:.3e}"
