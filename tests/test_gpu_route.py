"""GPU parity: router logits, top-k and the global sort against the reference's own outputs.

Top-k and sort fixtures come from the reference ``route.py`` (tests/golden/make_golden.py).
Indices and the permutation must match bit for bit; probs to fp32 rounding.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import route_ref

from gpu_util import rel_l2, to_np

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "route_cases.npz"


def _cases():
    d = np.load(GOLD)
    return d, sorted({k.split("/")[0] for k in d.files})


_D, _NAMES = _cases()


@pytest.mark.parametrize("name", _NAMES)
def test_topk_matches_reference(name):
    from flash_mh_moe import compute_topk_probs_and_indices
    d = _D
    H, S, E, K, nvg, tvg, rn, ub = (int(v) for v in d[name + "/meta"])
    sf = str(d[name + "/score_func"])
    logits = torch.from_numpy(d[name + "/logits"]).cuda()
    bias = torch.from_numpy(d[name + "/bias"]).cuda() if ub else None
    probs, idx = compute_topk_probs_and_indices(logits, K, sf, bias, nvg, tvg, bool(rn))
    ri, rp = d[name + "/idx"], d[name + "/probs"]
    gi, gp = to_np(idx), to_np(probs)
    if nvg > 1:   # reference returns the selected set unsorted (topk sorted=False)
        order_g, order_r = np.argsort(gi, -1), np.argsort(ri, -1)
        gi, gp = np.take_along_axis(gi, order_g, -1), np.take_along_axis(gp, order_g, -1)
        ri, rp = np.take_along_axis(ri, order_r, -1), np.take_along_axis(rp, order_r, -1)
    np.testing.assert_array_equal(gi, ri)
    np.testing.assert_allclose(gp, rp, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", _NAMES)
def test_global_sort_matches_reference(name):
    from flash_mh_moe import flash_mh_moe_global_sort
    d = _D
    E = int(d[name + "/meta"][2])
    probs = torch.from_numpy(d[name + "/probs"]).cuda()
    idx = torch.from_numpy(d[name + "/idx"]).cuda()
    g, p, o = flash_mh_moe_global_sort(probs, idx, E)
    np.testing.assert_array_equal(to_np(g), d[name + "/gather_ids"])
    np.testing.assert_array_equal(to_np(p), d[name + "/probs_sorted"])
    np.testing.assert_array_equal(to_np(o), d[name + "/expert_offsets"])


@pytest.mark.parametrize("H,S,K,E", [(1, 16384, 8, 128), (12, 2048, 6, 256), (1, 1, 2, 8), (3, 777, 5, 40),
                                     (2, 16000, 8, 120), (1, 32768, 8, 256), (12, 16384, 6, 256)])
def test_global_sort_large_matches_oracle(H, S, K, E):
    from flash_mh_moe.route import flash_mh_moe_global_sort_with_inverse
    rng = np.random.default_rng(H * 1000 + S)
    logits = rng.standard_normal((H, S, E)).astype(np.float32)
    logits[..., 0] += 3.0                         # crowded expert
    idx = np.argsort(-logits, -1, kind="stable")[..., :K].astype(np.int64)
    probs = rng.random((H, S, K)).astype(np.float32)
    g, p, o, inv = flash_mh_moe_global_sort_with_inverse(torch.from_numpy(probs).cuda(),
                                                         torch.from_numpy(idx).cuda(), E)
    rg, rp, ro = route_ref.flash_mh_moe_global_sort(probs, idx, E)
    np.testing.assert_array_equal(to_np(g), rg)
    np.testing.assert_array_equal(to_np(p), rp)
    np.testing.assert_array_equal(to_np(o), ro)
    # row_of_flat is the inverse permutation
    gidx = (idx + np.arange(H).reshape(H, 1, 1) * E).reshape(-1)
    order = np.argsort(gidx, kind="stable")
    ref_inv = np.empty_like(order)
    ref_inv[order] = np.arange(order.size)
    np.testing.assert_array_equal(to_np(inv), ref_inv)


@pytest.mark.parametrize("S,H,dh,E", [(512, 1, 1024, 8), (300, 2, 256, 64), (130, 12, 256, 256)])
def test_router_logits_fp32(S, H, dh, E):
    from flash_mh_moe.route import router_logits
    g = torch.Generator().manual_seed(S + E)
    x = torch.randn(S, H, dh, generator=g).to(torch.bfloat16)
    gate = torch.randn(H * E, dh, generator=g) * 0.02
    out = router_logits(x.cuda(), gate.cuda(), E)
    ref = route_ref.router_logits(x.float().numpy(), gate.numpy(), E)
    assert rel_l2(to_np(out), ref) < 1e-6
    np.testing.assert_allclose(to_np(out), ref, rtol=1e-4, atol=1e-5)


FUSED = [
    # S, H, dh, E, K, score, bias, route_scale, bf16_gate
    (512, 1, 1024, 8, 2, "softmax", False, 1.0, True),      # config-0 router
    (1000, 1, 3072, 128, 8, "softmax", False, 1.0, True),   # config-1 router (partial batch)
    (300, 2, 256, 64, 4, "sigmoid", True, 2.5, False),      # fp32 gate -> 3 planes
    (130, 12, 256, 256, 6, "sigmoid", True, 4.9, False),    # production head split
    (77, 1, 128, 40, 16, "softmax", True, 1.0, False),      # ragged E, K = 16
]


@pytest.mark.parametrize("path", ["default", "tensor_core"])
@pytest.mark.parametrize("S,H,dh,E,K,score,use_bias,scale,bf16_gate", FUSED)
def test_fused_router_matches_reference(S, H, dh, E, K, score, use_bias, scale, bf16_gate, path, monkeypatch):
    """Both router kernels: batches of a few 128-token tiles take the cluster split-K
    router by default (route_small.cu); MHMOE_ROUTER_TC_ONLY=1 forces the tensor-core
    router (router_tc.cu) the full-size batches use."""
    if path == "tensor_core":
        monkeypatch.setenv("MHMOE_ROUTER_TC_ONLY", "1")
    else:
        monkeypatch.delenv("MHMOE_ROUTER_TC_ONLY", raising=False)
    from flash_mh_moe.route import route_fused, router_prepare
    g = torch.Generator().manual_seed(S * 7 + E)
    x = torch.randn(S, H, dh, generator=g).to(torch.bfloat16)
    gate = torch.randn(H * E, dh, generator=g) * 0.02
    if bf16_gate:
        gate = gate.to(torch.bfloat16).float()
    bias = (torch.randn(H, E, generator=g) * 0.01) if use_bias else None
    planes, nsplit = router_prepare(gate.cuda())
    assert nsplit == (1 if bf16_gate else 3)
    probs, idx, logits = route_fused(x.cuda(), planes, nsplit, E, K, score, None if bias is None else bias.cuda(),
                                     True, 1e-12, scale, return_logits=True)
    ref_logits = route_ref.router_logits(x.float().numpy(), gate.numpy(), E)
    gl = to_np(logits)
    # Products are exact (x is bf16, the gate is split into exact bf16 planes); the
    # tensor core's fp32 accumulation is coarser than an IEEE FMA chain: measured
    # 3.3e-6 relative L2 at dh = 3072.  Bound: 1e-5.
    assert rel_l2(gl, ref_logits) < 1e-5
    # routing parity on the GPU's own logits (the reference contract is route.py on the logits)
    b = None if bias is None else bias.numpy()
    rp, ri = route_ref.compute_topk_probs_and_indices(gl, K, score, b)
    np.testing.assert_array_equal(to_np(idx), ri)
    np.testing.assert_allclose(to_np(probs), rp * np.float32(scale), rtol=3e-6, atol=1e-7)
    # near-tie flips against fp64 logits: only tokens whose k-th / (k+1)-th scores are
    # within the logit error may choose a different set
    _, ri64 = route_ref.compute_topk_probs_and_indices(ref_logits, K, score, b)
    flips = int((np.sort(ri, -1) != np.sort(ri64, -1)).any(-1).sum())
    print(f"logit rel L2 {rel_l2(gl, ref_logits):.2e}; top-{K} set flips vs fp64 logits: {flips}/{H * S}")
    assert flips <= max(1, H * S // 200)
