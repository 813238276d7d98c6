"""GPU parity: NVFP4 expert FFN (flash_mh_moe_fwd) against the CPU oracle.

The oracle (oracle/ffn_ref.py::mh_moe_fwd_nvfp4_ref) restates the reference kernel's
math on the same NVFP4 operands, quantising x and the SwiGLU7 output at the points the
GPU does.  Bar: relative L2 <= 1e-2; typical is ~1e-3.
"""
import numpy as np
import pytest
import torch

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

from gpu_util import bf16_tensor, rel_l2, seeded_moe, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _route(x, gate, S, H, dh, E, K, skew=0.0):
    logits = route_ref.router_logits(x.reshape(S, H, dh), gate, E)
    if skew:
        e = np.arange(E, dtype=np.float32)
        logits = logits + np.float32(skew) * np.log((e + 1.0) ** -1.2).astype(np.float32)
    probs, idx = route_ref.compute_topk_probs_and_indices(logits, K)
    return route_ref.flash_mh_moe_global_sort(probs, idx, E)


CASES = [
    # S, H, dh, de, E, K, seed, skew
    (256, 1, 256, 256, 8, 2, 0, 0.0),
    (200, 2, 256, 512, 4, 3, 1, 0.0),
    (333, 1, 512, 256, 16, 4, 2, 2.0),     # Zipf-skewed: empty and crowded experts
    (40, 1, 256, 256, 8, 1, 3, 0.0),       # fewer rows than one tile
    (96, 1, 3072, 512, 8, 4, 4, 0.0),      # config-1 head width: 3 blocks per lane in the quantiser
    (64, 1, 4096, 256, 4, 2, 5, 1.0),      # 4 blocks per lane, K > 3072 in the gate/up GEMM
]


@pytest.mark.parametrize("gemm", ["pair", "single"])
@pytest.mark.parametrize("scatter", ["combine", "atomic"])
@pytest.mark.parametrize("S,H,dh,de,E,K,seed,skew", CASES)
def test_ffn_nvfp4_matches_oracle(S, H, dh, de, E, K, seed, skew, scatter, gemm, monkeypatch):
    """combine: partial rows + fp32 combine (the oracle's order, ~0 error); atomic: bf16
    atomics from the down GEMM (bf16 accumulation in arrival order).  single: one CTA per
    tile, the default; pair: the CTA-pair (cta_group::2) GEMMs (MHMOE_GEMM_PAIR=1)."""
    from flash_mh_moe import flash_mh_moe_fwd
    monkeypatch.setenv("MHMOE_SCATTER", scatter)
    monkeypatch.setenv("MHMOE_GEMM_PAIR", "1" if gemm == "pair" else "0")
    x, gate, Wg, Wu, Wd = seeded_moe(S, H, dh, de, E, K, seed)
    gids, ps, offs = _route(x, gate, S, H, dh, E, K, skew)
    xh = x.reshape(S, H, dh)
    gu = nv.pack_gate_up(Wg, Wu)
    dn = nv.pack_down(Wd)
    ref = ffn_ref.mh_moe_fwd_nvfp4_ref(xh, gids, ps, offs, gu, dn)
    y = flash_mh_moe_fwd(bf16_tensor(xh), torch.from_numpy(gids).cuda(), torch.from_numpy(ps).cuda(),
                         torch.from_numpy(offs).cuda(), bf16_tensor(Wg), bf16_tensor(Wu), bf16_tensor(Wd))
    torch.cuda.synchronize()
    from flash_mh_moe import _lib
    _lib.check_device_status(y.device)
    got = to_np(y)
    assert np.isfinite(got).all()
    err = rel_l2(got, ref)
    assert err < TOL, f"rel L2 vs oracle {err:.3e}"
    # information only: distance to the unquantised bf16 reference restatement
    bf = ffn_ref.mh_moe_fwd_ref(xh, gids, ps, offs, Wg, Wu, Wd, dtype="bf16")
    print(f"rel L2 vs oracle {err:.2e}; vs bf16 reference (NVFP4 quantisation error) {rel_l2(got, bf):.3f}")


@pytest.mark.parametrize("scatter", ["combine", "atomic"])
def test_ffn_deterministic_and_empty(scatter, monkeypatch):
    from flash_mh_moe import flash_mh_moe_fwd
    monkeypatch.setenv("MHMOE_SCATTER", scatter)
    S, H, dh, de, E, K = 300, 1, 256, 256, 8, 2
    x, gate, Wg, Wu, Wd = seeded_moe(S, H, dh, de, E, K, 9)
    gids, ps, offs = _route(x, gate, S, H, dh, E, K)
    args = (bf16_tensor(x.reshape(S, H, dh)), torch.from_numpy(gids).cuda(), torch.from_numpy(ps).cuda(),
            torch.from_numpy(offs).cuda(), bf16_tensor(Wg), bf16_tensor(Wu), bf16_tensor(Wd))
    y1 = flash_mh_moe_fwd(*args)
    y2 = flash_mh_moe_fwd(*args)
    if scatter == "combine":
        assert torch.equal(y1, y2)
    else:   # atomic order may differ run to run: bf16 rounding only
        assert rel_l2(to_np(y1), to_np(y2)) < 1e-2
    # no routed rows -> zeros (reference mh_moe_fwd.py:257-258)
    z = flash_mh_moe_fwd(args[0], torch.empty(0, dtype=torch.int32, device="cuda"),
                         torch.empty(0, device="cuda"), torch.zeros(E + 1, dtype=torch.int64, device="cuda"),
                         *args[4:])
    assert torch.count_nonzero(z) == 0


@pytest.mark.parametrize("S,H,dh,de,E,K,seed,skew", [CASES[2], CASES[4], CASES[5]])
def test_ffn_quantise_paths_identical(S, H, dh, de, E, K, seed, skew, monkeypatch):
    """The A operand is the same bytes whichever way it is built: quantise + scatter in one
    kernel (the default for local tokens), or per-token quantisation then grouping by row
    (the path of expert-parallel records; MHMOE_QUANT_FUSED=0 selects it for local tokens)."""
    from flash_mh_moe import flash_mh_moe_fwd
    x, gate, Wg, Wu, Wd = seeded_moe(S, H, dh, de, E, K, seed)
    gids, ps, offs = _route(x, gate, S, H, dh, E, K, skew)
    args = (bf16_tensor(x.reshape(S, H, dh)), torch.from_numpy(gids).cuda(), torch.from_numpy(ps).cuda(),
            torch.from_numpy(offs).cuda(), bf16_tensor(Wg), bf16_tensor(Wu), bf16_tensor(Wd))
    outs = []
    for fused in ("1", "0"):
        monkeypatch.setenv("MHMOE_QUANT_FUSED", fused)
        outs.append(flash_mh_moe_fwd(*args))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
