"""CPU: the oracle is pinned against the reference's own outputs (golden fixtures) and
the NVFP4 codec against known answers.  No GPU needed."""
from pathlib import Path

import numpy as np
import pytest

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

GOLD = Path(__file__).resolve().parent / "golden"


# ───────────────────────── router / sort vs reference route.py ─────────────────────────

_R = np.load(GOLD / "route_cases.npz")
_NAMES = sorted({k.split("/")[0] for k in _R.files})


@pytest.mark.parametrize("name", _NAMES)
def test_route_oracle_matches_reference(name):
    d = _R
    H, S, E, K, nvg, tvg, rn, ub = (int(v) for v in d[name + "/meta"])
    sf = str(d[name + "/score_func"])
    bias = d[name + "/bias"] if ub else None
    p, i = route_ref.compute_topk_probs_and_indices(d[name + "/logits"], K, sf, bias, nvg, tvg, bool(rn))
    ri, rp = d[name + "/idx"], d[name + "/probs"]
    if nvg > 1:
        oi, orr = np.argsort(i, -1), np.argsort(ri, -1)
        i, p = np.take_along_axis(i, oi, -1), np.take_along_axis(p, oi, -1)
        ri, rp = np.take_along_axis(ri, orr, -1), np.take_along_axis(rp, orr, -1)
    np.testing.assert_array_equal(i, ri)
    np.testing.assert_allclose(p, rp, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", _NAMES)
def test_sort_oracle_matches_reference(name):
    d = _R
    E = int(d[name + "/meta"][2])
    g, p, o = route_ref.flash_mh_moe_global_sort(d[name + "/probs"], d[name + "/idx"], E)
    np.testing.assert_array_equal(g, d[name + "/gather_ids"])
    np.testing.assert_array_equal(p, d[name + "/probs_sorted"])
    np.testing.assert_array_equal(o, d[name + "/expert_offsets"])


def test_route_oracle_unknown_score_func():
    with pytest.raises(ValueError):
        route_ref.compute_topk_probs_and_indices(np.zeros((1, 2, 4), np.float32), 2, "relu")


# ───────────────────────── FFN restatement vs the reference Triton kernel ─────────────────────────

@pytest.mark.parametrize("name", ["small", "ragged"])
def test_ffn_oracle_matches_reference_kernel(name):
    f = np.load(GOLD / "ffn_fp32.npz")
    args = [f[name + "/" + k] for k in ["x", "gather_ids", "probs_sorted", "expert_offsets", "W_gate", "W_up",
                                         "W_down"]]
    y = ffn_ref.mh_moe_fwd_ref(*args, dtype="fp32")
    assert ffn_ref.rel_l2(y, f[name + "/y_det"]) < 1e-6
    assert ffn_ref.rel_l2(y, f[name + "/y_atomic"]) < 1e-6


def test_ffn_oracle_empty_rows():
    x = np.ones((4, 1, 64), np.float32)
    y = ffn_ref.mh_moe_fwd_ref(x, np.zeros(0, np.int32), np.zeros(0, np.float32), np.zeros(3, np.int64),
                               np.zeros((2, 64, 32)), np.zeros((2, 64, 32)), np.zeros((2, 32, 64)))
    assert not y.any()


def test_nvfp4_oracle_tracks_bf16_reference():
    """The fake-quant oracle stays within NVFP4 quantisation error of the bf16 reference
    restatement (information for the tolerance choice: ~0.1-0.2 relative L2)."""
    rng = np.random.default_rng(0)
    S, H, dh, de, E, K = 64, 1, 256, 256, 4, 2
    x = nv.bf16_round(rng.standard_normal((S, H, dh)).astype(np.float32))
    logits = rng.standard_normal((H, S, E)).astype(np.float32)
    p, i = route_ref.compute_topk_probs_and_indices(logits, K)
    g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    Wg = nv.bf16_round(rng.standard_normal((E, dh, de)).astype(np.float32) * 0.02)
    Wu = nv.bf16_round(rng.standard_normal((E, dh, de)).astype(np.float32) * 0.02)
    Wd = nv.bf16_round(rng.standard_normal((E, de, dh)).astype(np.float32) * 0.02)
    yq = ffn_ref.mh_moe_fwd_nvfp4_ref(x, g, ps, o, nv.pack_gate_up(Wg, Wu), nv.pack_down(Wd))
    yb = ffn_ref.mh_moe_fwd_ref(x, g, ps, o, Wg, Wu, Wd, dtype="bf16")
    err = ffn_ref.rel_l2(yq, yb)
    assert 0.02 < err < 0.3


# ───────────────────────── NVFP4 codec known answers ─────────────────────────

def test_e2m1_grid_and_ties():
    vals = np.array([0, 0.25, 0.2500001, 0.5, 0.75, 1.0, 1.25, 1.5, 1.75, 2.0, 2.5, 3.0, 3.5, 4.0, 5.0, 6.0, 7.0,
                     1e9], np.float32)
    want = np.array([0, 0, 1, 1, 2, 2, 2, 3, 4, 4, 4, 5, 6, 6, 6, 7, 7, 7], np.uint8)
    np.testing.assert_array_equal(nv.e2m1_encode(vals), want)
    np.testing.assert_array_equal(nv.e2m1_encode(-vals), want | 8)
    np.testing.assert_array_equal(nv.e2m1_decode(np.arange(8)), nv.E2M1_GRID)


def test_e4m3_known_answers():
    vals = np.array([0.0, 2.0 ** -9, 1.5 * 2.0 ** -9, 2.0 ** -6, 1.0, 1.0625, 1.125, 448.0, 1e6, 240.0, 0.1],
                    np.float32)
    want = np.array([0x00, 0x01, 0x02, 0x08, 0x38, 0x38, 0x39, 0x7E, 0x7E, 0x77, 0x1D], np.uint8)
    np.testing.assert_array_equal(nv.e4m3_encode(vals), want)
    np.testing.assert_array_equal(nv.e4m3_decode(np.array([0x38, 0x7E, 0x01, 0x08], np.uint8)),
                                  np.array([1.0, 448.0, 2.0 ** -9, 2.0 ** -6], np.float32))


def test_e4m3_matches_ml_dtypes():
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(3)
    t = np.minimum(np.exp(rng.uniform(-25, 6.2, 200000)).astype(np.float32), 448).astype(np.float32)
    np.testing.assert_array_equal(nv.e4m3_encode(t), t.astype(ml.float8_e4m3fn).view(np.uint8))


def test_nibble_order_and_roundtrip():
    codes = np.array([[1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 0]], np.uint8)
    packed = nv.pack_codes(codes)
    assert packed[0, 0] == 0x21 and packed[0, 7] == 0x0F
    np.testing.assert_array_equal(nv.unpack_codes(packed), codes)


def test_block_quant_known_answer():
    v = np.array([[6.0, -3.0, 1.5, 0.0] + [0.0] * 12], np.float32)
    codes, sf = nv.quantize_blocks(v, np.float32(1.0))
    assert sf[0, 0] == 0x38                                  # amax/6 = 1.0
    np.testing.assert_array_equal(codes[0, :4], [7, 13, 3, 0])
    np.testing.assert_allclose(nv.dequantize(codes, sf), v)


def test_hidden_block_scale_is_amax_times_8():
    """The gate/up epilogue computes the hidden's block scale as amax * 8: exact because
    6 * HIDDEN_GLOBAL rounds to 0.125 in fp32, so amax / (6 * g) is a power-of-two scaling."""
    g = nv.HIDDEN_GLOBAL
    assert np.float32(np.float32(6.0) * g) == np.float32(0.125)
    amax = np.random.default_rng(0).uniform(0, 60, 4096).astype(np.float32)
    amax[:4] = [0.0, 1e-40, 3.4e37, 7.0]
    np.testing.assert_array_equal((amax / (np.float32(6.0) * g)).astype(np.float32), amax * np.float32(8.0))


def test_sf_atom_layout():
    M, K = 256, 128
    sf = np.arange(M * K // 16, dtype=np.int64).reshape(M, K // 16) % 251
    sf = sf.astype(np.uint8)
    atoms = nv.sf_to_atoms(sf)
    assert atoms.size == M * K // 16
    # row 33, scale column 5: atom (0, 1), m=33 -> (33%32)*16 + (33//32)*4 + 1
    assert atoms[512 + 1 * 16 + 1 * 4 + 1] == sf[33, 5]
    np.testing.assert_array_equal(nv.atoms_to_sf(atoms, M, K), sf)


def test_pack_roundtrip_close():
    rng = np.random.default_rng(4)
    wg = rng.standard_normal((2, 128, 128)).astype(np.float32) * 0.02
    wu = rng.standard_normal((2, 128, 128)).astype(np.float32) * 0.02
    wd = rng.standard_normal((2, 128, 128)).astype(np.float32) * 0.02
    g2, u2 = nv.dequant_gate_up(nv.pack_gate_up(wg, wu))
    d2 = nv.dequant_down(nv.pack_down(wd))
    for a, b in ((g2, wg), (u2, wu), (d2, wd)):
        assert ffn_ref.rel_l2(a, b) < 0.12


# ───────────────────────── torch CPU path of the timed baseline ─────────────────────────

@pytest.mark.parametrize("H,dh,de,E,K,score,scale", [(1, 256, 512, 8, 2, "softmax", 1.0),
                                                     (3, 128, 256, 6, 3, "sigmoid", 4.9)])
def test_torch_cpu_layer_matches_oracle(H, dh, de, E, K, score, scale):
    """The CPU baseline's torch layer (oracle.ffn_torch_ref) equals the numpy restatement
    pinned against the reference kernel: routing and sort exactly, output within bf16
    rounding of the accumulation order.  With the reference package staged under
    oracle/_ref its own route.py and _scatter_back run, and must give the same result."""
    import torch

    from oracle import ffn_torch_ref, stage_ref
    from gpu_util import seeded_moe
    S = 96
    x, gate, Wg, Wu, Wd = seeded_moe(S, H, dh, de, E, K, seed=5)
    xh = x.reshape(S, H, dh)
    lg = route_ref.router_logits(xh, gate, E)
    p, i = route_ref.compute_topk_probs_and_indices(lg, K, score)
    p = (p * np.float32(scale)).astype(np.float32)
    g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, E)
    want = ffn_ref.mh_moe_fwd_ref(xh, g, ps, o, Wg, Wu, Wd, dtype="bf16")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16)
    args = (t(xh), torch.from_numpy(gate), t(Wg), t(Wu), t(Wd), E, K, score, scale)
    got = ffn_torch_ref.moe_layer_cpu(*args).float().numpy()
    assert ffn_ref.rel_l2(got, want) < 5e-3
    try:
        ref = stage_ref.import_ref()
    except ImportError:
        return
    got_ref = ffn_torch_ref.moe_layer_cpu(*args, ref=ref).float().numpy()
    np.testing.assert_array_equal(got_ref, got)


# ───────────────────────── MoE layer around the core vs the reference module ─────────────────────────

_L = np.load(GOLD / "layer_cases.npz")
_LNAMES = sorted({k.split("/")[0] for k in _L.files})


@pytest.mark.parametrize("name", _LNAMES)
def test_layer_oracle_matches_reference(name):
    """oracle.layer_ref's pre-norm and shared experts against the reference module's own
    MultiModalityRMSNorm and MultiHeadMoELayer._shared_expert_forward (bf16, CPU)."""
    from oracle import layer_ref
    d = lambda k: _L[f"{name}/{k}"]
    groups = [int(v) for v in d("groups")]
    norm = layer_ref.rmsnorm_ref(d("x"), d("pre_norm.weight"), groups)
    # one bf16 ulp at most (the mean's summation order differs)
    ulp = np.abs(norm - d("norm")) / np.maximum(np.abs(d("norm")), 1e-30)
    assert float(ulp.max()) <= 2.0 ** -7
    shared = layer_ref.shared_experts_ref(d("norm"), groups, d("shared_expert_fc1.weight"),
                                          d("shared_expert_fc2.weight"),
                                          d("modality_specific_shared_expert_fc1.weight"),
                                          d("modality_specific_shared_expert_fc2.weight"))
    assert ffn_ref.rel_l2(shared, d("shared")) < 2e-3
