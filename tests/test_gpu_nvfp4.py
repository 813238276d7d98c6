"""GPU parity: NVFP4 quantisers, weight packer and the raw tcgen05 block-scaled GEMM.

Quantiser and packer outputs are byte-compared with the CPU codec
(oracle/nvfp4_ref.py) on identical inputs; the GEMM accumulator is compared with an
fp64 product of the dequantised operands.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_ref as nv

from gpu_util import bf16_tensor, rel_l2, to_np

pytestmark = pytest.mark.gpu


def _lib():
    from flash_mh_moe import _lib
    return _lib


def test_quantize_rows_bit_exact():
    from flash_mh_moe.nvfp4 import quantize_rows
    rng = np.random.default_rng(0)
    M, K = 300, 3072
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[1] = 0.0                                   # all-zero row: g = 1, codes/sf 0
    x[2] *= 1e-30                                # tiny row
    x[3, :64] = 1e4                              # one hot block
    x[4] = np.exp(rng.uniform(-20, 5, K)) * np.sign(rng.standard_normal(K))   # wide dynamic range
    x[5, ::7] = -0.0
    xb = bf16_tensor(x)
    xr = nv.bf16_round(x)
    data, sf, g = quantize_rows(xb)
    codes, sfb, gg = nv.quantize_rows(xr)
    np.testing.assert_array_equal(to_np(g), gg)
    np.testing.assert_array_equal(to_np(data), nv.pack_codes(codes))
    atoms = to_np(sf)
    np.testing.assert_array_equal(nv.atoms_to_sf(atoms, M, K), sfb)


@pytest.mark.parametrize("n,dh,de", [(4, 256, 256), (2, 512, 384)])
def test_pack_weights_bit_exact(n, dh, de):
    from flash_mh_moe.nvfp4 import pack_down, pack_gate_up
    g = torch.Generator().manual_seed(5)
    Wg = (torch.randn(n, dh, de, generator=g) * 0.02).to(torch.bfloat16)
    Wu = (torch.randn(n, dh, de, generator=g) * 0.05).to(torch.bfloat16)
    Wd = (torch.randn(n, de, dh, generator=g) * 0.02).to(torch.bfloat16)
    Wg[0, :16, :16] = 0                          # an all-zero block
    gu = pack_gate_up(Wg.cuda(), Wu.cuda())
    dn = pack_down(Wd.cuda())
    # sizes that are not multiples of 256 are packed zero-padded up to one
    dhp, dep = (dh + 255) // 256 * 256, (de + 255) // 256 * 256
    pad = lambda w, a, b: np.pad(w.float().numpy(), ((0, 0), (0, a - w.shape[1]), (0, b - w.shape[2])))
    ref_gu = nv.pack_gate_up(pad(Wg, dhp, dep), pad(Wu, dhp, dep))
    ref_dn = nv.pack_down(pad(Wd, dep, dhp))
    assert gu.shape == (n, dh, de) and (gu.d_head, gu.d_expert) == (dhp, dep)
    np.testing.assert_array_equal(to_np(gu.gscale[0]), ref_gu["gscale_gate"])
    np.testing.assert_array_equal(to_np(gu.gscale[1]), ref_gu["gscale_up"])
    np.testing.assert_array_equal(to_np(gu.data), ref_gu["data"])
    np.testing.assert_array_equal(to_np(gu.sf), ref_gu["sf_atoms"])
    np.testing.assert_array_equal(to_np(dn.gscale), ref_dn["gscale"])
    np.testing.assert_array_equal(to_np(dn.data), ref_dn["data"])
    np.testing.assert_array_equal(to_np(dn.sf), ref_dn["sf_atoms"])


def _rand_operand(rng, rows, K, unit_scale):
    codes = rng.integers(0, 16, size=(rows, K), dtype=np.uint8)
    if unit_scale:
        sf = np.full((rows, K // 16), 0x38, np.uint8)            # E4M3 1.0
    else:
        e = rng.integers(4, 11, size=(rows, K // 16))
        m = rng.integers(0, 8, size=(rows, K // 16))
        sf = ((e << 3) | m).astype(np.uint8)
    return codes, sf


@pytest.mark.parametrize("unit_scale,N,K,n_mt", [(True, 512, 512, 3), (False, 512, 512, 3),
                                                  (False, 1536, 512, 3),    # 6 n-tiles: a full and a partial unit
                                                  (False, 512, 4096, 2)])   # K > 3072: A scales per stage
def test_gemm_raw_matches_dequantised_product(unit_scale, N, K, n_mt):
    L = _lib()
    rng = np.random.default_rng(1 if unit_scale else 2)
    n_exp = 2
    tile_expert = np.array([0, 1, 1][:n_mt], np.int32)
    a_codes, a_sf = _rand_operand(rng, n_mt * 128, K, unit_scale)
    b = [_rand_operand(rng, N, K, unit_scale) for _ in range(n_exp)]
    a_data = torch.from_numpy(nv.pack_codes(a_codes)).cuda()
    a_atoms = torch.from_numpy(nv.sf_to_atoms(a_sf)).cuda()
    b_data = torch.from_numpy(np.stack([nv.pack_codes(c) for c, _ in b])).cuda()
    b_atoms = torch.from_numpy(np.stack([nv.sf_to_atoms(s) for _, s in b])).cuda()
    te = torch.from_numpy(tile_expert).cuda()
    out = torch.full((n_mt * 128, N), float("nan"), dtype=torch.float32, device="cuda")
    st = L.device_status(out.device)
    L.check(L.lib().mhmoe_gemm_nvfp4_raw(a_data.data_ptr(), a_atoms.data_ptr(), n_mt, te.data_ptr(),
                                          b_data.data_ptr(), b_atoms.data_ptr(), n_exp, N, K, out.data_ptr(),
                                          st.data_ptr(), 0, L.stream_ptr()), "gemm_raw")
    torch.cuda.synchronize()
    L.check_device_status(out.device)
    a_deq = nv.dequantize(a_codes, a_sf).astype(np.float64)
    ref = np.empty((n_mt * 128, N))
    for mt in range(n_mt):
        e = tile_expert[mt]
        b_deq = nv.dequantize(b[e][0], b[e][1]).astype(np.float64)
        ref[mt * 128:(mt + 1) * 128] = a_deq[mt * 128:(mt + 1) * 128] @ b_deq.T
    got = to_np(out)
    assert np.isfinite(got).all()
    err = rel_l2(got, ref)
    assert err < 1e-5, f"raw GEMM rel L2 {err}"
