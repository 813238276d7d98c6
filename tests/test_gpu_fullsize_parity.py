"""GPU parity at the benchmark's full sizes, against the oracle.

BASELINE configs 1 and 2 (S=16384 tokens, d=3072 as one head, E=128, top-8 softmax,
SwiGLU7 d_expert 1024; config 2 adds the Zipf logit bias 2*ln((e+1)^-1.2)) and MAGI-2's
production head split (H=12 heads of 256, E=256 per head, top-6 sigmoid, route_scale 4.9,
d_expert 1280; configs/magi2_preview.json:40-88), with the seeds and generators the
benchmark uses.

* Routing, every token: the top-k indices the fused router returns equal the reference
  top-k (route.py:28-148, restated in oracle.route_ref) run on the fp32 logits the same
  kernel returned; probs within 3e-6 relative.
* Permutation, every routed row: gather_ids, probs_sorted and expert_offsets equal the
  reference global sort (route.py:209-253) of the GPU's own top-k output, bit for bit, and
  row_of_flat is its inverse.
* Layer output, sampled tokens: each sampled (token, head)'s K expert rows are computed on
  the CPU by the NVFP4 restatement of _mh_moe_fwd_kernel (mh_moe_fwd.py:50-181) from the
  weights the GPU packed (the packer is byte-exact against the CPU packer in
  test_gpu_nvfp4), summed in ascending row order in fp32 and rounded to bf16 once, as the
  combine does.  Bar: relative L2 <= 1e-2 (north star), max-abs reported.
"""
import numpy as np
import pytest
import torch

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

CONFIGS = {
    # name: S, H, dh, E, K, de, score, route_scale, seed, zipf, sampled tokens
    "config1": (16384, 1, 3072, 128, 8, 1024, "softmax", 1.0, 1, False, 256),
    "config2": (16384, 1, 3072, 128, 8, 1024, "softmax", 1.0, 2, True, 256),
    "prod_head_split": (16384, 12, 256, 256, 6, 1280, "sigmoid", 4.9, 5, False, 16),
}


def _layer(S, H, dh, E, K, de, score, scale, seed):
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    dev = torch.device("cuda", 0)
    cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                 expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                 score_func=score, route_norm=True, route_scale=scale)
    m = CoreMultiHeadMoE(cfg).to(dev)
    init_moe_params_(m, seed=seed, device=dev)          # as bench.py: generated on the device
    x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(seed * 1000)).to(torch.bfloat16).to(dev)
    return m, x


def _pack_np(gu, dn, experts):
    """The GPU-packed operands of the given flattened experts, as the oracle's pack dicts."""
    sel = torch.as_tensor(experts, dtype=torch.int64, device=gu.data.device)
    gu_pack = {"data": gu.data.index_select(0, sel).cpu().numpy(), "sf_atoms": gu.sf.index_select(0, sel).cpu().numpy(),
               "gscale_gate": gu.gscale[0].index_select(0, sel).cpu().numpy(),
               "gscale_up": gu.gscale[1].index_select(0, sel).cpu().numpy(),
               "N": 2 * gu.d_expert, "K": gu.d_head, "de": gu.d_expert}
    dn_pack = {"data": dn.data.index_select(0, sel).cpu().numpy(), "sf_atoms": dn.sf.index_select(0, sel).cpu().numpy(),
               "gscale": dn.gscale.index_select(0, sel).cpu().numpy(), "N": dn.d_head, "K": dn.d_expert}
    return gu_pack, dn_pack


def sampled_tokens_ref(x_heads, tokens, probs, idx, E, gu, dn):
    """Oracle output rows [len(tokens), H, dh] for the sampled tokens: per (token, head),
    its K rows bf16(down(swiglu7(gate/up)) * prob) in ascending expert order (the order of
    the stable sort), summed in fp32 and rounded to bf16 once."""
    H, _, K = idx.shape
    dh = x_heads.shape[2]
    n = len(tokens)
    xs = nv.bf16_round(x_heads[tokens].astype(np.float32))                       # [n, H, dh]
    codes, sf, g = nv.quantize_rows(xs.reshape(n * H, dh))
    codes = codes.reshape(n, H, dh)
    sf = sf.reshape(n, H, dh // 16)
    g = g.reshape(n, H)
    row_tok, row_code, row_sf, row_g, row_exp, row_prob = [], [], [], [], [], []
    for j, s in enumerate(tokens):
        for h in range(H):
            order = np.argsort(idx[h, s], kind="stable")                           # ascending expert
            for k in order:
                row_tok.append(j * H + h)
                row_code.append(codes[j, h])
                row_sf.append(sf[j, h])
                row_g.append(g[j, h])
                row_exp.append(h * E + int(idx[h, s, k]))
                row_prob.append(probs[h, s, k])
    experts = np.unique(row_exp)
    remap = {e: i for i, e in enumerate(experts)}
    gu_pack, dn_pack = _pack_np(gu, dn, experts)
    rows = ffn_ref.nvfp4_expert_rows_ref(np.stack(row_code), np.stack(row_sf), np.asarray(row_g, np.float32),
                                         np.array([remap[e] for e in row_exp]), np.asarray(row_prob, np.float32),
                                         gu_pack, dn_pack)
    out = np.zeros((n * H, dh), np.float32)
    for r, t in enumerate(row_tok):                                                  # ascending row order
        out[t] = (out[t] + rows[r]).astype(np.float32)
    return nv.bf16_round(out).reshape(n, H, dh)


@pytest.mark.parametrize("name", list(CONFIGS))
def test_fullsize_routing_sort_and_sampled_rows_match_oracle(name):
    from flash_mh_moe import _lib
    from flash_mh_moe.fwd import ffn_nvfp4
    from flash_mh_moe.route import flash_mh_moe_global_sort_with_inverse, route_fused
    S, H, dh, E, K, de, score, scale, seed, zipf, n_sample = CONFIGS[name]
    m, x = _layer(S, H, dh, E, K, de, score, scale, seed)
    dev = x.device
    x_heads = x.view(S, H, dh)
    planes, nsplit = m.router_planes()
    lbias = None
    if zipf:
        e = torch.arange(E, dtype=torch.float32, device=dev)
        lbias = (2.0 * torch.log((e + 1.0) ** -1.2)).repeat(H)
    ebias = m.router.expert_bias.view(H, E)
    probs, idx, logits = route_fused(x_heads, planes, nsplit, E, K, score, ebias, True, 1e-12, scale,
                                     return_logits=True, logit_bias=lbias)
    gids, ps, offs, inv = flash_mh_moe_global_sort_with_inverse(probs, idx, E)
    gu, dn = m.packed_weights()
    y = ffn_nvfp4(x_heads, gids, ps, offs, gu, dn, tok_rows=inv, k_fixed=K, deterministic=True)
    if lbias is None:
        assert torch.equal(m(x).view(S, H, dh), y)          # the module forward is this same path
    torch.cuda.synchronize()
    _lib.check_device_status(dev)

    # routing of every token, on the logits the kernel scored
    p_gpu, i_gpu = probs.cpu().numpy(), idx.cpu().numpy()
    p_ref, i_ref = route_ref.compute_topk_probs_and_indices(logits.cpu().numpy(), K, score,
                                                            ebias.cpu().numpy())
    p_ref = (p_ref * np.float32(scale)).astype(np.float32)
    n_bad = int((i_ref != i_gpu).any(-1).sum())
    assert n_bad == 0, f"{n_bad} (head, token) rows route differently from the reference top-k"
    np.testing.assert_allclose(p_gpu, p_ref, rtol=3e-6, atol=1e-7)

    # permutation of every routed row
    g_ref, ps_ref, o_ref = route_ref.flash_mh_moe_global_sort(p_gpu, i_gpu, E)
    assert np.array_equal(gids.cpu().numpy(), g_ref)
    assert np.array_equal(ps.cpu().numpy().view(np.uint32), ps_ref.view(np.uint32))
    assert np.array_equal(offs.cpu().numpy(), o_ref)
    inv_np = inv.cpu().numpy()
    assert np.array_equal(np.sort(inv_np), np.arange(H * S * K))
    assert np.array_equal(g_ref[inv_np], np.repeat(np.tile(np.arange(S), H), K))
    if zipf:   # the skew the config is about: empty and crowded experts
        counts = np.diff(o_ref)
        assert (counts == 0).sum() > 30 and counts.max() > S // 2

    # sampled tokens through the whole layer
    rng = np.random.default_rng(seed)
    tokens = np.sort(rng.choice(S, size=n_sample, replace=False))
    ref = sampled_tokens_ref(x_heads.float().cpu().numpy(), tokens, p_gpu, i_gpu, E, gu, dn)
    got = y.float().cpu().numpy()[tokens]
    err = rel_l2(got, ref)
    mabs = float(np.abs(got - ref).max())
    print(f"{name}: {n_sample} sampled tokens, rel L2 {err:.3e}, max abs {mabs:.3e}")
    assert np.isfinite(got).all() and err < 1e-2, err
