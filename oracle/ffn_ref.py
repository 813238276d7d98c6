"""numpy restatement of the reference expert FFN, plus its NVFP4 fake-quant twin.

Test infrastructure only (``tests/``, ``__graft_entry__.smoke()``, ``bench.py``'s
CPU-baseline leg).  The product path is the CUDA grouped GEMMs.

* ``mh_moe_fwd_ref``  restates ``inference/flash_mh_moe/triton/mh_moe_fwd.py:50-181``
  (``_mh_moe_fwd_kernel``), ``:189-215`` (``_scatter_back``) and ``:231-331``
  (``mh_moe_fwd_func``) with the reference's casts: operands in the weight dtype,
  fp32 accumulation, ``hidden.to(W_down.dtype)``, ``y_acc * probs`` in fp32, cast to
  ``y.dtype`` and a sequential per-row add in ``y.dtype``.  Pinned against the
  reference Triton kernel run under ``TRITON_INTERPRET=1`` in fp32
  (``tests/golden/make_golden.py``).
* ``mh_moe_fwd_nvfp4_ref`` is the same layer on NVFP4 operands, with x quantised
  per routed row and the SwiGLU7 output quantised with the static scale before
  the down GEMM — the exact points where the CUDA path quantises.  Partial rows are
  rounded to bf16 (as the reference rounds ``y_acc*probs`` to ``y.dtype``) and each
  (token, head) sums its rows in ascending sorted-row order in fp32.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4_ref as nv

SWIGLU7_ALPHA = np.float32(1.702)   # mh_moe_fwd.py:18-20
SWIGLU7_LIMIT = np.float32(7.0)
SWIGLU7_BIAS = np.float32(1.0)


def swiglu7(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """mh_moe_fwd.py:24-30 in fp32."""
    g = np.minimum(np.asarray(gate, np.float32), SWIGLU7_LIMIT)
    u = np.clip(np.asarray(up, np.float32), -SWIGLU7_LIMIT, SWIGLU7_LIMIT)
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-(SWIGLU7_ALPHA * g)).astype(np.float32))).astype(np.float32)
    return ((g * sig).astype(np.float32) * (u + SWIGLU7_BIAS)).astype(np.float32)


def _row_meta(gather_ids, expert_offsets, num_heads):
    """Per sorted row: global expert id and head id (mh_moe_fwd.py:93-97)."""
    offs = np.asarray(expert_offsets, np.int64)
    nflat = offs.size - 1
    counts = np.diff(offs)
    expert = np.repeat(np.arange(nflat), counts)
    head = expert // (nflat // num_heads)
    return expert, head


def _sequential_add(y_flat: np.ndarray, idx: np.ndarray, vals: np.ndarray, rnd) -> np.ndarray:
    """y[idx[i]] = rnd(y[idx[i]] + vals[i]) applied in increasing i (scatter_add_ order)."""
    order = np.argsort(idx, kind="stable")
    sidx = idx[order]
    first = np.r_[True, sidx[1:] != sidx[:-1]]
    grp_start = np.maximum.accumulate(np.where(first, np.arange(sidx.size), 0))
    level = np.arange(sidx.size) - grp_start
    for lv in range(int(level.max()) + 1 if level.size else 0):
        sel = order[level == lv]
        y_flat[idx[sel]] = rnd(y_flat[idx[sel]] + vals[sel])
    return y_flat


def mh_moe_fwd_ref(x, gather_ids, probs, expert_offsets, W_gate, W_up, W_down,
                   dtype: str = "bf16", deterministic: bool = True, round_weights: bool = True) -> np.ndarray:
    """Reference FFN restatement.  x [S,H,dh]; W_gate/W_up [H*E,dh,de]; W_down [H*E,de,dh].

    ``dtype`` is the operand / output dtype: "bf16" rounds operands, hidden and
    output to bf16; "fp32" keeps everything fp32 (the Triton-interpreter check).
    The bf16 atomic path adds in an unspecified order, so only the sequential
    (deterministic) order is restated; both round after every add.
    ``round_weights=False`` skips re-rounding weights the caller already holds as
    bf16 values (same result, less work for large layers).
    """
    rnd = nv.bf16_round if dtype == "bf16" else (lambda a: np.asarray(a, np.float32))
    x = rnd(np.asarray(x, np.float32))
    S, H, dh = x.shape
    R = int(np.asarray(gather_ids).size)
    if R == 0:                                                     # mh_moe_fwd.py:257-258
        return np.zeros_like(x)
    if round_weights:
        Wg, Wu, Wd = (rnd(np.asarray(w, np.float32)) for w in (W_gate, W_up, W_down))
    else:
        Wg, Wu, Wd = W_gate, W_up, W_down
    expert, head = _row_meta(gather_ids, expert_offsets, H)
    tok = np.asarray(gather_ids, np.int64)
    p = np.asarray(probs, np.float32)
    y_rows = np.zeros((R, dh), np.float32)
    offs = np.asarray(expert_offsets, np.int64)
    for e in range(offs.size - 1):
        lo, hi = offs[e], offs[e + 1]
        if hi == lo:
            continue
        h = e // ((offs.size - 1) // H)
        xe = x[tok[lo:hi], h, :]
        ga = (xe @ Wg[e]).astype(np.float32)
        ua = (xe @ Wu[e]).astype(np.float32)
        hid = rnd(swiglu7(ga, ua))
        ya = (hid @ Wd[e]).astype(np.float32)
        y_rows[lo:hi] = rnd((ya * p[lo:hi, None]).astype(np.float32))
    y = np.zeros((S * H, dh), np.float32)
    _sequential_add(y, tok * H + head, y_rows, rnd)
    return y.reshape(S, H, dh)


def mh_moe_fwd_nvfp4_ref(x, gather_ids, probs, expert_offsets, gu_pack: dict, down_pack: dict,
                         return_hidden: bool = False):
    """NVFP4 twin of the FFN (the CUDA path's oracle).

    gu_pack / down_pack come from ``nvfp4_ref.pack_gate_up`` / ``pack_down``.
    Returns y [S,H,dh] as bf16-valued fp32 (and the per-row hidden codes/sf when asked).
    """
    x = nv.bf16_round(np.asarray(x, np.float32))
    S, H, dh = x.shape
    R = int(np.asarray(gather_ids).size)
    if R == 0:
        return np.zeros_like(x)
    offs = np.asarray(expert_offsets, np.int64)
    nflat = offs.size - 1
    de = gu_pack["de"]
    tok = np.asarray(gather_ids, np.int64)
    p = np.asarray(probs, np.float32)
    expert, head = _row_meta(gather_ids, expert_offsets, H)

    # x quantised once per (token, head) row: g_row = amax(row)/2688
    xc, xsf, xg = nv.quantize_rows(x.reshape(S * H, dh))
    x_deq = nv.dequantize(xc, xsf)                                   # without g
    gu_codes = nv.unpack_codes(gu_pack["data"])
    dn_codes = nv.unpack_codes(down_pack["data"])
    y_rows = np.zeros((R, dh), np.float32)
    hid_codes = np.zeros((R, de), np.uint8)
    hid_sf = np.zeros((R, de // 16), np.uint8)
    is_up = ((np.arange(2 * de) // 16) % 2).astype(bool)
    for e in range(nflat):
        lo, hi = offs[e], offs[e + 1]
        if hi == lo:
            continue
        h = e // (nflat // H)
        rows = tok[lo:hi] * H + h
        a = x_deq[rows].astype(np.float64)
        b = nv.dequantize(gu_codes[e], nv.atoms_to_sf(gu_pack["sf_atoms"][e], 2 * de, dh)).astype(np.float64)
        acc = (a @ b.T).astype(np.float32)                           # [n, 2de]
        s_gate = (xg[rows] * gu_pack["gscale_gate"][e]).astype(np.float32)
        s_up = (xg[rows] * gu_pack["gscale_up"][e]).astype(np.float32)
        scale = np.where(is_up[None, :], s_up[:, None], s_gate[:, None]).astype(np.float32)
        v = (acc * scale).astype(np.float32).reshape(-1, de // 16, 2, 16)
        hid = swiglu7(v[:, :, 0, :], v[:, :, 1, :]).reshape(-1, de)
        hc, hsf = nv.quantize_blocks(hid, nv.HIDDEN_GLOBAL)
        hid_codes[lo:hi], hid_sf[lo:hi] = hc, hsf
        ha = nv.dequantize(hc, hsf).astype(np.float64)
        wd = nv.dequantize(dn_codes[e], nv.atoms_to_sf(down_pack["sf_atoms"][e], dh, de)).astype(np.float64)
        acc2 = (ha @ wd.T).astype(np.float32)                        # [n, dh]
        s_dn = np.float32(nv.HIDDEN_GLOBAL * down_pack["gscale"][e])
        y_rows[lo:hi] = nv.bf16_round(((acc2 * s_dn).astype(np.float32) * p[lo:hi, None]).astype(np.float32))
    # combine: fp32 sum over each (token, head)'s rows in ascending sorted-row order
    y = np.zeros((S * H, dh), np.float32)
    _sequential_add(y, tok * H + head, y_rows, lambda a: np.asarray(a, np.float32))
    y = nv.bf16_round(y).reshape(S, H, dh)
    if return_hidden:
        return y, hid_codes, hid_sf
    return y


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def nvfp4_expert_rows_ref(codes, sf, g, expert, prob, gu_pack: dict, down_pack: dict) -> np.ndarray:
    """Per-row NVFP4 expert FFN on already-quantised rows (the expert-parallel receiver's
    work): codes [R, dh] E2M1 codes, sf [R, dh/16] E4M3 bytes, g [R] row scales, expert
    [R] index into the packs, prob [R].  Returns bf16-valued fp32 rows [R, dh] =
    bf16(down(swiglu7(gate/up)) * prob) — the rows ``mh_moe_fwd_nvfp4_ref`` combines."""
    codes = np.asarray(codes, np.uint8)
    R, dh = codes.shape
    de = gu_pack["de"]
    out = np.zeros((R, dh), np.float32)
    x_deq = nv.dequantize(codes, sf)
    is_up = ((np.arange(2 * de) // 16) % 2).astype(bool)
    gu_codes = nv.unpack_codes(gu_pack["data"])
    dn_codes = nv.unpack_codes(down_pack["data"])
    expert = np.asarray(expert, np.int64)
    for e in np.unique(expert):
        rows = np.nonzero(expert == e)[0]
        b = nv.dequantize(gu_codes[e], nv.atoms_to_sf(gu_pack["sf_atoms"][e], 2 * de, dh)).astype(np.float64)
        acc = (x_deq[rows].astype(np.float64) @ b.T).astype(np.float32)
        s_gate = (np.asarray(g, np.float32)[rows] * gu_pack["gscale_gate"][e]).astype(np.float32)
        s_up = (np.asarray(g, np.float32)[rows] * gu_pack["gscale_up"][e]).astype(np.float32)
        scale = np.where(is_up[None, :], s_up[:, None], s_gate[:, None]).astype(np.float32)
        v = (acc * scale).astype(np.float32).reshape(-1, de // 16, 2, 16)
        hid = swiglu7(v[:, :, 0, :], v[:, :, 1, :]).reshape(-1, de)
        hc, hsf = nv.quantize_blocks(hid, nv.HIDDEN_GLOBAL)
        ha = nv.dequantize(hc, hsf).astype(np.float64)
        wd = nv.dequantize(dn_codes[e], nv.atoms_to_sf(down_pack["sf_atoms"][e], dh, de)).astype(np.float64)
        acc2 = (ha @ wd.T).astype(np.float32)
        s_dn = np.float32(nv.HIDDEN_GLOBAL * down_pack["gscale"][e])
        out[rows] = nv.bf16_round(((acc2 * s_dn).astype(np.float32) *
                                   np.asarray(prob, np.float32)[rows, None]).astype(np.float32))
    return out


def slice_packs(gu_pack: dict, down_pack: dict, lo: int, hi: int) -> tuple[dict, dict]:
    """Expert slice [lo, hi) of packed weights (an EP rank's shard)."""
    gu = dict(gu_pack)
    dn = dict(down_pack)
    for k in ("data", "sf_atoms", "gscale_gate", "gscale_up"):
        gu[k] = gu_pack[k][lo:hi]
    for k in ("data", "sf_atoms", "gscale"):
        dn[k] = down_pack[k][lo:hi]
    return gu, dn
