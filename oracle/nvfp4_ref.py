"""CPU NVFP4 codec — test infrastructure (the checker, never the product path).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this module.  The CUDA kernels under ``magi-2-preview_b200/csrc`` never call it.

Parity status: **unpinned with respect to the reference.**  The reference
(``inference/flash_mh_moe``) has no NVFP4 code at all — its experts are bf16
(``inference/model/magi2_preview.py:2547-2570``).  This file is the written
definition of the packed format the CUDA packer/quantisers must reproduce bit
for bit.  It restates NVIDIA's public NVFP4 definition:

* element: E2M1 (1 sign, 2 exponent, 1 mantissa bit), grid {0, .5, 1, 1.5, 2, 3, 4, 6};
* block scale: one unsigned E4M3 byte per 16 consecutive elements along K;
* second-level scale: one fp32 ``g`` per matrix (weights: per expert matrix;
  activations: per routed row; SwiGLU hidden: the static bound 56/2688);
* value = e2m1(code) * e4m3(scale) * g.

Exact fp32 operation sequence for one 16-element block ``v`` (every op IEEE
round-to-nearest-even, no FMA contraction — the CUDA side uses ``__fmul_rn`` /
``__fdiv_rn``):

    amax  = max_i |v_i|
    t     = amax / (6 * g)                       # fp32 mul, then fp32 div
    sf    = E4M3_RNE_SATFINITE(t)                # byte; sfv = decode(sf)
    inv   = 1 / (sfv * g)                        # fp32 mul, then fp32 div
    q_i   = E2M1_RNE_SATFINITE(v_i * inv)        # fp32 mul, then RNE to the grid
    if sfv == 0: every q_i = +0 (code 0)

Second-level scales: ``g = amax_matrix / 2688`` (fp32 div; 2688 = 6 * 448), or
1.0 when the matrix is all zero.  Packing: byte = code[2j] | code[2j+1] << 4
(low nibble = even k).  Negative values keep the sign bit (−0 encodes as 0x8),
as IEEE-style conversions do.

Scale-factor tile layout ("SF atoms", consumed by the tcgen05 block-scaled MMA
through ``tcgen05.cp ... 32x128b.warpx4``): rows are grouped by 128 and scale
columns by 4 (= 64 elements of K).  One atom is 512 contiguous bytes; inside it
row ``m`` (0..127) and scale column ``c`` (0..3) sit at byte
``(m % 32) * 16 + (m // 32) * 4 + c``.  Atoms are ordered K-fastest:
``atom(mb, kb) = (mb * (K // 64) + kb) * 512``.
"""
from __future__ import annotations

import numpy as np

E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E4M3_MAX = np.float32(448.0)
SF_DIVISOR = np.float32(2688.0)          # 6 * 448
HIDDEN_BOUND = np.float32(56.0)          # |swiglu7(g, u)| <= 7 * 8
HIDDEN_GLOBAL = np.float32(HIDDEN_BOUND / SF_DIVISOR)


def f32(x):
    return np.asarray(x, dtype=np.float32)


# ───────────────────────────── scalar format codecs ─────────────────────────────

def e2m1_encode(x: np.ndarray) -> np.ndarray:
    """Round fp32 to E2M1 codes (RNE, saturating to ±6). Returns uint8 codes 0..15."""
    x = f32(x)
    a = np.abs(x)
    # RNE on the grid: ties go to the code whose mantissa bit is 0 (0, 1, 2, 4).
    mag = np.where(a <= 0.25, 0,
          np.where(a < 0.75, 1,
          np.where(a <= 1.25, 2,
          np.where(a < 1.75, 3,
          np.where(a <= 2.5, 4,
          np.where(a < 3.5, 5,
          np.where(a <= 5.0, 6, 7))))))).astype(np.uint8)
    sign = np.signbit(x).astype(np.uint8) << 3
    return (mag | sign).astype(np.uint8)


def e2m1_decode(code: np.ndarray) -> np.ndarray:
    code = np.asarray(code, dtype=np.uint8)
    mag = E2M1_GRID[code & 7]
    return np.where(code & 8, -mag, mag).astype(np.float32)


def e4m3_encode(t: np.ndarray) -> np.ndarray:
    """Round non-negative fp32 to unsigned E4M3 bytes (RNE, saturating at 448)."""
    t = f32(t)
    if np.any(t < 0) or np.any(np.isnan(t)):
        raise ValueError("e4m3_encode expects finite non-negative inputs")
    t = np.minimum(t, E4M3_MAX)
    out = np.zeros(t.shape, dtype=np.uint8)
    sub = t < np.float32(2.0 ** -6)
    # subnormal range: step 2^-9; t * 512 is exact in fp32, rint is RNE
    qs = np.rint(t[sub] * np.float32(512.0)).astype(np.int32)     # 0..8; 8 == 2^-6 == code 0x08
    out[sub] = qs.astype(np.uint8)
    tn = t[~sub]
    if tn.size:
        e = np.floor(np.log2(tn)).astype(np.int32)
        # guard log2 rounding at exact binade edges
        e = np.where(np.ldexp(np.float32(1.0), e) > tn, e - 1, e)
        e = np.where(np.ldexp(np.float32(1.0), e + 1) <= tn, e + 1, e)
        step = np.ldexp(np.float32(1.0), e - 3).astype(np.float32)
        q = np.rint(tn / step).astype(np.int32)                     # 8..16, exact division by 2^k
        e = np.where(q == 16, e + 1, e)
        q = np.where(q == 16, 8, q)
        code = ((e + 7) << 3) | (q - 8)
        code = np.minimum(code, 0x7E)                               # 448
        out[~sub] = code.astype(np.uint8)
    return out


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int32)
    e = (b >> 3) & 0xF
    m = b & 7
    sub = np.ldexp(m.astype(np.float32), -9)
    nor = np.ldexp((8 + m).astype(np.float32), e - 10)
    return np.where(e == 0, sub, nor).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (RNE), returned as fp32 values."""
    x = np.ascontiguousarray(f32(x))
    u = x.view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)   # wraps only for NaN payloads
    return np.where(np.isnan(x), x, out).astype(np.float32)


# ───────────────────────────── block quantisation ─────────────────────────────

def global_scale(amax) -> np.float32:
    """Second-level fp32 scale g = amax / 2688 (1.0 for an all-zero matrix)."""
    amax = f32(amax)
    g = (amax / SF_DIVISOR).astype(np.float32)
    return np.where(amax > 0, g, np.float32(1.0)).astype(np.float32)


def quantize_blocks(v: np.ndarray, g) -> tuple[np.ndarray, np.ndarray]:
    """Quantise rows of ``v`` ([..., K], K % 16 == 0) with per-row-broadcast scale ``g``.

    ``g`` broadcasts against ``v[..., 0]``.  Returns (codes uint8 [..., K],
    sf bytes uint8 [..., K/16]).
    """
    v = f32(v)
    K = v.shape[-1]
    assert K % 16 == 0
    g = np.broadcast_to(f32(g), v.shape[:-1])[..., None]            # [..., 1]
    blk = v.reshape(*v.shape[:-1], K // 16, 16)
    amax = np.abs(blk).max(axis=-1)                                 # [..., K/16]
    t = (amax / (np.float32(6.0) * g).astype(np.float32)).astype(np.float32)
    sf = e4m3_encode(t)
    sfv = e4m3_decode(sf)
    denom = (sfv * g).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(sfv > 0, (np.float32(1.0) / np.where(sfv > 0, denom, 1)).astype(np.float32),
                       np.float32(0.0)).astype(np.float32)
    scaled = (blk * inv[..., None]).astype(np.float32)
    codes = e2m1_encode(scaled)
    codes = np.where((sfv > 0)[..., None], codes, np.uint8(0)).astype(np.uint8)
    return codes.reshape(v.shape), sf


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """[..., K] 4-bit codes -> [..., K/2] bytes, low nibble = even k."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_codes(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def dequantize(codes: np.ndarray, sf: np.ndarray, g=None) -> np.ndarray:
    """codes [..., K], sf [..., K/16] -> fp32 values (times g if given)."""
    vals = e2m1_decode(codes)
    K = vals.shape[-1]
    sfv = e4m3_decode(sf)
    out = (vals.reshape(*vals.shape[:-1], K // 16, 16) * sfv[..., None]).astype(np.float32)
    out = out.reshape(vals.shape)
    if g is not None:
        out = (out * np.broadcast_to(f32(g), out.shape[:-1])[..., None]).astype(np.float32)
    return out


# ───────────────────────────── SF atom layout ─────────────────────────────

def sf_atom_offset(rows: np.ndarray, sfcol: np.ndarray, K: int) -> np.ndarray:
    """Byte offset of scale (row, sf column) inside the SF-atom layout of a [*, K] matrix."""
    rows = np.asarray(rows, dtype=np.int64)
    sfcol = np.asarray(sfcol, dtype=np.int64)
    kb_per_row = K // 64
    atom = (rows // 128) * kb_per_row + sfcol // 4
    m = rows % 128
    return atom * 512 + (m % 32) * 16 + (m // 32) * 4 + (sfcol % 4)


def sf_to_atoms(sf: np.ndarray) -> np.ndarray:
    """[M, K/16] row-major scale bytes -> flat atom-layout bytes (M padded to 128, K/16 to 4)."""
    M, nsf = sf.shape
    assert nsf % 4 == 0, "K must be a multiple of 64"
    K = nsf * 16
    Mp = (M + 127) // 128 * 128
    out = np.zeros(Mp * nsf, dtype=np.uint8)
    r, c = np.meshgrid(np.arange(M), np.arange(nsf), indexing="ij")
    out[sf_atom_offset(r, c, K)] = sf
    return out


def atoms_to_sf(atoms: np.ndarray, M: int, K: int) -> np.ndarray:
    nsf = K // 16
    r, c = np.meshgrid(np.arange(M), np.arange(nsf), indexing="ij")
    return np.asarray(atoms, dtype=np.uint8)[sf_atom_offset(r, c, K)]


# ───────────────────────────── weight packing ─────────────────────────────

def pack_weight_nk(w_nk: np.ndarray) -> dict:
    """Pack one stack of K-major matrices ``w_nk`` [E, N, K] (fp32) to NVFP4.

    Returns dict(data uint8 [E, N, K/2], sf_atoms uint8 [E, N*K/16] (atom layout
    per expert), gscale fp32 [E]).
    """
    w = f32(w_nk)
    E, N, K = w.shape
    assert N % 128 == 0 and K % 64 == 0
    amax = np.abs(w.reshape(E, -1)).max(axis=1)
    g = global_scale(amax)                                          # [E]
    codes, sf = quantize_blocks(w, g[:, None])                      # sf [E, N, K/16]
    data = pack_codes(codes)
    atoms = np.stack([sf_to_atoms(sf[e]) for e in range(E)])
    return {"data": data, "sf_atoms": atoms, "gscale": g.astype(np.float32)}


def interleave_gate_up(w_gate_kn: np.ndarray, w_up_kn: np.ndarray) -> np.ndarray:
    """Reference-layout gate/up weights [E, K=dh, N=de] -> fused K-major [E, 2*de, dh].

    Rows are interleaved in groups of 16: for hidden column block j the fused rows
    32j..32j+15 are gate columns 16j..16j+15 and rows 32j+16..32j+31 the matching
    up columns, so one 32-column accumulator chunk yields one 16-wide hidden block.
    """
    wg = np.swapaxes(f32(w_gate_kn), 1, 2)      # [E, de, dh]
    wu = np.swapaxes(f32(w_up_kn), 1, 2)
    E, de, dh = wg.shape
    assert de % 16 == 0
    out = np.empty((E, de // 16, 2, 16, dh), dtype=np.float32)
    out[:, :, 0] = wg.reshape(E, de // 16, 16, dh)
    out[:, :, 1] = wu.reshape(E, de // 16, 16, dh)
    return out.reshape(E, 2 * de, dh)


def pack_gate_up(w_gate_kn: np.ndarray, w_up_kn: np.ndarray) -> dict:
    """NVFP4 pack of the fused gate/up operand; gate and up keep separate per-expert scales."""
    fused = interleave_gate_up(w_gate_kn, w_up_kn)
    E, N2, K = fused.shape
    de = N2 // 2
    g_gate = global_scale(np.abs(f32(w_gate_kn).reshape(E, -1)).max(axis=1))
    g_up = global_scale(np.abs(f32(w_up_kn).reshape(E, -1)).max(axis=1))
    # per fused row: the scale of the matrix the row came from
    is_up = ((np.arange(N2) // 16) % 2).astype(bool)
    g_rows = np.where(is_up[None, :], g_up[:, None], g_gate[:, None]).astype(np.float32)  # [E, 2de]
    codes, sf = quantize_blocks(fused, g_rows)
    data = pack_codes(codes)
    atoms = np.stack([sf_to_atoms(sf[e]) for e in range(E)])
    return {"data": data, "sf_atoms": atoms, "gscale_gate": g_gate, "gscale_up": g_up,
            "N": N2, "K": K, "de": de}


def pack_down(w_down_kn: np.ndarray) -> dict:
    """Reference-layout down weights [E, K=de, N=dh] -> NVFP4 of the K-major [E, dh, de]."""
    wd = np.swapaxes(f32(w_down_kn), 1, 2)      # [E, dh, de]
    p = pack_weight_nk(wd)
    p["N"], p["K"] = wd.shape[1], wd.shape[2]
    return p


def dequant_gate_up(p: dict) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of pack_gate_up: returns (W_gate, W_up) in reference layout [E, dh, de], fp32."""
    data, atoms = p["data"], p["sf_atoms"]
    E, N2, Kh = data.shape
    K = Kh * 2
    de = N2 // 2
    codes = unpack_codes(data)
    vals = np.stack([dequantize(codes[e], atoms_to_sf(atoms[e], N2, K)) for e in range(E)])
    vals = vals.reshape(E, de // 16, 2, 16, K)
    wg = vals[:, :, 0].reshape(E, de, K) * p["gscale_gate"][:, None, None]
    wu = vals[:, :, 1].reshape(E, de, K) * p["gscale_up"][:, None, None]
    return (np.swapaxes(wg, 1, 2).astype(np.float32), np.swapaxes(wu, 1, 2).astype(np.float32))


def dequant_down(p: dict) -> np.ndarray:
    data, atoms = p["data"], p["sf_atoms"]
    E, N, Kh = data.shape
    K = Kh * 2
    codes = unpack_codes(data)
    vals = np.stack([dequantize(codes[e], atoms_to_sf(atoms[e], N, K)) for e in range(E)])
    vals = vals * p["gscale"][:, None, None]
    return np.swapaxes(vals, 1, 2).astype(np.float32)


def quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-row NVFP4 of activations x [M, K]: g_row = amax(row)/2688.

    Returns (codes [M, K], sf [M, K/16], g [M]).
    """
    x = f32(x)
    g = global_scale(np.abs(x).max(axis=1))
    codes, sf = quantize_blocks(x, g)
    return codes, sf, g
