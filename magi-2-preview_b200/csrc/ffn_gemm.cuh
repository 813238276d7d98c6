// Block-scaled NVFP4 grouped GEMM for the MoE expert FFN (sm_100a, tcgen05).
//
// One persistent CTA per SM walks (m-tile, n-tile) work items of the grouped
// problem.  A m-tile is 128 consecutive rows of the expert-padded row space (every
// expert's rows start on a 128-row boundary); its expert comes from `tile_expert`.
//
//   D[128 x 256] (fp32, TMEM) = sum_k (A[128 x k] .* SFA) (B_e[256 x k] .* SFB)^T
//
// Warp roles (3 + EPW warps: EPW = 16 epilogue warps for the SwiGLU epilogue at K <= 1024,
// else 8):
//   warp 0      TMA producer into a 4-stage (EPI_DOWN: 3-stage) shared-memory ring, one
//               stage = 256 K-elements: A tile (128 x 256 FP4 = 16 KB) and B tile
//               (256 x 256 FP4 = 32 KB), 128-B swizzle, plus their UE4M3 scale atoms
//               (2 KB + 4 KB, untiled bulk copies).  The whole warp waits; lane 0 issues.
//   warp 1      TMEM owner + MMA issuer: per stage, once the stage's scale factors are in
//               TMEM, issues 4 x tcgen05.mma kind::mxf4nvf4 block16 (M128 N256 K64).
//   warps 2..    epilogue: drain the accumulator with tcgen05.ld into registers,
//               release TMEM, then apply the fused epilogue and store.  Warp w reads TMEM
//               lane quarter w % 4 and a 1024/EPW-column slice of the accumulator.  The
//               SwiGLU epilogue's arithmetic per accumulator element is several times the
//               MMA's at small K (d_head 256: one 256-K stage per tile), so there it
//               gets 16 warps.
//   last warp   scale-factor copier: per stage copies the 12 scale atoms into TMEM
//               (tcgen05.cp 32x128b.warpx4) and commits to the stage's sf-full barrier.
//               The copies cost the tcgen05 pipe more than the MMAs do; issued from their
//               own warp they run ahead of and beside the MMAs instead of between them.
//
// Ordering: the copier overwrites TMEM scale slot s only after full[s] of the next round,
// which the producer posts only after empty[s], which the MMA warp commits after the MMAs
// that read slot s; the MMA warp's empty[s] commit follows its wait on sf-full[s], so the
// copies' shared-memory reads are done before the stage is refilled.
//
// TMEM columns: [0,256) accumulator, [256 + 48*s, 256 + 48*(s+1)) the scale
// factors of stage s (16 columns SFA = 4 MMAs x 4, 32 columns SFB = 4 MMAs x 8).
//
// Epilogues:
//   EPI_SWIGLU  B = fused gate/up rows (interleaved by 16).  Each 32-column chunk
//               gives 16 hidden values: h = swiglu7(acc_g * s_gate, acc_u * s_up),
//               quantised to NVFP4 with the static hidden scale and written as the
//               A operand (data + SF atoms) of the down GEMM.
//   EPI_DOWN    bf16(acc * s_down * prob) staged in swizzled shared memory and written
//               with TMA stores into the padded partial buffer P[rows_pad, N].
//   EPI_DOWN_ATOMIC  the same bf16(acc * s_down * prob) values added into y[token, head]
//               with bf16 vector atomics (the reference's default, non-deterministic
//               scatter): no partial buffer, no combine pass.
//   EPI_RAW     fp32 accumulator written as is (verification only).
#pragma once

#include "mhmoe_common.cuh"

namespace mhmoe {

enum { EPI_SWIGLU = 0, EPI_DOWN = 1, EPI_RAW = 2, EPI_DOWN_ATOMIC = 3 };

constexpr int GEMM_BM = 128;
constexpr int GEMM_BN = 256;
constexpr int GEMM_BK = 256;          // FP4 elements per stage = 128 bytes per row
constexpr int GEMM_THREADS = 352;          // single-CTA kernel, 8 epilogue warps: warps 0-9 + the copier
constexpr int GEMMP_THREADS = 352;         // CTA-pair kernel: warps 0-9 + the leader's scale-factor copier
constexpr int GEMM_A_BYTES = GEMM_BM * GEMM_BK / 2;          // 16384
constexpr int GEMM_B_BYTES = GEMM_BN * GEMM_BK / 2;          // 32768
constexpr int GEMM_SFA_BYTES = GEMM_BM * GEMM_BK / 16;       // 2048
constexpr int GEMM_SFB_BYTES = GEMM_BN * GEMM_BK / 16;       // 4096
constexpr int GEMM_STAGE_TX = GEMM_A_BYTES + GEMM_B_BYTES + GEMM_SFA_BYTES + GEMM_SFB_BYTES;
constexpr int GEMM_STAGE_BYTES = GEMM_STAGE_TX;
constexpr int GEMM_STG_BYTES = 8 * 32 * 128;                 // EPI_DOWN: 4 KB store staging per epilogue warp
constexpr int GEMM_MISC_BYTES = 256 + 512;                    // mbarriers + TMEM slot, then the 128-float table
constexpr int GEMM_TMEM_COLS = 512;
constexpr int GEMM_SF_COL0 = 256;
constexpr int GEMM_SF_COLS_PER_STAGE = 48;

__host__ __device__ constexpr int gemm_stages(int epi) { return epi == EPI_DOWN ? 3 : 4; }
// Epilogue warps (a multiple of 4: each lane quarter of TMEM is read by EPW/4 warps): 16 for
// the SwiGLU epilogue when the reduction is short (K <= 1024: few MMAs per tile to hide the
// epilogue behind), else 8.
__host__ __device__ constexpr int gemm_epi_warps(int epi, int K) {
  return epi == EPI_SWIGLU && K <= 1024 ? 16 : 8;
}
__host__ __device__ constexpr int gemm_stg_bytes(int epi) { return epi == EPI_DOWN ? GEMM_STG_BYTES : 0; }
__host__ __device__ constexpr int gemm_smem_bytes(int epi) {
  return gemm_stages(epi) * GEMM_STAGE_BYTES + gemm_stg_bytes(epi) + GEMM_MISC_BYTES + 1024;
}

// CTA-pair variant (cluster of 2, cta_group::2): M = 256 rows per pair (128 per CTA), each
// CTA stages its own A rows, HALF of the 256-row B tile and the full B scale factors, so
// B crosses L2 -> SM once per pair instead of once per CTA.
constexpr int GEMMP_B_BYTES = (GEMM_BN / 2) * GEMM_BK / 2;    // 16384
constexpr int GEMMP_STAGE_TX = GEMM_A_BYTES + GEMMP_B_BYTES + GEMM_SFA_BYTES + GEMM_SFB_BYTES;   // per CTA
constexpr int GEMMP_STAGE_BYTES = GEMMP_STAGE_TX;
__host__ __device__ constexpr int gemmp_stages(int epi) { return epi == EPI_DOWN ? 4 : 5; }
__host__ __device__ constexpr int gemmp_smem_bytes(int epi) {
  return gemmp_stages(epi) * GEMMP_STAGE_BYTES + (epi == EPI_DOWN ? GEMM_STG_BYTES : 0) + GEMM_MISC_BYTES + 1024;
}

// Static second-level scale of the SwiGLU7 hidden: |swiglu7| <= 7 * 8 = 56, 56 / 2688.
constexpr float HIDDEN_GSCALE = 56.0f / 2688.0f;

struct FfnGemmParams {
  const uint8_t* sfa;        // A scale atoms (tiled A modes)
  const uint8_t* sfb;        // B scale atoms, per expert contiguous: N*K/16 bytes each
  const int* n_mtiles_dev;   // device scalar: number of valid m-tiles (or nullptr)
  int n_mtiles_host;         // m-tiles the buffers hold (caps n_mtiles_dev)
  const int* tile_expert;    // [m-tile] -> flattened expert id
  const int* tile_row0;      // [m-tile] -> first sorted row
  const int* tile_rows;      // [m-tile] -> valid rows in the tile
  int K;                     // reduction length in elements
  int N;                     // B rows per expert
  // EPI_SWIGLU
  const float* row_gscale;   // [128 * n_mtiles] second-level scale of each A row
  const float* gs_gate;      // [n_experts]
  const float* gs_up;        // [n_experts]
  uint8_t* h_data;           // [128 * n_mtiles, N/4]  (hidden has N/2 columns, 2 per byte)
  uint8_t* h_sf;             // SF atoms of the hidden, K_hidden = N/2
  // EPI_DOWN, EPI_DOWN_ATOMIC
  const float* probs;        // [R] sorted probs
  const float* gs_down;      // [n_experts]
  // EPI_DOWN_ATOMIC
  __nv_bfloat16* y;          // [S, H, N] (strides sy_s, sy_h; unit inner stride), zeroed before
  int64_t sy_s, sy_h;
  const int32_t* gather_ids; // [R] sorted row -> token
  int experts_per_head;
  // EPI_RAW
  float* out_f32;            // [128 * n_mtiles, N]
  int* status;
  uint64_t timeout_ns;
};

// SwiGLU7 of two (gate, up) pairs at once: min(g, 7) * sigmoid(1.702 min(g, 7)) *
// (clamp(u, -7, 7) + 1).  sigmoid(1.702 g) = 1 / (1 + 2^(g * -1.702 log2(e))): one scaled
// 2^x and one reciprocal from the special-function unit, the products and sums as
// two-lane fp32 (rounded like the scalar sequence (g * sig) * (u + 1)).
constexpr float SWIGLU7_NEG_ALPHA_LOG2E = -1.702f * 1.44269504088896341f;
__device__ __forceinline__ uint64_t swiglu7_x2(uint64_t g2, uint64_t u2) {
  float g0, g1, u0, u1;
  f2_unpack(g2, g0, g1);
  f2_unpack(u2, u0, u1);
  g0 = fminf(g0, 7.0f);
  g1 = fminf(g1, 7.0f);
  u0 = fminf(fmaxf(u0, -7.0f), 7.0f);
  u1 = fminf(fmaxf(u1, -7.0f), 7.0f);
  const uint64_t gc = f2_pack(g0, g1);
  float a0, a1;
  f2_unpack(f2_mul(gc, f2_pack(SWIGLU7_NEG_ALPHA_LOG2E, SWIGLU7_NEG_ALPHA_LOG2E)), a0, a1);
  float d0, d1;
  f2_unpack(f2_add(f2_pack(ex2_approx(a0), ex2_approx(a1)), f2_pack(1.0f, 1.0f)), d0, d1);
  const uint64_t gs = f2_mul(gc, f2_pack(rcp_approx(d0), rcp_approx(d1)));
  return f2_mul(gs, f2_add(f2_pack(u0, u1), f2_pack(1.0f, 1.0f)));
}

// 1 / (e4m3(sf) * HIDDEN_GSCALE) for every E4M3 scale byte (0 for sf = 0): the per-block
// factor of the hidden's quantisation, filled once per CTA into a 128-entry table.
__device__ __forceinline__ float hidden_inv_scale(uint32_t sf) {
  return sf ? __fdiv_rn(1.0f, __fmul_rn(e4m3_to_f32(sf), HIDDEN_GSCALE)) : 0.0f;
}

// NVFP4 quantisation of 16 hidden values (8 pairs) with the static second-level scale,
// the same results as quant_block16(v, HIDDEN_GSCALE): there the block scale is
// amax / (6 * HIDDEN_GSCALE), and 6 * HIDDEN_GSCALE rounds to exactly 0.125 in fp32, so the
// division is the exact amax * 8; the reciprocal comes from the table.
__device__ __forceinline__ uint32_t quant_hidden16(const uint64_t (&h2)[8], const float* inv_tab, uint32_t out[2]) {
  float h[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) f2_unpack(h2[i], h[2 * i], h[2 * i + 1]);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(h[i]));
  const uint32_t sf = cvt_e4m3(amax * 8.0f);
  const float inv = inv_tab[sf];
  const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    float s[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) f2_unpack(f2_mul(h2[4 * w + i], inv2), s[2 * i], s[2 * i + 1]);
    const uint32_t word = cvt_e2m1x8(s[0], s[1], s[2], s[3], s[4], s[5], s[6], s[7]);
    out[w] = sf ? word : 0u;
  }
  return sf;
}

// Per-tile scalars of one epilogue thread (row m of m-tile mt), loaded ahead of their use
// in two steps so that no load waits on another inside the tile loop: the loads indexed by
// the tile alone (expert, row scale, row range) two tiles ahead, the loads indexed by
// those (per-expert scales, probabilities) one tile ahead.  Products are formed at use.
struct EpiIndex {
  float gr;           // SwiGLU: second-level scale of the A row
  int e, rows, row0;  // expert; down: valid rows and first sorted row of the tile
};
struct EpiScalars {
  float gr, s0, s1;   // SwiGLU: row scale, gate / up weight scales; down: s0 = weight scale
  float pr;           // down: routing probability of the row
  int64_t tok;        // atomic scatter: token of the row
  int e, rows;
};

template <int EPI>
__device__ __forceinline__ EpiIndex epi_load_index(const FfnGemmParams& p, int mt, int m) {
  EpiIndex x{};
  x.e = p.tile_expert[mt];
  if constexpr (EPI == EPI_SWIGLU) {
    x.gr = p.row_gscale[(size_t)mt * GEMM_BM + m];
  } else if constexpr (EPI == EPI_DOWN || EPI == EPI_DOWN_ATOMIC) {
    x.rows = p.tile_rows[mt];
    x.row0 = p.tile_row0[mt];
  }
  return x;
}

template <int EPI>
__device__ __forceinline__ EpiScalars epi_load_scalars(const FfnGemmParams& p, const EpiIndex& x, int m) {
  EpiScalars v{};
  v.e = x.e;
  if constexpr (EPI == EPI_SWIGLU) {
    v.gr = x.gr;
    v.s0 = p.gs_gate[x.e];
    v.s1 = p.gs_up[x.e];
  } else if constexpr (EPI == EPI_DOWN || EPI == EPI_DOWN_ATOMIC) {
    v.rows = x.rows;
    v.s0 = p.gs_down[x.e];
    const bool valid = m < x.rows;
    const int64_t srow = (int64_t)x.row0 + m;
    v.pr = valid ? p.probs[srow] : 0.0f;
    if constexpr (EPI == EPI_DOWN_ATOMIC) v.tok = valid ? p.gather_ids[srow] : 0;
  }
  return v;
}

// The two-step prefetch of one epilogue thread over the tiles t0, t0 + step, ... (m-tile of
// tile t: mtile_of(t)).  next() returns the scalars of the current tile and issues the loads
// of the following two.
template <int EPI, class MtileOf>
struct EpiPrefetch {
  EpiScalars cur;
  EpiIndex ahead;     // index loads of the tile after the next
  __device__ __forceinline__ EpiPrefetch(const FfnGemmParams& p, MtileOf mtile_of, int t0, int step, int total, int m) {
    cur = EpiScalars{};
    ahead = EpiIndex{};
    if (t0 < total) cur = epi_load_scalars<EPI>(p, epi_load_index<EPI>(p, mtile_of(t0), m), m);
    if (t0 + step < total) ahead = epi_load_index<EPI>(p, mtile_of(t0 + step), m);
  }
  __device__ __forceinline__ EpiScalars next(const FfnGemmParams& p, MtileOf mtile_of, int t, int step, int total, int m) {
    const EpiScalars v = cur;
    if (t + step < total) cur = epi_load_scalars<EPI>(p, ahead, m);
    if (t + 2 * step < total) ahead = epi_load_index<EPI>(p, mtile_of(t + 2 * step), m);
    return v;
  }
};

// Fused epilogue of one 128 x 256 accumulator tile for one thread: row m of m-tile mt,
// accumulator columns [NCOL*half, NCOL*half + NCOL) already in registers (r), TMEM released,
// per-tile scalars in v.  stg: this warp's 4 KB store staging (EPI_DOWN); inv_tab: the
// hidden's reciprocal block scales (EPI_SWIGLU, hidden_inv_scale, in shared memory).
template <int EPI, int NCOL>
__device__ __forceinline__ void gemm_epilogue_tile(const FfnGemmParams& p, const CUtensorMap* tmC,
                                                   const uint32_t (&r)[NCOL], const EpiScalars& v, int mt, int nt,
                                                   int m, int q, int half, int lane, uint8_t* stg,
                                                   const float* inv_tab) {
  const int e = v.e;
  const size_t prow = (size_t)mt * GEMM_BM + m;   // padded row
  if constexpr (EPI == EPI_SWIGLU) {
    const float s_gate = __fmul_rn(v.gr, v.s0), s_up = __fmul_rn(v.gr, v.s1);
    const uint64_t s_gate2 = f2_pack(s_gate, s_gate);
    const uint64_t s_up2 = f2_pack(s_up, s_up);
    const int hid_cols = p.N / 2;
    constexpr int NB = NCOL / 32;            // SwiGLU blocks: 16 gate + 16 up columns -> 16 hidden
    uint32_t words[2 * NB];
    uint32_t sfw = 0;
#pragma unroll
    for (int c = 0; c < NB; ++c) {
      uint64_t h2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t* rg = r + c * 32 + 2 * i;
        const uint64_t g2 = f2_mul(f2_pack(__uint_as_float(rg[0]), __uint_as_float(rg[1])), s_gate2);
        const uint64_t u2 = f2_mul(f2_pack(__uint_as_float(rg[16]), __uint_as_float(rg[17])), s_up2);
        h2[i] = swiglu7_x2(g2, u2);
      }
      uint32_t w2[2];
      const uint32_t sf = quant_hidden16(h2, inv_tab, w2);
      words[2 * c] = w2[0];
      words[2 * c + 1] = w2[1];
      sfw |= sf << (8 * c);
    }
    const int hcol0 = nt * (GEMM_BN / 2) + half * (NCOL / 2);  // first hidden column of this thread
    uint4* dst = reinterpret_cast<uint4*>(p.h_data + prow * (size_t)(hid_cols / 2) + hcol0 / 2);
#pragma unroll
    for (int v = 0; v < NB / 2; ++v)
      dst[v] = make_uint4(words[4 * v], words[4 * v + 1], words[4 * v + 2], words[4 * v + 3]);
    uint8_t* sfd = p.h_sf + sf_atom_offset(prow, (uint32_t)(hcol0 / 16), (uint32_t)hid_cols);
    if constexpr (NB == 4)
      *reinterpret_cast<uint32_t*>(sfd) = sfw;
    else
      *reinterpret_cast<uint16_t*>(sfd) = (uint16_t)sfw;
  } else if constexpr (EPI == EPI_DOWN) {
    // this warp's 32 rows are all expert padding: nothing reads them, store nothing
    if (q * 32 >= v.rows) return;
    const float s = __fmul_rn(HIDDEN_GSCALE, v.s0);
    const uint64_t s2 = f2_pack(s, s);
    const uint64_t pr2 = f2_pack(v.pr, v.pr);
    const uint32_t stg_s = smem_u32(stg);
#pragma unroll
    for (int box = 0; box < 2; ++box) {
      // the previous box's TMA store must have finished reading the staging buffer
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) {            // 16-B chunk c of this row: columns box*64 + 8c .. +7
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = box * 64 + c * 8 + 2 * j;
          float a, b;   // (acc * s) * prob, rounded per step
          f2_unpack(f2_mul(f2_mul(f2_pack(__uint_as_float(r[col]), __uint_as_float(r[col + 1])), s2), pr2), a, b);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
          w[j] = *reinterpret_cast<uint32_t*>(&h2);
        }
        // 128-B swizzle: chunk c of row `lane` sits at chunk c ^ (lane & 7)
        *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, stg_s, nt * GEMM_BN + half * 128 + box * 64, mt * GEMM_BM + q * 32);
        bulk_commit();
      }
    }
  } else if constexpr (EPI == EPI_DOWN_ATOMIC) {
    if (m < v.rows) {
      const float s = __fmul_rn(HIDDEN_GSCALE, v.s0);
      const float pr = v.pr;
      const int64_t tok = v.tok;
      const int h = e / p.experts_per_head;
      __nv_bfloat16* yrow = p.y + tok * p.sy_s + (int64_t)h * p.sy_h + nt * GEMM_BN + half * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {           // 8 columns (16 B) per vector atomic
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = c * 8 + 2 * j;
          const float a = __fmul_rn(__fmul_rn(__uint_as_float(r[col]), s), pr);
          const float b = __fmul_rn(__fmul_rn(__uint_as_float(r[col + 1]), s), pr);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
          w[j] = *reinterpret_cast<uint32_t*>(&h2);
        }
        red_add_bf16x8(yrow + c * 8, w);
      }
    }
  } else {
    float4* dst = reinterpret_cast<float4*>(p.out_f32 + prow * (size_t)p.N + nt * GEMM_BN + half * 128);
#pragma unroll
    for (int v = 0; v < 32; ++v)
      dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                           __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
  }
}

// tmA: grouped A operand [128 * n_mtiles, K/2], box 128 x 128.
// tmB: B operand [n_experts * N, K/2], box 128 x 256.
// tmC: EPI_DOWN -> P [128 * n_mtiles, N] bf16, box 64 x 32 (store); unused otherwise.
template <int EPI, int EPW>
__global__ void __launch_bounds__(32 * (3 + EPW), 1)
    ffn_gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, const FfnGemmParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int STAGES = gemm_stages(EPI);
  static_assert(EPW == 8 || (EPW == 16 && EPI == EPI_SWIGLU), "16 epilogue warps: SwiGLU epilogue only");
  constexpr int NCOL = 4 * GEMM_BN / EPW;           // accumulator columns per epilogue thread
  constexpr int COPIER = 2 + EPW;                   // warp index of the scale-factor copier
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * GEMM_A_BYTES;
  uint8_t* sSFA = sB + STAGES * GEMM_B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * GEMM_SFA_BYTES;
  uint8_t* sSTG = sSFB + STAGES * GEMM_SFB_BYTES;                     // store staging (1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSTG + gemm_stg_bytes(EPI));
  uint64_t* full_bar = bars;                       // [STAGES]
  uint64_t* empty_bar = bars + STAGES;             // [STAGES]
  uint64_t* tfull_bar = bars + 2 * STAGES;         // accumulator ready
  uint64_t* tempty_bar = tfull_bar + 1;            // accumulator drained
  uint64_t* drain_bar = tfull_bar + 2;             // all issued tcgen05 ops retired
  uint64_t* sff_bar = tfull_bar + 3;               // [STAGES] scale factors of the stage in TMEM
  uint64_t* drain2_bar = sff_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain2_bar + 1);
  float* sInv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [128] hidden_inv_scale

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (EPI == EPI_SWIGLU && threadIdx.x < 128) sInv[threadIdx.x] = hidden_inv_scale(threadIdx.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(tfull_bar), 1);
    mbar_init(smem_u32(tempty_bar), EPW);
    mbar_init(smem_u32(drain_bar), 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&sff_bar[s]), 1);
    mbar_init(smem_u32(drain2_bar), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == EPI_DOWN) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), GEMM_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_mtiles = p.n_mtiles_dev ? min(*p.n_mtiles_dev, p.n_mtiles_host) : p.n_mtiles_host;
  const int n_ntiles = p.N / GEMM_BN;
  const int n_kblk = p.K / GEMM_BK;
  const int total = n_mtiles * n_ntiles;
  const uint64_t timeout = p.timeout_ns ? p.timeout_ns : 2000000000ull;

  if (warp == 0) {
    // ───────── producer (whole warp waits; lane 0 issues the TMA / bulk copies) ─────────
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = true;
    const size_t k_atoms = (size_t)(p.K / 64);
    const size_t sfb_expert_bytes = (size_t)p.N * (size_t)(p.K / 16);
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const int mt = t / n_ntiles, nt = t % n_ntiles;
      const int e = p.tile_expert[mt];
      const int brow = e * p.N + nt * GEMM_BN;
      for (int kb = 0; kb < n_kblk; ++kb) {
        if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, GEMM_STAGE_TX);
          tma_load_2d(smem_u32(sA + stage * GEMM_A_BYTES), &tmA, fb, kb * (GEMM_BK / 2), mt * GEMM_BM);
          tma_load_2d(smem_u32(sB + stage * GEMM_B_BYTES), &tmB, fb, kb * (GEMM_BK / 2), brow);
          const uint8_t* sfa_src = p.sfa + ((size_t)mt * k_atoms + (size_t)kb * 4) * 512;
          bulk_load(smem_u32(sSFA + stage * GEMM_SFA_BYTES), sfa_src, GEMM_SFA_BYTES, fb);
#pragma unroll
          for (int nb = 0; nb < 2; ++nb) {
            const uint8_t* sfb_src =
                p.sfb + (size_t)e * sfb_expert_bytes + ((size_t)(nt * 2 + nb) * k_atoms + (size_t)kb * 4) * 512;
            bulk_load(smem_u32(sSFB + stage * GEMM_SFB_BYTES + nb * 2048), sfb_src, 2048, fb);
          }
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // Every copy this CTA issued lands before it can exit.  Loads older than the last
    // STAGES were consumed already; on the normal path the last ones were too, so these
    // waits return at once — they matter when a consumer gave up on an error.
    for (int64_t i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
      mbar_wait(smem_u32(&full_bar[i % STAGES]), (uint32_t)((i / STAGES) & 1), nullptr, 0, MHMOE_DRAIN_NS);
  } else if (warp == 1) {
    // ───────── MMA issuer (whole warp waits; lane 0 issues) ─────────
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0;
    constexpr uint32_t idesc = idesc_nvf4(GEMM_BM, GEMM_BN);
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      if (!mbar_wait(smem_u32(tempty_bar), acc_phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
      tc_fence_after();
      for (int kb = 0; kb < n_kblk; ++kb) {
        if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
        if (!mbar_wait(smem_u32(&sff_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t tsfa = tmem_base + GEMM_SF_COL0 + stage * GEMM_SF_COLS_PER_STAGE;
          const uint32_t tsfb = tsfa + 16;
          const uint32_t a_s = smem_u32(sA + stage * GEMM_A_BYTES);
          const uint32_t b_s = smem_u32(sB + stage * GEMM_B_BYTES);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            mma_nvf4(tmem_base, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc,
                     tsfa + j * 4, tsfb + j * 8, (kb | j) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&empty_bar[stage]));
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (lane == 0) tc_commit(smem_u32(tfull_bar));
      __syncwarp();
      acc_phase ^= 1;
    }
  } else if (warp == COPIER) {
    // ───────── scale-factor copier (whole warp waits; lane 0 issues) ─────────
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      for (int kb = 0; kb < n_kblk; ++kb) {
        if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t tsfa = tmem_base + GEMM_SF_COL0 + stage * GEMM_SF_COLS_PER_STAGE;
          const uint32_t tsfb = tsfa + 16;
          const uint32_t sfa_s = smem_u32(sSFA + stage * GEMM_SFA_BYTES);
          const uint32_t sfb_s = smem_u32(sSFB + stage * GEMM_SFB_BYTES);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tc_cp_32x128b_warpx4(tsfa + j * 4, sdesc_sf_chunk(sfa_s + j * 512));
            tc_cp_32x128b_warpx4(tsfb + j * 8, sdesc_sf_chunk(sfb_s + j * 512));
            tc_cp_32x128b_warpx4(tsfb + j * 8 + 4, sdesc_sf_chunk(sfb_s + 2048 + j * 512));
          }
          tc_commit(smem_u32(&sff_bar[stage]));
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ───────── epilogue warps 2 .. 2+EPW-1 ─────────
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;       // accumulator columns [NCOL*half, NCOL*half + NCOL)
    const int m = q * 32 + lane;            // tile row owned by this thread
    uint32_t acc_phase = 0;
    // Per-tile scalars arrive ahead of their tile (EpiPrefetch): their global-memory latency
    // hides under the epilogues before, which matters when the epilogue is the bottleneck.
    const auto mtile_of = [n_ntiles](int t) { return t / n_ntiles; };
    EpiPrefetch<EPI, decltype(mtile_of)> pf(p, mtile_of, (int)blockIdx.x, (int)gridDim.x, total, m);
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int mt = t / n_ntiles, nt = t % n_ntiles;
      const EpiScalars sc = pf.next(p, mtile_of, t, (int)gridDim.x, total, m);
      if (!mbar_wait(smem_u32(tfull_bar), acc_phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) break;
      acc_phase ^= 1;
      tc_fence_after();
      uint32_t r[NCOL];
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * NCOL);
#pragma unroll
      for (int c = 0; c < NCOL; c += 32) MHMOE_TMEM_LD_32x32b_X32(taddr + c, (r + c));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tempty_bar));

      gemm_epilogue_tile<EPI, NCOL>(p, &tmC, r, sc, mt, nt, m, q, half, lane, sSTG + (warp - 2) * (32 * 128), sInv);
    }
    if constexpr (EPI == EPI_DOWN) {
      if (lane == 0) bulk_wait_all();     // stores complete before the CTA exits
    }
  }
done:
  if (warp == 1 && lane == 0) {
    // Retire every tcgen05 op this thread issued before TMEM is released
    // (matters only on an error path; on the normal path they are done already).
    tc_commit(smem_u32(drain_bar));
    mbar_wait(smem_u32(drain_bar), 0, nullptr, 0, MHMOE_DRAIN_NS);
  }
  if (warp == COPIER && lane == 0) {
    tc_commit(smem_u32(drain2_bar));
    mbar_wait(smem_u32(drain2_bar), 0, nullptr, 0, MHMOE_DRAIN_NS);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, GEMM_TMEM_COLS);
  }
}

// ───────────────────────────── CTA-pair kernel ─────────────────────────────
// Work item = (pair of m-tiles 2*pt, 2*pt+1 of one expert, n-tile).  CTA rank r of the
// cluster owns m-tile 2*pt + r.  Roles as in the single-CTA kernel, except:
//   producer (both CTAs): TMA loads into its own shared memory (A rows, B rows
//     [nt*256 + 128*r, +128), SFA, full SFB) that signal the LEADER's full barrier; the
//     leader's producer posts the expected bytes of both CTAs.
//   copier (warp 10, leader only): tcgen05.cp with cta_group::2 (each CTA's shared memory at
//     the same offsets -> its own TMEM), committed to the leader's sf-full barrier.
//   MMA (leader only): tcgen05.mma with cta_group::2 once the stage's data and scale
//     factors are in, commits to the stage's empty barrier of both CTAs and, per tile, to
//     both CTAs' accumulator-full barrier.
//   epilogue (both CTAs): its own 128 rows; releases the accumulator on the leader's
//     barrier (16 arrivals per tile).
// tmSFA / tmSFB: the SF atom arrays viewed as [bytes/256, 256] u8, box 256 x 8 (2 KB).
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMMP_THREADS, 1)
    ffn_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmSFA,
                         const __grid_constant__ CUtensorMap tmSFB, const FfnGemmParams p) {
  constexpr int STAGES = gemmp_stages(EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * GEMM_A_BYTES;
  uint8_t* sSFA = sB + STAGES * GEMMP_B_BYTES;
  uint8_t* sSFB = sSFA + STAGES * GEMM_SFA_BYTES;
  uint8_t* sSTG = sSFB + STAGES * GEMM_SFB_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSTG + (EPI == EPI_DOWN ? GEMM_STG_BYTES : 0));
  uint64_t* full_bar = bars;                       // [STAGES] (leader's are used)
  uint64_t* empty_bar = bars + STAGES;             // [STAGES]
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = tfull_bar + 1;            // (leader's is used)
  uint64_t* drain_bar = tfull_bar + 2;
  uint64_t* sff_bar = tfull_bar + 3;               // [STAGES] scale factors of the stage in TMEM (leader's)
  uint64_t* drain2_bar = sff_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain2_bar + 1);
  float* sInv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [128] hidden_inv_scale

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (EPI == EPI_SWIGLU && threadIdx.x < 128) sInv[threadIdx.x] = hidden_inv_scale(threadIdx.x);
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(tfull_bar), 1);
    mbar_init(smem_u32(tempty_bar), 16);
    mbar_init(smem_u32(drain_bar), 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&sff_bar[s]), 1);
    mbar_init(smem_u32(drain2_bar), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmSFA);
    tma_prefetch_desc(&tmSFB);
    if (EPI == EPI_DOWN) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), GEMM_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();                                  // barriers initialised, TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_mtiles = p.n_mtiles_dev ? min(*p.n_mtiles_dev, p.n_mtiles_host) : p.n_mtiles_host;
  const int n_pairs = n_mtiles / 2;
  const int n_ntiles = p.N / GEMM_BN;
  const int n_kblk = p.K / GEMM_BK;
  const int total = n_pairs * n_ntiles;
  const int cluster_id = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
  const uint64_t timeout = p.timeout_ns ? p.timeout_ns : 2000000000ull;

  if (warp == 0) {
    // ───────── producer (both CTAs; whole warp waits, lane 0 issues) ─────────
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = true;
    const int k_atoms = p.K / 64;
    const int64_t sfb_rows_per_expert = (int64_t)p.N * (p.K / 16) / 256;
    for (int t = cluster_id; ok && t < total; t += n_clusters) {
      const int pt = t / n_ntiles, nt = t % n_ntiles;
      const int mt = 2 * pt + (int)crank;
      const int e = p.tile_expert[mt];
      const int brow = e * p.N + nt * GEMM_BN + (int)crank * (GEMM_BN / 2);
      for (int kb = 0; kb < n_kblk; ++kb) {
        if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t fb_local = smem_u32(&full_bar[stage]);
          const uint32_t fb = mapa_shared(fb_local, 0);
          if (leader) mbar_arrive_expect_tx(fb_local, 2u * GEMMP_STAGE_TX);
          tma_load_2d_pair(smem_u32(sA + stage * GEMM_A_BYTES), &tmA, fb, kb * (GEMM_BK / 2), mt * GEMM_BM);
          tma_load_2d_pair(smem_u32(sB + stage * GEMMP_B_BYTES), &tmB, fb, kb * (GEMM_BK / 2), brow);
          tma_load_2d_pair(smem_u32(sSFA + stage * GEMM_SFA_BYTES), &tmSFA, fb, 0, (mt * k_atoms + kb * 4) * 2);
#pragma unroll
          for (int nb = 0; nb < 2; ++nb)
            tma_load_2d_pair(smem_u32(sSFB + stage * GEMM_SFB_BYTES + nb * 2048), &tmSFB, fb, 0,
                             (int)(e * sfb_rows_per_expert + ((nt * 2 + nb) * k_atoms + kb * 4) * 2));
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // The leader's full barriers count both CTAs' bytes: once the last STAGES of them
    // completed, every copy of the pair has landed (returns at once on the normal path).
    if (leader)
      for (int64_t i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
        mbar_wait(smem_u32(&full_bar[i % STAGES]), (uint32_t)((i / STAGES) & 1), nullptr, 0, MHMOE_DRAIN_NS);
  } else if (warp == 1) {
    // ───────── MMA issuer: the leader CTA only ─────────
    if (leader) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      constexpr uint32_t idesc = idesc_nvf4(2 * GEMM_BM, GEMM_BN);
      for (int t = cluster_id; t < total; t += n_clusters) {
        if (!mbar_wait(smem_u32(tempty_bar), acc_phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
        tc_fence_after();
        for (int kb = 0; kb < n_kblk; ++kb) {
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
          if (!mbar_wait(smem_u32(&sff_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t tsfa = tmem_base + GEMM_SF_COL0 + stage * GEMM_SF_COLS_PER_STAGE;
            const uint32_t tsfb = tsfa + 16;
            const uint32_t a_s = smem_u32(sA + stage * GEMM_A_BYTES);
            const uint32_t b_s = smem_u32(sB + stage * GEMMP_B_BYTES);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              mma_nvf4_pair(tmem_base, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc,
                            tsfa + j * 4, tsfb + j * 8, (kb | j) != 0 ? 1u : 0u);
            const uint32_t eb = smem_u32(&empty_bar[stage]);
            tc_commit_pair(mapa_shared(eb, 0));
            tc_commit_pair(mapa_shared(eb, 1));
          }
          __syncwarp();
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (lane == 0) {
          tc_commit_pair(mapa_shared(smem_u32(tfull_bar), 0));
          tc_commit_pair(mapa_shared(smem_u32(tfull_bar), 1));
        }
        __syncwarp();
        acc_phase ^= 1;
      }
    }
  } else if (warp == 10) {
    // ───────── scale-factor copier: the leader CTA only (pair copies reach both CTAs' TMEM) ─────────
    // Slot s is rewritten only after full[s] of the next round, posted after empty[s], which
    // the MMA warp commits after the MMAs that read slot s (as in the single-CTA kernel).
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = cluster_id; t < total; t += n_clusters) {
        for (int kb = 0; kb < n_kblk; ++kb) {
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t tsfa = tmem_base + GEMM_SF_COL0 + stage * GEMM_SF_COLS_PER_STAGE;
            const uint32_t tsfb = tsfa + 16;
            const uint32_t sfa_s = smem_u32(sSFA + stage * GEMM_SFA_BYTES);
            const uint32_t sfb_s = smem_u32(sSFB + stage * GEMM_SFB_BYTES);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tc_cp_32x128b_warpx4_pair(tsfa + j * 4, sdesc_sf_chunk(sfa_s + j * 512));
              tc_cp_32x128b_warpx4_pair(tsfb + j * 8, sdesc_sf_chunk(sfb_s + j * 512));
              tc_cp_32x128b_warpx4_pair(tsfb + j * 8 + 4, sdesc_sf_chunk(sfb_s + 2048 + j * 512));
            }
            tc_commit_pair(mapa_shared(smem_u32(&sff_bar[stage]), 0));
          }
          __syncwarp();
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else {
    // ───────── epilogue warps 2..9 (both CTAs, own 128 rows) ─────────
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int m = q * 32 + lane;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty_bar), 0);
    uint32_t acc_phase = 0;
    const int crank_i = (int)crank;
    const auto mtile_of = [n_ntiles, crank_i](int t) { return 2 * (t / n_ntiles) + crank_i; };
    EpiPrefetch<EPI, decltype(mtile_of)> pf(p, mtile_of, cluster_id, n_clusters, total, m);   // per-tile scalars
    for (int t = cluster_id; t < total; t += n_clusters) {
      const int pt = t / n_ntiles, nt = t % n_ntiles;
      const int mt = 2 * pt + (int)crank;
      const EpiScalars sc = pf.next(p, mtile_of, t, n_clusters, total, m);
      if (!mbar_wait(smem_u32(tfull_bar), acc_phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) break;
      acc_phase ^= 1;
      tc_fence_after();
      uint32_t r[128];
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * 128);
      MHMOE_TMEM_LD_32x32b_X32(taddr + 0, (r + 0));
      MHMOE_TMEM_LD_32x32b_X32(taddr + 32, (r + 32));
      MHMOE_TMEM_LD_32x32b_X32(taddr + 64, (r + 64));
      MHMOE_TMEM_LD_32x32b_X32(taddr + 96, (r + 96));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader);
      gemm_epilogue_tile<EPI, 128>(p, &tmC, r, sc, mt, nt, m, q, half, lane, sSTG + (warp - 2) * (32 * 128), sInv);
    }
    if constexpr (EPI == EPI_DOWN) {
      if (lane == 0) bulk_wait_all();
    }
  }
done:
  if (leader && warp == 1 && lane == 0) {
    tc_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
    mbar_wait(smem_u32(drain_bar), 0, nullptr, 0, MHMOE_DRAIN_NS);
  }
  if (leader && warp == 10 && lane == 0) {
    tc_commit_pair(mapa_shared(smem_u32(drain2_bar), 0));
    mbar_wait(smem_u32(drain2_bar), 0, nullptr, 0, MHMOE_DRAIN_NS);
  }
  tc_fence_before();
  cluster_sync();                                  // neither CTA leaves while the pair still uses it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, GEMM_TMEM_COLS);
  }
}

}  // namespace mhmoe
