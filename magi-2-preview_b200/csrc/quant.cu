// NVFP4 quantisers: activation gather+quantise for the gate/up GEMM, generic per-row
// quantisation, and the weight packer (quantise on load).
//
// The exact fp32 op sequence of a 16-element block is quant_block16() in
// mhmoe_common.cuh; oracle/nvfp4_ref.py states the same sequence for the CPU.
#include "kernels.cuh"

namespace mhmoe {

// Load 8 bf16 (16 B) and widen to fp32.
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Quantise one bf16 row of K elements (K % 64 == 0) with a warp: amax -> g, then
// lanes take 64-element groups (4 blocks), write 32 packed bytes + one 4-byte SF word.
__device__ __forceinline__ void warp_quant_row(const __nv_bfloat16* src, int K, uint64_t out_row, uint8_t* data,
                                               uint8_t* sf, float* gscale, int lane, bool sf_rowmajor = false) {
  float amax = 0.f;
  if (src) {
    for (int i = lane; i < K / 8; i += 32) {
      float f[8];
      load8_bf16(src + i * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float g = amax > 0.f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  if (lane == 0 && gscale) gscale[out_row] = g;
  uint8_t* drow = data + out_row * (uint64_t)(K / 2);
  for (int grp = lane; grp < K / 64; grp += 32) {
    uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t sfw = 0;
    if (src) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float v[16];
        load8_bf16(src + grp * 64 + b * 16, v);
        load8_bf16(src + grp * 64 + b * 16 + 8, v + 8);
        uint32_t w2[2];
        const uint32_t s = quant_block16(v, g, w2);
        words[2 * b] = w2[0];
        words[2 * b + 1] = w2[1];
        sfw |= s << (8 * b);
      }
    }
    uint4* d = reinterpret_cast<uint4*>(drow + grp * 32);
    d[0] = make_uint4(words[0], words[1], words[2], words[3]);
    d[1] = make_uint4(words[4], words[5], words[6], words[7]);
    const uint64_t so = sf_rowmajor ? out_row * (uint64_t)(K / 16) + (uint64_t)grp * 4
                                    : sf_atom_offset(out_row, (uint32_t)(grp * 4), (uint32_t)K);
    *reinterpret_cast<uint32_t*>(sf + so) = sfw;
  }
}

// Grouped A operand of the gate/up GEMM: warps walk the padded rows of the expert-grouped
// row space (grid-stride, up to the device's tile count: the grid is sized for the rows
// actually present, not for the host's upper bound); each copies its token's NVFP4 row
// (per-token quantised x: data, row-major scales, row scale) into place, scales into the
// SF-atom layout.  Padding rows are zeroed.
__global__ void group_rows_kernel(const uint8_t* __restrict__ xq, int64_t xq_pitch, const uint8_t* __restrict__ xsf,
                                  int64_t xsf_pitch, const uint8_t* __restrict__ xg, int64_t xg_pitch, int64_t T,
                                  int dh, int H, int E_per_head,
                                  const int32_t* __restrict__ gather_ids, const int* __restrict__ cu_tiles, int HE,
                                  const int* __restrict__ tile_expert, const int* __restrict__ tile_row0,
                                  const int* __restrict__ tile_rows, uint8_t* __restrict__ a_data,
                                  uint8_t* __restrict__ a_sf, float* __restrict__ a_gscale,
                                  int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t n_rows = (int64_t)cu_tiles[HE] * 128;
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t prow = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); prow < n_rows; prow += stride) {
    const int mt = (int)(prow >> 7);
    const int m = (int)(prow & 127);
    int64_t t = -1;
    if (m < tile_rows[mt]) {
      const int s = gather_ids[tile_row0[mt] + m];
      t = (int64_t)s * H + tile_expert[mt] / E_per_head;
      if (s < 0 || t >= T) {
        if (lane == 0) record_error(status, MHMOE_ERR_ARGS);
        t = -1;
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(a_data + prow * (dh / 2));
    const uint4* src = t >= 0 ? reinterpret_cast<const uint4*>(xq + t * xq_pitch) : nullptr;
    for (int i = lane; i < dh / 32; i += 32) dst[i] = src ? src[i] : make_uint4(0, 0, 0, 0);
    const uint32_t* ssrc = t >= 0 ? reinterpret_cast<const uint32_t*>(xsf + t * xsf_pitch) : nullptr;
    for (int w = lane; w < dh / 64; w += 32) {
      const uint32_t v = ssrc ? ssrc[w] : 0u;
      *reinterpret_cast<uint32_t*>(a_sf + sf_atom_offset((uint64_t)prow, (uint32_t)(4 * w), (uint32_t)dh)) = v;
    }
    if (lane == 0) a_gscale[prow] = t >= 0 ? *reinterpret_cast<const float*>(xg + t * xg_pitch) : 1.0f;
  }
}

// Per-token quantisation: row t = s * H + h of x [S, H, dh]; scales row-major [T, dh/16].
// Each token is quantised once, however many experts it is routed to.
__global__ void quant_tokens_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx_s, int64_t sx_h, int S, int H,
                                    int dh, uint8_t* __restrict__ xq, uint8_t* __restrict__ xsf,
                                    float* __restrict__ xg) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= (int64_t)S * H) return;
  const int64_t s = t / H, h = t % H;
  warp_quant_row(x + s * sx_s + h * sx_h, dh, (uint64_t)t, xq, xsf, xg, lane, true);
}

// Fused quantise + group (local path, inverse map known): a pair of warps per key (h, s)
// quantises x[s, h, :] once and writes the NVFP4 row (data, scale atoms, row scale) to
// each of the key's padded rows of the grouped A operand, so the per-token intermediate
// never exists.  Lane l of warp half w owns the 16-element blocks b = 32 w + l + 64 i:
// every data store of a destination row is 256 contiguous bytes per warp, and the four
// scales of a 64-element chunk (lanes 4c'..4c'+3 of one warp) are packed into one word
// with two shuffles; the two warps' partial row amax meet in shared memory.  The op
// sequence per block is quant_block16 with g = amax / 2688, as in warp_quant_row.
template <int MAXNB>
__global__ void __launch_bounds__(256, MAXNB <= 3 ? 4 : 2)
    quant_scatter_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx_s, int64_t sx_h, int S, int H, int dh,
                         const int32_t* __restrict__ tok_rows, const int32_t* __restrict__ tok_offsets, int k_fixed,
                         int64_t R, const int32_t* __restrict__ pad_of_row, int64_t rows,
                         uint8_t* __restrict__ a_data, uint8_t* __restrict__ a_sf, float* __restrict__ a_gscale,
                         int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float pair_amax[4][2];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int pair = warp >> 1, half = warp & 1;
  const int64_t key = (int64_t)blockIdx.x * 4 + pair;   // key = h * S + s
  if (key >= (int64_t)H * S) return;                    // both warps of a pair leave together
  const int64_t h = key / S, s = key % S;
  const __nv_bfloat16* src = x + s * sx_s + h * sx_h;
  const int nblk = dh / 16;
  // destinations first (two dependent lookups), so their latency hides under the x loads
  int64_t begin;
  int cnt;
  if (tok_offsets) {
    begin = tok_offsets[key];
    cnt = tok_offsets[key + 1] - (int)begin;
  } else {
    begin = key * k_fixed;
    cnt = k_fixed;
  }
  int r0 = -1;
  if (lane < cnt) r0 = tok_rows[begin + lane];
  uint4 raw[MAXNB][2];
#pragma unroll
  for (int i = 0; i < MAXNB; ++i) {
    const int b = 32 * half + lane + 64 * i;
    if (b < nblk) {
      raw[i][0] = *reinterpret_cast<const uint4*>(src + 16 * b);
      raw[i][1] = *reinterpret_cast<const uint4*>(src + 16 * b + 8);
    } else {
      raw[i][0] = raw[i][1] = make_uint4(0, 0, 0, 0);
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < MAXNB; ++i) {
    float f[16];
    load8_bf16(reinterpret_cast<const __nv_bfloat16*>(&raw[i][0]), f);
    load8_bf16(reinterpret_cast<const __nv_bfloat16*>(&raw[i][1]), f + 8);
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  int32_t p0 = -1;
  if (r0 >= 0 && r0 < R) p0 = pad_of_row[r0];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) pair_amax[pair][half] = amax;
  asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");     // the pair's two warps
  amax = fmaxf(pair_amax[pair][0], pair_amax[pair][1]);
  const float g = amax > 0.f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  uint32_t codes[MAXNB][2], sfw[MAXNB];
#pragma unroll
  for (int i = 0; i < MAXNB; ++i) {
    float f[16];
    load8_bf16(reinterpret_cast<const __nv_bfloat16*>(&raw[i][0]), f);
    load8_bf16(reinterpret_cast<const __nv_bfloat16*>(&raw[i][1]), f + 8);
    uint32_t sf = quant_block16(f, g, codes[i]);
    // lane 4c' collects the scales of lanes 4c'..4c'+3 (bytes 0..3 of the chunk's word)
    sf |= __shfl_down_sync(0xffffffffu, sf, 1) << 8;
    sf |= __shfl_down_sync(0xffffffffu, sf, 2) << 16;
    sfw[i] = sf;
  }
  for (int j0 = 0; j0 < cnt; j0 += 32) {
    int64_t mine = -1;
    if (j0 + lane < cnt) {
      int32_t pr = p0;
      if (j0 > 0) {
        const int r = tok_rows[begin + j0 + lane];
        pr = r >= 0 && r < R ? pad_of_row[r] : -1;
      }
      if (pr >= 0 && pr < rows) mine = pr;
      if (mine < 0 && half == 0) record_error(status, MHMOE_ERR_ARGS);
    }
    const int n = min(32, cnt - j0);
    for (int j = 0; j < n; ++j) {
      const int64_t prow = __shfl_sync(0xffffffffu, mine, j);
      if (prow < 0) continue;
      uint8_t* drow = a_data + prow * (int64_t)(dh / 2);
#pragma unroll
      for (int i = 0; i < MAXNB; ++i) {
        const int b = 32 * half + lane + 64 * i;
        if (b < nblk) {
          *reinterpret_cast<uint2*>(drow + 8 * b) = make_uint2(codes[i][0], codes[i][1]);
          if ((lane & 3) == 0)
            *reinterpret_cast<uint32_t*>(a_sf + sf_atom_offset((uint64_t)prow, (uint32_t)b, (uint32_t)dh)) = sfw[i];
        }
      }
      if (lane == 0 && half == 0) a_gscale[prow] = g;
    }
  }
}

// The same fused quantise + group for short head rows (dh = 16 * LPK: 256 or 512): LPK
// lanes per key, one 16-element block per lane, 32 / LPK keys per warp, so every lane has a
// block (the warp-pair kernel above leaves most lanes idle at dh = 256).  Same op sequence
// and outputs.  Lanes of a warp loop over the largest destination count of its keys, so the
// shuffles always see the whole warp.
template <int LPK>
__global__ void __launch_bounds__(256)
    quant_scatter_short_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx_s, int64_t sx_h, int S, int H,
                               const int32_t* __restrict__ tok_rows, const int32_t* __restrict__ tok_offsets,
                               int k_fixed, int64_t R, const int32_t* __restrict__ pad_of_row, int64_t rows,
                               uint8_t* __restrict__ a_data, uint8_t* __restrict__ a_sf, float* __restrict__ a_gscale,
                               int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  constexpr int dh = 16 * LPK;
  constexpr int KPW = 32 / LPK;                                  // keys per warp
  const int lane = threadIdx.x & 31;
  const int sl = lane % LPK;                                     // block of this lane
  const int gbase = lane - sl;                                   // first lane of this key's group
  const int64_t key = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * KPW + lane / LPK;
  const bool live = key < (int64_t)H * S;
  const int64_t h = live ? key / S : 0, s = live ? key % S : 0;
  int64_t begin = 0;
  int cnt = 0;
  if (live) {
    if (tok_offsets) {
      begin = tok_offsets[key];
      cnt = tok_offsets[key + 1] - (int)begin;
    } else {
      begin = key * k_fixed;
      cnt = k_fixed;
    }
  }
  float f[16];
  if (live) {
    const __nv_bfloat16* src = x + s * sx_s + h * sx_h + 16 * sl;
    load8_bf16(src, f);
    load8_bf16(src + 8, f + 8);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(f[j]));
#pragma unroll
  for (int o = LPK / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float g = amax > 0.f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  uint32_t codes[2];
  uint32_t sfw = quant_block16(f, g, codes);
  // lane 4c collects the scales of lanes 4c..4c+3 (bytes 0..3 of the chunk's word)
  sfw |= __shfl_down_sync(0xffffffffu, sfw, 1) << 8;
  sfw |= __shfl_down_sync(0xffffffffu, sfw, 2) << 16;
  int maxcnt = cnt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxcnt = max(maxcnt, __shfl_xor_sync(0xffffffffu, maxcnt, o));
  for (int j0 = 0; j0 < maxcnt; j0 += LPK) {
    int64_t mine = -1;                                           // padded row of destination j0 + sl
    if (j0 + sl < cnt) {
      const int r = tok_rows[begin + j0 + sl];
      const int32_t pr = r >= 0 && r < R ? pad_of_row[r] : -1;
      if (pr >= 0 && pr < rows) mine = pr;
      else record_error(status, MHMOE_ERR_ARGS);
    }
    const int n = min(LPK, maxcnt - j0);
    for (int j = 0; j < n; ++j) {
      const int64_t prow = __shfl_sync(0xffffffffu, mine, gbase + j);
      if (j0 + j >= cnt || prow < 0) continue;
      *reinterpret_cast<uint2*>(a_data + prow * (int64_t)(dh / 2) + 8 * sl) = make_uint2(codes[0], codes[1]);
      if ((sl & 3) == 0)
        *reinterpret_cast<uint32_t*>(a_sf + sf_atom_offset((uint64_t)prow, (uint32_t)sl, (uint32_t)dh)) = sfw;
      if (sl == 0) a_gscale[prow] = g;
    }
  }
}

__global__ void quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t pitch, int64_t M, int K,
                                     uint8_t* __restrict__ data, uint8_t* __restrict__ sf,
                                     float* __restrict__ gscale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  warp_quant_row(x + row * pitch, K, (uint64_t)row, data, sf, gscale, lane);
}

// ───────────────────────────── weight packer ─────────────────────────────

// amax[mat] over each [rows x cols] matrix; grid (chunks, n_mats).  Non-negative
// floats order like their bit patterns, so an integer atomicMax is exact.
__global__ void amax_kernel(const __nv_bfloat16* __restrict__ w, int64_t mat_elems, float* __restrict__ amax) {
  const __nv_bfloat16* base = w + (int64_t)blockIdx.y * mat_elems;
  float a = 0.f;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < mat_elems;
       i += (int64_t)gridDim.x * blockDim.x * 8) {
    float f[8];
    load8_bf16(base + i, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(f[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(amax) + blockIdx.y, __float_as_int(a));
}

__global__ void gscale_kernel(const float* __restrict__ amax, int n, float* __restrict__ g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) g[i] = amax[i] > 0.f ? __fdiv_rn(amax[i], 2688.0f) : 1.0f;
}

// Transposing quantiser: source matrix w[e] is [Kdim, Ndim] (N contiguous, the
// reference layout); the packed operand is K-major [Nrows, Kdim/2].  One CTA handles a
// 64(k) x 64(n) tile; thread (n, kq) quantises the 16-element k-block kq of column n.
// For kind 0 the source column n of matrix `which` (0 gate, 1 up) lands on fused row
// 32*(n/16) + 16*which + n%16 of a 2*Ndim-row operand.
__global__ void pack_tile_kernel(const __nv_bfloat16* __restrict__ w, int Kdim, int Ndim, int which, int fused,
                                 const float* __restrict__ gscale, uint8_t* __restrict__ data,
                                 uint8_t* __restrict__ sf) {
  __shared__ float tile[64][65];
  const int e = blockIdx.z;
  const int k0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const __nv_bfloat16* src = w + (int64_t)e * Kdim * Ndim;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int kk = i / 64, nn = i % 64;
    tile[kk][nn] = __bfloat162float(src[(int64_t)(k0 + kk) * Ndim + n0 + nn]);
  }
  __syncthreads();
  const int nn = threadIdx.x & 63, kq = threadIdx.x >> 6;   // 256 threads: 64 columns x 4 k-blocks
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = tile[kq * 16 + i][nn];
  const int Nrows = fused ? 2 * Ndim : Ndim;
  const float g = gscale[(fused ? which * gridDim.z : 0) + e];
  uint32_t w2[2];
  const uint32_t s = quant_block16(v, g, w2);
  const int n = n0 + nn;
  const int64_t row = fused ? (int64_t)32 * (n / 16) + 16 * which + (n % 16) : n;
  const int k = k0 + kq * 16;
  uint8_t* drow = data + ((int64_t)e * Nrows + row) * (Kdim / 2);
  *reinterpret_cast<uint2*>(drow + k / 2) = make_uint2(w2[0], w2[1]);
  uint8_t* sfe = sf + (int64_t)e * Nrows * (Kdim / 16);
  sfe[sf_atom_offset((uint64_t)row, (uint32_t)(k / 16), (uint32_t)Kdim)] = (uint8_t)s;
}

// ───────────────────────────── launchers ─────────────────────────────

cudaError_t launch_group_rows(const uint8_t* xq, int64_t xq_pitch, const uint8_t* xsf, int64_t xsf_pitch,
                              const uint8_t* xg, int64_t xg_pitch, int64_t T, int dh, int H, int E_per_head,
                              const int32_t* gather_ids, const int* cu_tiles, int HE, int64_t max_mtiles,
                              const int* tile_expert, const int* tile_row0, const int* tile_rows, uint8_t* a_data,
                              uint8_t* a_sf, float* a_gscale, int* status, cudaStream_t st) {
  const int64_t rows = max_mtiles * 128;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(rows / 8, (int64_t)16 * num_sms()));
  MHMOE_LAUNCH_PDL(group_rows_kernel, (unsigned)blocks, 256, 0, st, xq, xq_pitch, xsf, xsf_pitch, xg, xg_pitch, T,
                   dh, H, E_per_head, gather_ids, cu_tiles, HE, tile_expert, tile_row0, tile_rows, a_data, a_sf,
                   a_gscale, status);
  return cudaGetLastError();
}

cudaError_t launch_quant_tokens(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh,
                                uint8_t* xq, uint8_t* xsf, float* xg, cudaStream_t st) {
  const int64_t T = (int64_t)S * H;
  MHMOE_LAUNCH_PDL(quant_tokens_kernel, (unsigned)((T + 7) / 8), 256, 0, st, x, sx_s, sx_h, S, H, dh, xq, xsf, xg);
  return cudaGetLastError();
}

int quant_scatter_max_dh() { return 16 * 512; }

cudaError_t launch_quant_scatter(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh,
                                 const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R,
                                 const int32_t* pad_of_row, int64_t rows, uint8_t* a_data, uint8_t* a_sf,
                                 float* a_gscale, int* status, cudaStream_t st) {
  const int64_t keys = (int64_t)S * H;
  if (dh == 256 || dh == 512) {                          // short rows: LPK lanes per key, 8 warps per block
    const int lpk = dh / 16;
    const int64_t warps = (keys + 32 / lpk - 1) / (32 / lpk);
    const unsigned g2 = (unsigned)((warps + 7) / 8);
    if (lpk == 16)
      MHMOE_LAUNCH_PDL(quant_scatter_short_kernel<16>, g2, 256, 0, st, x, sx_s, sx_h, S, H, tok_rows, tok_offsets,
                       k_fixed, R, pad_of_row, rows, a_data, a_sf, a_gscale, status);
    else
      MHMOE_LAUNCH_PDL(quant_scatter_short_kernel<32>, g2, 256, 0, st, x, sx_s, sx_h, S, H, tok_rows, tok_offsets,
                       k_fixed, R, pad_of_row, rows, a_data, a_sf, a_gscale, status);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((keys + 3) / 4);      // 4 keys (warp pairs) per 256-thread block
  const int nb = (dh / 16 + 63) / 64;                    // blocks per lane
#define MHMOE_QS(NB)                                                                                       \
  MHMOE_LAUNCH_PDL(quant_scatter_kernel<NB>, grid, 256, 0, st, x, sx_s, sx_h, S, H, dh, tok_rows, tok_offsets, \
                   k_fixed, R, pad_of_row, rows, a_data, a_sf, a_gscale, status)
  if (nb <= 1) MHMOE_QS(1);
  else if (nb <= 2) MHMOE_QS(2);
  else if (nb <= 3) MHMOE_QS(3);
  else if (nb <= 4) MHMOE_QS(4);
  else if (nb <= 6) MHMOE_QS(6);
  else if (nb <= 8) MHMOE_QS(8);
  else return cudaErrorInvalidValue;
#undef MHMOE_QS
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int64_t pitch, int64_t M, int K, uint8_t* data, uint8_t* sf,
                                 float* gscale, cudaStream_t st) {
  quantize_rows_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(x, pitch, M, K, data, sf, gscale);
  return cudaGetLastError();
}

cudaError_t launch_pack_weights(int kind, const __nv_bfloat16* w0, const __nv_bfloat16* w1, int n_experts, int dh,
                                int de, uint8_t* data, uint8_t* sf, float* gscale, float* amax, cudaStream_t st) {
  // kind 0: w0 = W_gate, w1 = W_up, each [E, dh, de]; operand [E, 2de, dh/2]
  // kind 1: w0 = W_down [E, de, dh];                     operand [E, dh, de/2]
  const int nmat = kind == 0 ? 2 : 1;
  const int64_t elems = (int64_t)dh * de;
  cudaMemsetAsync(amax, 0, sizeof(float) * nmat * n_experts, st);
  const dim3 ag(64, n_experts);
  amax_kernel<<<ag, 256, 0, st>>>(w0, elems, amax);
  if (kind == 0) amax_kernel<<<ag, 256, 0, st>>>(w1, elems, amax + n_experts);
  gscale_kernel<<<(nmat * n_experts + 255) / 256, 256, 0, st>>>(amax, nmat * n_experts, gscale);
  if (kind == 0) {
    const dim3 grid(de / 64, dh / 64, n_experts);
    pack_tile_kernel<<<grid, 256, 0, st>>>(w0, dh, de, 0, 1, gscale, data, sf);
    pack_tile_kernel<<<grid, 256, 0, st>>>(w1, dh, de, 1, 1, gscale, data, sf);
  } else {
    const dim3 grid(dh / 64, de / 64, n_experts);
    pack_tile_kernel<<<grid, 256, 0, st>>>(w0, de, dh, 0, 0, gscale, data, sf);
  }
  return cudaGetLastError();
}

}  // namespace mhmoe
