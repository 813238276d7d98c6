// Router: fp32 logits and top-k gating.
//
// * router_logits_kernel restates CoreMultiHeadMoE._route's fp32 einsum
//   (inference/model/magi2_preview.py:2588-2591): logits[h,s,e] = sum_d x[s,h,d] *
//   gate[h*E+e, d], with x widened from bf16 and fp32 products/accumulation.
// * topk_kernel restates _compute_topk_probs_and_indices_torch_impl
//   (inference/flash_mh_moe/route.py:28-148): softmax/sigmoid scores, selection on
//   scores + expert_bias, optional virtual-group pre-selection (group score = sum of
//   its top-2, masked experts read 0.0), top-k sorted descending (ties -> lower id),
//   probs gathered from the unbiased scores, L1 normalisation x / max(sum|x|, eps),
//   then the module's route_scale (magi2_preview.py:2600).
#include "kernels.cuh"

namespace mhmoe {

// 64 tokens x 64 experts per CTA, 256 threads (4x4 outputs each), d in steps of 32.
__global__ void __launch_bounds__(256) router_logits_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx_s,
                                                            int64_t sx_h, const float* __restrict__ gate, int S,
                                                            int dh, int E, float* __restrict__ logits) {
  __shared__ float xs[32][68];
  __shared__ float gs[32][68];
  const int h = blockIdx.z;
  const int s0 = blockIdx.x * 64, e0 = blockIdx.y * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int d0 = 0; d0 < dh; d0 += 32) {
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
      const int r = i >> 5, c = i & 31;
      const int s = s0 + r, e = e0 + r;
      xs[c][r] = s < S ? __bfloat162float(x[(int64_t)s * sx_s + (int64_t)h * sx_h + d0 + c]) : 0.f;
      gs[c][r] = e < E ? gate[((int64_t)h * E + e) * dh + d0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < 32; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[c][ty * 4 + i];
        b[i] = gs[c][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = s0 + ty * 4 + i;
    if (s >= S) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) logits[((int64_t)h * S + s) * E + e] = acc[i][j];
    }
  }
}

// Warp-wide argmax over (value, index) pairs: larger value wins, ties -> smaller index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

constexpr int TOPK_WARPS = 4;

// One warp per (h, s) row.  Dynamic smem per warp: score[E], sel[E], plus 32 group slots.
__global__ void topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int H, int S, int E,
                            int K, int score_func, int nvg, int tvg, int route_norm, float norm_eps,
                            float route_scale, float* __restrict__ probs, int64_t* __restrict__ idx) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * TOPK_WARPS + warp;
  if (row >= (int64_t)H * S) return;
  const int h = (int)(row / S);
  float* score = sm + warp * (2 * E + 64);
  float* sel = score + E;
  float* gsc = sel + E;                 // group scores (<= 64 groups)
  const float* lg = logits + row * E;

  if (score_func == 0) {
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) {
      const float ex = expf(lg[e] - mx);
      score[e] = ex;
      sum += ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int e = lane; e < E; e += 32) score[e] = __fdiv_rn(score[e], sum);
  } else {
    for (int e = lane; e < E; e += 32) score[e] = __fdiv_rn(1.0f, 1.0f + expf(-lg[e]));
  }
  for (int e = lane; e < E; e += 32) sel[e] = bias ? __fadd_rn(score[e], bias[(int64_t)h * E + e]) : score[e];
  __syncwarp();

  if (nvg > 1) {
    const int epg = E / nvg;
    for (int g = lane; g < nvg; g += 32) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int j = 0; j < epg; ++j) {
        const float v = sel[g * epg + j];
        if (v > b1) {
          b2 = b1;
          b1 = v;
        } else if (v > b2) {
          b2 = v;
        }
      }
      gsc[g] = epg >= 2 ? __fadd_rn(b1, b2) : b1;
    }
    __syncwarp();
    // pick tvg groups; chosen groups are marked by -inf in gsc copy
    unsigned long long chosen = 0ull;
    for (int t = 0; t < tvg; ++t) {
      float v = -INFINITY;
      int gi = 0x7fffffff;
      for (int g = lane; g < nvg; g += 32) {
        if (chosen >> g & 1ull) continue;
        const float gv = gsc[g];
        if (gv > v || (gv == v && g < gi)) {
          v = gv;
          gi = g;
        }
      }
      warp_argmax(v, gi);
      if (gi < nvg) chosen |= 1ull << gi;
    }
    for (int e = lane; e < E; e += 32)
      if (!(chosen >> (e / epg) & 1ull)) sel[e] = 0.0f;
    __syncwarp();
  }

  // top-K by repeated warp argmax; selected entries are excluded through a lane-local bitmask
  unsigned taken = 0u;   // bit j: expert lane + 32*j taken (E <= 1024)
  float my_p = 0.f;
  int my_i = 0;
  for (int k = 0; k < K; ++k) {
    float v = -INFINITY;
    int vi = 0x7fffffff;
    for (int j = 0, e = lane; e < E; ++j, e += 32) {
      if (taken >> j & 1u) continue;
      const float sv = sel[e];
      if (sv > v || (sv == v && e < vi)) {
        v = sv;
        vi = e;
      }
    }
    warp_argmax(v, vi);
    if (vi >= E) vi = 0;                       // all remaining are NaN: deterministic fallback
    if ((vi & 31) == lane) taken |= 1u << (vi >> 5);
    if (lane == k) {
      my_i = vi;
      my_p = score[vi];
    }
  }
  if (route_norm) {
    float s = lane < K ? fabsf(my_p) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    my_p = __fdiv_rn(my_p, fmaxf(s, norm_eps));
  }
  if (lane < K) {
    probs[row * K + lane] = __fmul_rn(my_p, route_scale);
    idx[row * K + lane] = my_i;
  }
}

cudaError_t launch_router_logits(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, const float* gate, int S, int H,
                                 int dh, int E, float* logits, cudaStream_t st) {
  const dim3 grid((S + 63) / 64, (E + 63) / 64, H);
  router_logits_kernel<<<grid, 256, 0, st>>>(x, sx_s, sx_h, gate, S, dh, E, logits);
  return cudaGetLastError();
}

cudaError_t launch_topk(const float* logits, const float* bias, int H, int S, int E, int K, int score_func, int nvg,
                        int tvg, int route_norm, float norm_eps, float route_scale, float* probs, int64_t* idx,
                        cudaStream_t st) {
  const int64_t rows = (int64_t)H * S;
  const size_t smem = (size_t)TOPK_WARPS * (2 * E + 64) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  topk_kernel<<<(unsigned)((rows + TOPK_WARPS - 1) / TOPK_WARPS), TOPK_WARPS * 32, smem, st>>>(
      logits, bias, H, S, E, K, score_func, nvg, tvg, route_norm, norm_eps, route_scale, probs, idx);
  return cudaGetLastError();
}

}  // namespace mhmoe
