// Router for small batches: the fused router's contract (fp32-accurate logits, scoring,
// +expert_bias for selection, top-k sorted descending with ties to the lower expert, L1
// normalisation, route_scale; CoreMultiHeadMoE._route, inference/model/magi2_preview.py:
// 2588-2601 and inference/flash_mh_moe/route.py:28-148) for batches too small to occupy
// the GPU with one 128-token tensor-core tile per SM.
//
// At 256 tokens the tensor-core router runs two CTAs, each streaming 128 x dh of x and
// the whole gate through one SM (~50 us).  Here a cluster of 8 CTAs splits the reduction
// dimension of a 32-token tile: CTA r accumulates x[:, r*dh/8 : (r+1)*dh/8] against the
// same slice of the gate, on the CUDA cores, as an fp32 FMA chain in ascending k of the
// bf16 x values and the fp32 gate (rebuilt exactly from its bf16 planes: their sum is the
// fp32 weight, each partial sum representable), with the slice streamed through shared
// memory by asynchronous copies.  One FMA per (token, expert, k) whatever the number of
// planes; the result is the fp32 dot product to rounding.  The leader CTA sums
// the eight partial tiles through distributed shared memory in rank order (run-to-run
// identical), then scores and selects, one warp per token.  No scratch memory.
#include "kernels.cuh"

namespace mhmoe {

constexpr int RS_TOK = 32;            // tokens per cluster tile
constexpr int RS_SPLIT = 8;           // CTAs per cluster (reduction-dimension split)
constexpr int RS_SMEM_MAX = 200 * 1024;
constexpr int RS_THREADS = 256;

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Warp-wide argmax: larger value wins, ties to the smaller index.
__device__ __forceinline__ void rs_argmax(float& v, int& i) {
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// EP = experts per lane (E <= 32 * EP).  The CTA's reduction slice is streamed in chunks of
// kch elements through two shared-memory buffers with asynchronous 16-B copies (the next
// chunk loads while this one is consumed), kept as bf16: x [32][kch + 8] and the gate
// planes [nsplit][32*EP][kch + 8].  The row pitch (kch + 8) * 2 B is 16 mod 128 B, so the
// 16-B reads of eight consecutive experts hit distinct banks.
template <int EP>
__global__ void __cluster_dims__(RS_SPLIT, 1, 1) __launch_bounds__(RS_THREADS, 1)
    router_small_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx_s, const __nv_bfloat16* __restrict__ planes,
                        int nsplit, int S, int H, int dh, int E, int K, int score_func,
                        const float* __restrict__ logit_bias, const float* __restrict__ bias, int route_norm,
                        float norm_eps, float route_scale, float* __restrict__ probs, int64_t* __restrict__ idx,
                        float* __restrict__ logits, int kch) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float rs_smem[];
  constexpr int EPAD = 32 * EP;
  float* red = rs_smem;                                   // [RS_TOK][EPAD] partial (leader: final) logits
  const int pitch = kch + 8;                              // bf16 elements per buffered row
  const int buf_elems = (RS_TOK + nsplit * EPAD) * pitch;
  __nv_bfloat16* bufs = reinterpret_cast<__nv_bfloat16*>(red + RS_TOK * EPAD);   // 2 x [x rows | gate rows]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const int tiles_per_head = (S + RS_TOK - 1) / RS_TOK;
  const int tile = blockIdx.x / RS_SPLIT;
  const int h = tile / tiles_per_head;
  const int s0 = (tile % tiles_per_head) * RS_TOK;
  const int kspan = dh / RS_SPLIT;
  const int k_begin = (int)rank * kspan;
  const int64_t prow = (int64_t)nsplit * dh;              // plane row pitch (elements)
  const int nch = kspan / kch;
  const int vpr = kch / 8;                                // 16-B pieces per buffered row

  auto issue = [&](int c) {
    __nv_bfloat16* buf = bufs + (size_t)(c & 1) * buf_elems;
    const int k0 = k_begin + c * kch;
    const int rows = RS_TOK + nsplit * E;
    for (int u = tid; u < rows * vpr; u += RS_THREADS) {
      const int row = u / vpr, v = u % vpr;
      const int k = k0 + 8 * v;
      const __nv_bfloat16* src;
      uint32_t nbytes = 16;
      __nv_bfloat16* dst;
      if (row < RS_TOK) {                                  // x row of token s0 + row
        const int s = s0 + row;
        src = s < S ? x + (int64_t)s * sx_s + (int64_t)h * dh + k : x;
        nbytes = s < S ? 16u : 0u;                         // zero-filled past the batch
        dst = buf + (size_t)row * pitch + 8 * v;
      } else {                                             // plane p of expert e
        const int pe = row - RS_TOK, p = pe / E, e = pe % E;
        src = planes + (int64_t)(h * E + e) * prow + (int64_t)((k / 64) * nsplit + p) * 64 + k % 64;
        dst = buf + (size_t)(RS_TOK + p * EPAD + e) * pitch + 8 * v;
      }
      cp_async16(smem_u32(dst), src, nbytes);
    }
    cp_async_commit();
  };

  float acc[4][EP];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < EP; ++j) acc[i][j] = 0.f;

  issue(0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) {
      issue(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* buf = bufs + (size_t)(c & 1) * buf_elems;
    for (int kk = 0; kk < kch; kk += 8) {
      float xa[4][8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 raw = *reinterpret_cast<const uint4*>(buf + (size_t)(warp * 4 + i) * pitch + kk);
        const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(r2[q]);
          xa[i][2 * q] = f.x;
          xa[i][2 * q + 1] = f.y;
        }
      }
#pragma unroll
      for (int j = 0; j < EP; ++j) {
        const int e = lane + 32 * j;
        if (e >= E) continue;
        // the fp32 gate weights k .. k+7 of expert e: the sum of its planes, plane by plane
        float gv[8];
        for (int p = 0; p < nsplit; ++p) {
          const uint4 raw = *reinterpret_cast<const uint4*>(buf + (size_t)(RS_TOK + p * EPAD + e) * pitch + kk);
          const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 g = __bfloat1622float2(r2[q]);
            gv[2 * q] = p ? __fadd_rn(gv[2 * q], g.x) : g.x;
            gv[2 * q + 1] = p ? __fadd_rn(gv[2 * q + 1], g.y) : g.y;
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i][j] = __fmaf_rn(xa[i][q], gv[q], acc[i][j]);
      }
    }
    __syncthreads();                        // this buffer is refilled by chunk c + 2
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < EP; ++j) red[(warp * 4 + i) * EPAD + lane + 32 * j] = acc[i][j];
  cluster_sync();                         // every partial tile written

  if (rank == 0) {
    // fixed-order sum of the eight partials (rank 0 first), plus the optional logit bias
    const uint32_t red_s = smem_u32(red);
    uint32_t remote[RS_SPLIT];
#pragma unroll
    for (int r = 0; r < RS_SPLIT; ++r) remote[r] = mapa_shared(red_s, (uint32_t)r);
    for (int u = tid; u < RS_TOK * E; u += RS_THREADS) {
      const int t = u / E, e = u % E;
      const int o = t * EPAD + e;
      float v = red[o];
#pragma unroll
      for (int r = 1; r < RS_SPLIT; ++r) v += ld_dsmem_f32(remote[r] + (uint32_t)o * 4u);
      if (logit_bias) v = __fadd_rn(v, logit_bias[(int64_t)h * E + e]);
      red[o] = v;
    }
  }
  cluster_sync();                         // the leader has read every partial: the others may exit
  if (rank != 0) return;
  __syncthreads();

  // scoring and top-k: one warp per token
  for (int t = warp; t < RS_TOK; t += RS_THREADS / 32) {
    const int s = s0 + t;
    if (s >= S) break;
    const int64_t row = (int64_t)h * S + s;
    const float* lg = red + t * EPAD;
    if (logits)
      for (int e = lane; e < E; e += 32) logits[row * E + e] = lg[e];
    float mx = -INFINITY, sum = 0.f;
    if (score_func == 0) {
      for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      for (int e = lane; e < E; e += 32) sum += expf(lg[e] - mx);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    float sc[EP], sel[EP];
#pragma unroll
    for (int j = 0; j < EP; ++j) {
      const int e = lane + 32 * j;
      sc[j] = 0.f;
      sel[j] = -INFINITY;
      if (e < E) {
        const float l = lg[e];
        sc[j] = score_func == 0 ? __fdiv_rn(expf(l - mx), sum) : __fdiv_rn(1.0f, 1.0f + expf(-l));
        sel[j] = bias ? __fadd_rn(sc[j], bias[(int64_t)h * E + e]) : sc[j];
      }
    }
    float my_p = 0.f;
    int my_i = 0;
    for (int k = 0; k < K; ++k) {
      float v = -INFINITY;
      int vi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EP; ++j) {
        const int e = lane + 32 * j;
        if (e < E && (sel[j] > v || (sel[j] == v && e < vi))) {
          v = sel[j];
          vi = e;
        }
      }
      rs_argmax(v, vi);
      if (vi >= E) vi = 0;                  // every remaining value is NaN: deterministic fallback
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < EP; ++j)
        if (lane + 32 * j == vi) {
          p = sc[j];
          sel[j] = -INFINITY;               // taken (never selected again: -inf < any score)
        }
      p = __shfl_sync(0xffffffffu, p, vi & 31);
      if (lane == k) {
        my_p = p;
        my_i = vi;
      }
    }
    if (route_norm) {
      float a = lane < K ? fabsf(my_p) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      my_p = __fdiv_rn(my_p, fmaxf(a, norm_eps));
    }
    if (lane < K) {
      probs[row * K + lane] = __fmul_rn(my_p, route_scale);
      idx[row * K + lane] = my_i;
    }
  }
}

// Largest chunk (a multiple of 16 dividing the CTA's slice) whose two buffers fit.
static int rs_chunk(int dh, int E, int nsplit, size_t* smem) {
  const int epad = E <= 32 ? 32 : E <= 64 ? 64 : E <= 128 ? 128 : 256;
  const int kspan = dh / RS_SPLIT;
  for (int kch = kspan; kch >= 16; kch -= 16) {
    if (kspan % kch) continue;
    const size_t bytes = sizeof(float) * RS_TOK * epad + 2 * sizeof(__nv_bfloat16) * (RS_TOK + (size_t)nsplit * epad) *
                                                             (kch + 8);
    if (bytes <= RS_SMEM_MAX) {
      if (smem) *smem = bytes;
      return kch;
    }
  }
  return 0;
}

bool router_small_supported(int S, int H, int dh, int E, int K) {
  const int tc_tiles = H * ((S + 127) / 128);
  return tc_tiles * 4 <= num_sms() && dh % (RS_SPLIT * 16) == 0 && E <= 256 && K <= 32 && K <= E &&
         rs_chunk(dh, E, 3, nullptr) > 0;
}

cudaError_t launch_router_small(const __nv_bfloat16* x, int64_t sx_s, const __nv_bfloat16* planes, int nsplit,
                                int S, int H, int dh, int E, int K, int score_func, const float* logit_bias,
                                const float* bias, int route_norm, float norm_eps, float route_scale, float* probs,
                                int64_t* idx, float* logits, cudaStream_t st) {
  if (S == 0) return cudaSuccess;
  const int ep0 = (E + 31) / 32;
  const int ep = ep0 <= 1 ? 1 : ep0 <= 2 ? 2 : ep0 <= 4 ? 4 : 8;    // instantiated lane widths
  size_t smem = 0;
  const int kch = rs_chunk(dh, E, nsplit, &smem);
  if (kch == 0) return cudaErrorInvalidValue;
  const int tiles = H * ((S + RS_TOK - 1) / RS_TOK);
  const dim3 grid(tiles * RS_SPLIT);
#define MHMOE_RS_CASE(N)                                                                                          \
  case N: {                                                                                                       \
    static PerDeviceOnce once;                                                                                    \
    const cudaError_t a = once.run([](int) {                                                                      \
      return cudaFuncSetAttribute(router_small_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, RS_SMEM_MAX); \
    });                                                                                                           \
    if (a != cudaSuccess) return a;                                                                               \
    MHMOE_LAUNCH_PDL(router_small_kernel<N>, grid, RS_THREADS, smem, st, x, sx_s, planes, nsplit, S, H, dh, E, K,  \
                     score_func, logit_bias, bias, route_norm, norm_eps, route_scale, probs, idx, logits, kch);  \
    break;                                                                                                        \
  }
  switch (ep) {
    MHMOE_RS_CASE(1)
    MHMOE_RS_CASE(2)
    MHMOE_RS_CASE(4)
    MHMOE_RS_CASE(8)
    default:
      return cudaErrorInvalidValue;
  }
#undef MHMOE_RS_CASE
  return cudaGetLastError();
}

}  // namespace mhmoe
