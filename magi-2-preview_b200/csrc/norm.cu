// Multi-modality RMSNorm: the pre-norm of MAGI-2's MoE layer.
//
//   y[t, :] = bf16( x[t, :] * rsqrt(mean(x[t, :]^2) + eps) * (w[m(t), :] + weight_bias) )
//
// in fp32, where m(t) is the modality group of row t: rows are grouped by modality
// ([cu_groups[m], cu_groups[m+1]) holds modality m, the layout MAGI-2's ModalityDispatcher
// gives), and w holds one fp32 weight row per modality.  Replaces MultiModalityRMSNorm's
// forward (inference/model/magi2_preview.py:497-623: single- and multi-modality paths,
// weight_bias = 1).
//
// One warp per row; 16-B vectorised loads and stores, the row kept in registers between
// the reduction and the scaling (dim <= 8192).  HBM-bound: reads dim*2 B and writes dim*2 B
// per row (the weight rows stay in L2).
#include "kernels.cuh"

namespace mhmoe {

constexpr int NORM_WARPS = 8;
constexpr int NORM_MAX_CHUNKS = 32;          // 16-B chunks per lane: dim <= 32 * 32 * 8 = 8192

template <int CHUNKS>
__global__ void __launch_bounds__(NORM_WARPS * 32)
    rmsnorm_modality_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, const float* __restrict__ w,
                            const int32_t* __restrict__ cu_groups, int n_groups, int64_t rows, int dim,
                            float eps, float weight_bias, __nv_bfloat16* __restrict__ y, int64_t sy) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NORM_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * sx);
  const int nchunk = dim / 8;
  uint4 v[CHUNKS];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nchunk ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(__fdiv_rn(ss, (float)dim) + eps);
  int m = 0;
  if (cu_groups)
    while (m + 1 < n_groups && row >= (int64_t)__ldg(cu_groups + m + 1)) ++m;
  const float4* wr = reinterpret_cast<const float4*>(w + (int64_t)m * dim);
  uint4* yr = reinterpret_cast<uint4*>(y + row * sy);
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    const int c = lane + 32 * i;
    if (c >= nchunk) break;
    const float4 w0 = __ldg(wr + 2 * c), w1 = __ldg(wr + 2 * c + 1);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
    uint32_t out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      const float a = __fmul_rn(__fmul_rn(f.x, r), __fadd_rn(wv[2 * j], weight_bias));
      const float b = __fmul_rn(__fmul_rn(f.y, r), __fadd_rn(wv[2 * j + 1], weight_bias));
      __nv_bfloat162 o2 = __floats2bfloat162_rn(a, b);
      out[j] = *reinterpret_cast<uint32_t*>(&o2);
    }
    yr[c] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

cudaError_t launch_rmsnorm_modality(const __nv_bfloat16* x, int64_t sx, const float* w, const int32_t* cu_groups,
                                    int n_groups, int64_t rows, int dim, float eps, float weight_bias,
                                    __nv_bfloat16* y, int64_t sy, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + NORM_WARPS - 1) / NORM_WARPS);
  const int chunks = (dim / 8 + 31) / 32;
  if (chunks <= 4) {
    MHMOE_LAUNCH_PDL(rmsnorm_modality_kernel<4>, grid, NORM_WARPS * 32, 0, st, x, sx, w, cu_groups, n_groups, rows,
                     dim, eps, weight_bias, y, sy);
  } else if (chunks <= 12) {
    MHMOE_LAUNCH_PDL(rmsnorm_modality_kernel<12>, grid, NORM_WARPS * 32, 0, st, x, sx, w, cu_groups, n_groups,
                     rows, dim, eps, weight_bias, y, sy);
  } else {
    MHMOE_LAUNCH_PDL(rmsnorm_modality_kernel<NORM_MAX_CHUNKS>, grid, NORM_WARPS * 32, 0, st, x, sx, w, cu_groups,
                     n_groups, rows, dim, eps, weight_bias, y, sy);
  }
  return cudaGetLastError();
}

}  // namespace mhmoe
