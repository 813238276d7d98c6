// Expert-parallel (token -> expert) dispatch support kernels.
//
// The reference shards heads across the EP group and moves the whole activation with
// one all_to_all_single each way (inference/model/magi2_preview.py:3277-3327).  Here the
// flattened experts [0, H*E) are split into contiguous per-rank ranges and only routed
// rows travel, as NVFP4 (dh/2 data bytes + dh/16 scale bytes + a 16-byte meta record):
//
//   ep_pack_kernel    sorted row r of the source -> send buffers (rows are already grouped
//                     by destination rank because expert ranges are contiguous):
//                     data/scales copied from the per-token quantised x, meta =
//                     {token row scale g, local expert id, routing prob, 0}.
//   ep_unpack_kernel  received meta -> g [R], local expert id as int64 [R], prob [R]
//                     (the inputs of the receiver's local sort and FFN).
#include "kernels.cuh"

namespace mhmoe {

// One warp per sorted row.
__global__ void ep_pack_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xsf,
                               const float* __restrict__ xg, int64_t T, int dh, int H, int E, int E_loc, int64_t R,
                               const int32_t* __restrict__ gather_ids, const float* __restrict__ probs_sorted,
                               const int64_t* __restrict__ expert_offsets, int HE, uint8_t* __restrict__ send_xq,
                               uint8_t* __restrict__ send_xsf, float4* __restrict__ send_meta,
                               int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= R) return;
  // expert of sorted row r: largest e with expert_offsets[e] <= r
  int lo = 0, hi = HE - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (expert_offsets[mid] <= r) lo = mid; else hi = mid - 1;
  }
  const int e = lo;
  const int s = gather_ids[r];
  const int64_t t = (int64_t)s * H + e / E;
  if (s < 0 || t >= T) {
    if (lane == 0) record_error(status, MHMOE_ERR_ARGS);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(xq + t * (dh / 2));
  uint4* dst = reinterpret_cast<uint4*>(send_xq + r * (dh / 2));
  for (int i = lane; i < dh / 32; i += 32) dst[i] = src[i];
  const uint4* ssrc = reinterpret_cast<const uint4*>(xsf + t * (dh / 16));
  uint4* sdst = reinterpret_cast<uint4*>(send_xsf + r * (dh / 16));
  for (int i = lane; i < dh / 256; i += 32) sdst[i] = ssrc[i];
  if (lane == 0) send_meta[r] = make_float4(xg[t], __int_as_float(e % E_loc), probs_sorted[r], 0.f);
}

__global__ void ep_unpack_kernel(const float4* __restrict__ meta, int64_t R, int E_loc, float* __restrict__ g,
                                 int64_t* __restrict__ local_expert, float* __restrict__ prob,
                                 int* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const float4 m = meta[i];
  int e = __float_as_int(m.y);
  if (e < 0 || e >= E_loc) {
    record_error(status, MHMOE_ERR_ARGS);
    e = 0;
  }
  g[i] = m.x;
  local_expert[i] = e;
  prob[i] = m.z;
}

cudaError_t launch_ep_pack(const uint8_t* xq, const uint8_t* xsf, const float* xg, int64_t T, int dh, int H, int E,
                           int E_loc, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                           const int64_t* expert_offsets, int HE, uint8_t* send_xq, uint8_t* send_xsf,
                           void* send_meta, int* status, cudaStream_t st) {
  ep_pack_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>(xq, xsf, xg, T, dh, H, E, E_loc, R, gather_ids,
                                                          probs_sorted, expert_offsets, HE, send_xq, send_xsf,
                                                          static_cast<float4*>(send_meta), status);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const void* meta, int64_t R, int E_loc, float* g, int64_t* local_expert, float* prob,
                             int* status, cudaStream_t st) {
  ep_unpack_kernel<<<(unsigned)((R + 255) / 256), 256, 0, st>>>(static_cast<const float4*>(meta), R, E_loc, g,
                                                                local_expert, prob, status);
  return cudaGetLastError();
}

}  // namespace mhmoe
