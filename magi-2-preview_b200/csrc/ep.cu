// Expert-parallel (token -> expert) dispatch support kernels.
//
// The reference shards heads across the EP group and moves the whole activation with
// one all_to_all_single each way (inference/model/magi2_preview.py:3277-3327).  Here the
// flattened experts [0, H*E) are split into contiguous per-rank ranges of E_loc experts
// and only routed token rows travel, once per destination rank, in NVFP4:
//
//   ep_dest_kernel    key t = h*S + s (a (head, token) row): dest[t, d] = d when any of
//                     its K experts lives on rank d, else -1.  A stable sort of these
//                     entries by d gives the send order (grouped by destination).
//   ep_pack_kernel    send row j -> one packed record: the token row's NVFP4 data
//                     (dh/2 B), its scales (dh/16 B) and a meta block {g, count, pad,
//                     K x (local expert, prob)} listing the experts of that rank.
//   ep_unpack_kernel  received records -> local expert ids int64 [R, K] (-1 past the
//                     count) and probs [R, K]; the NVFP4 data is read in place.
#include "kernels.cuh"

namespace mhmoe {

__global__ void ep_dest_kernel(const int64_t* __restrict__ idx, int H, int S, int K, int E, int n_ranks, int E_loc,
                               int64_t* __restrict__ dest, int* __restrict__ status) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // key = h*S + s
  if (t >= (int64_t)H * S) return;
  const int h = (int)(t / S);
  uint32_t mask = 0;                                                  // n_ranks <= 32
  for (int k = 0; k < K; ++k) {
    const int64_t e = idx[t * K + k];
    if (e < 0 || e >= E) {
      if (e >= E) record_error(status, MHMOE_ERR_ARGS);
      continue;
    }
    mask |= 1u << (int)((h * (int64_t)E + e) / E_loc);
  }
  for (int d = 0; d < n_ranks; ++d) dest[t * n_ranks + d] = (mask >> d) & 1u ? d : -1;
}

// One warp per send row.
__global__ void ep_pack_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xsf,
                               const float* __restrict__ xg, int H, int S, int dh, const int64_t* __restrict__ idx,
                               const float* __restrict__ probs, int K, int E, int E_loc,
                               const int32_t* __restrict__ send_key, const int64_t* __restrict__ send_offsets,
                               int n_ranks, int64_t R_send, uint8_t* __restrict__ send, int64_t row_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (j >= R_send || j >= send_offsets[n_ranks]) return;
  int d = 0;
  while (d + 1 < n_ranks && send_offsets[d + 1] <= j) ++d;            // destination of row j
  const int64_t t = send_key[j];                                       // h*S + s
  const int h = (int)(t / S), s = (int)(t % S);
  const int64_t q = (int64_t)s * H + h;                                // quantised token row
  uint8_t* row = send + j * row_bytes;
  const uint4* src = reinterpret_cast<const uint4*>(xq + q * (dh / 2));
  uint4* dst = reinterpret_cast<uint4*>(row);
  for (int i = lane; i < dh / 32; i += 32) dst[i] = src[i];
  const uint4* ssrc = reinterpret_cast<const uint4*>(xsf + q * (dh / 16));
  uint4* sdst = reinterpret_cast<uint4*>(row + dh / 2);
  for (int i = lane; i < dh / 256; i += 32) sdst[i] = ssrc[i];
  if (lane == 0) {
    uint8_t* meta = row + dh / 2 + dh / 16;
    int c = 0;
    int2* pairs = reinterpret_cast<int2*>(meta + 16);
    for (int k = 0; k < K; ++k) {
      const int64_t e = idx[t * K + k];
      if (e < 0 || e >= E) continue;
      const int64_t ge = (int64_t)h * E + e;
      if (ge / E_loc == d) pairs[c++] = make_int2((int)(ge % E_loc), __float_as_int(probs[t * K + k]));
    }
    for (int k = c; k < K; ++k) pairs[k] = make_int2(-1, 0);
    *reinterpret_cast<float4*>(meta) = make_float4(xg[q], __int_as_float(c), 0.f, 0.f);
  }
}

__global__ void ep_unpack_kernel(const uint8_t* __restrict__ recv, int64_t R, int64_t row_bytes, int dh, int K,
                                 int E_loc, int64_t* __restrict__ idx, float* __restrict__ probs,
                                 int* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const uint8_t* meta = recv + i * row_bytes + dh / 2 + dh / 16;
  const int c = __float_as_int(reinterpret_cast<const float4*>(meta)->y);
  const int2* pairs = reinterpret_cast<const int2*>(meta + 16);
  for (int k = 0; k < K; ++k) {
    int e = -1;
    float p = 0.f;
    if (k < c) {
      const int2 pr = pairs[k];
      e = pr.x;
      p = __int_as_float(pr.y);
      if (e < 0 || e >= E_loc) {
        record_error(status, MHMOE_ERR_ARGS);
        e = -1;
      }
    }
    idx[i * K + k] = e;
    probs[i * K + k] = p;
  }
}

int64_t ep_row_bytes(int dh, int K) { return dh / 2 + dh / 16 + ((16 + 8 * (int64_t)K + 15) / 16) * 16; }

cudaError_t launch_ep_dest(const int64_t* idx, int H, int S, int K, int E, int n_ranks, int E_loc, int64_t* dest,
                           int* status, cudaStream_t st) {
  const int64_t T = (int64_t)H * S;
  ep_dest_kernel<<<(unsigned)((T + 255) / 256), 256, 0, st>>>(idx, H, S, K, E, n_ranks, E_loc, dest, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                           const int64_t* idx, const float* probs, int K, int E, int E_loc, const int32_t* send_key,
                           const int64_t* send_offsets, int n_ranks, int64_t R_send, uint8_t* send, cudaStream_t st) {
  ep_pack_kernel<<<(unsigned)((R_send + 7) / 8), 256, 0, st>>>(xq, xsf, xg, H, S, dh, idx, probs, K, E, E_loc,
                                                               send_key, send_offsets, n_ranks, R_send, send,
                                                               ep_row_bytes(dh, K));
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const uint8_t* recv, int64_t R, int dh, int K, int E_loc, int64_t* idx, float* probs,
                             int* status, cudaStream_t st) {
  ep_unpack_kernel<<<(unsigned)((R + 255) / 256), 256, 0, st>>>(recv, R, ep_row_bytes(dh, K), dh, K, E_loc, idx,
                                                                probs, status);
  return cudaGetLastError();
}

}  // namespace mhmoe
