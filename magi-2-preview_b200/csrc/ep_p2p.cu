// Expert-parallel exchange over NVLink peer memory (no host synchronisation, no NCCL).
//
// Replaces the two all_to_all_single calls of ep_dispatch / ep_undispatch
// (inference/model/magi2_preview.py:3277-3327) with token->expert records that the
// kernels write straight into the destination rank's buffer (CUDA IPC mapping, plain
// stores over NVLink), each kernel ending with a system-scope release of a per-source
// arrival counter in every peer.  Buffer layout: EpLayout (kernels.cuh).
//
//   ep_send_records_kernel   send row j (grouped by destination d, from the counting sort)
//                            -> record at d's rx[me*cap + j - send_offsets[d]], destinations
//                            interleaved across warps; the last
//                            CTA writes {count, send offset} into d's meta[me] and raises
//                            d's records flag [0][me].
//   ep_wait_kernel           bounded wait until every source's flag of one kind reaches
//                            the layer call's epoch (MHMOE_ERR_PEER on expiry).
//   ep_unpack_slots_kernel   rx slot -> local expert ids / probs [n*cap, K], -1 for slots
//                            past the source's count.
// The receiver's FFN ends in combine_return_kernel (combine.cu), which writes each
// record's bf16 sum into the source's back area and raises the return flag [1][me].
//
// Ordering argument: a source writes a destination's rx/meta only in layer call t+1,
// after it has seen that destination's return flag of call t, which the destination
// raises after every kernel that reads rx/meta for call t; a destination writes a
// source's back area for call t+1 only after receiving the source's call-t+1 records,
// which the source sends after its combine of call t has read back.
#include <cstdlib>

#include "kernels.cuh"

namespace mhmoe {

// One warp per send row; grid-stride over the send rows (count read on the device).
__global__ void ep_send_records_kernel(const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xsf,
                                       const float* __restrict__ xg, int H, int S, int dh,
                                       const int64_t* __restrict__ idx, const float* __restrict__ probs, int K, int E,
                                       int E_loc, const int32_t* __restrict__ send_key,
                                       const int64_t* __restrict__ send_offsets, int n, int me, int64_t cap,
                                       int64_t row_bytes, const EpPeers peers, EpLayout L, uint8_t* local,
                                       int* status, int bulk, int stage) {
  extern __shared__ __align__(128) uint8_t rec_stage[];
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  int issued = 0;
  // Work item w -> destination d = (w + me) % n, its k = w / n-th row: consecutive warps
  // write to different ranks (and each rank starts at a different one), so every link
  // carries traffic at once instead of all ranks filling one destination after another.
  const int64_t items = (int64_t)n * cap;
  for (int64_t w = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); w < items; w += (int64_t)gridDim.x * warps) {
    const int d = (int)((w + me) % n);
    const int64_t slot = w / n;
    const int64_t cnt = send_offsets[d + 1] - send_offsets[d];
    if (slot >= cnt) continue;
    if (cnt > cap) {                                                    // more rows than the buffer holds
      if (lane == 0) record_error(status, MHMOE_ERR_CAPACITY);
      continue;
    }
    const int64_t j = send_offsets[d] + slot;
    const int64_t t = send_key[j];                                      // h*S + s
    const int h = (int)(t / S), s = (int)(t % S);
    const int64_t q = (int64_t)s * H + h;                               // quantised token row
    // stage: into this rank's slab for destination d (moved later by the copy engines)
    uint8_t* const dst_row = stage ? local + L.off_slab + ((int64_t)d * cap + slot) * row_bytes
                                   : peers.base[d] + L.off_rx + ((int64_t)me * cap + slot) * row_bytes;
    // bulk: the record is built in one of the warp's two shared-memory buffers and sent with
    // one bulk copy (the buffer's previous copy must have read it out first)
    uint8_t* row = dst_row;
    if (bulk) {
      row = rec_stage + ((size_t)(threadIdx.x >> 5) * 2 + (issued & 1)) * row_bytes;
      if (issued >= 2) {
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
      }
    }
    const uint4* src = reinterpret_cast<const uint4*>(xq + q * (dh / 2));
    uint4* dst = reinterpret_cast<uint4*>(row);
    for (int i = lane; i < dh / 32; i += 32) dst[i] = src[i];
    const uint4* ssrc = reinterpret_cast<const uint4*>(xsf + q * (dh / 16));
    uint4* sdst = reinterpret_cast<uint4*>(row + dh / 2);
    for (int i = lane; i < dh / 256; i += 32) sdst[i] = ssrc[i];
    // meta: lane k < K builds pair k of this rank's experts (in k order), lane 0 the header
    int is_mine = 0;
    int2 pr = make_int2(-1, 0);
    if (lane < K) {
      const int64_t e = idx[t * K + lane];
      if (e >= 0 && e < E) {
        const int64_t ge = (int64_t)h * E + e;
        if (ge / E_loc == d) {
          is_mine = 1;
          pr = make_int2((int)(ge % E_loc), __float_as_int(probs[t * K + lane]));
        }
      }
    }
    const uint32_t mine = __ballot_sync(0xffffffffu, is_mine);
    int2* pairs = reinterpret_cast<int2*>(row + dh / 2 + dh / 16 + 16);
    if (is_mine) pairs[__popc(mine & ((1u << lane) - 1u))] = pr;       // compacted, k order kept
    const int c = __popc(mine);
    if (lane >= c && lane < K) pairs[lane] = make_int2(-1, 0);
    if (lane == 0)
      *reinterpret_cast<float4*>(row + dh / 2 + dh / 16) = make_float4(xg[q], __int_as_float(c), 0.f, 0.f);
    if (bulk) {
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        bulk_store(dst_row, smem_u32(row), (uint32_t)row_bytes);
        bulk_commit();
      }
      ++issued;
    }
  }
  if (bulk && lane == 0 && issued > 0) {
    bulk_wait_all();                 // records written at the destinations before the flag release
    fence_proxy_async_global();
  }
  if (stage) {                        // counts for the copies; no flags (the push raises them)
    if (blockIdx.x == 0)
      for (int d = threadIdx.x; d < n; d += blockDim.x) {
        int64_t* mo = reinterpret_cast<int64_t*>(local + L.off_mout) + 2 * d;
        mo[0] = send_offsets[d + 1] - send_offsets[d];
        mo[1] = send_offsets[d];
      }
    return;
  }
  if (ep_last_cta(reinterpret_cast<int*>(local + L.off_done)) && threadIdx.x == 0) {
    for (int d = 0; d < n; ++d) {
      int64_t* meta = reinterpret_cast<int64_t*>(peers.base[d] + L.off_meta) + 2 * me;
      meta[0] = send_offsets[d + 1] - send_offsets[d];
      meta[1] = send_offsets[d];
    }
    __threadfence_system();
    for (int d = 0; d < n; ++d) red_release_sys_add(reinterpret_cast<int*>(peers.base[d] + L.off_flags) + me, 1);
  }
}

__global__ void ep_wait_kernel(const int* flags, int n, int target, uint64_t timeout_ns, int* status) {
  const int s = threadIdx.x;
  if (s < n) flag_wait_geq(flags + s, target, status, MHMOE_ERR_PEER, timeout_ns);
}

__global__ void ep_unpack_slots_kernel(const uint8_t* __restrict__ local, EpLayout L, int n, int64_t cap,
                                       int64_t row_bytes, int dh, int K, int E_loc, int64_t* __restrict__ idx,
                                       float* __restrict__ probs, int* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * cap) return;
  const int src = (int)(i / cap);
  const int64_t slot = i % cap;
  const int64_t cnt = reinterpret_cast<const int64_t*>(local + L.off_meta)[2 * src];
  const bool ok = ld_volatile_i32(status) == 0 && cnt >= 0 && cnt <= cap && slot < cnt;
  const uint8_t* meta = local + L.off_rx + i * row_bytes + dh / 2 + dh / 16;
  const int c = ok ? __float_as_int(reinterpret_cast<const float4*>(meta)->y) : 0;
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

cudaError_t launch_ep_send_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                                   const int64_t* idx, const float* probs, int K, int E, int E_loc,
                                   const int32_t* send_key, const int64_t* send_offsets, int n, int me, int64_t cap,
                                   const EpPeers& peers, uint8_t* local, int* status, cudaStream_t st, bool stage) {
  const int64_t rb = ep_row_bytes(dh, K);
  const EpLayout L = ep_layout(n, cap, dh, rb);
  const int64_t items = (int64_t)n * cap;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, 4 * num_sms()));
  // bulk copies when MHMOE_EP_BULK=1 (two record buffers per warp, at most 6 KB each); the
  // default stores from registers measured as fast at 2 GPUs
  const char* env = std::getenv("MHMOE_EP_BULK");
  const int bulk = (env && env[0] == '1') && rb <= 6144 ? 1 : 0;
  const size_t smem = bulk ? (size_t)8 * 2 * rb : 0;
  if (bulk) {
    static PerDeviceOnce once;
    const cudaError_t e = once.run([](int) {
      return cudaFuncSetAttribute(ep_send_records_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  8 * 2 * 6144);
    });
    if (e != cudaSuccess) return e;
  }
  ep_send_records_kernel<<<(unsigned)blocks, 256, smem, st>>>(xq, xsf, xg, H, S, dh, idx, probs, K, E, E_loc,
                                                                     send_key, send_offsets, n, me, cap, rb, peers, L,
                                                                     local, status, bulk, stage ? 1 : 0);
  return cudaGetLastError();
}

// Raise this rank's flag of `kind` in every peer (after the copies before it in the stream).
__global__ void ep_flag_kernel(const EpPeers peers, int64_t off_flags, int kind, int n, int me) {
  const int d = threadIdx.x;
  if (d >= n) return;
  __threadfence_system();
  red_release_sys_add(reinterpret_cast<int*>(peers.base[d] + off_flags) + 32 * kind + me, 1);
}

// Copy-engine transport: one cudaMemcpyAsync per peer (whole slabs: the counts live on the
// device, the receiver reads them from the copied meta), then the flags.
//   kind 0: slab[d] -> d's rx[me], mout[d] -> d's meta[me]
//   kind 1: stage[s] -> s's back[me]
cudaError_t launch_ep_push(uint8_t* local, int kind, int n, int me, int64_t cap, int dh, int K, const EpPeers& peers,
                           cudaStream_t st) {
  const int64_t rb = ep_row_bytes(dh, K);
  const EpLayout L = ep_layout(n, cap, dh, rb);
  for (int i = 0; i < n; ++i) {
    const int d = (me + 1 + i) % n;        // every rank starts with a different peer
    cudaError_t e;
    if (kind == 0) {
      e = cudaMemcpyAsync(peers.base[d] + L.off_rx + (int64_t)me * cap * rb, local + L.off_slab + (int64_t)d * cap * rb,
                          (size_t)(cap * rb), cudaMemcpyDeviceToDevice, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(peers.base[d] + L.off_meta + 16 * me, local + L.off_mout + 16 * d, 16,
                            cudaMemcpyDeviceToDevice, st);
    } else {
      const int64_t rowb = (int64_t)dh * 2;
      e = cudaMemcpyAsync(peers.base[d] + L.off_back + (int64_t)me * cap * rowb,
                          local + L.off_stage + (int64_t)d * cap * rowb, (size_t)(cap * rowb), cudaMemcpyDeviceToDevice,
                          st);
    }
    if (e != cudaSuccess) return e;
  }
  ep_flag_kernel<<<1, 32, 0, st>>>(peers, L.off_flags, kind, n, me);
  return cudaGetLastError();
}

cudaError_t launch_ep_wait(const uint8_t* local, int kind, int n, int target, uint64_t timeout_ns, int* status,
                           cudaStream_t st) {
  const int* flags = reinterpret_cast<const int*>(local) + 32 * kind;    // EpLayout.off_flags == 0
  ep_wait_kernel<<<1, 32, 0, st>>>(flags, n, target, timeout_ns, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack_slots(const uint8_t* local, int n, int64_t cap, int dh, int K, int E_loc,
                                   int64_t* idx, float* probs, int* status, cudaStream_t st) {
  const int64_t rb = ep_row_bytes(dh, K);
  const EpLayout L = ep_layout(n, cap, dh, rb);
  const int64_t slots = (int64_t)n * cap;
  ep_unpack_slots_kernel<<<(unsigned)std::max<int64_t>(1, (slots + 255) / 256), 256, 0, st>>>(
      local, L, n, cap, rb, dh, K, E_loc, idx, probs, status);
  return cudaGetLastError();
}

}  // namespace mhmoe
