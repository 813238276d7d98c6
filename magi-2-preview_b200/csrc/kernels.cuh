// Internal launcher declarations shared by the .cu files of libmhmoe.
#pragma once

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "mhmoe_common.cuh"

namespace mhmoe {

// Upper bound of 128-row tiles for R rows spread over n_experts groups.
// align: tiles per expert rounded up to a multiple of align (2 for the CTA-pair GEMM).
// Launch with programmatic stream serialization (see pdl_wait / pdl_trigger).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_pdl from a function returning cudaError_t: returns the launch error, if any.
#define MHMOE_LAUNCH_PDL(kernel, grid, block, smem, st, ...)                                              \
  do {                                                                                                     \
    const cudaError_t mhmoe_le_ = launch_pdl(kernel, dim3(grid), dim3(block), (size_t)(smem), st, __VA_ARGS__); \
    if (mhmoe_le_ != cudaSuccess) return mhmoe_le_;                                                        \
  } while (0)

inline int64_t mtiles_upper_bound(int64_t R, int64_t n_experts, int align = 1) {
  return (R + 127) / 128 + (int64_t)align * n_experts;
}

// Set-up that belongs to one device's context (kernel attributes such as the dynamic
// shared-memory limit, occupancy queries): run(f) calls f(device) the first time it runs
// with that device current and returns the recorded result on every later call there.
// A process that drives several GPUs (one host thread per device, or one thread switching
// devices) gets the set-up on each of them.
constexpr int MHMOE_MAX_DEVICES = 64;
struct PerDeviceOnce {
  std::mutex mu;
  bool done[MHMOE_MAX_DEVICES] = {};
  cudaError_t err[MHMOE_MAX_DEVICES] = {};
  template <class F>
  cudaError_t run(F&& f) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MHMOE_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      err[dev] = f(dev);
      done[dev] = true;
    }
    return err[dev];
  }
};

// ───────── expert-parallel peer buffers (ep_p2p.cu, combine.cu) ─────────
// Every rank allocates one buffer with this layout and maps every peer's (CUDA IPC):
//   flags  int32 [2][32]  arrival counters raised by peers: [0][s] records from s landed,
//                         [1][s] returns from s landed (one increment per layer call)
//   meta   int64 [32][2]  written by source s before its record flag: {record count,
//                         offset of this rank's group in s's send order}
//   done   int32 [8]      this rank's own last-CTA counters
//   rx     [n][cap][row_bytes]  records from source s at slot s*cap + j
//   back   [n*cap][dh] bf16     returned sums: row = this rank's send position (stores
//                               from the kernels), or d*cap + slot (copy-engine transport)
//   copy-engine transport only (local staging, moved by cudaMemcpyAsync):
//   slab   [n][cap][row_bytes]  this rank's records for destination d at d*cap + slot
//   mout   int64 [32][2]        {count, send offset} for destination d
//   stage  [n][cap][dh] bf16    sums of the records received from source s at s*cap + slot
constexpr int EP_MAX_RANKS = 32;
struct EpLayout {
  int64_t off_flags, off_meta, off_done, off_rx, off_back, off_slab, off_mout, off_stage, bytes;
};
inline EpLayout ep_layout(int n, int64_t cap, int dh, int64_t row_bytes) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  EpLayout L;
  L.off_flags = 0;
  L.off_meta = 256;
  L.off_done = 768;
  L.off_rx = 1024;
  L.off_back = L.off_rx + up((int64_t)n * cap * row_bytes);
  L.off_slab = L.off_back + up((int64_t)n * cap * dh * 2);
  L.off_mout = L.off_slab + up((int64_t)n * cap * row_bytes);
  L.off_stage = L.off_mout + 512;
  L.bytes = L.off_stage + up((int64_t)n * cap * dh * 2);
  return L;
}
struct EpPeers {
  uint8_t* base[EP_MAX_RANKS];
};
struct EpReturn {
  EpPeers peers;     // every rank's buffer base as mapped here (peers.base[me] = local)
  uint8_t* local;
  EpLayout layout;
  int64_t cap;
  int n, me;
  int* status;
  int stage;         // 1: sums into this rank's stage area (copy-engine transport), no flags
};

// Last-CTA detection: every thread's stores (peer stores included) are ordered at system
// scope before this CTA's increment of *done; returns true in the CTA that completes the
// grid, after which *done is back to 0.  Called by all threads of the block.
__device__ __forceinline__ bool ep_last_cta(int* done) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    if (last) {
      __threadfence_system();
      *done = 0;
    }
  }
  __syncthreads();
  return last != 0;
}

// permute.cu
// Sort chunks hold at least min_chunk flat entries (256 by default; larger chunks shrink the
// histogram scratch).
int sort_chunk_size(int64_t R, int64_t HE, int min_chunk = 256);
size_t global_sort_ws_bytes(int H, int S, int K, int E, int min_chunk = 256);
cudaError_t launch_global_sort(const float* probs, const int64_t* idx, int H, int S, int K, int E, void* ws,
                               int32_t* gather_ids, float* probs_sorted, int64_t* expert_offsets,
                               int32_t* row_of_flat, int* status, cudaStream_t st, int min_chunk = 256);
cudaError_t launch_tile_tables(const int64_t* expert_offsets, int HE, int64_t max_tiles, int* cu_tiles,
                               int* tile_expert, int* tile_row0, int* tile_rows, int* status, cudaStream_t st,
                               int align = 1);
size_t token_rows_ws_bytes(int64_t T);
cudaError_t launch_token_rows(const int32_t* gather_ids, int64_t max_mtiles, const int* cu_tiles, int HE, int E,
                              int S, int H, const int* tile_expert, const int* tile_row0, const int* tile_rows,
                              void* ws, int32_t* tok_offsets, int32_t* tok_rows, int* status, cudaStream_t st);

// quant.cu
cudaError_t launch_group_rows(const uint8_t* xq, int64_t xq_pitch, const uint8_t* xsf, int64_t xsf_pitch,
                              const uint8_t* xg, int64_t xg_pitch, int64_t T, int dh, int H, int E_per_head,
                              const int32_t* gather_ids, const int* cu_tiles, int HE, int64_t max_mtiles,
                              const int* tile_expert, const int* tile_row0, const int* tile_rows, uint8_t* a_data,
                              uint8_t* a_sf, float* a_gscale, int* status, cudaStream_t st);
// Fused quantise + group of x into the padded A operand through the inverse map (tok_rows
// with tok_offsets or k_fixed); dh <= quant_scatter_max_dh(), dh % 64 == 0.
int quant_scatter_max_dh();
cudaError_t launch_quant_scatter(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh,
                                 const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R,
                                 const int32_t* pad_of_row, int64_t rows, uint8_t* a_data, uint8_t* a_sf,
                                 float* a_gscale, int* status, cudaStream_t st);
cudaError_t launch_quant_tokens(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh,
                                uint8_t* xq, uint8_t* xsf, float* xg, cudaStream_t st);
cudaError_t launch_quantize_rows(const __nv_bfloat16* x, int64_t pitch, int64_t M, int K, uint8_t* data, uint8_t* sf,
                                 float* gscale, cudaStream_t st);
cudaError_t launch_pack_weights(int kind, const __nv_bfloat16* w0, const __nv_bfloat16* w1, int n_experts, int dh,
                                int de, uint8_t* data, uint8_t* sf, float* gscale, float* amax, cudaStream_t st);

// route.cu
cudaError_t launch_router_logits(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, const float* gate, int S, int H,
                                 int dh, int E, float* logits, cudaStream_t st);
cudaError_t launch_topk(const float* logits, const float* bias, int H, int S, int E, int K, int score_func, int nvg,
                        int tvg, int route_norm, float norm_eps, float route_scale, float* probs, int64_t* idx,
                        cudaStream_t st);

// combine.cu
// sorted row -> padded row
cudaError_t launch_pad_rows(const int* cu_tiles, int HE, int64_t max_mtiles, const int* tile_row0,
                            const int* tile_rows, int32_t* pad_of_row, cudaStream_t st);
cudaError_t launch_combine(const __nv_bfloat16* P, const int32_t* pad_of_row, int dh, int S, int H,
                           const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R,
                           int64_t P_rows, __nv_bfloat16* y, int64_t sy_s, int64_t sy_h, cudaStream_t st);

// capi.cu: text returned by mhmoe_last_error() on this host thread
void set_last_error(const std::string& msg);

// ffn.cu
int num_sms();
size_t ffn_workspace_bytes(int64_t R, int64_t T, int dh, int de, int HE);
int ffn_nvfp4(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh, int de, int HE, int64_t R,
              const int32_t* gather_ids, const float* probs_sorted, const int64_t* expert_offsets,
              const uint8_t* gu_data, const uint8_t* gu_sf, const float* gu_gscale, const uint8_t* dn_data,
              const uint8_t* dn_sf, const float* dn_gscale, const int32_t* tok_rows, const int32_t* tok_offsets,
              int k_fixed, void* workspace, __nv_bfloat16* y, int64_t sy_s, int64_t sy_h, int* status,
              uint64_t timeout_ns, const cudaEvent_t* events, cudaStream_t st, cudaError_t* cerr,
              const uint8_t* xq_in = nullptr, const uint8_t* xsf_in = nullptr, const uint8_t* xg_in = nullptr,
              int64_t xq_pitch = 0, int64_t xsf_pitch = 0, int64_t xg_pitch = 0, const EpReturn* ret = nullptr,
              bool atomic_scatter = false);

// combine.cu: y[s, h, 0:dh] = 0 for every (s, h)
cudaError_t launch_zero_rows(__nv_bfloat16* y, int S, int H, int dh, int64_t sy_s, int64_t sy_h, cudaStream_t st);

// combine.cu (expert-parallel return)
cudaError_t launch_combine_return(const __nv_bfloat16* P, const int32_t* pad_of_row, int dh,
                                  const int32_t* tok_rows, int k_fixed, int64_t R, int64_t P_rows, const EpReturn& r,
                                  cudaStream_t st);

// ep_p2p.cu
cudaError_t launch_ep_send_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                                   const int64_t* idx, const float* probs, int K, int E, int E_loc,
                                   const int32_t* send_key, const int64_t* send_offsets, int n, int me, int64_t cap,
                                   const EpPeers& peers, uint8_t* local, int* status, cudaStream_t st,
                                   bool stage = false);
cudaError_t launch_ep_push(uint8_t* local, int kind, int n, int me, int64_t cap, int dh, int K, const EpPeers& peers,
                           cudaStream_t st);
cudaError_t launch_ep_wait(const uint8_t* local, int kind, int n, int target, uint64_t timeout_ns, int* status,
                           cudaStream_t st);
cudaError_t launch_ep_unpack_slots(const uint8_t* local, int n, int64_t cap, int dh, int K, int E_loc,
                                   int64_t* idx, float* probs, int* status, cudaStream_t st);

// ep.cu
int64_t ep_row_bytes(int dh, int K);
cudaError_t launch_ep_dest(const int64_t* idx, int H, int S, int K, int E, int n_ranks, int E_loc, int64_t* dest,
                           int* status, cudaStream_t st);
cudaError_t launch_ep_pack(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                           const int64_t* idx, const float* probs, int K, int E, int E_loc, const int32_t* send_key,
                           const int64_t* send_offsets, int n_ranks, int64_t R_send, uint8_t* send, cudaStream_t st);
cudaError_t launch_ep_unpack(const uint8_t* recv, int64_t R, int dh, int K, int E_loc, int64_t* idx, float* probs,
                             int* status, cudaStream_t st);

// ffn.cu (continued)
int gemm_nvfp4_raw(const uint8_t* a_data, const uint8_t* a_sf, int n_mtiles, const int32_t* tile_expert,
                   const uint8_t* b_data, const uint8_t* b_sf, int n_experts, int N, int K, float* out, int* status,
                   uint64_t timeout_ns, cudaStream_t st, cudaError_t* cerr);
cudaError_t encode_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows,
                              uint32_t box_inner, uint32_t box_rows);
cudaError_t encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                           uint64_t inner, uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                           uint32_t box_rows, bool swizzle128 = true);

// route_small.cu: the router for batches of a few 128-token tiles (cluster split of the
// reduction dimension, CUDA cores); same contract as router_tc
bool router_small_supported(int S, int H, int dh, int E, int K);
cudaError_t launch_router_small(const __nv_bfloat16* x, int64_t sx_s, const __nv_bfloat16* planes, int nsplit,
                                int S, int H, int dh, int E, int K, int score_func, const float* logit_bias,
                                const float* bias, int route_norm, float norm_eps, float route_scale, float* probs,
                                int64_t* idx, float* logits, cudaStream_t st);

// norm.cu
cudaError_t launch_rmsnorm_modality(const __nv_bfloat16* x, int64_t sx, const float* w, const int32_t* cu_groups,
                                    int n_groups, int64_t rows, int dim, float eps, float weight_bias,
                                    __nv_bfloat16* y, int64_t sy, cudaStream_t st);

// wait_selftest.cu
cudaError_t launch_wait_selftest(const int* flag, int expected, int mode, uint64_t timeout_ns, int* status,
                                 int64_t* elapsed_ns, cudaStream_t st);

// router_tc.cu
cudaError_t launch_split_gate(const float* gate, int64_t HE, int dh, int nsplit, __nv_bfloat16* out, int* flags,
                              cudaStream_t st);
int router_tc(const __nv_bfloat16* x, int64_t sx_s, const __nv_bfloat16* gate_planes, int nsplit, int S, int H,
              int dh, int E, int K, int score_func, const float* logit_bias, const float* bias, int route_norm,
              float norm_eps, float route_scale, float* probs, int64_t* idx, float* logits, int* status,
              cudaStream_t st, cudaError_t* cerr);

}  // namespace mhmoe
