// extern "C" entry points of libmhmoe (declared in include/mhmoe.h).
//
// Each entry point validates shapes, strides and alignment on the host, checks the
// device architecture once per device, enqueues its kernels on the caller's stream and
// maps CUDA errors to mhmoe_status.  No entry point allocates device memory.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail_cuda(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return MHMOE_ERR_LAUNCH;
}

int fail_args(const char* what) {
  g_last_error = std::string("invalid argument: ") + what;
  return MHMOE_ERR_ARGS;
}

// sm_100 check, cached per device ordinal.
int check_arch() {
  static int cached[64];   // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    g_last_error = "no current CUDA device";
    return MHMOE_ERR_ARCH;
  }
  if (cached[dev] == 0) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cached[dev] = major == 10 ? 1 : 2;
  }
  if (cached[dev] != 1) {
    g_last_error = "libmhmoe requires an sm_100 (B200) device";
    return MHMOE_ERR_ARCH;
  }
  return MHMOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define MHMOE_CHECK_ARCH()          \
  do {                              \
    const int a_ = check_arch();    \
    if (a_ != MHMOE_OK) return a_;  \
  } while (0)

#define MHMOE_REQUIRE(cond)                   \
  do {                                        \
    if (!(cond)) return fail_args(#cond);     \
  } while (0)

}  // namespace

namespace mhmoe {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace mhmoe

using namespace mhmoe;

extern "C" {

int mhmoe_version(void) { return 1; }

const char* mhmoe_status_string(int status) {
  switch (status) {
    case MHMOE_OK: return "ok";
    case MHMOE_ERR_ARGS: return "invalid argument";
    case MHMOE_ERR_ARCH: return "unsupported device (sm_100 required)";
    case MHMOE_ERR_LAUNCH: return "CUDA launch/runtime error";
    case MHMOE_ERR_TIMEOUT: return "device-side wait timed out";
    case MHMOE_ERR_DRIVER: return "CUDA driver entry point or tensor-map encode failed";
    case MHMOE_ERR_PEER: return "expert-parallel peer wait timed out";
    case MHMOE_ERR_CAPACITY: return "size exceeds a compiled-in maximum";
    default: return "unknown status";
  }
}

const char* mhmoe_last_error(void) { return g_last_error.c_str(); }

int mhmoe_router_logits(const void* x, int64_t x_stride_s, int64_t x_stride_h, const float* gate, int S, int H,
                        int dh, int E, float* logits, void* stream) {
  MHMOE_REQUIRE(x && gate && logits);
  MHMOE_REQUIRE(S >= 0 && H > 0 && E > 0 && dh > 0 && dh % 32 == 0);
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  const cudaError_t e = launch_router_logits(static_cast<const __nv_bfloat16*>(x), x_stride_s, x_stride_h, gate, S,
                                             H, dh, E, logits, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "router_logits");
}

int mhmoe_router_prepare(const float* gate, int n_experts, int dh, int nsplit, void* planes, int* flags,
                         void* stream) {
  MHMOE_REQUIRE(gate && planes && n_experts > 0 && dh > 0 && dh % 64 == 0 && nsplit >= 1 && nsplit <= 3);
  MHMOE_CHECK_ARCH();
  const cudaError_t e = launch_split_gate(gate, n_experts, dh, nsplit, static_cast<__nv_bfloat16*>(planes), flags,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "router_prepare");
}

int mhmoe_route(const void* x, int64_t x_stride_s, int64_t x_stride_h, const void* planes, int nsplit, int S, int H,
                int dh, int E, int K, int score_func, const float* logit_bias, const float* expert_bias, int route_norm,
                float norm_eps, float route_scale, float* probs, int64_t* idx, float* logits, int* dev_status,
                void* stream) {
  MHMOE_REQUIRE(x && planes && probs && idx);
  MHMOE_REQUIRE(S >= 0 && H > 0 && dh > 0 && dh % 64 == 0 && E > 0 && E <= 256 && K > 0 && K <= 16 && K <= E);
  MHMOE_REQUIRE(nsplit >= 1 && nsplit <= 3 && (score_func == 0 || score_func == 1));
  MHMOE_REQUIRE(x_stride_h == dh && x_stride_s % 8 == 0 && x_stride_s >= (int64_t)H * dh && aligned16(x));
  MHMOE_REQUIRE(aligned16(planes));
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  cudaError_t ce = cudaSuccess;
  const int rc = router_tc(static_cast<const __nv_bfloat16*>(x), x_stride_s, static_cast<const __nv_bfloat16*>(planes),
                           nsplit, S, H, dh, E, K, score_func, logit_bias, expert_bias, route_norm, norm_eps,
                           route_scale, probs, idx, logits, dev_status, static_cast<cudaStream_t>(stream), &ce);
  if (rc == MHMOE_ERR_LAUNCH) return fail_cuda(ce, "route");
  if (rc == MHMOE_ERR_DRIVER) g_last_error = "cuTensorMapEncodeTiled failed (route)";
  return rc;
}

int mhmoe_topk(const float* logits, const float* expert_bias, int H, int S, int E, int K, int score_func,
               int num_virtual_group, int topk_virtual_group, int route_norm, float norm_eps, float route_scale,
               float* probs, int64_t* idx, void* stream) {
  MHMOE_REQUIRE(logits && probs && idx);
  MHMOE_REQUIRE(H > 0 && S >= 0 && E > 0 && E <= 1024 && K > 0 && K <= 32 && K <= E);
  MHMOE_REQUIRE(score_func == 0 || score_func == 1);
  if (num_virtual_group > 1) {
    MHMOE_REQUIRE(num_virtual_group <= 64 && E % num_virtual_group == 0);
    MHMOE_REQUIRE(topk_virtual_group > 0 && topk_virtual_group <= num_virtual_group);
  }
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  const cudaError_t e = launch_topk(logits, expert_bias, H, S, E, K, score_func, num_virtual_group,
                                    topk_virtual_group, route_norm, norm_eps, route_scale, probs, idx,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "topk");
}

size_t mhmoe_global_sort_workspace_bytes(int H, int S, int K, int E) { return global_sort_ws_bytes(H, S, K, E); }

int mhmoe_global_sort(const float* topk_probs, const int64_t* topk_idx, int H, int S, int K, int E,
                      void* workspace, int32_t* gather_ids, float* probs_sorted, int64_t* expert_offsets,
                      int32_t* row_of_flat, int* dev_status, void* stream) {
  MHMOE_REQUIRE(topk_probs && topk_idx && workspace && gather_ids && probs_sorted && expert_offsets);
  MHMOE_REQUIRE(H > 0 && S >= 0 && K > 0 && E > 0);
  MHMOE_REQUIRE((int64_t)H * E <= 12288);
  MHMOE_REQUIRE((int64_t)H * S * K < (int64_t)1 << 31);
  MHMOE_CHECK_ARCH();
  if (S == 0) {
    const cudaError_t e =
        cudaMemsetAsync(expert_offsets, 0, sizeof(int64_t) * (H * E + 1), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "global_sort");
  }
  const cudaError_t e = launch_global_sort(topk_probs, topk_idx, H, S, K, E, workspace, gather_ids, probs_sorted,
                                           expert_offsets, row_of_flat, dev_status,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "global_sort");
}

int64_t mhmoe_max_mtiles(int64_t R, int n_experts) { return mtiles_upper_bound(R, n_experts); }

size_t mhmoe_ffn_workspace_bytes(int64_t R, int S, int H, int dh, int de, int n_experts) {
  return ffn_workspace_bytes(R, (int64_t)S * H, dh, de, n_experts);
}

int mhmoe_pack_weights_nvfp4(int kind, const void* w0, const void* w1, int n_experts, int dh, int de,
                             uint8_t* data, uint8_t* sf, float* gscale, float* amax_scratch, void* stream) {
  MHMOE_REQUIRE(kind == 0 || kind == 1);
  MHMOE_REQUIRE(w0 && data && sf && gscale && amax_scratch);
  MHMOE_REQUIRE(kind == 1 || w1);
  MHMOE_REQUIRE(n_experts > 0 && dh > 0 && de > 0 && dh % 128 == 0 && de % 128 == 0);
  MHMOE_REQUIRE(aligned16(w0) && (kind == 1 || aligned16(w1)) && aligned16(data));
  MHMOE_CHECK_ARCH();
  const cudaError_t e = launch_pack_weights(kind, static_cast<const __nv_bfloat16*>(w0),
                                            static_cast<const __nv_bfloat16*>(w1), n_experts, dh, de, data, sf,
                                            gscale, amax_scratch, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "pack_weights_nvfp4");
}

static int ffn_entry(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh, int de,
                     int n_experts, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                     const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                     const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                     const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, void* workspace,
                     void* y, int64_t y_stride_s, int64_t y_stride_h, int* dev_status, uint64_t timeout_ns,
                     void* const* stage_events, void* stream, bool atomic, const char* what) {
  MHMOE_REQUIRE(x && y && expert_offsets && gu_data && gu_sf && gu_gscale && dn_data && dn_sf && dn_gscale);
  MHMOE_REQUIRE(S >= 0 && H > 0 && n_experts > 0 && n_experts % H == 0 && R >= 0);
  MHMOE_REQUIRE(dh % 256 == 0 && de % 256 == 0 && dh > 0 && de > 0);
  MHMOE_REQUIRE(R < ((int64_t)1 << 31) - 128 * (int64_t)n_experts);
  MHMOE_REQUIRE(aligned16(x) && x_stride_s % 8 == 0 && x_stride_h % 8 == 0);
  MHMOE_REQUIRE(aligned16(y) && y_stride_s % 8 == 0 && y_stride_h % 8 == 0);
  MHMOE_REQUIRE(aligned16(gu_data) && aligned16(dn_data) && aligned16(gu_sf) && aligned16(dn_sf));
  MHMOE_REQUIRE(tok_rows || !tok_offsets);
  MHMOE_REQUIRE(!tok_rows || tok_offsets || k_fixed > 0);
  MHMOE_CHECK_ARCH();
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (S == 0) return MHMOE_OK;
  if (R == 0) {   // no routed rows: y = 0 (reference: mh_moe_fwd.py:257-258)
    cudaError_t e;
    if (y_stride_h == dh && y_stride_s == (int64_t)H * dh) {
      e = cudaMemsetAsync(y, 0, sizeof(__nv_bfloat16) * (size_t)S * H * dh, st);
    } else {
      e = cudaSuccess;
      for (int64_t s = 0; s < S && e == cudaSuccess; ++s)
        e = cudaMemset2DAsync(static_cast<__nv_bfloat16*>(y) + s * y_stride_s, sizeof(__nv_bfloat16) * y_stride_h, 0,
                              sizeof(__nv_bfloat16) * dh, H, st);
    }
    return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ffn_nvfp4 (zero fill)");
  }
  MHMOE_REQUIRE(workspace && gather_ids && probs_sorted);
  cudaError_t ce = cudaSuccess;
  const int rc = ffn_nvfp4(static_cast<const __nv_bfloat16*>(x), x_stride_s, x_stride_h, S, H, dh, de, n_experts, R,
                           gather_ids, probs_sorted, expert_offsets, gu_data, gu_sf, gu_gscale, dn_data, dn_sf,
                           dn_gscale, tok_rows, tok_offsets, k_fixed, workspace, static_cast<__nv_bfloat16*>(y),
                           y_stride_s, y_stride_h, dev_status, timeout_ns,
                           reinterpret_cast<cudaEvent_t const*>(stage_events), st, &ce, nullptr, nullptr, nullptr,
                           0, 0, 0, nullptr, atomic);
  if (rc == MHMOE_ERR_LAUNCH) return fail_cuda(ce, what);
  if (rc == MHMOE_ERR_DRIVER) g_last_error = "cuTensorMapEncodeTiled failed";
  return rc;
}

int mhmoe_ffn_nvfp4(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh, int de,
                    int n_experts, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                    const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                    const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                    const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, void* workspace,
                    void* y, int64_t y_stride_s, int64_t y_stride_h, int* dev_status, uint64_t timeout_ns,
                    void* const* stage_events, void* stream) {
  return ffn_entry(x, x_stride_s, x_stride_h, S, H, dh, de, n_experts, R, gather_ids, probs_sorted, expert_offsets,
                   gu_data, gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, tok_rows, tok_offsets, k_fixed, workspace, y,
                   y_stride_s, y_stride_h, dev_status, timeout_ns, stage_events, stream, false, "ffn_nvfp4");
}

int mhmoe_ffn_nvfp4_atomic(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh, int de,
                           int n_experts, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                           const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                           const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf,
                           const float* dn_gscale, void* workspace, void* y, int64_t y_stride_s, int64_t y_stride_h,
                           int* dev_status, uint64_t timeout_ns, void* const* stage_events, void* stream) {
  return ffn_entry(x, x_stride_s, x_stride_h, S, H, dh, de, n_experts, R, gather_ids, probs_sorted, expert_offsets,
                   gu_data, gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, nullptr, nullptr, 0, workspace, y,
                   y_stride_s, y_stride_h, dev_status, timeout_ns, stage_events, stream, true, "ffn_nvfp4_atomic");
}

int mhmoe_ffn_nvfp4_quantized(const uint8_t* xq, int64_t xq_pitch, const uint8_t* xsf, int64_t xsf_pitch,
                              const uint8_t* xg, int64_t xg_pitch, int T, int dh, int de,
                              int n_experts, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                              const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                              const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf,
                              const float* dn_gscale, const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed,
                              void* workspace, void* y, int64_t y_stride, int* dev_status, uint64_t timeout_ns,
                              void* const* stage_events, void* stream) {
  MHMOE_REQUIRE(xq && xsf && xg && y && expert_offsets && gu_data && gu_sf && gu_gscale && dn_data && dn_sf &&
                dn_gscale);
  MHMOE_REQUIRE(T >= 0 && n_experts > 0 && R >= 0 && dh % 256 == 0 && de % 256 == 0 && dh > 0 && de > 0);
  MHMOE_REQUIRE(aligned16(xq) && aligned16(xsf) && aligned16(y) && y_stride % 8 == 0);
  MHMOE_REQUIRE(xq_pitch >= dh / 2 && xq_pitch % 16 == 0 && xsf_pitch >= dh / 16 && xsf_pitch % 16 == 0);
  MHMOE_REQUIRE(xg_pitch >= 4 && xg_pitch % 4 == 0 && (reinterpret_cast<uintptr_t>(xg) & 3) == 0);
  MHMOE_REQUIRE(tok_rows || !tok_offsets);
  MHMOE_REQUIRE(!tok_rows || tok_offsets || k_fixed > 0);
  MHMOE_CHECK_ARCH();
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) return MHMOE_OK;
  if (R == 0) {
    const cudaError_t e = cudaMemset2DAsync(y, sizeof(__nv_bfloat16) * y_stride, 0, sizeof(__nv_bfloat16) * dh, T, st);
    return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ffn_nvfp4_quantized (zero fill)");
  }
  MHMOE_REQUIRE(workspace && gather_ids && probs_sorted);
  cudaError_t ce = cudaSuccess;
  const int rc = ffn_nvfp4(nullptr, 0, 0, T, 1, dh, de, n_experts, R, gather_ids, probs_sorted, expert_offsets,
                           gu_data, gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, tok_rows, tok_offsets, k_fixed,
                           workspace, static_cast<__nv_bfloat16*>(y), y_stride, dh, dev_status, timeout_ns,
                           reinterpret_cast<cudaEvent_t const*>(stage_events), st, &ce, xq, xsf, xg, xq_pitch,
                           xsf_pitch, xg_pitch);
  if (rc == MHMOE_ERR_LAUNCH) return fail_cuda(ce, "ffn_nvfp4_quantized");
  if (rc == MHMOE_ERR_DRIVER) g_last_error = "cuTensorMapEncodeTiled failed";
  return rc;
}

int mhmoe_quant_tokens(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh, uint8_t* xq,
                       uint8_t* xsf, float* xg, void* stream) {
  MHMOE_REQUIRE(x && xq && xsf && xg && S >= 0 && H > 0 && dh > 0 && dh % 256 == 0);
  MHMOE_REQUIRE(aligned16(x) && x_stride_s % 8 == 0 && x_stride_h % 8 == 0 && aligned16(xq) && aligned16(xsf));
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  const cudaError_t e = launch_quant_tokens(static_cast<const __nv_bfloat16*>(x), x_stride_s, x_stride_h, S, H, dh,
                                            xq, xsf, xg, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "quant_tokens");
}

int mhmoe_combine(const void* P, int64_t P_rows, const int32_t* pad_of_row, int dh, int S, int H,
                  const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R, void* y,
                  int64_t y_stride_s, int64_t y_stride_h, void* stream) {
  MHMOE_REQUIRE(y && S >= 0 && H > 0 && dh > 0 && dh % 8 == 0 && R >= 0);
  MHMOE_REQUIRE(tok_rows && (tok_offsets || k_fixed > 0));
  MHMOE_REQUIRE(aligned16(y) && y_stride_s % 8 == 0 && y_stride_h % 8 == 0 && (R == 0 || (P && aligned16(P))));
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  const cudaError_t e = launch_combine(static_cast<const __nv_bfloat16*>(P), pad_of_row, dh, S, H, tok_rows,
                                       tok_offsets, k_fixed, R, P_rows, static_cast<__nv_bfloat16*>(y), y_stride_s,
                                       y_stride_h, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "combine");
}

int64_t mhmoe_ep_row_bytes(int dh, int K) { return ep_row_bytes(dh, K); }

int mhmoe_ep_dest(const int64_t* topk_idx, int H, int S, int K, int E, int n_ranks, int64_t* dest, int* dev_status,
                  void* stream) {
  MHMOE_REQUIRE(topk_idx && dest && H > 0 && S >= 0 && K > 0 && E > 0 && n_ranks > 0 && n_ranks <= 32);
  MHMOE_REQUIRE(((int64_t)H * E) % n_ranks == 0);
  MHMOE_CHECK_ARCH();
  if (S == 0) return MHMOE_OK;
  const cudaError_t e = launch_ep_dest(topk_idx, H, S, K, E, n_ranks, H * E / n_ranks, dest, dev_status,
                                       static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_dest");
}

int mhmoe_ep_pack(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                  const int64_t* topk_idx, const float* topk_probs, int K, int E, int n_ranks, const int32_t* send_key,
                  const int64_t* send_offsets, int64_t R_send, uint8_t* send, void* stream) {
  MHMOE_REQUIRE(xq && xsf && xg && topk_idx && topk_probs && send_key && send_offsets && send);
  MHMOE_REQUIRE(H > 0 && S >= 0 && dh > 0 && dh % 256 == 0 && K > 0 && E > 0 && n_ranks > 0 && n_ranks <= 32);
  MHMOE_REQUIRE(((int64_t)H * E) % n_ranks == 0 && R_send >= 0);
  MHMOE_REQUIRE(aligned16(xq) && aligned16(xsf) && aligned16(send));
  MHMOE_CHECK_ARCH();
  if (R_send == 0) return MHMOE_OK;
  const cudaError_t e = launch_ep_pack(xq, xsf, xg, H, S, dh, topk_idx, topk_probs, K, E, H * E / n_ranks, send_key,
                                       send_offsets, n_ranks, R_send, send, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_pack");
}

int mhmoe_ep_unpack(const uint8_t* recv, int64_t R, int dh, int K, int E_loc, int64_t* local_expert, float* probs,
                    int* dev_status, void* stream) {
  MHMOE_REQUIRE(recv && local_expert && probs && R >= 0 && dh > 0 && dh % 256 == 0 && K > 0 && E_loc > 0);
  MHMOE_CHECK_ARCH();
  if (R == 0) return MHMOE_OK;
  const cudaError_t e = launch_ep_unpack(recv, R, dh, K, E_loc, local_expert, probs, dev_status,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_unpack");
}

int mhmoe_quantize_rows_nvfp4(const void* x, int64_t row_pitch, int64_t M, int K, uint8_t* data, uint8_t* sf,
                              float* gscale, void* stream) {
  MHMOE_REQUIRE(x && data && sf && gscale);
  MHMOE_REQUIRE(M >= 0 && K > 0 && K % 64 == 0 && row_pitch % 8 == 0 && aligned16(x) && aligned16(data));
  MHMOE_CHECK_ARCH();
  if (M == 0) return MHMOE_OK;
  const cudaError_t e = launch_quantize_rows(static_cast<const __nv_bfloat16*>(x), row_pitch, M, K, data, sf, gscale,
                                             static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "quantize_rows_nvfp4");
}

int mhmoe_gemm_nvfp4_raw(const uint8_t* a_data, const uint8_t* a_sf, int n_mtiles, const int32_t* tile_expert,
                         const uint8_t* b_data, const uint8_t* b_sf, int n_experts, int N, int K, float* out,
                         int* dev_status, uint64_t timeout_ns, void* stream) {
  MHMOE_REQUIRE(a_data && a_sf && tile_expert && b_data && b_sf && out);
  MHMOE_REQUIRE(n_mtiles > 0 && n_experts > 0 && N % 256 == 0 && K % 256 == 0 && N > 0 && K > 0);
  MHMOE_REQUIRE(aligned16(a_data) && aligned16(b_data) && aligned16(a_sf) && aligned16(b_sf));
  MHMOE_CHECK_ARCH();
  cudaError_t ce = cudaSuccess;
  const int rc = gemm_nvfp4_raw(a_data, a_sf, n_mtiles, tile_expert, b_data, b_sf, n_experts, N, K, out, dev_status,
                                timeout_ns, static_cast<cudaStream_t>(stream), &ce);
  if (rc == MHMOE_ERR_LAUNCH) return fail_cuda(ce, "gemm_nvfp4_raw");
  return rc;
}

int mhmoe_wait_selftest(const int* flag, int expected, int mode, uint64_t timeout_ns, int* dev_status,
                        int64_t* elapsed_ns, void* stream) {
  MHMOE_REQUIRE(dev_status && mode >= 0 && mode <= 3 && (!(mode & 2) || flag));
  MHMOE_REQUIRE(timeout_ns >= 1000ull && timeout_ns <= 10000000000ull);
  MHMOE_CHECK_ARCH();
  const cudaError_t e = launch_wait_selftest(flag, expected, mode, timeout_ns, dev_status, elapsed_ns,
                                             static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "wait_selftest");
}

/* ───────── MoE layer around the routed core ───────── */

int mhmoe_rmsnorm(const void* x, int64_t x_stride, const float* weight, const int32_t* cu_group_rows, int n_groups,
                  int64_t rows, int dim, float eps, float weight_bias, void* y, int64_t y_stride, void* stream) {
  MHMOE_REQUIRE(x && y && weight && rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= 8192);
  MHMOE_REQUIRE(n_groups >= 1 && (n_groups == 1 || cu_group_rows));
  MHMOE_REQUIRE(x_stride >= dim && y_stride >= dim && x_stride % 8 == 0 && y_stride % 8 == 0);
  MHMOE_REQUIRE(aligned16(x) && aligned16(y) && aligned16(weight));
  MHMOE_CHECK_ARCH();
  const cudaError_t e = launch_rmsnorm_modality(
      static_cast<const __nv_bfloat16*>(x), x_stride, weight, n_groups > 1 ? cu_group_rows : nullptr, n_groups, rows,
      dim, eps, weight_bias, static_cast<__nv_bfloat16*>(y), y_stride, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "rmsnorm");
}

/* ───────── expert-parallel exchange over peer memory ───────── */

size_t mhmoe_ep_sym_bytes(int n_ranks, int64_t cap, int dh, int K) {
  if (n_ranks <= 0 || n_ranks > EP_MAX_RANKS || cap < 0 || dh <= 0 || K <= 0) return 0;
  return (size_t)ep_layout(n_ranks, cap, dh, ep_row_bytes(dh, K)).bytes;
}

int mhmoe_ep_sym_offsets(int n_ranks, int64_t cap, int dh, int K, int64_t* out) {
  MHMOE_REQUIRE(out && n_ranks > 0 && n_ranks <= EP_MAX_RANKS && cap >= 0 && dh > 0 && K > 0);
  const EpLayout L = ep_layout(n_ranks, cap, dh, ep_row_bytes(dh, K));
  out[0] = L.off_flags;
  out[1] = L.off_meta;
  out[2] = L.off_rx;
  out[3] = L.off_back;
  out[4] = L.bytes;
  return MHMOE_OK;
}

int mhmoe_ep_sym_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  MHMOE_REQUIRE(ptr && ipc_handle && bytes > 0);
  MHMOE_CHECK_ARCH();
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail_cuda(e, "ep_sym_alloc (cudaMalloc)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail_cuda(e, "ep_sym_alloc (ipc handle)");
  }
  *ptr = p;
  return MHMOE_OK;
}

int mhmoe_ep_sym_open(const void* ipc_handle, void** peer_ptr) {
  MHMOE_REQUIRE(ipc_handle && peer_ptr);
  MHMOE_CHECK_ARCH();
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_sym_open (cudaIpcOpenMemHandle)");
}

int mhmoe_ep_sym_close(void* peer_ptr) {
  MHMOE_REQUIRE(peer_ptr);
  const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_sym_close");
}

int mhmoe_ep_sym_free(void* ptr) {
  MHMOE_REQUIRE(ptr);
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_sym_free");
}

static bool fill_peers(void* const* peer_bases, int n, EpPeers* peers) {
  for (int d = 0; d < EP_MAX_RANKS; ++d) peers->base[d] = nullptr;
  for (int d = 0; d < n; ++d) {
    if (!peer_bases[d] || !aligned16(peer_bases[d])) return false;
    peers->base[d] = static_cast<uint8_t*>(peer_bases[d]);
  }
  return true;
}

static int ep_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh, const int64_t* idx,
                      const float* probs, int K, int E, const int32_t* send_key, const int64_t* send_offsets,
                      int n_ranks, int rank, int64_t cap, void* const* peer_bases, int* dev_status, void* stream,
                      bool stage) {
  MHMOE_REQUIRE(xq && xsf && xg && idx && probs && send_key && send_offsets && peer_bases && dev_status);
  MHMOE_REQUIRE(H > 0 && S >= 0 && dh > 0 && dh % 256 == 0 && K > 0 && K <= 16 && E > 0);
  MHMOE_REQUIRE(n_ranks > 0 && n_ranks <= EP_MAX_RANKS && rank >= 0 && rank < n_ranks && (H * E) % n_ranks == 0);
  MHMOE_REQUIRE(cap >= (int64_t)H * S);
  MHMOE_CHECK_ARCH();
  EpPeers peers;
  MHMOE_REQUIRE(fill_peers(peer_bases, n_ranks, &peers));
  const cudaError_t e = launch_ep_send_records(xq, xsf, xg, H, S, dh, idx, probs, K, E, H * E / n_ranks, send_key,
                                               send_offsets, n_ranks, rank, cap, peers, peers.base[rank], dev_status,
                                               static_cast<cudaStream_t>(stream), stage);
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, stage ? "ep_stage_records" : "ep_send_records");
}

int mhmoe_ep_send_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                          const int64_t* idx, const float* probs, int K, int E, const int32_t* send_key,
                          const int64_t* send_offsets, int n_ranks, int rank, int64_t cap, void* const* peer_bases,
                          int* dev_status, void* stream) {
  return ep_records(xq, xsf, xg, H, S, dh, idx, probs, K, E, send_key, send_offsets, n_ranks, rank, cap, peer_bases,
                    dev_status, stream, false);
}

int mhmoe_ep_stage_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                           const int64_t* idx, const float* probs, int K, int E, const int32_t* send_key,
                           const int64_t* send_offsets, int n_ranks, int rank, int64_t cap, void* const* peer_bases,
                           int* dev_status, void* stream) {
  return ep_records(xq, xsf, xg, H, S, dh, idx, probs, K, E, send_key, send_offsets, n_ranks, rank, cap, peer_bases,
                    dev_status, stream, true);
}

int mhmoe_ep_push(void* local_base, int kind, int n_ranks, int rank, int64_t cap, int dh, int K,
                  void* const* peer_bases, void* stream) {
  MHMOE_REQUIRE(local_base && peer_bases && (kind == 0 || kind == 1));
  MHMOE_REQUIRE(n_ranks > 0 && n_ranks <= EP_MAX_RANKS && rank >= 0 && rank < n_ranks && cap >= 0);
  MHMOE_REQUIRE(dh > 0 && dh % 256 == 0 && K > 0 && K <= 16);
  MHMOE_CHECK_ARCH();
  EpPeers peers;
  MHMOE_REQUIRE(fill_peers(peer_bases, n_ranks, &peers));
  MHMOE_REQUIRE(peers.base[rank] == local_base);
  const cudaError_t e = launch_ep_push(static_cast<uint8_t*>(local_base), kind, n_ranks, rank, cap, dh, K, peers,
                                       static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_push");
}

int mhmoe_ep_wait(const void* local_base, int kind, int n_ranks, int epoch, uint64_t timeout_ns, int* dev_status,
                  void* stream) {
  MHMOE_REQUIRE(local_base && dev_status && (kind == 0 || kind == 1) && n_ranks > 0 && n_ranks <= EP_MAX_RANKS);
  MHMOE_REQUIRE(epoch > 0 && timeout_ns >= 1000ull && timeout_ns <= 600000000000ull);
  MHMOE_CHECK_ARCH();
  const cudaError_t e = launch_ep_wait(static_cast<const uint8_t*>(local_base), kind, n_ranks, epoch, timeout_ns,
                                       dev_status, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_wait");
}

int mhmoe_ep_unpack_slots(const void* local_base, int n_ranks, int64_t cap, int dh, int K, int E_loc,
                          int64_t* local_expert, float* probs, int* dev_status, void* stream) {
  MHMOE_REQUIRE(local_base && local_expert && probs && dev_status && n_ranks > 0 && n_ranks <= EP_MAX_RANKS);
  MHMOE_REQUIRE(cap >= 0 && dh > 0 && dh % 256 == 0 && K > 0 && K <= 16 && E_loc > 0);
  MHMOE_CHECK_ARCH();
  if ((int64_t)n_ranks * cap == 0) return MHMOE_OK;
  const cudaError_t e = launch_ep_unpack_slots(static_cast<const uint8_t*>(local_base), n_ranks, cap, dh, K, E_loc,
                                               local_expert, probs, dev_status, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MHMOE_OK : fail_cuda(e, "ep_unpack_slots");
}

static int ep_ffn(const void* local_base, int n_ranks, int rank, int64_t cap, int dh, int de, int K, int E_loc, int64_t R,
                  const int32_t* gather_ids, const float* probs_sorted, const int64_t* expert_offsets,
                  const uint8_t* gu_data, const uint8_t* gu_sf, const float* gu_gscale, const uint8_t* dn_data,
                  const uint8_t* dn_sf, const float* dn_gscale, const int32_t* row_of_flat, void* workspace,
                  void* const* peer_bases, int* dev_status, uint64_t timeout_ns, void* const* stage_events,
                  void* stream, int stage) {
  MHMOE_REQUIRE(local_base && gather_ids && probs_sorted && expert_offsets && gu_data && gu_sf && gu_gscale &&
                dn_data && dn_sf && dn_gscale && row_of_flat && workspace && peer_bases && dev_status);
  MHMOE_REQUIRE(n_ranks > 0 && n_ranks <= EP_MAX_RANKS && rank >= 0 && rank < n_ranks && cap > 0);
  MHMOE_REQUIRE(dh > 0 && dh % 256 == 0 && de > 0 && de % 256 == 0 && K > 0 && K <= 16 && E_loc > 0);
  MHMOE_REQUIRE(R == (int64_t)n_ranks * cap * K);
  MHMOE_CHECK_ARCH();
  EpPeers peers;
  MHMOE_REQUIRE(fill_peers(peer_bases, n_ranks, &peers));
  MHMOE_REQUIRE(peers.base[rank] == local_base);
  const int64_t rb = ep_row_bytes(dh, K);
  EpReturn ret;
  ret.peers = peers;
  ret.local = static_cast<uint8_t*>(const_cast<void*>(local_base));
  ret.layout = ep_layout(n_ranks, cap, dh, rb);
  ret.cap = cap;
  ret.n = n_ranks;
  ret.me = rank;
  ret.status = dev_status;
  ret.stage = stage;
  const uint8_t* rx = ret.local + ret.layout.off_rx;
  const int64_t T = (int64_t)n_ranks * cap;
  MHMOE_REQUIRE(T <= 0x7fffffff);
  cudaError_t ce = cudaSuccess;
  const int rc = ffn_nvfp4(nullptr, 0, 0, (int)T, 1, dh, de, E_loc, R, gather_ids, probs_sorted, expert_offsets,
                           gu_data, gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, row_of_flat, nullptr, K, workspace,
                           nullptr, dh, dh, dev_status, timeout_ns,
                           reinterpret_cast<cudaEvent_t const*>(stage_events), static_cast<cudaStream_t>(stream), &ce,
                           rx, rx + dh / 2, rx + dh / 2 + dh / 16, rb, rb, rb, &ret);
  if (rc == MHMOE_ERR_LAUNCH) return fail_cuda(ce, stage ? "ep_ffn_stage" : "ep_ffn_return");
  if (rc == MHMOE_ERR_DRIVER) g_last_error = "cuTensorMapEncodeTiled failed";
  return rc;
}

int mhmoe_ep_ffn_return(const void* local_base, int n_ranks, int rank, int64_t cap, int dh, int de, int K, int E_loc,
                        int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                        const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                        const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                        const int32_t* row_of_flat, void* workspace, void* const* peer_bases, int* dev_status,
                        uint64_t timeout_ns, void* const* stage_events, void* stream) {
  return ep_ffn(local_base, n_ranks, rank, cap, dh, de, K, E_loc, R, gather_ids, probs_sorted, expert_offsets, gu_data,
                gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, row_of_flat, workspace, peer_bases, dev_status, timeout_ns,
                stage_events, stream, 0);
}

int mhmoe_ep_ffn_stage(const void* local_base, int n_ranks, int rank, int64_t cap, int dh, int de, int K, int E_loc,
                       int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                       const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                       const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                       const int32_t* row_of_flat, void* workspace, void* const* peer_bases, int* dev_status,
                       uint64_t timeout_ns, void* const* stage_events, void* stream) {
  return ep_ffn(local_base, n_ranks, rank, cap, dh, de, K, E_loc, R, gather_ids, probs_sorted, expert_offsets, gu_data,
                gu_sf, gu_gscale, dn_data, dn_sf, dn_gscale, row_of_flat, workspace, peer_bases, dev_status, timeout_ns,
                stage_events, stream, 1);
}

}  // extern "C"
