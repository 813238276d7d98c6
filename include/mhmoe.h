/*
 * mhmoe.h — C ABI of the B200 (sm_100a) MAGI-2 MoE expert hot path.
 *
 * Drop-in replacement for the reference's `inference/flash_mh_moe` package
 * (router top-k, global sort, fused expert FFN) plus the expert-parallel
 * dispatch/combine.  Every entry point takes raw device pointers, shapes and a
 * cudaStream_t (passed as void*), enqueues work on that stream and returns an
 * mhmoe_status.  The compute entry points allocate no device memory: callers own
 * every buffer, including the scratch buffers whose sizes the *_bytes queries give.
 * The one exception is mhmoe_ep_sym_alloc, the set-up call that allocates (and
 * exports for CUDA IPC) an expert-parallel exchange buffer; mhmoe_ep_sym_free
 * releases it.  No compute entry point synchronises the stream.
 *
 * Kernels that wait on on-chip barriers give up after `timeout_ns` (0 selects
 * the default of 2 s) and record MHMOE_ERR_TIMEOUT in the optional device word
 * `dev_status` (int32, caller-zeroed); the host reads it when convenient.
 *
 * Layout conventions (row-major unless stated):
 *   x            bf16 [S, H, dh]   strides in elements; dh stride must be 1
 *   logits       fp32 [H, S, E]
 *   probs / idx  fp32 / int64 [H, S, K]
 *   gather_ids   int32 [R], probs_sorted fp32 [R], expert_offsets int64 [H*E+1]
 *   NVFP4 matrix: packed E2M1 bytes [rows, K/2] (low nibble = even k), UE4M3
 *                 scales in 512-byte "SF atoms" (128 rows x 64 K-elements each;
 *                 row m, scale column c at (m%32)*16 + (m/32)*4 + c; atoms
 *                 K-fastest), one fp32 second-level scale per matrix or row.
 */
#ifndef MHMOE_H_
#define MHMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MHMOE_API __attribute__((visibility("default")))
#else
#define MHMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MHMOE_OK = 0,
  MHMOE_ERR_ARGS = 1,      /* bad shape, stride, alignment or null pointer */
  MHMOE_ERR_ARCH = 2,      /* device is not sm_100 */
  MHMOE_ERR_LAUNCH = 3,    /* CUDA launch / runtime error */
  MHMOE_ERR_TIMEOUT = 4,   /* a bounded on-chip wait gave up (device-side) */
  MHMOE_ERR_DRIVER = 5,    /* driver entry point / tensor-map encode failed */
  MHMOE_ERR_PEER = 6,      /* expert-parallel peer wait gave up (device-side) */
  MHMOE_ERR_CAPACITY = 7   /* a size exceeds a compiled-in maximum */
} mhmoe_status;

/* Library identity and diagnostics. */
MHMOE_API int mhmoe_version(void);
MHMOE_API const char* mhmoe_status_string(int status);
/* Last CUDA error text recorded by a failing call on this host thread. */
MHMOE_API const char* mhmoe_last_error(void);

/* ───────────────────────── router ───────────────────────── */

/* Router logits: logits[h,s,e] = sum_d x[s,h,d] * gate[h*E+e, d] in fp32.
 * Replaces the fp32 einsum of CoreMultiHeadMoE._route
 * (inference/model/magi2_preview.py:2588-2591).  gate is fp32 [H*E, dh]. */
MHMOE_API int mhmoe_router_logits(const void* x, int64_t x_stride_s, int64_t x_stride_h, const float* gate, int S, int H,
                        int dh, int E, float* logits, void* stream);

/* Router weight preparation (at load, not per step): split the fp32 gate [H*E, dh]
 * into nsplit (1..3) bf16 planes hi, lo, lo2 (g = hi + lo + lo2 exactly for nsplit 3),
 * stored interleaved per 64-column block: planes [H*E, nsplit*dh] bf16.
 * flags (optional, int32[3], caller-zeroed): flags[1] / flags[2] set when the lo / lo2
 * plane is non-zero, i.e. the smallest exact nsplit is 1 + flags[1]|flags[2] + flags[2]. */
MHMOE_API int mhmoe_router_prepare(const float* gate, int n_experts, int dh, int nsplit, void* planes, int* flags,
                                   void* stream);

/* Fused router on the tensor cores.  Replaces CoreMultiHeadMoE._route
 * (inference/model/magi2_preview.py:2588-2601): fp32-accurate logits (bf16 tcgen05 MMAs
 * over the prepared planes) followed, in the same kernel, by softmax/sigmoid, +expert_bias
 * for selection, top-k (sorted desc, ties to the lower id), L1 normalisation and
 * route_scale (route.py:28-148 without virtual groups).  x bf16 [S, H, dh] with heads
 * contiguous (x_stride_h == dh).  E <= 256, K <= 16, dh % 64 == 0.
 * logit_bias (optional, fp32 [H*E]) is added to the logits before scoring (a gate bias
 * term; the reference has none, pass NULL).  logits (optional) receives the fp32 [H, S, E]
 * logits the scores were computed from.  Batches of a few 128-token tiles (H*ceil(S/128)
 * at most a quarter of the SMs, dh % 128 == 0) run a cluster kernel that splits the
 * reduction over 8 CTAs instead (same contract, exact products summed in fp32). */
MHMOE_API int mhmoe_route(const void* x, int64_t x_stride_s, int64_t x_stride_h, const void* planes, int nsplit,
                          int S, int H, int dh, int E, int K, int score_func, const float* logit_bias,
                          const float* expert_bias, int route_norm, float norm_eps, float route_scale, float* probs,
                          int64_t* idx, float* logits, int* dev_status, void* stream);

/* Top-k gating from logits.  Replaces compute_topk_probs_and_indices
 * (inference/flash_mh_moe/route.py:157-199 -> :28-148).
 * score_func: 0 softmax, 1 sigmoid.  expert_bias fp32 [H*E] or NULL.
 * num_virtual_group > 1 enables the two-stage group selection (route.py:61-104).
 * route_scale multiplies the (normalised) probs, as CoreMultiHeadMoE._route does
 * (magi2_preview.py:2600); pass 1.0 for the plain route.py contract.
 * Outputs: probs fp32 [H,S,K]; idx int64 [H,S,K], sorted by descending score,
 * ties to the lower expert id.  E <= 1024, K <= 32. */
MHMOE_API int mhmoe_topk(const float* logits, const float* expert_bias, int H, int S, int E, int K, int score_func,
               int num_virtual_group, int topk_virtual_group, int route_norm, float norm_eps, float route_scale,
               float* probs, int64_t* idx, void* stream);

/* ───────────────────────── permutation ───────────────────────── */

/* Scratch bytes for mhmoe_global_sort (int32 chunk histograms). */
MHMOE_API size_t mhmoe_global_sort_workspace_bytes(int H, int S, int K, int E);

/* Stable counting sort of the flat (h,s,k) entries by global expert h*E+idx.
 * Replaces flash_mh_moe_global_sort (inference/flash_mh_moe/route.py:209-253):
 * gather_ids int32 [R], probs_sorted fp32 [R], expert_offsets int64 [H*E+1],
 * bit-identical to argsort(stable=True).  row_of_flat int32 [R] (optional):
 * the sorted position of flat entry f (-1 for dropped entries).  H*E <= 12288.
 * A negative expert id marks an empty slot and is skipped (the reference never emits
 * one; expert-parallel packing uses them); an id >= E is never used as an index: the
 * entry is dropped and MHMOE_ERR_ARGS is recorded in dev_status. */
MHMOE_API int mhmoe_global_sort(const float* topk_probs, const int64_t* topk_idx, int H, int S, int K, int E,
                      void* workspace, int32_t* gather_ids, float* probs_sorted, int64_t* expert_offsets,
                      int32_t* row_of_flat, int* dev_status, void* stream);

/* Same contract and outputs as mhmoe_global_sort, for callers that cannot allocate
 * device memory: it takes no workspace and allocates nothing.  No counterpart in the
 * reference (the reference sort allocates through PyTorch).  Its scratch is a fixed
 * ~1.05 MB array inside the library, held by every GPU that loads it; limits:
 * H*S*K <= 262144 routed rows and H*E <= 1024 experts, else MHMOE_ERR_CAPACITY with
 * nothing launched.  The first call on a device (with it current) resolves the
 * array's device address; make that call before any stream capture.  The address is
 * cached per device for the life of the process: do not use this entry point across a
 * device reset (cudaDeviceReset) of that device.  All calls share the array: calls that
 * overlap on the GPU race, so order them. */
MHMOE_API int mhmoe_global_sort_noalloc(const float* topk_probs, const int64_t* topk_idx, int H, int S, int K, int E,
                                        int32_t* gather_ids, float* probs_sorted, int64_t* expert_offsets,
                                        int32_t* row_of_flat, int* dev_status, void* stream);

/* ───────────────────────── expert FFN (NVFP4) ───────────────────────── */

/* Upper bound of 128-row tiles for R routed rows over n_experts groups. */
MHMOE_API int64_t mhmoe_max_mtiles(int64_t R, int n_experts);

/* Scratch bytes of mhmoe_ffn_nvfp4 for R rows, S tokens, H heads, dh, de, H*E experts. */
MHMOE_API size_t mhmoe_ffn_workspace_bytes(int64_t R, int S, int H, int dh, int de, int n_experts);

/* Pack reference-layout weights into the NVFP4 operand layout (quantise on load).
 *   kind 0 (gate/up): w0 = W_gate, w1 = W_up, both [n_experts, dh, de] (bf16);
 *        out data [n_experts, 2*de, dh/2] with gate/up rows interleaved in groups
 *        of 16, sf atoms [n_experts, 2*de*dh/16], gscale [2, n_experts] (gate, up).
 *   kind 1 (down): w0 = W_down [n_experts, de, dh] (bf16), w1 = NULL;
 *        out data [n_experts, dh, de/2], sf atoms [n_experts, dh*de/16], gscale [n_experts].
 * gscale = amax(matrix)/2688.  Scratch: amax fp32 [2*n_experts] (caller-zeroed not required). */
MHMOE_API int mhmoe_pack_weights_nvfp4(int kind, const void* w0, const void* w1, int n_experts, int dh, int de,
                             uint8_t* data, uint8_t* sf, float* gscale, float* amax_scratch, void* stream);

/* Fused expert FFN on NVFP4 operands.  Replaces flash_mh_moe_fwd / mh_moe_fwd_func
 * (inference/flash_mh_moe/fwd.py:16-40, triton/mh_moe_fwd.py:231-331): gather ->
 * x quantise (per row) -> grouped GEMM gate/up + SwiGLU7 + hidden quantise ->
 * grouped GEMM down x prob -> deterministic combine into y [S,H,dh] bf16.
 * R = number of routed rows, n_experts = H*E (flattened).  dh % 256 == 0,
 * de % 256 == 0.  `tok_rows`/`tok_offsets` (optional) give each (s,h) its rows
 * (row_of_flat with fixed K when tok_offsets == NULL and k_fixed > 0); when both
 * are NULL the mapping is derived from gather_ids.  workspace: see
 * mhmoe_ffn_workspace_bytes.  stage_events (optional): 5 cudaEvent_t recorded on
 * `stream` before the tile tables, before the gate/up GEMM, before the down GEMM,
 * before the combine and at the end (per-stage timing without a profiler). */
MHMOE_API int mhmoe_ffn_nvfp4(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh, int de,
                    int n_experts, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                    const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                    const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                    const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, void* workspace,
                    void* y, int64_t y_stride_s, int64_t y_stride_h, int* dev_status, uint64_t timeout_ns,
                    void* const* stage_events, void* stream);

/* mhmoe_ffn_nvfp4 with the reference's default (non-deterministic) scatter: the down
 * GEMM adds each routed row's bf16(y_acc * prob) into y with bf16 atomics
 * (_mh_moe_fwd_kernel with deterministic=False, triton/mh_moe_fwd.py:172-181, selected
 * when MAGI2_DETERMINISTIC is not "1", fwd.py:12-13).  y is zeroed first; no partial
 * buffer and no combine pass.  Results may differ run to run in the last bf16 bits. */
MHMOE_API int mhmoe_ffn_nvfp4_atomic(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh,
                                     int de, int n_experts, int64_t R, const int32_t* gather_ids,
                                     const float* probs_sorted, const int64_t* expert_offsets, const uint8_t* gu_data,
                                     const uint8_t* gu_sf, const float* gu_gscale, const uint8_t* dn_data,
                                     const uint8_t* dn_sf, const float* dn_gscale, void* workspace, void* y,
                                     int64_t y_stride_s, int64_t y_stride_h, int* dev_status, uint64_t timeout_ns,
                                     void* const* stage_events, void* stream);

/* The FFN above on rows that are already NVFP4 (per-row scales): row t has its dh/2
 * data bytes at xq + t*xq_pitch, its dh/16 row-major scale bytes at xsf + t*xsf_pitch
 * and its fp32 row scale at xg + t*xg_pitch (byte pitches, 16-B aligned data/scales);
 * gather_ids index these T rows (H = 1).  Used by the expert-parallel receiver, which
 * reads the received records in place.  y: [T, dh] bf16 rows with pitch y_stride
 * (combined through tok_rows / tok_offsets / k_fixed as above).  stage_events: as for
 * mhmoe_ffn_nvfp4 (optional). */
MHMOE_API int mhmoe_ffn_nvfp4_quantized(const uint8_t* xq, int64_t xq_pitch, const uint8_t* xsf, int64_t xsf_pitch,
                                        const uint8_t* xg, int64_t xg_pitch, int T, int dh, int de,
                                        int n_experts, int64_t R, const int32_t* gather_ids,
                                        const float* probs_sorted, const int64_t* expert_offsets,
                                        const uint8_t* gu_data, const uint8_t* gu_sf, const float* gu_gscale,
                                        const uint8_t* dn_data, const uint8_t* dn_sf, const float* dn_gscale,
                                        const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed,
                                        void* workspace, void* y, int64_t y_stride, int* dev_status,
                                        uint64_t timeout_ns, void* const* stage_events, void* stream);

/* ───────────────────────── building blocks (tests, EP) ───────────────────────── */

/* Per-token NVFP4 of x [S, H, dh] (bf16): row t = s*H + h of xq [T, dh/2], xsf [T, dh/16]
 * (row-major scales), xg [T] = amax(row)/2688.  dh % 256 == 0. */
MHMOE_API int mhmoe_quant_tokens(const void* x, int64_t x_stride_s, int64_t x_stride_h, int S, int H, int dh,
                                 uint8_t* xq, uint8_t* xsf, float* xg, void* stream);

/* Deterministic combine: y[s,h,:] = bf16(sum, in ascending row id, of P[map(r), :] over
 * the rows r of key h*S + s), rows from tok_rows/tok_offsets (or k_fixed rows per key);
 * map = pad_of_row when given, else identity.  Replaces the scatter of the reference
 * FFN (triton/mh_moe_fwd.py:172-181, :189-215) and, in expert parallelism, the head
 * un-dispatch (magi2_preview.py:3303-3327). */
MHMOE_API int mhmoe_combine(const void* P, int64_t P_rows, const int32_t* pad_of_row, int dh, int S, int H,
                            const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R, void* y,
                            int64_t y_stride_s, int64_t y_stride_h, void* stream);

/* Expert-parallel dispatch (token -> expert sharding over n_ranks contiguous ranges of
 * E_loc flattened experts).  Replaces the head-sharded ep_dispatch / ep_undispatch of
 * the reference (magi2_preview.py:3277-3327).  A token row travels once to each rank
 * owning any of its K experts, as one record of mhmoe_ep_row_bytes(dh, K) bytes:
 * [dh/2 NVFP4 data][dh/16 scales][16 B {g, count, 0, 0}][K x {local expert, prob}].
 *   mhmoe_ep_dest: dest [H*S, n_ranks] int64 (key h*S + s): d if the row goes to rank
 *     d, else -1 (sorting it with mhmoe_global_sort, H = 1, K = n_ranks, E = n_ranks,
 *     gives the send order, per-rank counts and the (key, rank) -> send row map).
 *   mhmoe_ep_pack: send row j (key send_key[j], destination from send_offsets) ->
 *     its record, from the per-token quantised x (mhmoe_quant_tokens) and the routing.
 *   mhmoe_ep_unpack: received records -> local expert ids int64 [R, K] (-1 past the
 *     count) and probs [R, K]. */
MHMOE_API int64_t mhmoe_ep_row_bytes(int dh, int K);
MHMOE_API int mhmoe_ep_dest(const int64_t* topk_idx, int H, int S, int K, int E, int n_ranks, int64_t* dest,
                            int* dev_status, void* stream);
MHMOE_API int mhmoe_ep_pack(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                            const int64_t* topk_idx, const float* topk_probs, int K, int E, int n_ranks,
                            const int32_t* send_key, const int64_t* send_offsets, int64_t R_send, uint8_t* send,
                            void* stream);
MHMOE_API int mhmoe_ep_unpack(const uint8_t* recv, int64_t R, int dh, int K, int E_loc, int64_t* local_expert,
                              float* probs, int* dev_status, void* stream);

/* Per-row NVFP4 quantisation of bf16 rows x[r, 0:K] (row pitch in elements):
 * data [M, K/2], sf atoms, gscale [M] = amax(row)/2688.  K % 64 == 0. */
MHMOE_API int mhmoe_quantize_rows_nvfp4(const void* x, int64_t row_pitch, int64_t M, int K, uint8_t* data, uint8_t* sf,
                              float* gscale, void* stream);

/* Raw block-scaled grouped GEMM for verification: acc[rows, N] fp32 =
 * A (NVFP4, rows grouped in 128-row tiles by tile_expert) x B[e]^T (NVFP4) with
 * no second-level scales applied.  a rows = 128 * n_mtiles. */
MHMOE_API int mhmoe_gemm_nvfp4_raw(const uint8_t* a_data, const uint8_t* a_sf, int n_mtiles, const int32_t* tile_expert,
                         const uint8_t* b_data, const uint8_t* b_sf, int n_experts, int N, int K, float* out,
                         int* dev_status, uint64_t timeout_ns, void* stream);

/* ─────────────── expert-parallel exchange over peer memory ───────────────
 * Replaces the two all_to_all_single calls of ep_dispatch / ep_undispatch
 * (inference/model/magi2_preview.py:3277-3327) for ranks on the GPUs of one node: the
 * record and return kernels store straight into the destination rank's buffer (mapped
 * with CUDA IPC; plain NVLink stores, no multicast) and raise per-source arrival
 * counters there; no host synchronisation.  One buffer per rank, same layout on all:
 * flags, meta, rx records [n][cap][mhmoe_ep_row_bytes] and a return area
 * [n*cap][dh] bf16.  cap >= H*S (rows per rank).  Every call of one layer step passes
 * the same epoch, 1 for the first step and +1 per step, identically on all ranks. */

/* Bytes of the per-rank buffer (0 on bad arguments). */
MHMOE_API size_t mhmoe_ep_sym_bytes(int n_ranks, int64_t cap, int dh, int K);

/* Byte offsets of the buffer's parts: out[5] = {flags, meta, rx, back, total}. */
MHMOE_API int mhmoe_ep_sym_offsets(int n_ranks, int64_t cap, int dh, int K, int64_t* out);

/* Allocate and zero a buffer on the current device and export it: ipc_handle receives
 * the 64-byte CUDA IPC handle the other ranks open. */
MHMOE_API int mhmoe_ep_sym_alloc(size_t bytes, void** ptr, void* ipc_handle);

/* Map another rank's buffer from its 64-byte handle (peer access enabled lazily). */
MHMOE_API int mhmoe_ep_sym_open(const void* ipc_handle, void** peer_ptr);
MHMOE_API int mhmoe_ep_sym_close(void* peer_ptr);
MHMOE_API int mhmoe_ep_sym_free(void* ptr);

/* Source side: one record per send row (send_key / send_offsets from mhmoe_global_sort
 * of mhmoe_ep_dest's mask, grouped by destination) stored into destination d's rx at
 * slot rank*cap + (row - send_offsets[d]); then {count, send_offsets[d]} into d's meta
 * and d's records flag for this rank raised.  peer_bases: host array of n_ranks buffer
 * pointers as mapped on this device (this rank's own at [rank]). */
MHMOE_API int mhmoe_ep_send_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                                    const int64_t* topk_idx, const float* topk_probs, int K, int E,
                                    const int32_t* send_key, const int64_t* send_offsets, int n_ranks, int rank,
                                    int64_t cap, void* const* peer_bases, int* dev_status, void* stream);

/* Copy-engine transport, step 1: the same records as mhmoe_ep_send_records, written into this
 * rank's own slab (one cap-row slab per destination, send order within it) with the
 * per-destination {count, offset} beside it; nothing crosses NVLink and no flag is raised.
 * Replaces, like mhmoe_ep_send_records, the dispatch all_to_all of
 * inference/model/magi2_preview.py:3277-3299. */
MHMOE_API int mhmoe_ep_stage_records(const uint8_t* xq, const uint8_t* xsf, const float* xg, int H, int S, int dh,
                                     const int64_t* topk_idx, const float* topk_probs, int K, int E,
                                     const int32_t* send_key, const int64_t* send_offsets, int n_ranks, int rank,
                                     int64_t cap, void* const* peer_bases, int* dev_status, void* stream);

/* Copy-engine transport, step 2: one cudaMemcpyAsync per peer on `stream` (whole cap-row
 * slabs: the counts stay on the device) and then this rank's flag of `kind` in every peer.
 * kind 0: staged records -> each destination's receive area (+ their counts);
 * kind 1: staged sums (mhmoe_ep_ffn_stage) -> each source's return area, row d*cap + slot.
 * Only copies and a one-warp flag kernel: run it on a stream of its own to overlap the
 * transfer with compute.  Replaces the all_to_all calls of
 * inference/model/magi2_preview.py:3277-3327. */
MHMOE_API int mhmoe_ep_push(void* local_base, int kind, int n_ranks, int rank, int64_t cap, int dh, int K,
                            void* const* peer_bases, void* stream);

/* Wait on the device until every source's flag of `kind` (0 records, 1 returns) in this
 * rank's buffer reaches `epoch`; gives up after timeout_ns with MHMOE_ERR_PEER in
 * dev_status.  Later work on the stream runs after it. */
MHMOE_API int mhmoe_ep_wait(const void* local_base, int kind, int n_ranks, int epoch, uint64_t timeout_ns,
                            int* dev_status, void* stream);

/* Receiver: rx slot i -> local expert ids int64 [n_ranks*cap, K] and probs, -1 / 0 for
 * unused pairs and for slots past the source's count. */
MHMOE_API int mhmoe_ep_unpack_slots(const void* local_base, int n_ranks, int64_t cap, int dh, int K, int E_loc,
                                    int64_t* local_expert, float* probs, int* dev_status, void* stream);

/* Receiver: the expert FFN over the rx records in place (as mhmoe_ffn_nvfp4_quantized,
 * R = n_ranks*cap*K entries from the sort of mhmoe_ep_unpack_slots' output), whose
 * combine stores each record's bf16 expert sum into the source rank's return area at
 * row (source's send position) and raises the source's return flag for this rank. */
MHMOE_API int mhmoe_ep_ffn_return(const void* local_base, int n_ranks, int rank, int64_t cap, int dh, int de, int K,
                                  int E_loc, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                                  const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                                  const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf,
                                  const float* dn_gscale, const int32_t* row_of_flat, void* workspace,
                                  void* const* peer_bases, int* dev_status, uint64_t timeout_ns,
                                  void* const* stage_events, void* stream);

/* Copy-engine transport, step 3: mhmoe_ep_ffn_return with each record's sum written into this
 * rank's own stage area (source s's records at s*cap + slot) instead of the source's memory;
 * mhmoe_ep_push(kind 1) moves them.  Same arguments. */
MHMOE_API int mhmoe_ep_ffn_stage(const void* local_base, int n_ranks, int rank, int64_t cap, int dh, int de, int K,
                                 int E_loc, int64_t R, const int32_t* gather_ids, const float* probs_sorted,
                                 const int64_t* expert_offsets, const uint8_t* gu_data, const uint8_t* gu_sf,
                                 const float* gu_gscale, const uint8_t* dn_data, const uint8_t* dn_sf,
                                 const float* dn_gscale, const int32_t* row_of_flat, void* workspace,
                                 void* const* peer_bases, int* dev_status, uint64_t timeout_ns,
                                 void* const* stage_events, void* stream);

/* ───────────────────────── MoE layer around the routed core ───────────────────────── */

/* Multi-modality RMSNorm, the MoE layer's pre-norm.  Replaces MultiModalityRMSNorm.forward
 * (inference/model/magi2_preview.py:497-623, used as MultiHeadMoELayer.pre_norm at :2734):
 * y[t,:] = bf16(x[t,:] * rsqrt(mean(x[t,:]^2) + eps) * (weight[m(t),:] + weight_bias)) in
 * fp32, with rows grouped by modality: rows [cu_group_rows[m], cu_group_rows[m+1]) use
 * weight row m (fp32 [n_groups, dim]).  cu_group_rows: device int32 [n_groups+1] (may be
 * NULL when n_groups == 1).  x, y bf16 rows with the given strides (elements); dim % 8 == 0,
 * dim <= 8192, 16-B aligned pointers and strides. */
MHMOE_API int mhmoe_rmsnorm(const void* x, int64_t x_stride, const float* weight, const int32_t* cu_group_rows,
                            int n_groups, int64_t rows, int dim, float eps, float weight_bias, void* y,
                            int64_t y_stride, void* stream);

/* ───────────────────────── failure detection ───────────────────────── */

/* Self test of the bounded device waits (no counterpart in the reference).  Every
 * kernel here waits only with a time limit: on expiry it records MHMOE_ERR_TIMEOUT in
 * dev_status, finishes its copies in flight, frees its tensor memory and returns, so
 * the CUDA context stays usable.  This entry runs those waits against conditions that
 * never complete: mode bit 0 waits on a shared-memory barrier nothing arrives on, bit 1
 * waits for the int at `flag` to reach `expected` (flag may be NULL when bit 1 is
 * clear).  Each wait gives up after timeout_ns (must be 1 us .. 10 s).  elapsed_ns
 * (device, may be NULL) receives the total time waited.  Asynchronous: read dev_status
 * after synchronising the stream. */
MHMOE_API int mhmoe_wait_selftest(const int* flag, int expected, int mode, uint64_t timeout_ns, int* dev_status,
                                  int64_t* elapsed_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MHMOE_H_ */
