// mhmoe_global_sort_noalloc: the stable expert sort of mhmoe_global_sort for callers
// that cannot allocate device memory.
//
// Who needs it: hosts that bind libmhmoe directly through its C ABI and own no device
// allocator (no PyTorch caching allocator behind them), and callers that must not
// allocate on their hot path because cudaMalloc/cudaFree can synchronise the device
// and fragment memory between steps.  Such a caller still passes its inputs and
// outputs; only the sort's scratch (per-chunk histograms, per-expert totals and the
// 128-row tile tables) moves into a fixed array compiled into the library.
//
// The scratch is one file-scope __device__ array of NOALLOC_SCRATCH_BYTES (about
// 1.05 MB).  Every GPU that loads the library holds it until the process exits.
// Limits: at most NOALLOC_MAX_ROWS routed rows (H*S*K) and NOALLOC_MAX_EXPERTS
// flattened experts (H*E); larger problems are rejected with MHMOE_ERR_CAPACITY
// before anything is launched.
//
// All calls share the array and it keeps the previous call's contents.  Nothing in it
// has to start at zero: every scratch word the kernels read is written earlier in the
// same call.  Calls whose kernels overlap on the GPU (different streams, or different
// host threads, without ordering between them) race on the array; order them.
//
// Host code cannot pass the array's name to a kernel (on the host it names a shadow
// variable, not device memory), so the first call on each device, with that device
// current, asks the runtime for the array's device address (cudaGetSymbolAddress) and
// caches it.  Make that first call on a device before any stream capture begins.
#include <mutex>

#include "kernels.cuh"

namespace mhmoe {
namespace {

constexpr int64_t NOALLOC_MAX_ROWS = 262144;
constexpr int64_t NOALLOC_MAX_EXPERTS = 1024;
// This entry point sorts in chunks of >= 1024 rows, so at the limits the scratch holds
// 256 chunk histograms (global_sort_ws_bytes(..., NOALLOC_MIN_CHUNK)).
constexpr int NOALLOC_MIN_CHUNK = 1024;
constexpr int64_t NOALLOC_CHUNKS = NOALLOC_MAX_ROWS / NOALLOC_MIN_CHUNK;
constexpr int64_t NOALLOC_MTILES = NOALLOC_MAX_ROWS / 128 + NOALLOC_MAX_EXPERTS;
constexpr size_t NOALLOC_SCRATCH_BYTES =
    ((size_t)(NOALLOC_CHUNKS + 2) * NOALLOC_MAX_EXPERTS + 1 + 3 * (size_t)NOALLOC_MTILES) * sizeof(int) + 256;

__device__ __align__(256) unsigned char g_sort_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_sort_scratch on the current device (resolved once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sort_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace mhmoe

extern "C" MHMOE_API int mhmoe_global_sort_noalloc(const float* topk_probs, const int64_t* topk_idx, int H, int S,
                                                   int K, int E, int32_t* gather_ids, float* probs_sorted,
                                                   int64_t* expert_offsets, int32_t* row_of_flat, int* dev_status,
                                                   void* stream) {
  using namespace mhmoe;
  if (!topk_probs || !topk_idx || !gather_ids || !probs_sorted || !expert_offsets || H <= 0 || S < 0 || K <= 0 ||
      E <= 0)
    return MHMOE_ERR_ARGS;
  const int64_t R = (int64_t)H * S * K;
  const int64_t HE = (int64_t)H * E;
  if (R > NOALLOC_MAX_ROWS || HE > NOALLOC_MAX_EXPERTS ||
      global_sort_ws_bytes(H, S, K, E, NOALLOC_MIN_CHUNK) > NOALLOC_SCRATCH_BYTES) {
    set_last_error("mhmoe_global_sort_noalloc: " + std::to_string(R) + " routed rows / " + std::to_string(HE) +
                   " experts exceed the built-in scratch limits (" + std::to_string(NOALLOC_MAX_ROWS) +
                   " rows, " + std::to_string(NOALLOC_MAX_EXPERTS) + " experts); use mhmoe_global_sort");
    return MHMOE_ERR_CAPACITY;
  }
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) {
    set_last_error("mhmoe_global_sort_noalloc requires an sm_100 (B200) device");
    return MHMOE_ERR_ARCH;
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (S == 0) {
    return cudaMemsetAsync(expert_offsets, 0, sizeof(int64_t) * (HE + 1), st) == cudaSuccess ? MHMOE_OK
                                                                                            : MHMOE_ERR_LAUNCH;
  }
  void* ws = nullptr;
  cudaError_t e = scratch_address(&ws);
  if (e == cudaSuccess)
    e = launch_global_sort(topk_probs, topk_idx, H, S, K, E, ws, gather_ids, probs_sorted, expert_offsets,
                           row_of_flat, dev_status, st, NOALLOC_MIN_CHUNK);
  if (e != cudaSuccess) {
    set_last_error(std::string("mhmoe_global_sort_noalloc: ") + cudaGetErrorString(e));
    return MHMOE_ERR_LAUNCH;
  }
  return MHMOE_OK;
}
