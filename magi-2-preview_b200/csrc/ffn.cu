// Host orchestration of the NVFP4 expert FFN: workspace carving, TMA descriptors and
// the launch sequence  tile tables -> gather/quantise -> gate/up GEMM (+SwiGLU7,
// hidden quantise) -> down GEMM (x prob) -> token map -> combine.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ffn_gemm.cuh"
#include "kernels.cuh"

namespace mhmoe {

// ───────────────────────────── driver entry points ─────────────────────────────

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// 2-D tensor map over [rows, inner] elements with the given row stride, 128-B swizzle.
cudaError_t encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                           uint64_t inner, uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                           uint32_t box_rows, bool swizzle128) {
  PFN_encodeTiled fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 2-D uint8 tensor map over [rows, inner_bytes] (row pitch = inner_bytes), 128-B swizzle.
cudaError_t encode_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows,
                              uint32_t box_inner, uint32_t box_rows) {
  return encode_tmap_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inner_bytes, rows, inner_bytes, box_inner,
                        box_rows);
}

int num_sms() {
  static int n_sms[MHMOE_MAX_DEVICES] = {};
  static PerDeviceOnce once;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MHMOE_MAX_DEVICES) return 148;
  once.run([](int d) {
    int n = 0;
    const cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    n_sms[d] = (e == cudaSuccess && n > 0) ? n : 148;
    return e;
  });
  return n_sms[dev];
}

// SF atom array of `bytes` bytes as [bytes/256, 256] u8 rows, box 256 x 8 (one 2 KB m/n-tile stage).
static cudaError_t encode_sf_map(CUtensorMap* map, const void* base, uint64_t bytes) {
  return encode_tmap_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 256, bytes / 256, 256, 256, 8, false);
}

// The CTA-pair GEMM is used when MHMOE_GEMM_PAIR=1.  It is correct but measured slower
// than one CTA per tile here: the tcgen05 pipe (scale-factor copies + MMAs) and load
// latency limit both, the pair pads every expert to 256 rows and couples two SMs.
static bool use_pair_gemm() {
  const char* v = std::getenv("MHMOE_GEMM_PAIR");
  return v && v[0] == '1';
}

template <int EPI>
static cudaError_t launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                                    const CUtensorMap& tsfa, const CUtensorMap& tsfb, const FfnGemmParams& p,
                                    int64_t max_work, cudaStream_t st) {
  // per device: the shared-memory attribute and the cluster occupancy of its context
  static PerDeviceOnce once;
  static int max_clusters[MHMOE_MAX_DEVICES] = {};
  const cudaError_t attr_err = once.run([](int dev) {
    cudaError_t e = cudaFuncSetAttribute(ffn_gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemmp_smem_bytes(EPI));
    if (e != cudaSuccess) return e;
    // the kernel's cluster shape (2, 1, 1) is compiled in, so the query config names none
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(GEMMP_THREADS);
    cfg.dynamicSmemBytes = gemmp_smem_bytes(EPI);
    e = cudaOccupancyMaxActiveClusters(&max_clusters[dev], ffn_gemm_pair_kernel<EPI>, &cfg);
    if (e == cudaSuccess && max_clusters[dev] <= 0) e = cudaErrorInvalidConfiguration;
    return e;
  });
  if (attr_err != cudaSuccess) return attr_err;
  int dev = 0;
  cudaGetDevice(&dev);
  const int clusters = (int)std::max<int64_t>(1, std::min<int64_t>(max_clusters[dev], max_work));
  ffn_gemm_pair_kernel<EPI><<<2 * clusters, GEMMP_THREADS, gemmp_smem_bytes(EPI), st>>>(ta, tb, tc, tsfa, tsfb, p);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                               const FfnGemmParams& p, int64_t max_work, cudaStream_t st) {
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), max_work));
  static PerDeviceOnce once[2];
  auto go = [&](auto kernel, int epw) -> cudaError_t {
    const cudaError_t attr_err = once[epw == 16].run([&](int) {
      return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(EPI));
    });
    if (attr_err != cudaSuccess) return attr_err;
    MHMOE_LAUNCH_PDL(kernel, grid, 32 * (3 + epw), gemm_smem_bytes(EPI), st, ta, tb, tc, p);
    return cudaGetLastError();
  };
  if constexpr (EPI == EPI_SWIGLU) {
    if (gemm_epi_warps(EPI, p.K) == 16) return go(ffn_gemm_nvfp4_kernel<EPI, 16>, 16);
  }
  return go(ffn_gemm_nvfp4_kernel<EPI, 8>, 8);
}

// ───────────────────────────── workspace layout ─────────────────────────────

struct FfnWorkspace {
  int* cu_tiles;
  int* tile_expert;
  int* tile_row0;
  int* tile_rows;
  int32_t* pad_of_row;   // [R] sorted row -> padded row
  uint8_t* xq;           // [T, dh/2]  per-token quantised x (T = S*H rows, row = s*H + h)
  uint8_t* xsf;          // [T, dh/16] row-major scales
  float* xg;             // [T]
  uint8_t* a_data;       // [rows_pad, dh/2] grouped A operand of the gate/up GEMM
  uint8_t* a_sf;         // SF atoms of a_data
  float* a_gscale;       // [rows_pad]
  uint8_t* h_data;       // [rows_pad, de/2] quantised SwiGLU hidden
  uint8_t* h_sf;         // SF atoms of the hidden
  __nv_bfloat16* P;      // [rows_pad, dh] bf16(y_acc * prob) per padded row
  int32_t* tok_offsets;
  int32_t* tok_rows;
  void* tok_ws;
  size_t bytes;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static FfnWorkspace carve(uint8_t* base, int64_t R, int64_t T, int dh, int de, int HE) {
  FfnWorkspace w{};
  const int64_t mt = mtiles_upper_bound(R, HE, 2);     // covers both tile alignments
  const int64_t rows = mt * 128;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off = align_up(off + bytes, 1024);
    return p;
  };
  w.cu_tiles = reinterpret_cast<int*>(take(sizeof(int) * (HE + 1)));
  w.tile_expert = reinterpret_cast<int*>(take(sizeof(int) * mt));
  w.tile_row0 = reinterpret_cast<int*>(take(sizeof(int) * mt));
  w.tile_rows = reinterpret_cast<int*>(take(sizeof(int) * mt));
  w.pad_of_row = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(R, 1)));
  w.xq = take((size_t)T * dh / 2);
  w.xsf = take((size_t)T * dh / 16);
  w.xg = reinterpret_cast<float*>(take(sizeof(float) * T));
  w.a_data = take((size_t)rows * dh / 2);
  w.a_sf = take((size_t)rows * dh / 16);
  w.a_gscale = reinterpret_cast<float*>(take(sizeof(float) * rows));
  w.h_data = take((size_t)rows * de / 2);
  w.h_sf = take((size_t)rows * de / 16);
  w.P = reinterpret_cast<__nv_bfloat16*>(take(sizeof(__nv_bfloat16) * (size_t)rows * dh));
  w.tok_offsets = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (T + 1)));
  w.tok_rows = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * std::max<int64_t>(R, 1)));
  w.tok_ws = take(token_rows_ws_bytes(T));
  w.bytes = off;
  return w;
}

size_t ffn_workspace_bytes(int64_t R, int64_t T, int dh, int de, int HE) {
  return carve(nullptr, R, T, dh, de, HE).bytes;
}

int ffn_nvfp4(const __nv_bfloat16* x, int64_t sx_s, int64_t sx_h, int S, int H, int dh, int de, int HE, int64_t R,
              const int32_t* gather_ids, const float* probs_sorted, const int64_t* expert_offsets,
              const uint8_t* gu_data, const uint8_t* gu_sf, const float* gu_gscale, const uint8_t* dn_data,
              const uint8_t* dn_sf, const float* dn_gscale, const int32_t* tok_rows, const int32_t* tok_offsets,
              int k_fixed, void* workspace, __nv_bfloat16* y, int64_t sy_s, int64_t sy_h, int* status,
              uint64_t timeout_ns, const cudaEvent_t* events, cudaStream_t st, cudaError_t* cerr,
              const uint8_t* xq_in, const uint8_t* xsf_in, const uint8_t* xg_in, int64_t xq_pitch, int64_t xsf_pitch,
              int64_t xg_pitch, const EpReturn* ret, bool atomic_scatter) {
  const int64_t T = (int64_t)S * H;
  FfnWorkspace w = carve(static_cast<uint8_t*>(workspace), R, T, dh, de, HE);
  const bool prequant = xq_in != nullptr;
  const uint8_t* xq = prequant ? xq_in : w.xq;
  const uint8_t* xsf = prequant ? xsf_in : w.xsf;
  const uint8_t* xg = prequant ? xg_in : reinterpret_cast<const uint8_t*>(w.xg);
  if (!prequant) {
    xq_pitch = dh / 2;
    xsf_pitch = dh / 16;
    xg_pitch = sizeof(float);
  }
  const bool pair = use_pair_gemm();
  const int64_t max_mt = mtiles_upper_bound(R, HE, 2);
  const int64_t rows = max_mt * 128;
  cudaError_t e;
#define MHMOE_TRY(call)        \
  do {                         \
    e = (call);                \
    if (e != cudaSuccess) {    \
      *cerr = e;               \
      return MHMOE_ERR_LAUNCH; \
    }                          \
  } while (0)

  auto mark = [&](int i) {
    if (events && events[i]) cudaEventRecord(events[i], st);
  };
  mark(0);
  MHMOE_TRY(launch_tile_tables(expert_offsets, HE, max_mt, w.cu_tiles, w.tile_expert, w.tile_row0, w.tile_rows,
                               status, st, pair ? 2 : 1));
  // key (h, s) -> its sorted rows: the caller's inverse map, else built from the tile tables
  const int32_t* rows_map = tok_rows;
  const int32_t* offs_map = tok_offsets;
  int kf = k_fixed;
  if (!tok_rows) {
    MHMOE_TRY(launch_token_rows(gather_ids, max_mt, w.cu_tiles, HE, HE / H, S, H, w.tile_expert, w.tile_row0,
                                w.tile_rows, w.tok_ws, w.tok_offsets, w.tok_rows, status, st));
    rows_map = w.tok_rows;
    offs_map = w.tok_offsets;
    kf = 0;
  }
  // Local tokens are quantised once and written straight into their grouped rows; tokens
  // that arrive pre-quantised (expert-parallel receive) are grouped by copy.
  const char* qenv = std::getenv("MHMOE_QUANT_FUSED");
  const bool fused = !prequant && dh <= quant_scatter_max_dh() && !(qenv && qenv[0] == '0');
  // (the A operand's padding rows stay unwritten: each row's GEMM results depend on that row
  // alone, and nothing reads a padding row's hidden or partial output)
  MHMOE_TRY(launch_pad_rows(w.cu_tiles, HE, max_mt, w.tile_row0, w.tile_rows, w.pad_of_row, st));
  if (fused) {
    MHMOE_TRY(launch_quant_scatter(x, sx_s, sx_h, S, H, dh, rows_map, offs_map, kf, R, w.pad_of_row, rows, w.a_data,
                                   w.a_sf, w.a_gscale, status, st));
  } else {
    if (!prequant) MHMOE_TRY(launch_quant_tokens(x, sx_s, sx_h, S, H, dh, w.xq, w.xsf, w.xg, st));
    MHMOE_TRY(launch_group_rows(xq, xq_pitch, xsf, xsf_pitch, xg, xg_pitch, T, dh, H, HE / H, gather_ids, w.cu_tiles,
                                HE, max_mt, w.tile_expert, w.tile_row0, w.tile_rows, w.a_data, w.a_sf, w.a_gscale,
                                status, st));
  }

  CUtensorMap ta1, tb1, ta2, tb2, tc2;
  if (encode_tmap_2d_u8(&ta1, w.a_data, dh / 2, rows, 128, 128) != cudaSuccess ||
      encode_tmap_2d_u8(&tb1, gu_data, dh / 2, (uint64_t)HE * 2 * de, 128, 256) != cudaSuccess ||
      encode_tmap_2d_u8(&ta2, w.h_data, de / 2, rows, 128, 128) != cudaSuccess ||
      encode_tmap_2d_u8(&tb2, dn_data, de / 2, (uint64_t)HE * dh, 128, 256) != cudaSuccess ||
      encode_tmap_2d(&tc2, w.P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dh, rows, (uint64_t)dh * 2, 64, 32) !=
          cudaSuccess)
    return MHMOE_ERR_DRIVER;
  // CTA-pair operands: B tiles of 128 rows, SF atoms through TMA
  CUtensorMap tb1p, tb2p, tsfa1, tsfb1, tsfa2, tsfb2;
  if (pair && (encode_tmap_2d_u8(&tb1p, gu_data, dh / 2, (uint64_t)HE * 2 * de, 128, 128) != cudaSuccess ||
               encode_tmap_2d_u8(&tb2p, dn_data, de / 2, (uint64_t)HE * dh, 128, 128) != cudaSuccess ||
               encode_sf_map(&tsfa1, w.a_sf, (uint64_t)rows * dh / 16) != cudaSuccess ||
               encode_sf_map(&tsfb1, gu_sf, (uint64_t)HE * 2 * de * dh / 16) != cudaSuccess ||
               encode_sf_map(&tsfa2, w.h_sf, (uint64_t)rows * de / 16) != cudaSuccess ||
               encode_sf_map(&tsfb2, dn_sf, (uint64_t)HE * dh * de / 16) != cudaSuccess))
    return MHMOE_ERR_DRIVER;

  mark(1);
  FfnGemmParams p1{};
  p1.sfa = w.a_sf;
  p1.sfb = gu_sf;
  p1.n_mtiles_dev = w.cu_tiles + HE;
  p1.n_mtiles_host = (int)max_mt;
  p1.tile_expert = w.tile_expert;
  p1.tile_row0 = w.tile_row0;
  p1.tile_rows = w.tile_rows;
  p1.K = dh;
  p1.N = 2 * de;
  p1.row_gscale = w.a_gscale;
  p1.gs_gate = gu_gscale;
  p1.gs_up = gu_gscale + HE;
  p1.h_data = w.h_data;
  p1.h_sf = w.h_sf;
  p1.status = status;
  p1.timeout_ns = timeout_ns;
  if (pair)
    MHMOE_TRY(launch_gemm_pair<EPI_SWIGLU>(ta1, tb1p, ta1, tsfa1, tsfb1, p1, max_mt / 2 * (2 * de / GEMM_BN), st));
  else
    MHMOE_TRY(launch_gemm<EPI_SWIGLU>(ta1, tb1, ta1, p1, max_mt * (2 * de / GEMM_BN), st));

  mark(2);
  FfnGemmParams p2 = p1;
  p2.sfa = w.h_sf;
  p2.sfb = dn_sf;
  p2.K = de;
  p2.N = dh;
  p2.probs = probs_sorted;
  p2.gs_down = dn_gscale;
  if (atomic_scatter) {
    // reference default scatter: bf16 atomics into the zeroed output, no partials / combine
    p2.y = y;
    p2.sy_s = sy_s;
    p2.sy_h = sy_h;
    p2.gather_ids = gather_ids;
    p2.experts_per_head = HE / H;
    MHMOE_TRY(launch_zero_rows(y, S, H, dh, sy_s, sy_h, st));
    if (pair)
      MHMOE_TRY(launch_gemm_pair<EPI_DOWN_ATOMIC>(ta2, tb2p, tc2, tsfa2, tsfb2, p2, max_mt / 2 * (dh / GEMM_BN), st));
    else
      MHMOE_TRY(launch_gemm<EPI_DOWN_ATOMIC>(ta2, tb2, tc2, p2, max_mt * (dh / GEMM_BN), st));
    mark(3);
    mark(4);
    return MHMOE_OK;
  }
  if (pair)
    MHMOE_TRY(launch_gemm_pair<EPI_DOWN>(ta2, tb2p, tc2, tsfa2, tsfb2, p2, max_mt / 2 * (dh / GEMM_BN), st));
  else
    MHMOE_TRY(launch_gemm<EPI_DOWN>(ta2, tb2, tc2, p2, max_mt * (dh / GEMM_BN), st));

  mark(3);
  if (ret)
    MHMOE_TRY(launch_combine_return(w.P, w.pad_of_row, dh, rows_map, kf, R, rows, *ret, st));
  else
    MHMOE_TRY(launch_combine(w.P, w.pad_of_row, dh, S, H, rows_map, offs_map, kf, R, rows, y, sy_s, sy_h, st));
  mark(4);
#undef MHMOE_TRY
  return MHMOE_OK;
}

int gemm_nvfp4_raw(const uint8_t* a_data, const uint8_t* a_sf, int n_mtiles, const int32_t* tile_expert,
                   const uint8_t* b_data, const uint8_t* b_sf, int n_experts, int N, int K, float* out, int* status,
                   uint64_t timeout_ns, cudaStream_t st, cudaError_t* cerr) {
  CUtensorMap ta, tb;
  if (encode_tmap_2d_u8(&ta, a_data, K / 2, (uint64_t)n_mtiles * 128, 128, 128) != cudaSuccess ||
      encode_tmap_2d_u8(&tb, b_data, K / 2, (uint64_t)n_experts * N, 128, 256) != cudaSuccess)
    return MHMOE_ERR_DRIVER;
  FfnGemmParams p{};
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.n_mtiles_dev = nullptr;
  p.n_mtiles_host = n_mtiles;
  p.tile_expert = tile_expert;
  p.K = K;
  p.N = N;
  p.out_f32 = out;
  p.status = status;
  p.timeout_ns = timeout_ns;
  const cudaError_t e = launch_gemm<EPI_RAW>(ta, tb, ta, p, (int64_t)n_mtiles * (N / GEMM_BN), st);
  if (e != cudaSuccess) {
    *cerr = e;
    return MHMOE_ERR_LAUNCH;
  }
  return MHMOE_OK;
}

}  // namespace mhmoe
