// Fused router on the tensor cores: fp32-accurate logits from bf16 tcgen05 MMAs, with
// scoring, top-k, normalisation and route_scale in the epilogue.
//
// Replaces CoreMultiHeadMoE._route (inference/model/magi2_preview.py:2588-2601): the
// fp32 einsum("shd,hed->hse") and compute_topk_probs_and_indices
// (inference/flash_mh_moe/route.py:28-148, no virtual groups — MAGI-2 does not use them).
//
// Precision: x is bf16, so x * g for an fp32 gate weight g = hi + lo + lo2 (three bf16
// planes, hi = bf16(g), lo = bf16(g - hi), lo2 = bf16(g - hi - lo)) is the sum of three
// exactly representable products; the MMA accumulates them in fp32.  The logits match an
// fp32 GEMM to fp32 rounding.  Gate planes that are all zero are skipped (nsplit < 3),
// e.g. a bf16-valued gate needs one plane.
//
// GEMM shape per tile: M = 128 tokens (one head), N = E rounded up to 16 (<= 256),
// K' = nsplit * dh, iterated as (dh block of 64, plane) so each x tile is re-read from L2
// right after its first load.  Warp 0: TMA producer (x tile 128x64 bf16, gate tile
// Nx64 bf16, 128-B swizzle, up to 8 stages); warp 1: TMEM owner + MMA issuer
// (tcgen05.mma kind::f16, M128 N<=256 K16); warps 2-17: epilogue.  Epilogue warp w reads
// TMEM lane quarter q = w % 4 (rows 32q..32q+31, one per lane) and column group
// g = (w - 2) / 4, a contiguous quarter of the 32-column chunks, so each row's scoring is
// spread over four warps: partial row max and softmax sums are combined through shared
// memory in group order, each warp keeps a top-k list of its columns in registers
// (branch-free insertion; 8 entries for K <= 8, else 16), and the four lists of a row are
// merged in two rounds (group 1 into 0 and 3 into 2, then 2 into 0) — lower groups hold
// lower experts, so the merge keeps the order (score desc, expert asc) of one sequential
// pass.
#include <cstdlib>
#include <mutex>

#include "kernels.cuh"

namespace mhmoe {

constexpr int RT_BM = 128;
constexpr int RT_BK = 64;                // bf16 elements per stage row (128 B)
constexpr int RT_MAX_STAGES = 8;        // as many as shared memory holds (6 at N = 128)
constexpr int RT_EPI_WARPS = 16;
constexpr int RT_THREADS = 64 + 32 * RT_EPI_WARPS;
// shared scratch after the barriers: row max and softmax partials [4 groups][128 rows] fp32,
// then the merge buffer [4 quarters][2 slots][KM][32 lanes] x (value, expert, score)
constexpr int RT_RED_BYTES = 2 * 4 * 128 * 4;
__host__ __device__ constexpr int rt_merge_bytes(int km) { return 4 * 2 * km * 32 * 12; }


struct RouterParams {
  const float* logit_bias; // [H*E] or null: added to the logits before scoring
  const float* bias;       // [H*E] or null
  float* probs;            // [H, S, K]
  int64_t* idx;            // [H, S, K]
  float* logits;           // [H, S, E] or null
  int S, H, dh, E, Npad, K, nsplit, score_func, route_norm, stages;
  float norm_eps, route_scale;
  int* status;
  uint64_t timeout_ns;
};

// Insert (v, e, sc) into the descending list tv[0..KM) without branches: every entry
// takes its new value by selects, so lanes never diverge.  v enters above an entry only
// when strictly larger, and values arrive in ascending expert order, so equal values keep
// the lower expert first.  NaN and -inf never enter.
template <int KM>
__device__ __forceinline__ void topk_insert(float v, int e, float sc, float (&tv)[KM], int (&ti)[KM],
                                            float (&ts)[KM]) {
#pragma unroll
  for (int j = KM - 1; j >= 1; --j) {
    const bool above_prev = v > tv[j - 1];
    const bool above_cur = v > tv[j];
    tv[j] = above_prev ? tv[j - 1] : (above_cur ? v : tv[j]);
    ti[j] = above_prev ? ti[j - 1] : (above_cur ? e : ti[j]);
    ts[j] = above_prev ? ts[j - 1] : (above_cur ? sc : ts[j]);
  }
  const bool top = v > tv[0];
  tv[0] = top ? v : tv[0];
  ti[0] = top ? e : ti[0];
  ts[0] = top ? sc : ts[0];
}

// SF: the score function (0 softmax, 1 sigmoid), fixed per instantiation so the per-score
// code carries no branch on it.
template <int KM, int SF>
__global__ void __launch_bounds__(RT_THREADS, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
                     const RouterParams p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = RT_BM * RT_BK * 2;
  const int b_bytes = p.Npad * RT_BK * 2;
  uint8_t* sA = smem;
  const int STAGES = p.stages;
  uint8_t* sB = sA + STAGES * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * b_bytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + RT_MAX_STAGES;
  uint64_t* tfull_bar = bars + 2 * RT_MAX_STAGES;
  uint64_t* tempty_bar = tfull_bar + 1;
  uint64_t* drain_bar = tfull_bar + 2;
  uint64_t* qbar = drain_bar + 1;                  // [4] the four epilogue warps of a lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qbar + 4);
  float* red_max = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [4][128]
  float* red_sum = red_max + 4 * 128;                                                  // [4][128]
  float* mg_v = red_sum + 4 * 128;                                                     // [4][2][KM][32]
  int* mg_e = reinterpret_cast<int*>(mg_v + 4 * 2 * KM * 32);
  float* mg_s = reinterpret_cast<float*>(mg_e + 4 * 2 * KM * 32);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tcols = p.Npad <= 32 ? 32 : p.Npad <= 64 ? 64 : p.Npad <= 128 ? 128 : 256;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(tfull_bar), 1);
    mbar_init(smem_u32(tempty_bar), RT_EPI_WARPS);
    mbar_init(smem_u32(drain_bar), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&qbar[i]), 128);
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmG);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int mtiles = (p.S + RT_BM - 1) / RT_BM;
  const int total = mtiles * p.H;
  const int nkb = p.dh / RT_BK;
  const int nk = nkb * p.nsplit;
  const uint64_t timeout = p.timeout_ns ? p.timeout_ns : 2000000000ull;

  if (warp == 0) {
    // producer: the whole warp loops and waits, lane 0 issues
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const int h = t / mtiles, mt = t % mtiles;
      for (int k = 0; k < nk; ++k) {
        const int kb = k / p.nsplit, sp = k % p.nsplit;
        if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, (uint32_t)(a_bytes + b_bytes));
          tma_load_2d(smem_u32(sA + stage * a_bytes), &tmX, fb, h * p.dh + kb * RT_BK, mt * RT_BM);
          tma_load_2d(smem_u32(sB + stage * b_bytes), &tmG, fb, (kb * p.nsplit + sp) * RT_BK, h * p.E);
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // every load issued lands before the CTA exits (returns at once on the normal path)
    for (int64_t i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
      mbar_wait(smem_u32(&full_bar[i % STAGES]), (uint32_t)((i / STAGES) & 1), nullptr, 0, MHMOE_DRAIN_NS);
  } else if (warp == 1) {
    // MMA issuer: the whole warp loops and waits, lane 0 issues
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0;
    const uint32_t idesc = idesc_bf16(RT_BM, p.Npad);
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      if (!mbar_wait(smem_u32(tempty_bar), acc_phase ^ 1, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
      tc_fence_after();
      for (int k = 0; k < nk; ++k) {
        if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) goto done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_s = smem_u32(sA + stage * a_bytes);
          const uint32_t b_s = smem_u32(sB + stage * b_bytes);
#pragma unroll
          for (int j = 0; j < RT_BK / 16; ++j)
            mma_bf16(tmem_base, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc,
                     (k | j) != 0 ? 1u : 0u);
          tc_commit(smem_u32(&empty_bar[stage]));
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (lane == 0) tc_commit(smem_u32(tfull_bar));
      __syncwarp();
      acc_phase ^= 1;
    }
  } else {
    // epilogue: lane quarter q, column group g; one token row per lane
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    const int m = q * 32 + lane;
    const int nchunk = p.Npad / 32 + (p.Npad % 32 ? 1 : 0);
    const int cpg = (nchunk + 3) / 4;                    // chunks per group (contiguous)
    const int c0 = min(nchunk, g * cpg), c1 = min(nchunk, c0 + cpg);
    uint32_t acc_phase = 0, q_phase = 0;
    // every thread of the quarter's four warps arrives, then waits (bounded) for the rest
    auto quarter_sync = [&]() -> bool {
      mbar_arrive(smem_u32(&qbar[q]));
      const bool ok = mbar_wait(smem_u32(&qbar[q]), q_phase, p.status, MHMOE_ERR_TIMEOUT, timeout);
      q_phase ^= 1;
      return ok;
    };
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int h = t / mtiles, mt = t % mtiles;
      if (!mbar_wait(smem_u32(tfull_bar), acc_phase, p.status, MHMOE_ERR_TIMEOUT, timeout)) break;
      acc_phase ^= 1;
      tc_fence_after();
      const int s = mt * RT_BM + m;
      const bool valid = s < p.S;
      const int64_t row = (int64_t)h * p.S + s;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);
      const float* lb = p.logit_bias ? p.logit_bias + (int64_t)h * p.E : nullptr;
      uint32_t r[32];
      // pass 1: row max over this group's columns (and the optional logits output); the
      // sigmoid scores need neither, so without a logits output the pass is skipped
      float mx = -INFINITY;
      const bool pass1 = SF == 0 || p.logits;
      for (int c = c0; pass1 && c < c1; ++c) {
        MHMOE_TMEM_LD_32x32b_X32(taddr + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int e = c * 32 + i;
          if (e < p.E) {
            const float l = lb ? __fadd_rn(__uint_as_float(r[i]), lb[e]) : __uint_as_float(r[i]);
            mx = fmaxf(mx, l);
            if (valid && p.logits) p.logits[row * p.E + e] = l;
          }
        }
      }
      if (SF == 0) {
        red_max[g * 128 + m] = mx;
        if (!quarter_sync()) break;
        mx = fmaxf(fmaxf(red_max[m], red_max[128 + m]), fmaxf(red_max[256 + m], red_max[384 + m]));
      }
      // pass 2: softmax denominator, ascending experts within the group, groups in order
      float sum = 0.f;
      if (SF == 0) {
        float part = 0.f;
        for (int c = c0; c < c1; ++c) {
          MHMOE_TMEM_LD_32x32b_X32(taddr + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int e = c * 32 + i;
            if (e < p.E) part += expf((lb ? __fadd_rn(__uint_as_float(r[i]), lb[e]) : __uint_as_float(r[i])) - mx);
          }
        }
        red_sum[g * 128 + m] = part;
        if (!quarter_sync()) break;
        sum = red_sum[m];
        sum += red_sum[128 + m];
        sum += red_sum[256 + m];
        sum += red_sum[384 + m];
      }
      // pass 3: scores and selection values, inserted into this group's top-KM list
      float tv[KM], ts[KM];
      int ti[KM];
#pragma unroll
      for (int j = 0; j < KM; ++j) {
        tv[j] = -INFINITY;
        ts[j] = 0.f;
        ti[j] = 0;
      }
      // score of logit l: softmax exp(l - max) / sum, or sigmoid 1 / (1 + exp(-l)) (the
      // correctly rounded reciprocal equals the correctly rounded quotient 1 / y)
      auto score_of = [&](float l) -> float {
        if constexpr (SF == 0) return __fdiv_rn(expf(l - mx), sum);
        else return __frcp_rn(1.0f + expf(-l));
      };
      // without logit or selection bias the selection value is the score: a loop with no
      // per-score branches
      const bool plain = lb == nullptr && p.bias == nullptr;
      for (int c = c0; c < c1; ++c) {
        MHMOE_TMEM_LD_32x32b_X32(taddr + c * 32, r);
        tmem_wait_ld();
        if (plain) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int e = c * 32 + i;
            const float sc = score_of(__uint_as_float(r[i]));
            topk_insert<KM>(e < p.E ? sc : -INFINITY, e, sc, tv, ti, ts);
          }
          continue;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int e = c * 32 + i;
          float v = -INFINITY, sc = 0.f;
          if (e < p.E) {
            const float l = lb ? __fadd_rn(__uint_as_float(r[i]), lb[e]) : __uint_as_float(r[i]);
            sc = score_of(l);
            v = p.bias ? __fadd_rn(sc, p.bias[(int64_t)h * p.E + e]) : sc;
          }
          topk_insert<KM>(v, e, sc, tv, ti, ts);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tempty_bar));
      // merge: first step 1 -> 0 and 3 -> 2, second step 2 -> 0; slot index [q][slot][j][lane]
      auto put = [&](int slot) {
#pragma unroll
        for (int j = 0; j < KM; ++j) {
          const int o = ((q * 2 + slot) * KM + j) * 32 + lane;
          mg_v[o] = tv[j];
          mg_e[o] = ti[j];
          mg_s[o] = ts[j];
        }
      };
      auto take = [&](int slot) {
#pragma unroll
        for (int j = 0; j < KM; ++j) {
          const int o = ((q * 2 + slot) * KM + j) * 32 + lane;
          topk_insert<KM>(mg_v[o], mg_e[o], mg_s[o], tv, ti, ts);
        }
      };
      if (g & 1) put(g >> 1);
      if (!quarter_sync()) break;
      if (!(g & 1)) take(g >> 1);
      if (!quarter_sync()) break;
      if (g == 2) put(0);
      if (!quarter_sync()) break;
      if (g == 0) {
        take(0);
        if (valid) {
          float nrm = 1.f;
          if (p.route_norm) {
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < KM; ++j)
              if (j < p.K) a += fabsf(ts[j]);
            nrm = fmaxf(a, p.norm_eps);
          }
#pragma unroll
          for (int j = 0; j < KM; ++j) {
            if (j < p.K) {
              const float pr = p.route_norm ? __fdiv_rn(ts[j], nrm) : ts[j];
              p.probs[row * p.K + j] = __fmul_rn(pr, p.route_scale);
              p.idx[row * p.K + j] = ti[j];
            }
          }
        }
      }
    }
  }
done:
  if (warp == 1 && lane == 0) {
    tc_commit(smem_u32(drain_bar));
    mbar_wait(smem_u32(drain_bar), 0, nullptr, 0, MHMOE_DRAIN_NS);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

// gate fp32 [HE, dh] -> planes bf16 [HE, nsplit*dh], interleaved per 64-column block:
// out[r, (kb*nsplit + s)*64 + j] = plane_s[r, kb*64 + j].  flags[s] |= plane s non-zero.
__global__ void split_gate_kernel(const float* __restrict__ gate, int64_t HE, int dh, int nsplit,
                                  __nv_bfloat16* __restrict__ out, int* __restrict__ flags) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= HE * dh) return;
  const int64_t r = i / dh;
  const int d = (int)(i % dh);
  const float g = gate[i];
  const __nv_bfloat16 hi = __float2bfloat16_rn(g);
  const float rem1 = g - __bfloat162float(hi);
  const __nv_bfloat16 lo = __float2bfloat16_rn(rem1);
  const float rem2 = rem1 - __bfloat162float(lo);
  const __nv_bfloat16 lo2 = __float2bfloat16_rn(rem2);
  const __nv_bfloat16 planes[3] = {hi, lo, lo2};
  const int kb = d / 64, j = d % 64;
  for (int s = 0; s < nsplit; ++s) {
    out[r * (int64_t)nsplit * dh + (int64_t)(kb * nsplit + s) * 64 + j] = planes[s];
  }
  if (flags) {
    if (__bfloat162float(lo) != 0.f) atomicOr(&flags[1], 1);
    if (__bfloat162float(lo2) != 0.f) atomicOr(&flags[2], 1);
  }
}

// 2-D bf16 tensor map [rows, inner] with the given row stride, 128-B swizzle.
static cudaError_t encode_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  return encode_tmap_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, rows, row_stride_bytes, box_inner,
                        box_rows);
}

cudaError_t launch_split_gate(const float* gate, int64_t HE, int dh, int nsplit, __nv_bfloat16* out, int* flags,
                              cudaStream_t st) {
  const int64_t n = HE * dh;
  split_gate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(gate, HE, dh, nsplit, out, flags);
  return cudaGetLastError();
}

int router_tc(const __nv_bfloat16* x, int64_t sx_s, const __nv_bfloat16* gate_planes, int nsplit, int S, int H,
              int dh, int E, int K, int score_func, const float* logit_bias, const float* bias, int route_norm,
              float norm_eps, float route_scale, float* probs, int64_t* idx, float* logits, int* status,
              cudaStream_t st, cudaError_t* cerr) {
  if (router_small_supported(S, H, dh, E, K) && !std::getenv("MHMOE_ROUTER_TC_ONLY")) {
    // a batch of a few tiles: split the reduction over clusters of CTAs instead
    const cudaError_t e = launch_router_small(x, sx_s, gate_planes, nsplit, S, H, dh, E, K, score_func, logit_bias,
                                              bias, route_norm, norm_eps, route_scale, probs, idx, logits, st);
    if (e != cudaSuccess) {
      *cerr = e;
      return MHMOE_ERR_LAUNCH;
    }
    return MHMOE_OK;
  }
  const int Npad = std::max(16, (E + 15) / 16 * 16);
  CUtensorMap tx, tg;
  if (encode_bf16_2d(&tx, x, (uint64_t)H * dh, (uint64_t)S, (uint64_t)sx_s * 2, RT_BK, RT_BM) != cudaSuccess ||
      encode_bf16_2d(&tg, gate_planes, (uint64_t)nsplit * dh, (uint64_t)H * E, (uint64_t)nsplit * dh * 2, RT_BK,
                     (uint32_t)Npad) != cudaSuccess)
    return MHMOE_ERR_DRIVER;
  RouterParams p{};
  p.logit_bias = logit_bias;
  p.bias = bias;
  p.probs = probs;
  p.idx = idx;
  p.logits = logits;
  p.S = S;
  p.H = H;
  p.dh = dh;
  p.E = E;
  p.Npad = Npad;
  p.K = K;
  p.nsplit = nsplit;
  p.score_func = score_func;
  p.route_norm = route_norm;
  p.norm_eps = norm_eps;
  p.route_scale = route_scale;
  p.status = status;
  const int stage_bytes = RT_BM * RT_BK * 2 + Npad * RT_BK * 2;
  const int fixed = 256 + RT_RED_BYTES + rt_merge_bytes(K <= 8 ? 8 : 16) + 1024;
  p.stages = std::min(RT_MAX_STAGES, (227 * 1024 - fixed) / stage_bytes);
  const int smem = p.stages * stage_bytes + fixed;
  // top-K lists of 8 entries cover K <= 8; 16 entries otherwise (K <= 16)
  auto kernel = K <= 8 ? (score_func == 0 ? router_tc_kernel<8, 0> : router_tc_kernel<8, 1>)
                       : (score_func == 0 ? router_tc_kernel<16, 0> : router_tc_kernel<16, 1>);
  static PerDeviceOnce once;
  const cudaError_t attr = once.run([](int) {
    cudaError_t e = cudaSuccess;
    for (auto k : {router_tc_kernel<8, 0>, router_tc_kernel<8, 1>, router_tc_kernel<16, 0>, router_tc_kernel<16, 1>})
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    return e;
  });
  if (attr != cudaSuccess) {
    *cerr = attr;
    return MHMOE_ERR_LAUNCH;
  }
  const int tiles = ((S + RT_BM - 1) / RT_BM) * H;
  const int grid = std::max(1, std::min(tiles, num_sms()));
  const cudaError_t e = launch_pdl(kernel, dim3(grid), dim3(RT_THREADS), (size_t)smem, st, tx, tg, p);
  if (e != cudaSuccess) {
    *cerr = e;
    return MHMOE_ERR_LAUNCH;
  }
  return MHMOE_OK;
}

}  // namespace mhmoe
