// tcgen05 rates on one B200: the block-scaled FP4 MMA (M128 N256 K64, kind::mxf4nvf4
// block16) against the tcgen05.cp copies that bring its scale factors into tensor memory,
// with operands resident in shared memory (no TMA, no epilogue): the ceilings the expert
// GEMM (csrc/ffn_gemm.cuh) works against.  Timing only: operands are random bytes, scales
// 1.0, and the copy-shape variants do not lay the scales out the way the MMA reads them.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr \
//        -o tcgen05_rates magi-2-preview_b200/microbench/tcgen05_rates.cu
//   ./tcgen05_rates 20000           # single-CTA and CTA-pair variants
//   ./tcgen05_rates 20000 copies    # copy-shape variants
//
// One CTA per SM (120 KB of shared memory each; every CTA allocates all 512 TMEM columns).
// Every wait is bounded (2 s) and records an error code instead of hanging.
// Single CTA, per 256-K stage (4 MMAs): 0 MMAs only; 1 the 12 scale copies only
// (32x128b.warpx4: 4 A atoms + 8 B atoms); 2 copies + MMAs from one thread; 3 a copier warp
// and an MMA warp (the GEMM's split).  Copy shapes: 4 six 128x256b copies (the same bytes)
// only; 5 the same from a copier warp beside the MMA warp; 6 twelve 128x128b copies only.
// CTA pairs (cta_group::2, M = 256): 10 MMAs only; 11 twelve pair copies only; 12 copier +
// MMA warps; 13 the same with 8 copies.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../csrc/mhmoe_common.cuh"

using namespace mhmoe;

__device__ __forceinline__ uint32_t hash32(uint32_t x) {
  x ^= x >> 16; x *= 0x7feb352dU; x ^= x >> 15; x *= 0x846ca68bU; x ^= x >> 16;
  return x;
}

template <int VARIANT>
__global__ void __launch_bounds__(128, 1) mma_bench(int iters, long long* cyc, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + 16384;
  uint8_t* sSF = sB + 32768;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + 6144);   // [0,4) mma done per slot, [4,8) sf full per slot
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < (16384 + 32768) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = hash32(i * 2654435761u + blockIdx.x);
  for (int i = tid; i < 6144 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sSF)[i] = 0x38383838u;
  if (tid == 0) {
    for (int b = 0; b < 8; ++b) mbar_init(smem_u32(&bar[b]), 1);
    fence_mbar_init();
  }
  fence_proxy_async_shared();
  if (warp == 0) {
    tmem_alloc(smem_u32(tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tslot;
  const uint32_t a_s = smem_u32(sA), b_s = smem_u32(sB), sfa_s = smem_u32(sSF), sfb_s = sfa_s + 2048;
  constexpr uint32_t idesc = idesc_nvf4(128, 256);
  const uint64_t TO = 2000000000ull;
  if (VARIANT <= 2) {
    if (warp == 0 && lane == 0) {
      const long long t0 = clock64();
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
        if (VARIANT >= 1) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tc_cp_32x128b_warpx4(tsfa + j * 4, sdesc_sf_chunk(sfa_s + j * 512));
            tc_cp_32x128b_warpx4(tsfb + j * 8, sdesc_sf_chunk(sfb_s + j * 512));
            tc_cp_32x128b_warpx4(tsfb + j * 8 + 4, sdesc_sf_chunk(sfb_s + 2048 + j * 512));
          }
        }
        if (VARIANT != 1) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_nvf4(tb, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc, tsfa + j * 4,
                     tsfb + j * 8, (it | j) != 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bar[slot]));
        if (it >= 2) {
          const int w = it - 2;
          if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
        }
      }
      for (int w = iters >= 2 ? iters - 2 : 0; w < iters; ++w) mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
      cyc[blockIdx.x] = clock64() - t0;
    }
  } else {
    // warp 1: copier (slot s reused only after the MMAs that read it completed: bar[s]);
    // warp 0: MMA issuer, waits the slot's copies (bar[4+s]).
    if (warp == 1 && lane == 0) {
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        if (it >= 4) {
          const int w = it - 4;
          if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
        }
        const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          tc_cp_32x128b_warpx4(tsfa + j * 4, sdesc_sf_chunk(sfa_s + j * 512));
          tc_cp_32x128b_warpx4(tsfb + j * 8, sdesc_sf_chunk(sfb_s + j * 512));
          tc_cp_32x128b_warpx4(tsfb + j * 8 + 4, sdesc_sf_chunk(sfb_s + 2048 + j * 512));
        }
        tc_commit(smem_u32(&bar[4 + slot]));
      }
    }
    if (warp == 0 && lane == 0) {
      const long long t0 = clock64();
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        if (!mbar_wait(smem_u32(&bar[4 + slot]), (it >> 2) & 1, err, 4, TO)) break;
        tc_fence_after();
        const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_nvf4(tb, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc, tsfa + j * 4,
                   tsfb + j * 8, (it | j) != 0 ? 1u : 0u);
        tc_commit(smem_u32(&bar[slot]));
      }
      const int w = iters - 1;
      mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
      cyc[blockIdx.x] = clock64() - t0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tb, 512);
}

template <int V>
void run(int iters, int nsm) {
  const int smem = 120 * 1024;   // more than half the SM: one CTA per SM (each allocates all 512 TMEM columns)
  cudaFuncSetAttribute(mma_bench<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  long long* cyc;
  int* err;
  cudaMalloc(&cyc, nsm * sizeof(long long));
  cudaMalloc(&err, sizeof(int));
  cudaMemset(err, 0, sizeof(int));
  mma_bench<V><<<nsm, 128, smem>>>(100, cyc, err);   // warm-up
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  mma_bench<V><<<nsm, 128, smem>>>(iters, cyc, err);
  cudaEventRecord(e1);
  cudaError_t ce = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  std::vector<long long> h(nsm);
  int herr = 0;
  cudaMemcpy(h.data(), cyc, nsm * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (long long v : h) avg += (double)v;
  avg /= nsm;
  const double flops = 2.0 * 128 * 256 * 256 * (double)iters * nsm;
  printf("variant %d on %d SMs: %s err=%d  %.1f cycles/stage (%s)  %.3f ms  %.1f TFLOP/s\n", V, nsm,
         cudaGetErrorString(ce), herr, avg / iters,
         V == 1 ? "12 copies only" : (V == 0 ? "4 MMAs, no copies" : (V == 2 ? "12 copies + 4 MMAs, one thread"
                                                                               : "copier warp + MMA warp")),
         ms, V == 1 ? 0.0 : flops / (ms * 1e-3) / 1e12);
  cudaFree(cyc);
  cudaFree(err);
}


// Pair variants (cluster of 2, cta_group::2, M=256 per MMA across the pair): V 10 MMAs only,
// 11 12 copies only, 12 copier warp + MMA warp with 12 copies, 13 the same with 8 copies
// (4 SFA + 4 SFB: timing only).  All issued by the leader CTA.
template <int VARIANT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) mma_bench_pair(int iters, long long* cyc, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + 16384;            // 128 B-rows per CTA (half of N = 256)
  uint8_t* sSF = sB + 16384;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + 6144);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool leader = cluster_ctarank() == 0;
  for (int i = tid; i < (16384 + 16384) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = hash32(i * 2654435761u + blockIdx.x);
  for (int i = tid; i < 6144 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sSF)[i] = 0x38383838u;
  if (tid == 0) {
    for (int b = 0; b < 8; ++b) mbar_init(smem_u32(&bar[b]), 1);
    fence_mbar_init();
  }
  fence_proxy_async_shared();
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(tslot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tb = *tslot;
  const uint32_t a_s = smem_u32(sA), b_s = smem_u32(sB), sfa_s = smem_u32(sSF), sfb_s = sfa_s + 2048;
  constexpr uint32_t idesc = idesc_nvf4(256, 256);
  const uint64_t TO = 2000000000ull;
  constexpr int NCP = VARIANT == 13 ? 8 : 12;
  auto copies = [&](uint32_t tsfa, uint32_t tsfb) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      tc_cp_32x128b_warpx4_pair(tsfa + j * 4, sdesc_sf_chunk(sfa_s + j * 512));
      tc_cp_32x128b_warpx4_pair(tsfb + j * 8, sdesc_sf_chunk(sfb_s + j * 512));
      if (NCP == 12) tc_cp_32x128b_warpx4_pair(tsfb + j * 8 + 4, sdesc_sf_chunk(sfb_s + 2048 + j * 512));
    }
  };
  auto mmas = [&](uint32_t tsfa, uint32_t tsfb, int it) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      mma_nvf4_pair(tb, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc, tsfa + j * 4,
                    tsfb + j * 8, (it | j) != 0 ? 1u : 0u);
  };
  if (leader) {
    if (VARIANT <= 11) {
      if (warp == 0 && lane == 0) {
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
          const int slot = it & 3;
          const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
          if (VARIANT == 11) copies(tsfa, tsfb); else mmas(tsfa, tsfb, it);
          tc_commit_pair(mapa_shared(smem_u32(&bar[slot]), 0));
          if (it >= 2) {
            const int w = it - 2;
            if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
          }
        }
        for (int w = iters >= 2 ? iters - 2 : 0; w < iters; ++w) mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
        cyc[blockIdx.x / 2] = clock64() - t0;
      }
    } else {
      if (warp == 1 && lane == 0) {
        for (int it = 0; it < iters; ++it) {
          const int slot = it & 3;
          if (it >= 4) {
            const int w = it - 4;
            if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
          }
          const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
          copies(tsfa, tsfb);
          tc_commit_pair(mapa_shared(smem_u32(&bar[4 + slot]), 0));
        }
      }
      if (warp == 0 && lane == 0) {
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
          const int slot = it & 3;
          if (!mbar_wait(smem_u32(&bar[4 + slot]), (it >> 2) & 1, err, 4, TO)) break;
          tc_fence_after();
          const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
          mmas(tsfa, tsfb, it);
          tc_commit_pair(mapa_shared(smem_u32(&bar[slot]), 0));
        }
        const int w = iters - 1;
        mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
        cyc[blockIdx.x / 2] = clock64() - t0;
      }
    }
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tb, 512);
}

template <int V>
void run_pair(int iters, int nsm) {
  const int smem = 120 * 1024;
  cudaFuncSetAttribute(mma_bench_pair<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int nclu = nsm / 2;
  long long* cyc;
  int* err;
  cudaMalloc(&cyc, nclu * sizeof(long long));
  cudaMalloc(&err, sizeof(int));
  cudaMemset(err, 0, sizeof(int));
  mma_bench_pair<V><<<2 * nclu, 128, smem>>>(100, cyc, err);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  mma_bench_pair<V><<<2 * nclu, 128, smem>>>(iters, cyc, err);
  cudaEventRecord(e1);
  cudaError_t ce = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  std::vector<long long> h(nclu);
  int herr = 0;
  cudaMemcpy(h.data(), cyc, nclu * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (long long v : h) avg += (double)v;
  avg /= nclu;
  const double flops = 2.0 * 256 * 256 * 256 * (double)iters * nclu;
  printf("pair variant %d on %d clusters: %s err=%d  %.1f cycles/stage (%s)  %.3f ms  %.1f TFLOP/s\n", V, nclu,
         cudaGetErrorString(ce), herr, avg / iters,
         V == 10 ? "4 pair MMAs" : V == 11 ? "12 pair copies only" : V == 12 ? "copier + MMA, 12 copies"
                                                                            : "copier + MMA, 8 copies",
         ms, V == 11 ? 0.0 : flops / (ms * 1e-3) / 1e12);
  cudaFree(cyc);
  cudaFree(err);
}

__device__ __forceinline__ void tc_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_cp_128x128b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Copy-shape variants (timing only; the data layout is not the MMA's): 4: 6 x 128x256b
// copies only; 5: copier warp (6 x 128x256b) + MMA warp; 6: 12 x 128x128b copies only.
template <int VARIANT>
__global__ void __launch_bounds__(128, 1) cp_bench(int iters, long long* cyc, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + 16384;
  uint8_t* sSF = sB + 32768;                 // 6 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + 6144);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < (16384 + 32768) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = hash32(i * 2654435761u + blockIdx.x);
  for (int i = tid; i < 6144 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sSF)[i] = 0x38383838u;
  if (tid == 0) {
    for (int b = 0; b < 8; ++b) mbar_init(smem_u32(&bar[b]), 1);
    fence_mbar_init();
  }
  fence_proxy_async_shared();
  if (warp == 0) {
    tmem_alloc(smem_u32(tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tslot;
  const uint32_t a_s = smem_u32(sA), b_s = smem_u32(sB), sf_s = smem_u32(sSF);
  constexpr uint32_t idesc = idesc_nvf4(128, 256);
  const uint64_t TO = 2000000000ull;
  auto copies = [&](uint32_t tcol) {
    if (VARIANT == 6) {
#pragma unroll
      for (int j = 0; j < 12; ++j) tc_cp_128x128b(tcol + j * 4, make_sdesc(sf_s + (j & 1) * 2048, 0, 128, 0));
    } else {
#pragma unroll
      for (int j = 0; j < 6; ++j) tc_cp_128x256b(tcol + j * 8, make_sdesc(sf_s, 128, 256, 0));
    }
  };
  if (VARIANT != 5) {
    if (warp == 0 && lane == 0) {
      const long long t0 = clock64();
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        copies(tb + 256 + slot * 48);
        tc_commit(smem_u32(&bar[slot]));
        if (it >= 2) {
          const int w = it - 2;
          if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
        }
      }
      for (int w = iters >= 2 ? iters - 2 : 0; w < iters; ++w) mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
      cyc[blockIdx.x] = clock64() - t0;
    }
  } else {
    if (warp == 1 && lane == 0) {
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        if (it >= 4) {
          const int w = it - 4;
          if (!mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO)) break;
        }
        copies(tb + 256 + slot * 48);
        tc_commit(smem_u32(&bar[4 + slot]));
      }
    }
    if (warp == 0 && lane == 0) {
      const long long t0 = clock64();
      for (int it = 0; it < iters; ++it) {
        const int slot = it & 3;
        if (!mbar_wait(smem_u32(&bar[4 + slot]), (it >> 2) & 1, err, 4, TO)) break;
        tc_fence_after();
        const uint32_t tsfa = tb + 256 + slot * 48, tsfb = tsfa + 16;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_nvf4(tb, sdesc_kmajor_sw128(a_s + j * 32), sdesc_kmajor_sw128(b_s + j * 32), idesc, tsfa + j * 4,
                   tsfb + j * 8, (it | j) != 0 ? 1u : 0u);
        tc_commit(smem_u32(&bar[slot]));
      }
      const int w = iters - 1;
      mbar_wait(smem_u32(&bar[w & 3]), (w >> 2) & 1, err, 4, TO);
      cyc[blockIdx.x] = clock64() - t0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tb, 512);
}

template <int V>
void run_cp(int iters, int nsm) {
  const int smem = 120 * 1024;
  cudaFuncSetAttribute(cp_bench<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  long long* cyc;
  int* err;
  cudaMalloc(&cyc, nsm * sizeof(long long));
  cudaMalloc(&err, sizeof(int));
  cudaMemset(err, 0, sizeof(int));
  cp_bench<V><<<nsm, 128, smem>>>(100, cyc, err);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  cp_bench<V><<<nsm, 128, smem>>>(iters, cyc, err);
  cudaEventRecord(e1);
  cudaError_t ce = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  std::vector<long long> h(nsm);
  int herr = 0;
  cudaMemcpy(h.data(), cyc, nsm * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (long long v : h) avg += (double)v;
  avg /= nsm;
  const double flops = 2.0 * 128 * 256 * 256 * (double)iters * nsm;
  printf("copy variant %d: %s err=%d  %.1f cycles/stage (%s)  %.3f ms  %.1f TFLOP/s\n", V, cudaGetErrorString(ce),
         herr, avg / iters,
         V == 4 ? "6 x 128x256b only" : V == 5 ? "copier 6 x 128x256b + MMA warp" : "12 x 128x128b only", ms,
         V == 5 ? flops / (ms * 1e-3) / 1e12 : 0.0);
  cudaFree(cyc);
  cudaFree(err);
}

int main(int argc, char** argv) {
  int iters = argc > 1 ? atoi(argv[1]) : 20000;
  int nsm = 0;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0);
  run<0>(iters, nsm);
  run<1>(iters, nsm);
  run<2>(iters, nsm);
  run<3>(iters, nsm);
  run<0>(iters, 1);
  run<2>(iters, 1);
  if (argc > 2) {
    run_cp<4>(iters, nsm);
    run_cp<5>(iters, nsm);
    run_cp<6>(iters, nsm);
    return 0;
  }
  run_pair<10>(iters, nsm);
  run_pair<11>(iters, nsm);
  run_pair<12>(iters, nsm);
  run_pair<13>(iters, nsm);
  return 0;
}
