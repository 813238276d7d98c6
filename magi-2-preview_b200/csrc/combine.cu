// Deterministic weighted combine: y[s, h, :] = bf16( sum over the (token, head)'s
// routed rows r, in ascending r, of P[r, :] ) with fp32 accumulation.
//
// Replaces the scatter of the reference FFN: the bf16 atomic_add of
// _mh_moe_fwd_kernel (inference/flash_mh_moe/triton/mh_moe_fwd.py:172-181) and the
// deterministic _scatter_back (:189-215).  P already holds bf16(y_acc * prob) per
// sorted row, exactly the values the reference scatters; the sum is taken in fp32
// in a fixed order, so the result is run-to-run identical.
#include <cstdlib>

#include "kernels.cuh"

namespace mhmoe {

constexpr int COMBINE_WARPS = 4;

// pad_of_row[r] = padded row of sorted row r: mt * 128 + m for tile rows m < tile_rows[mt].
__global__ void pad_rows_kernel(const int* __restrict__ cu_tiles, int HE, const int* __restrict__ tile_row0,
                                const int* __restrict__ tile_rows, int32_t* __restrict__ pad_of_row) {
  pdl_wait();
  pdl_trigger();
  const int mt = blockIdx.x;
  if (mt >= cu_tiles[HE]) return;
  const int m = threadIdx.x;
  if (m < tile_rows[mt]) pad_of_row[tile_row0[mt] + m] = mt * 128 + m;
}

// Sum of one key's rows (cnt ids at tok_rows[begin..]) into yrow, one warp.
// srt: this warp's 32-entry shared scratch.  U: row loads issued together.  The warp sums
// the 8-column groups part, part + parts, ... (lane-strided): parts > 1 lets several warps
// share one key's row when there are few keys.
template <int U = 8>
__device__ __forceinline__ void combine_key(const __nv_bfloat16* __restrict__ P, const int32_t* __restrict__ pad_of_row,
                                            int dh, const int32_t* __restrict__ tok_rows, int64_t begin, int cnt,
                                            int64_t R, int64_t P_rows, __nv_bfloat16* yrow, int* srt, int part = 0,
                                            int parts = 1) {
  const int lane = threadIdx.x & 31;
  const int nvec = dh / 8;
  const int c_first = part * 32 + lane, c_step = 32 * parts;
  if (cnt <= 32) {
    // rank sort of <= 32 row ids (ascending; ids are distinct)
    int r = lane < cnt ? tok_rows[begin + lane] : 0x7fffffff;
    if (r < 0 || r >= R) r = 0x7fffffff;            // invalid id: dropped
    int prow = r == 0x7fffffff ? 0x7fffffff : (pad_of_row ? pad_of_row[r] : r);
    if (prow < 0 || prow >= P_rows) {               // never read outside P
      prow = 0x7fffffff;
      r = 0x7fffffff;
    }
    int rank = 0;
    for (int j = 0; j < 32; ++j) {
      const int o = __shfl_sync(0xffffffffu, r, j);
      rank += (o < r) || (o == r && j < lane);
    }
    srt[rank] = prow;   // ascending sorted row <=> ascending padded row
    __syncwarp();
    int nvalid = 0;
    for (int j = 0; j < cnt; ++j) nvalid += srt[j] != 0x7fffffff;
    for (int c = c_first; c < nvec; c += c_step) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j0 = 0; j0 < nvalid; j0 += U) {
        // issue up to U independent row loads before accumulating (in ascending row order)
        uint4 u[U];
#pragma unroll
        for (int jj = 0; jj < U; ++jj)
          if (j0 + jj < nvalid) u[jj] = *reinterpret_cast<const uint4*>(P + (int64_t)srt[j0 + jj] * dh + c * 8);
#pragma unroll
        for (int jj = 0; jj < U; ++jj) {
          if (j0 + jj < nvalid) {
            const uint32_t w[4] = {u[jj].x, u[jj].y, u[jj].z, u[jj].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc[2 * i] = __fadd_rn(acc[2 * i], __uint_as_float(w[i] << 16));
              acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u));
            }
          }
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<uint32_t*>(&b);
      }
      *reinterpret_cast<uint4*>(yrow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncwarp();
  } else {
    // rare long lists: ascending selection, one row at a time
    for (int c = c_first; c < nvec; c += c_step) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      int last = -1;
      for (int it = 0; it < cnt; ++it) {
        int best = 0x7fffffff;
        for (int j = 0; j < cnt; ++j) {
          const int rr = tok_rows[begin + j];
          if (rr > last && rr < best && rr < R) best = rr;
        }
        if (best == 0x7fffffff) break;
        last = best;
        const int64_t prow = pad_of_row ? pad_of_row[best] : best;
        if (prow < 0 || prow >= P_rows) continue;
        const uint4 u = *reinterpret_cast<const uint4*>(P + prow * dh + c * 8);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = __fadd_rn(acc[2 * i], __uint_as_float(w[i] << 16));
          acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u));
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<uint32_t*>(&b);
      }
      *reinterpret_cast<uint4*>(yrow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ P, const int32_t* __restrict__ pad_of_row, int dh,
                               int S, int H,
                               const int32_t* __restrict__ tok_rows, const int32_t* __restrict__ tok_offsets,
                               int k_fixed, int64_t R, int64_t P_rows, __nv_bfloat16* __restrict__ y, int64_t sy_s,
                               int64_t sy_h, int parts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int srt[COMBINE_WARPS][32];
  const int warp = threadIdx.x >> 5;
  const int64_t w = (int64_t)blockIdx.x * COMBINE_WARPS + warp;
  const int64_t key = w / parts;                                      // key = h * S + s
  const int part = (int)(w % parts);
  if (key >= (int64_t)H * S) return;
  const int h = (int)(key / S), s = (int)(key % S);
  int64_t begin;
  int cnt;
  if (tok_offsets) {
    begin = tok_offsets[key];
    cnt = tok_offsets[key + 1] - (int)begin;
  } else {
    begin = key * k_fixed;
    cnt = k_fixed;
  }
  combine_key(P, pad_of_row, dh, tok_rows, begin, cnt, R, P_rows, y + (int64_t)s * sy_s + (int64_t)h * sy_h,
              srt[warp], part, parts);
}

// Expert-parallel receiver: key = received record slot src * cap + slot.  The record's sum
// goes into the source rank's return area, row (source's send position of the record) =
// meta offset + slot, over NVLink; slots past the source's count are skipped.  The last CTA
// to finish raises the return flag of this rank in every peer (system-scope release after
// every CTA's stores).
// Work item w -> source (w + me) % n, slot w / n: consecutive warps write to different
// ranks, so all links carry the returns at once (no rank is the target of everyone).
// Warps walk the items grid-stride.
// bulk != 0: each sum is built in one of two shared-memory buffers of the warp and sent
// with one bulk copy; a buffer is rewritten once its previous copy has been read out
// (wait_group.read), so a warp keeps a copy in flight while it sums the next record, and
// waits for completion once, before the flag.  bulk == 0: stored from registers.
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    combine_return_kernel(const __nv_bfloat16* __restrict__ P, const int32_t* __restrict__ pad_of_row, int dh,
                          const int32_t* __restrict__ tok_rows, int k_fixed, int64_t R, int64_t P_rows,
                          const EpReturn r, int bulk) {
  __shared__ int srt[WARPS][32];
  extern __shared__ __align__(128) uint8_t stage_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t slots = (int64_t)r.n * r.cap;
  const int64_t* meta = reinterpret_cast<const int64_t*>(r.local + r.layout.off_meta);
  int issued = 0;
  for (int64_t w = (int64_t)blockIdx.x * WARPS + warp; w < slots; w += (int64_t)gridDim.x * WARPS) {
    if (ld_volatile_i32(r.status) != 0) break;
    const int src = (int)((w + r.me) % r.n);
    const int64_t slot = w / r.n;
    const int64_t key = (int64_t)src * r.cap + slot;
    const int64_t cnt = meta[2 * src], off = meta[2 * src + 1];
    if (!(slot < cnt && cnt <= r.cap && off >= 0 && off + cnt <= slots)) continue;
    __nv_bfloat16* yrow =
        r.stage ? reinterpret_cast<__nv_bfloat16*>(r.local + r.layout.off_stage) + key * dh   // copied by the push
                : reinterpret_cast<__nv_bfloat16*>(r.peers.base[src] + r.layout.off_back) + (off + slot) * dh;
    if (bulk) {
      __nv_bfloat16* srow = reinterpret_cast<__nv_bfloat16*>(stage_raw) + ((size_t)warp * 2 + (issued & 1)) * dh;
      if (issued >= 2) {
        if (lane == 0) bulk_wait_read_1();      // the copy that last used this buffer has read it
        __syncwarp();
      }
      combine_key<4>(P, pad_of_row, dh, tok_rows, key * k_fixed, k_fixed, R, P_rows, srow, srt[warp]);
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        bulk_store(yrow, smem_u32(srow), (uint32_t)dh * 2);
        bulk_commit();
      }
      ++issued;
    } else {
      combine_key<4>(P, pad_of_row, dh, tok_rows, key * k_fixed, k_fixed, R, P_rows, yrow, srt[warp]);
    }
  }
  if (bulk && lane == 0 && issued > 0) {
    bulk_wait_all();                            // written at the destinations before the flag release
    fence_proxy_async_global();
  }
  if (r.stage) return;                          // the push raises the flags after its copies
  if (ep_last_cta(reinterpret_cast<int*>(r.local + r.layout.off_done) + 1) && threadIdx.x == 0) {
    for (int d = 0; d < r.n; ++d)
      red_release_sys_add(reinterpret_cast<int*>(r.peers.base[d] + r.layout.off_flags) + 32 + r.me, 1);
  }
}

// One warp per (s, h) row, 16-B stores.
__global__ void zero_rows_kernel(__nv_bfloat16* __restrict__ y, int S, int H, int dh, int64_t sy_s, int64_t sy_h) {
  pdl_wait();
  pdl_trigger();
  const int64_t key = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (key >= (int64_t)S * H) return;
  const int64_t s = key / H, h = key % H;
  uint4* row = reinterpret_cast<uint4*>(y + s * sy_s + h * sy_h);
  for (int c = threadIdx.x & 31; c < dh / 8; c += 32) row[c] = make_uint4(0u, 0u, 0u, 0u);
}

cudaError_t launch_zero_rows(__nv_bfloat16* y, int S, int H, int dh, int64_t sy_s, int64_t sy_h, cudaStream_t st) {
  const int64_t rows = (int64_t)S * H;
  if (rows == 0) return cudaSuccess;
  MHMOE_LAUNCH_PDL(zero_rows_kernel, (unsigned)((rows + 7) / 8), 256, 0, st, y, S, H, dh, sy_s, sy_h);
  return cudaGetLastError();
}

cudaError_t launch_pad_rows(const int* cu_tiles, int HE, int64_t max_mtiles, const int* tile_row0,
                            const int* tile_rows, int32_t* pad_of_row, cudaStream_t st) {
  MHMOE_LAUNCH_PDL(pad_rows_kernel, (unsigned)max_mtiles, 128, 0, st, cu_tiles, HE, tile_row0, tile_rows, pad_of_row);
  return cudaGetLastError();
}

cudaError_t launch_combine(const __nv_bfloat16* P, const int32_t* pad_of_row, int dh, int S, int H,
                           const int32_t* tok_rows, const int32_t* tok_offsets, int k_fixed, int64_t R,
                           int64_t P_rows, __nv_bfloat16* y, int64_t sy_s, int64_t sy_h, cudaStream_t st) {
  const int64_t keys = (int64_t)H * S;
  // few keys (small batches): several warps per key, each a share of the row's columns, so
  // that the launch still has ~16 warps per SM
  const int64_t want = 16 * (int64_t)num_sms();
  const int parts = (int)std::max<int64_t>(1, std::min<int64_t>((want + keys - 1) / std::max<int64_t>(keys, 1),
                                                                 (dh / 8 + 31) / 32));
  const int64_t warps = keys * parts;
  MHMOE_LAUNCH_PDL(combine_kernel, (unsigned)((warps + COMBINE_WARPS - 1) / COMBINE_WARPS), COMBINE_WARPS * 32, 0, st,
                   P, pad_of_row, dh, S, H, tok_rows, tok_offsets, k_fixed, R, P_rows, y, sy_s, sy_h, parts);
  return cudaGetLastError();
}

cudaError_t launch_combine_return(const __nv_bfloat16* P, const int32_t* pad_of_row, int dh,
                                  const int32_t* tok_rows, int k_fixed, int64_t R, int64_t P_rows, const EpReturn& r,
                                  cudaStream_t st) {
  const int64_t keys = (int64_t)r.n * r.cap;
  // bulk copies when MHMOE_EP_BULK=1, for rows of at most 8 KB (two 8 KB buffers per warp);
  // measured slower than stores from registers at 2 GPUs (the default)
  const char* env = std::getenv("MHMOE_EP_BULK");
  const int bulk = (env && env[0] == '1') && dh * 2 <= 8192 ? 1 : 0;
  const size_t smem = bulk ? (size_t)COMBINE_WARPS * 2 * dh * 2 : 0;
  if (bulk) {
    static PerDeviceOnce once;
    const cudaError_t e = once.run([](int) {
      return cudaFuncSetAttribute(combine_return_kernel<COMBINE_WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  COMBINE_WARPS * 2 * 8192);
    });
    if (e != cudaSuccess) return e;
  }
  // warps walk the records grid-stride: a few CTAs per SM keep copies in flight on every link
  const int64_t want = std::max<int64_t>(1, (keys + COMBINE_WARPS - 1) / COMBINE_WARPS);
  const int64_t blocks = std::min<int64_t>(want, (int64_t)(bulk ? 3 : 16) * num_sms());
  combine_return_kernel<COMBINE_WARPS><<<(unsigned)blocks, COMBINE_WARPS * 32, smem, st>>>(
      P, pad_of_row, dh, tok_rows, k_fixed, R, P_rows, r, bulk);
  return cudaGetLastError();
}

}  // namespace mhmoe
