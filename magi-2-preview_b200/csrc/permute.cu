// Token permutation for the MoE hot path: stable counting sort by expert, CSR
// offsets, 128-row tile tables, and the inverse (token -> rows) map.
//
// Replaces flash_mh_moe_global_sort (inference/flash_mh_moe/route.py:209-253) and the
// tile-count prep of mh_moe_fwd_func (inference/flash_mh_moe/triton/mh_moe_fwd.py:275-282).
//
// Stable sort = argsort(stable=True) over the flat (h, s, k) order:
//   1. chunk histograms   hist[c][g]  (one CTA per chunk, shared-memory counters)
//   2. column scan        hist[c][g] <- sum_{c' < c} hist[c'][g];  total[g]
//   3. key scan           expert_offsets = exclusive scan of total; tile tables
//   4. ordered scatter    one warp per chunk walks its entries in order; lanes that
//                         share a key get consecutive slots via __match_any_sync, so
//                         equal keys keep their flat order (stability).
// Up to 8192 entries and 256 keys the same result comes from one single-CTA kernel
// (sort_small_kernel).
#include "kernels.cuh"

namespace mhmoe {

__global__ void sort_hist_kernel(const int64_t* __restrict__ idx, int64_t R, int SK, int E, int HE, int chunk,
                                 int* __restrict__ hist, int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sh[];
  for (int g = threadIdx.x; g < HE; g += blockDim.x) sh[g] = 0;
  __syncthreads();
  const int64_t f0 = (int64_t)blockIdx.x * chunk;
  const int64_t f1 = min(f0 + chunk, R);
  for (int64_t f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
    const int64_t e = idx[f];
    if (e < 0) continue;              // negative id: "no expert" slot, skipped
    if (e >= E) {                     // out-of-range expert id: record, never index with it
      record_error(status, MHMOE_ERR_ARGS);
      continue;
    }
    const int h = (int)(f / SK);
    atomicAdd(&sh[h * E + (int)e], 1);
  }
  __syncthreads();
  int* row = hist + (size_t)blockIdx.x * HE;
  for (int g = threadIdx.x; g < HE; g += blockDim.x) row[g] = sh[g];
}

// One warp per key: exclusive prefix over the chunk histograms, 32 chunks per step; the
// loads of 16 steps are issued together so their latencies overlap.
__global__ void sort_colscan_kernel(int* __restrict__ hist, int nchunks, int HE, int* __restrict__ total) {
  pdl_wait();
  pdl_trigger();
  constexpr int U = 16;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g >= HE) return;
  int run = 0;
  for (int c0 = 0; c0 < nchunks; c0 += 32 * U) {
    int v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + 32 * u + lane;
      v[u] = c < nchunks ? hist[(size_t)c * HE + g] : 0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + 32 * u + lane;
      int incl = v[u];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      if (c < nchunks) hist[(size_t)c * HE + g] = run + incl - v[u];
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (lane == 0) total[g] = run;
}

// Single CTA: expert_offsets / tile tables from per-expert counts (counts != nullptr)
// or from given expert_offsets (counts == nullptr).
__global__ void tile_tables_kernel(const int* __restrict__ counts, const int64_t* __restrict__ offsets_in,
                                   int HE, int64_t* __restrict__ offsets_out, int* __restrict__ cu_tiles,
                                   int* __restrict__ tile_expert, int* __restrict__ tile_row0,
                                   int* __restrict__ tile_rows, int64_t max_mtiles, int* __restrict__ status,
                                   int align) {
  pdl_wait();
  pdl_trigger();
  __shared__ int64_t s_carry_rows;
  __shared__ int s_carry_tiles;
  __shared__ int64_t s_rows[1024];
  __shared__ int s_tiles[1024];
  if (threadIdx.x == 0) {
    s_carry_rows = 0;
    s_carry_tiles = 0;
  }
  __syncthreads();
  for (int base = 0; base < HE; base += 1024) {
    const int g = base + threadIdx.x;
    int64_t cnt = 0;
    if (g < HE) cnt = counts ? (int64_t)counts[g] : (offsets_in[g + 1] - offsets_in[g]);
    if (cnt < 0) {                    // non-monotonic offsets from a caller
      record_error(status, MHMOE_ERR_ARGS);
      cnt = 0;
    }
    const int nt = (int)(((cnt + 127) / 128 + align - 1) / align * align);
    s_rows[threadIdx.x] = cnt;
    s_tiles[threadIdx.x] = nt;
    __syncthreads();
    // Hillis-Steele inclusive scan over 1024 entries (two arrays)
    for (int off = 1; off < 1024; off <<= 1) {
      int64_t vr = 0;
      int vt = 0;
      if (threadIdx.x >= off) {
        vr = s_rows[threadIdx.x - off];
        vt = s_tiles[threadIdx.x - off];
      }
      __syncthreads();
      s_rows[threadIdx.x] += vr;
      s_tiles[threadIdx.x] += vt;
      __syncthreads();
    }
    const int64_t row_excl = s_carry_rows + s_rows[threadIdx.x] - cnt;
    const int tile_excl = s_carry_tiles + s_tiles[threadIdx.x] - nt;
    if (g < HE) {
      const int64_t row0 = counts ? row_excl : offsets_in[g];
      if (offsets_out) offsets_out[g] = row0;
      cu_tiles[g] = tile_excl;
      for (int j = 0; j < nt; ++j) {
        if (tile_excl + j >= max_mtiles) {   // more rows than the caller sized for
          record_error(status, MHMOE_ERR_ARGS);
          break;
        }
        tile_expert[tile_excl + j] = g;
        tile_row0[tile_excl + j] = (int)(row0 + 128 * j);
        const int64_t left = cnt - 128 * (int64_t)j;           // <= 0 on alignment padding tiles
        tile_rows[tile_excl + j] = (int)(left < 0 ? 0 : left < 128 ? left : 128);
      }
    }
    __syncthreads();
    if (threadIdx.x == 1023) {
      s_carry_rows += s_rows[1023];
      s_carry_tiles += s_tiles[1023];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (offsets_out) offsets_out[HE] = counts ? s_carry_rows : offsets_in[HE];
    cu_tiles[HE] = (int)((int64_t)s_carry_tiles < max_mtiles ? (int64_t)s_carry_tiles : max_mtiles);
  }
}

// One warp per chunk; entries of the chunk are visited in flat order, 32 at a time, the
// ids and probs of 8 steps loaded together so their latencies overlap.
__global__ void sort_scatter_kernel(const int64_t* __restrict__ idx, const float* __restrict__ probs, int64_t R,
                                    int S, int K, int E, int HE, int chunk, const int* __restrict__ hist,
                                    const int64_t* __restrict__ offsets, int32_t* __restrict__ gather_ids,
                                    float* __restrict__ probs_sorted, int32_t* __restrict__ row_of_flat) {
  pdl_wait();
  pdl_trigger();
  // Entries with a negative ("no expert") or out-of-range id get no slot; their
  // row_of_flat entry is -1.
  extern __shared__ int cursor[];
  const int lane = threadIdx.x;
  const int* row = hist + (size_t)blockIdx.x * HE;
  for (int g = lane; g < HE; g += 32) cursor[g] = (int)offsets[g] + row[g];
  __syncwarp();
  constexpr int U = 8;
  const int SK = S * K;
  const int64_t f0 = (int64_t)blockIdx.x * chunk;
  const int64_t f1 = min(f0 + chunk, R);
  for (int64_t fb0 = f0; fb0 < f1; fb0 += 32 * U) {
    int64_t ev[U];
    float pv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t f = fb0 + 32 * u + lane;
      ev[u] = f < f1 ? idx[f] : -1;
      pv[u] = f < f1 ? probs[f] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t f = fb0 + 32 * u + lane;
      int g = -1 - lane;   // distinct sentinel per invalid lane
      bool ok = false;
      if (f < f1) {
        const int64_t e = ev[u];
        ok = e >= 0 && e < E;
        if (ok) g = (int)(f / SK) * E + (int)e;
      }
      const bool valid_key = ok;
      const unsigned peers = __match_any_sync(0xffffffffu, g);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      int base = 0;
      if (valid_key) base = cursor[g];
      __syncwarp();
      if (valid_key && rank == 0) cursor[g] = base + __popc(peers);
      __syncwarp();
      if (valid_key) {
        const int pos = base + rank;
        gather_ids[pos] = (int32_t)((f / K) % S);
        probs_sorted[pos] = pv[u];
        if (row_of_flat) row_of_flat[f] = pos;
      } else if (f < f1 && row_of_flat) {
        row_of_flat[f] = -1;
      }
    }
  }
}

// Small problems (R <= SORT_SMALL_MAX entries, H*E <= SORT_SMALL_MAX_KEYS): the same
// stable counting sort in one CTA of 1024 threads — warp w owns a contiguous chunk of the
// flat entries; per-warp key histograms in shared memory, a column scan over the 32 warps
// and a key scan give every (warp, key) its first slot; each warp then walks its chunk in
// order and lanes sharing a key take consecutive slots (__match_any_sync), so equal keys
// keep their flat order.  Keys and probs are staged in shared memory.  One launch instead
// of four, whose latency dominates at small R.
constexpr int SORT_SMALL_MAX = 8192;
constexpr int SORT_SMALL_MAX_KEYS = 256;
constexpr int SORT_SMALL_SMEM = (32 * SORT_SMALL_MAX_KEYS + 2 * SORT_SMALL_MAX) * 4;   // 96 KB

__global__ void __launch_bounds__(1024, 1)
    sort_small_kernel(const int64_t* __restrict__ idx, const float* __restrict__ probs, int R, int S, int K, int E,
                      int HE, int64_t* __restrict__ expert_offsets, int32_t* __restrict__ gather_ids,
                      float* __restrict__ probs_sorted, int32_t* __restrict__ row_of_flat, int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sort_small_smem[];
  int* hist = sort_small_smem;                                   // [32][HE]: count, then first slot
  int* key = hist + 32 * SORT_SMALL_MAX_KEYS;                   // [R]
  float* prob = reinterpret_cast<float*>(key + SORT_SMALL_MAX);  // [R]
  __shared__ int tot[1024];
  __shared__ int wsum[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * HE; i += 1024) hist[i] = 0;
  __syncthreads();
  const int SK = S * K;
  const int chunk = (R + 31) / 32;
  const int f0 = warp * chunk, f1 = min(f0 + chunk, R);
  int* my = hist + warp * HE;
  for (int f = f0 + lane; f < f1; f += 32) {
    const int64_t e = idx[f];
    int g = -1;
    if (e >= E) record_error(status, MHMOE_ERR_ARGS);
    else if (e >= 0) g = (f / SK) * E + (int)e;
    key[f] = g;
    prob[f] = probs[f];
    if (g >= 0) atomicAdd(&my[g], 1);
  }
  __syncthreads();
  // column scan over warps: hist[w][g] <- entries of key g in warps before w
  int total = 0;
  if (tid < HE) {
    for (int w = 0; w < 32; ++w) {
      const int c = hist[w * HE + tid];
      hist[w * HE + tid] = total;
      total += c;
    }
  }
  // exclusive scan of the key totals (tid < 1024 covers HE <= 256)
  const int v = total;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = wsum[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    wsum[lane] = wi - w;
  }
  __syncthreads();
  const int excl = wsum[warp] + incl - v;
  tot[tid] = excl;
  if (tid < HE) expert_offsets[tid] = excl;
  if (tid == HE - 1) expert_offsets[HE] = excl + v;
  __syncthreads();
  for (int i = tid; i < 32 * HE; i += 1024) hist[i] += tot[i % HE];
  __syncthreads();
  // ordered scatter, each warp over its own chunk
  for (int fb = f0; fb < f1; fb += 32) {
    const int f = fb + lane;
    const int g = f < f1 ? key[f] : -1;
    const bool valid = g >= 0;
    const unsigned peers = __match_any_sync(0xffffffffu, valid ? g : -1 - lane);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    int base = 0;
    if (valid) base = my[g];
    __syncwarp();
    if (valid && rank == 0) my[g] = base + __popc(peers);
    __syncwarp();
    if (valid) {
      const int pos = base + rank;
      gather_ids[pos] = (int32_t)((f / K) % S);
      probs_sorted[pos] = prob[f];
      if (row_of_flat) row_of_flat[f] = pos;
    } else if (f < f1 && row_of_flat) {
      row_of_flat[f] = -1;
    }
  }
}

// ───────────── token -> rows map for arbitrary (gather_ids, expert_offsets) ─────────────

// counts[h*S + s] += 1 for every row; one CTA per m-tile of the tile tables.
__global__ void tok_count_kernel(const int32_t* __restrict__ gather_ids, const int* __restrict__ cu_tiles,
                                 int HE, int E, int S, const int* __restrict__ tile_expert,
                                 const int* __restrict__ tile_row0, const int* __restrict__ tile_rows,
                                 int* __restrict__ tok_count, int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int mt = blockIdx.x;
  if (mt >= cu_tiles[HE]) return;
  const int m = threadIdx.x;
  if (m >= tile_rows[mt]) return;
  const int h = tile_expert[mt] / E;
  const int r = tile_row0[mt] + m;
  const int s = gather_ids[r];
  if (s < 0 || s >= S) {
    record_error(status, MHMOE_ERR_ARGS);
    return;
  }
  atomicAdd(&tok_count[h * S + s], 1);
}

// Exclusive scan, pass 1: per-block scan of 4096 entries, block sums out.
__global__ void scan_block_kernel(const int* __restrict__ in, int n, int* __restrict__ out,
                                  int* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sh[1024];
  const int base = blockIdx.x * 4096 + threadIdx.x * 4;
  int v[4], s = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = (base + i < n) ? in[base + i] : 0;
    s += v[i];
  }
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int t = threadIdx.x >= off ? sh[threadIdx.x - off] : 0;
    __syncthreads();
    sh[threadIdx.x] += t;
    __syncthreads();
  }
  int run = sh[threadIdx.x] - s;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (base + i < n) out[base + i] = run;
    run += v[i];
  }
  if (threadIdx.x == 1023) block_sums[blockIdx.x] = sh[1023];
}

// Pass 2: exclusive scan of the block sums in place (single CTA, serial carry) and
// the grand total into out_total.
__global__ void scan_sums_kernel(int* __restrict__ block_sums, int nblocks, int* __restrict__ out_total) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sh[1024];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nblocks; base += 1024) {
    const int i = base + threadIdx.x;
    const int v = i < nblocks ? block_sums[i] : 0;
    sh[threadIdx.x] = v;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
      const int t = threadIdx.x >= off ? sh[threadIdx.x - off] : 0;
      __syncthreads();
      sh[threadIdx.x] += t;
      __syncthreads();
    }
    if (i < nblocks) block_sums[i] = carry + sh[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == 1023) carry += sh[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out_total = carry;
}

// Pass 3: add block offsets.
__global__ void scan_add_kernel(int* __restrict__ out, int n, const int* __restrict__ block_sums) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] += block_sums[i / 4096];
}

__global__ void tok_fill_kernel(const int32_t* __restrict__ gather_ids, const int* __restrict__ cu_tiles, int HE,
                                int E, int S, const int* __restrict__ tile_expert,
                                const int* __restrict__ tile_row0, const int* __restrict__ tile_rows,
                                const int* __restrict__ tok_offsets, int* __restrict__ tok_cursor,
                                int32_t* __restrict__ tok_rows) {
  pdl_wait();
  pdl_trigger();
  const int mt = blockIdx.x;
  if (mt >= cu_tiles[HE]) return;
  const int m = threadIdx.x;
  if (m >= tile_rows[mt]) return;
  const int h = tile_expert[mt] / E;
  const int r = tile_row0[mt] + m;
  const int s = gather_ids[r];
  if (s < 0 || s >= S) return;      // recorded by tok_count_kernel
  const int t = h * S + s;
  const int pos = tok_offsets[t] + atomicAdd(&tok_cursor[t], 1);
  tok_rows[pos] = r;
}

// ───────────────────────────── host launchers ─────────────────────────────

// Chunk of flat entries per histogram row: 256 entries (8 warp steps in the scatter) up to
// 2048 chunks, larger chunks beyond that so the histogram stays <= 2048 x H*E ints.
// Entries per chunk: at most ~2048 chunks, and chunks x keys at most 2^21 histogram
// counters (the column scan reads each counter once per key-warp step; with thousands of
// keys, as in the production head split's 12 x 256, many small chunks made that scan the
// slowest step of the sort).
int sort_chunk_size(int64_t R, int64_t HE, int min_chunk) {
  int64_t c = std::max<int64_t>((R + 2047) / 2048, (R * std::max<int64_t>(HE, 1) + (1 << 21) - 1) >> 21);
  c = (c + 31) / 32 * 32;
  return (int)std::max<int64_t>(min_chunk, c);
}

cudaError_t launch_global_sort(const float* probs, const int64_t* idx, int H, int S, int K, int E, void* ws,
                               int32_t* gather_ids, float* probs_sorted, int64_t* expert_offsets,
                               int32_t* row_of_flat, int* status, cudaStream_t st, int min_chunk) {
  const int64_t R = (int64_t)H * S * K;
  const int HE = H * E;
  const int chunk = sort_chunk_size(R, HE, min_chunk);
  const int nchunks = (int)((R + chunk - 1) / chunk);
  const int64_t mt = mtiles_upper_bound(R, HE);
  int* hist = static_cast<int*>(ws);
  int* total = hist + (size_t)nchunks * HE;
  int* cu_tiles = total + HE;
  int* tile_expert = cu_tiles + HE + 1;
  int* tile_row0 = tile_expert + mt;
  int* tile_rows = tile_row0 + mt;
  if (R <= SORT_SMALL_MAX && HE <= SORT_SMALL_MAX_KEYS) {
    static PerDeviceOnce once;
    const cudaError_t attr = once.run([](int) {
      return cudaFuncSetAttribute(sort_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SORT_SMALL_SMEM);
    });
    if (attr != cudaSuccess) return attr;
    MHMOE_LAUNCH_PDL(sort_small_kernel, 1, 1024, SORT_SMALL_SMEM, st, idx, probs, (int)R, S, K, E, HE, expert_offsets,
                     gather_ids, probs_sorted, row_of_flat, status);
    return cudaGetLastError();
  }
  const size_t shb = (size_t)HE * sizeof(int);
  MHMOE_LAUNCH_PDL(sort_hist_kernel, nchunks, 256, shb, st, idx, R, S * K, E, HE, chunk, hist, status);
  MHMOE_LAUNCH_PDL(sort_colscan_kernel, (HE + 7) / 8, 256, 0, st, hist, nchunks, HE, total);
  MHMOE_LAUNCH_PDL(tile_tables_kernel, 1, 1024, 0, st, total, nullptr, HE, expert_offsets, cu_tiles, tile_expert,
                   tile_row0, tile_rows, mtiles_upper_bound(R, HE), status, 1);
  MHMOE_LAUNCH_PDL(sort_scatter_kernel, nchunks, 32, shb, st, idx, probs, R, S, K, E, HE, chunk, hist, expert_offsets,
                   gather_ids, probs_sorted, row_of_flat);
  return cudaGetLastError();
}

size_t global_sort_ws_bytes(int H, int S, int K, int E, int min_chunk) {
  const int64_t R = (int64_t)H * S * K;
  const int chunk = sort_chunk_size(R, (int64_t)H * E, min_chunk);
  const int64_t nchunks = (R + chunk - 1) / chunk;
  const int64_t mt = mtiles_upper_bound(R, (int64_t)H * E);
  return ((size_t)(nchunks + 2) * (size_t)(H * E) + 1 + 3 * (size_t)mt) * sizeof(int) + 256;
}

cudaError_t launch_tile_tables(const int64_t* expert_offsets, int HE, int64_t max_tiles, int* cu_tiles,
                               int* tile_expert, int* tile_row0, int* tile_rows, int* status, cudaStream_t st,
                               int align) {
  MHMOE_LAUNCH_PDL(tile_tables_kernel, 1, 1024, 0, st, nullptr, expert_offsets, HE, nullptr, cu_tiles, tile_expert,
                   tile_row0, tile_rows, max_tiles, status, align);
  return cudaGetLastError();
}

size_t token_rows_ws_bytes(int64_t T) {
  const int64_t nblk = (T + 4095) / 4096;
  return (size_t)(2 * T + nblk + 64) * sizeof(int);
}

cudaError_t launch_token_rows(const int32_t* gather_ids, int64_t max_mtiles, const int* cu_tiles, int HE, int E,
                              int S, int H, const int* tile_expert, const int* tile_row0, const int* tile_rows,
                              void* ws, int32_t* tok_offsets, int32_t* tok_rows, int* status, cudaStream_t st) {
  const int64_t T = (int64_t)H * S;
  int* cnt = static_cast<int*>(ws);
  int* cursor = cnt + T;
  int* bsums = cursor + T;
  const int nblk = (int)((T + 4095) / 4096);
  cudaMemsetAsync(cnt, 0, (size_t)(2 * T) * sizeof(int), st);
  MHMOE_LAUNCH_PDL(tok_count_kernel, (unsigned)max_mtiles, 128, 0, st, gather_ids, cu_tiles, HE, E, S, tile_expert,
                   tile_row0, tile_rows, cnt, status);
  MHMOE_LAUNCH_PDL(scan_block_kernel, nblk, 1024, 0, st, cnt, (int)T, tok_offsets, bsums);
  MHMOE_LAUNCH_PDL(scan_sums_kernel, 1, 1024, 0, st, bsums, nblk, tok_offsets + T);
  MHMOE_LAUNCH_PDL(scan_add_kernel, (unsigned)((T + 255) / 256), 256, 0, st, tok_offsets, (int)T, bsums);
  MHMOE_LAUNCH_PDL(tok_fill_kernel, (unsigned)max_mtiles, 128, 0, st, gather_ids, cu_tiles, HE, E, S, tile_expert,
                   tile_row0, tile_rows, tok_offsets, cursor, tok_rows);
  return cudaGetLastError();
}

}  // namespace mhmoe
