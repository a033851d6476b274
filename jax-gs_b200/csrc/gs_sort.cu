// Stage 2: duplication of each visible Gaussian into (tile << 13 | depth)
// keys, a stable device LSD radix sort, and the per-tile range search.
//
// Replaces get_tile_interactions (jax_gs/renderer/rasterizer.py:12-116) and the
// searchsorted of rasterizer.py:158-160 / renderer.py:57-61. The reference
// materialises all N*256 candidate slots and sorts them; here only the valid
// pairs are emitted (in Gaussian order, tiles ascending within a Gaussian, the
// order of its offset grid), so a stable sort on the same 32-bit key gives the
// reference's valid segment exactly.
//
// The radix sort is reduce-then-scan over a FIXED grid of kSortGrid CTAs: each
// CTA owns one contiguous slice, so no CTA ever waits on another (no spin
// loops) and launch shapes are independent of the data-dependent pair count,
// which the kernels read from device memory.
#include "gs_kernels.cuh"

namespace gs {

// Slice [begin, end) of CTA b for n keys.
__device__ __forceinline__ void sort_slice(int n, int b, int& begin, int& end) {
  int per = (n + kSortGrid - 1) / kSortGrid;
  per = (per + kSortTileKeys - 1) / kSortTileKeys * kSortTileKeys;
  long long bb = (long long)b * per;
  long long nn = n;
  begin = (int)(bb < nn ? bb : nn);
  end = (int)(bb + per < nn ? bb + per : nn);
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Exclusive scan over 256 threads (one value each). Returns the exclusive
// prefix; *total receives the sum. Uses s_tmp[8].
__device__ __forceinline__ int block_exclusive_scan_256(int v, int* s_tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_tmp[warp] = x;
  __syncthreads();
  int wpre = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    int t = s_tmp[w];
    if (w < warp) wpre += t;
    tot += t;
  }
  __syncthreads();
  *total = tot;
  return wpre + x - v;
}

// ---------------------------------------------------------------------------
// Exclusive scan of per-CTA pair counts (single CTA, 64-bit running sum).
__global__ void __launch_bounds__(1024)
k_scan_block_counts(const int* __restrict__ counts, int nb, int* __restrict__ offsets,
                    Scalars* __restrict__ sc, long long cap, int num_tiles,
                    GsExtras* __restrict__ ex) {
  __shared__ long long s_warp[32];
  __shared__ long long s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < nb; base += 1024) {
    int i = base + tid;
    long long v = (i < nb) ? counts[i] : 0;
    long long x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      long long w = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    long long wpre = (warp > 0) ? s_warp[warp - 1] : 0;
    long long excl = s_carry + wpre + x - v;
    if (i < nb) offsets[i] = (int)excl;
    long long blk = s_warp[31];
    __syncthreads();
    if (tid == 0) s_carry += blk;
    __syncthreads();
  }
  if (tid == 0) {
    long long total = s_carry;
    long long emit = total < cap ? total : cap;
    sc->n_total = (int)total;
    sc->n_emit = (int)emit;
    if (ex) {
      ex->n_interactions = (int)total;
      ex->mean_interactions_per_tile = (float)(int)total / (float)(num_tiles > 1 ? num_tiles : 1);
      ex->capacity_overflow = (int)(total - emit);
      ex->num_tiles = num_tiles;
    }
  }
}

// ---------------------------------------------------------------------------
// Key emission: one CTA per 256 Gaussians; the CTA's pairs are spread over
// its threads so stores are contiguous regardless of per-Gaussian counts.
__global__ void __launch_bounds__(256)
k_emit_keys(const int2* __restrict__ bins, const int* __restrict__ block_offsets, int n,
            int tiles_x, const Scalars* __restrict__ sc, long long cap, int* __restrict__ keys,
            int* __restrict__ ids) {
  __shared__ int s_pre[257];
  __shared__ int2 s_bin[256];
  __shared__ int s_tmp[8];
  const int tid = threadIdx.x;
  const int i = blockIdx.x * 256 + tid;
  int2 b = (i < n) ? bins[i] : make_int2(0, 0);
  int cnt = (b.y & 31) * ((b.y >> 5) & 31);
  int total;
  int ex = block_exclusive_scan_256(cnt, s_tmp, &total);
  s_pre[tid] = ex;
  s_bin[tid] = b;
  if (tid == 0) s_pre[256] = total;
  __syncthreads();
  const int base = block_offsets[blockIdx.x];
  for (int e = tid; e < total; e += 256) {
    int lo = 0, hi = 255;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (s_pre[mid] <= e) lo = mid; else hi = mid - 1;
    }
    int2 bb = s_bin[lo];
    int j = e - s_pre[lo];
    int nx = bb.y & 31;
    int dq = (bb.y >> 10) & 0x1FFF;
    int oy = j / nx, ox = j - oy * nx;
    int tx0 = bb.x & 0xFFFF, ty0 = bb.x >> 16;
    int tile = (ty0 + oy) * tiles_x + (tx0 + ox);
    long long pos = (long long)base + e;
    if (pos < cap) {
      keys[pos] = (tile << kDepthBits) | dq;
      ids[pos] = blockIdx.x * 256 + lo;
    }
  }
}

// ---------------------------------------------------------------------------
// Radix sort, pass part 1: digit histogram of each CTA slice, digit-major.
__global__ void __launch_bounds__(kSortThreads)
k_sort_upsweep(const int* __restrict__ keys, const Scalars* __restrict__ sc, int shift, int mask,
               int* __restrict__ hist, int* __restrict__ digit_total) {
  __shared__ int s_h[8][kRadix];
  const int tid = threadIdx.x, warp = tid >> 5;
#pragma unroll
  for (int w = 0; w < 8; ++w) s_h[w][tid] = 0;
  __syncthreads();
  int begin, end;
  sort_slice(sc->n_emit, blockIdx.x, begin, end);
  for (int i = begin + tid; i < end; i += kSortThreads) {
    unsigned d = ((unsigned)__ldg(keys + i) >> shift) & (unsigned)mask;
    atomicAdd(&s_h[warp][d], 1);
  }
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) s += s_h[w][tid];
  hist[tid * kSortGrid + blockIdx.x] = s;
  if (s) atomicAdd(digit_total + tid, s);
}

// Pass part 2: exclusive scan of the kRadix x kSortGrid histogram (in place),
// digit-major, so entry (d, b) becomes the first output slot of digit d in CTA
// slice b. One warp per digit: its base is the sum of the smaller digits'
// totals (accumulated by the upsweep), then the warp scans its contiguous row
// over the CTA slices that hold keys.
constexpr int kScanWarps = 8;
__global__ void __launch_bounds__(32 * kScanWarps)
k_sort_scan(int* __restrict__ hist, const int* __restrict__ digit_total,
            const Scalars* __restrict__ sc) {
  const int lane = threadIdx.x & 31;
  const int d = blockIdx.x * kScanWarps + (threadIdx.x >> 5);
  int part = 0;
#pragma unroll
  for (int k = 0; k < kRadix / 32; ++k) {
    int dd = lane * (kRadix / 32) + k;
    if (dd < d) part += digit_total[dd];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  int carry = part;
  const int n = sc->n_emit;
  int per = (n + kSortGrid - 1) / kSortGrid;
  per = (per + kSortTileKeys - 1) / kSortTileKeys * kSortTileKeys;
  const int used = per > 0 ? min(kSortGrid, (n + per - 1) / per) : 0;
  int* row = hist + d * kSortGrid;
  for (int b0 = 0; b0 < used; b0 += 32) {
    const int b = b0 + lane;
    const int v = (b < used) ? row[b] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (b < used) row[b] = carry + x - v;
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
}

// Pass part 3: stable scatter. Each CTA walks its slice in tiles of
// kSortTileKeys keys; within a tile, warp w ranks keys [w*256, w*256+256)
// in 8 rounds of 32 with __match_any_sync, which keeps the original order of
// equal digits; the tile is staged in shared memory in digit order so the
// global stores form contiguous runs.
__global__ void __launch_bounds__(kSortThreads)
k_sort_downsweep(const int* __restrict__ keys_in, const int* __restrict__ ids_in,
                 int* __restrict__ keys_out, int* __restrict__ ids_out,
                 const Scalars* __restrict__ sc, int shift, int mask,
                 const int* __restrict__ offsets) {
  __shared__ int s_whist[8][kRadix];
  __shared__ int s_tile_start[kRadix];
  __shared__ int s_tile_count[kRadix];
  __shared__ int s_gbase[kRadix];
  __shared__ int s_keys[kSortTileKeys];
  __shared__ int s_ids[kSortTileKeys];
  __shared__ int s_tmp[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lt = lanemask_lt();
  int begin, end;
  sort_slice(sc->n_emit, blockIdx.x, begin, end);
  s_gbase[tid] = offsets[tid * kSortGrid + blockIdx.x];
  for (int t0 = begin; t0 < end; t0 += kSortTileKeys) {
#pragma unroll
    for (int k = 0; k < kRadix / 32; ++k) s_whist[warp][lane + 32 * k] = 0;
    __syncwarp();
    int key[kSortItems], id[kSortItems], rank[kSortItems];
    unsigned dig[kSortItems];
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      int idx = t0 + warp * 256 + r * 32 + lane;
      bool ok = idx < end;
      key[r] = ok ? keys_in[idx] : 0;
      id[r] = ok ? ids_in[idx] : 0;
      unsigned d = ok ? (((unsigned)key[r] >> shift) & (unsigned)mask) : (unsigned)kRadix;
      unsigned peers = __match_any_sync(0xffffffffu, d);
      int before = 0;
      if (ok) before = s_whist[warp][d];
      __syncwarp();
      if (ok && lane == __ffs(peers) - 1) s_whist[warp][d] = before + __popc(peers);
      __syncwarp();
      rank[r] = before + __popc(peers & lt);
      dig[r] = d;
    }
    __syncthreads();
    {
      int run = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        int c = s_whist[w][tid];
        s_whist[w][tid] = run;
        run += c;
      }
      s_tile_count[tid] = run;
      int tot;
      int ex = block_exclusive_scan_256(run, s_tmp, &tot);
      s_tile_start[tid] = ex;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      if (dig[r] < (unsigned)kRadix) {
        int pos = s_tile_start[dig[r]] + s_whist[warp][dig[r]] + rank[r];
        s_keys[pos] = key[r];
        s_ids[pos] = id[r];
      }
    }
    __syncthreads();
    const int tile_n = min(kSortTileKeys, end - t0);
    for (int i = tid; i < tile_n; i += kSortThreads) {
      int k = s_keys[i];
      unsigned d = ((unsigned)k >> shift) & (unsigned)mask;
      int out = s_gbase[d] + (i - s_tile_start[d]);
      keys_out[out] = k;
      ids_out[out] = s_ids[i];
    }
    __syncthreads();
    s_gbase[tid] += s_tile_count[tid];
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Tile ranges: ranges[t] = first index whose tile id >= t, for t in [0, T].
constexpr int kRangeGrid = 592;

__global__ void __launch_bounds__(256)
k_ranges_from_keys(const int* __restrict__ keys, const Scalars* __restrict__ sc, int T,
                   int* __restrict__ ranges) {
  const int n = sc->n_emit;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i <= n; i += (long long)gridDim.x * 256) {
    int cur = (i < n) ? (keys[i] >> kDepthBits) : T;
    int prev = (i == 0) ? -1 : (keys[i - 1] >> kDepthBits);
    if (cur > T) cur = T;
    for (int t = prev + 1; t <= cur; ++t) ranges[t] = (int)i;
  }
}

__global__ void __launch_bounds__(256)
k_ranges_from_ids(const int* __restrict__ tiles, long long ns, int T, int* __restrict__ ranges) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i <= ns; i += (long long)gridDim.x * 256) {
    long long cur = (i < ns) ? (long long)tiles[i] : (long long)T;
    long long prev = (i == 0) ? -1 : (long long)tiles[i - 1];
    long long lo = prev + 1 < 0 ? 0 : prev + 1;
    long long hi = cur > T ? T : cur;
    for (long long t = lo; t <= hi; ++t) ranges[t] = (int)i;
  }
}

__global__ void __launch_bounds__(256)
k_export(const int* __restrict__ keys, const int* __restrict__ ids, const Scalars* __restrict__ sc,
         long long cap, int T, int* __restrict__ out_tiles, int* __restrict__ out_ids,
         int* __restrict__ out_count) {
  const int n = sc->n_emit;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < cap; i += (long long)gridDim.x * 256) {
    bool ok = i < n;
    out_tiles[i] = ok ? (keys[i] >> kDepthBits) : T;
    out_ids[i] = ok ? ids[i] : 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && out_count) *out_count = sc->n_total;
}

// ---------------------------------------------------------------------------
void launch_scan_block_counts(const int* block_counts, int n_blocks, int* block_offsets,
                              Scalars* sc, int64_t capacity, int num_tiles, GsExtras* extras,
                              cudaStream_t st) {
  GS_TIMED("scan_block_counts", st);
  k_scan_block_counts<<<1, 1024, 0, st>>>(block_counts, n_blocks, block_offsets, sc, capacity,
                                          num_tiles, extras);
}

void launch_emit_keys(const int2* bins, const int* block_offsets, int n, int tiles_x,
                      const Scalars* sc, int64_t capacity, int* keys, int* ids, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("emit_keys", st);
  k_emit_keys<<<nb, 256, 0, st>>>(bins, block_offsets, n, tiles_x, sc, capacity, keys, ids);
}

int launch_radix_sort(int* keys0, int* ids0, int* keys1, int* ids1, int* hist, const Scalars* sc,
                      int total_bits, cudaStream_t st) {
  int cur = 0;
  int* kb[2] = {keys0, keys1};
  int* ib[2] = {ids0, ids1};
  // per-pass digit totals live after the kRadix x kSortGrid histogram
  int* totals = hist + kRadix * kSortGrid;
  cudaMemsetAsync(totals, 0, sizeof(int) * kRadix * kMaxSortPasses, st);
  int pass = 0;
  for (int shift = 0; shift < total_bits; shift += kRadixBits, ++pass) {
    int bits = total_bits - shift < kRadixBits ? total_bits - shift : kRadixBits;
    int mask = (1 << bits) - 1;
    int* dt = totals + kRadix * pass;
    {
      GS_TIMED("sort_upsweep", st);
      k_sort_upsweep<<<kSortGrid, kSortThreads, 0, st>>>(kb[cur], sc, shift, mask, hist, dt);
    }
    {
      GS_TIMED("sort_scan", st);
      k_sort_scan<<<kRadix / kScanWarps, 32 * kScanWarps, 0, st>>>(hist, dt, sc);
    }
    GS_TIMED("sort_downsweep", st);
    k_sort_downsweep<<<kSortGrid, kSortThreads, 0, st>>>(kb[cur], ib[cur], kb[cur ^ 1], ib[cur ^ 1], sc,
                                                         shift, mask, hist);
    cur ^= 1;
  }
  return cur;
}

void launch_tile_ranges_from_keys(const int* sorted_keys, const Scalars* sc, int num_tiles,
                                  int* ranges, cudaStream_t st) {
  GS_TIMED("tile_ranges", st);
  k_ranges_from_keys<<<kRangeGrid, 256, 0, st>>>(sorted_keys, sc, num_tiles, ranges);
}

void launch_tile_ranges_from_ids(const int* sorted_tile_ids, int64_t n_sorted, int num_tiles,
                                 int* ranges, cudaStream_t st) {
  GS_TIMED("tile_ranges_ids", st);
  k_ranges_from_ids<<<kRangeGrid, 256, 0, st>>>(sorted_tile_ids, n_sorted, num_tiles, ranges);
}

void launch_export_interactions(const int* keys, const int* ids, const Scalars* sc,
                                int64_t capacity, int num_tiles, int* out_tiles, int* out_ids,
                                int* out_count, cudaStream_t st) {
  GS_TIMED("export", st);
  k_export<<<kRangeGrid, 256, 0, st>>>(keys, ids, sc, capacity, num_tiles, out_tiles, out_ids,
                                       out_count);
}

}  // namespace gs
