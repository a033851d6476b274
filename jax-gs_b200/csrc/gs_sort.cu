// Stage 2: the (tile, depth)-sorted list of (Gaussian, tile) pairs and the
// per-tile range search.
//
// Replaces get_tile_interactions (jax_gs/renderer/rasterizer.py:12-116) and the
// searchsorted of rasterizer.py:158-160 / renderer.py:57-61. The reference
// materialises all N*256 candidate slots, keys them (tile << 13 | depth >> 18
// bits) and stable-sorts them, so its valid segment is ordered by tile, then
// by the 13-bit depth key, then by Gaussian index (each Gaussian has at most
// one pair per tile). Only the valid pairs are built here, by one of two
// paths that give the same order:
//
// Direct (n < kPresortMinN): the pairs are emitted in Gaussian order with the
// reference's key and stable-sorted on 13 + log2(T) bits. Each 8-bit pass is
// one launch: a CTA takes the next 2048-key tile from an atomic counter, ranks
// its keys by digit (stable), publishes its per-digit counts and obtains the
// counts of all earlier tiles by a decoupled look-back (single-pass prefix
// scan: Merrill & Garland 2016; its use for LSD radix sorting: Adinets &
// Merrill 2022, "Onesweep"). Tiles are claimed in order by running CTAs, so a
// look-back only waits on CTAs that are already resident; every wait is
// bounded and counted in Scalars::sort_timeouts if it gives up. Best for small
// inputs, where launches dominate.
//
// Pre-sort (n >= kPresortMinN): the Gaussians that have pairs are compacted
// and stable-sorted by their 13-bit depth key (N_v keys, two passes); their
// pairs are emitted in that order with the tile id alone as key and
// stable-sorted by tile (M keys, ceil(log2 T / 8) passes instead of
// ceil((13 + log2 T) / 8)). A stable sort by tile of a list already in
// (depth, index) order is the reference's order. Its passes are three
// launches with no inter-CTA waiting (large inputs make a look-back chain
// long): per 2048-key tile its digit counts ([digit][tile]); per digit a scan
// of its row; per tile a stable rank and the scatter to base + rank. The
// emission's output offsets come from the pair counts of the depth-sorted
// 256-Gaussian blocks, summed by the last depth pass.
//
// Both paths stage each sorted tile in shared memory in digit order so that
// the global stores form contiguous runs.
#include "gs_kernels.cuh"

namespace gs {

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

// Lanes of the warp holding the same value d < 2^nbits (nbits <= 9,
// warp-uniform): the AND over bits of the ballots that agree with d. A few
// ballots issue faster than one match.any on this GPU. Whole warp.
__device__ __forceinline__ unsigned same_value_lanes(unsigned d, int nbits) {
  unsigned m = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < 9; ++b) {
    if (b < nbits) {
      const bool bit = (d >> b) & 1u;
      const unsigned v = __ballot_sync(0xffffffffu, bit);
      m &= bit ? v : ~v;
    }
  }
  return m;
}

// 16-byte asynchronous copy global -> shared of src_bytes (0..16) bytes,
// the rest of the 16 zero-filled (nothing is read past src_bytes).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Totals of the per-256-Gaussian block counts [pairs | visible] (single CTA):
// n_total / n_emit from the pairs, and the exclusive scan of the visible
// counts (compaction offsets) with n_vis.
__global__ void __launch_bounds__(1024)
k_scan_block_counts(const int* __restrict__ counts, int nb, int* __restrict__ pair_offsets,
                    int* __restrict__ vis_offsets, Scalars* __restrict__ sc, long long cap,
                    int num_tiles, GsExtras* __restrict__ ex) {
  GS_PDL_ENTRY();
  __shared__ long long s_warp[2][32];
  __shared__ long long s_carry[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 2) s_carry[tid] = 0;
  __syncthreads();
  for (int base = 0; base < nb; base += 1024) {
    const int i = base + tid;
    long long v[2], x[2];
    v[0] = (i < nb) ? counts[i] : 0;       // pairs
    v[1] = (i < nb) ? counts[nb + i] : 0;  // visible Gaussians
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      x[a] = v[a];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, x[a], o);
        if (lane >= o) x[a] += y;
      }
      if (lane == 31) s_warp[a][warp] = x[a];
    }
    __syncthreads();
    if (warp < 2) {
      long long w = s_warp[warp][lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[warp][lane] = w;  // inclusive over warps
    }
    __syncthreads();
    if (i < nb) {
      const long long p = s_carry[0] + (warp > 0 ? s_warp[0][warp - 1] : 0) + x[0] - v[0];
      pair_offsets[i] = (int)(p < cap ? p : cap);  // emission writes only below cap
      vis_offsets[i] = (int)(s_carry[1] + (warp > 0 ? s_warp[1][warp - 1] : 0) + x[1] - v[1]);
    }
    const long long b0 = s_warp[0][31], b1 = s_warp[1][31];
    __syncthreads();
    if (tid == 0) {
      s_carry[0] += b0;
      s_carry[1] += b1;
    }
    __syncthreads();
  }
  if (tid == 0) {
    const long long total = s_carry[0];
    const long long emit = total < cap ? total : cap;
    sc->n_total = (int)total;
    sc->n_emit = (int)emit;
    sc->n_vis = (int)s_carry[1];
    if (ex) {
      ex->n_interactions = (int)total;
      ex->mean_interactions_per_tile = (float)(int)total / (float)(num_tiles > 1 ? num_tiles : 1);
      ex->capacity_overflow = (int)(total - emit);
      ex->num_tiles = num_tiles;
    }
  }
}

// ---------------------------------------------------------------------------
// The Gaussians with pairs, in index order, keyed by their 13-bit depth key.
// Also clears the per-block pair counts that the last depth pass sums.
__global__ void __launch_bounds__(256)
k_compact_visible(const int2* __restrict__ bins, int n, const int* __restrict__ vis_offsets,
                  int* __restrict__ dkeys, int* __restrict__ dids, int* __restrict__ sorted_counts) {
  GS_PDL_ENTRY();
  __shared__ int s_tmp[8];
  const int tid = threadIdx.x;
  const int i = blockIdx.x * 256 + tid;
  if (i < (n + 255) / 256) sorted_counts[i] = 0;  // grid has ceil(n/256) CTAs x 256 threads
  const int2 b = (i < n) ? bins[i] : make_int2(0, 0);
  const bool vis = (b.y & 31) * ((b.y >> 5) & 31) > 0;
  int tot;
  const int ex = block_exclusive_scan_256(vis ? 1 : 0, s_tmp, &tot);
  if (vis) {
    const int pos = vis_offsets[blockIdx.x] + ex;
    dkeys[pos] = (b.y >> 10) & 0x1FFF;
    dids[pos] = i;
  }
}

// Exclusive scan of the pair counts of the depth-sorted 256-Gaussian blocks
// (single CTA): the emission's output offsets.
__global__ void __launch_bounds__(1024)
k_scan_sorted_counts(const int* __restrict__ counts, const Scalars* __restrict__ sc,
                     int* __restrict__ offsets) {
  GS_PDL_ENTRY();
  __shared__ int s_warp[32];
  __shared__ int s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (sc->n_vis + 255) / 256;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < nb; base += 1024) {
    const int i = base + tid;
    const int v = (i < nb) ? counts[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[lane] = w;
    }
    __syncthreads();
    const int wpre = (warp > 0) ? s_warp[warp - 1] : 0;
    if (i < nb) offsets[i] = s_carry + wpre + x - v;
    const int blk = s_warp[31];
    __syncthreads();
    if (tid == 0) s_carry += blk;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Pair emission in depth order, one CTA per block of 256 depth-sorted
// Gaussians and one warp per 32 of them: the warp's pairs are a contiguous
// run of the output (block offset + the earlier warps' pairs), which its
// lanes write 32 consecutive pairs at a time; lane l finds the Gaussian of
// pair e by a 5-step search of the warp's 32 exclusive pair offsets. Within
// a Gaussian the tiles ascend (the order of its offset grid).
__global__ void __launch_bounds__(256)
k_emit_sorted(const int2* __restrict__ bins, const int* __restrict__ order,
                    const Scalars* __restrict__ sc, const int* __restrict__ offsets, int tiles_x,
                    int* __restrict__ keys, int* __restrict__ ids) {
  GS_PDL_ENTRY();
  __shared__ int s_ex[8][33];
  __shared__ int2 s_bin[8][32];
  __shared__ int s_gid[8][32];
  __shared__ int s_wtot[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_vis = sc->n_vis, n_emit = sc->n_emit;
  const int b = blockIdx.x;
  if (b * 256 >= n_vis) return;  // grid covers the capacity; uniform per CTA
  const int i = b * 256 + tid;
  const int g = (i < n_vis) ? order[i] : 0;
  const int2 bb = (i < n_vis) ? bins[g] : make_int2(0, 0);
  const int cnt = (bb.y & 31) * ((bb.y >> 5) & 31);
  int x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  const int wtot = __shfl_sync(0xffffffffu, x, 31);
  s_ex[warp][lane] = x - cnt;
  s_bin[warp][lane] = bb;
  s_gid[warp][lane] = g;
  if (lane == 0) {
    s_ex[warp][32] = wtot;
    s_wtot[warp] = wtot;
  }
  __syncthreads();
  int base = offsets[b];
  for (int w = 0; w < warp; ++w) base += s_wtot[w];
  for (int e0 = 0; e0 < wtot; e0 += 32) {  // warp-uniform trip count
    const int e = e0 + lane;
    if (e < wtot && base + e < n_emit) {
      int lo = 0;  // largest lo with s_ex[lo] <= e: a Gaussian with pairs
#pragma unroll
      for (int step = 16; step > 0; step >>= 1)
        if (s_ex[warp][lo + step] <= e) lo += step;
      const int2 q = s_bin[warp][lo];
      const int j = e - s_ex[warp][lo];
      const int nx = q.y & 31;
      // j / nx for j < 256, nx <= 16: (j + 1/2) / nx is at least 1/32
      // away from an integer, far more than the float rounding
      const int oy = (int)__fmul_rn((float)j + 0.5f, __frcp_rn((float)nx)), ox = j - oy * nx;
      keys[base + e] = ((q.x >> 16) + oy) * tiles_x + ((q.x & 0xFFFF) + ox);
      ids[base + e] = s_gid[warp][lo];
    }
  }
}

// ---------------------------------------------------------------------------
// Radix pass, part 1: digit counts of every 2048-key tile, digit-major
// (counts[d * max_tiles + t]), and their totals per digit (atomics). Keys
// come in as int4 loads, one shared-memory increment per key into the
// warp's own histogram, and the next tile's loads are issued before the
// current tile is counted.
__device__ __forceinline__ void load_tile_keys(const int* __restrict__ keys, int n, int t, int tid, int4 v[2]) {
  const int t0 = t * kSortTileKeys;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int li = 4 * (r * kSortThreads + tid);  // key index in the tile
    if (t0 + li + 3 < n) {
      v[r] = __ldg(reinterpret_cast<const int4*>(keys + t0 + li));  // tiles start 16-byte aligned
    } else {
      v[r].x = (t0 + li < n) ? __ldg(keys + t0 + li) : 0;
      v[r].y = (t0 + li + 1 < n) ? __ldg(keys + t0 + li + 1) : 0;
      v[r].z = (t0 + li + 2 < n) ? __ldg(keys + t0 + li + 2) : 0;
      v[r].w = (t0 + li + 3 < n) ? __ldg(keys + t0 + li + 3) : 0;
    }
  }
}

__global__ void __launch_bounds__(kSortThreads)
k_sort_count(const int* __restrict__ keys, const int* __restrict__ count, int shift, int mask,
             int* __restrict__ counts, int max_tiles, int* __restrict__ totals) {
  GS_PDL_ENTRY();
  __shared__ int s_h[kSortThreads / 32][kRadix];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = *count;
  const int ntiles = (n + kSortTileKeys - 1) / kSortTileKeys;
  int tot = 0;
  int4 v[2];
  if (blockIdx.x < ntiles) load_tile_keys(keys, n, blockIdx.x, tid, v);
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
#pragma unroll
    for (int k = 0; k < kRadix / 32; ++k) s_h[warp][lane + 32 * k] = 0;
    __syncwarp();
    int4 cur[2] = {v[0], v[1]};
    if (t + (int)gridDim.x < ntiles) load_tile_keys(keys, n, t + gridDim.x, tid, v);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int kv[4] = {cur[r].x, cur[r].y, cur[r].z, cur[r].w};
      const int left = n - (t * kSortTileKeys + 4 * (r * kSortThreads + tid));  // keys of this int4 in range
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < left) atomicAdd(&s_h[warp][((unsigned)kv[c] >> shift) & (unsigned)mask], 1);
    }
    __syncthreads();
    int c = 0;
#pragma unroll
    for (int w = 0; w < kSortThreads / 32; ++w) c += s_h[w][tid];
    counts[(size_t)tid * max_tiles + t] = c;
    tot += c;
    __syncthreads();
  }
  if (tot) atomicAdd(totals + tid, tot);
}

// Part 2: CTA d turns row d into output bases: the sum of the smaller
// digits' totals plus the exclusive prefix of the row.
__global__ void __launch_bounds__(1024)
k_sort_scan(int* __restrict__ counts, const int* __restrict__ count, int max_tiles,
            const int* __restrict__ totals) {
  GS_PDL_ENTRY();
  __shared__ int s_warp[32];
  __shared__ int s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = blockIdx.x;
  const int ntiles = (*count + kSortTileKeys - 1) / kSortTileKeys;
  // base of digit d: sum of totals[0, d)
  int part = (tid < d) ? totals[tid] : 0;  // 1024 threads >= 256 digits
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) s_warp[warp] = part;
  __syncthreads();
  if (tid == 0) {
    int b = 0;
    for (int w = 0; w < 32; ++w) b += s_warp[w];
    s_carry = b;
  }
  __syncthreads();
  int* row = counts + (size_t)d * max_tiles;
  for (int base = 0; base < ntiles; base += 1024) {
    const int i = base + tid;
    const int v = (i < ntiles) ? row[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[lane] = w;
    }
    __syncthreads();
    const int wpre = (warp > 0) ? s_warp[warp - 1] : 0;
    if (i < ntiles) row[i] = s_carry + wpre + x - v;
    const int blk = s_warp[31];
    __syncthreads();
    if (tid == 0) s_carry += blk;
    __syncthreads();
  }
}

// Part 3: stable scatter of each tile to bases[digit][tile] + rank. With
// bins / sorted_counts set (last depth pass), also sums the pair counts of
// every 256-Gaussian block of the output. The next tile's keys and ids are
// copied into the other half of a shared double buffer (cp.async) while the
// current one is ranked, so the global loads stay off the critical path.
__device__ __forceinline__ void prefetch_tile(const int* __restrict__ keys_in, const int* __restrict__ ids_in,
                                              int n, int t, int* s_k, int* s_i, int tid) {
  const int t0 = t * kSortTileKeys;
  const int tile_n = min(kSortTileKeys, n - t0);
#pragma unroll
  for (int c = tid; c < kSortTileKeys / 4; c += kSortThreads) {
    const int left = tile_n - 4 * c;  // keys of this 16-byte chunk in range
    if (left > 0) {
      const int bytes = left >= 4 ? 16 : 4 * left;  // tiles start 16-byte aligned
      cp_async16(s_k + 4 * c, keys_in + t0 + 4 * c, bytes);
      cp_async16(s_i + 4 * c, ids_in + t0 + 4 * c, bytes);
    }
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(kSortThreads, 4)
k_sort_scatter(const int* __restrict__ keys_in, const int* __restrict__ ids_in,
               int* __restrict__ keys_out, int* __restrict__ ids_out, const int* __restrict__ count,
               int shift, int mask, const int* __restrict__ bases, int max_tiles,
               const int2* __restrict__ bins, int* __restrict__ sorted_counts) {
  GS_PDL_ENTRY();
  __shared__ int s_whist[8][kRadix];
  __shared__ int s_tile_start[kRadix];
  __shared__ int s_gbase[kRadix];
  __shared__ __align__(16) int s_kbuf[2][kSortTileKeys];  // input tile, then its digit-ordered copy
  __shared__ __align__(16) int s_ibuf[2][kSortTileKeys];
  __shared__ int s_tmp[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lt = lanemask_lt();
  const int n = *count;
  const int ntiles = (n + kSortTileKeys - 1) / kSortTileKeys;
  const unsigned none = (unsigned)mask + 1u;  // digit of a missing key
  const int nbits = 33 - __clz(mask);          // bits of `none`: ballots per rank
  int buf = 0;
  if (blockIdx.x < ntiles) prefetch_tile(keys_in, ids_in, n, blockIdx.x, s_kbuf[0], s_ibuf[0], tid);
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    if (t + (int)gridDim.x < ntiles)
      prefetch_tile(keys_in, ids_in, n, t + gridDim.x, s_kbuf[buf ^ 1], s_ibuf[buf ^ 1], tid);
    else
      cp_async_commit();  // an empty group keeps the wait below uniform
    const int t0 = t * kSortTileKeys;
    const int tile_n = min(kSortTileKeys, n - t0);
#pragma unroll
    for (int k = 0; k < kRadix / 32; ++k) s_whist[warp][lane + 32 * k] = 0;
    s_gbase[tid] = bases[(size_t)tid * max_tiles + t];
    cp_async_wait_1();  // this thread's copies of tile t are done
    __syncthreads();    // and everyone's
    int* s_keys = s_kbuf[buf];
    int* s_ids = s_ibuf[buf];
    int key[kSortItems], id[kSortItems], rank[kSortItems];
    unsigned dig[kSortItems];
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      const int li = warp * (32 * kSortItems) + r * 32 + lane;
      const bool ok = li < tile_n;
      key[r] = s_keys[li];
      id[r] = s_ids[li];
      dig[r] = ok ? (((unsigned)key[r] >> shift) & (unsigned)mask) : none;
    }
    // rank within the warp's 256 keys, in order: 8 rounds of 32
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      const unsigned d = dig[r];
      const unsigned peers = same_value_lanes(d, nbits);
      int before = 0;
      if (d < none) before = s_whist[warp][d];
      __syncwarp();
      if (d < none && (peers & lt) == 0) s_whist[warp][d] = before + __popc(peers);
      __syncwarp();
      rank[r] = before + __popc(peers & lt);
    }
    __syncthreads();  // ranks done; every thread has read its keys from the buffer
    {
      int run = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int c = s_whist[w][tid];
        s_whist[w][tid] = run;
        run += c;
      }
      int tot;
      s_tile_start[tid] = block_exclusive_scan_256(run, s_tmp, &tot);
    }
    __syncthreads();  // s_tile_start complete before any thread stages
    // stage the tile in digit order (over its own input buffer) so that the
    // global stores form runs
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      if (dig[r] < none) {
        const int pos = s_tile_start[dig[r]] + s_whist[warp][dig[r]] + rank[r];
        s_keys[pos] = key[r];
        s_ids[pos] = id[r];
      }
    }
    __syncthreads();
    for (int i0 = warp * 32; i0 < tile_n; i0 += kSortThreads) {  // warp-uniform trip count
      const int i = i0 + lane;
      int out = -1, c = 0;
      if (i < tile_n) {
        const int k = s_keys[i];
        const unsigned d = ((unsigned)k >> shift) & (unsigned)mask;
        out = s_gbase[d] + (i - s_tile_start[d]);
        keys_out[out] = k;
        ids_out[out] = s_ids[i];
        if (sorted_counts) {
          const int2 b = bins[s_ids[i]];
          c = (b.y & 31) * ((b.y >> 5) & 31);
        }
      }
      if (sorted_counts) {
        // sum c over the lanes writing into the same 256-Gaussian output
        // block (one or two blocks per warp in practice); one add per block
        unsigned rem = __ballot_sync(0xffffffffu, out >= 0);
        while (rem) {
          const int l = __ffs(rem) - 1;
          const int b = __shfl_sync(0xffffffffu, out >> 8, l);
          const unsigned m = __ballot_sync(0xffffffffu, out >= 0 && (out >> 8) == b);
          int v = ((m >> lane) & 1u) ? c : 0;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == l) atomicAdd(sorted_counts + b, v);
          rem &= ~m;
        }
      }
    }
    __syncthreads();  // the buffer is refilled two tiles from now
    buf ^= 1;
  }
}

// ---------------------------------------------------------------------------
// Direct path. Look-back status word: high 32 bits the flag (0 = not yet
// published, 1 = this tile's own count, 2 = inclusive count of it and all
// earlier tiles), low 32 bits the count.
constexpr unsigned long long kOsAggregate = 1ull << 32;
constexpr unsigned long long kOsInclusive = 2ull << 32;
constexpr int kOsSpinLimit = 1 << 22;  // default bound of a wait: about a second of polling
constexpr int kLookback = 32;          // status words read per look-back round trip

__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Look-back over entry t of a sequence whose entries are `stride` words
// apart: publish_aggregate() makes `own` visible to the later entries at
// once (entry 0 inclusive); walk_back() then sums the earlier entries until
// an inclusive one, publishes its own inclusive count and returns the sum.
// Entries >= t are never read.
__device__ __forceinline__ void publish_aggregate(unsigned long long* words, size_t stride, int t, unsigned own) {
  st_relaxed(words + (size_t)t * stride, (t == 0 ? kOsInclusive : kOsAggregate) | own);
}

// A wait gives up after spin_limit rounds that found nothing new, adds 1 to
// *timeouts and goes on with the partial sum (the output is then invalid;
// every store stays in bounds). blind (a test setting, gs_test_set_sort_wait)
// reads every earlier word as unpublished, so the wait always runs out.
__device__ __forceinline__ long long walk_back(unsigned long long* words, size_t stride, int t, unsigned own,
                                               int* timeouts, int spin_limit, bool blind) {
  if (t == 0) return 0;
  unsigned long long* mine = words + (size_t)t * stride;
  long long excl = 0;
  int j = t - 1, spins = 0;
  for (;;) {
    unsigned long long w[kLookback];
#pragma unroll
    for (int k = 0; k < kLookback; ++k)
      w[k] = (j - k >= 0) ? ld_relaxed(words + (size_t)(j - k) * stride) : kOsInclusive;
    if (blind) {
#pragma unroll
      for (int k = 0; k < kLookback; ++k) w[k] = 0ull;
    }
    int used = 0;
    bool done = false;
#pragma unroll
    for (int k = 0; k < kLookback; ++k) {
      if (!done && used == k) {
        const unsigned f = (unsigned)(w[k] >> 32);
        if (f != 0u) {
          excl += (long long)(w[k] & 0xffffffffull);
          used = k + 1;
          done = (f == 2u);
        }
      }
    }
    if (done) break;
    j -= used;
    if (used == 0 && ++spins > spin_limit) {
      atomicAdd(timeouts, 1);
      break;
    }
  }
  st_relaxed(mine, kOsInclusive | (unsigned long long)(excl + own));
  return excl;
}

// Direct-path emission: one CTA per 256 Gaussians (index order) writes their
// (tile << 13 | depth) keys from pair_offsets[b] on; one warp per 32 of them
// writes the warp's contiguous run 32 pairs at a time, lane l finding the
// Gaussian of its pair by a 5-step search of the warp's exclusive offsets;
// within a Gaussian the tiles ascend. Counts the first pass's digits and
// clears the first pass's look-back words.
__global__ void __launch_bounds__(256)
k_emit_keys(const int2* __restrict__ bins, const int* __restrict__ pair_offsets, int n, int tiles_x,
            const Scalars* __restrict__ sc, long long cap, int* __restrict__ keys, int* __restrict__ ids,
            int* __restrict__ hist0, unsigned long long* __restrict__ status0) {
  GS_PDL_ENTRY();
  __shared__ int s_ex[8][33];
  __shared__ int2 s_bin[8][32];
  __shared__ int s_wtot[8];
  __shared__ int s_hist[kRadix];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  {
    const long long words = (long long)((sc->n_emit + kOsTileKeys - 1) / kOsTileKeys) * kRadix;
    for (long long w = blockIdx.x * 256ll + tid; w < words; w += (long long)gridDim.x * 256) status0[w] = 0ull;
  }
  s_hist[tid] = 0;
  const int i = blockIdx.x * 256 + tid;
  const int2 b = (i < n) ? bins[i] : make_int2(0, 0);
  const int cnt = (b.y & 31) * ((b.y >> 5) & 31);
  int x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  const int wtot = __shfl_sync(0xffffffffu, x, 31);
  s_ex[warp][lane] = x - cnt;
  s_bin[warp][lane] = b;
  if (lane == 0) s_wtot[warp] = wtot;
  __syncthreads();
  long long base = pair_offsets[blockIdx.x];
  for (int w = 0; w < warp; ++w) base += s_wtot[w];
  for (int e0 = 0; e0 < wtot; e0 += 32) {  // warp-uniform trip count
    const int e = e0 + lane;
    const long long pos = base + e;
    if (e < wtot && pos < cap) {
      int lo = 0;  // largest lo with s_ex[lo] <= e: a Gaussian with pairs
#pragma unroll
      for (int step = 16; step > 0; step >>= 1)
        if (s_ex[warp][lo + step] <= e) lo += step;
      const int2 q = s_bin[warp][lo];
      const int j = e - s_ex[warp][lo];
      const int nx = q.y & 31;
      const int dq = (q.y >> 10) & 0x1FFF;
      // j / nx for j < 256, nx <= 16: (j + 1/2) / nx is at least 1/32 away
      // from an integer, far more than the float rounding of the product
      const int oy = (int)__fmul_rn((float)j + 0.5f, __frcp_rn((float)nx)), ox = j - oy * nx;
      const int tx0 = q.x & 0xFFFF, ty0 = q.x >> 16;
      const int key = (((ty0 + oy) * tiles_x + (tx0 + ox)) << kDepthBits) | dq;
      keys[pos] = key;
      ids[pos] = blockIdx.x * 256 + warp * 32 + lo;
      atomicAdd(&s_hist[key & (kRadix - 1)], 1);
    }
  }
  __syncthreads();
  if (s_hist[tid]) atomicAdd(hist0 + tid, s_hist[tid]);
}

// Direct-path radix pass over *count keys: stable scatter by digit
// (key >> shift) & mask with a look-back for the earlier tiles' counts.
// hist holds this pass's global digit counts; with hist_next the pass also
// counts digit (key >> next_shift) & 255 for the next pass.
__global__ void __launch_bounds__(kSortThreads, 2)  // registers for a 32-word look-back window
k_sort_onesweep(const int* __restrict__ keys_in, const int* __restrict__ ids_in,
                int* __restrict__ keys_out, int* __restrict__ ids_out, const int* __restrict__ count,
                unsigned* __restrict__ sweep, int* __restrict__ timeouts, int spin_limit, int blind,
                int shift, int mask,
                const int* __restrict__ hist, int* __restrict__ hist_next, int next_shift,
                unsigned long long* __restrict__ status_cur,
                unsigned long long* __restrict__ status_next) {
  GS_PDL_ENTRY();
  __shared__ int s_whist[8][kRadix];
  __shared__ int s_tile_start[kRadix];
  __shared__ int s_gbase[kRadix];
  __shared__ int s_dbase[kRadix];
  __shared__ int s_keys[kOsTileKeys];
  __shared__ int s_ids[kOsTileKeys];
  __shared__ int s_tmp[8];
  __shared__ int s_tile;
  __shared__ int s_next[kRadix];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lt = lanemask_lt();
  const int n = *count;
  const int ntiles = (n + kOsTileKeys - 1) / kOsTileKeys;
  const unsigned none = (unsigned)mask + 1u;  // rank value of a missing key
  const int nbits = 33 - __clz(mask);
  s_next[tid] = 0;
  {
    int tot;
    s_dbase[tid] = block_exclusive_scan_256(hist[tid], s_tmp, &tot);
  }
  for (;;) {
    if (tid == 0) s_tile = (int)atomicAdd(sweep, 1u);
    __syncthreads();
    const int t = s_tile;
    if (t >= ntiles) {
      if (hist_next && s_next[tid]) atomicAdd(hist_next + tid, s_next[tid]);
      break;
    }
    status_next[(size_t)t * kRadix + tid] = 0ull;  // the next pass's word, unread until then
    const int t0 = t * kOsTileKeys;
    const int tile_n = min(kOsTileKeys, n - t0);
#pragma unroll
    for (int k = 0; k < kRadix / 32; ++k) s_whist[warp][lane + 32 * k] = 0;
    int key[kOsItems], id[kOsItems], rank[kOsItems];
    unsigned dig[kOsItems];
#pragma unroll
    for (int r = 0; r < kOsItems; ++r) {
      const int li = warp * (32 * kOsItems) + r * 32 + lane;
      const bool ok = li < tile_n;
      key[r] = ok ? keys_in[t0 + li] : 0;
      id[r] = ok ? ids_in[t0 + li] : 0;
      dig[r] = ok ? (((unsigned)key[r] >> shift) & (unsigned)mask) : (unsigned)kRadix;
    }
    if (hist_next) {
#pragma unroll
      for (int r = 0; r < kOsItems; ++r)
        if (dig[r] < (unsigned)kRadix) atomicAdd(&s_next[((unsigned)key[r] >> next_shift) & (kRadix - 1)], 1);
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < kOsItems; ++r) {
      const unsigned d = dig[r];
      const unsigned peers = same_value_lanes(d < (unsigned)kRadix ? d : none, nbits);
      int before = 0;
      if (d < (unsigned)kRadix) before = s_whist[warp][d];
      __syncwarp();
      if (d < (unsigned)kRadix && (peers & lt) == 0) s_whist[warp][d] = before + __popc(peers);
      __syncwarp();
      rank[r] = before + __popc(peers & lt);
    }
    __syncthreads();
    int cnt;
    {
      int run = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int c = s_whist[w][tid];
        s_whist[w][tid] = run;
        run += c;
      }
      cnt = run;
      publish_aggregate(status_cur + tid, kRadix, t, (unsigned)cnt);
      int tot;
      s_tile_start[tid] = block_exclusive_scan_256(run, s_tmp, &tot);
    }
    __syncthreads();  // s_tile_start complete
    // stage the tile in digit order first, so that the look-back runs with
    // the keys out of registers
#pragma unroll
    for (int r = 0; r < kOsItems; ++r) {
      if (dig[r] < (unsigned)kRadix) {
        const int pos = s_tile_start[dig[r]] + s_whist[warp][dig[r]] + rank[r];
        s_keys[pos] = key[r];
        s_ids[pos] = id[r];
      }
    }
    const long long excl = walk_back(status_cur + tid, kRadix, t, (unsigned)cnt, timeouts, spin_limit, blind != 0);
    s_gbase[tid] = s_dbase[tid] + (int)excl;
    __syncthreads();  // staging and s_gbase complete
    for (int i = tid; i < tile_n; i += kSortThreads) {
      const int k = s_keys[i];
      const unsigned d = ((unsigned)k >> shift) & (unsigned)mask;
      const int out = s_gbase[d] + (i - s_tile_start[d]);
      keys_out[out] = k;
      ids_out[out] = s_ids[i];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Tile ranges: ranges[t] = first index whose tile id >= t, for t in [0, T].
constexpr int kRangeGrid = 592;

// Tile ranges from the sorted keys: each thread looks at groups of 4 keys
// (one int4 load) and the key before them, and writes ranges[t] = i for the
// tiles t that start at position i. A grid-stride loop over the n_emit + 1
// positions (the grid is sized on the host from the capacity, capped).
__global__ void __launch_bounds__(256)
k_ranges_from_keys(const int* __restrict__ keys, int shift, const Scalars* __restrict__ sc, int T,
                   int* __restrict__ ranges) {
  GS_PDL_ENTRY();
  const int n = sc->n_emit;
  for (long long i0 = 4 * (blockIdx.x * 256ll + threadIdx.x); i0 <= n; i0 += 4ll * gridDim.x * 256) {
    int k[5];
    k[0] = (i0 == 0) ? -1 : min(max(keys[i0 - 1] >> shift, -1), T);
    if (i0 + 3 < n) {
      const int4 v = __ldg(reinterpret_cast<const int4*>(keys + i0));  // 16-byte aligned: i0 % 4 == 0
      k[1] = v.x >> shift; k[2] = v.y >> shift; k[3] = v.z >> shift; k[4] = v.w >> shift;
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) k[q + 1] = (i0 + q < n) ? (keys[i0 + q] >> shift) : T;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const long long i = i0 + q;
      if (i > n) break;
      // tile ids are in [0, T); the clamps keep writes in ranges[0, T]
      const int cur = min(max(k[q + 1], 0), T), prev = min(max(k[q], -1), T);
      for (int t = prev + 1; t <= cur; ++t) ranges[t] = (int)i;
      k[q + 1] = cur;
    }
  }
}

__global__ void __launch_bounds__(256)
k_ranges_from_ids(const int* __restrict__ tiles, long long ns, int T, int* __restrict__ ranges) {
  GS_PDL_ENTRY();
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i <= ns; i += (long long)gridDim.x * 256) {
    long long cur = (i < ns) ? (long long)tiles[i] : (long long)T;
    long long prev = (i == 0) ? -1 : (long long)tiles[i - 1];
    long long lo = prev + 1 < 0 ? 0 : prev + 1;
    long long hi = cur > T ? T : cur;
    for (long long t = lo; t <= hi; ++t) ranges[t] = (int)i;
  }
}

__global__ void __launch_bounds__(256)
k_export(const int* __restrict__ keys, int shift, const int* __restrict__ ids,
         const Scalars* __restrict__ sc, long long cap, int T, int* __restrict__ out_tiles,
         int* __restrict__ out_ids, int* __restrict__ out_count) {
  GS_PDL_ENTRY();
  const int n = sc->n_emit;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < cap; i += (long long)gridDim.x * 256) {
    bool ok = i < n;
    out_tiles[i] = ok ? (keys[i] >> shift) : T;
    out_ids[i] = ok ? ids[i] : 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && out_count) *out_count = sc->n_total;
}

// ---------------------------------------------------------------------------
static int resident_grid(const void* fn, int threads) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0);
  return sms * (per_sm > 0 ? per_sm : 1);
}

void launch_scan_block_counts(const int* block_counts, int n_blocks, int* pair_offsets, int* vis_offsets,
                              Scalars* sc, int64_t capacity, int num_tiles, GsExtras* extras,
                              cudaStream_t st) {
  GS_TIMED("scan_block_counts", st);
  launch_kernel(k_scan_block_counts, 1, 1024, 0, st, block_counts, n_blocks, pair_offsets, vis_offsets, sc, capacity,
                                          num_tiles, extras);
}

void launch_emit_keys(const int2* bins, const int* pair_offsets, int n, int tiles_x, const Scalars* sc,
                      int64_t capacity, int* keys, int* ids, int* hist0, unsigned long long* status0,
                      cudaStream_t st) {
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("emit_pairs", st);
  launch_kernel(k_emit_keys, nb, 256, 0, st, bins, pair_offsets, n, tiles_x, sc, capacity, keys, ids, hist0, status0);
}

// Bounded-wait setting of the look-back (gs_test_set_sort_wait): 0 = default.
static int g_sort_spin_limit = 0;
static int g_sort_blind = 0;

void set_sort_wait(int spin_limit, int blind) {
  g_sort_spin_limit = spin_limit > 0 ? spin_limit : 0;
  g_sort_blind = blind ? 1 : 0;
}

int launch_radix_sort_onesweep(int* keys0, int* ids0, int* keys1, int* ids1, const int* count, Scalars* sc,
                               int* hist, unsigned long long* status0, unsigned long long* status1,
                               int total_bits, cudaStream_t st) {
  static int grid = 0;  // resident CTAs (the GPUs of one node have the same SM count)
  if (grid == 0) grid = resident_grid((const void*)k_sort_onesweep, kSortThreads);
  int cur = 0;
  int* kb[2] = {keys0, keys1};
  int* ib[2] = {ids0, ids1};
  unsigned long long* sb[2] = {status0, status1};
  int pass = 0;
  for (int shift = 0; shift < total_bits; shift += kRadixBits, ++pass) {
    const int bits = total_bits - shift < kRadixBits ? total_bits - shift : kRadixBits;
    const int mask = (1 << bits) - 1;
    const int next_shift = shift + kRadixBits < total_bits ? shift + kRadixBits : -1;
    GS_TIMED("sort_keys", st);
    launch_kernel(k_sort_onesweep, grid, kSortThreads, 0, st,
        kb[cur], ib[cur], kb[cur ^ 1], ib[cur ^ 1], count, &sc->sweep_tile[pass], &sc->sort_timeouts,
        g_sort_spin_limit > 0 ? g_sort_spin_limit : kOsSpinLimit, g_sort_blind, shift,
        mask, hist + pass * kRadix, next_shift >= 0 ? hist + (pass + 1) * kRadix : nullptr, next_shift,
        sb[pass & 1], sb[(pass & 1) ^ 1]);
    cur ^= 1;
  }
  return cur;
}

void launch_compact_visible(const int2* bins, int n, const int* vis_offsets, int* dkeys, int* dids,
                            int* sorted_counts, cudaStream_t st) {
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("compact_visible", st);
  launch_kernel(k_compact_visible, nb, 256, 0, st, bins, n, vis_offsets, dkeys, dids, sorted_counts);
}

void launch_emit_sorted(const int2* bins, const int* order, int n, const Scalars* sc,
                        const int* sorted_counts, int* offsets, int tiles_x, int64_t capacity, int* keys,
                        int* ids, cudaStream_t st) {
  (void)capacity;  // n_emit <= capacity bounds every write
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  {
    GS_TIMED("scan_sorted_counts", st);
    launch_kernel(k_scan_sorted_counts, 1, 1024, 0, st, sorted_counts, sc, offsets);
  }
  GS_TIMED("emit_pairs", st);
  launch_kernel(k_emit_sorted, nb, 256, 0, st, bins, order, sc, offsets, tiles_x, keys, ids);
}

int launch_radix_sort(int* keys0, int* ids0, int* keys1, int* ids1, const int* count, int max_tiles,
                      int* counts, int* totals, int total_bits, const int2* bins, int* sorted_counts,
                      const char* name, cudaStream_t st) {
  static int grid_count = 0, grid_scatter = 0;  // resident CTAs (same SM count on every GPU of a node)
  if (grid_scatter == 0) {
    grid_count = resident_grid((const void*)k_sort_count, kSortThreads);
    grid_scatter = resident_grid((const void*)k_sort_scatter, kSortThreads);
  }
  int cur = 0;
  int* kb[2] = {keys0, keys1};
  int* ib[2] = {ids0, ids1};
  int pass = 0;
  const int passes = (total_bits + kRadixBits - 1) / kRadixBits;
  if (passes > 0) cudaMemsetAsync(totals, 0, sizeof(int) * kRadix * passes, st);
  for (int shift = 0; shift < total_bits; shift += kRadixBits, ++pass) {
    const int bits = total_bits - shift < kRadixBits ? total_bits - shift : kRadixBits;
    const int mask = (1 << bits) - 1;
    int* tot = totals + pass * kRadix;
    const bool last = pass == passes - 1;
    GS_TIMED(name, st);
    launch_kernel(k_sort_count, grid_count, kSortThreads, 0, st, kb[cur], count, shift, mask, counts, max_tiles, tot);
    launch_kernel(k_sort_scan, kRadix, 1024, 0, st, counts, count, max_tiles, tot);
    launch_kernel(k_sort_scatter, grid_scatter, kSortThreads, 0, st, kb[cur], ib[cur], kb[cur ^ 1], ib[cur ^ 1], count,
                                                          shift, mask, counts, max_tiles,
                                                          last ? bins : nullptr, last ? sorted_counts : nullptr);
    cur ^= 1;
  }
  return cur;
}

void launch_tile_ranges_from_keys(const int* sorted_keys, int shift, const Scalars* sc, int num_tiles,
                                  int64_t capacity, int* ranges, cudaStream_t st) {
  GS_TIMED("tile_ranges", st);
  const long long groups = (capacity + 4) / 4;  // 4 keys per thread, positions 0 .. capacity
  const long long grid = (groups + 255) / 256;
  launch_kernel(k_ranges_from_keys, (unsigned)(grid < 2368 ? grid : 2368), 256, 0, st, sorted_keys, shift, sc, num_tiles,
                                                                           ranges);
}

void launch_tile_ranges_from_ids(const int* sorted_tile_ids, int64_t n_sorted, int num_tiles,
                                 int* ranges, cudaStream_t st) {
  GS_TIMED("tile_ranges_ids", st);
  launch_kernel(k_ranges_from_ids, kRangeGrid, 256, 0, st, sorted_tile_ids, n_sorted, num_tiles, ranges);
}

void launch_export_interactions(const int* keys, int shift, const int* ids, const Scalars* sc,
                                int64_t capacity, int num_tiles, int* out_tiles, int* out_ids, int* out_count,
                                cudaStream_t st) {
  GS_TIMED("export", st);
  launch_kernel(k_export, kRangeGrid, 256, 0, st, keys, shift, ids, sc, capacity, num_tiles, out_tiles, out_ids,
                                       out_count);
}

}  // namespace gs
