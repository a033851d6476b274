// Stages 3 and 4: the front-to-back compositor and its backward.
//
// Compositing rule of the reference (rasterizer.py:202-215,
// rasterizer_tpu.py:308-336): a splat is applied while T > 1e-4 (tested
// before the splat), only where power > -10, with alpha = min(0.99,
// exp(power) sigmoid(o)); at most MAX_TILE_INTERACTIONS splats per tile;
// out = C + T bg.
//
// Forward: one CTA per 16x16 tile, PIX pixels per thread (a column of PIX
// rows), so each splat record staged in shared memory is read once per PIX
// pixels. The tile's sorted splats are processed in batches (kBatch, or
// kBatchSmall on small images: compositor_batch); before
// each batch the CTA checkpoints every pixel's (T, C) and names the batch a
// work item (tile, batch). A CTA stops as soon as every pixel has T <= 1e-4
// (the reference's scans run on but contribute nothing).
//
// Backward: every (tile, batch) work item is independent. With
// S_{j+1} = image - C_{<=j} (the colour still to come, background included),
//   dL/dalpha_j = T_j (c_j . G) - (image - C_{<=j}) . G / (1 - alpha_j)
//   dL/dc_j     = alpha_j T_j G,
// so an item replays its batch front to back from the forward's checkpoint,
// with the forward's own arithmetic (bit-identical T and decisions). A
// persistent grid takes items from an atomic counter (no CTA ever waits), so
// heavy tiles no longer form a tail. Per-splat gradients are reduced over
// each warp (transposed 14-shuffle reduction), summed over the CTA's warps
// with shared-memory atomics and added to the Gaussian's accumulator with
// float4 global atomics.
#include "gs_kernels.cuh"

namespace gs {

// e^x = 2^(x log2 e), with the PTX ex2.approx instruction; one helper so the
// forward and the backward evaluate identical values.
__device__ __forceinline__ float splat_exp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, 1.4426950408889634f)));
  return y;
}

// Paired fp32 arithmetic (sm_100 FFMA2 / FMUL2 / FADD2): each half is the
// IEEE single-precision operation, rounded as the scalar one, so the
// backward's two-pixel loop gives the forward's bits of T and alpha. (The
// forward stays scalar: there the pairs of broadcast splat values cost
// more register moves than the paired operations save.)
__device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// e^power for two pixels, as splat_exp on each.
__device__ __forceinline__ float2 splat_exp2(float2 power) {
  const float2 x = __fmul2_rn(power, dup2(1.4426950408889634f));
  return make_float2(ex2_approx(x.x), ex2_approx(x.y));
}

// ---------------------------------------------------------------------------
constexpr int kTileBuckets = 256;

// Work items per tile and the tile-count statistics (renderer.py:61,76-88).
// sort_timeouts (nullable): the sort's count of bounded waits that gave up;
// if it is nonzero the pair order is unknown, so every range is emptied
// (nothing is composited) and the count goes to GsExtras.device_timeouts.
__global__ void __launch_bounds__(1024)
k_tile_items(int* __restrict__ ranges, int T, int batch, int* __restrict__ tile_items,
             Scalars* __restrict__ sc, GsExtras* __restrict__ ex, const int* __restrict__ sort_timeouts,
             int* __restrict__ tile_order) {
  GS_PDL_ENTRY();
  __shared__ int s_warp[32];
  __shared__ int s_carry;
  __shared__ int s_stat[5][32];
  __shared__ int s_thist[kTileBuckets];
  __shared__ int s_tnext[kTileBuckets];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int timeouts = sort_timeouts ? *sort_timeouts : 0;
  if (timeouts != 0) {
    for (int t = tid; t <= T; t += 1024) ranges[t] = 0;
    __syncthreads();
  }
  if (tid == 0) s_carry = 0;
  int mx = 0, ovt = 0, ovi = 0, trt = 0, tri = 0;
  __syncthreads();
  for (int base = 0; base < T; base += 1024) {
    const int t = base + tid;
    int cnt = 0;
    if (t < T) cnt = ranges[t + 1] - ranges[t];
    const int v = (min(cnt, kMaxTileInteractions) + batch - 1) / batch;
    mx = max(mx, cnt);
    if (cnt > kBlockSize) { ovt += 1; ovi += cnt - kBlockSize; }
    if (cnt > kMaxTileInteractions) { trt += 1; tri += cnt - kMaxTileInteractions; }
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
    const int excl = s_carry + ((warp > 0) ? s_warp[warp - 1] : 0) + x - v;
    if (t < T) tile_items[t] = excl;
    const int blk = s_warp[31];
    __syncthreads();
    if (tid == 0) s_carry += blk;
    __syncthreads();
  }
  // statistics: warp then CTA reduction
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    ovt += __shfl_xor_sync(0xffffffffu, ovt, o);
    ovi += __shfl_xor_sync(0xffffffffu, ovi, o);
    trt += __shfl_xor_sync(0xffffffffu, trt, o);
    tri += __shfl_xor_sync(0xffffffffu, tri, o);
  }
  if (lane == 0) {
    s_stat[0][warp] = mx; s_stat[1][warp] = ovt; s_stat[2][warp] = ovi;
    s_stat[3][warp] = trt; s_stat[4][warp] = tri;
  }
  __syncthreads();
  if (tile_order) {
    // the forward's CTA order: tiles by pair count, most first (a counting
    // sort in buckets of 16 pairs). Consecutive CTAs go to different SMs, so
    // the heaviest tiles are spread one per SM instead of clustering (image
    // centres are dense) on a few.
    if (tid < kTileBuckets) s_thist[tid] = 0;
    __syncthreads();
    for (int t = tid; t < T; t += 1024)
      atomicAdd(&s_thist[min(min(ranges[t + 1] - ranges[t], kMaxTileInteractions) >> 4, kTileBuckets - 1)], 1);
    __syncthreads();
    if (warp == 0) {
      // bucket kTileBuckets - 1 first: lane l holds buckets 255 - 8l .. 248 - 8l
      constexpr int per = kTileBuckets / 32;
      int h[per], sum = 0;
#pragma unroll
      for (int j = 0; j < per; ++j) {
        h[j] = s_thist[kTileBuckets - 1 - per * lane - j];
        sum += h[j];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int run = incl - sum;
#pragma unroll
      for (int j = 0; j < per; ++j) {
        s_tnext[kTileBuckets - 1 - per * lane - j] = run;
        run += h[j];
      }
    }
    __syncthreads();
    for (int t = tid; t < T; t += 1024) {
      const int bkt = min(min(ranges[t + 1] - ranges[t], kMaxTileInteractions) >> 4, kTileBuckets - 1);
      tile_order[atomicAdd(&s_tnext[bkt], 1)] = t;
    }
  }
  if (tid == 0) {
    int a = 0, b = 0, c = 0, d = 0, e = 0;
    for (int w = 0; w < 32; ++w) {
      a = max(a, s_stat[0][w]); b += s_stat[1][w]; c += s_stat[2][w];
      d += s_stat[3][w]; e += s_stat[4][w];
    }
    tile_items[T] = s_carry;
    sc->n_items = s_carry;
    if (ex) {
      ex->max_interactions_per_tile = a;
      ex->overflow_tiles = b;
      ex->overflow_interactions = c;
      ex->truncated_tiles = d;
      ex->truncated_interactions = e;
      ex->device_timeouts = timeouts;
    }
  }
}

// ---------------------------------------------------------------------------
// Pixel ownership of the compositor kernels. A tile CTA has NT = 256 / PIX
// threads in NW warps; warp w owns a WX x WY block of the tile's pixels and
// each thread a column of PIX rows inside it.
template <int PIX, int WX>
struct Foot {
  static constexpr int NT = kTilePixels / PIX;
  static constexpr int NW = NT / 32;
  static constexpr int WY = 32 * PIX / WX;
  static constexpr int WPR = kTile / WX;  // warps per block row
  static_assert(WX * WY * NW == kTilePixels && WPR * WX == kTile, "bad pixel ownership");
  __device__ static int col(int warp, int lane) { return (warp % WPR) * WX + lane % WX; }
  __device__ static int row0(int warp, int lane) { return (warp / WPR) * WY + (lane / WX) * PIX; }
  // Bit w set: the splat's power > -10 region (box of half-extents hx, hy
  // around (mx, my), then the exact ellipse test splat_meets_rect) can meet
  // the pixel centres of warp w of tile (tx, ty).
  __device__ static unsigned warp_mask(float mx, float my, float hx, float hy, float ha, float hb, float hc,
                                       int tx, int ty) {
    unsigned m = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float x0 = (float)(tx * kTile + (w % WPR) * WX) + 0.5f, x1 = x0 + (float)(WX - 1);
      const float y0 = (float)(ty * kTile + (w / WPR) * WY) + 0.5f, y1 = y0 + (float)(WY - 1);
      const bool miss = (mx + hx < x0) | (mx - hx > x1) | (my + hy < y0) | (my - hy > y1);
      if (!miss && splat_meets_rect(mx, my, ha, hb, hc, x0, x1, y0, y1)) m |= 1u << w;
    }
    return m;
  }
};

__device__ __forceinline__ unsigned lane_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// The batch positions (ascending) whose bit `warp` is set in s_mask[0, nb),
// written to list; returns their count. Whole warp.
__device__ __forceinline__ int warp_list(const unsigned char* s_mask, int nb, int warp, int lane,
                                         unsigned char* list) {
  int cnt = 0;
  const unsigned lt = lane_lt();
  for (int r = 0; r < nb; r += 32) {
    const int j = r + lane;
    const bool in = (j < nb) && ((s_mask[j] >> warp) & 1u);
    const unsigned bal = __ballot_sync(0xffffffffu, in);
    if (in) list[cnt + __popc(bal & lt)] = (unsigned char)j;
    cnt += __popc(bal);
  }
  __syncwarp();
  return cnt;
}

// Forward. Per batch, the loading threads test each splat's power > -10 box
// against every warp's pixels once; each warp then composites only the
// splats on its own list, in batch (depth) order. A skipped splat has
// alpha = 0 at all of the warp's pixels, so skipping it changes nothing.
// ckpt == nullptr: no checkpoints or work items (no backward will follow).
template <int PIX, int WX, int BATCH>
__global__ void __launch_bounds__(kTilePixels / PIX, 4 * PIX)  // 32 warps per SM
k_raster_fwd(const Splat* __restrict__ splats, const int* __restrict__ ids,
             const int* __restrict__ ranges, const int* __restrict__ tile_items, int n,
             const float* __restrict__ bg, int width, int height, int tiles_x,
             float* __restrict__ image, float* __restrict__ img_copy, float* __restrict__ pix_T,
             float4* __restrict__ ckpt, int* __restrict__ item_info, int* __restrict__ item_cost,
             const int* __restrict__ tile_order) {
  GS_PDL_ENTRY();
  using F = Foot<PIX, WX>;
  constexpr int NT = F::NT;
  __shared__ float4 s_a[BATCH];
  __shared__ float4 s_b[BATCH];
  __shared__ float4 s_c[BATCH];
  __shared__ unsigned char s_mask[BATCH];
  __shared__ unsigned char s_list[F::NW][BATCH];
  __shared__ int s_cost;  // splat steps of the current batch, summed over the warps
  const int tile = tile_order ? tile_order[blockIdx.x] : (int)blockIdx.x;
  const int tx = tile % tiles_x, ty = tile / tiles_x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lx = F::col(warp, lane), ly0 = F::row0(warp, lane);
  const int px = tx * kTile + lx;
  const float fpx = (float)px + 0.5f;
  const int start = ranges[tile];
  const int count = min(ranges[tile + 1] - start, kMaxTileInteractions);
  const int nbt = (count + BATCH - 1) / BATCH;
  const int it0 = tile_items ? tile_items[tile] : 0;
  float T[PIX], C0[PIX], C1[PIX], C2[PIX], fpy[PIX];
#pragma unroll
  for (int i = 0; i < PIX; ++i) {
    const int py = ty * kTile + ly0 + i;
    fpy[i] = (float)py + 0.5f;
    T[i] = (px < width && py < height) ? 1.f : 0.f;  // outside pixels never contribute
    C0[i] = C1[i] = C2[i] = 0.f;
  }
  if (tid == 0) s_cost = 0;
  int b = 0;
  for (; b < nbt; ++b) {
    bool alive = false;
#pragma unroll
    for (int i = 0; i < PIX; ++i) alive |= (T[i] > 1e-4f);
    const int n_alive = __syncthreads_count(alive);
    if (ckpt && tid == 0 && b > 0) {  // the previous batch is complete (barrier above)
      item_cost[it0 + b - 1] = s_cost;
      s_cost = 0;
    }
    if (n_alive == 0) {
      if (ckpt)
        for (int bb = b + tid; bb < nbt; bb += NT) {
          item_info[it0 + bb] = pack_item(tile, bb, true);
          item_cost[it0 + bb] = 0;
        }
      break;
    }
    if (ckpt) {
      if (tid == 0) item_info[it0 + b] = pack_item(tile, b, false);
      float4* ck = ckpt + (size_t)(it0 + b) * kTilePixels;
#pragma unroll
      for (int i = 0; i < PIX; ++i) ck[(ly0 + i) * kTile + lx] = make_float4(T[i], C0[i], C1[i], C2[i]);
    }
    const int b0 = b * BATCH;
    const int nb = min(BATCH, count - b0);
    for (int j = tid; j < nb; j += NT) {
      int g = ids[start + b0 + j];
      g = min(max(g, 0), n - 1);
      const Splat* sp = splats + g;
      const float4 a = __ldg(&sp->a), bb = __ldg(&sp->b), c = __ldg(&sp->c);
      s_a[j] = a;
      s_b[j] = bb;
      s_c[j] = c;
      s_mask[j] = (unsigned char)F::warp_mask(a.x, a.y, c.y, c.z, a.z, a.w, bb.x, tx, ty);
    }
    __syncthreads();
    const int cnt = warp_list(s_mask, nb, warp, lane, s_list[warp]);
    const unsigned char* list = s_list[warp];
    int q = 0;
    for (; alive && q < cnt; ++q) {
      const int k = list[q];
      const float4 A = s_a[k];
      const float4 B = s_b[k];
      const float4 Cc = s_c[k];
      const float dx = fpx - A.x;
      const float q0 = splat_q0(dx, A.z), q1 = splat_q1(dx, A.w);
#pragma unroll
      for (int i = 0; i < PIX; ++i) {
        const float power = splat_power(fpy[i] - A.y, q0, q1, B.x);
        const float a_raw = fminf(0.99f, __fmul_rn(splat_exp(power), B.y));
        const float alpha = ((T[i] > 1e-4f) & (power > -10.f)) ? a_raw : 0.f;
        const float w = __fmul_rn(alpha, T[i]);
        C0[i] = __fmaf_rn(w, B.z, C0[i]);
        C1[i] = __fmaf_rn(w, B.w, C1[i]);
        C2[i] = __fmaf_rn(w, Cc.x, C2[i]);
        T[i] = __fmul_rn(T[i], __fsub_rn(1.f, alpha));
      }
      if ((q & 15) == 15) {
        alive = false;
#pragma unroll
        for (int i = 0; i < PIX; ++i) alive |= (T[i] > 1e-4f);
      }
    }
    // the backward replays this warp's list until no lane of it is alive:
    // the largest q of its lanes
    if (ckpt) {
      const int qm = (int)__reduce_max_sync(0xffffffffu, (unsigned)q);
      if (lane == 0) atomicAdd(&s_cost, qm);
    }
  }
  if (ckpt && b == nbt && nbt > 0) {  // the last batch ran to its end: its cost is not written yet
    __syncthreads();
    if (tid == 0) item_cost[it0 + nbt - 1] = s_cost;
  }
  float b0 = 0.f, b1 = 0.f, b2 = 0.f;
  if (bg) { b0 = bg[0]; b1 = bg[1]; b2 = bg[2]; }
#pragma unroll
  for (int i = 0; i < PIX; ++i) {
    const int py = ty * kTile + ly0 + i;
    if (px < width && py < height) {
      const int pix = py * width + px;
      const float o0 = C0[i] + T[i] * b0, o1 = C1[i] + T[i] * b1, o2 = C2[i] + T[i] * b2;
      image[3 * pix] = o0;
      image[3 * pix + 1] = o1;
      image[3 * pix + 2] = o2;
      if (img_copy) {
        img_copy[3 * pix] = o0;
        img_copy[3 * pix + 1] = o1;
        img_copy[3 * pix + 2] = o2;
      }
      if (pix_T) pix_T[pix] = T[i];
    }
  }
}

// Warp sum of nine per-lane values with 14 shuffles: values 0..7 by recursive
// halving (each exchange keeps half of the vector: 4 + 2 + 1 shuffles, then
// 2 more over the last two lane bits), value 8 by a plain butterfly. On
// return, lanes 4i..4i+3 hold the total of value i in v[0] (i < 8) and every
// lane holds the total of value 8 in v[8].
__device__ __forceinline__ void warp_sum9(float v[9], int lane) {
  const bool h4 = lane & 16, h2 = lane & 8, h1 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float send = h4 ? v[i] : v[i + 4];
    float keep = h4 ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float send = h2 ? v[i] : v[i + 2];
    float keep = h2 ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    float send = h1 ? v[0] : v[1];
    float keep = h1 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v[8] += __shfl_xor_sync(0xffffffffu, v[8], o);
}

template <int PIX, int WX, int BATCH>
__global__ void __launch_bounds__(kTilePixels / PIX)
k_raster_bwd(const Splat* __restrict__ splats, const int* __restrict__ ids,
             const int* __restrict__ ranges, int n, int width, int height, int tiles_x,
             const float* __restrict__ grad_image, const float* __restrict__ img,
             const float4* __restrict__ ckpt, const int* __restrict__ item_info,
             const int* __restrict__ item_order, Scalars* __restrict__ sc, SplatGrad* __restrict__ grads) {
  GS_PDL_ENTRY();
  using F = Foot<PIX, WX>;
  constexpr int NT = F::NT;
  __shared__ float4 s_a[BATCH];
  __shared__ float4 s_b[BATCH];
  __shared__ float4 s_c[BATCH];
  __shared__ int s_gid[BATCH];
  __shared__ float s_acc[9][BATCH + 1];  // +1: the 9 rows of one splat in 9 banks
  __shared__ unsigned char s_mask[BATCH];
  __shared__ unsigned char s_list[F::NW][BATCH];
  __shared__ int s_item;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lx = F::col(warp, lane), ly0 = F::row0(warp, lane);
  const int n_items = sc->n_items;
  const bool sorted = sc->item_sorted != 0;
  for (int j = tid; j < 9 * (BATCH + 1); j += NT) (&s_acc[0][0])[j] = 0.f;
  for (;;) {
    if (tid == 0) {
      const int c = (int)atomicAdd(&sc->item_counter, 1u);
      s_item = c < n_items ? (sorted ? item_order[c] : c) : n_items;  // longest items first when sorted
    }
    __syncthreads();
    const int item = s_item;
    __syncthreads();
    if (item >= n_items) break;
    const int info = item_info[item];
    if (item_skipped(info)) continue;  // the forward stopped before this batch
    const int tile = item_tile(info), b = item_batch(info);
    const int tx = tile % tiles_x, ty = tile / tiles_x;
    const int start = ranges[tile];
    const int count = min(ranges[tile + 1] - start, kMaxTileInteractions);
    const int b0 = b * BATCH;
    const int nb = min(BATCH, count - b0);
    const int px = tx * kTile + lx;
    const float fpx = (float)px + 0.5f;
    float T[PIX], G0[PIX], G1[PIX], G2[PIX], IG[PIX], CG[PIX], fpy[PIX];
    const float4* ck = ckpt + (size_t)item * kTilePixels;
#pragma unroll
    for (int i = 0; i < PIX; ++i) {
      const int py = ty * kTile + ly0 + i;
      fpy[i] = (float)py + 0.5f;
      G0[i] = G1[i] = G2[i] = IG[i] = CG[i] = 0.f;
      T[i] = 0.f;
      if (px < width && py < height) {
        const int pix = py * width + px;
        G0[i] = grad_image[3 * pix];
        G1[i] = grad_image[3 * pix + 1];
        G2[i] = grad_image[3 * pix + 2];
        IG[i] = img[3 * pix] * G0[i] + img[3 * pix + 1] * G1[i] + img[3 * pix + 2] * G2[i];
        const float4 c = ck[(ly0 + i) * kTile + lx];
        T[i] = c.x;
        CG[i] = c.y * G0[i] + c.z * G1[i] + c.w * G2[i];
      }
    }
    for (int j = tid; j < nb; j += NT) {
      int g = ids[start + b0 + j];
      g = min(max(g, 0), n - 1);
      const Splat* sp = splats + g;
      const float4 a = __ldg(&sp->a), bb = __ldg(&sp->b), c = __ldg(&sp->c);
      s_gid[j] = g;
      s_a[j] = a;
      s_b[j] = bb;
      s_c[j] = c;
      s_mask[j] = (unsigned char)F::warp_mask(a.x, a.y, c.y, c.z, a.z, a.w, bb.x, tx, ty);
    }
    __syncthreads();
    const int cnt = warp_list(s_mask, nb, warp, lane, s_list[warp]);
    const unsigned char* list = s_list[warp];
    bool alive = false;
#pragma unroll
    for (int i = 0; i < PIX; ++i) alive |= (T[i] > 1e-4f);
    alive = __any_sync(0xffffffffu, alive);
    float2 T2, G0_2, G1_2, G2_2, IG2, CG2, fpy2;
    if constexpr (PIX == 2) {
      T2 = make_float2(T[0], T[1]);
      G0_2 = make_float2(G0[0], G0[1]);
      G1_2 = make_float2(G1[0], G1[1]);
      G2_2 = make_float2(G2[0], G2[1]);
      IG2 = make_float2(IG[0], IG[1]);
      CG2 = make_float2(CG[0], CG[1]);
      fpy2 = make_float2(fpy[0], fpy[1]);
    }
    for (int q = 0; alive && q < cnt; ++q) {
      const int k = list[q];
      const float4 A = s_a[k];
      const float4 B = s_b[k];
      const float4 Cc = s_c[k];
      const float dx = fpx - A.x;
      const float q0 = splat_q0(dx, A.z), q1 = splat_q1(dx, A.w);
      // The thread's pixels share dx, so the exponent's gradients follow from
      // three sums over them: S0 = sum dpow, S1 = sum dpow dy, S2 = sum dpow dy^2.
      float v[9];
      float S0 = 0.f, S1 = 0.f, S2 = 0.f;
      v[6] = v[7] = v[8] = 0.f;
      bool contrib = false;
      if constexpr (PIX == 2) {
        // the forward's arithmetic on the pixel pair (same bits of T and alpha)
        const float2 dy = __fadd2_rn(fpy2, dup2(-A.y));
        const float2 power = __ffma2_rn(dy, __ffma2_rn(dy, dup2(B.x), dup2(q1)), dup2(q0));
        const float2 e = splat_exp2(power);
        const float2 ea = __fmul2_rn(e, dup2(B.y));
        const bool act0 = (T2.x > 1e-4f) & (power.x > -10.f), act1 = (T2.y > 1e-4f) & (power.y > -10.f);
        const float2 alpha = make_float2(act0 ? fminf(0.99f, ea.x) : 0.f, act1 ? fminf(0.99f, ea.y) : 0.f);
        const float2 one_m = __ffma2_rn(alpha, dup2(-1.f), dup2(1.f));
        const float2 cG = __ffma2_rn(dup2(Cc.x), G2_2, __ffma2_rn(dup2(B.w), G1_2, __fmul2_rn(dup2(B.z), G0_2)));
        const float2 w = __fmul2_rn(alpha, T2);
        CG2 = __ffma2_rn(w, cG, CG2);
        // dalpha = T cG - (IG - C) / (1 - alpha)
        const float2 rem = __ffma2_rn(CG2, dup2(-1.f), IG2);
        const float2 nrcp = make_float2(__fdividef(-1.f, one_m.x), __fdividef(-1.f, one_m.y));
        const float2 dalpha = __ffma2_rn(rem, nrcp, __fmul2_rn(T2, cG));
        T2 = __fmul2_rn(T2, one_m);
        // u = dL/d(ea) e, with jnp.minimum(0.99, ea)'s gradient 1 below, 1/2
        // at the tie, 0 above (and 0 where the splat is not applied)
        const float fe0 = act0 ? ((ea.x < 0.99f) ? e.x : ((ea.x == 0.99f) ? 0.5f * e.x : 0.f)) : 0.f;
        const float fe1 = act1 ? ((ea.y < 0.99f) ? e.y : ((ea.y == 0.99f) ? 0.5f * e.y : 0.f)) : 0.f;
        const float2 u = __fmul2_rn(dalpha, make_float2(fe0, fe1));
        v[6] = __fmaf_rn(w.y, G0_2.y, w.x * G0_2.x);
        v[7] = __fmaf_rn(w.y, G1_2.y, w.x * G1_2.x);
        v[8] = __fmaf_rn(w.y, G2_2.y, w.x * G2_2.x);
        const float2 uy = __fmul2_rn(u, dy);
        S0 = u.x + u.y;
        v[5] = S0;
        S1 = uy.x + uy.y;
        S2 = __fmaf_rn(uy.y, dy.y, uy.x * dy.x);
        contrib = act0 | act1;
      } else
#pragma unroll
      for (int i = 0; i < PIX; ++i) {
        const float dy = fpy[i] - A.y;
        const float power = splat_power(dy, q0, q1, B.x);
        const float e = splat_exp(power);
        const float ea = __fmul_rn(e, B.y);
        const bool act = (T[i] > 1e-4f) & (power > -10.f);
        const float alpha = act ? fminf(0.99f, ea) : 0.f;
        const float one_m = __fsub_rn(1.f, alpha);
        const float cG = B.z * G0[i] + B.w * G1[i] + Cc.x * G2[i];
        const float w = __fmul_rn(alpha, T[i]);
        CG[i] += w * cG;
        const float dalpha = T[i] * cG - __fdividef(IG[i] - CG[i], one_m);
        T[i] = __fmul_rn(T[i], one_m);
        // u = dL/d(ea) e, as in the two-pixel path
        const float fe = act ? ((ea < 0.99f) ? e : ((ea == 0.99f) ? 0.5f * e : 0.f)) : 0.f;
        const float u = dalpha * fe;
        v[6] += w * G0[i];
        v[7] += w * G1[i];
        v[8] += w * G2[i];
        S0 += u;
        const float uy = u * dy;
        S1 += uy;
        S2 += uy * dy;
        contrib |= act;
      }
      if constexpr (PIX != 2) v[5] = S0;
      // The mean and conic gradients are linear in the sums below with the
      // splat's constants, so they are reduced raw and combined once per
      // splat when the batch is flushed (see there).
      const float dxS0 = dx * S0;
      v[0] = dxS0;
      v[1] = S1;
      v[2] = dx * dxS0;
      v[3] = dx * S1;
      v[4] = S2;
      if (__any_sync(0xffffffffu, contrib)) {
        warp_sum9(v, lane);
        if ((lane & 3) == 0) atomicAdd(&s_acc[lane >> 2][k], v[0]);
        if (lane == 1) atomicAdd(&s_acc[8][k], v[8]);
      }
      if ((q & 15) == 15) {
        bool al = false;
        if constexpr (PIX == 2) al = (T2.x > 1e-4f) | (T2.y > 1e-4f); else
#pragma unroll
        for (int i = 0; i < PIX; ++i) al |= (T[i] > 1e-4f);
        alive = __any_sync(0xffffffffu, al);
      }
    }
    __syncthreads();
    for (int j = tid; j < nb; j += NT) {
      float a[9];
#pragma unroll
      for (int q = 0; q < 9; ++q) {
        a[q] = s_acc[q][j];
        s_acc[q][j] = 0.f;
      }
      if ((a[0] != 0.f) | (a[1] != 0.f) | (a[2] != 0.f) | (a[3] != 0.f) | (a[4] != 0.f) |
          (a[5] != 0.f) | (a[6] != 0.f) | (a[7] != 0.f) | (a[8] != 0.f)) {
        // power = ha dx^2 + hb dx dy + hc dy^2 with (ha, hb, hc) = -(a, b2, c) / 2
        // and mean = pixel - (dx, dy); dL/dpower = u sig per pixel (ea = e sig,
        // sig the splat's opacity). From the sums R0 = sum dx S0, R1 = sum S1,
        // R2 = sum dx^2 S0, R3 = sum dx S1, R4 = sum S2 (S0 = u, S1 = u dy,
        // S2 = u dy^2 per thread) the gradients of mean x, y and of (a, b2, c)
        const float ha = s_a[j].z, hb = s_a[j].w, hc = s_b[j].x, sig = s_b[j].y;
        const float r0 = sig * a[0], r1 = sig * a[1], hs = -0.5f * sig;
        a[0] = -2.f * ha * r0 - hb * r1;
        a[1] = -2.f * hc * r1 - hb * r0;
        a[2] = hs * a[2];
        a[3] = hs * a[3];
        a[4] = hs * a[4];
        SplatGrad* gp = grads + s_gid[j];
        atomicAdd(&gp->a, make_float4(a[0], a[1], a[2], a[3]));
        atomicAdd(&gp->b, make_float4(a[4], a[5], a[6], a[7]));
        atomicAdd(&gp->c.x, a[8]);
      }
    }
  }
}

// The backward's work-item order: items sorted by decreasing cost (the
// splat steps the forward ran for them, in buckets of 8), so that the
// persistent grid starts the long items first and ends on short ones
// (longest-processing-time-first scheduling). That matters while the items
// are few for the grid (about one per resident CTA at 504x378); with
// lpt_below items or more the tail is short anyway and the kernel only
// clears sc->item_sorted, so the backward takes the items in index order.
// One CTA: a histogram of the buckets, their exclusive scan from the top
// bucket down, a scatter. The order inside a bucket follows the
// shared-memory atomics (the gradient sums are order-dependent in their last
// bits anyway: float atomics).
constexpr int kCostBuckets = 128;

__global__ void __launch_bounds__(1024)
k_item_order(const int* __restrict__ item_cost, Scalars* __restrict__ sc, int lpt_below, int* __restrict__ order) {
  GS_PDL_ENTRY();
  __shared__ int s_hist[kCostBuckets];
  __shared__ int s_next[kCostBuckets];
  const int tid = threadIdx.x;
  const int n = sc->n_items;
  if (n >= lpt_below) {
    if (tid == 0) sc->item_sorted = 0;
    return;
  }
  if (tid == 0) sc->item_sorted = 1;
  if (tid < kCostBuckets) s_hist[tid] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += 1024) atomicAdd(&s_hist[min(item_cost[i] >> 3, kCostBuckets - 1)], 1);
  __syncthreads();
  if (tid < 32) {
    // bucket kCostBuckets - 1 first: lane l holds buckets 127 - 4l .. 124 - 4l
    int h[4], sum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = s_hist[kCostBuckets - 1 - 4 * tid - j];
      sum += h[j];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += y;
    }
    int run = incl - sum;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s_next[kCostBuckets - 1 - 4 * tid - j] = run;
      run += h[j];
    }
  }
  __syncthreads();
  for (int i = tid; i < n; i += 1024) {
    const int pos = atomicAdd(&s_next[min(item_cost[i] >> 3, kCostBuckets - 1)], 1);
    order[pos] = i;
  }
}

// d image / d background = T_final per pixel (renderer.py:230): sum T * G.
__global__ void __launch_bounds__(256)
k_grad_bg(const float* __restrict__ pix_T, const float* __restrict__ grad_image, int P,
          float* __restrict__ grad_bg) {
  GS_PDL_ENTRY();
  float v0 = 0.f, v1 = 0.f, v2 = 0.f;
  for (int p = blockIdx.x * 256 + threadIdx.x; p < P; p += gridDim.x * 256) {
    const float t = pix_T[p];
    v0 += t * grad_image[3 * p];
    v1 += t * grad_image[3 * p + 1];
    v2 += t * grad_image[3 * p + 2];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v0 += __shfl_xor_sync(0xffffffffu, v0, o);
    v1 += __shfl_xor_sync(0xffffffffu, v1, o);
    v2 += __shfl_xor_sync(0xffffffffu, v2, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(grad_bg, v0);
    atomicAdd(grad_bg + 1, v1);
    atomicAdd(grad_bg + 2, v2);
  }
}

// Pixels per thread and warp block width of the two compositor kernels.
#ifndef GS_FWD_PIX
#define GS_FWD_PIX 2
#endif
#ifndef GS_FWD_WX
#define GS_FWD_WX 8
#endif
#ifndef GS_BWD_PIX
#define GS_BWD_PIX 2
#endif
#ifndef GS_BWD_WX
#define GS_BWD_WX 8
#endif
constexpr int kFwdPix = GS_FWD_PIX, kFwdWx = GS_FWD_WX;
constexpr int kBwdPix = GS_BWD_PIX, kBwdWx = GS_BWD_WX;

static int persistent_ctas(const void* fn, int threads) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0);
  return sms * (per_sm > 0 ? per_sm : 1);
}

void launch_tile_items(int* ranges, int num_tiles, int* tile_items, Scalars* sc,
                       GsExtras* extras, const int* sort_timeouts, int* tile_order, cudaStream_t st) {
  GS_TIMED("tile_items", st);
  launch_kernel(k_tile_items, 1, 1024, 0, st, ranges, num_tiles, compositor_batch(num_tiles), tile_items, sc, extras,
                                   sort_timeouts, tile_order);
}

void launch_raster_fwd(const Splat* splats, const int* ids, const int* ranges,
                       const int* tile_items, int n, const float* bg, int width, int height,
                       int tiles_x, int num_tiles, float* image, float* img_copy, float* pix_T,
                       float4* ckpt, int* item_info, int* item_cost, const int* tile_order, cudaStream_t st) {
  if (num_tiles == 0) return;
  GS_TIMED("raster_fwd", st);
  if (compositor_batch(num_tiles) == kBatchSmall)
    launch_kernel(k_raster_fwd<kFwdPix, kFwdWx, kBatchSmall>, num_tiles, kTilePixels / kFwdPix, 0, st,
        splats, ids, ranges, tile_items, n, bg, width, height, tiles_x, image, img_copy, pix_T, ckpt,
        item_info, item_cost, tile_order);
  else
    launch_kernel(k_raster_fwd<kFwdPix, kFwdWx, kBatch>, num_tiles, kTilePixels / kFwdPix, 0, st,
        splats, ids, ranges, tile_items, n, bg, width, height, tiles_x, image, img_copy, pix_T, ckpt,
        item_info, item_cost, tile_order);
}

template <int BATCH>
static void raster_bwd_batch(const Splat* splats, const int* ids, const int* ranges, int n, int width,
                             int height, int tiles_x, const float* grad_image, const float* img,
                             const float4* ckpt, const int* item_info, const int* item_cost, int* item_order,
                             Scalars* sc, SplatGrad* grads, cudaStream_t st) {
  static int ctas = 0;  // per process: the GPUs of one node have the same SM count
  if (ctas == 0)
    ctas = persistent_ctas((const void*)k_raster_bwd<kBwdPix, kBwdWx, BATCH>, kTilePixels / kBwdPix);
  cudaMemsetAsync(&sc->item_counter, 0, sizeof(unsigned), st);
  {
    GS_TIMED("item_order", st);
    launch_kernel(k_item_order, 1, 1024, 0, st, item_cost, sc, 4 * ctas, item_order);
  }
  GS_TIMED("raster_bwd", st);
  launch_kernel(k_raster_bwd<kBwdPix, kBwdWx, BATCH>, ctas, kTilePixels / kBwdPix, 0, st,
      splats, ids, ranges, n, width, height, tiles_x, grad_image, img, ckpt, item_info, item_order, sc, grads);
}

void launch_raster_bwd(const Splat* splats, const int* ids, const int* ranges, int n, int width,
                       int height, int tiles_x, int num_tiles, const float* grad_image,
                       const float* img, const float4* ckpt, const int* item_info, const int* item_cost,
                       int* item_order, Scalars* sc, SplatGrad* grads, const float* pix_T, float* grad_bg,
                       cudaStream_t st) {
  if (num_tiles == 0) return;
  if (compositor_batch(num_tiles) == kBatchSmall)
    raster_bwd_batch<kBatchSmall>(splats, ids, ranges, n, width, height, tiles_x, grad_image, img, ckpt, item_info,
                                  item_cost, item_order, sc, grads, st);
  else
    raster_bwd_batch<kBatch>(splats, ids, ranges, n, width, height, tiles_x, grad_image, img, ckpt, item_info,
                             item_cost, item_order, sc, grads, st);
  if (grad_bg) {
    GS_TIMED("grad_bg", st);
    launch_kernel(k_grad_bg, device_sms(), 256, 0, st, pix_T, grad_image, width * height, grad_bg);
  }
}

}  // namespace gs
