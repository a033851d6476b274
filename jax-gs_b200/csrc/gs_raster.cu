// Stages 3 and 4: the front-to-back compositor and its backward.
//
// One CTA per 16x16 tile, one thread per pixel. The tile's sorted Gaussians
// are staged through shared memory 256 records at a time (three 16-byte loads
// per record); every pixel of the tile then walks the staged batch. The
// compositing rule is the reference's (rasterizer.py:202-215,
// rasterizer_tpu.py:308-336): a Gaussian is applied while T > 1e-4 (tested
// before the splat), only where power > -10, with alpha = min(0.99,
// exp(power) sigmoid(o)); at most MAX_TILE_INTERACTIONS Gaussians per tile;
// out = C + T bg. A pixel stops at the first splat that leaves T <= 1e-4; the
// CTA stops when every pixel has stopped (reference scans run to the end but
// contribute nothing after that point).
#include "gs_kernels.cuh"

namespace gs {

__global__ void __launch_bounds__(kTilePixels)
k_raster_fwd(const Splat* __restrict__ splats, const int* __restrict__ ids,
             const int* __restrict__ ranges, int n, const float* __restrict__ bg, int width,
             int height, int tiles_x, float* __restrict__ image, float* __restrict__ pix_T,
             int* __restrict__ pix_last, GsExtras* __restrict__ extras) {
  __shared__ float4 s_a[kTilePixels];
  __shared__ float4 s_b[kTilePixels];
  __shared__ float s_c[kTilePixels];
  const int tile = blockIdx.x;
  const int tx = tile % tiles_x, ty = tile / tiles_x;
  const int tid = threadIdx.x;
  const int px = tx * kTile + (tid & (kTile - 1));
  const int py = ty * kTile + (tid / kTile);
  const bool inside = (px < width) && (py < height);
  const float fpx = (float)px + 0.5f, fpy = (float)py + 0.5f;
  const int start = ranges[tile];
  const int full = ranges[tile + 1] - start;
  const int count = min(full, kMaxTileInteractions);
  if (extras != nullptr && tid == 0) {
    // renderer.py:61,76-77,84-88 tile-count statistics.
    atomicMax(&extras->max_interactions_per_tile, full);
    if (full > kBlockSize) {
      atomicAdd(&extras->overflow_tiles, 1);
      atomicAdd(&extras->overflow_interactions, full - kBlockSize);
    }
    if (full > kMaxTileInteractions) {
      atomicAdd(&extras->truncated_tiles, 1);
      atomicAdd(&extras->truncated_interactions, full - kMaxTileInteractions);
    }
  }
  float T = 1.f, C0 = 0.f, C1 = 0.f, C2 = 0.f;
  int last = -1;
  bool done = !inside;
  for (int b0 = 0; b0 < count; b0 += kTilePixels) {
    if (__syncthreads_count(!done) == 0) break;
    const int j = b0 + tid;
    if (j < count) {
      int g = ids[start + j];
      g = min(max(g, 0), n - 1);
      const Splat* sp = splats + g;
      s_a[tid] = __ldg(&sp->a);
      s_b[tid] = __ldg(&sp->b);
      s_c[tid] = __ldg(&sp->c.x);
    }
    __syncthreads();
    const int nb = min(kTilePixels, count - b0);
    if (!done) {
      for (int k = 0; k < nb; ++k) {
        const float4 A = s_a[k];
        const float4 B = s_b[k];
        const float dx = fpx - A.x, dy = fpy - A.y;
        const float power = -0.5f * (dx * dx * A.z + dx * dy * A.w + dy * dy * B.x);
        if (power > -10.f) {
          const float alpha = fminf(0.99f, __expf(power) * B.y);
          const float w = alpha * T;
          C0 += w * B.z;
          C1 += w * B.w;
          C2 += w * s_c[k];
          T = T * (1.f - alpha);
          last = b0 + k;
          if (T <= 1e-4f) {
            done = true;
            break;
          }
        }
      }
    }
  }
  if (inside) {
    const int pix = py * width + px;
    float b0 = 0.f, b1 = 0.f, b2 = 0.f;
    if (bg) { b0 = bg[0]; b1 = bg[1]; b2 = bg[2]; }
    image[3 * pix] = C0 + T * b0;
    image[3 * pix + 1] = C1 + T * b1;
    image[3 * pix + 2] = C2 + T * b2;
    if (pix_T) pix_T[pix] = T;
    if (pix_last) pix_last[pix] = last;
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

// Backward: replays each pixel's contributors back to front, reconstructing
// the transmittance before each splat by division (alpha <= 0.99), and
// reduces the per-Gaussian gradient over the tile (warp shuffles, then
// shared-memory atomics) before one set of global vector atomics per
// (Gaussian, tile) pair.
//
// Per pixel with colour gradient G, splats j = L..0 that contributed:
//   dL/dc_j     = alpha_j T_j G
//   dL/dalpha_j = T_j (c_j . G) - S_{j+1} / (1 - alpha_j)
// where S_{j+1} = sum_{k>j} alpha_k T_k (c_k . G) + T_final (bg . G).
__global__ void __launch_bounds__(kTilePixels)
k_raster_bwd(const Splat* __restrict__ splats, const int* __restrict__ ids,
             const int* __restrict__ ranges, int n, const float* __restrict__ bg, int width,
             int height, int tiles_x, const float* __restrict__ grad_image,
             const float* __restrict__ pix_T, const int* __restrict__ pix_last,
             SplatGrad* __restrict__ grads, float* __restrict__ grad_bg) {
  __shared__ float4 s_a[kTilePixels];
  __shared__ float4 s_b[kTilePixels];
  __shared__ float s_c[kTilePixels];
  __shared__ int s_gid[kTilePixels];
  __shared__ float s_acc[9][kTilePixels];
  __shared__ int s_maxlast;
  __shared__ float s_bg[3][8];
  const int tile = blockIdx.x;
  const int tx = tile % tiles_x, ty = tile / tiles_x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int px = tx * kTile + (tid & (kTile - 1));
  const int py = ty * kTile + (tid / kTile);
  const bool inside = (px < width) && (py < height);
  const float fpx = (float)px + 0.5f, fpy = (float)py + 0.5f;
  const int start = ranges[tile];
  float G0 = 0.f, G1 = 0.f, G2 = 0.f, T = 1.f;
  int last = -1;
  if (inside) {
    const int pix = py * width + px;
    G0 = grad_image[3 * pix];
    G1 = grad_image[3 * pix + 1];
    G2 = grad_image[3 * pix + 2];
    T = pix_T[pix];
    last = pix_last[pix];
  }
  float bg0 = 0.f, bg1 = 0.f, bg2 = 0.f;
  if (bg) { bg0 = bg[0]; bg1 = bg[1]; bg2 = bg[2]; }
  float s = T * (bg0 * G0 + bg1 * G1 + bg2 * G2);
  if (grad_bg) {
    float v0 = inside ? T * G0 : 0.f, v1 = inside ? T * G1 : 0.f, v2 = inside ? T * G2 : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      v0 += __shfl_down_sync(0xffffffffu, v0, o);
      v1 += __shfl_down_sync(0xffffffffu, v1, o);
      v2 += __shfl_down_sync(0xffffffffu, v2, o);
    }
    if (lane == 0) { s_bg[0][warp] = v0; s_bg[1][warp] = v1; s_bg[2][warp] = v2; }
  }
  if (tid == 0) s_maxlast = -1;
#pragma unroll
  for (int k = 0; k < 9; ++k) s_acc[k][tid] = 0.f;
  __syncthreads();
  if (grad_bg && tid < 3) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += s_bg[tid][w];
    atomicAdd(grad_bg + tid, t);
  }
  {
    int m = last;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_down_sync(0xffffffffu, m, o));
    if (lane == 0) atomicMax(&s_maxlast, m);
  }
  __syncthreads();
  const int maxlast = s_maxlast;
  for (int bend = maxlast + 1; bend > 0; bend -= kTilePixels) {
    const int b0 = max(0, bend - kTilePixels);
    const int nb = bend - b0;
    __syncthreads();
    if (tid < nb) {
      int g = ids[start + b0 + tid];
      g = min(max(g, 0), n - 1);
      const Splat* sp = splats + g;
      s_gid[tid] = g;
      s_a[tid] = __ldg(&sp->a);
      s_b[tid] = __ldg(&sp->b);
      s_c[tid] = __ldg(&sp->c.x);
    }
    __syncthreads();
    for (int k = nb - 1; k >= 0; --k) {
      const int j = b0 + k;
      float v[9];
#pragma unroll
      for (int q = 0; q < 9; ++q) v[q] = 0.f;
      bool contrib = false;
      if (j <= last) {
        const float4 A = s_a[k];
        const float4 B = s_b[k];
        const float cb = s_c[k];
        const float dx = fpx - A.x, dy = fpy - A.y;
        const float power = -0.5f * (dx * dx * A.z + dx * dy * A.w + dy * dy * B.x);
        if (power > -10.f) {
          const float e = __expf(power);
          const float ea = e * B.y;
          const float alpha = fminf(0.99f, ea);
          const float inv_oma = 1.f / (1.f - alpha);
          T = T * inv_oma;
          const float cG = B.z * G0 + B.w * G1 + cb * G2;
          const float w = alpha * T;
          v[6] = w * G0;
          v[7] = w * G1;
          v[8] = w * G2;
          const float dalpha = T * cG - s * inv_oma;
          s += w * cG;
          // jnp.minimum(0.99, ea): gradient 1 below, 1/2 at the tie, 0 above.
          const float dea = (ea < 0.99f) ? dalpha : ((ea == 0.99f) ? 0.5f * dalpha : 0.f);
          const float dpow = dea * ea;
          v[5] = dea * e;
          v[2] = dpow * (-0.5f * dx * dx);
          v[3] = dpow * (-0.5f * dx * dy);
          v[4] = dpow * (-0.5f * dy * dy);
          v[0] = dpow * (dx * A.z + 0.5f * dy * A.w);
          v[1] = dpow * (dy * B.x + 0.5f * dx * A.w);
          contrib = true;
        }
      }
      if (__any_sync(0xffffffffu, contrib)) {
        warp_sum9(v, lane);
        if ((lane & 3) == 0) atomicAdd(&s_acc[lane >> 2][k], v[0]);
        if (lane == 1) atomicAdd(&s_acc[8][k], v[8]);
      }
    }
    __syncthreads();
    if (tid < nb) {
      float a0 = s_acc[0][tid], a1 = s_acc[1][tid], a2 = s_acc[2][tid], a3 = s_acc[3][tid],
            a4 = s_acc[4][tid], a5 = s_acc[5][tid], a6 = s_acc[6][tid], a7 = s_acc[7][tid],
            a8 = s_acc[8][tid];
#pragma unroll
      for (int q = 0; q < 9; ++q) s_acc[q][tid] = 0.f;
      if ((a0 != 0.f) | (a1 != 0.f) | (a2 != 0.f) | (a3 != 0.f) | (a4 != 0.f) | (a5 != 0.f) |
          (a6 != 0.f) | (a7 != 0.f) | (a8 != 0.f)) {
        SplatGrad* gp = grads + s_gid[tid];
        atomicAdd(&gp->a, make_float4(a0, a1, a2, a3));
        atomicAdd(&gp->b, make_float4(a4, a5, a6, a7));
        atomicAdd(&gp->c.x, a8);
      }
    }
  }
}

void launch_raster_fwd(const Splat* splats, const int* ids, const int* ranges, int n,
                       const float* bg, int width, int height, int tiles_x, int num_tiles,
                       float* image, float* pix_T, int* pix_last, GsExtras* extras,
                       cudaStream_t st) {
  if (num_tiles == 0) return;
  GS_TIMED("raster_fwd", st);
  k_raster_fwd<<<num_tiles, kTilePixels, 0, st>>>(splats, ids, ranges, n, bg, width, height, tiles_x,
                                                  image, pix_T, pix_last, extras);
}

void launch_raster_bwd(const Splat* splats, const int* ids, const int* ranges, int n,
                       const float* bg, int width, int height, int tiles_x, int num_tiles,
                       const float* grad_image, const float* pix_T, const int* pix_last,
                       SplatGrad* grads, float* grad_bg, cudaStream_t st) {
  if (num_tiles == 0) return;
  GS_TIMED("raster_bwd", st);
  k_raster_bwd<<<num_tiles, kTilePixels, 0, st>>>(splats, ids, ranges, n, bg, width, height, tiles_x,
                                                  grad_image, pix_T, pix_last, grads, grad_bg);
}

}  // namespace gs
