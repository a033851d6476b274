// Shared definitions of the sm_100a Gaussian-splat renderer kernels.
//
// Data layout in HBM (all per-view scratch lives in the caller's workspace):
//   Splat        48 B per Gaussian: the compositor's record (means2D, conic,
//                sigmoid opacity, RGB) -- three 16-byte vectors so a tile
//                stages it with three 128-bit loads.
//   BinInfo      8 B per Gaussian: tile rectangle origin, span and 13-bit
//                depth key (what the key-emission kernel needs).
//   keys / ids   int32 (tile << 13 | depth) keys and Gaussian ids, double
//                buffered for the LSD radix sort.
//   tile ranges  int32 (T+1), searchsorted boundaries.
//   pixel state  final transmittance and index of the last contributor.
//   SplatGrad    48 B per Gaussian gradient accumulator of the compositor.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gsb200.h"

namespace gs {

constexpr int kTile = GS_TILE_SIZE;                       // rasterizer.py:6
constexpr int kOffset = GS_OFFSET_SIZE;                   // rasterizer.py:7
constexpr int kBlockSize = GS_BLOCK_SIZE;                 // rasterizer.py:8
constexpr int kMaxTileInteractions = GS_MAX_TILE_INTERACTIONS;  // rasterizer.py:10
constexpr int kDepthBits = GS_DEPTH_BITS;                 // rasterizer.py:84
constexpr int kTilePixels = kTile * kTile;                // 256 threads per tile CTA

// Radix sort geometry: 8-bit digits, one kernel per digit pass over tiles of
// kSortTileKeys keys (256 threads x kSortItems), at most kMaxSortPasses passes
// (32-bit keys).
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTileKeys = kSortThreads * kSortItems;  // 2048
constexpr int kMaxSortPasses = 4;
// Key tile of the direct path's single-pass-per-digit sort (256 threads x
// kOsItems keys). 8 measured faster than 4 at config 2 (50.9 vs 56.5 us for
// the three passes: the shorter tiles' look-back chain is twice as long).
#ifndef GS_OS_ITEMS
#define GS_OS_ITEMS 8
#endif
constexpr int kOsItems = GS_OS_ITEMS;
constexpr int kOsTileKeys = kSortThreads * kOsItems;
// Gaussian count from which the pairs are sorted after a depth pre-sort of
// the Gaussians (two M-key passes fewer) instead of directly on 13 + log2(T)
// bits: below it the extra launches cost more than the passes they save.
constexpr int kPresortMinN = 1 << 18;

// Spherical-harmonic constants, jax_gs/renderer/sh.py:6-23.
constexpr float kC0 = 0.28209479177387814f;
constexpr float kC1 = 0.4886025119029199f;
constexpr float kC2_0 = 1.0925484305920792f;
constexpr float kC2_1 = -1.0925484305920792f;
constexpr float kC2_2 = 0.31539156525252005f;
constexpr float kC2_3 = -1.0925484305920792f;
constexpr float kC2_4 = 0.5462742152960396f;
constexpr float kC3_0 = -0.5900435899266435f;
constexpr float kC3_1 = 2.890611442640554f;
constexpr float kC3_2 = -0.4570457994644658f;
constexpr float kC3_3 = 0.3731763325901154f;
constexpr float kC3_4 = -0.4570457994644658f;
constexpr float kC3_5 = 1.445305721320277f;
constexpr float kC3_6 = -0.5900435899266435f;

struct __align__(16) Splat {
  float4 a;  // means2D x, y, ha = -inv[0,0] / 2, hb = -inv[0,1]
  float4 b;  // hc = -inv[1,1] / 2, sigmoid(opacity), r, g
  float4 c;  // b, half-width and half-height of the power > -10 region (bbox_halfext), unused
};

// Half-extents of the region where a splat's exponent exceeds -10
// (x^T Q x < 20 for the clamped inverse Q = adj(cov) / max(det, 1e-6)),
// widened by 1 % + 0.5 px so that a float evaluation of the exponent outside
// them is always <= -10. Infinite when the form is not positive definite.
__device__ __forceinline__ float2 bbox_halfext(float c00, float c01, float c11) {
  const float det = c00 * c11 - c01 * c01;
  if (!(det > 0.f) || !(c00 > 0.f) || !(c11 > 0.f)) return make_float2(INFINITY, INFINITY);
  const float s = 20.f * (fmaxf(det, 1e-6f) / det);
  return make_float2(sqrtf(s * c00) * 1.01f + 0.5f, sqrtf(s * c11) * 1.01f + 0.5f);
}

// Whether the exponent power(dx, dy) = ha dx^2 + hb dx dy + hc dy^2 of a
// splat at (mx, my) (dx, dy = pixel centre - mean) can exceed -10 at a pixel
// centre in [x0, x1] x [y0, y1]. The maximum over the continuous rectangle
// (an upper bound of the centres') is at the mean when it lies inside,
// otherwise on an edge facing the mean, where power is a parabola in the
// free coordinate. It is compared with -10 minus a margin that covers the
// float evaluation of this test and of the compositor's exponent (rounding
// relative to the terms' magnitude, and of dx, dy relative to the slope).
// Forms that are not negative definite, non-finite values and NaN keep the
// splat, so a splat is only dropped where the compositor's alpha is 0.
__device__ __forceinline__ bool splat_meets_rect(float mx, float my, float ha, float hb, float hc, float x0,
                                                 float x1, float y0, float y1) {
  if (!(ha < 0.f) || !(hc < 0.f) || !(4.f * ha * hc > hb * hb)) return true;
  if (!(fabsf(mx) < 1e30f) || !(fabsf(my) < 1e30f)) return true;
  const float lx = x0 - mx, ux = x1 - mx, ly = y0 - my, uy = y1 - my;
  const float ex = fminf(fmaxf(0.f, lx), ux), ey = fminf(fmaxf(0.f, ly), uy);
  if (ex == 0.f && ey == 0.f) return true;  // the mean is inside
  float best = -INFINITY;
  if (ex != 0.f) {  // the vertical edge dx = ex
    const float dy = fminf(fmaxf(__fdividef(-hb * ex, 2.f * hc), ly), uy);
    best = fmaxf(best, (ha * ex + hb * dy) * ex + hc * dy * dy);
  }
  if (ey != 0.f) {  // the horizontal edge dy = ey
    const float dx = fminf(fmaxf(__fdividef(-hb * ey, 2.f * ha), lx), ux);
    best = fmaxf(best, (ha * dx + hb * ey) * dx + hc * ey * ey);
  }
  const float DX = fmaxf(fabsf(lx), fabsf(ux)), DY = fmaxf(fabsf(ly), fabsf(uy));
  const float mag = (fabsf(hb) * DY - ha * DX) * DX - hc * DY * DY;
  const float slope = fabsf(hb) * (DX + DY) - 2.f * (ha * DX + hc * DY);
  return !(best <= -10.05f - 1e-4f * mag - 1e-3f * slope);
}

struct __align__(16) SplatGrad {
  float4 a;  // d mx, d my, d a, d b2
  float4 b;  // d c, d sigmoid(opacity), d r, d g
  float4 c;  // d b, 0, 0, 0
};

// Rounded IEEE single-precision arithmetic with FMA contraction forbidden.
// The projection path uses these so that means2D, radii and depth -- which
// decide the integer tile keys through floor() and ceil() -- are bitwise the
// same as a CPU evaluation of the same expressions in the same order.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float sqrt_rn(float a) { return __fsqrt_rn(a); }
// exp rounded once from a double-precision evaluation: the correctly rounded
// float result except in cases within one double ulp of a float midpoint.
__device__ __forceinline__ float exp_cr(float a) { return (float)exp((double)a); }
// jnp.maximum / jnp.minimum propagate NaN (fmaxf/fminf would drop it).
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a != a) ? a : ((a > b) ? a : b);
}
__device__ __forceinline__ float nan_min(float a, float b) {
  return (a != a) ? a : ((a < b) ? a : b);
}

// Per-view camera scalars.
struct Cam {
  float W[12];  // rows 0..2 of W2C (row-major 3x4)
  float fx, fy, cx, cy;
  int width, height;
  int tiles_x, tiles_y;
};

// Result of projecting one Gaussian (projection.py:21-79).
struct Proj {
  float x, y, z;        // camera-space mean
  float u, v;           // means2D
  float c00, c01, c11;  // cov2D entries [0,0], [0,1], [1,1] (0.3 added on diagonal)
  float radius;         // ceil(3 sqrt(lambda_max))
  // Intermediates the backward pass reuses.
  float R[9];           // rotation from the normalised quaternion
  float s[3];           // exp(scales)
  float qn[4];          // normalised quaternion
  float qnorm;          // |q|
  float Sig[6];         // Sigma 00 01 02 11 12 22
  float Mj[6];          // J @ W_rot, rows 0 and 1
  float inv_z;          // 1 / max(z, 0.01)
};

// get_covariance_3d (jax_gs/core/gaussians.py:58-93) and project_gaussians
// (jax_gs/renderer/projection.py:21-79), evaluated in a fixed order: matrix
// products are summed in increasing k, the zero entries of J are skipped
// (adding a signed zero to a non-zero value is exact).
__device__ __forceinline__ void project_one(const float m[3], const float sc[3], const float q[4],
                                            const Cam& cam, Proj& p) {
  const float* W = cam.W;
  // projection.py:133-134  means_cam = [m, 1] @ W2C^T
  p.x = add_rn(add_rn(add_rn(mul_rn(W[0], m[0]), mul_rn(W[1], m[1])), mul_rn(W[2], m[2])), W[3]);
  p.y = add_rn(add_rn(add_rn(mul_rn(W[4], m[0]), mul_rn(W[5], m[1])), mul_rn(W[6], m[2])), W[7]);
  p.z = add_rn(add_rn(add_rn(mul_rn(W[8], m[0]), mul_rn(W[9], m[1])), mul_rn(W[10], m[2])), W[11]);

  // gaussians.py:70  q / |q|
  float n2 = add_rn(add_rn(add_rn(mul_rn(q[0], q[0]), mul_rn(q[1], q[1])), mul_rn(q[2], q[2])),
                    mul_rn(q[3], q[3]));
  p.qnorm = sqrt_rn(n2);
  float r = div_rn(q[0], p.qnorm), x = div_rn(q[1], p.qnorm), y = div_rn(q[2], p.qnorm),
        z = div_rn(q[3], p.qnorm);
  p.qn[0] = r; p.qn[1] = x; p.qn[2] = y; p.qn[3] = z;
  // gaussians.py:78-82
  float xx2 = mul_rn(2.f, mul_rn(x, x)), yy2 = mul_rn(2.f, mul_rn(y, y)),
        zz2 = mul_rn(2.f, mul_rn(z, z));
  float x2 = mul_rn(2.f, x), r2 = mul_rn(2.f, r), y2 = mul_rn(2.f, y);
  p.R[0] = sub_rn(sub_rn(1.f, yy2), zz2);
  p.R[1] = sub_rn(mul_rn(x2, y), mul_rn(r2, z));
  p.R[2] = add_rn(mul_rn(x2, z), mul_rn(r2, y));
  p.R[3] = add_rn(mul_rn(x2, y), mul_rn(r2, z));
  p.R[4] = sub_rn(sub_rn(1.f, xx2), zz2);
  p.R[5] = sub_rn(mul_rn(y2, z), mul_rn(r2, x));
  p.R[6] = sub_rn(mul_rn(x2, z), mul_rn(r2, y));
  p.R[7] = add_rn(mul_rn(y2, z), mul_rn(r2, x));
  p.R[8] = sub_rn(sub_rn(1.f, xx2), yy2);
  // gaussians.py:85-91  M = R * exp(s);  Sigma = M M^T
  p.s[0] = exp_cr(sc[0]); p.s[1] = exp_cr(sc[1]); p.s[2] = exp_cr(sc[2]);
  float M[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) M[i * 3 + j] = mul_rn(p.R[i * 3 + j], p.s[j]);
  float S[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      S[i * 3 + j] = add_rn(add_rn(mul_rn(M[i * 3 + 0], M[j * 3 + 0]), mul_rn(M[i * 3 + 1], M[j * 3 + 1])),
                            mul_rn(M[i * 3 + 2], M[j * 3 + 2]));
  p.Sig[0] = S[0]; p.Sig[1] = S[1]; p.Sig[2] = S[2]; p.Sig[3] = S[4]; p.Sig[4] = S[5]; p.Sig[5] = S[8];

  // projection.py:150-164  J (2x3), M = J W_rot, cov2D = M Sigma M^T
  float sz = nan_max(p.z, 0.01f);
  p.inv_z = div_rn(1.f, sz);
  float inv_z2 = mul_rn(p.inv_z, p.inv_z);
  float J00 = mul_rn(cam.fx, p.inv_z);
  float J02 = mul_rn(mul_rn(-cam.fx, p.x), inv_z2);
  float J11 = mul_rn(cam.fy, p.inv_z);
  float J12 = mul_rn(mul_rn(-cam.fy, p.y), inv_z2);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    p.Mj[k] = add_rn(mul_rn(J00, W[0 * 4 + k]), mul_rn(J02, W[2 * 4 + k]));
    p.Mj[3 + k] = add_rn(mul_rn(J11, W[1 * 4 + k]), mul_rn(J12, W[2 * 4 + k]));
  }
  float T[6];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      T[i * 3 + k] = add_rn(add_rn(mul_rn(p.Mj[i * 3 + 0], S[0 * 3 + k]), mul_rn(p.Mj[i * 3 + 1], S[1 * 3 + k])),
                            mul_rn(p.Mj[i * 3 + 2], S[2 * 3 + k]));
  float cov00 = add_rn(add_rn(mul_rn(T[0], p.Mj[0]), mul_rn(T[1], p.Mj[1])), mul_rn(T[2], p.Mj[2]));
  float cov01 = add_rn(add_rn(mul_rn(T[0], p.Mj[3]), mul_rn(T[1], p.Mj[4])), mul_rn(T[2], p.Mj[5]));
  float cov11 = add_rn(add_rn(mul_rn(T[3], p.Mj[3]), mul_rn(T[4], p.Mj[4])), mul_rn(T[5], p.Mj[5]));
  // projection.py:168-169  + 0.3 I
  p.c00 = add_rn(cov00, 0.3f);
  p.c01 = cov01;
  p.c11 = add_rn(cov11, 0.3f);
  // projection.py:172-175
  p.u = add_rn(div_rn(mul_rn(cam.fx, p.x), p.z), cam.cx);
  p.v = add_rn(div_rn(mul_rn(cam.fy, p.y), p.z), cam.cy);
  // projection.py:178-184
  float det = sub_rn(mul_rn(p.c00, p.c11), mul_rn(p.c01, p.c01));
  float trace = add_rn(p.c00, p.c11);
  float mid = div_rn(trace, 2.f);
  float term = sqrt_rn(nan_max(sub_rn(mul_rn(mid, mid), det), 0.f));
  float lam = add_rn(mid, term);
  p.radius = ceilf(mul_rn(3.f, sqrt_rn(lam)));
}

// Tile rectangle of a projected splat (rasterizer.py:36-51, renderer.py:63-75).
struct Rect {
  int tx0, ty0, tx1, ty1;  // inclusive tile bounds before the 16-tile span cap
  bool on_screen;
};

__device__ __forceinline__ Rect tile_rect(float u, float v, float r, int width, int height) {
  Rect t;
  float umr = sub_rn(u, r), upr = add_rn(u, r), vmr = sub_rn(v, r), vpr = add_rn(v, r);
  t.on_screen = (upr > 0.f) && (umr < (float)width) && (vpr > 0.f) && (vmr < (float)height);
  if (!t.on_screen) {
    t.tx0 = t.ty0 = 0; t.tx1 = t.ty1 = -1;
    return t;
  }
  float wm1 = (float)(width - 1), hm1 = (float)(height - 1);
  float min_x = fminf(fmaxf(umr, 0.f), wm1), max_x = fminf(fmaxf(upr, 0.f), wm1);
  float min_y = fminf(fmaxf(vmr, 0.f), hm1), max_y = fminf(fmaxf(vpr, 0.f), hm1);
  // x // 16 for x >= 0: the division by a power of two is exact.
  t.tx0 = (int)floorf(min_x * (1.f / kTile));
  t.tx1 = (int)floorf(max_x * (1.f / kTile));
  t.ty0 = (int)floorf(min_y * (1.f / kTile));
  t.ty1 = (int)floorf(max_y * (1.f / kTile));
  return t;
}

// 13-bit depth key: bitcast(z) >> 18 (arithmetic), rasterizer.py:93-94.
__device__ __forceinline__ int depth_key(float z) { return __float_as_int(z) >> (31 - kDepthBits); }

// Packed emission info of one Gaussian: x = tx0 | ty0 << 16,
// y = nx | ny << 5 | dq << 10 (nx, ny in 0..16 after the span cap).
__device__ __forceinline__ int2 pack_bin(int tx0, int ty0, int nx, int ny, int dq) {
  return make_int2((tx0 & 0xFFFF) | (ty0 << 16), nx | (ny << 5) | ((dq & 0x1FFF) << 10));
}

// Spherical-harmonic colour, jax_gs/renderer/sh.py:25-74; sh points at the
// (K,3) coefficients of one Gaussian.
// The first 3 (deg + 1)^2 coefficients of one Gaussian's SH row (sh_k
// coefficients x 3 channels) into registers. With 16-byte aligned rows
// (sh_k a multiple of 4 and an aligned base) as float4 loads: a warp's
// thread-per-Gaussian loads then touch a quarter of the sectors that
// scalar loads of the 192-byte rows would.
__device__ __forceinline__ void load_sh_row(const float* __restrict__ row, int sh_k, int deg, float v[48]) {
  const int nf = 3 * (deg + 1) * (deg + 1);
  if ((sh_k & 3) == 0 && (((uintptr_t)row) & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll
    for (int k = 0; k < 12; ++k) {
      if (4 * k < nf) {  // (4k + 3) < 3 sh_k: the row holds at least 4 ceil(nf / 4) floats
        const float4 t = __ldg(r4 + k);
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
      } else {
        v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = 0.f;
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < 48; ++k) v[k] = (k < nf) ? __ldg(row + k) : 0.f;
  }
}

__device__ __forceinline__ void eval_sh_one(int deg, const float* __restrict__ sh, float dx, float dy,
                                            float dz, float out[3]) {
#pragma unroll
  for (int c = 0; c < 3; ++c) out[c] = kC0 * sh[c];
  if (deg > 0) {
    float x = dx, y = dy, z = dz;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      out[c] = out[c] - kC1 * y * sh[3 + c] + kC1 * z * sh[6 + c] - kC1 * x * sh[9 + c];
    if (deg > 1) {
      float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        out[c] = out[c] + kC2_0 * xy * sh[12 + c] + kC2_1 * yz * sh[15 + c] +
                 kC2_2 * (2.f * zz - xx - yy) * sh[18 + c] + kC2_3 * xz * sh[21 + c] +
                 kC2_4 * (xx - yy) * sh[24 + c];
      if (deg > 2) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
          out[c] = out[c] + kC3_0 * y * (3.f * xx - yy) * sh[27 + c] + kC3_1 * xy * z * sh[30 + c] +
                   kC3_2 * y * (4.f * zz - xx - yy) * sh[33 + c] +
                   kC3_3 * z * (2.f * zz - 3.f * xx - 3.f * yy) * sh[36 + c] +
                   kC3_4 * x * (4.f * zz - xx - yy) * sh[39 + c] + kC3_5 * z * (xx - yy) * sh[42 + c] +
                   kC3_6 * x * (xx - 3.f * yy) * sh[45 + c];
      }
    }
  }
}

__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

// Workspace layout shared by every entry point (host and device agree on it).
struct Layout {
  size_t splats, bins, block_counts, block_offsets, vis_offsets, keys0, ids0, keys1, ids1, hist, status0,
      status1, tcounts, dcounts, dkeys0, dids0, dkeys1, dids1, sorted_counts, emit_offsets, ranges,
      tile_items, tile_order, item_info, item_cost, item_order, ckpt, pix_T, img, grads, scalars, loss_partials,
      total;
  int n, width, height, tiles_x, tiles_y, num_tiles, n_blocks;
  int64_t capacity;
  int64_t max_items;  // upper bound of (tile, 256-splat batch) work items
  int sort_tiles, depth_tiles;  // 2048-key tiles of the tile sort (capacity) and depth sort (n)
  bool presort;                 // depth pre-sort path (large n) or direct 13+log2(T)-bit sort
};

// Device-side scalars kept in the workspace.
struct Scalars {
  int32_t n_emit;        // min(total pairs, capacity): keys actually written
  int32_t n_total;       // total pairs (may exceed capacity)
  uint32_t loss_ticket;  // last-block-done counter of the loss reduction
  int32_t n_items;       // (tile, batch) work items of the compositor backward
  uint32_t item_counter;  // next work item of the persistent backward grid
  int32_t n_vis;          // Gaussians with at least one pair
  // zeroed together before every single-pass radix sort:
  int32_t sort_timeouts;   // look-back waits that gave up (0 unless a GPU stalls)
  uint32_t sweep_tile[4];  // next key tile of each single-pass radix pass
  int32_t item_sorted;  // 1: the backward takes items through the longest-first order
  int32_t pad[4];
};

// A compositor work item: one tile and one batch of sorted splats -- kBatch
// (256) of them, or kBatchSmall (128) on images of at most kSmallImageTiles
// tiles, where the backward's items are few for the GPU and shorter ones
// shorten the persistent grid's tail. (The 2DGS compositor uses kBatch.)
constexpr int kBatch = 256;
#ifndef GS_BATCH_SMALL
#define GS_BATCH_SMALL 128
#endif
constexpr int kBatchSmall = GS_BATCH_SMALL;
#ifndef GS_SMALL_IMAGE_TILES
#define GS_SMALL_IMAGE_TILES 2048
#endif
constexpr int kSmallImageTiles = GS_SMALL_IMAGE_TILES;
static_assert(kBatchSmall >= 64 && kBatchSmall <= kBatch && kBatch % kBatchSmall == 0, "compositor batch");
__host__ __device__ inline int compositor_batch(int num_tiles) {
  return num_tiles <= kSmallImageTiles ? kBatchSmall : kBatch;
}
// item_info word: tile (18 bits) | batch index (6 bits: up to 4096 / 64
// batches) << 18 | skipped << 24
__device__ __forceinline__ int pack_item(int tile, int batch, bool skip) {
  return tile | (batch << 18) | ((skip ? 1 : 0) << 24);
}
__device__ __forceinline__ bool item_skipped(int info) { return (info >> 24) != 0; }
__device__ __forceinline__ int item_tile(int info) { return info & 0x3FFFF; }
__device__ __forceinline__ int item_batch(int info) { return (info >> 18) & 63; }

// Gaussian exponent of one splat at a pixel, power = -0.5 (a dx^2 + b2 dx dy
// + c dy^2) = ha dx^2 + hb dx dy + hc dy^2 with the record's halved conic
// (ha, hb, hc) = -(a, b2, c) / 2, as q0 + dy (q1 + dy hc) from the per-column
// terms q0 = ha dx^2 and q1 = hb dx (a thread's pixels share dx). Written with
// explicit fused operations so that the forward compositor and the backward
// replay evaluate bit-identical values (the backward re-derives the forward's
// transmittance and its T > 1e-4 / power > -10 decisions).
__device__ __forceinline__ float splat_q0(float dx, float ha) { return __fmul_rn(__fmul_rn(dx, dx), ha); }
__device__ __forceinline__ float splat_q1(float dx, float hb) { return __fmul_rn(dx, hb); }
__device__ __forceinline__ float splat_power(float dy, float q0, float q1, float hc) {
  return __fmaf_rn(dy, __fmaf_rn(dy, hc, q1), q0);
}

// Deterministic sum of per-thread doubles over a 256-thread block: shuffle
// tree, then the 8 warp totals in order. Result valid in thread 0; every
// thread must call it (two barriers). s_w: 8 doubles of shared memory.
__device__ __forceinline__ double block_sum_d256(double v, double* s_w) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < 8; ++w) t += s_w[w];
  __syncthreads();
  return t;
}

// Shared per-Gaussian helpers of the 3DGS and 2DGS preprocess kernels.
__device__ __forceinline__ void load_cam_rows(const float* __restrict__ w2c, Cam& cam) {
#pragma unroll
  for (int k = 0; k < 12; ++k) cam.W[k] = __ldg(w2c + k);
}

// Sums over a 256-thread block of three ints at once: one warp reduction
// instruction per value, one pass through shared memory and one barrier (the
// kernel's last use of s_red). The totals are valid in thread 0.
__device__ __forceinline__ int3 block_sum3_256(int a, int b, int c, int (*s_red)[3]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = __reduce_add_sync(0xffffffffu, a);
  b = __reduce_add_sync(0xffffffffu, b);
  c = __reduce_add_sync(0xffffffffu, c);
  if (lane == 0) {
    s_red[warp][0] = a;
    s_red[warp][1] = b;
    s_red[warp][2] = c;
  }
  __syncthreads();
  int3 t = make_int3(0, 0, 0);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      t.x += s_red[w][0];
      t.y += s_red[w][1];
      t.z += s_red[w][2];
    }
  }
  return t;
}


// JVP weight of jnp.maximum / jnp.minimum at a tie (0.5), else 1 or 0.
__device__ __forceinline__ float tie_weight(float x, float bound, bool upper_is_x_larger) {
  if (x == bound) return 0.5f;
  return upper_is_x_larger ? (x > bound ? 1.f : 0.f) : (x < bound ? 1.f : 0.f);
}

// Gradient of the conic (a, 2*inv01, c) w.r.t. cov2D entries c00, c01, c11
// through det' = max(c00 c11 - c01^2, 1e-6) (rasterizer.py:147-153).
__device__ __forceinline__ void conic_backward(float c00, float c01, float c11, float ga, float gb2,
                                               float gc, float& g00, float& g01, float& g11) {
  float det_raw = c00 * c11 - c01 * c01;
  float det = fmaxf(det_raw, 1e-6f);
  float id = 1.f / det;
  float ia = c11 * id, i01 = -c01 * id, ic = c00 * id;
  float gi01 = 2.f * gb2;
  float gdet = -(ga * ia + gi01 * i01 + gc * ic) * id;
  float w = tie_weight(det_raw, 1e-6f, true);
  gdet *= w;
  g00 = gc * id + gdet * c11;
  g11 = ga * id + gdet * c00;
  g01 = -gi01 * id + gdet * (-2.f * c01);
}

}  // namespace gs
