// 2DGS surfel renderer (jax_2dgs): projection of 2D Gaussian disks, the
// 9-channel compositor (colour, depth, depth^2, normal, 1 - T), its backward,
// the depth-distortion / normal-consistency regularisers, and the flat Adam
// step of the 2DGS trainer (optax.adam over every parameter).
//
// The pairs are the 3DGS ones (same tile keys, gs_sort.cu); the compositor
// keeps the reference's rule (rasterizer_2d.py:62-92: T > 1e-4 before the
// splat, power > -10, alpha = min(0.99, e^power sigmoid(o))) and composites the
// first BLOCK_SIZE = 512 sorted splats of a tile (rasterizer_2d.py:35-37).
// Forward: one CTA per tile, warps own 8x8 blocks and composite only their
// own lists of splats (as in gs_raster.cu). Backward: the same CTA layout
// replays the tile from T = 1 (at most two batches of 256), with
// dL/dalpha_j = T_j gy_j - (F - R_j) / (1 - alpha_j), gy_j the splat's
// channels dotted with the output gradients (accum counts as a channel of
// value 1, since 1 - T = sum of the weights), F the same dot product of the
// final outputs and R_j its running sum.
#include "gs_kernels.cuh"

namespace gs {

struct __align__(16) Splat2 {
  float4 a;  // means2D x, y, ha, hb (halved conic, as in Splat)
  float4 b;  // hc, sigmoid(opacity), r, g
  float4 c;  // b, half-width, half-height of the power > -10 box, depth z
  float4 d;  // camera-space normal x, y, z, z * z
};

struct __align__(16) Splat2Grad {
  float4 a;  // d mx, d my, d a, d b2
  float4 b;  // d c, d sigmoid(opacity), d r, d g
  float4 c;  // d b, d z (both depth channels), d nx, d ny
  float4 d;  // d nz, 0, 0, 0
};

constexpr int k2dMaxSplats = 512;  // BLOCK_SIZE: splats composited per tile
constexpr float kShC0 = 0.28209479177387814f;

// 2D Gaussian projection (projection_2d.py:6-87) in a fixed evaluation order.
struct Proj2 {
  float x, y, z, u, v;
  float c00, c01, c11, radius;
  float qn[4], qnorm;
  float U[3], V[3], Nc[3];  // camera-space tangents and normal
  float s[2];
  float J00, J02, J11, J12, inv_z;
  float A0, A1, B0, B1;  // rows of J [u | v] before the scales
};

__device__ __forceinline__ void project_surfel(const float m[3], const float sc[2], const float q[4],
                                               const Cam& cam, Proj2& p) {
  const float* W = cam.W;
  p.x = add_rn(add_rn(add_rn(mul_rn(W[0], m[0]), mul_rn(W[1], m[1])), mul_rn(W[2], m[2])), W[3]);
  p.y = add_rn(add_rn(add_rn(mul_rn(W[4], m[0]), mul_rn(W[5], m[1])), mul_rn(W[6], m[2])), W[7]);
  p.z = add_rn(add_rn(add_rn(mul_rn(W[8], m[0]), mul_rn(W[9], m[1])), mul_rn(W[10], m[2])), W[11]);
  // gaussians_2d.py:26-54 tangent vectors of q / |q|
  const float n2 = add_rn(add_rn(add_rn(mul_rn(q[0], q[0]), mul_rn(q[1], q[1])), mul_rn(q[2], q[2])),
                          mul_rn(q[3], q[3]));
  p.qnorm = sqrt_rn(n2);
  const float r = div_rn(q[0], p.qnorm), x = div_rn(q[1], p.qnorm), y = div_rn(q[2], p.qnorm),
              z = div_rn(q[3], p.qnorm);
  p.qn[0] = r; p.qn[1] = x; p.qn[2] = y; p.qn[3] = z;
  const float xx2 = mul_rn(2.f, mul_rn(x, x)), yy2 = mul_rn(2.f, mul_rn(y, y)), zz2 = mul_rn(2.f, mul_rn(z, z));
  const float xy2 = mul_rn(2.f, mul_rn(x, y)), rz2 = mul_rn(2.f, mul_rn(r, z)), xz2 = mul_rn(2.f, mul_rn(x, z));
  const float ry2 = mul_rn(2.f, mul_rn(r, y)), yz2 = mul_rn(2.f, mul_rn(y, z)), rx2 = mul_rn(2.f, mul_rn(r, x));
  const float u[3] = {sub_rn(sub_rn(1.f, yy2), zz2), add_rn(xy2, rz2), sub_rn(xz2, ry2)};
  const float v[3] = {sub_rn(xy2, rz2), sub_rn(sub_rn(1.f, xx2), zz2), add_rn(yz2, rx2)};
  const float n[3] = {add_rn(xz2, ry2), sub_rn(yz2, rx2), sub_rn(sub_rn(1.f, xx2), yy2)};
  // projection_2d.py:37-40: (u, v, n) @ W_rot^T
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float* Wk = W + 4 * k;
    p.U[k] = add_rn(add_rn(mul_rn(u[0], Wk[0]), mul_rn(u[1], Wk[1])), mul_rn(u[2], Wk[2]));
    p.V[k] = add_rn(add_rn(mul_rn(v[0], Wk[0]), mul_rn(v[1], Wk[1])), mul_rn(v[2], Wk[2]));
    p.Nc[k] = add_rn(add_rn(mul_rn(n[0], Wk[0]), mul_rn(n[1], Wk[1])), mul_rn(n[2], Wk[2]));
  }
  // :43-51 J, :55-61 M = J [u | v] diag(exp(s))
  p.inv_z = div_rn(1.f, nan_max(p.z, 0.01f));
  const float iz2 = mul_rn(p.inv_z, p.inv_z);
  p.J00 = mul_rn(cam.fx, p.inv_z);
  p.J02 = mul_rn(mul_rn(-cam.fx, p.x), iz2);
  p.J11 = mul_rn(cam.fy, p.inv_z);
  p.J12 = mul_rn(mul_rn(-cam.fy, p.y), iz2);
  p.s[0] = exp_cr(sc[0]);
  p.s[1] = exp_cr(sc[1]);
  p.A0 = add_rn(mul_rn(p.J00, p.U[0]), mul_rn(p.J02, p.U[2]));
  p.A1 = add_rn(mul_rn(p.J00, p.V[0]), mul_rn(p.J02, p.V[2]));
  p.B0 = add_rn(mul_rn(p.J11, p.U[1]), mul_rn(p.J12, p.U[2]));
  p.B1 = add_rn(mul_rn(p.J11, p.V[1]), mul_rn(p.J12, p.V[2]));
  const float Ms00 = mul_rn(p.A0, p.s[0]), Ms01 = mul_rn(p.A1, p.s[1]);
  const float Ms10 = mul_rn(p.B0, p.s[0]), Ms11 = mul_rn(p.B1, p.s[1]);
  // :65-69 cov2D = Ms Ms^T + 0.3 I
  p.c00 = add_rn(add_rn(mul_rn(Ms00, Ms00), mul_rn(Ms01, Ms01)), 0.3f);
  p.c01 = add_rn(mul_rn(Ms00, Ms10), mul_rn(Ms01, Ms11));
  p.c11 = add_rn(add_rn(mul_rn(Ms10, Ms10), mul_rn(Ms11, Ms11)), 0.3f);
  // :72-75 means2D with the raw z
  p.u = add_rn(div_rn(mul_rn(cam.fx, p.x), p.z), cam.cx);
  p.v = add_rn(div_rn(mul_rn(cam.fy, p.y), p.z), cam.cy);
  // :78-85 radius
  const float det = sub_rn(mul_rn(p.c00, p.c11), mul_rn(p.c01, p.c01));
  const float mid = div_rn(add_rn(p.c00, p.c11), 2.f);
  const float term = sqrt_rn(nan_max(sub_rn(mul_rn(mid, mid), det), 0.f));
  p.radius = ceilf(mul_rn(3.f, sqrt_rn(add_rn(mid, term))));
}

// ---------------------------------------------------------------------------
// Forward preprocess: projection, DC colour, conic, Splat2 record, tile bins
// and the per-block [pairs | visible] counts (the 3DGS sort's input).
__global__ void __launch_bounds__(256)
k_pre2d_fwd(const float* __restrict__ means, const float* __restrict__ scales, const float* __restrict__ quats,
            const float* __restrict__ opac, const float* __restrict__ sh, int n, int sh_k,
            const float* __restrict__ w2c, CamParams cp, Splat2* __restrict__ splats, int2* __restrict__ bins,
            int* __restrict__ block_counts, float* __restrict__ radii_out, uint8_t* __restrict__ valid_out,
            GsExtras* __restrict__ extras) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ int s_red3[8][3];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  int count = 0, capv = 0;
  if (i < n) {
    Cam cam;
    load_cam_rows(w2c, cam);
    cam.fx = cp.fx; cam.fy = cp.fy; cam.cx = cp.cx; cam.cy = cp.cy;
    const float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
    const float sc[2] = {scales[2 * i], scales[2 * i + 1]};
    const float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
    Proj2 p;
    project_surfel(m, sc, q, cam, p);
    const bool valid = p.z > 0.01f;  // projection_2d.py:31 (no active mask in 2DGS)
    radii_out[i] = p.radius;
    valid_out[i] = valid ? 1 : 0;
    const Rect rc = tile_rect(p.u, p.v, p.radius, cp.width, cp.height);
    int nx = 0, ny = 0, tx0 = 0, ty0 = 0, dq = 0;
    if (valid && rc.on_screen) {
      const int spx = rc.tx1 - rc.tx0 + 1, spy = rc.ty1 - rc.ty0 + 1;
      capv = (spx > kOffset || spy > kOffset) ? 1 : 0;
      if (spx > 0 && spy > 0) {
        nx = min(spx, kOffset);
        ny = min(spy, kOffset);
        tx0 = rc.tx0; ty0 = rc.ty0;
        dq = depth_key(p.z);
      }
    }
    count = nx * ny;
    bins[i] = pack_bin(tx0, ty0, nx, ny, dq);
    if (count > 0) {
      // rasterizer_2d.py:18-26 conic with the det clamp, sigmoid; renderer.py:27-28 DC colour
      const float det = fmaxf(p.c00 * p.c11 - p.c01 * p.c01, 1e-6f);
      const float ia = p.c11 / det, i01 = -p.c01 / det, ic = p.c00 / det;
      const float* s0 = sh + (size_t)i * sh_k * 3;
      float col[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) col[c] = fminf(fmaxf(add_rn(mul_rn(s0[c], kShC0), 0.5f), 0.f), 1.f);
      const float2 h = bbox_halfext(p.c00, p.c01, p.c11);
      Splat2 s;
      s.a = make_float4(p.u, p.v, -0.5f * ia, -i01);
      s.b = make_float4(-0.5f * ic, sigmoidf(opac[i]), col[0], col[1]);
      s.c = make_float4(col[2], h.x, h.y, p.z);
      s.d = make_float4(p.Nc[0], p.Nc[1], p.Nc[2], mul_rn(p.z, p.z));
      splats[i] = s;
    }
  }
  // pairs, visible surfels and radius-cap violations of the block
  const int3 t = block_sum3_256(count, count > 0 ? 1 : 0, capv, s_red3);
  if (threadIdx.x == 0) {
    block_counts[blockIdx.x] = t.x;
    block_counts[gridDim.x + blockIdx.x] = t.y;
    if (t.z && extras) atomicAdd(&extras->radius_cap_violations, t.z);
  }
}

// ---------------------------------------------------------------------------
// Pixel ownership as in gs_raster.cu: 128 threads, warp w owns an 8x8 block,
// a thread a column of 2 pixels.
constexpr int k2Pix = 2, k2Wx = 8, k2NT = kTilePixels / k2Pix, k2NW = k2NT / 32, k2Wy = 32 * k2Pix / k2Wx;
constexpr int k2Wpr = kTile / k2Wx;

__device__ __forceinline__ unsigned warp_mask2(float mx, float my, float hx, float hy, float ha, float hb, float hc,
                                               int tx, int ty) {
  unsigned m = 0;
#pragma unroll
  for (int w = 0; w < k2NW; ++w) {
    const float x0 = (float)(tx * kTile + (w % k2Wpr) * k2Wx) + 0.5f, x1 = x0 + (float)(k2Wx - 1);
    const float y0 = (float)(ty * kTile + (w / k2Wpr) * k2Wy) + 0.5f, y1 = y0 + (float)(k2Wy - 1);
    const bool miss = (mx + hx < x0) | (mx - hx > x1) | (my + hy < y0) | (my - hy > y1);
    if (!miss && splat_meets_rect(mx, my, ha, hb, hc, x0, x1, y0, y1)) m |= 1u << w;
  }
  return m;
}

__device__ __forceinline__ int warp_list2(const unsigned char* s_mask, int nb, int warp, int lane,
                                          unsigned char* list) {
  int cnt = 0;
  unsigned lt;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
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

__device__ __forceinline__ float surfel_exp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, 1.4426950408889634f)));
  return y;
}

// Stages batch b of the tile's splats (records, warp masks, per-warp lists).
__device__ __forceinline__ int stage_batch2(const Splat2* __restrict__ splats, const int* __restrict__ ids, int n,
                                            int start, int count, int b, int tx, int ty, float4 (*s_r)[kBatch],
                                            int* s_gid, unsigned char* s_mask, unsigned char (*s_list)[kBatch],
                                            int tid, int warp, int lane, int& nb) {
  const int b0 = b * kBatch;
  nb = min(kBatch, count - b0);
  for (int j = tid; j < nb; j += k2NT) {
    int g = ids[start + b0 + j];
    g = min(max(g, 0), n - 1);
    const Splat2* sp = splats + g;
    const float4 a = __ldg(&sp->a), bb = __ldg(&sp->b), c = __ldg(&sp->c);
    s_r[0][j] = a;
    s_r[1][j] = bb;
    s_r[2][j] = c;
    s_r[3][j] = __ldg(&sp->d);
    if (s_gid) s_gid[j] = g;
    s_mask[j] = (unsigned char)warp_mask2(a.x, a.y, c.y, c.z, a.z, a.w, bb.x, tx, ty);
  }
  __syncthreads();
  return warp_list2(s_mask, nb, warp, lane, s_list[warp]);
}

__global__ void __launch_bounds__(k2NT, 8)
k_raster2d_fwd(const Splat2* __restrict__ splats, const int* __restrict__ ids, const int* __restrict__ ranges,
               int n, const float* __restrict__ bg, int width, int height, int tiles_x,
               float* __restrict__ image, float* __restrict__ depth, float* __restrict__ depth_sq,
               float* __restrict__ normals, float* __restrict__ accum, float* __restrict__ pix_T) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float4 s_r[4][kBatch];
  __shared__ unsigned char s_mask[kBatch];
  __shared__ unsigned char s_list[k2NW][kBatch];
  const int tile = blockIdx.x, tx = tile % tiles_x, ty = tile / tiles_x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lx = (warp % k2Wpr) * k2Wx + lane % k2Wx, ly0 = (warp / k2Wpr) * k2Wy + (lane / k2Wx) * k2Pix;
  const int px = tx * kTile + lx;
  const float fpx = (float)px + 0.5f;
  const int start = ranges[tile];
  const int count = min(ranges[tile + 1] - start, k2dMaxSplats);
  float T[k2Pix], acc[k2Pix][8], fpy[k2Pix];
#pragma unroll
  for (int i = 0; i < k2Pix; ++i) {
    const int py = ty * kTile + ly0 + i;
    fpy[i] = (float)py + 0.5f;
    T[i] = (px < width && py < height) ? 1.f : 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
  }
  const int nbt = (count + kBatch - 1) / kBatch;
  for (int b = 0; b < nbt; ++b) {
    bool alive = false;
#pragma unroll
    for (int i = 0; i < k2Pix; ++i) alive |= (T[i] > 1e-4f);
    if (__syncthreads_count(alive) == 0) break;
    int nb;
    const int cnt = stage_batch2(splats, ids, n, start, count, b, tx, ty, s_r, nullptr, s_mask, s_list, tid,
                                 warp, lane, nb);
    const unsigned char* list = s_list[warp];
    for (int q = 0; alive && q < cnt; ++q) {
      const int k = list[q];
      const float4 A = s_r[0][k], B = s_r[1][k], Cc = s_r[2][k], D = s_r[3][k];
      const float dx = fpx - A.x;
      const float q0 = splat_q0(dx, A.z), q1 = splat_q1(dx, A.w);
      const float ch[8] = {B.z, B.w, Cc.x, Cc.w, D.w, D.x, D.y, D.z};  // r g b z z^2 nx ny nz
#pragma unroll
      for (int i = 0; i < k2Pix; ++i) {
        const float power = splat_power(fpy[i] - A.y, q0, q1, B.x);
        const float a_raw = fminf(0.99f, __fmul_rn(surfel_exp(power), B.y));
        const float alpha = ((T[i] > 1e-4f) & (power > -10.f)) ? a_raw : 0.f;
        const float w = __fmul_rn(alpha, T[i]);
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[i][c] = __fmaf_rn(w, ch[c], acc[i][c]);
        T[i] = __fmul_rn(T[i], __fsub_rn(1.f, alpha));
      }
      if ((q & 15) == 15) {
        alive = false;
#pragma unroll
        for (int i = 0; i < k2Pix; ++i) alive |= (T[i] > 1e-4f);
      }
    }
  }
  float b0 = 0.f, b1 = 0.f, b2 = 0.f;
  if (bg) { b0 = bg[0]; b1 = bg[1]; b2 = bg[2]; }
#pragma unroll
  for (int i = 0; i < k2Pix; ++i) {
    const int py = ty * kTile + ly0 + i;
    if (px < width && py < height) {
      const int pix = py * width + px;
      image[3 * pix] = acc[i][0] + T[i] * b0;
      image[3 * pix + 1] = acc[i][1] + T[i] * b1;
      image[3 * pix + 2] = acc[i][2] + T[i] * b2;
      depth[pix] = acc[i][3];
      depth_sq[pix] = acc[i][4];
      normals[3 * pix] = acc[i][5];
      normals[3 * pix + 1] = acc[i][6];
      normals[3 * pix + 2] = acc[i][7];
      accum[pix] = 1.f - T[i];
      pix_T[pix] = T[i];
    }
  }
}

// Warp sum of 16 per-lane values by recursive halving (8 + 4 + 2 + 1
// shuffles), then a butterfly over the last lane bit: lanes 2i and 2i + 1
// hold the total of value i in v[0].
__device__ __forceinline__ void warp_sum16(float v[16], int lane) {
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = h16 ? v[i] : v[i + 8], keep = h16 ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h8 ? v[i] : v[i + 4], keep = h8 ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h4 ? v[i] : v[i + 2], keep = h4 ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const float send = h2 ? v[0] : v[1], keep = h2 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// Backward: per tile, replay from T = 1. Output gradients: image (3), depth,
// depth_sq, normals (3), accum (nullable).
constexpr int k2Grads = 13;  // mx my a b2 c sigma r g b z nx ny nz

__global__ void __launch_bounds__(k2NT, 4)
k_raster2d_bwd(const Splat2* __restrict__ splats, const int* __restrict__ ids, const int* __restrict__ ranges,
               int n, int width, int height, int tiles_x, const float* __restrict__ image,
               const float* __restrict__ depth, const float* __restrict__ depth_sq,
               const float* __restrict__ normals, const float* __restrict__ accum, const float* __restrict__ pix_T,
               const float* __restrict__ g_image, const float* __restrict__ g_depth,
               const float* __restrict__ g_depth_sq, const float* __restrict__ g_normals,
               const float* __restrict__ g_accum, Splat2Grad* __restrict__ grads) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float4 s_r[4][kBatch];
  __shared__ int s_gid[kBatch];
  __shared__ float s_acc[k2Grads][kBatch + 1];
  __shared__ unsigned char s_mask[kBatch];
  __shared__ unsigned char s_list[k2NW][kBatch];
  const int tile = blockIdx.x, tx = tile % tiles_x, ty = tile / tiles_x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lx = (warp % k2Wpr) * k2Wx + lane % k2Wx, ly0 = (warp / k2Wpr) * k2Wy + (lane / k2Wx) * k2Pix;
  const int px = tx * kTile + lx;
  const float fpx = (float)px + 0.5f;
  const int start = ranges[tile];
  const int count = min(ranges[tile + 1] - start, k2dMaxSplats);
  if (count <= 0) return;
  for (int j = tid; j < k2Grads * (kBatch + 1); j += k2NT) (&s_acc[0][0])[j] = 0.f;
  // per-pixel output gradients G (9 channels) and F = G . outputs
  float T[k2Pix], G[k2Pix][9], F[k2Pix], R[k2Pix], fpy[k2Pix];
#pragma unroll
  for (int i = 0; i < k2Pix; ++i) {
    const int py = ty * kTile + ly0 + i;
    fpy[i] = (float)py + 0.5f;
    T[i] = 0.f;
    F[i] = R[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 9; ++c) G[i][c] = 0.f;
    if (px < width && py < height) {
      const int pix = py * width + px;
      T[i] = 1.f;
      G[i][0] = g_image[3 * pix]; G[i][1] = g_image[3 * pix + 1]; G[i][2] = g_image[3 * pix + 2];
      G[i][3] = g_depth ? g_depth[pix] : 0.f;
      G[i][4] = g_depth_sq ? g_depth_sq[pix] : 0.f;
      if (g_normals) {
        G[i][5] = g_normals[3 * pix]; G[i][6] = g_normals[3 * pix + 1]; G[i][7] = g_normals[3 * pix + 2];
      }
      G[i][8] = g_accum ? g_accum[pix] : 0.f;
      F[i] = G[i][0] * image[3 * pix] + G[i][1] * image[3 * pix + 1] + G[i][2] * image[3 * pix + 2] +
             G[i][3] * depth[pix] + G[i][4] * depth_sq[pix] + G[i][5] * normals[3 * pix] +
             G[i][6] * normals[3 * pix + 1] + G[i][7] * normals[3 * pix + 2] + G[i][8] * accum[pix];
      (void)pix_T;
    }
  }
  const int nbt = (count + kBatch - 1) / kBatch;
  for (int b = 0; b < nbt; ++b) {
    bool al = false;
#pragma unroll
    for (int i = 0; i < k2Pix; ++i) al |= (T[i] > 1e-4f);
    if (__syncthreads_count(al) == 0) break;
    int nb;
    const int cnt = stage_batch2(splats, ids, n, start, count, b, tx, ty, s_r, s_gid, s_mask, s_list, tid, warp,
                                 lane, nb);
    const unsigned char* list = s_list[warp];
    bool alive = __any_sync(0xffffffffu, al);
    for (int q = 0; alive && q < cnt; ++q) {
      const int k = list[q];
      const float4 A = s_r[0][k], B = s_r[1][k], Cc = s_r[2][k], D = s_r[3][k];
      const float dx = fpx - A.x;
      const float q0 = splat_q0(dx, A.z), q1 = splat_q1(dx, A.w);
      const float ch[8] = {B.z, B.w, Cc.x, Cc.w, D.w, D.x, D.y, D.z};
      float v[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) v[c] = 0.f;
      float S0 = 0.f, S1 = 0.f, S2 = 0.f;
      bool contrib = false;
#pragma unroll
      for (int i = 0; i < k2Pix; ++i) {
        const float dy = fpy[i] - A.y;
        const float power = splat_power(dy, q0, q1, B.x);
        const float e = surfel_exp(power);
        const float ea = __fmul_rn(e, B.y);
        const bool act = (T[i] > 1e-4f) & (power > -10.f);
        const float alpha = act ? fminf(0.99f, ea) : 0.f;
        const float one_m = __fsub_rn(1.f, alpha);
        float gy = G[i][8];
#pragma unroll
        for (int c = 0; c < 8; ++c) gy += G[i][c] * ch[c];
        const float w = __fmul_rn(alpha, T[i]);
        R[i] += w * gy;
        const float dalpha = T[i] * gy - __fdividef(F[i] - R[i], one_m);
        T[i] = __fmul_rn(T[i], one_m);
        // u = dL/d(ea) e (jnp.minimum(0.99, ea): gradient 1 below, 1/2 at
        // the tie, 0 above); dL/dpower = u sigmoid(opacity)
        const float fe = act ? ((ea < 0.99f) ? e : ((ea == 0.99f) ? 0.5f * e : 0.f)) : 0.f;
        const float u = dalpha * fe;
        v[6] += w * G[i][0];                         // d r, g, b
        v[7] += w * G[i][1];
        v[8] += w * G[i][2];
        v[9] += w * (G[i][3] + 2.f * Cc.w * G[i][4]);  // d z through z and z^2
        v[10] += w * G[i][5];                        // d normal
        v[11] += w * G[i][6];
        v[12] += w * G[i][7];
        S0 += u;
        const float uy = u * dy;
        S1 += uy;
        S2 += uy * dy;
        contrib |= act;
      }
      v[5] = S0;  // d sigmoid
      // reduced raw, combined with the splat's conic and opacity once per
      // batch (flush)
      const float dxS0 = dx * S0;
      v[0] = dxS0;
      v[1] = S1;
      v[2] = dx * dxS0;
      v[3] = dx * S1;
      v[4] = S2;
      if (__any_sync(0xffffffffu, contrib)) {
        warp_sum16(v, lane);
        if ((lane & 1) == 0 && (lane >> 1) < k2Grads) atomicAdd(&s_acc[lane >> 1][k], v[0]);
      }
      if ((q & 15) == 15) {
        bool a2 = false;
#pragma unroll
        for (int i = 0; i < k2Pix; ++i) a2 |= (T[i] > 1e-4f);
        alive = __any_sync(0xffffffffu, a2);
      }
    }
    __syncthreads();
    for (int j = tid; j < nb; j += k2NT) {
      float a[k2Grads];
      bool any = false;
#pragma unroll
      for (int qq = 0; qq < k2Grads; ++qq) {
        a[qq] = s_acc[qq][j];
        s_acc[qq][j] = 0.f;
        any |= a[qq] != 0.f;
      }
      if (any) {
        // power = ha dx^2 + hb dx dy + hc dy^2, dL/dpower = u sig per pixel:
        // gradients of mean x, y and of (a, b2, c) from R0 = sum dx S0,
        // R1 = sum S1, R2 = sum dx^2 S0, R3 = sum dx S1, R4 = sum S2
        // (S0 = u, S1 = u dy, S2 = u dy^2)
        const float ha = s_r[0][j].z, hb = s_r[0][j].w, hc = s_r[1][j].x, sig = s_r[1][j].y;
        const float r0 = sig * a[0], r1 = sig * a[1], hs = -0.5f * sig;
        a[0] = -2.f * ha * r0 - hb * r1;
        a[1] = -2.f * hc * r1 - hb * r0;
        a[2] = hs * a[2];
        a[3] = hs * a[3];
        a[4] = hs * a[4];
        Splat2Grad* gp = grads + s_gid[j];
        atomicAdd(&gp->a, make_float4(a[0], a[1], a[2], a[3]));
        atomicAdd(&gp->b, make_float4(a[4], a[5], a[6], a[7]));
        atomicAdd(&gp->c, make_float4(a[8], a[9], a[10], a[11]));
        atomicAdd(&gp->d.x, a[12]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Preprocess backward: Splat2Grad -> means, scales (2), quaternions,
// opacities, sh (DC only). One thread per surfel; the DC gradient is returned
// in gsh[3] for the CTA's coalesced store of the sh rows.
__device__ __forceinline__ void pre2d_bwd_one(const float* __restrict__ means, const float* __restrict__ scales,
                                              const float* __restrict__ quats, const float* __restrict__ opac,
                                              const float* __restrict__ sh, int i, int sh_k,
                                              const float* __restrict__ w2c, const CamParams& cp,
                                              const Splat2Grad* __restrict__ sgrad, float* __restrict__ g_means,
                                              float* __restrict__ g_scales, float* __restrict__ g_quats,
                                              float* __restrict__ g_opac, float gsh[3]) {
  const Splat2Grad gr = sgrad[i];
  const bool any = (gr.a.x != 0.f) | (gr.a.y != 0.f) | (gr.a.z != 0.f) | (gr.a.w != 0.f) | (gr.b.x != 0.f) |
                   (gr.b.y != 0.f) | (gr.b.z != 0.f) | (gr.b.w != 0.f) | (gr.c.x != 0.f) | (gr.c.y != 0.f) |
                   (gr.c.z != 0.f) | (gr.c.w != 0.f) | (gr.d.x != 0.f);
  if (!any) {
    g_means[3 * i] = g_means[3 * i + 1] = g_means[3 * i + 2] = 0.f;
    g_scales[2 * i] = g_scales[2 * i + 1] = 0.f;
    g_quats[4 * i] = g_quats[4 * i + 1] = g_quats[4 * i + 2] = g_quats[4 * i + 3] = 0.f;
    g_opac[i] = 0.f;
    gsh[0] = gsh[1] = gsh[2] = 0.f;
    return;
  }
  Cam cam;
  load_cam_rows(w2c, cam);
  cam.fx = cp.fx; cam.fy = cp.fy; cam.cx = cp.cx; cam.cy = cp.cy;
  const float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
  const float sc[2] = {scales[2 * i], scales[2 * i + 1]};
  const float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
  Proj2 p;
  project_surfel(m, sc, q, cam, p);
  const float* W = cam.W;
  // colour: clip(sh0 C0 + 0.5, 0, 1), half weight at either bound
  const float gcol[3] = {gr.b.z, gr.b.w, gr.c.x};
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float raw = sh[(size_t)i * sh_k * 3 + c] * kShC0 + 0.5f;
    const float w = (raw > 0.f && raw < 1.f) ? 1.f : ((raw == 0.f || raw == 1.f) ? 0.5f : 0.f);
    gsh[c] = gcol[c] * w * kShC0;
  }
  // opacity (rasterizer_2d.py:26)
  {
    const float s = sigmoidf(opac[i]);
    g_opac[i] = gr.b.y * s * (1.f - s);
  }
  // conic -> cov2D entries (det clamp), cov2D = Ms Ms^T (only [0,1] of the
  // off-diagonal is read downstream)
  float g00, g01, g11;
  conic_backward(p.c00, p.c01, p.c11, gr.a.z, gr.a.w, gr.b.x, g00, g01, g11);
  const float Ms00 = p.A0 * p.s[0], Ms01 = p.A1 * p.s[1], Ms10 = p.B0 * p.s[0], Ms11 = p.B1 * p.s[1];
  const float dMs00 = 2.f * g00 * Ms00 + g01 * Ms10, dMs01 = 2.f * g00 * Ms01 + g01 * Ms11;
  const float dMs10 = g01 * Ms00 + 2.f * g11 * Ms10, dMs11 = g01 * Ms01 + 2.f * g11 * Ms11;
  g_scales[2 * i] = (dMs00 * p.A0 + dMs10 * p.B0) * p.s[0];
  g_scales[2 * i + 1] = (dMs01 * p.A1 + dMs11 * p.B1) * p.s[1];
  const float dA0 = dMs00 * p.s[0], dA1 = dMs01 * p.s[1], dB0 = dMs10 * p.s[0], dB1 = dMs11 * p.s[1];
  const float dJ00 = dA0 * p.U[0] + dA1 * p.V[0], dJ02 = dA0 * p.U[2] + dA1 * p.V[2];
  const float dJ11 = dB0 * p.U[1] + dB1 * p.V[1], dJ12 = dB0 * p.U[2] + dB1 * p.V[2];
  const float dU[3] = {dA0 * p.J00, dB0 * p.J11, dA0 * p.J02 + dB0 * p.J12};
  const float dV[3] = {dA1 * p.J00, dB1 * p.J11, dA1 * p.J02 + dB1 * p.J12};
  const float dN[3] = {gr.c.z, gr.c.w, gr.d.x};
  // J -> camera-space mean (max(z, 0.01) passes half the gradient at the tie)
  const float iz = p.inv_z, iz2 = iz * iz, iz3 = iz2 * iz;
  float gpx = dJ02 * (-cp.fx * iz2);
  float gpy = dJ12 * (-cp.fy * iz2);
  const float gsz = dJ00 * (-cp.fx * iz2) + dJ02 * (2.f * cp.fx * p.x * iz3) + dJ11 * (-cp.fy * iz2) +
                    dJ12 * (2.f * cp.fy * p.y * iz3);
  float gpz = gsz * tie_weight(p.z, 0.01f, true);
  // means2D (raw z) and depth
  {
    const float mx = gr.a.x, my = gr.a.y, izr = 1.f / p.z;
    gpx += mx * cp.fx * izr;
    gpy += my * cp.fy * izr;
    gpz += -(mx * cp.fx * p.x + my * cp.fy * p.y) * izr * izr;
    gpz += gr.c.y;
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) g_means[3 * i + k] = W[0 * 4 + k] * gpx + W[1 * 4 + k] * gpy + W[2 * 4 + k] * gpz;
  // camera-space (u, v, n) -> world: W_rot^T
  float du[3], dv[3], dn[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    du[k] = W[0 * 4 + k] * dU[0] + W[1 * 4 + k] * dU[1] + W[2 * 4 + k] * dU[2];
    dv[k] = W[0 * 4 + k] * dV[0] + W[1 * 4 + k] * dV[1] + W[2 * 4 + k] * dV[2];
    dn[k] = W[0 * 4 + k] * dN[0] + W[1 * 4 + k] * dN[1] + W[2 * 4 + k] * dN[2];
  }
  // (u, v, n) of the normalised quaternion (gaussians_2d.py:33-52)
  const float r = p.qn[0], x = p.qn[1], y = p.qn[2], z = p.qn[3];
  const float gr_ = 2.f * (z * du[1] - y * du[2] - z * dv[0] + x * dv[2] + y * dn[0] - x * dn[1]);
  const float gx = 2.f * (y * du[1] + z * du[2] + y * dv[0] - 2.f * x * dv[1] + r * dv[2] + z * dn[0] - r * dn[1] -
                          2.f * x * dn[2]);
  const float gy = 2.f * (-2.f * y * du[0] + x * du[1] - r * du[2] + x * dv[0] + z * dv[2] + r * dn[0] + z * dn[1] -
                          2.f * y * dn[2]);
  const float gz = 2.f * (-2.f * z * du[0] + r * du[1] + x * du[2] - r * dv[0] - 2.f * z * dv[1] + y * dv[2] +
                          x * dn[0] + y * dn[1]);
  const float dot = r * gr_ + x * gx + y * gy + z * gz;
  const float in = 1.f / p.qnorm;
  g_quats[4 * i] = (gr_ - r * dot) * in;
  g_quats[4 * i + 1] = (gx - x * dot) * in;
  g_quats[4 * i + 2] = (gy - y * dot) * in;
  g_quats[4 * i + 3] = (gz - z * dot) * in;
}

__global__ void __launch_bounds__(256)
k_pre2d_bwd(const float* __restrict__ means, const float* __restrict__ scales, const float* __restrict__ quats,
            const float* __restrict__ opac, const float* __restrict__ sh, int n, int sh_k,
            const float* __restrict__ w2c, CamParams cp, const Splat2Grad* __restrict__ sgrad,
            float* __restrict__ g_means, float* __restrict__ g_scales, float* __restrict__ g_quats,
            float* __restrict__ g_opac, float* __restrict__ g_sh) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_dc[256 * 3];
  const int tid = threadIdx.x, base = blockIdx.x * 256, i = base + tid;
  float dc[3] = {0.f, 0.f, 0.f};
  if (i < n) pre2d_bwd_one(means, scales, quats, opac, sh, i, sh_k, w2c, cp, sgrad, g_means, g_scales, g_quats,
                           g_opac, dc);
  s_dc[3 * tid] = dc[0];
  s_dc[3 * tid + 1] = dc[1];
  s_dc[3 * tid + 2] = dc[2];
  __syncthreads();
  // sh rows of L = 3 sh_k floats, the DC coefficient first and zeros after it
  // (only the DC coefficient is used, renderer.py:27): warp w stores rows
  // w, w + 8, ..., lane l element l (and l + 32) of each
  const int cnt = min(256, n - base), L = 3 * sh_k, warp = tid >> 5, lane = tid & 31;
  float* dst = g_sh + (size_t)L * base;
  for (int g = warp; g < cnt; g += 8) {
    if (lane < L) dst[(size_t)g * L + lane] = (lane < 3) ? s_dc[3 * g + lane] : 0.f;
    if (lane + 32 < L) dst[(size_t)g * L + lane + 32] = 0.f;
  }
}

// ---------------------------------------------------------------------------
// Regularisers (jax_2dgs/training/losses.py): depth distortion (:4-32) and
// normal consistency (:34-78), means over H x W, with their gradients w.r.t.
// depth, depth_sq and normals (accum_weight and the normal loss's weight are
// stop-gradient in the reference). Deterministic last-CTA reduction.
struct RegScalars {
  unsigned ticket;
  float pad[3];
};

__global__ void __launch_bounds__(256)
k_reg2d(const float* __restrict__ depth, const float* __restrict__ depth_sq, const float* __restrict__ normals,
        const float* __restrict__ accum, int H, int W, float lam_dist, float lam_normal,
        float* __restrict__ part, RegScalars* __restrict__ rs, float* __restrict__ dist_out,
        float* __restrict__ normal_out, float* __restrict__ g_depth, float* __restrict__ g_depth_sq,
        float* __restrict__ g_normals) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ double s_w[8];
  __shared__ float s_red[2][8];
  __shared__ bool s_last;
  const int P = H * W;
  const float inv_p = 1.f / (float)P;
  float acc_d = 0.f, acc_n = 0.f;
  for (int pix = blockIdx.x * 256 + threadIdx.x; pix < P; pix += gridDim.x * 256) {
    const int y = pix / W, x = pix - y * W;
    // depth distortion
    const float w = accum[pix];
    float gd = 0.f, gd2 = 0.f;
    if (w > 1e-4f) {
      const float ed = depth[pix] / w, ed2 = depth_sq[pix] / w;
      const float vr = ed2 - ed * ed;
      acc_d += fmaxf(vr, 0.f) * w;
      const float tw = (vr > 0.f) ? 1.f : ((vr == 0.f) ? 0.5f : 0.f);
      // d (var w) / d depth_sq = 1, d / d depth = -2 E[d] (w is a constant)
      gd2 = lam_dist * inv_p * tw;
      gd = -2.f * ed * lam_dist * inv_p * tw;
    }
    // normal consistency: depth normal from the (constant) depth map with
    // wrap-around central differences (jnp.roll)
    const int xl = (x == 0) ? W - 1 : x - 1, xr = (x == W - 1) ? 0 : x + 1;
    const int yu = (y == 0) ? H - 1 : y - 1, yd = (y == H - 1) ? 0 : y + 1;
    const float dzdx = (depth[y * W + xr] - depth[y * W + xl]) / 2.f;
    const float dzdy = (depth[yd * W + x] - depth[yu * W + x]) / 2.f;
    float nd0 = -dzdx, nd1 = -dzdy, nd2 = 1.f;
    const float ndn = sqrtf(nd0 * nd0 + nd1 * nd1 + nd2 * nd2 + 1e-6f);
    nd0 /= ndn; nd1 /= ndn; nd2 /= ndn;
    const float n0 = normals[3 * pix], n1 = normals[3 * pix + 1], n2 = normals[3 * pix + 2];
    const float rn = sqrtf(n0 * n0 + n1 * n1 + n2 * n2 + 1e-8f);
    const float r0 = n0 / rn, r1 = n1 / rn, r2 = n2 / rn;
    const float cs = r0 * nd0 + r1 * nd1 + r2 * nd2;
    acc_n += (1.f - cs) * rn;
    // d/dn of (1 - cos) * stop(rn): -stop(rn) (nd - nr cos) / rn
    const float gsc = -lam_normal * inv_p * rn / rn;
    if (g_depth) {
      g_depth[pix] = gd;
      g_depth_sq[pix] = gd2;
      g_normals[3 * pix] = gsc * (nd0 - r0 * cs);
      g_normals[3 * pix + 1] = gsc * (nd1 - r1 * cs);
      g_normals[3 * pix + 2] = gsc * (nd2 - r2 * cs);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_d += __shfl_down_sync(0xffffffffu, acc_d, o);
    acc_n += __shfl_down_sync(0xffffffffu, acc_n, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_red[0][threadIdx.x >> 5] = acc_d;
    s_red[1][threadIdx.x >> 5] = acc_n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < 8; ++w) {
      a += s_red[0][w];
      b += s_red[1][w];
    }
    part[blockIdx.x] = a;
    part[gridDim.x + blockIdx.x] = b;
    __threadfence();
    s_last = (atomicAdd(&rs->ticket, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double td = 0.0, tn = 0.0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += 256) {
    td += (double)((volatile float*)part)[b];
    tn += (double)((volatile float*)part)[gridDim.x + b];
  }
  td = block_sum_d256(td, s_w);
  tn = block_sum_d256(tn, s_w);
  if (threadIdx.x == 0) {
    if (dist_out) *dist_out = (float)(td / (double)P);
    if (normal_out) *normal_out = (float)(tn / (double)P);
    rs->ticket = 0u;
  }
}

// Bias corrections from a device-side optax count (state[0], before this
// update), as the host computes them for gs_adam_step_flat; and the count
// advance by the last CTA to finish (state[1] is its ticket, no waiting).
__device__ __forceinline__ void flat_bias(const int* state, float b1, float b2, float& inv_bc1, float& inv_bc2) {
  if (!state) return;
  const double step = (double)(*(volatile const int*)state) + 1.0;
  inv_bc1 = 1.f / (1.f - (float)pow((double)b1, step));
  inv_bc2 = 1.f / (1.f - (float)pow((double)b2, step));
}
__device__ __forceinline__ void flat_advance(int* state) {
  if (!state) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(reinterpret_cast<unsigned*>(state + 1), 1u);
    if (t == gridDim.x - 1) {
      state[0] = state[0] + 1;
      state[1] = 0;
    }
  }
}

// optax.adam on a flat buffer (the 2DGS trainer's optimizer, one learning rate).
__global__ void __launch_bounds__(256)
k_adam_flat_scalar(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                   float* __restrict__ v, int count, float lr, float b1, float b2, float omb1, float omb2,
                   float inv_bc1, float inv_bc2, float eps, int* state) {
  GS_PDL_ENTRY_PLAIN();
  flat_bias(state, b1, b2, inv_bc1, inv_bc2);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < count; e += gridDim.x * blockDim.x) {
    const float gg = g[e];
    const float mm = omb1 * gg + b1 * m[e];
    const float vv = omb2 * (gg * gg) + b2 * v[e];
    m[e] = mm;
    v[e] = vv;
    p[e] += -lr * __fdividef(mm * inv_bc1, __fsqrt_rn(vv * inv_bc2) + eps);
  }
  flat_advance(state);
}

// The same, four elements per thread (16-byte aligned buffers).
__global__ void __launch_bounds__(256)
k_adam_flat(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
            int count, float lr, float b1, float b2, float omb1, float omb2, float inv_bc1, float inv_bc2,
            float eps, int* state) {
  GS_PDL_ENTRY_PLAIN();
  flat_bias(state, b1, b2, inv_bc1, inv_bc2);
  auto one = [&](float& pp, float gg, float& mm, float& vv) {
    mm = omb1 * gg + b1 * mm;
    vv = omb2 * (gg * gg) + b2 * vv;
    pp += -lr * __fdividef(mm * inv_bc1, __fsqrt_rn(vv * inv_bc2) + eps);
  };
  const int stride = gridDim.x * blockDim.x;
  const int n4 = count / 4;  // the buffers are 16-byte aligned (cudaMalloc / torch)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 P = reinterpret_cast<float4*>(p)[i], G = reinterpret_cast<const float4*>(g)[i];
    float4 M = reinterpret_cast<float4*>(m)[i], V = reinterpret_cast<float4*>(v)[i];
    one(P.x, G.x, M.x, V.x);
    one(P.y, G.y, M.y, V.y);
    one(P.z, G.z, M.z, V.z);
    one(P.w, G.w, M.w, V.w);
    reinterpret_cast<float4*>(p)[i] = P;
    reinterpret_cast<float4*>(m)[i] = M;
    reinterpret_cast<float4*>(v)[i] = V;
  }
  for (int e = 4 * n4 + blockIdx.x * blockDim.x + threadIdx.x; e < count; e += stride) one(p[e], g[e], m[e], v[e]);
  flat_advance(state);
}

// ---------------------------------------------------------------------------
size_t splat2_bytes() { return sizeof(Splat2); }
size_t splat2_grad_bytes() { return sizeof(Splat2Grad); }

void launch_pre2d_fwd(const float* means, const float* scales, const float* quats, const float* opac,
                      const float* sh, int n, int sh_k, const float* w2c, const CamParams& cp, void* splats,
                      int2* bins, int* block_counts, float* radii, uint8_t* valid, GsExtras* extras,
                      cudaStream_t st) {
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("preprocess2d_fwd", st);
  launch_kernel_plain(k_pre2d_fwd, nb, 256, 0, st, means, scales, quats, opac, sh, n, sh_k, w2c, cp, (Splat2*)splats, bins,
                                  block_counts, radii, valid, extras);
}

void launch_raster2d_fwd(const void* splats, const int* ids, const int* ranges, int n, const float* bg, int width,
                         int height, int tiles_x, int num_tiles, float* image, float* depth, float* depth_sq,
                         float* normals, float* accum, float* pix_T, cudaStream_t st) {
  if (num_tiles == 0) return;
  GS_TIMED("raster2d_fwd", st);
  launch_kernel_plain(k_raster2d_fwd, num_tiles, k2NT, 0, st, (const Splat2*)splats, ids, ranges, n, bg, width, height, tiles_x,
                                             image, depth, depth_sq, normals, accum, pix_T);
}

void launch_raster2d_bwd(const void* splats, const int* ids, const int* ranges, int n, int width, int height,
                         int tiles_x, int num_tiles, const float* image, const float* depth, const float* depth_sq,
                         const float* normals, const float* accum, const float* pix_T, const float* g_image,
                         const float* g_depth, const float* g_depth_sq, const float* g_normals,
                         const float* g_accum, void* grads, cudaStream_t st) {
  cudaMemsetAsync(grads, 0, sizeof(Splat2Grad) * (size_t)n, st);
  if (num_tiles == 0) return;
  GS_TIMED("raster2d_bwd", st);
  launch_kernel_plain(k_raster2d_bwd, num_tiles, k2NT, 0, st, (const Splat2*)splats, ids, ranges, n, width, height, tiles_x, image,
                                             depth, depth_sq, normals, accum, pix_T, g_image, g_depth, g_depth_sq,
                                             g_normals, g_accum, (Splat2Grad*)grads);
}

void launch_pre2d_bwd(const float* means, const float* scales, const float* quats, const float* opac,
                      const float* sh, int n, int sh_k, const float* w2c, const CamParams& cp, const void* grads,
                      float* g_means, float* g_scales, float* g_quats, float* g_opac, float* g_sh,
                      cudaStream_t st) {
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("preprocess2d_bwd", st);
  launch_kernel_plain(k_pre2d_bwd, nb, 256, 0, st, means, scales, quats, opac, sh, n, sh_k, w2c, cp, (const Splat2Grad*)grads,
                                  g_means, g_scales, g_quats, g_opac, g_sh);
}

constexpr int kRegGrid = 296;

size_t reg2d_workspace_bytes() { return 256 + 2 * kRegGrid * sizeof(float); }

void launch_reg2d(const float* depth, const float* depth_sq, const float* normals, const float* accum, int h, int w,
                  float lam_dist, float lam_normal, float* dist_out, float* normal_out, float* g_depth,
                  float* g_depth_sq, float* g_normals, void* ws, cudaStream_t st) {
  RegScalars* rs = (RegScalars*)ws;
  float* part = (float*)((char*)ws + 256);
  cudaMemsetAsync(rs, 0, sizeof(RegScalars), st);
  GS_TIMED("regularizers2d", st);
  launch_kernel_plain(k_reg2d, kRegGrid, 256, 0, st, depth, depth_sq, normals, accum, h, w, lam_dist, lam_normal, part, rs,
                                    dist_out, normal_out, g_depth, g_depth_sq, g_normals);
}

void launch_adam_flat(float* p, const float* g, float* m, float* v, int count, float lr, float b1, float b2,
                      float omb1, float omb2, float inv_bc1, float inv_bc2, float eps, int* state, cudaStream_t st) {
  if (count <= 0) return;
  // the float4 path needs 16-byte aligned buffers
  const bool aligned = ((((uintptr_t)p) | ((uintptr_t)g) | ((uintptr_t)m) | ((uintptr_t)v)) & 15) == 0;
  GS_TIMED("adam_flat", st);
  if (!aligned) {
    launch_kernel_plain(k_adam_flat_scalar, device_sms() * 4, 256, 0, st, p, g, m, v, count, lr, b1, b2, omb1, omb2, inv_bc1, inv_bc2, eps,
                                            state);
    return;
  }
  launch_kernel_plain(k_adam_flat, device_sms() * 4, 256, 0, st, p, g, m, v, count, lr, b1, b2, omb1, omb2, inv_bc1, inv_bc2, eps, state);
}

}  // namespace gs
