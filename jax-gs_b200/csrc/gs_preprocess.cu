// Per-Gaussian stages: projection + SH colour + tile rectangle (forward), the
// chain rule back to the Gaussian parameters (backward), and the small
// per-Gaussian kernels behind the stage-level entry points.
//
// One thread per Gaussian; every kernel is a flat grid over the static
// capacity N, so launch shapes never depend on data (graph-capturable).
#include "gs_kernels.cuh"

namespace gs {

// Camera centre -R^T t (jax_gs/core/camera.py:14-21).
__device__ __forceinline__ void cam_center(const Cam& cam, float c[3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
    c[i] = -(cam.W[0 * 4 + i] * cam.W[3] + cam.W[1 * 4 + i] * cam.W[7] + cam.W[2 * 4 + i] * cam.W[11]);
}

// ---------------------------------------------------------------------------
// Fused forward preprocess: renderer.py:36-49 + rasterizer.py:36-65 +
// rasterizer.py:146-156 for one Gaussian.
// Resident CTAs per SM the two per-Gaussian kernels ask of the compiler.
// Both are bound by global-load latency (long-scoreboard stalls; 72 and 127
// registers, 3 and 4 resident CTAs per SM), but capping registers for more
// CTAs measured slower at config 2: preprocess_bwd 23.1 us at 96 registers
// (5 CTAs) and 22.0 at 80 (6) against 20.8, preprocess_fwd 17.3 at 64
// registers (4 CTAs) against 17.2; the spills and the shorter load runs per
// thread cost more than the extra warps hide.
#ifndef GS_PRE_FWD_MIN_CTAS
#define GS_PRE_FWD_MIN_CTAS 1
#endif
#ifndef GS_PRE_BWD_MIN_CTAS
#define GS_PRE_BWD_MIN_CTAS 1
#endif
__global__ void __launch_bounds__(256, GS_PRE_FWD_MIN_CTAS)
k_preprocess_fwd(const float* __restrict__ means, const float* __restrict__ scales,
                 const float* __restrict__ quats, const float* __restrict__ opac,
                 const float* __restrict__ sh, int n, int sh_k, int sh_degree,
                 const uint8_t* __restrict__ mask, const float* __restrict__ w2c, CamParams cp,
                 Splat* __restrict__ splats, int2* __restrict__ bins,
                 int* __restrict__ block_counts,  // [pairs per block | visible per block]
                 float* __restrict__ radii_out, uint8_t* __restrict__ valid_out,
                 GsExtras* __restrict__ extras) {
  GS_PDL_ENTRY();
  __shared__ int s_red3[8][3];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  int count = 0, capv = 0;
  if (i < n) {
    Cam cam;
    load_cam_rows(w2c, cam);
    cam.fx = cp.fx; cam.fy = cp.fy; cam.cx = cp.cx; cam.cy = cp.cy;
    float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
    float sc[3] = {scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
    float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
    Proj p;
    project_one(m, sc, q, cam, p);
    bool valid = p.z > 0.01f;
    if (mask) valid = valid && (mask[i] != 0);
    radii_out[i] = p.radius;
    valid_out[i] = valid ? 1 : 0;
    Rect rc = tile_rect(p.u, p.v, p.radius, cp.width, cp.height);
    int nx = 0, ny = 0, tx0 = 0, ty0 = 0, dq = 0;
    if (valid && rc.on_screen) {
      int spx = rc.tx1 - rc.tx0 + 1, spy = rc.ty1 - rc.ty0 + 1;
      capv = (spx > kOffset || spy > kOffset) ? 1 : 0;  // renderer.py:73-75
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
      // rasterizer.py:147-153 conic with det clamp, :156 sigmoid
      float det = fmaxf(p.c00 * p.c11 - p.c01 * p.c01, 1e-6f);
      float ia = p.c11 / det, i01 = -p.c01 / det, ic = p.c00 / det;
      float op = sigmoidf(opac[i]);
      // renderer.py:40-49 view-dependent colour
      float cc[3];
      cam_center(cam, cc);
      float d0 = m[0] - cc[0], d1 = m[1] - cc[1], d2 = m[2] - cc[2];
      float inv = 1.f / sqrtf(d0 * d0 + d1 * d1 + d2 * d2);
      float col[3];
      float shv[48];
      load_sh_row(sh + (size_t)i * sh_k * 3, sh_k, sh_degree, shv);
      eval_sh_one(sh_degree, shv, d0 * inv, d1 * inv, d2 * inv, col);
      Splat s;
      s.a = make_float4(p.u, p.v, -0.5f * ia, -i01);
      s.b = make_float4(-0.5f * ic, op, fminf(fmaxf(col[0] + 0.5f, 0.f), 1.f),
                        fminf(fmaxf(col[1] + 0.5f, 0.f), 1.f));
      const float2 h = bbox_halfext(p.c00, p.c01, p.c11);
      s.c = make_float4(fminf(fmaxf(col[2] + 0.5f, 0.f), 1.f), h.x, h.y, p.z);
      splats[i] = s;
    }
  }
  // pairs, visible Gaussians and radius-cap violations of the block
  const int3 t = block_sum3_256(count, count > 0 ? 1 : 0, capv, s_red3);
  if (threadIdx.x == 0) {
    block_counts[blockIdx.x] = t.x;
    block_counts[gridDim.x + blockIdx.x] = t.y;
    if (t.z) atomicAdd(&extras->radius_cap_violations, t.z);
  }
}

// ---------------------------------------------------------------------------
// Stage: project_gaussians (projection.py:6-79).
__global__ void __launch_bounds__(256)
k_project(const float* __restrict__ means, const float* __restrict__ scales,
          const float* __restrict__ quats, int n, const uint8_t* __restrict__ mask,
          const float* __restrict__ w2c, CamParams cp, float* __restrict__ means2d,
          float* __restrict__ cov2d, float* __restrict__ radii, uint8_t* __restrict__ valid,
          float* __restrict__ depths) {
  GS_PDL_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  Cam cam;
  load_cam_rows(w2c, cam);
  cam.fx = cp.fx; cam.fy = cp.fy; cam.cx = cp.cx; cam.cy = cp.cy;
  float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
  float sc[3] = {scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
  float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
  Proj p;
  project_one(m, sc, q, cam, p);
  // cov2D[1,0] is its own sum of products (projection.py:164), not a copy of [0,1].
  float MS1[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float* S = p.Sig;
    float Sk0 = (k == 0) ? S[0] : (k == 1) ? S[1] : S[2];
    float Sk1 = (k == 0) ? S[1] : (k == 1) ? S[3] : S[4];
    float Sk2 = (k == 0) ? S[2] : (k == 1) ? S[4] : S[5];
    MS1[k] = add_rn(add_rn(mul_rn(p.Mj[3], Sk0), mul_rn(p.Mj[4], Sk1)), mul_rn(p.Mj[5], Sk2));
  }
  float cov10 = add_rn(add_rn(mul_rn(MS1[0], p.Mj[0]), mul_rn(MS1[1], p.Mj[1])), mul_rn(MS1[2], p.Mj[2]));
  means2d[2 * i] = p.u;
  means2d[2 * i + 1] = p.v;
  cov2d[4 * i + 0] = p.c00;
  cov2d[4 * i + 1] = p.c01;
  cov2d[4 * i + 2] = cov10;
  cov2d[4 * i + 3] = p.c11;
  radii[i] = p.radius;
  bool v = p.z > 0.01f;
  if (mask) v = v && (mask[i] != 0);
  valid[i] = v ? 1 : 0;
  depths[i] = p.z;
}

// Stage: get_covariance_3d (gaussians.py:58-93) alone. project_one's Sigma,
// evaluated for a mean on the optical axis of an identity camera (the camera
// does not enter Sigma), expanded to the symmetric (3,3): its [i][j] and
// [j][i] are the same sum of the same products in the same order.
__global__ void __launch_bounds__(256)
k_covariance_3d(const float* __restrict__ scales, const float* __restrict__ quats, int n,
                float* __restrict__ cov) {
  GS_PDL_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  Cam cam;
#pragma unroll
  for (int k = 0; k < 12; ++k) cam.W[k] = (k == 0 || k == 5 || k == 10) ? 1.f : 0.f;
  cam.fx = cam.fy = 1.f;
  cam.cx = cam.cy = 0.f;
  cam.width = cam.height = 1;
  cam.tiles_x = cam.tiles_y = 1;
  const float m[3] = {0.f, 0.f, 1.f};
  const float sc[3] = {scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
  const float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
  Proj p;
  project_one(m, sc, q, cam, p);
  const float* S = p.Sig;  // 00 01 02 11 12 22
  float* o = cov + 9 * (size_t)i;
  o[0] = S[0]; o[1] = S[1]; o[2] = S[2];
  o[3] = S[1]; o[4] = S[3]; o[5] = S[4];
  o[6] = S[2]; o[7] = S[4]; o[8] = S[5];
}

// Stage: eval_sh (sh.py:25-74).
__global__ void __launch_bounds__(256)
k_eval_sh(int deg, const float* __restrict__ sh, int n, int sh_k, const float* __restrict__ dirs,
          float* __restrict__ out) {
  GS_PDL_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float col[3];
  eval_sh_one(deg, sh + (size_t)i * sh_k * 3, dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2], col);
  out[3 * i] = col[0];
  out[3 * i + 1] = col[1];
  out[3 * i + 2] = col[2];
}

// Stage: tile rectangles from caller-supplied means2D / radii / valid / depth
// (get_tile_interactions, rasterizer.py:36-51).
__global__ void __launch_bounds__(256)
k_bin_prep(const float* __restrict__ means2d, const float* __restrict__ radii,
           const uint8_t* __restrict__ valid, const float* __restrict__ depths, int n, int width,
           int height, int2* __restrict__ bins, int* __restrict__ block_counts) {
  GS_PDL_ENTRY();
  __shared__ int s_red3[8][3];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  int count = 0;
  if (i < n) {
    float u = means2d[2 * i], v = means2d[2 * i + 1], r = radii[i];
    Rect rc = tile_rect(u, v, r, width, height);
    int nx = 0, ny = 0, tx0 = 0, ty0 = 0, dq = 0;
    if (valid[i] && rc.on_screen && rc.tx1 >= rc.tx0 && rc.ty1 >= rc.ty0) {
      nx = min(rc.tx1 - rc.tx0 + 1, kOffset);
      ny = min(rc.ty1 - rc.ty0 + 1, kOffset);
      tx0 = rc.tx0; ty0 = rc.ty0;
      dq = depth_key(depths[i]);
    }
    count = nx * ny;
    bins[i] = pack_bin(tx0, ty0, nx, ny, dq);
  }
  const int3 t = block_sum3_256(count, count > 0 ? 1 : 0, 0, s_red3);
  if (threadIdx.x == 0) {
    block_counts[blockIdx.x] = t.x;
    block_counts[gridDim.x + blockIdx.x] = t.y;
  }
}

// Stage: compositor records from caller-supplied means2D / cov2D / raw opacity
// / colours (render_tiles, rasterizer.py:146-156).
__global__ void __launch_bounds__(256)
k_pack_splats(const float* __restrict__ means2d, const float* __restrict__ cov2d,
              const float* __restrict__ opac, const float* __restrict__ colors, int n,
              Splat* __restrict__ splats) {
  GS_PDL_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float c00 = cov2d[4 * i], c01 = cov2d[4 * i + 1], c11 = cov2d[4 * i + 3];
  float det = fmaxf(c00 * c11 - c01 * c01, 1e-6f);
  Splat s;
  s.a = make_float4(means2d[2 * i], means2d[2 * i + 1], -0.5f * (c11 / det), -(-c01 / det));
  s.b = make_float4(-0.5f * (c00 / det), sigmoidf(opac[i]), colors[3 * i], colors[3 * i + 1]);
  const float2 h = bbox_halfext(c00, c01, c11);
  s.c = make_float4(colors[3 * i + 2], h.x, h.y, 0.f);
  splats[i] = s;
}

// Stage backward: compositor-record gradients -> means2D, cov2D, raw opacity,
// colour gradients (what jax.vjp of render_tiles returns).
__global__ void __launch_bounds__(256)
k_splat_grads_to_inputs(const float* __restrict__ cov2d, const float* __restrict__ opac,
                        const SplatGrad* __restrict__ sg, int n, float* __restrict__ g_means2d,
                        float* __restrict__ g_cov2d, float* __restrict__ g_opac,
                        float* __restrict__ g_colors) {
  GS_PDL_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  SplatGrad g = sg[i];
  if (g_means2d) {
    g_means2d[2 * i] = g.a.x;
    g_means2d[2 * i + 1] = g.a.y;
  }
  if (g_cov2d) {
    float g00, g01, g11;
    conic_backward(cov2d[4 * i], cov2d[4 * i + 1], cov2d[4 * i + 3], g.a.z, g.a.w, g.b.x, g00, g01,
                   g11);
    g_cov2d[4 * i] = g00;
    g_cov2d[4 * i + 1] = g01;
    g_cov2d[4 * i + 2] = 0.f;
    g_cov2d[4 * i + 3] = g11;
  }
  if (g_opac) {
    float s = sigmoidf(opac[i]);
    g_opac[i] = g.b.y * s * (1.f - s);
  }
  if (g_colors) {
    g_colors[3 * i] = g.b.z;
    g_colors[3 * i + 1] = g.b.w;
    g_colors[3 * i + 2] = g.c.x;
  }
}

// SH backward of one Gaussian: basis[k] receives the basis value Y_k(dir)
// (0 above the degree), so that d colour_c / d sh[k][c] = Y_k and the
// coefficient gradient is basis[k] * gcol[c]; gdir receives d(colour)/d(dir)
// contracted with the colour gradient.
__device__ __forceinline__ void sh_backward_one(int deg, const float* __restrict__ sh, float x, float y,
                                                float z, const float gcol[3], float* __restrict__ basis,
                                                float gdir[3]) {
  // basis values
  float b[16];
#pragma unroll
  for (int k = 1; k < 16; ++k) b[k] = 0.f;
  b[0] = kC0;
  int nb = 1;
  gdir[0] = gdir[1] = gdir[2] = 0.f;
  float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  if (deg > 0) {
    b[1] = -kC1 * y; b[2] = kC1 * z; b[3] = -kC1 * x;
    nb = 4;
    if (deg > 1) {
      b[4] = kC2_0 * xy; b[5] = kC2_1 * yz; b[6] = kC2_2 * (2.f * zz - xx - yy);
      b[7] = kC2_3 * xz; b[8] = kC2_4 * (xx - yy);
      nb = 9;
      if (deg > 2) {
        b[9] = kC3_0 * y * (3.f * xx - yy); b[10] = kC3_1 * xy * z;
        b[11] = kC3_2 * y * (4.f * zz - xx - yy); b[12] = kC3_3 * z * (2.f * zz - 3.f * xx - 3.f * yy);
        b[13] = kC3_4 * x * (4.f * zz - xx - yy); b[14] = kC3_5 * z * (xx - yy);
        b[15] = kC3_6 * x * (xx - 3.f * yy);
        nb = 16;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) basis[k] = (k < nb) ? b[k] : 0.f;
  if (deg == 0) return;
  // dot of each coefficient with the colour gradient
  float d[16];
#pragma unroll
  for (int k = 1; k < 16; ++k)
    d[k] = (k < nb) ? sh[3 * k] * gcol[0] + sh[3 * k + 1] * gcol[1] + sh[3 * k + 2] * gcol[2] : 0.f;
  float gx = -kC1 * d[3], gy = -kC1 * d[1], gz = kC1 * d[2];
  if (deg > 1) {
    gx += kC2_0 * y * d[4] + kC2_2 * (-2.f * x) * d[6] + kC2_3 * z * d[7] + kC2_4 * (2.f * x) * d[8];
    gy += kC2_0 * x * d[4] + kC2_1 * z * d[5] + kC2_2 * (-2.f * y) * d[6] + kC2_4 * (-2.f * y) * d[8];
    gz += kC2_1 * y * d[5] + kC2_2 * (4.f * z) * d[6] + kC2_3 * x * d[7];
    if (deg > 2) {
      gx += kC3_0 * y * (6.f * x) * d[9] + kC3_1 * yz * d[10] + kC3_2 * y * (-2.f * x) * d[11] +
            kC3_3 * z * (-6.f * x) * d[12] + kC3_4 * (4.f * zz - 3.f * xx - yy) * d[13] +
            kC3_5 * z * (2.f * x) * d[14] + kC3_6 * (3.f * xx - 3.f * yy) * d[15];
      gy += kC3_0 * (3.f * xx - 3.f * yy) * d[9] + kC3_1 * xz * d[10] +
            kC3_2 * (4.f * zz - xx - 3.f * yy) * d[11] + kC3_3 * z * (-6.f * y) * d[12] +
            kC3_4 * x * (-2.f * y) * d[13] + kC3_5 * z * (-2.f * y) * d[14] + kC3_6 * x * (-6.f * y) * d[15];
      gz += kC3_1 * xy * d[10] + kC3_2 * y * (8.f * z) * d[11] +
            kC3_3 * (6.f * zz - 3.f * xx - 3.f * yy) * d[12] + kC3_4 * x * (8.f * z) * d[13] +
            kC3_5 * (xx - yy) * d[14];
    }
  }
  gdir[0] = gx; gdir[1] = gy; gdir[2] = gz;
}

// ---------------------------------------------------------------------------
// Fused preprocess backward: the chain rule of renderer.py:36-49,
// projection.py:21-79, gaussians.py:58-93 and rasterizer.py:146-156 from the
// compositor-record gradients to the Gaussian parameters. One thread per
// Gaussian computes into shared memory; the CTA then writes each output
// array as one contiguous run (a thread-per-Gaussian store of 59 strided
// floats would make every store instruction touch 32 cache lines). The SH
// gradient, sh[k][c] -> Y_k gcol[c], is kept factored (16 basis values at an
// odd stride and 3 colour gradients per Gaussian: no bank conflicts) and
// multiplied out by the warp that stores it.
constexpr int kPBT = 128;
constexpr int kBasisStride = 17;

__device__ __forceinline__ void copy_out(float* __restrict__ dst, const float* __restrict__ src, int nf) {
  if ((((uintptr_t)dst) & 15) == 0) {
    const int n4 = nf >> 2;
    for (int j = threadIdx.x; j < n4; j += kPBT)
      reinterpret_cast<float4*>(dst)[j] = reinterpret_cast<const float4*>(src)[j];
    for (int j = 4 * n4 + threadIdx.x; j < nf; j += kPBT) dst[j] = src[j];
  } else {
    for (int j = threadIdx.x; j < nf; j += kPBT) dst[j] = src[j];
  }
}

__global__ void __launch_bounds__(kPBT, GS_PRE_BWD_MIN_CTAS)
k_preprocess_bwd(const float* __restrict__ means, const float* __restrict__ scales,
                 const float* __restrict__ quats, const float* __restrict__ opac,
                 const float* __restrict__ sh, int n, int sh_k, int sh_degree,
                 const float* __restrict__ w2c, CamParams cp, const SplatGrad* __restrict__ sgrad,
                 float* __restrict__ g_means, float* __restrict__ g_scales,
                 float* __restrict__ g_quats, float* __restrict__ g_opac,
                 float* __restrict__ g_sh, uint8_t* __restrict__ touched) {
  GS_PDL_ENTRY();
  __shared__ __align__(16) float s_m[kPBT * 3];
  __shared__ __align__(16) float s_s[kPBT * 3];
  __shared__ __align__(16) float s_q[kPBT * 4];
  __shared__ __align__(16) float s_o[kPBT];
  __shared__ float s_basis[kPBT * kBasisStride];
  __shared__ float s_gcol[kPBT * 3];
  const int tid = threadIdx.x;
  const int base = blockIdx.x * kPBT;
  const int i = base + tid;
  float* basis = s_basis + tid * kBasisStride;
  float* gcol = s_gcol + 3 * tid;
  float* gm_out = s_m + 3 * tid;
  float* gs_out = s_s + 3 * tid;
  float* gq_out = s_q + 4 * tid;
  SplatGrad gr;
  bool any = false;
  if (i < n) {
    gr = sgrad[i];
    any = (gr.a.x != 0.f) | (gr.a.y != 0.f) | (gr.a.z != 0.f) | (gr.a.w != 0.f) | (gr.b.x != 0.f) |
          (gr.b.y != 0.f) | (gr.b.z != 0.f) | (gr.b.w != 0.f) | (gr.c.x != 0.f);
    // 0: this Gaussian's whole gradient row is written as exact +0 below
    if (touched) touched[i] = any ? 1 : 0;
  }
  if (!any) {
    gm_out[0] = gm_out[1] = gm_out[2] = 0.f;
    gs_out[0] = gs_out[1] = gs_out[2] = 0.f;
    gq_out[0] = gq_out[1] = gq_out[2] = gq_out[3] = 0.f;
    s_o[tid] = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) basis[k] = 0.f;
    gcol[0] = gcol[1] = gcol[2] = 0.f;
  } else {
    Cam cam;
    load_cam_rows(w2c, cam);
    cam.fx = cp.fx; cam.fy = cp.fy; cam.cx = cp.cx; cam.cy = cp.cy;
    float m[3] = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
    float sc[3] = {scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]};
    float q[4] = {quats[4 * i], quats[4 * i + 1], quats[4 * i + 2], quats[4 * i + 3]};
    Proj p;
    project_one(m, sc, q, cam, p);
    const float* W = cam.W;
    float gm[3] = {0.f, 0.f, 0.f};
    // ---- colour path (renderer.py:40-49, sh.py) ----
    {
      float cc[3];
      cam_center(cam, cc);
      float v0 = m[0] - cc[0], v1 = m[1] - cc[1], v2 = m[2] - cc[2];
      float nrm = sqrtf(v0 * v0 + v1 * v1 + v2 * v2);
      float inv = 1.f / nrm;
      float dx = v0 * inv, dy = v1 * inv, dz = v2 * inv;
      float shi[48];
      load_sh_row(sh + (size_t)i * sh_k * 3, sh_k, sh_degree, shi);
      float col[3];
      eval_sh_one(sh_degree, shi, dx, dy, dz, col);
      float gin[3] = {gr.b.z, gr.b.w, gr.c.x};
      float gc[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        float raw = col[c] + 0.5f;
        // clip(x, 0, 1) = minimum(maximum(x, 0), 1): half weight at either bound.
        float w = (raw > 0.f && raw < 1.f) ? 1.f : ((raw == 0.f || raw == 1.f) ? 0.5f : 0.f);
        gc[c] = gin[c] * w;
        gcol[c] = gc[c];
      }
      float gdir[3];
      sh_backward_one(sh_degree, shi, dx, dy, dz, gc, basis, gdir);
      if (sh_degree > 0) {
        float dotg = dx * gdir[0] + dy * gdir[1] + dz * gdir[2];
        gm[0] += (gdir[0] - dx * dotg) * inv;
        gm[1] += (gdir[1] - dy * dotg) * inv;
        gm[2] += (gdir[2] - dz * dotg) * inv;
      }
    }
    // ---- opacity (rasterizer.py:156) ----
    {
      float s = sigmoidf(opac[i]);
      s_o[tid] = gr.b.y * s * (1.f - s);
    }
    // ---- conic -> cov2D (rasterizer.py:147-153) ----
    float g00, g01, g11;
    conic_backward(p.c00, p.c01, p.c11, gr.a.z, gr.a.w, gr.b.x, g00, g01, g11);
    // ---- cov2D = Mj Sigma Mj^T (projection.py:163-164) ----
    // loss depends on cov[0,1] only (cov[1,0] is unused): Gs = G + G^T.
    float Gs00 = 2.f * g00, Gs01 = g01, Gs11 = 2.f * g11;
    const float* Mj = p.Mj;
    float S[9] = {p.Sig[0], p.Sig[1], p.Sig[2], p.Sig[1], p.Sig[3], p.Sig[4], p.Sig[2], p.Sig[4], p.Sig[5]};
    float MS[6];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int k = 0; k < 3; ++k)
        MS[r * 3 + k] = Mj[r * 3 + 0] * S[0 * 3 + k] + Mj[r * 3 + 1] * S[1 * 3 + k] + Mj[r * 3 + 2] * S[2 * 3 + k];
    float dMj[6];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      dMj[k] = Gs00 * MS[k] + Gs01 * MS[3 + k];
      dMj[3 + k] = Gs01 * MS[k] + Gs11 * MS[3 + k];
    }
    // P = Mj^T Gs Mj (3x3), dL/dA = P A with A = R diag(s)
    float GM[6];  // Gs Mj
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      GM[k] = Gs00 * Mj[k] + Gs01 * Mj[3 + k];
      GM[3 + k] = Gs01 * Mj[k] + Gs11 * Mj[3 + k];
    }
    float P[9];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) P[a * 3 + b] = Mj[a] * GM[b] + Mj[3 + a] * GM[3 + b];
    float A[9];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) A[a * 3 + b] = p.R[a * 3 + b] * p.s[b];
    float dA[9];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        dA[a * 3 + b] = P[a * 3 + 0] * A[0 * 3 + b] + P[a * 3 + 1] * A[1 * 3 + b] + P[a * 3 + 2] * A[2 * 3 + b];
    float dR[9];
    float ds[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        dR[a * 3 + b] = dA[a * 3 + b] * p.s[b];
        ds[b] += dA[a * 3 + b] * p.R[a * 3 + b];
      }
    gs_out[0] = ds[0] * p.s[0];
    gs_out[1] = ds[1] * p.s[1];
    gs_out[2] = ds[2] * p.s[2];
    // rotation from quaternion (gaussians.py:78-82)
    {
      float r = p.qn[0], x = p.qn[1], y = p.qn[2], z = p.qn[3];
      float gr_ = 2.f * (-z * dR[1] + y * dR[2] + z * dR[3] - x * dR[5] - y * dR[6] + x * dR[7]);
      float gx = 2.f * (y * dR[1] + z * dR[2] + y * dR[3] - 2.f * x * dR[4] - r * dR[5] + z * dR[6] +
                        r * dR[7] - 2.f * x * dR[8]);
      float gy = 2.f * (-2.f * y * dR[0] + x * dR[1] + r * dR[2] + x * dR[3] + z * dR[5] - r * dR[6] +
                        z * dR[7] - 2.f * y * dR[8]);
      float gz = 2.f * (-2.f * z * dR[0] - r * dR[1] + x * dR[2] + r * dR[3] - 2.f * z * dR[4] +
                        y * dR[5] + x * dR[6] + y * dR[7]);
      // q / |q|  (gaussians.py:70)
      float dot = r * gr_ + x * gx + y * gy + z * gz;
      float in = 1.f / p.qnorm;
      gq_out[0] = (gr_ - r * dot) * in;
      gq_out[1] = (gx - x * dot) * in;
      gq_out[2] = (gy - y * dot) * in;
      gq_out[3] = (gz - z * dot) * in;
    }
    // ---- J (projection.py:150-157) ----
    float dJ00 = dMj[0] * W[0] + dMj[1] * W[1] + dMj[2] * W[2];
    float dJ02 = dMj[0] * W[8] + dMj[1] * W[9] + dMj[2] * W[10];
    float dJ11 = dMj[3] * W[4] + dMj[4] * W[5] + dMj[5] * W[6];
    float dJ12 = dMj[3] * W[8] + dMj[4] * W[9] + dMj[5] * W[10];
    float iz = p.inv_z, iz2 = iz * iz, iz3 = iz2 * iz;
    float gpx = dJ02 * (-cp.fx * iz2);
    float gpy = dJ12 * (-cp.fy * iz2);
    float gsz = dJ00 * (-cp.fx * iz2) + dJ02 * (2.f * cp.fx * p.x * iz3) + dJ11 * (-cp.fy * iz2) +
                dJ12 * (2.f * cp.fy * p.y * iz3);
    float gpz = gsz * tie_weight(p.z, 0.01f, true);
    // ---- means2D (projection.py:172-175), raw z ----
    {
      float mx = gr.a.x, my = gr.a.y;
      float izr = 1.f / p.z;
      gpx += mx * cp.fx * izr;
      gpy += my * cp.fy * izr;
      gpz += -(mx * cp.fx * p.x + my * cp.fy * p.y) * izr * izr;
    }
    // ---- means_cam = W_rot m + t ----
#pragma unroll
    for (int k = 0; k < 3; ++k) gm[k] += W[0 * 4 + k] * gpx + W[1 * 4 + k] * gpy + W[2 * 4 + k] * gpz;
    gm_out[0] = gm[0];
    gm_out[1] = gm[1];
    gm_out[2] = gm[2];
  }
  __syncthreads();
  const int cnt = min(kPBT, n - base);
  copy_out(g_means + 3 * (size_t)base, s_m, 3 * cnt);
  copy_out(g_scales + 3 * (size_t)base, s_s, 3 * cnt);
  copy_out(g_quats + 4 * (size_t)base, s_q, 4 * cnt);
  copy_out(g_opac + (size_t)base, s_o, cnt);
  // g_sh rows of L = 3 sh_k floats: warp w stores rows w, w + 4, ..., lane
  // l element l (and l + 32) of each, (k, c) = divmod(element, 3)
  {
    const int L = 3 * sh_k, warp = tid >> 5, lane = tid & 31;
    const int k0 = lane / 3, c0 = lane - 3 * k0;
    const int k1 = (lane + 32) / 3, c1 = lane + 32 - 3 * k1;
    float* dst = g_sh + (size_t)L * base;
    for (int g = warp; g < cnt; g += kPBT / 32) {
      const float* bs = s_basis + g * kBasisStride;
      const float* gc = s_gcol + 3 * g;
      if (lane < L) dst[(size_t)g * L + lane] = bs[k0] * gc[c0];
      if (lane + 32 < L) dst[(size_t)g * L + lane + 32] = bs[k1] * gc[c1];
    }
  }
}

// ---------------------------------------------------------------------------
// Host launchers.
void launch_preprocess_fwd(const float* means, const float* scales, const float* quats,
                           const float* opac, const float* sh, int n, int sh_k, int sh_degree,
                           const uint8_t* mask, const float* w2c, const CamParams& cp, Splat* splats,
                           int2* bins, int* block_counts, float* radii, uint8_t* valid,
                           GsExtras* extras, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("preprocess_fwd", st);
  launch_kernel(k_preprocess_fwd, nb, 256, 0, st, means, scales, quats, opac, sh, n, sh_k, sh_degree, mask, w2c,
                                       cp, splats, bins, block_counts, radii, valid, extras);
}

void launch_project(const float* means, const float* scales, const float* quats, int n,
                    const uint8_t* mask, const float* w2c, const CamParams& cp, float* means2d,
                    float* cov2d, float* radii, uint8_t* valid, float* depths, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("project", st);
  launch_kernel(k_project, nb, 256, 0, st, means, scales, quats, n, mask, w2c, cp, means2d, cov2d, radii, valid,
                                depths);
}

void launch_eval_sh(int deg, const float* sh, int n, int sh_k, const float* dirs, float* out,
                    cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("eval_sh", st);
  launch_kernel(k_eval_sh, nb, 256, 0, st, deg, sh, n, sh_k, dirs, out);
}

void launch_covariance_3d(const float* scales, const float* quats, int n, float* cov, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("covariance_3d", st);
  launch_kernel(k_covariance_3d, nb, 256, 0, st, scales, quats, n, cov);
}

void launch_bin_prep(const float* means2d, const float* radii, const uint8_t* valid,
                     const float* depths, int n, int width, int height, int2* bins,
                     int* block_counts, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("bin_prep", st);
  launch_kernel(k_bin_prep, nb, 256, 0, st, means2d, radii, valid, depths, n, width, height, bins, block_counts);
}

void launch_pack_splats(const float* means2d, const float* cov2d, const float* opac,
                        const float* colors, int n, Splat* splats, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("pack_splats", st);
  launch_kernel(k_pack_splats, nb, 256, 0, st, means2d, cov2d, opac, colors, n, splats);
}

void launch_splat_grads_to_inputs(const float* cov2d, const float* opac, const SplatGrad* sg, int n,
                                  float* g_means2d, float* g_cov2d, float* g_opac, float* g_colors,
                                  cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("splat_grads_to_inputs", st);
  launch_kernel(k_splat_grads_to_inputs, nb, 256, 0, st, cov2d, opac, sg, n, g_means2d, g_cov2d, g_opac, g_colors);
}

void launch_preprocess_bwd(const float* means, const float* scales, const float* quats,
                           const float* opac, const float* sh, int n, int sh_k, int sh_degree,
                           const float* w2c, const CamParams& cp, const SplatGrad* sg,
                           float* g_means, float* g_scales, float* g_quats, float* g_opac,
                           float* g_sh, uint8_t* touched, cudaStream_t st) {
  int nb = (n + kPBT - 1) / kPBT;
  if (nb == 0) return;
  GS_TIMED("preprocess_bwd", st);
  launch_kernel(k_preprocess_bwd, nb, kPBT, 0, st, means, scales, quats, opac, sh, n, sh_k, sh_degree, w2c, cp, sg,
                                       g_means, g_scales, g_quats, g_opac, g_sh, touched);
}

}  // namespace gs
