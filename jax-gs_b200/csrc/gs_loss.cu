// The training loss of the reference's step, (1 - lambda) L1 + lambda D-SSIM
// (jax_gs/training/trainer.py:18-26 over losses.py:4-8 and :16-75), with its
// gradient with respect to the rendered image, in two kernels:
//
//   k_loss_fwd  per 32x16 output tile and every channel: the halo tile of
//               pred and target in shared memory (asynchronous copies, whole
//               interleaved rows of W x C floats), the
//               five 11-tap blurred maps (separable, SAME zero padding; each
//               thread blurs a run of outputs from inputs held in
//               registers), the SSIM map and the
//               three per-pixel coefficient maps of its gradient (written
//               planar, [c][y][x]), and the tile's sums of |pred - target|
//               and of the clamped SSIM map. The last CTA to finish (atomic
//               ticket) reduces the per-CTA sums in a fixed order -- the
//               result does not depend on scheduling -- and sets the loss
//               values and the D-SSIM gradient factor.
//   k_loss_bwd  per tile and channel (one CTA each, so the channels run
//               side by side): blurs the channel's coefficient maps (the
//               window is symmetric, so the adjoint blur is the same blur)
//               and writes that channel of
//               dL/dpred = (1 - lambda) sign(pred - target) / count
//               + factor (blur(g_mu1) + 2 pred blur(g_s11) + target blur(g_s12)).
//               It reads and writes every C-th float of the interleaved
//               (H, W, C) rows; the C CTAs of a tile touch the same lines,
//               which L2 merges. Measured against one CTA per tile for all
//               channels (the channels one after another behind six
//               barriers at about 21 warps per SM): 14.8 vs 18.9 us at
//               504x378, 94 vs 105 us at 1920x1080. The same split of the
//               forward measured 18.4 vs 18.8 and 101.6 vs 90 us, so the
//               forward keeps a CTA per tile.
#include "gs_kernels.cuh"

namespace gs {

constexpr int kLTW = 32, kLTH = 16, kLR = 5, kLK = 11;
constexpr int kLLW = kLTW + 2 * kLR;  // 42
constexpr int kLLH = kLTH + 2 * kLR;  // 26
constexpr int kLVR = 4;               // rows per thread in the vertical pass
constexpr int kLHX = 2;               // columns per thread in the horizontal pass

struct LossWin {
  float k[kLK];
};

struct LossScalars {
  unsigned ticket;
  float factor;  // lambda * d d_ssim / d mean(ssim_map) / count
  float pad[2];
};

// 4-byte asynchronous copy global -> shared; ok = false writes 0 and reads
// nothing (src must still be a valid address).
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, bool ok) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa), "l"(gmem), "r"(ok ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Register-blocked taps: out[o] = sum_i k[i] in[o + i] (i ascending, one
// fused multiply-add per tap) for NO consecutive outputs from NO + 10
// inputs, the outputs taken in pairs on paired-fp32 FMAs (FFMA2: each lane
// rounds like a scalar FMA). A tap that exists for one output of a pair only
// (the pair's first and last) stays scalar, so no input outside an output's
// window enters it, not even as 0 * x.
template <int NO>
__device__ __forceinline__ void blur_run_x2(const float* in, const LossWin& win, float* out) {
  static_assert(NO % 2 == 0, "outputs in pairs");
  float2 acc[NO / 2];
#pragma unroll
  for (int p = 0; p < NO / 2; ++p) acc[p] = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NO + kLK - 1; ++j) {
#pragma unroll
    for (int p = 0; p < NO / 2; ++p) {
      const int i0 = j - 2 * p, i1 = j - 2 * p - 1;  // tap of each output of the pair
      const bool b0 = i0 >= 0 && i0 < kLK, b1 = i1 >= 0 && i1 < kLK;
      if (b0 && b1)
        acc[p] = __ffma2_rn(make_float2(win.k[i0], win.k[i1]), make_float2(in[j], in[j]), acc[p]);
      else if (b0)
        acc[p].x = __fmaf_rn(win.k[i0], in[j], acc[p].x);
      else if (b1)
        acc[p].y = __fmaf_rn(win.k[i1], in[j], acc[p].y);
    }
  }
#pragma unroll
  for (int p = 0; p < NO / 2; ++p) {
    out[2 * p] = acc[p].x;
    out[2 * p + 1] = acc[p].y;
  }
}

// Rows [0, rows) of a tile-shaped region copied to shared memory by the
// CTA's NW warps: row r (global row y_first + r) holds `rowlen` elements,
// element u read at offset col0 + u * ES of the image row (ES = 1 for a
// planar map, C for one channel of an interleaved image); `valid(u)` says
// whether element u lies inside the image.
template <int ROWLEN, int ROWS, int PITCH, int ES, int NW, typename V>
__device__ __forceinline__ void copy_rows(float* dst, const float* __restrict__ src, int H, long long row_stride,
                                          long long col0, int y_first, V valid, int warp, int lane) {
  for (int r = warp; r < ROWS; r += NW) {
    const int y = y_first + r;
    const bool yin = (y >= 0) && (y < H);
    const float* row = src + (long long)y * row_stride + col0;
#pragma unroll
    for (int u = lane; u < ROWLEN; u += 32) {
      const bool ok = yin && valid(u);
      cp_async4(dst + r * PITCH + u, ok ? row + (long long)u * ES : src, ok);
    }
  }
}

// Threads of a k_loss_bwd CTA; one CTA per (32x16 output tile, channel), so
// a 504x378 RGB image gives 1152 CTAs of 128 threads, resident at once.
constexpr int kLT = 128;
constexpr int kLW = kLT / 32;

template <int C>
__global__ void __launch_bounds__(256)
k_loss_fwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, LossWin win,
           float lambda, float* __restrict__ gmu, float* __restrict__ gs11, float* __restrict__ gs12,
           float* __restrict__ part_ssim, float* __restrict__ part_l1, LossScalars* __restrict__ ls,
           float* __restrict__ l1_out, float* __restrict__ dssim_out, float* __restrict__ ssim_out,
           float* __restrict__ loss_out) {
  GS_PDL_ENTRY_PLAIN();
  // halo tile, interleaved like the image: row r holds kLLW * C floats
  __shared__ float s_a[kLLH][kLLW * C];
  __shared__ float s_b[kLLH][kLLW * C];
  __shared__ float s_v[5][kLTH][kLLW];
  __shared__ float s_red[2][8];
  __shared__ double s_w[8];
  __shared__ bool s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int x0 = blockIdx.x * kLTW, y0 = blockIdx.y * kLTH;
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  {
    auto valid = [&](int u) {
      const int x = x0 - kLR + u / C;
      return x >= 0 && x < W;
    };
    const long long col0 = (long long)(x0 - kLR) * C;
    copy_rows<kLLW * C, kLLH, kLLW * C, 1, 8>(&s_a[0][0], x1, H, (long long)W * C, col0, y0 - kLR, valid, warp, lane);
    copy_rows<kLLW * C, kLLH, kLLW * C, 1, 8>(&s_b[0][0], x2, H, (long long)W * C, col0, y0 - kLR, valid, warp, lane);
    cp_async_wait_all();
  }
  __syncthreads();
  float acc_ssim = 0.f, acc_l1 = 0.f;
  const size_t plane = (size_t)H * W;
  constexpr int nvr = kLTH / kLVR, nhx = kLTW / kLHX;
  for (int c = 0; c < C; ++c) {
    // vertical pass: thread = (column, run of kLVR rows)
    for (int it = tid; it < kLLW * nvr; it += 256) {
      const int q = it / nvr, r0 = (it - q * nvr) * kLVR;
      // (mu1, mu2) and (e11, e22) share each tap weight: paired-fp32 FMAs,
      // each lane the same rounding and order as a scalar FMA
      float2 mm[kLVR], ee[kLVR];
      float e12[kLVR];
#pragma unroll
      for (int o = 0; o < kLVR; ++o) {
        mm[o] = ee[o] = make_float2(0.f, 0.f);
        e12[o] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < kLVR + kLK - 1; ++j) {
        const float a = s_a[r0 + j][q * C + c], b = s_b[r0 + j][q * C + c];
        const float2 ab2 = make_float2(a, b);
        const float2 sq = __fmul2_rn(ab2, ab2);
        const float ab = __fmul_rn(a, b);
#pragma unroll
        for (int o = 0; o < kLVR; ++o) {
          if (j - o >= 0 && j - o < kLK) {
            const float k = win.k[j - o];
            const float2 k2 = make_float2(k, k);
            mm[o] = __ffma2_rn(k2, ab2, mm[o]);
            ee[o] = __ffma2_rn(k2, sq, ee[o]);
            e12[o] = __fmaf_rn(k, ab, e12[o]);
          }
        }
      }
#pragma unroll
      for (int o = 0; o < kLVR; ++o) {
        s_v[0][r0 + o][q] = mm[o].x;
        s_v[1][r0 + o][q] = mm[o].y;
        s_v[2][r0 + o][q] = ee[o].x;
        s_v[3][r0 + o][q] = ee[o].y;
        s_v[4][r0 + o][q] = e12[o];
      }
    }
    __syncthreads();
    // horizontal pass + SSIM: thread = (row, run of kLHX columns)
    for (int it = tid; it < kLTH * nhx; it += 256) {
      const int r = it / nhx, q0 = (it - r * nhx) * kLHX;
      float v[5][kLHX];
#pragma unroll
      for (int p = 0; p < 5; ++p) {
        float w[kLHX + kLK - 1];
#pragma unroll
        for (int j = 0; j < kLHX + kLK - 1; ++j) w[j] = s_v[p][r][q0 + j];
        blur_run_x2<kLHX>(w, win, v[p]);
      }
#pragma unroll
      for (int h = 0; h < kLHX; ++h) {
        const int y = y0 + r, x = x0 + q0 + h;
        if (y >= H || x >= W) continue;
        const int u = (q0 + h + kLR) * C + c;
        acc_l1 += fabsf(s_a[r + kLR][u] - s_b[r + kLR][u]);
        const float mu1 = v[0][h], mu2 = v[1][h];
        const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
        const float s11r = v[2][h] - mu1_sq, s22r = v[3][h] - mu2_sq;
        const float s11 = fmaxf(0.f, s11r), s22 = fmaxf(0.f, s22r);
        const float s12 = v[4][h] - mu12;
        const float A = 2.f * mu12 + C1, B = 2.f * s12 + C2;
        const float Cc = mu1_sq + mu2_sq + C1, D = s11 + s22 + C2;
        const float map = (A * B) / (Cc * D);
        acc_ssim += fminf(fmaxf(map, -1.f), 1.f);
        if (gmu) {
          // clip's and maximum's ties pass half the cotangent (JAX)
          const float g = (map > -1.f && map < 1.f) ? 1.f : ((map == -1.f || map == 1.f) ? 0.5f : 0.f);
          const float inv = 1.f / (Cc * D);
          const float gA = g * B * inv, gB = g * A * inv, gC = -g * map / Cc, gD = -g * map / D;
          const float w11 = (s11r > 0.f) ? 1.f : ((s11r == 0.f) ? 0.5f : 0.f);
          const float g_s12 = 2.f * gB;
          const float g_s11 = gD * w11;
          const float g_mu1 = 2.f * mu2 * gA + 2.f * mu1 * gC - mu2 * g_s12 - 2.f * mu1 * g_s11;
          const size_t pidx = c * plane + (size_t)y * W + x;
          gmu[pidx] = g_mu1;
          gs11[pidx] = g_s11;
          gs12[pidx] = g_s12;
        }
      }
    }
    __syncthreads();  // s_v reused by the next channel
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_ssim += __shfl_down_sync(0xffffffffu, acc_ssim, o);
    acc_l1 += __shfl_down_sync(0xffffffffu, acc_l1, o);
  }
  if ((tid & 31) == 0) {
    s_red[0][tid >> 5] = acc_ssim;
    s_red[1][tid >> 5] = acc_l1;
  }
  __syncthreads();
  const unsigned nblocks = gridDim.x * gridDim.y;
  const unsigned bid = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) {
    float t0 = 0.f, t1 = 0.f;
    for (int w = 0; w < 8; ++w) {
      t0 += s_red[0][w];
      t1 += s_red[1][w];
    }
    part_ssim[bid] = t0;
    part_l1[bid] = t1;
    __threadfence();
    s_last = (atomicAdd(&ls->ticket, 1u) == nblocks - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double ts = 0.0, tl = 0.0;
  for (unsigned b = tid; b < nblocks; b += 256) {
    ts += (double)((volatile float*)part_ssim)[b];
    tl += (double)((volatile float*)part_l1)[b];
  }
  ts = block_sum_d256(ts, s_w);
  tl = block_sum_d256(tl, s_w);
  if (tid == 0) {
    const double cnt = (double)H * W * C;
    const float mean = (float)(ts / cnt);
    const float l1 = (float)(tl / cnt);
    const float d = (1.f - mean) / 2.f;
    const float dssim = fmaxf(0.f, d);
    const float w = (d > 0.f) ? 1.f : ((d == 0.f) ? 0.5f : 0.f);
    if (l1_out) *l1_out = l1;
    if (dssim_out) *dssim_out = dssim;
    if (ssim_out) *ssim_out = mean;
    if (loss_out) *loss_out = (1.f - lambda) * l1 + lambda * dssim;
    ls->factor = (float)(lambda * w * -0.5 / cnt);
    ls->ticket = 0u;
  }
}

template <int C>
__global__ void __launch_bounds__(kLT)
k_loss_bwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, LossWin win,
           float l1_scale, const float* __restrict__ gmu, const float* __restrict__ gs11,
           const float* __restrict__ gs12, const LossScalars* __restrict__ ls, float* __restrict__ grad) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_m[3][kLLH][kLLW];
  __shared__ float s_v[3][kLTH][kLLW];
  // the tile's pred and target in this channel
  __shared__ float s_p[kLTH][kLTW];
  __shared__ float s_t[kLTH][kLTW];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int x0 = blockIdx.x * kLTW, y0 = blockIdx.y * kLTH, c = blockIdx.z;
  const float factor = ls->factor;
  const size_t plane = (size_t)H * W;
  {
    auto valid = [&](int u) { return x0 + u < W; };
    const long long col0 = (long long)x0 * C + c;
    copy_rows<kLTW, kLTH, kLTW, C, kLW>(&s_p[0][0], x1, H, (long long)W * C, col0, y0, valid, warp, lane);
    copy_rows<kLTW, kLTH, kLTW, C, kLW>(&s_t[0][0], x2, H, (long long)W * C, col0, y0, valid, warp, lane);
    // halo tiles of the channel's three coefficient maps (planar rows)
    auto valid_m = [&](int u) {
      const int x = x0 - kLR + u;
      return x >= 0 && x < W;
    };
    copy_rows<kLLW, kLLH, kLLW, 1, kLW>(&s_m[0][0][0], gmu + c * plane, H, W, x0 - kLR, y0 - kLR, valid_m, warp,
                                        lane);
    copy_rows<kLLW, kLLH, kLLW, 1, kLW>(&s_m[1][0][0], gs11 + c * plane, H, W, x0 - kLR, y0 - kLR, valid_m, warp,
                                        lane);
    copy_rows<kLLW, kLLH, kLLW, 1, kLW>(&s_m[2][0][0], gs12 + c * plane, H, W, x0 - kLR, y0 - kLR, valid_m, warp,
                                        lane);
    cp_async_wait_all();
  }
  __syncthreads();
  constexpr int nvr = kLTH / kLVR, nhx = kLTW / kLHX;
  // vertical pass: thread = (map, column, run of kLVR rows)
  for (int it = tid; it < 3 * kLLW * nvr; it += kLT) {
    const int m = it / (kLLW * nvr), rem = it - m * (kLLW * nvr);
    const int q = rem / nvr, r0 = (rem - q * nvr) * kLVR;
    float a[kLVR + kLK - 1], o[kLVR];
#pragma unroll
    for (int j = 0; j < kLVR + kLK - 1; ++j) a[j] = s_m[m][r0 + j][q];
    blur_run_x2<kLVR>(a, win, o);
#pragma unroll
    for (int k = 0; k < kLVR; ++k) s_v[m][r0 + k][q] = o[k];
  }
  __syncthreads();
  // horizontal pass and the gradient: thread = (row, run of kLHX columns);
  // written in place into the interleaved (H, W, C) gradient
  for (int it = tid; it < kLTH * nhx; it += kLT) {
    const int r = it / nhx, q0 = (it - r * nhx) * kLHX;
    float o[3][kLHX];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      float w[kLHX + kLK - 1];
#pragma unroll
      for (int j = 0; j < kLHX + kLK - 1; ++j) w[j] = s_v[m][r][q0 + j];
      blur_run_x2<kLHX>(w, win, o[m]);
    }
#pragma unroll
    for (int h = 0; h < kLHX; ++h) {
      const int y = y0 + r, x = x0 + q0 + h;
      if (y >= H || x >= W) continue;
      const float p = s_p[r][q0 + h], t = s_t[r][q0 + h];
      const float diff = p - t;
      const float l1g = (diff > 0.f) ? l1_scale : ((diff < 0.f) ? -l1_scale : 0.f);
      grad[((size_t)y * W + x) * C + c] = l1g + factor * (o[0][h] + 2.f * p * o[1][h] + t * o[2][h]);
    }
  }
}

static LossWin loss_window() {
  // losses.py:193-198: exp(-x^2 / (2 sigma^2)) normalised, x = -5..5, sigma 1.5
  LossWin w;
  double k[kLK], s = 0.0;
  for (int i = 0; i < kLK; ++i) {
    double x = (double)(i - kLR);
    k[i] = (double)(float)exp((double)(float)(-(x * x) / 4.5));
    s += k[i];
  }
  for (int i = 0; i < kLK; ++i) w.k[i] = (float)(k[i] / s);
  return w;
}

static inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t l1_dssim_workspace_bytes(int h, int w, int c) {
  const size_t map = al256((size_t)h * w * c * sizeof(float));
  const size_t nb = (size_t)((w + kLTW - 1) / kLTW) * ((h + kLTH - 1) / kLTH);  // k_loss_fwd CTAs
  return al256(sizeof(LossScalars)) + 2 * al256(nb * sizeof(float)) + 3 * map;
}

void launch_l1_dssim(const float* pred, const float* target, int h, int w, int c, float lambda,
                     float* l1_out, float* dssim_out, float* ssim_out, float* loss_out, float* grad, void* ws,
                     cudaStream_t st) {
  const size_t map = al256((size_t)h * w * c * sizeof(float));
  const dim3 grid((w + kLTW - 1) / kLTW, (h + kLTH - 1) / kLTH);     // k_loss_fwd: a tile, all channels
  const dim3 grid_c((w + kLTW - 1) / kLTW, (h + kLTH - 1) / kLTH, c);  // k_loss_bwd: a tile and channel
  const size_t nb = (size_t)grid.x * grid.y;
  char* base = (char*)ws;
  LossScalars* ls = (LossScalars*)base;
  float* part_ssim = (float*)(base + al256(sizeof(LossScalars)));
  float* part_l1 = (float*)(base + al256(sizeof(LossScalars)) + al256(nb * sizeof(float)));
  float* gmu = (float*)(base + al256(sizeof(LossScalars)) + 2 * al256(nb * sizeof(float)));
  float* gs11 = (float*)((char*)gmu + map);
  float* gs12 = (float*)((char*)gmu + 2 * map);
  const LossWin win = loss_window();
  cudaMemsetAsync(ls, 0, sizeof(LossScalars), st);
  {
    GS_TIMED("loss_fwd", st);
#define GS_LOSS_FWD(CC)                                                                                     \
  launch_kernel_plain(k_loss_fwd<CC>, grid, 256, 0, st, pred, target, h, w, win, lambda, grad ? gmu : nullptr, gs11, gs12, \
                                       part_ssim, part_l1, ls, l1_out, dssim_out, ssim_out, loss_out)
    if (c == 1) GS_LOSS_FWD(1); else if (c == 2) GS_LOSS_FWD(2); else GS_LOSS_FWD(3);
#undef GS_LOSS_FWD
  }
  if (grad) {
    GS_TIMED("loss_bwd", st);
    const float l1_scale = (1.f - lambda) / (float)((double)h * w * c);
#define GS_LOSS_BWD(CC) \
  launch_kernel_plain(k_loss_bwd<CC>, grid_c, kLT, 0, st, pred, target, h, w, win, l1_scale, gmu, gs11, gs12, ls, grad)
    if (c == 1) GS_LOSS_BWD(1); else if (c == 2) GS_LOSS_BWD(2); else GS_LOSS_BWD(3);
#undef GS_LOSS_BWD
  }
}

}  // namespace gs
