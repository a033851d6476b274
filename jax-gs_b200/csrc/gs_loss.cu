// The training loss of the reference's step, (1 - lambda) L1 + lambda D-SSIM
// (jax_gs/training/trainer.py:18-26 over losses.py:4-8 and :16-75), with its
// gradient with respect to the rendered image, in two kernels:
//
//   k_loss_fwd  per 32x16 output tile and every channel: the halo tile of
//               pred and target in shared memory, the five 11-tap blurred
//               maps (separable, SAME zero padding), the SSIM map and the
//               three per-pixel coefficient maps of its gradient (written
//               planar, [c][y][x]), and the tile's sums of |pred - target|
//               and of the clamped SSIM map. The last CTA to finish (atomic
//               ticket) reduces the per-CTA sums in a fixed order -- the
//               result does not depend on scheduling -- and sets the loss
//               values and the D-SSIM gradient factor.
//   k_loss_bwd  per tile: blurs the coefficient maps (the window is
//               symmetric, so the adjoint blur is the same blur) and writes
//               dL/dpred = (1 - lambda) sign(pred - target) / count
//               + factor (blur(g_mu1) + 2 pred blur(g_s11) + target blur(g_s12)).
//
// Loads and stores of the interleaved (H, W, C) images walk whole tile rows
// (W x C contiguous floats), so they coalesce.
#include "gs_kernels.cuh"

namespace gs {

constexpr int kLTW = 32, kLTH = 16, kLR = 5, kLK = 11;
constexpr int kLLW = kLTW + 2 * kLR;  // 42
constexpr int kLLH = kLTH + 2 * kLR;  // 26
constexpr int kLMaxC = 3;

struct LossWin {
  float k[kLK];
};

struct LossScalars {
  unsigned ticket;
  float factor;  // lambda * d d_ssim / d mean(ssim_map) / count
  float pad[2];
};

__global__ void __launch_bounds__(256)
k_loss_fwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, int C, LossWin win,
           float lambda, float* __restrict__ gmu, float* __restrict__ gs11, float* __restrict__ gs12,
           float* __restrict__ part_ssim, float* __restrict__ part_l1, LossScalars* __restrict__ ls,
           float* __restrict__ l1_out, float* __restrict__ dssim_out, float* __restrict__ ssim_out,
           float* __restrict__ loss_out) {
  __shared__ float s_a[kLMaxC][kLLH][kLLW];
  __shared__ float s_b[kLMaxC][kLLH][kLLW];
  __shared__ float s_v[5][kLTH][kLLW];
  __shared__ float s_red[2][8];
  __shared__ double s_w[8];
  __shared__ bool s_last;
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kLTW, y0 = blockIdx.y * kLTH;
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  // halo tile, all channels: row r holds kLLW * C consecutive floats
  const int rowlen = kLLW * C;
  for (int e = tid; e < kLLH * rowlen; e += 256) {
    const int r = e / rowlen, u = e - r * rowlen;
    const int q = u / C, c = u - q * C;
    const int y = y0 + r - kLR, x = x0 + q - kLR;
    const bool in = (y >= 0) && (y < H) && (x >= 0) && (x < W);
    const size_t idx = ((size_t)y * W + x) * C + c;
    s_a[c][r][q] = in ? x1[idx] : 0.f;
    s_b[c][r][q] = in ? x2[idx] : 0.f;
  }
  __syncthreads();
  float acc_ssim = 0.f, acc_l1 = 0.f;
  const size_t plane = (size_t)H * W;
  for (int c = 0; c < C; ++c) {
    for (int e = tid; e < kLTH * kLLW; e += 256) {
      const int r = e / kLLW, q = e - r * kLLW;
      float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
      for (int i = 0; i < kLK; ++i) {
        const float a = s_a[c][r + i][q], b = s_b[c][r + i][q], k = win.k[i];
        m1 += k * a;
        m2 += k * b;
        e11 += k * (a * a);
        e22 += k * (b * b);
        e12 += k * (a * b);
      }
      s_v[0][r][q] = m1; s_v[1][r][q] = m2; s_v[2][r][q] = e11; s_v[3][r][q] = e22; s_v[4][r][q] = e12;
    }
    __syncthreads();
    // horizontal pass: each thread two neighbouring outputs from 12 loads per map
    for (int e = tid; e < kLTH * kLTW / 2; e += 256) {
      const int r = e / (kLTW / 2), q = 2 * (e - r * (kLTW / 2));
      float v0[5], v1[5];
#pragma unroll
      for (int p = 0; p < 5; ++p) {
        float w[kLK + 1];
#pragma unroll
        for (int j = 0; j <= kLK; ++j) w[j] = s_v[p][r][q + j];
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int j = 0; j < kLK; ++j) {
          t0 += win.k[j] * w[j];
          t1 += win.k[j] * w[j + 1];
        }
        v0[p] = t0;
        v1[p] = t1;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int y = y0 + r, x = x0 + q + h;
        if (y >= H || x >= W) continue;
        acc_l1 += fabsf(s_a[c][r + kLR][q + h + kLR] - s_b[c][r + kLR][q + h + kLR]);
        const float* v = h ? v1 : v0;
        const float mu1 = v[0], mu2 = v[1];
        const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
        const float s11r = v[2] - mu1_sq, s22r = v[3] - mu2_sq;
        const float s11 = fmaxf(0.f, s11r), s22 = fmaxf(0.f, s22r);
        const float s12 = v[4] - mu12;
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
    __syncthreads();
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

__global__ void __launch_bounds__(256)
k_loss_bwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, int C, LossWin win,
           float l1_scale, const float* __restrict__ gmu, const float* __restrict__ gs11,
           const float* __restrict__ gs12, const LossScalars* __restrict__ ls, float* __restrict__ grad) {
  __shared__ float s_m[3][kLLH][kLLW];
  __shared__ float s_v[3][kLTH][kLLW];
  // the tile's pred, target and gradient, interleaved like the image
  __shared__ float s_p[kLTH][kLTW * kLMaxC];
  __shared__ float s_t[kLTH][kLTW * kLMaxC];
  __shared__ float s_out[kLTH][kLTW * kLMaxC];
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kLTW, y0 = blockIdx.y * kLTH;
  const float factor = ls->factor;
  const size_t plane = (size_t)H * W;
  const int rowlen = kLTW * C;
  for (int e = tid; e < kLTH * rowlen; e += 256) {
    const int r = e / rowlen, u = e - r * rowlen;
    const int y = y0 + r, x = x0 + u / C;
    const bool in = y < H && x < W;
    const size_t idx = ((size_t)y * W + x0) * C + u;
    s_p[r][u] = in ? x1[idx] : 0.f;
    s_t[r][u] = in ? x2[idx] : 0.f;
  }
  for (int c = 0; c < C; ++c) {
    const float* maps[3] = {gmu + c * plane, gs11 + c * plane, gs12 + c * plane};
    for (int e = tid; e < kLLH * kLLW; e += 256) {
      const int r = e / kLLW, q = e - r * kLLW;
      const int y = y0 + r - kLR, x = x0 + q - kLR;
      const bool in = (y >= 0) && (y < H) && (x >= 0) && (x < W);
      const size_t idx = (size_t)y * W + x;
#pragma unroll
      for (int m = 0; m < 3; ++m) s_m[m][r][q] = in ? maps[m][idx] : 0.f;
    }
    __syncthreads();
    for (int e = tid; e < kLTH * kLLW; e += 256) {
      const int r = e / kLLW, q = e - r * kLLW;
      float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
      for (int i = 0; i < kLK; ++i) {
        const float k = win.k[i];
        a += k * s_m[0][r + i][q];
        b += k * s_m[1][r + i][q];
        d += k * s_m[2][r + i][q];
      }
      s_v[0][r][q] = a; s_v[1][r][q] = b; s_v[2][r][q] = d;
    }
    __syncthreads();
    for (int e = tid; e < kLTH * kLTW / 2; e += 256) {  // two outputs per thread
      const int r = e / (kLTW / 2), q = 2 * (e - r * (kLTW / 2));
      float o0[3], o1[3];
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        float w[kLK + 1];
#pragma unroll
        for (int j = 0; j <= kLK; ++j) w[j] = s_v[m][r][q + j];
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int j = 0; j < kLK; ++j) {
          t0 += win.k[j] * w[j];
          t1 += win.k[j] * w[j + 1];
        }
        o0[m] = t0;
        o1[m] = t1;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float* o = h ? o1 : o0;
        const int u = (q + h) * C + c;
        const float p = s_p[r][u], t = s_t[r][u];
        const float diff = p - t;
        const float l1g = (diff > 0.f) ? l1_scale : ((diff < 0.f) ? -l1_scale : 0.f);
        s_out[r][u] = l1g + factor * (o[0] + 2.f * p * o[1] + t * o[2]);
      }
    }
    __syncthreads();  // s_m / s_v reused by the next channel
  }
  // coalesced store of the tile's rows
  for (int e = tid; e < kLTH * rowlen; e += 256) {
    const int r = e / rowlen, u = e - r * rowlen;
    const int y = y0 + r, x = x0 + u / C;
    if (y < H && x < W) grad[((size_t)y * W + x0) * C + u] = s_out[r][u];
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
  const size_t nb = (size_t)((w + kLTW - 1) / kLTW) * ((h + kLTH - 1) / kLTH);
  return al256(sizeof(LossScalars)) + 2 * al256(nb * sizeof(float)) + 3 * map;
}

void launch_l1_dssim(const float* pred, const float* target, int h, int w, int c, float lambda,
                     float* l1_out, float* dssim_out, float* ssim_out, float* loss_out, float* grad, void* ws,
                     cudaStream_t st) {
  const size_t map = al256((size_t)h * w * c * sizeof(float));
  const dim3 grid((w + kLTW - 1) / kLTW, (h + kLTH - 1) / kLTH);
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
    k_loss_fwd<<<grid, 256, 0, st>>>(pred, target, h, w, c, win, lambda, grad ? gmu : nullptr, gs11, gs12,
                                     part_ssim, part_l1, ls, l1_out, dssim_out, ssim_out, loss_out);
  }
  if (grad) {
    GS_TIMED("loss_bwd", st);
    const float l1_scale = (1.f - lambda) / (float)((double)h * w * c);
    k_loss_bwd<<<grid, 256, 0, st>>>(pred, target, h, w, c, win, l1_scale, gmu, gs11, gs12, ls, grad);
  }
}

}  // namespace gs
