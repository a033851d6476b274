// D-SSIM loss (jax_gs/training/losses.py:16-75) forward and gradient.
//
// ssim uses an 11-tap Gaussian window (sigma 1.5) applied separably, first
// along H then along W, with SAME zero padding, per channel. The forward
// kernel computes the five blurred maps of a 32x16 output tile from a
// shared-memory halo tile, the SSIM map, its mean (deterministic last-CTA
// reduction) and three per-pixel coefficient maps; the backward kernel blurs
// those maps (the window is symmetric, so the adjoint blur is the same blur)
// and forms dL/dpred = blur(g_mu1) + 2 pred blur(g_s11) + target blur(g_s12).
#include "gs_kernels.cuh"

namespace gs {

constexpr int kSsimTW = 32, kSsimTH = 16, kSsimR = 5, kSsimK = 11;
constexpr int kSsimLW = kSsimTW + 2 * kSsimR;  // 42
constexpr int kSsimLH = kSsimTH + 2 * kSsimR;  // 26

struct SsimWin {
  float k[kSsimK];
};

struct SsimScalars {
  unsigned ticket;
  float factor;  // scale * d loss / d mean(ssim_map) (includes the 1/count)
  float pad[2];
};

__global__ void __launch_bounds__(256)
k_ssim_fwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, int C,
           SsimWin win, float scale, float* __restrict__ gmu, float* __restrict__ gs11,
           float* __restrict__ gs12, float* __restrict__ partials, SsimScalars* __restrict__ ss,
           float* __restrict__ loss, float* __restrict__ ssim_out) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_a[kSsimLH][kSsimLW];
  __shared__ float s_b[kSsimLH][kSsimLW];
  __shared__ float s_v[5][kSsimTH][kSsimLW];
  __shared__ float s_red[8];
  __shared__ double s_w[8];
  __shared__ bool s_last;
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kSsimTW, y0 = blockIdx.y * kSsimTH;
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  float acc = 0.f;
  for (int c = 0; c < C; ++c) {
    for (int e = tid; e < kSsimLH * kSsimLW; e += 256) {
      int r = e / kSsimLW, q = e - r * kSsimLW;
      int y = y0 + r - kSsimR, x = x0 + q - kSsimR;
      bool in = (y >= 0) && (y < H) && (x >= 0) && (x < W);
      size_t idx = ((size_t)y * W + x) * C + c;
      s_a[r][q] = in ? x1[idx] : 0.f;
      s_b[r][q] = in ? x2[idx] : 0.f;
    }
    __syncthreads();
    for (int e = tid; e < kSsimTH * kSsimLW; e += 256) {
      int r = e / kSsimLW, q = e - r * kSsimLW;
      float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
      for (int i = 0; i < kSsimK; ++i) {
        float a = s_a[r + i][q], b = s_b[r + i][q], k = win.k[i];
        m1 += k * a;
        m2 += k * b;
        e11 += k * (a * a);
        e22 += k * (b * b);
        e12 += k * (a * b);
      }
      s_v[0][r][q] = m1; s_v[1][r][q] = m2; s_v[2][r][q] = e11; s_v[3][r][q] = e22; s_v[4][r][q] = e12;
    }
    __syncthreads();
    for (int e = tid; e < kSsimTH * kSsimTW; e += 256) {
      int r = e / kSsimTW, q = e - r * kSsimTW;
      int y = y0 + r, x = x0 + q;
      if (y >= H || x >= W) continue;
      float v[5];
#pragma unroll
      for (int p = 0; p < 5; ++p) {
        float t = 0.f;
#pragma unroll
        for (int j = 0; j < kSsimK; ++j) t += win.k[j] * s_v[p][r][q + j];
        v[p] = t;
      }
      float mu1 = v[0], mu2 = v[1];
      float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
      float s11r = v[2] - mu1_sq, s22r = v[3] - mu2_sq;
      float s11 = fmaxf(0.f, s11r), s22 = fmaxf(0.f, s22r);
      float s12 = v[4] - mu12;
      float A = 2.f * mu12 + C1, B = 2.f * s12 + C2;
      float Cc = mu1_sq + mu2_sq + C1, D = s11 + s22 + C2;
      float map = (A * B) / (Cc * D);
      acc += fminf(fmaxf(map, -1.f), 1.f);
      float g = (map > -1.f && map < 1.f) ? 1.f : ((map == -1.f || map == 1.f) ? 0.5f : 0.f);
      float inv = 1.f / (Cc * D);
      float gA = g * B * inv, gB = g * A * inv, gC = -g * map / Cc, gD = -g * map / D;
      float w11 = (s11r > 0.f) ? 1.f : ((s11r == 0.f) ? 0.5f : 0.f);
      float g_s12 = 2.f * gB;
      float g_s11 = gD * w11;
      float g_mu1 = 2.f * mu2 * gA + 2.f * mu1 * gC - mu2 * g_s12 - 2.f * mu1 * g_s11;
      size_t idx = ((size_t)y * W + x) * C + c;
      if (gmu) {
        gmu[idx] = g_mu1;
        gs11[idx] = g_s11;
        gs12[idx] = g_s12;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((tid & 31) == 0) s_red[tid >> 5] = acc;
  __syncthreads();
  const unsigned nblocks = gridDim.x * gridDim.y;
  const unsigned bid = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += s_red[w];
    partials[bid] = t;
    __threadfence();
    unsigned ticket = atomicAdd(&ss->ticket, 1u);
    s_last = (ticket == nblocks - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double t = 0.0;  // fixed order: thread i sums partials i, i + 256, ...
  for (unsigned b = tid; b < nblocks; b += 256) t += (double)((volatile float*)partials)[b];
  t = block_sum_d256(t, s_w);
  if (tid == 0) {
    double cnt = (double)H * W * C;
    float mean = (float)(t / cnt);
    float d = (1.f - mean) / 2.f;
    float dssim = fmaxf(0.f, d);
    float w = (d > 0.f) ? 1.f : ((d == 0.f) ? 0.5f : 0.f);
    if (loss) *loss = dssim;
    if (ssim_out) *ssim_out = mean;
    ss->factor = (float)(scale * w * -0.5 / cnt);
    ss->ticket = 0u;
  }
}

__global__ void __launch_bounds__(256)
k_ssim_bwd(const float* __restrict__ x1, const float* __restrict__ x2, int H, int W, int C,
           SsimWin win, const float* __restrict__ gmu, const float* __restrict__ gs11,
           const float* __restrict__ gs12, const SsimScalars* __restrict__ ss,
           float* __restrict__ grad) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_m[3][kSsimLH][kSsimLW];
  __shared__ float s_v[3][kSsimTH][kSsimLW];
  const int tid = threadIdx.x;
  const int x0 = blockIdx.x * kSsimTW, y0 = blockIdx.y * kSsimTH;
  const float factor = ss->factor;
  for (int c = 0; c < C; ++c) {
    for (int e = tid; e < kSsimLH * kSsimLW; e += 256) {
      int r = e / kSsimLW, q = e - r * kSsimLW;
      int y = y0 + r - kSsimR, x = x0 + q - kSsimR;
      bool in = (y >= 0) && (y < H) && (x >= 0) && (x < W);
      size_t idx = ((size_t)y * W + x) * C + c;
      s_m[0][r][q] = in ? gmu[idx] : 0.f;
      s_m[1][r][q] = in ? gs11[idx] : 0.f;
      s_m[2][r][q] = in ? gs12[idx] : 0.f;
    }
    __syncthreads();
    for (int e = tid; e < kSsimTH * kSsimLW; e += 256) {
      int r = e / kSsimLW, q = e - r * kSsimLW;
      float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
      for (int i = 0; i < kSsimK; ++i) {
        float k = win.k[i];
        a += k * s_m[0][r + i][q];
        b += k * s_m[1][r + i][q];
        d += k * s_m[2][r + i][q];
      }
      s_v[0][r][q] = a; s_v[1][r][q] = b; s_v[2][r][q] = d;
    }
    __syncthreads();
    for (int e = tid; e < kSsimTH * kSsimTW; e += 256) {
      int r = e / kSsimTW, q = e - r * kSsimTW;
      int y = y0 + r, x = x0 + q;
      if (y >= H || x >= W) continue;
      float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
      for (int j = 0; j < kSsimK; ++j) {
        float k = win.k[j];
        a += k * s_v[0][r][q + j];
        b += k * s_v[1][r][q + j];
        d += k * s_v[2][r][q + j];
      }
      size_t idx = ((size_t)y * W + x) * C + c;
      grad[idx] += factor * (a + 2.f * x1[idx] * b + x2[idx] * d);
    }
    __syncthreads();
  }
}

static SsimWin make_window() {
  // losses.py:193-198: exp(-x^2 / (2 sigma^2)) normalised, x = -5..5, sigma 1.5
  SsimWin w;
  double k[kSsimK], s = 0.0;
  for (int i = 0; i < kSsimK; ++i) {
    double x = (double)(i - kSsimR);
    k[i] = (double)(float)exp((double)(float)(-(x * x) / 4.5));
    s += k[i];
  }
  for (int i = 0; i < kSsimK; ++i) w.k[i] = (float)(k[i] / s);
  return w;
}

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Workspace of an (h, w, c) image: three coefficient maps, one partial sum
// per CTA of the grid below, then the ticket block (SsimScalars).
static size_t dssim_scalars_offset(int h, int w, int c) {
  size_t map = align256((size_t)h * w * c * sizeof(float));
  size_t nb = (size_t)((w + kSsimTW - 1) / kSsimTW) * ((h + kSsimTH - 1) / kSsimTH);
  return 3 * map + align256(nb * sizeof(float));
}

size_t dssim_workspace_bytes(int h, int w, int c) {
  return dssim_scalars_offset(h, w, c) + align256(sizeof(SsimScalars));
}

cudaError_t clear_dssim_ticket(void* ws, int h, int w, int c, cudaStream_t st) {
  return cudaMemsetAsync(static_cast<char*>(ws) + dssim_scalars_offset(h, w, c), 0, sizeof(SsimScalars), st);
}

void launch_dssim(const float* pred, const float* target, int h, int w, int c, float scale,
                  float* loss, float* ssim_out, float* grad, void* ws, cudaStream_t st) {
  size_t map = align256((size_t)h * w * c * sizeof(float));
  char* base = (char*)ws;
  float* gmu = (float*)base;
  float* gs11 = (float*)(base + map);
  float* gs12 = (float*)(base + 2 * map);
  dim3 grid((w + kSsimTW - 1) / kSsimTW, (h + kSsimTH - 1) / kSsimTH);
  size_t nb = (size_t)grid.x * grid.y;
  float* partials = (float*)(base + 3 * map);
  SsimScalars* ss = (SsimScalars*)(base + dssim_scalars_offset(h, w, c));
  SsimWin win = make_window();
  {
    GS_TIMED("ssim_fwd", st);
    launch_kernel_plain(k_ssim_fwd, grid, 256, 0, st, pred, target, h, w, c, win, scale, grad ? gmu : nullptr, gs11,
                                   gs12, partials, ss, loss, ssim_out);
  }
  GS_TIMED("ssim_bwd", st);
  if (grad) launch_kernel_plain(k_ssim_bwd, grid, 256, 0, st, pred, target, h, w, c, win, gmu, gs11, gs12, ss, grad);
}

}  // namespace gs
