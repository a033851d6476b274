// Training-step kernels around the renderer: L1 loss, the masked multi-group
// Adam step and the densification statistics (jax_gs/training/losses.py,
// trainer.py). All are flat, bandwidth-bound element loops.
#include <algorithm>

#include "gs_kernels.cuh"

namespace gs {

// ---------------------------------------------------------------------------
// L1: mean |pred - target| (losses.py:4-8) with its gradient
// sign(pred - target) * scale / count (d|x|/dx = 0 at x = 0, as in JAX).
// Deterministic: fixed grid, per-CTA partials, the last CTA to finish
// (atomic ticket, no waiting) sums the partials in a fixed order.
__global__ void __launch_bounds__(256)
k_l1(const float* __restrict__ pred, const float* __restrict__ target, long long count, float gscale,
     float* __restrict__ loss, float* __restrict__ grad, float* __restrict__ partials,
     Scalars* __restrict__ sc) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_red[8];
  __shared__ double s_w[8];
  __shared__ bool s_last;
  float acc = 0.f;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < count; i += (long long)gridDim.x * 256) {
    float d = pred[i] - target[i];
    acc += fabsf(d);
    if (grad) grad[i] = (d > 0.f) ? gscale : ((d < 0.f) ? -gscale : 0.f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += s_red[w];
    partials[blockIdx.x] = t;
    __threadfence();
    unsigned ticket = atomicAdd(&sc->loss_ticket, 1u);
    s_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double t = 0.0;  // fixed order: thread i sums partials i, i + 256, ...
  for (unsigned b = threadIdx.x; b < gridDim.x; b += 256) t += (double)((volatile float*)partials)[b];
  t = block_sum_d256(t, s_w);
  if (threadIdx.x == 0) {
    *loss = (float)(t / (double)count);
    sc->loss_ticket = 0u;
  }
}

void launch_l1_loss(const float* pred, const float* target, int64_t count, float scale,
                    float* loss, float* grad, float* partials, Scalars* sc, cudaStream_t st) {
  float gscale = count > 0 ? scale / (float)count : 0.f;
  GS_TIMED("l1_loss", st);
  launch_kernel_plain(k_l1, kLossGrid, 256, 0, st, pred, target, count, gscale, loss, grad, partials, sc);
}

// mse_loss (losses.py:10-14): the same grid, partials and fixed-order
// last-CTA reduction as k_l1, of (pred - target)^2; gradient 2 d scale / count.
__global__ void __launch_bounds__(256)
k_mse(const float* __restrict__ pred, const float* __restrict__ target, long long count, float gscale,
      float* __restrict__ loss, float* __restrict__ grad, float* __restrict__ partials,
      Scalars* __restrict__ sc) {
  GS_PDL_ENTRY_PLAIN();
  __shared__ float s_red[8];
  __shared__ double s_w[8];
  __shared__ bool s_last;
  float acc = 0.f;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < count; i += (long long)gridDim.x * 256) {
    const float d = pred[i] - target[i];
    acc += d * d;
    if (grad) grad[i] = d * gscale;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += s_red[w];
    partials[blockIdx.x] = t;
    __threadfence();
    unsigned ticket = atomicAdd(&sc->loss_ticket, 1u);
    s_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double t = 0.0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += 256) t += (double)((volatile float*)partials)[b];
  t = block_sum_d256(t, s_w);
  if (threadIdx.x == 0) {
    *loss = (float)(t / (double)count);
    sc->loss_ticket = 0u;
  }
}

void launch_mse_loss(const float* pred, const float* target, int64_t count, float scale,
                     float* loss, float* grad, float* partials, Scalars* sc, cudaStream_t st) {
  float gscale = count > 0 ? 2.f * scale / (float)count : 0.f;
  GS_TIMED("mse_loss", st);
  launch_kernel_plain(k_mse, kLossGrid, 256, 0, st, pred, target, count, gscale, loss, grad, partials, sc);
}

// ---------------------------------------------------------------------------
// Adam (optax.scale_by_adam + scale_by_learning_rate) per parameter group,
// then the active-mask update masking (trainer.py:44-53) and apply_updates.
// blockIdx.y selects the group, so the group's learning rate, start and
// per-Gaussian width are uniform per CTA; the width is a template constant
// so the Gaussian index (for the active mask) is a cheap 32-bit division.
// The bias corrections are applied as reciprocals and the final quotient
// with the fast divide: each differs from optax's float32 divisions by at
// most a couple of ulps.
struct AdamArgs {
  float lr[5];
  int start[5];
  int count[5];
  float b1, b2, omb1, omb2, inv_bc1, inv_bc2, eps;
  int sh_width;
  // device schedule (state != nullptr): lr = lr_init * decay ^ (count / steps)
  int* state;
  float lr_init[5], decay[5], steps[5];
  // 1-D grid: CTAs [cta[g], cta[g+1]) stream group g, in proportion to its width
  int cta[6];
};

struct AdamHyper {
  float lr, inv_bc1, inv_bc2;
};

__device__ __forceinline__ float adam_update(float g, float& m, float& v, const AdamHyper& h,
                                             const AdamArgs& a) {
  m = a.omb1 * g + a.b1 * m;
  v = a.omb2 * (g * g) + a.b2 * v;
  const float mh = m * h.inv_bc1;
  const float vh = v * h.inv_bc2;
  return -h.lr * __fdividef(mh, __fsqrt_rn(vh) + a.eps);
}

template <int WIDTH>
__device__ __forceinline__ void adam_group(float* __restrict__ p, const float* __restrict__ g,
                                           float* __restrict__ m, float* __restrict__ v, int count,
                                           int width_rt, const AdamHyper& lr,
                                           const uint8_t* __restrict__ active, const AdamArgs& a,
                                           bool vec, int blk, int nblk) {
  const unsigned width = WIDTH > 0 ? (unsigned)WIDTH : (unsigned)width_rt;
  const int stride = nblk * blockDim.x;
  const int first = blk * blockDim.x + threadIdx.x;
  if (vec) {
    float4* p4 = reinterpret_cast<float4*>(p);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    // two chunks per iteration, every load of both issued before either is
    // used (twice the bytes in flight per thread)
    const int n4 = count / 4;
    for (int i0 = first; i0 < n4; i0 += 2 * stride) {
      bool act[2][4], any[2], in[2];
      float4 P[2], G[2], M0[2], V0[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = i0 + h * stride;
        in[h] = i < n4;
        const unsigned e = 4u * (unsigned)i;
#pragma unroll
        for (int q = 0; q < 4; ++q) act[h][q] = in[h] && (!active || active[(e + q) / width] != 0);
        // masked elements keep their value: no read or write of the parameter
        any[h] = act[h][0] | act[h][1] | act[h][2] | act[h][3];
        P[h] = any[h] ? p4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        if (in[h]) {
          G[h] = __ldg(g4 + i);
          M0[h] = m4[i];
          V0[h] = v4[i];
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!in[h]) continue;
        const int i = i0 + h * stride;
        float4 M = M0[h], V = V0[h];
        const float u0 = adam_update(G[h].x, M.x, V.x, lr, a), u1 = adam_update(G[h].y, M.y, V.y, lr, a);
        const float u2 = adam_update(G[h].z, M.z, V.z, lr, a), u3 = adam_update(G[h].w, M.w, V.w, lr, a);
        if (any[h]) {
          float4 Q = P[h];
          Q.x += act[h][0] ? u0 : 0.f;
          Q.y += act[h][1] ? u1 : 0.f;
          Q.z += act[h][2] ? u2 : 0.f;
          Q.w += act[h][3] ? u3 : 0.f;
          p4[i] = Q;
        }
        // moments that did not change (zero gradient and zero moments: slots
        // that were never active) are not stored again
        if (!same_bits(M, M0[h])) m4[i] = M;
        if (!same_bits(V, V0[h])) v4[i] = V;
      }
    }
  } else {
    for (int e = first; e < count; e += stride) {
      float M = m[e], V = v[e];
      const float u = adam_update(g[e], M, V, lr, a);
      if (!active || active[(unsigned)e / width]) p[e] += u;
      m[e] = M;
      v[e] = V;
    }
  }
}

__global__ void __launch_bounds__(256)
k_adam(float* __restrict__ params, const float* __restrict__ grads, float* __restrict__ mu,
       float* __restrict__ nu, const uint8_t* __restrict__ active, AdamArgs a, bool vec) {
  GS_PDL_ENTRY_PLAIN();
  int grp = 0;
#pragma unroll
  for (int q = 1; q < 5; ++q)
    if ((int)blockIdx.x >= a.cta[q]) grp = q;
  const int blk = (int)blockIdx.x - a.cta[grp], nblk = a.cta[grp + 1] - a.cta[grp];
  AdamHyper h;
  if (a.state) {
    // optax count before this update; every CTA evaluates the same schedule
    const float cf = (float)(*(volatile int*)a.state);
    h.lr = a.lr_init[grp] * powf(a.decay[grp], cf / a.steps[grp]);
    h.inv_bc1 = 1.f / (1.f - powf(a.b1, cf + 1.f));
    h.inv_bc2 = 1.f / (1.f - powf(a.b2, cf + 1.f));
  } else {
    h.lr = a.lr[grp];
    h.inv_bc1 = a.inv_bc1;
    h.inv_bc2 = a.inv_bc2;
  }
  const int o = a.start[grp];
  float* p = params + o;
  const float* g = grads + o;
  float* m = mu + o;
  float* v = nu + o;
  const AdamHyper& lr = h;
  const int c = a.count[grp];
  switch (grp) {
    case 0:
    case 1: adam_group<3>(p, g, m, v, c, 3, lr, active, a, vec, blk, nblk); break;
    case 2: adam_group<4>(p, g, m, v, c, 4, lr, active, a, vec, blk, nblk); break;
    case 3: adam_group<1>(p, g, m, v, c, 1, lr, active, a, vec, blk, nblk); break;
    default:
      if (a.sh_width == 48) adam_group<48>(p, g, m, v, c, 48, lr, active, a, vec, blk, nblk);
      else adam_group<0>(p, g, m, v, c, a.sh_width, lr, active, a, vec, blk, nblk);
  }
  if (a.state) {
    // the last CTA to finish (atomic ticket, no waiting) advances the count
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned total = gridDim.x;
      const unsigned t = atomicAdd(reinterpret_cast<unsigned*>(a.state + 1), 1u);
      if (t == total - 1) {
        a.state[0] = a.state[0] + 1;
        a.state[1] = 0;
      }
    }
  }
}

#ifndef GS_ADAM_CTAS_PER_SM
#define GS_ADAM_CTAS_PER_SM 8
#endif
constexpr int kAdamCtasPerSm = GS_ADAM_CTAS_PER_SM;

void launch_adam(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                 const uint8_t* active, const float lrs[5], float bc1, float bc2, float b1,
                 float b2, float omb1, float omb2, float eps, int* state, const float* sched_lr,
                 const float* sched_decay, const float* sched_steps, cudaStream_t st) {
  AdamArgs a;
  const int widths[5] = {3, 3, 4, 1, 3 * sh_k};
  long long acc = 0;
  for (int s = 0; s < 5; ++s) {
    a.lr[s] = lrs[s];
    a.start[s] = (int)acc;
    a.count[s] = widths[s] * n;
    acc += a.count[s];
  }
  a.sh_width = 3 * sh_k;
  a.b1 = b1; a.b2 = b2; a.omb1 = omb1; a.omb2 = omb2; a.eps = eps;
  a.inv_bc1 = 1.f / bc1;
  a.inv_bc2 = 1.f / bc2;
  a.state = state;
  for (int g = 0; g < 5; ++g) {
    a.lr_init[g] = sched_lr ? sched_lr[g] : 0.f;
    a.decay[g] = sched_decay ? sched_decay[g] : 1.f;
    a.steps[g] = sched_steps ? sched_steps[g] : 1.f;
  }
  if (acc == 0) return;
  // every group starts on a 16-byte boundary when n is a multiple of 4
  const bool vec = (n % 4 == 0) &&
                   ((((uintptr_t)params) | ((uintptr_t)grads) | ((uintptr_t)mu) | ((uintptr_t)nu)) & 15) == 0;
  // GS_ADAM_CTAS_PER_SM CTAs of 256 per SM, shared among the groups by width
  const int total = device_sms() * kAdamCtasPerSm;
  const long long all = acc > 0 ? acc : 1;
  a.cta[0] = 0;
  for (int g = 0; g < 5; ++g)
    a.cta[g + 1] = a.cta[g] + (int)std::max<long long>(1, (long long)total * a.count[g] / all);
  GS_TIMED("adam", st);
  launch_kernel_plain(k_adam, a.cta[5], 256, 0, st, params, grads, mu, nu, active, a, vec);
}

// ---------------------------------------------------------------------------
// grad_2d_mag (trainer.py:143-150 / :83-94).
__global__ void __launch_bounds__(256)
k_grad2d(const float* __restrict__ gmeans, const float* __restrict__ means,
         const float* __restrict__ w2c, int n, float focal, float pix3, float* __restrict__ out) {
  GS_PDL_ENTRY_PLAIN();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  float W20 = __ldg(w2c + 8), W21 = __ldg(w2c + 9), W22 = __ldg(w2c + 10), W23 = __ldg(w2c + 11);
  float z = add_rn(add_rn(add_rn(mul_rn(W20, means[3 * i]), mul_rn(W21, means[3 * i + 1])),
                          mul_rn(W22, means[3 * i + 2])),
                   W23);
  z = nan_max(z, 0.01f);
  float g0 = gmeans[3 * i], g1 = gmeans[3 * i + 1], g2 = gmeans[3 * i + 2];
  float nrm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
  out[i] = (nrm * (z / focal)) * pix3;
}

void launch_grad2d(const float* grad_means, const float* means, const float* w2c, int n, float fx,
                   float fy, int width, int height, float* out, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  float focal = (float)(((double)fx + (double)fy) / 2.0);
  float pix3 = (float)((double)width * (double)height * 3.0);
  GS_TIMED("grad2d", st);
  launch_kernel_plain(k_grad2d, nb, 256, 0, st, grad_means, means, w2c, n, focal, pix3, out);
}

// grad_accum / denom / max_radii updates (trainer.py:100-113, :152-159).
__global__ void __launch_bounds__(256)
k_density_stats(const float* __restrict__ grad2d, const float* __restrict__ radii,
                const uint8_t* __restrict__ valid, const uint8_t* __restrict__ radii_valid,
                const uint8_t* __restrict__ active, int n, float* __restrict__ grad_accum,
                int32_t* __restrict__ denom, float* __restrict__ max_radii) {
  GS_PDL_ENTRY_PLAIN();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  grad_accum[i] = grad_accum[i] + grad2d[i];
  const bool a = active ? (active[i] != 0) : true;
  if (valid[i] != 0 && a) denom[i] = denom[i] + 1;
  if (radii_valid[i] != 0) max_radii[i] = nan_max(max_radii[i], radii[i]);
}

// Single device, trainer.py:143-159 in one pass: grad_2d_mag of the
// (pre-update) means, then the accumulators, with the arithmetic of
// k_grad2d and k_density_stats (radii_valid = valid).
__global__ void __launch_bounds__(256)
k_step_stats(const float* __restrict__ gmeans, const float* __restrict__ means, const float* __restrict__ w2c,
             int n, float focal, float pix3, const float* __restrict__ radii, const uint8_t* __restrict__ valid,
             const uint8_t* __restrict__ active, float* __restrict__ grad_accum, int32_t* __restrict__ denom,
             float* __restrict__ max_radii, float* __restrict__ grad2d_out) {
  GS_PDL_ENTRY_PLAIN();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  const float W20 = __ldg(w2c + 8), W21 = __ldg(w2c + 9), W22 = __ldg(w2c + 10), W23 = __ldg(w2c + 11);
  float z = add_rn(add_rn(add_rn(mul_rn(W20, means[3 * i]), mul_rn(W21, means[3 * i + 1])),
                          mul_rn(W22, means[3 * i + 2])),
                   W23);
  z = nan_max(z, 0.01f);
  const float g0 = gmeans[3 * i], g1 = gmeans[3 * i + 1], g2 = gmeans[3 * i + 2];
  const float nrm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
  const float g2d = (nrm * (z / focal)) * pix3;
  if (grad2d_out) grad2d_out[i] = g2d;
  grad_accum[i] = grad_accum[i] + g2d;
  const bool v = valid[i] != 0;
  const bool a = active ? (active[i] != 0) : true;
  if (v && a) denom[i] = denom[i] + 1;
  if (v) max_radii[i] = nan_max(max_radii[i], radii[i]);
}

void launch_step_stats(const float* grad_means, const float* means, const float* w2c, int n, float fx, float fy,
                       int width, int height, const float* radii, const uint8_t* valid, const uint8_t* active,
                       float* grad_accum, int32_t* denom, float* max_radii, float* grad2d, cudaStream_t st) {
  const int nb = (n + 255) / 256;
  if (nb == 0) return;
  const float focal = (float)(((double)fx + (double)fy) / 2.0);
  const float pix3 = (float)((double)width * (double)height * 3.0);
  GS_TIMED("step_stats", st);
  launch_kernel_plain(k_step_stats, nb, 256, 0, st, grad_means, means, w2c, n, focal, pix3, radii, valid, active, grad_accum, denom,
                                    max_radii, grad2d);
}

void launch_density_stats(const float* grad2d, const float* radii, const uint8_t* valid,
                          const uint8_t* radii_valid, const uint8_t* active, int n,
                          float* grad_accum, int32_t* denom, float* max_radii, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("density_stats", st);
  launch_kernel_plain(k_density_stats, nb, 256, 0, st, grad2d, radii, valid, radii_valid, active, n, grad_accum, denom,
                                       max_radii);
}

}  // namespace gs

namespace gs {

// gs_train_step_metrics: one thread per output value.
__global__ void k_step_metrics(const float* __restrict__ tail, const GsExtras* __restrict__ ex, float lambda,
                               const int* __restrict__ wait_status, float* __restrict__ out) {
  GS_PDL_ENTRY_PLAIN();
  const int t = threadIdx.x;
  if (t == 0) out[0] = (1.f - lambda) * tail[0] + lambda * tail[1];
  if (t == 1) out[1] = tail[0];
  if (t == 2) out[2] = 1.f - tail[1] * 2.f;
  if (t >= 3 && t < 11) {
    const int c = t - 3;
    float v;
    if (ex) {
      const int32_t* e = reinterpret_cast<const int32_t*>(ex);
      v = (c == 1) ? ex->mean_interactions_per_tile : (float)e[c];
    } else {
      v = tail[3 + c];
    }
    out[t] = v;
  }
  // bounded device waits that gave up: the sort's (this render, or the
  // tail's copy averaged over ranks) and the rendezvous word's
  if (t == 11) out[t] = (ex ? (float)ex->device_timeouts : tail[11]) + (wait_status ? (float)*wait_status : 0.f);
}

void launch_step_metrics(const float* tail, const GsExtras* ex, float lambda, const int* wait_status, float* out,
                         cudaStream_t st) {
  launch_kernel_plain(k_step_metrics, 1, 32, 0, st, tail, ex, lambda, wait_status, out);
}

}  // namespace gs
