// Training-step kernels around the renderer: L1 loss, the masked multi-group
// Adam step and the densification statistics (jax_gs/training/losses.py,
// trainer.py). All are flat, bandwidth-bound element loops.
#include "gs_kernels.cuh"

namespace gs {

// ---------------------------------------------------------------------------
// L1: mean |pred - target| (losses.py:4-8) with its gradient
// sign(pred - target) * scale / count (d|x|/dx = 0 at x = 0, as in JAX).
// Deterministic: fixed grid, per-CTA partials, the last CTA to finish
// (atomic ticket, no waiting) sums the partials in CTA order.
__global__ void __launch_bounds__(256)
k_l1(const float* __restrict__ pred, const float* __restrict__ target, long long count, float gscale,
     float* __restrict__ loss, float* __restrict__ grad, float* __restrict__ partials,
     Scalars* __restrict__ sc) {
  __shared__ float s_red[8];
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
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    double t = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) t += (double)((volatile float*)partials)[b];
    *loss = (float)(t / (double)count);
    sc->loss_ticket = 0u;
  }
}

void launch_l1_loss(const float* pred, const float* target, int64_t count, float scale,
                    float* loss, float* grad, float* partials, Scalars* sc, cudaStream_t st) {
  float gscale = count > 0 ? scale / (float)count : 0.f;
  GS_TIMED("l1_loss", st);
  k_l1<<<kLossGrid, 256, 0, st>>>(pred, target, count, gscale, loss, grad, partials, sc);
}

// ---------------------------------------------------------------------------
// Adam (optax.scale_by_adam + scale_by_learning_rate) per parameter group,
// then the active-mask update masking (trainer.py:44-53) and apply_updates.
struct AdamArgs {
  float lr[5];
  long long bound[5];  // end offsets of the groups in the flat buffer
  int width[5];        // elements per Gaussian in each group
  float b1, b2, omb1, omb2, bc1, bc2, eps;
};

__device__ __forceinline__ void adam_elem(long long e, float& p, float g, float& m, float& v,
                                          const uint8_t* __restrict__ active, const AdamArgs& a) {
  int seg = 0;
#pragma unroll
  for (int s = 0; s < 4; ++s) seg += (e >= a.bound[s]) ? 1 : 0;
  long long seg_start = seg == 0 ? 0 : a.bound[seg - 1];
  long long gid = (e - seg_start) / a.width[seg];
  m = a.omb1 * g + a.b1 * m;
  v = a.omb2 * (g * g) + a.b2 * v;
  float mh = m / a.bc1;
  float vh = v / a.bc2;
  float u = -a.lr[seg] * (mh / (sqrtf(vh) + a.eps));
  if (active != nullptr && active[gid] == 0) u = 0.f;
  p = p + u;
}

__global__ void __launch_bounds__(256)
k_adam_vec4(float4* __restrict__ params, const float4* __restrict__ grads, float4* __restrict__ mu,
            float4* __restrict__ nu, long long n4, const uint8_t* __restrict__ active, AdamArgs a) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n4; i += (long long)gridDim.x * 256) {
    float4 p = params[i], g = __ldg(grads + i), m = mu[i], v = nu[i];
    long long e = 4 * i;
    adam_elem(e, p.x, g.x, m.x, v.x, active, a);
    adam_elem(e + 1, p.y, g.y, m.y, v.y, active, a);
    adam_elem(e + 2, p.z, g.z, m.z, v.z, active, a);
    adam_elem(e + 3, p.w, g.w, m.w, v.w, active, a);
    params[i] = p;
    mu[i] = m;
    nu[i] = v;
  }
}

__global__ void __launch_bounds__(256)
k_adam_scalar(float* __restrict__ params, const float* __restrict__ grads, float* __restrict__ mu,
              float* __restrict__ nu, long long total, const uint8_t* __restrict__ active,
              AdamArgs a) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    float p = params[i], m = mu[i], v = nu[i];
    adam_elem(i, p, grads[i], m, v, active, a);
    params[i] = p;
    mu[i] = m;
    nu[i] = v;
  }
}

void launch_adam(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                 const uint8_t* active, const float lrs[5], float bc1, float bc2, float b1,
                 float b2, float eps, cudaStream_t st) {
  AdamArgs a;
  const int widths[5] = {3, 3, 4, 1, 3 * sh_k};
  long long acc = 0;
  for (int s = 0; s < 5; ++s) {
    a.lr[s] = lrs[s];
    a.width[s] = widths[s];
    acc += (long long)widths[s] * n;
    a.bound[s] = acc;
  }
  a.b1 = b1; a.b2 = b2; a.omb1 = 1.f - b1; a.omb2 = 1.f - b2; a.bc1 = bc1; a.bc2 = bc2; a.eps = eps;
  const long long total = acc;
  if (total == 0) return;
  const int grid = 148 * 8;
  bool aligned = ((((uintptr_t)params) | ((uintptr_t)grads) | ((uintptr_t)mu) | ((uintptr_t)nu)) & 15) == 0;
  GS_TIMED("adam", st);
  if (aligned && (total % 4) == 0) {
    k_adam_vec4<<<grid, 256, 0, st>>>((float4*)params, (const float4*)grads, (float4*)mu, (float4*)nu,
                                      total / 4, active, a);
  } else {
    k_adam_scalar<<<grid, 256, 0, st>>>(params, grads, mu, nu, total, active, a);
  }
}

// ---------------------------------------------------------------------------
// grad_2d_mag (trainer.py:143-150 / :83-94).
__global__ void __launch_bounds__(256)
k_grad2d(const float* __restrict__ gmeans, const float* __restrict__ means,
         const float* __restrict__ w2c, int n, float focal, float pix3, float* __restrict__ out) {
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
  k_grad2d<<<nb, 256, 0, st>>>(grad_means, means, w2c, n, focal, pix3, out);
}

// grad_accum / denom / max_radii updates (trainer.py:100-113, :152-159).
__global__ void __launch_bounds__(256)
k_density_stats(const float* __restrict__ grad2d, const float* __restrict__ radii,
                const uint8_t* __restrict__ valid, const uint8_t* __restrict__ active, int n,
                float* __restrict__ grad_accum, int32_t* __restrict__ denom,
                float* __restrict__ max_radii) {
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  grad_accum[i] = grad_accum[i] + grad2d[i];
  bool v = valid[i] != 0;
  bool a = active ? (active[i] != 0) : true;
  if (v && a) denom[i] = denom[i] + 1;
  if (v) max_radii[i] = nan_max(max_radii[i], radii[i]);
}

void launch_density_stats(const float* grad2d, const float* radii, const uint8_t* valid,
                          const uint8_t* active, int n, float* grad_accum, int32_t* denom,
                          float* max_radii, cudaStream_t st) {
  int nb = (n + 255) / 256;
  if (nb == 0) return;
  GS_TIMED("density_stats", st);
  k_density_stats<<<nb, 256, 0, st>>>(grad2d, radii, valid, active, n, grad_accum, denom, max_radii);
}

}  // namespace gs
