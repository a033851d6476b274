// Data-parallel gradient average + Adam + densification statistics over
// NVLink peer memory (gs_dp_update, include/gsb200.h).
//
// One kernel per rank (k_dp_adam), on the rank's own GPU, in two CTA ranges:
//   means + statistics  one thread per Gaussian of the rank's slice: averaged
//               means gradient -> grad_2d of every rank's camera, averaged
//               (trainer.py:83-97); max over ranks of masked radii and of the
//               valid mask (:108-111); grad_accum / denom / max_radii written
//               into every rank's buffers (denom with that rank's own mask);
//               then masked Adam on the Gaussian's three means elements (the
//               statistics read the pre-update means the same thread updates).
//   groups 1..4  one thread per 4 elements of the slice in each of the other
//               parameter groups: gradient averaged over the ranks' buffers,
//               masked Adam with this rank's mu / nu, new value stored to every
//               rank.
// Peer traffic per rank: reads (R-1)/R and writes (R-1)/R of the 59-float
// per-Gaussian parameter record -- the volume of a ring all-reduce -- with
// Adam and the statistics computed on 1/R of the data while it streams. The
// peer loads of a thread (one per rank) are issued together, so a thread
// waits for one NVLink round trip, not one per rank.
// The kernel first reads the caller's rendezvous status word: nonzero means
// a gs_dp_barrier wait gave up (a peer may be late, gone or its memory
// unmapped), and then it touches no peer memory and changes nothing.
// Inactive Gaussians (active_mask 0) have zero gradients on every rank and
// masked updates, so their parameters and statistics are the same on every
// replica before and after the step: their peer reads and writes are
// skipped (only their Adam moments, which are rank-local, still decay).
// With touched inboxes (gs_dp_publish_barrier), a rank's gradient row of a
// Gaussian its view did not touch (exact zeros) is not read either; the
// flags are local by then, so the skip costs no extra NVLink round trip.
// The loss / metric tail is averaged in CTA 0, the render counters read from
// every rank's GsExtras when the peer set carries them.
//
// Measured (config 2, 200 k slots, 100 k active): the update is bound by
// NVLink and by round trips, not by HBM. At 2 GPUs, plain peer reads reach
// about 600 GB/s and writes 645 GB/s, but reads and writes together about
// 330 GB/s each way (the incoming link carries this rank's read data and the
// peer's writes). The update plus one rendezvous takes 60 us at 2 GPUs
// and 90-105 us at 8, where the time varies from machine to machine.
#include <algorithm>
#include <cstring>

#include "gs_kernels.cuh"

namespace gs {

struct DpArgs {
  GsPeerSet p;
  int n, sh_k;
  int mine;  // stripes of GS_DP_STRIPE Gaussians this rank owns: s = k R + rank, k < mine
  float focal, pix3;
  float inv_world;
  // k_dp_adam's 1-D grid: CTAs [cta[g], cta[g+1]) stream parameter group g,
  // in proportion to its width (the SH group is 48 of the 59 floats)
  int cta[6];
};

// Rank r owns the stripes of kStripe consecutive Gaussians whose index is r
// modulo R: an interleaving, so every rank gets its share of the active
// Gaussians whatever their layout (a capacity's first half active, or holes
// left by pruning), and every stripe starts 16-byte aligned in every group.
constexpr int kStripe = GS_DP_STRIPE;

static int dp_stripes_owned(int n, int world, int rank) {
  const int total = (n + kStripe - 1) / kStripe;
  return rank < total ? (total - rank + world - 1) / world : 0;
}

// Global index of the Gaussian at position j of this rank's stripes.
__device__ __forceinline__ int dp_gaussian(const DpArgs& a, int j) {
  return ((j / kStripe) * a.p.world + a.p.rank) * kStripe + (j % kStripe);
}

struct DpAdam {
  float lr_init[5], decay[5], steps[5];
  float b1, b2, omb1, omb2, eps;
  int* state;
};

// The means group together with the statistics, one thread per Gaussian of
// this rank's slice (so the statistics read the pre-update means that the
// same thread then updates, and no other CTA writes them):
//  - the averaged means gradient -> grad_2d under every rank's camera,
//    averaged (trainer.py:83-97); the max over ranks of the masked radii and
//    of the valid mask (:108-111); grad_accum / max_radii written into every
//    rank's buffers, denom with each rank's own mask;
//  - masked Adam on the three means elements, the new values stored to
//    every rank; the moments stay with this rank.
// The first CTA also averages the loss / metric tail (trainer.py:70-71).
template <int RMAX>
__device__ __forceinline__ void dp_means_and_stats(const DpArgs& a, const DpAdam& h, float* __restrict__ mu,
                                                   float* __restrict__ nu, const uint8_t* __restrict__ active,
                                                   float lr, float inv_bc1, float inv_bc2, int blk, int nblk,
                                                   int tail_len, float* __restrict__ tail_out) {
  const int R = a.p.world;
  const uint8_t* __restrict__ inbox = a.p.touched_in[a.p.rank];  // R rows of n touched flags, or NULL
  __shared__ float s_w[RMAX][4];  // row 2 of every rank's W2C (the camera depth)
  if (threadIdx.x < 4 * R) s_w[threadIdx.x >> 2][threadIdx.x & 3] = a.p.w2c[threadIdx.x >> 2][8 + (threadIdx.x & 3)];
  if (blk == 0 && threadIdx.x < tail_len) {
    const int k = threadIdx.x;
    const size_t off = (size_t)a.n * (11 + 3 * a.sh_k) + k;
    float t = 0.f;
    for (int r = 0; r < R; ++r) {
      const int32_t* ex = a.p.extras[r];
      if (ex && k >= 3 && k <= 11) {
        // the render's health counters straight from that rank's GsExtras:
        // tail[3..10] = words 0..7 (word 1 is a float), tail[11] = device_timeouts
        t += k == 4 ? __int_as_float(ex[1]) : (float)ex[k <= 10 ? k - 3 : 10];
      } else {
        t += a.p.grads[r][off];
      }
    }
    tail_out[k] = t * a.inv_world;
  }
  __syncthreads();
  for (int j = blk * blockDim.x + threadIdx.x; j < a.mine * kStripe; j += nblk * blockDim.x) {
    const int i = dp_gaussian(a, j);
    if (i >= a.n) continue;  // the last stripe may be partial
    const bool act = active ? (active[i] != 0) : true;
    const size_t e = 3 * (size_t)i;
    float g0 = 0.f, g1 = 0.f, g2 = 0.f;
    if (act) {
      // every peer's loads are issued before any is used (the statistics in
      // one NVLink round trip, the gradient rows that may be nonzero by the
      // local touched flags); the sums keep the rank order 0 .. R-1
      float gx[RMAX][3], rr_[RMAX];
      uint8_t vv_[RMAX];
      int dn[RMAX];
      bool tc[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          vv_[r] = a.p.valid[r][i];
          rr_[r] = a.p.radii[r][i];
          dn[r] = a.p.denom[r][i];
          tc[r] = !inbox || inbox[(size_t)r * a.n + i] != 0;
        }
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R && tc[r]) {
          const float* g = a.p.grads[r] + e;
          gx[r][0] = g[0]; gx[r][1] = g[1]; gx[r][2] = g[2];
        }
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R && tc[r]) {
          g0 += gx[r][0];
          g1 += gx[r][1];
          g2 += gx[r][2];
        }
      }
      g0 *= a.inv_world; g1 *= a.inv_world; g2 *= a.inv_world;
      const float nrm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
      const float* m = a.p.params[a.p.rank] + e;  // pre-update means (own replica)
      const float m0 = m[0], m1 = m[1], m2 = m[2];
      float g2d = 0.f, rmax = 0.f;
      bool any_valid = false;
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          float z = add_rn(add_rn(add_rn(mul_rn(s_w[r][0], m0), mul_rn(s_w[r][1], m1)), mul_rn(s_w[r][2], m2)),
                           s_w[r][3]);
          z = nan_max(z, 0.01f);
          g2d += (nrm * (z / a.focal)) * a.pix3;
          const bool v = vv_[r] != 0;
          any_valid |= v;
          rmax = nan_max(rmax, v ? rr_[r] : 0.f);
        }
      }
      g2d *= a.inv_world;
      const float acc = a.p.grad_accum[a.p.rank][i] + g2d;
      const float mr0 = a.p.max_radii[a.p.rank][i];
      const float mr = any_valid ? nan_max(mr0, rmax) : mr0;
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          a.p.grad_accum[r][i] = acc;
          a.p.max_radii[r][i] = mr;
          if (vv_[r] != 0) a.p.denom[r][i] = dn[r] + 1;
        }
      }
    }
    // masked Adam on the three means elements (an inactive Gaussian has a
    // zero gradient everywhere: only its own moments decay)
    const float gv[3] = {g0, g1, g2};
    float pv[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float m_old = mu[e + c], v_old = nu[e + c];
      const float mv = h.omb1 * gv[c] + h.b1 * m_old;
      const float vv = h.omb2 * (gv[c] * gv[c]) + h.b2 * v_old;
      const float u = -lr * __fdividef(mv * inv_bc1, __fsqrt_rn(vv * inv_bc2) + h.eps);
      if (__float_as_uint(mv) != __float_as_uint(m_old)) mu[e + c] = mv;
      if (__float_as_uint(vv) != __float_as_uint(v_old)) nu[e + c] = vv;
      pv[c] = act ? a.p.params[a.p.rank][e + c] + u : 0.f;
    }
    if (act) {
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
          float* P = a.p.params[r] + e;
          P[0] = pv[0]; P[1] = pv[1]; P[2] = pv[2];
        }
      }
    }
  }
}


// Chunks of 4 elements a thread of groups 1..4 keeps in flight: every load
// of all of them (the R gradient rows, both moments, the parameter) is
// issued before any is used. The update is bound by NVLink bandwidth, not
// by round trips (at 2 GPUs the incoming link carries this rank's gradient
// reads and the peer's parameter writes, about 650 GB/s of payload
// together), so 1 is the default: 2 chunks take 80 registers at RMAX 2
// instead of 56 and measured 65 vs 60 us for update + rendezvous.
#ifndef GS_DP_UNROLL
#define GS_DP_UNROLL 1
#endif
constexpr int kDpUnroll = GS_DP_UNROLL;
// CTAs of the means + statistics phase, in units of one float of Adam
// streaming per Gaussian (the other groups weigh their width: 3, 4, 1, 3K)
#ifndef GS_DP_MEANS_WORK
#define GS_DP_MEANS_WORK 12
#endif
constexpr int kDpMeansWork = GS_DP_MEANS_WORK;

// Whether a rank's gradient row may be nonzero at the float4 chunk starting
// at element el of a group of the given width: that rank's touched flag (its
// row t of this rank's inbox, local memory) of every Gaussian the chunk
// covers. gs_render_backward writes 0 only where the whole gradient row is
// exact +0, and skipping a +0 leaves every sum the update uses as it was.
// NULL: no flags, read the row.
template <int WIDTH>
__device__ __forceinline__ bool row_touched(const uint8_t* __restrict__ t, unsigned el, unsigned width) {
  if (!t) return true;
  if (WIDTH == 1) return *reinterpret_cast<const uint32_t*>(t + el) != 0u;  // el % 4 == 0: 4 Gaussians
  if (WIDTH > 0 && WIDTH % 4 == 0) return t[el / WIDTH] != 0;                // one Gaussian
  const unsigned g0 = el / width, g1 = (el + 3) / width;
  bool any = false;
  for (unsigned g = g0; g <= g1; ++g) any |= t[g] != 0;
  return any;
}

template <int RMAX, int WIDTH>
__device__ __forceinline__ void dp_adam_group(const DpArgs& a, const DpAdam& h, size_t seg, int width_rt,
                                              float* __restrict__ mu, float* __restrict__ nu,
                                              const uint8_t* __restrict__ active, float lr, float inv_bc1,
                                              float inv_bc2, int blk, int nblk) {
  const unsigned width = WIDTH > 0 ? (unsigned)WIDTH : (unsigned)width_rt;
  const unsigned per_stripe = (unsigned)kStripe * width;  // elements of one stripe in this group
  const unsigned group_end = (unsigned)a.n * width;
  const int R = a.p.world;
  const uint8_t* __restrict__ inbox = a.p.touched_in[a.p.rank];  // R rows of n touched flags, or NULL
  const int stride = nblk * blockDim.x;
  const int first = blk * blockDim.x + threadIdx.x;
  // float4 chunks never straddle the group's end when n % 4 == 0
  const bool vec = (a.n & 3) == 0;
  if (vec) {
    const int chunks = (int)(per_stripe / 4);
    const int total = a.mine * chunks;
    for (int j0 = first; j0 < total; j0 += kDpUnroll * stride) {
      bool in[kDpUnroll], any[kDpUnroll], act[kDpUnroll][4];
      unsigned el[kDpUnroll], need[kDpUnroll];
      float4 xr[kDpUnroll][RMAX], M[kDpUnroll], V[kDpUnroll], P[kDpUnroll];
#pragma unroll
      for (int u = 0; u < kDpUnroll; ++u) {
        const int j = j0 + u * stride;
        const int k = j / chunks, c = j - k * chunks;
        el[u] = (unsigned)((k * R + a.p.rank) * kStripe) * width + 4u * (unsigned)c;
        // past the end of this rank's stripes, or of the last (partial) stripe
        in[u] = j < total && el[u] < group_end;
        // an inactive Gaussian has a zero gradient on every rank and keeps
        // its parameters: its peer rows are neither read nor written
        if (WIDTH > 0 && WIDTH % 4 == 0) {
          const bool g_act = in[u] && (!active || active[el[u] / width] != 0);
#pragma unroll
          for (int q = 0; q < 4; ++q) act[u][q] = g_act;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) act[u][q] = in[u] && (!active || active[(el[u] + q) / width] != 0);
        }
        any[u] = act[u][0] | act[u][1] | act[u][2] | act[u][3];
        need[u] = 0u;
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
          if (any[u] && r < R && row_touched<WIDTH>(inbox ? inbox + (size_t)r * a.n : nullptr, el[u], width))
            need[u] |= 1u << r;
        const size_t e = seg + el[u];
        if (in[u]) {
          M[u] = *reinterpret_cast<const float4*>(mu + e);
          V[u] = *reinterpret_cast<const float4*>(nu + e);
        }
        if (any[u]) P[u] = *reinterpret_cast<const float4*>(a.p.params[a.p.rank] + e);
      }
      // the gradient rows that may be nonzero, after the touched flags
#pragma unroll
      for (int u = 0; u < kDpUnroll; ++u) {
        const size_t e = seg + el[u];
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
          if ((need[u] >> r) & 1u) xr[u][r] = *reinterpret_cast<const float4*>(a.p.grads[r] + e);
      }
#pragma unroll
      for (int u = 0; u < kDpUnroll; ++u) {
        if (!in[u]) continue;
        const size_t e = seg + el[u];
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          if ((need[u] >> r) & 1u) {
            g.x += xr[u][r].x; g.y += xr[u][r].y; g.z += xr[u][r].z; g.w += xr[u][r].w;
          }
        }
        g.x *= a.inv_world; g.y *= a.inv_world; g.z *= a.inv_world; g.w *= a.inv_world;
        float gv[4] = {g.x, g.y, g.z, g.w}, mv[4] = {M[u].x, M[u].y, M[u].z, M[u].w};
        float vv[4] = {V[u].x, V[u].y, V[u].z, V[u].w};
        float pv[4] = {0.f, 0.f, 0.f, 0.f};
        if (any[u]) { pv[0] = P[u].x; pv[1] = P[u].y; pv[2] = P[u].z; pv[3] = P[u].w; }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          mv[q] = h.omb1 * gv[q] + h.b1 * mv[q];
          vv[q] = h.omb2 * (gv[q] * gv[q]) + h.b2 * vv[q];
          const float d = -lr * __fdividef(mv[q] * inv_bc1, __fsqrt_rn(vv[q] * inv_bc2) + h.eps);
          pv[q] += act[u][q] ? d : 0.f;
        }
        // moments that did not change (no gradient, zero moments) are not stored again
        const float4 M1 = make_float4(mv[0], mv[1], mv[2], mv[3]), V1 = make_float4(vv[0], vv[1], vv[2], vv[3]);
        if (!same_bits(M1, M[u])) *reinterpret_cast<float4*>(mu + e) = M1;
        if (!same_bits(V1, V[u])) *reinterpret_cast<float4*>(nu + e) = V1;
        const float4 out = make_float4(pv[0], pv[1], pv[2], pv[3]);
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
          if (any[u] && r < R) *reinterpret_cast<float4*>(a.p.params[r] + e) = out;
      }
    }
  } else {
    for (int j = first; j < a.mine * (int)per_stripe; j += stride) {
      const int k = j / (int)per_stripe, c = j - k * (int)per_stripe;
      const unsigned el = (unsigned)((k * R + a.p.rank) * kStripe) * width + (unsigned)c;
      if (el >= group_end) continue;
      const size_t e = seg + el;
      const unsigned gid = el / width;
      const bool act = !active || active[gid] != 0;
      bool tc[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) tc[r] = act && r < R && (!inbox || inbox[(size_t)r * a.n + gid] != 0);
      float xr[RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (tc[r]) xr[r] = a.p.grads[r][e];
      float g = 0.f;
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (tc[r]) g += xr[r];
      g *= a.inv_world;
      float mv = h.omb1 * g + h.b1 * mu[e];
      float vv = h.omb2 * (g * g) + h.b2 * nu[e];
      float u = -lr * __fdividef(mv * inv_bc1, __fsqrt_rn(vv * inv_bc2) + h.eps);
      if (!act) u = 0.f;
      mu[e] = mv;
      nu[e] = vv;
      const float out = a.p.params[a.p.rank][e] + u;
#pragma unroll
      for (int r = 0; r < RMAX; ++r)
        if (act && r < R) a.p.params[r][e] = out;
    }
  }
}

// Rendezvous over peer memory (gs_dp_barrier): thread r < R raises this
// rank's word in rank r's flags array to the new epoch, then waits for rank
// r's word in this rank's array. Bounded: after kBarrierSpins polls the
// thread counts a timeout and stops waiting.
constexpr int kBarrierSpins = 1 << 22;  // about a second of polling

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The rendezvous itself, run by one whole CTA (threads r < R do the work).
__device__ __forceinline__ void rendezvous(const GsPeerSet& p, int* __restrict__ epoch, int* __restrict__ status) {
  __shared__ int s_epoch;
  const int t = threadIdx.x;
  if (t == 0) {
    s_epoch = *epoch + 1;
    *epoch = s_epoch;
  }
  __syncthreads();
  const int e = s_epoch;
  if (t < p.world) {
    // this GPU's earlier writes (the previous kernels', ordered before this
    // thread by the kernel boundary, and the publishing CTAs', ordered by
    // their fences and tickets; the fence is cumulative) before the flag.
    // (Relaxed polls with one acquire fence after them measured slower:
    // 10.7 vs 7.0 us per back-to-back rendezvous at 2 GPUs.)
    __threadfence_system();
    st_release_sys(p.flags[t] + p.rank, e);
    const int* mine = p.flags[p.rank] + t;
    int spins = 0;
    while (ld_acquire_sys(mine) < e) {
      if (++spins > kBarrierSpins) {
        atomicAdd(status, 1);
        break;
      }
    }
  }
  __syncthreads();
}

__global__ void k_dp_barrier(GsPeerSet p, int* __restrict__ epoch, int* __restrict__ status) {
  GS_PDL_ENTRY_PLAIN();
  rendezvous(p, epoch, status);
}

// gs_dp_publish_barrier: this rank's touched flags into row `rank` of every
// owner's inbox (p.touched_in[owner], GS_MAX_RANKS rows of n bytes), 16
// Gaussians per thread and store (16 consecutive Gaussians lie in one stripe,
// so they have one owner), then the rendezvous, run by the last CTA to finish
// (each CTA fences its peer writes at system scope before taking its ticket
// in epoch[1]). The inbox rows are rewritten in full every step.
constexpr int kPublishThreads = 256;

__global__ void __launch_bounds__(kPublishThreads)
k_dp_publish_barrier(GsPeerSet p, const uint8_t* __restrict__ touched, int n, int* __restrict__ epoch,
                     int* __restrict__ status) {
  GS_PDL_ENTRY_PLAIN();
  const int R = p.world;
  // after a rendezvous gave up (status word set) no peer's inbox is written
  const int groups = *(volatile const int*)status == 0 ? (n + 15) / 16 : 0;
  const bool vec = (n & 15) == 0;  // every row, and so every 16-byte group, 16-byte aligned
  for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += gridDim.x * blockDim.x) {
    const int i0 = gi * 16;
    const int owner = (i0 / kStripe) % R;
    uint8_t* dst = p.touched_in[owner] + (size_t)p.rank * (size_t)n + i0;
    if (vec) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(touched + i0);
    } else {
      for (int q = 0; q < 16 && i0 + q < n; ++q) dst[q] = touched[i0 + q];
    }
  }
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned t = atomicAdd(reinterpret_cast<unsigned*>(epoch + 1), 1u);
    s_last = t == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) epoch[1] = 0;  // every ticket is in: ready for the next call
  rendezvous(p, epoch, status);
}

// The data-parallel update as one launch: CTAs [cta[0], cta[1]) run the means
// and the statistics (dp_means_and_stats), the others stream parameter groups
// 1..4 (scales, quaternions, opacities, SH) by float4 chunks. RMAX bounds the
// world size (2, 4 or 8): the per-rank load registers are sized by it.
// Minimum resident CTAs per SM asked of the 8-rank kernel: 3 caps it at 80
// registers with a small spill (1 would leave 98 registers, 2 CTAs per SM).
// Measured back to back on one 8-GPU machine: 100.0 / 100.4 vs 105.4 / 104.9
// us per exchange (publish rendezvous + update + rendezvous) with the
// touched-row skip, 102.5 / 103.4 vs 103.7 / 104.3 without it.
#ifndef GS_DP_MIN_CTAS_8
#define GS_DP_MIN_CTAS_8 3
#endif
// The same for the 4-rank kernel: 80 registers and no spill at 3 CTAs per SM
// (86 and 2 CTAs per SM unbounded); not timed at 4 GPUs on its own.
#ifndef GS_DP_MIN_CTAS_4
#define GS_DP_MIN_CTAS_4 3
#endif
template <int RMAX>
__global__ void __launch_bounds__(256, (RMAX >= 8 ? GS_DP_MIN_CTAS_8 : RMAX >= 4 ? GS_DP_MIN_CTAS_4 : 1))
k_dp_adam(DpArgs a, DpAdam h, float* __restrict__ mu, float* __restrict__ nu,
          const uint8_t* __restrict__ active, const int* __restrict__ barrier_status, int tail_len,
          float* __restrict__ tail_out) {
  GS_PDL_ENTRY_PLAIN();
  if (barrier_status && *(volatile const int*)barrier_status != 0) return;  // every CTA: no ticket, no count
  int grp = 0;
#pragma unroll
  for (int g = 1; g < 5; ++g)
    if ((int)blockIdx.x >= a.cta[g]) grp = g;
  const int blk = (int)blockIdx.x - a.cta[grp], nblk = a.cta[grp + 1] - a.cta[grp];
  const float cf = (float)(*(volatile int*)h.state);
  float li = 0.f, de = 1.f, stp = 1.f;
#pragma unroll
  for (int g = 0; g < 5; ++g)
    if (g == grp) {
      li = h.lr_init[g];
      de = h.decay[g];
      stp = h.steps[g];
    }
  const float lr = li * powf(de, cf / stp);
  const float inv_bc1 = 1.f / (1.f - powf(h.b1, cf + 1.f));
  const float inv_bc2 = 1.f / (1.f - powf(h.b2, cf + 1.f));
  const size_t n = (size_t)a.n;
  switch (grp) {
    case 0:
      dp_means_and_stats<RMAX>(a, h, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk, tail_len, tail_out);
      break;
    case 1: dp_adam_group<RMAX, 3>(a, h, 3 * n, 3, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk); break;
    case 2: dp_adam_group<RMAX, 4>(a, h, 6 * n, 4, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk); break;
    case 3: dp_adam_group<RMAX, 1>(a, h, 10 * n, 1, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk); break;
    default:
      if (a.sh_k == 16)
        dp_adam_group<RMAX, 48>(a, h, 11 * n, 48, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk);
      else
        dp_adam_group<RMAX, 0>(a, h, 11 * n, 3 * a.sh_k, mu, nu, active, lr, inv_bc1, inv_bc2, blk, nblk);
  }
  // the last CTA to finish (atomic ticket, no waiting) advances the count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned total = gridDim.x;
    const unsigned t = atomicAdd(reinterpret_cast<unsigned*>(h.state + 1), 1u);
    if (t == total - 1) {
      h.state[0] = h.state[0] + 1;
      h.state[1] = 0;
    }
  }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_dp_barrier(const GsPeerSet* peers, int32_t* epoch, int32_t* status, gs_stream_t stream) {
  if (!peers || !epoch || !status) return GS_ERR_INVALID_ARGUMENT;
  if (peers->world < 1 || peers->world > GS_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->world)
    return GS_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < peers->world; ++r)
    if (!peers->flags[r]) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  GS_TIMED("dp_barrier", st);
  launch_kernel_plain(k_dp_barrier, 1, 32, 0, st, *peers, epoch, status);
  return cudaPeekAtLastError() == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

extern "C" int gs_dp_publish_barrier(const GsPeerSet* peers, const uint8_t* touched, int n, int32_t* epoch,
                                     int32_t* status, gs_stream_t stream) {
  if (!peers || !touched || n < 1 || !epoch || !status) return GS_ERR_INVALID_ARGUMENT;
  if (peers->world < 1 || peers->world > GS_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->world)
    return GS_ERR_INVALID_ARGUMENT;
  if ((long long)n * GS_MAX_RANKS > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < peers->world; ++r)
    if (!peers->flags[r] || !peers->touched_in[r]) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  GS_TIMED("dp_barrier", st);
  const int groups = (n + 15) / 16;
  const int grid = std::max(1, std::min(device_sms(), (groups + kPublishThreads - 1) / kPublishThreads));
  launch_kernel_plain(k_dp_publish_barrier, grid, kPublishThreads, 0, st, *peers, touched, n, epoch, status);
  return cudaPeekAtLastError() == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

extern "C" int gs_dp_update(const GsPeerSet* peers, float* mu, float* nu, int n, int sh_k,
                            const uint8_t* active_mask, const GsAdamSchedule* schedule,
                            int32_t* adam_state, float fx, float fy, int width, int height,
                            int tail_len, float* tail_out, const int32_t* barrier_status,
                            gs_stream_t stream) {
  if (!peers || !schedule || !adam_state || n < 0 || sh_k < 1 || sh_k > 16 || width <= 0 || height <= 0)
    return GS_ERR_INVALID_ARGUMENT;
  if (peers->world < 1 || peers->world > GS_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->world)
    return GS_ERR_INVALID_ARGUMENT;
  if (tail_len < 0 || tail_len > 256 || (tail_len > 0 && !tail_out)) return GS_ERR_INVALID_ARGUMENT;
  if ((long long)n * (11 + 3 * sh_k) + tail_len > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < peers->world; ++r)
    if (!peers->params[r] || !peers->grads[r] || !peers->radii[r] || !peers->valid[r] || !peers->w2c[r] ||
        !peers->grad_accum[r] || !peers->denom[r] || !peers->max_radii[r])
      return GS_ERR_INVALID_ARGUMENT;
  for (int g = 0; g < 5; ++g)
    if (!(schedule->transition_steps[g] > 0.f)) return GS_ERR_INVALID_ARGUMENT;
  DpArgs a;
  a.p = *peers;
  a.n = n;
  a.sh_k = sh_k;
  a.mine = dp_stripes_owned(n, peers->world, peers->rank);
  a.focal = (float)(((double)fx + (double)fy) / 2.0);
  a.pix3 = (float)((double)width * (double)height * 3.0);
  a.inv_world = 1.f / (float)peers->world;
  DpAdam h;
  for (int g = 0; g < 5; ++g) {
    h.lr_init[g] = schedule->lr_init[g];
    h.decay[g] = schedule->decay_rate[g];
    h.steps[g] = schedule->transition_steps[g];
  }
  h.b1 = (float)schedule->b1;
  h.b2 = (float)schedule->b2;
  h.omb1 = (float)(1.0 - schedule->b1);
  h.omb2 = (float)(1.0 - schedule->b2);
  h.eps = (float)schedule->eps;
  h.state = adam_state;
  {
    GS_TIMED("dp_update", stream);
    // one resident wave: the CTAs that fit on the GPU at once, shared among
    // the means + statistics phase and groups 1..4 in proportion to their
    // work (a Gaussian's statistics and means cost about 12 floats of Adam
    // streaming), so that every phase runs concurrently from the start
    const int R = peers->world;
    const int which = R <= 2 ? 0 : R <= 4 ? 1 : 2;
    const void* kernel = which == 0 ? (const void*)k_dp_adam<2> : which == 1 ? (const void*)k_dp_adam<4>
                                                                              : (const void*)k_dp_adam<8>;
    static int per_sm[3] = {0, 0, 0};
    if (per_sm[which] == 0) {
      int b = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, 256, 0);
      per_sm[which] = b > 0 ? b : 1;
    }
    const int total = device_sms() * per_sm[which];
    const int work[5] = {kDpMeansWork, 3, 4, 1, 3 * sh_k};
    const int wsum = kDpMeansWork + 8 + 3 * sh_k;
    a.cta[0] = 0;
    for (int g = 0; g < 5; ++g) a.cta[g + 1] = a.cta[g] + std::max(1, total * work[g] / wsum);
    if (which == 0)
      launch_kernel_plain(k_dp_adam<2>, a.cta[5], 256, 0, stream, a, h, mu, nu, active_mask, barrier_status, tail_len, tail_out);
    else if (which == 1)
      launch_kernel_plain(k_dp_adam<4>, a.cta[5], 256, 0, stream, a, h, mu, nu, active_mask, barrier_status, tail_len, tail_out);
    else
      launch_kernel_plain(k_dp_adam<8>, a.cta[5], 256, 0, stream, a, h, mu, nu, active_mask, barrier_status, tail_len, tail_out);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

extern "C" int gs_ipc_open(const void* handle64, void** base_out) {
  if (!handle64 || !base_out) return GS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return GS_ERR_CUDA;
  }
  *base_out = p;
  return GS_OK;
}

extern "C" int gs_ipc_close(void* base) {
  if (!base) return GS_ERR_INVALID_ARGUMENT;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return GS_ERR_CUDA;
  }
  return GS_OK;
}

