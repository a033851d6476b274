// Density control: densify_and_prune and reset_opacities
// (jax_gs/training/density.py:76-211) on the flat training buffers
// [means | scales | quats | opacities | sh] (and the Adam moments in the same
// layout).
//
// The reference routes new Gaussians with three argsorts over the capacity
// (density.py:153-169): the k-th empty slot in index order receives the k-th
// clone source, then the split sources, in index order. The same routing is a
// stream compaction here: per-Gaussian flags and per-block counts, one scan,
// the list of empty slots, then one pass in which every clone / split source
// copies its row (parameters and both moments) to its slot. A slot only ever
// receives one row and sources are never slots, so rows move in place.
#include "gs_kernels.cuh"

namespace gs {

constexpr unsigned kFlagKeep = 1u, kFlagClone = 2u, kFlagSplit = 4u, kFlagEmpty = 8u, kFlagPruned = 16u;

struct DensArgs {
  int n, sh_k;
  int enabled;
  float grad_threshold, min_opacity, max_scale_prune, max_scale_split, max_screen;
  float log16;  // float32 log(1.6)
};

__device__ __forceinline__ int block_count_256(bool v, int* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = __popc(__ballot_sync(0xffffffffu, v));
  if (lane == 0) s_red[warp] = c;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += s_red[w];
  __syncthreads();
  return t;
}

// Exclusive rank of the threads with v set among the block's 256, in order.
__device__ __forceinline__ int block_rank_256(bool v, int* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned b = __ballot_sync(0xffffffffu, v);
  if (lane == 0) s_red[warp] = __popc(b);
  __syncthreads();
  int before = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) before += (w < warp) ? s_red[w] : 0;
  __syncthreads();
  unsigned lt;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
  return before + __popc(b & lt);
}

// density.py:114-135: prune / keep / densify / split / clone flags and the
// per-block counts [empty, clone, split, pruned].
__global__ void __launch_bounds__(256)
k_dens_classify(const float* __restrict__ params, const uint8_t* __restrict__ active,
                const float* __restrict__ grad_accum, const int* __restrict__ denom,
                const float* __restrict__ max_radii, DensArgs a, uint8_t* __restrict__ flags,
                int* __restrict__ counts) {
  __shared__ int s_red[8];
  const int i = blockIdx.x * 256 + threadIdx.x;
  const size_t n = (size_t)a.n;
  unsigned f = 0;
  if (i < a.n) {
    const bool act = active[i] != 0;
    const float op = params[10 * n + i];
    const float sig = (float)(1.0 / (1.0 + exp(-(double)op)));
    float ms = -INFINITY;
#pragma unroll
    for (int k = 0; k < 3; ++k) ms = fmaxf(ms, (float)exp((double)params[3 * n + 3 * (size_t)i + k]));
    bool prune = (sig < a.min_opacity) | (ms > a.max_scale_prune) | (max_radii[i] > a.max_screen);
    prune = prune & act;
    const bool keep = act & !prune;
    const int dn = denom[i];
    const float avg = dn > 0 ? __fdiv_rn(grad_accum[i], (float)dn) : 0.f;
    const bool dens = (avg >= a.grad_threshold) & keep;
    const bool split = dens & (ms > a.max_scale_split);
    const bool clone = dens & !split;
    f = (keep ? kFlagKeep : 0u) | (clone ? kFlagClone : 0u) | (split ? kFlagSplit : 0u) |
        (keep ? 0u : kFlagEmpty) | (prune ? kFlagPruned : 0u);
    flags[i] = (uint8_t)f;
  }
  const int ce = block_count_256(f & kFlagEmpty, s_red);
  const int cc = block_count_256(f & kFlagClone, s_red);
  const int cs = block_count_256(f & kFlagSplit, s_red);
  const int cp = block_count_256(f & kFlagPruned, s_red);
  if (threadIdx.x == 0) {
    const int nb = gridDim.x;
    counts[blockIdx.x] = ce;
    counts[nb + blockIdx.x] = cc;
    counts[2 * nb + blockIdx.x] = cs;
    counts[3 * nb + blockIdx.x] = cp;
  }
}

// Exclusive scans of the [empty, clone, split] block counts (single CTA) and
// the capacity decision (density.py:141-151); info = [pruned, clones, splits,
// applied].
__global__ void __launch_bounds__(1024)
k_dens_scan(const int* __restrict__ counts, int nb, int enabled, int* __restrict__ offsets,
            int* __restrict__ info) {
  __shared__ int s_warp[32];
  __shared__ int s_carry[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int a = 0; a < 4; ++a) {
    if (tid == 0) s_carry[a] = 0;
    __syncthreads();
    for (int base = 0; base < nb; base += 1024) {
      const int i = base + tid;
      const int v = (i < nb) ? counts[a * nb + i] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) s_warp[warp] = x;
      __syncthreads();
      if (warp == 0) {
        int w = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, w, o);
          if (lane >= o) w += y;
        }
        s_warp[lane] = w;
      }
      __syncthreads();
      if (a < 3 && i < nb) offsets[a * nb + i] = s_carry[a] + (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
      const int blk = s_warp[31];
      __syncthreads();
      if (tid == 0) s_carry[a] += blk;
      __syncthreads();
    }
  }
  if (tid == 0) {
    const int empty = s_carry[0], clones = s_carry[1], splits = s_carry[2];
    const bool can = enabled && (clones + splits <= empty);
    info[0] = s_carry[3];
    info[1] = can ? clones : 0;
    info[2] = can ? splits : 0;
    info[3] = (can && clones + splits > 0) ? 1 : 0;
  }
}

// Slot list: empty_list[r] = the r-th empty slot in index order.
__global__ void __launch_bounds__(256)
k_dens_empty_list(const uint8_t* __restrict__ flags, int n, const int* __restrict__ offsets,
                  int* __restrict__ empty_list) {
  __shared__ int s_red[8];
  const int i = blockIdx.x * 256 + threadIdx.x;
  const bool e = (i < n) && (flags[i] & kFlagEmpty);
  const int r = block_rank_256(e, s_red);
  if (e) empty_list[offsets[blockIdx.x] + r] = i;
}

__device__ __forceinline__ void copy_row(float* __restrict__ buf, size_t n, int sh_k, int src, int dst) {
  float* b = buf;
#pragma unroll
  for (int k = 0; k < 3; ++k) b[3 * (size_t)dst + k] = b[3 * (size_t)src + k];
  b += 3 * n;
#pragma unroll
  for (int k = 0; k < 3; ++k) b[3 * (size_t)dst + k] = b[3 * (size_t)src + k];
  b += 3 * n;
#pragma unroll
  for (int k = 0; k < 4; ++k) b[4 * (size_t)dst + k] = b[4 * (size_t)src + k];
  b += 4 * n;
  b[dst] = b[src];
  b += n;
  const int w = 3 * sh_k;
  for (int k = 0; k < w; ++k) b[(size_t)w * dst + k] = b[(size_t)w * src + k];
}

// density.py:183-190 on row r: scales -= log(1.6), means += noise[r] * exp(scales).
__device__ __forceinline__ void split_row(float* __restrict__ params, size_t n, int r, float log16,
                                          const float* __restrict__ noise) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    float& s = params[3 * n + 3 * (size_t)r + k];
    s = __fsub_rn(s, log16);
    const float e = (float)exp((double)s);
    float& m = params[3 * (size_t)r + k];
    m = __fadd_rn(m, __fmul_rn(noise[3 * (size_t)r + k], e));
  }
}

// Clone / split sources copy their rows to their slots; every Gaussian sets
// its own final active flag and resets its accumulators (density.py:171-206).
__global__ void __launch_bounds__(256)
k_dens_move(float* __restrict__ params, float* __restrict__ mu, float* __restrict__ nu,
            uint8_t* __restrict__ active, float* __restrict__ grad_accum, int* __restrict__ denom,
            const uint8_t* __restrict__ flags, const int* __restrict__ offsets,
            const int* __restrict__ empty_list, const int* __restrict__ info, const float* __restrict__ noise,
            DensArgs a) {
  __shared__ int s_red[8];
  const int i = blockIdx.x * 256 + threadIdx.x;
  const int nb = gridDim.x;
  const int nc = info[1], ns = info[2];
  const unsigned f = (i < a.n) ? flags[i] : 0u;
  const bool clone = (f & kFlagClone) && nc > 0;  // nc, ns are 0 when densification is off
  const bool split = (f & kFlagSplit) && ns > 0;
  const int rc = block_rank_256(clone, s_red);
  const int rs = block_rank_256(split, s_red);
  const int re = block_rank_256(f & kFlagEmpty, s_red);
  if (i >= a.n) return;
  const size_t n = (size_t)a.n;
  if (clone || split) {
    const int k = clone ? offsets[nb + blockIdx.x] + rc : nc + offsets[2 * nb + blockIdx.x] + rs;
    const int d = empty_list[k];
    copy_row(params, n, a.sh_k, i, d);
    copy_row(mu, n, a.sh_k, i, d);
    copy_row(nu, n, a.sh_k, i, d);
    if (split) {
      split_row(params, n, d, a.log16, noise);
      split_row(params, n, i, a.log16, noise);
    }
  }
  const bool dest = (f & kFlagEmpty) && (offsets[blockIdx.x] + re < nc + ns);
  active[i] = ((f & kFlagKeep) || dest) ? 1 : 0;
  grad_accum[i] = 0.f;
  denom[i] = 0;
}

// density.py:76-96: active opacities set to inv (the logit of reset_val).
__global__ void __launch_bounds__(256)
k_reset_opacities(float* __restrict__ params, int n, const uint8_t* __restrict__ active, float inv) {
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < n && active[i]) params[10 * (size_t)n + i] = inv;
}

size_t density_workspace_bytes(int n) {
  const size_t nb = (size_t)((n + 255) / 256);
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  return al((size_t)n) + al(4 * nb * sizeof(int)) + al(3 * nb * sizeof(int)) + al((size_t)n * sizeof(int));
}

void launch_densify_and_prune(float* params, float* mu, float* nu, int n, int sh_k, uint8_t* active,
                              float* grad_accum, int* denom, const float* max_radii, const float* noise,
                              int enabled, float grad_threshold, float min_opacity, float extent,
                              float max_screen_size, void* ws, int* info, cudaStream_t st) {
  const int nb = (n + 255) / 256;
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  char* base = (char*)ws;
  uint8_t* flags = (uint8_t*)base;
  int* counts = (int*)(base + al((size_t)n));
  int* offsets = (int*)((char*)counts + al(4 * (size_t)nb * sizeof(int)));
  int* empty_list = (int*)((char*)offsets + al(3 * (size_t)nb * sizeof(int)));
  DensArgs a;
  a.n = n;
  a.sh_k = sh_k;
  a.enabled = enabled;
  a.grad_threshold = grad_threshold;
  a.min_opacity = min_opacity;
  // JAX compares the float32 arrays with the Python products as float32
  a.max_scale_prune = (float)(0.1 * (double)extent);
  a.max_scale_split = (float)(0.01 * (double)extent);
  a.max_screen = max_screen_size;
  a.log16 = (float)log((double)1.6f);
  if (nb == 0) {
    cudaMemsetAsync(info, 0, 4 * sizeof(int), st);
    return;
  }
  GS_TIMED("densify", st);
  k_dens_classify<<<nb, 256, 0, st>>>(params, active, grad_accum, denom, max_radii, a, flags, counts);
  k_dens_scan<<<1, 1024, 0, st>>>(counts, nb, enabled, offsets, info);
  k_dens_empty_list<<<nb, 256, 0, st>>>(flags, n, offsets, empty_list);
  k_dens_move<<<nb, 256, 0, st>>>(params, mu, nu, active, grad_accum, denom, flags, offsets, empty_list, info,
                                  noise, a);
}

void launch_reset_opacities(float* params, int n, const uint8_t* active, float reset_val, cudaStream_t st) {
  if (n <= 0) return;
  const float inv = (float)log((double)(float)((double)reset_val / (1.0 - (double)reset_val)));
  GS_TIMED("reset_opacities", st);
  k_reset_opacities<<<(n + 255) / 256, 256, 0, st>>>(params, n, active, inv);
}

}  // namespace gs
