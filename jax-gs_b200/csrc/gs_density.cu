// Density control: densify_and_prune and reset_opacities
// (jax_gs/training/density.py:76-211) on the flat training buffers
// [means | scales | quats | opacities | sh] (and the Adam moments in the same
// layout).
//
// The reference routes new Gaussians with three argsorts over the capacity
// (density.py:153-169): the k-th empty slot in index order receives the k-th
// clone source, then the split sources, in index order. The same routing is a
// stream compaction here: per-Gaussian flags and per-block counts, one scan,
// the list of empty slots, the list of moves (source, slot), then one warp per
// move copies the row (parameters and both moments). A slot only ever
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
  GS_PDL_ENTRY_PLAIN();
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
  GS_PDL_ENTRY_PLAIN();
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
  GS_PDL_ENTRY_PLAIN();
  __shared__ int s_red[8];
  const int i = blockIdx.x * 256 + threadIdx.x;
  const bool e = (i < n) && (flags[i] & kFlagEmpty);
  const int r = block_rank_256(e, s_red);
  if (e) empty_list[offsets[blockIdx.x] + r] = i;
}

// One row move by a whole warp: the 11 + 3K floats of Gaussian src copied to
// dst in params, mu and nu (lanes over each group's floats, so the accesses
// coalesce).
__device__ __forceinline__ void warp_copy_row(float* __restrict__ buf, size_t n, int w_sh, int src, int dst,
                                              int lane) {
  const int seg_w[5] = {3, 3, 4, 1, w_sh};
  size_t base = 0;
#pragma unroll
  for (int g = 0; g < 5; ++g) {
    const int w = seg_w[g];
    for (int k = lane; k < w; k += 32) buf[base + (size_t)w * dst + k] = buf[base + (size_t)w * src + k];
    base += (size_t)w * n;
  }
}

// density.py:183-190 on coordinate k of row r: scales -= log(1.6),
// means += noise[r] * exp(scales).
__device__ __forceinline__ void split_row(float* __restrict__ params, size_t n, int r, float log16,
                                          const float* __restrict__ noise, int k) {
  float& s = params[3 * n + 3 * (size_t)r + k];
  s = __fsub_rn(s, log16);
  const float e = (float)exp((double)s);
  float& m = params[3 * (size_t)r + k];
  m = __fadd_rn(m, __fmul_rn(noise[3 * (size_t)r + k], e));
}

// Every Gaussian sets its own final active flag, resets its accumulators and,
// as a clone / split source, records its move: move k goes to the k-th empty
// slot, clones first, then splits, each in index order (density.py:153-195).
__global__ void __launch_bounds__(256)
k_dens_route(uint8_t* __restrict__ active, float* __restrict__ grad_accum, int* __restrict__ denom,
             const uint8_t* __restrict__ flags, const int* __restrict__ offsets,
             const int* __restrict__ empty_list, const int* __restrict__ info, int2* __restrict__ moves,
             DensArgs a) {
  GS_PDL_ENTRY_PLAIN();
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
  if (clone || split) {
    const int k = clone ? offsets[nb + blockIdx.x] + rc : nc + offsets[2 * nb + blockIdx.x] + rs;
    moves[k] = make_int2(i, split ? -1 - empty_list[k] : empty_list[k]);  // split: slot coded negative
  }
  const bool dest = (f & kFlagEmpty) && (offsets[blockIdx.x] + re < nc + ns);
  active[i] = ((f & kFlagKeep) || dest) ? 1 : 0;
  grad_accum[i] = 0.f;
  denom[i] = 0;
}

// The moves, one warp each, over a persistent grid.
__global__ void __launch_bounds__(256)
k_dens_copy(float* __restrict__ params, float* __restrict__ mu, float* __restrict__ nu,
            const int2* __restrict__ moves, const int* __restrict__ info, const float* __restrict__ noise,
            DensArgs a) {
  GS_PDL_ENTRY_PLAIN();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int total = info[1] + info[2];
  const size_t n = (size_t)a.n;
  const int w_sh = 3 * a.sh_k;
  for (int m = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); m < total; m += warps) {
    const int2 mv = moves[m];
    const bool split = mv.y < 0;
    const int src = mv.x, dst = split ? -1 - mv.y : mv.y;
    warp_copy_row(params, n, w_sh, src, dst, lane);
    warp_copy_row(mu, n, w_sh, src, dst, lane);
    warp_copy_row(nu, n, w_sh, src, dst, lane);
    __syncwarp();  // the source row is read before the split changes it
    if (split && lane < 3) {
      split_row(params, n, dst, a.log16, noise, lane);
      split_row(params, n, src, a.log16, noise, lane);
    }
  }
}

// density.py:76-96: active opacities set to inv (the logit of reset_val).
__global__ void __launch_bounds__(256)
k_reset_opacities(float* __restrict__ params, int n, const uint8_t* __restrict__ active, float inv) {
  GS_PDL_ENTRY_PLAIN();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < n && active[i]) params[10 * (size_t)n + i] = inv;
}

size_t density_workspace_bytes(int n) {
  const size_t nb = (size_t)((n + 255) / 256);
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  return al((size_t)n) + al(4 * nb * sizeof(int)) + al(3 * nb * sizeof(int)) + al((size_t)n * sizeof(int)) +
         al((size_t)n * sizeof(int2));
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
  int2* moves = (int2*)((char*)empty_list + al((size_t)n * sizeof(int)));
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
  launch_kernel_plain(k_dens_classify, nb, 256, 0, st, params, active, grad_accum, denom, max_radii, a, flags, counts);
  launch_kernel_plain(k_dens_scan, 1, 1024, 0, st, counts, nb, enabled, offsets, info);
  launch_kernel_plain(k_dens_empty_list, nb, 256, 0, st, flags, n, offsets, empty_list);
  launch_kernel_plain(k_dens_route, nb, 256, 0, st, active, grad_accum, denom, flags, offsets, empty_list, info, moves, a);
  static int grid = 0;  // resident CTAs (the GPUs of one node have the same SM count)
  if (grid == 0) {
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_dens_copy, 256, 0);
    grid = sms * (per_sm > 0 ? per_sm : 1);
  }
  launch_kernel_plain(k_dens_copy, grid, 256, 0, st, params, mu, nu, moves, info, noise, a);
}

void launch_reset_opacities(float* params, int n, const uint8_t* active, float reset_val, cudaStream_t st) {
  if (n <= 0) return;
  const float inv = (float)log((double)(float)((double)reset_val / (1.0 - (double)reset_val)));
  GS_TIMED("reset_opacities", st);
  launch_kernel_plain(k_reset_opacities, (n + 255) / 256, 256, 0, st, params, n, active, inv);
}

}  // namespace gs
