// Internal launcher declarations shared by the kernel files and the C ABI.
#pragma once

#include "gs_common.cuh"
#include "gs_timing.cuh"

#include <utility>

namespace gs {

// Programmatic dependent launch. The render path's kernels (projection,
// pair sort, compositor) are launched by launch_kernel with programmatic
// stream serialization and start with GS_PDL_ENTRY: each first waits until
// the previous grid in the stream has completed and its writes are visible
// (griddepcontrol.wait, before any memory access of the kernel), then lets
// the next grid be launched once all of its own CTAs have started
// (griddepcontrol.launch_dependents). The next kernel's launch and CTA
// set-up then overlap this kernel's tail instead of following its
// completion; the data dependence is unchanged. After anything that is not
// such a kernel (a memset, another library's kernel, a plain launch) the
// order is the usual one. The training-step kernels around the render
// (loss, Adam, statistics, data parallel, density, 2DGS) use plain launches
// (launch_kernel_plain, GS_PDL_ENTRY_PLAIN): measured on the config 2 train
// step, PDL everywhere was 2 % slower (0.426 vs 0.418 ms) while the render
// chain alone gains (config 1's fwd + L1 + bwd graph: 0.160 vs 0.166 ms) and
// the train step is unchanged. GS_PDL=0 builds plain launches throughout.
#ifndef GS_PDL
#define GS_PDL 1
#endif
#ifndef GS_PDL_TRIGGER
#define GS_PDL_TRIGGER 1
#endif
// kernels launched by launch_kernel_plain: the wait only (a no-op there)
#define GS_PDL_ENTRY_PLAIN()                                  \
  do {                                                        \
    if (GS_PDL) asm volatile("griddepcontrol.wait;" ::: "memory"); \
  } while (0)
#if GS_PDL
#define GS_PDL_ENTRY()                                                          \
  do {                                                                          \
    asm volatile("griddepcontrol.wait;" ::: "memory");                          \
    if (GS_PDL_TRIGGER) asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); \
  } while (0)
#else
#define GS_PDL_ENTRY() \
  do {                 \
  } while (0)
#endif

template <bool PDL, typename... KArgs, typename... Args>
inline cudaError_t launch_kernel_as(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (GS_PDL && PDL) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// the render path's kernels (projection, pair sort, compositor)
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args&&... args) {
  return launch_kernel_as<true>(kernel, grid, block, smem, st, std::forward<Args>(args)...);
}
// the training-step kernels around it (loss, Adam, statistics, data parallel)
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel_plain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                       cudaStream_t st, Args&&... args) {
  return launch_kernel_as<false>(kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

// Streaming multiprocessors of the current device (148 on a B200), looked up
// once per device; grids of the streaming kernels are sized from it.
inline int device_sms() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int s = 0;
    if (cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || s <= 0) s = 148;
    cache[dev] = s;
  }
  return cache[dev];
}

// True when two float4 hold the same bits (a store of one over the other
// would change nothing).
__device__ __forceinline__ bool same_bits(const float4& a, const float4& b) {
  return ((__float_as_uint(a.x) ^ __float_as_uint(b.x)) | (__float_as_uint(a.y) ^ __float_as_uint(b.y)) |
          (__float_as_uint(a.z) ^ __float_as_uint(b.z)) | (__float_as_uint(a.w) ^ __float_as_uint(b.w))) == 0u;
}

// Static camera scalars passed by value to kernels (the W2C matrix itself is
// a device buffer, read by the kernels).
struct CamParams {
  float fx, fy, cx, cy;
  int width, height, tiles_x, tiles_y;
};

// gs_preprocess.cu
void launch_preprocess_fwd(const float* means, const float* scales, const float* quats,
                           const float* opac, const float* sh, int n, int sh_k, int sh_degree,
                           const uint8_t* mask, const float* w2c, const CamParams& cp, Splat* splats,
                           int2* bins, int* block_counts, float* radii, uint8_t* valid,
                           GsExtras* extras, cudaStream_t st);
void launch_project(const float* means, const float* scales, const float* quats, int n,
                    const uint8_t* mask, const float* w2c, const CamParams& cp, float* means2d,
                    float* cov2d, float* radii, uint8_t* valid, float* depths, cudaStream_t st);
void launch_eval_sh(int deg, const float* sh, int n, int sh_k, const float* dirs, float* out,
                    cudaStream_t st);
void launch_covariance_3d(const float* scales, const float* quats, int n, float* cov, cudaStream_t st);
void launch_bin_prep(const float* means2d, const float* radii, const uint8_t* valid,
                     const float* depths, int n, int width, int height, int2* bins,
                     int* block_counts, cudaStream_t st);
void launch_pack_splats(const float* means2d, const float* cov2d, const float* opac,
                        const float* colors, int n, Splat* splats, cudaStream_t st);
void launch_splat_grads_to_inputs(const float* cov2d, const float* opac, const SplatGrad* sg, int n,
                                  float* g_means2d, float* g_cov2d, float* g_opac, float* g_colors,
                                  cudaStream_t st);
void launch_preprocess_bwd(const float* means, const float* scales, const float* quats,
                           const float* opac, const float* sh, int n, int sh_k, int sh_degree,
                           const float* w2c, const CamParams& cp, const SplatGrad* sg,
                           float* g_means, float* g_scales, float* g_quats, float* g_opac,
                           float* g_sh, uint8_t* touched, cudaStream_t st);

// gs_sort.cu
// Totals of the per-block [pairs | visible] counts (n_total, n_emit, n_vis,
// extras) and their exclusive scans (pair offsets, capped at capacity, and
// the compaction offsets of the visible Gaussians).
void launch_scan_block_counts(const int* block_counts, int n_blocks, int* pair_offsets, int* vis_offsets,
                              Scalars* sc, int64_t capacity, int num_tiles, GsExtras* extras,
                              cudaStream_t st);
// Direct path: (tile << 13 | depth) keys in Gaussian order, then a stable
// single-pass-per-digit sort on total_bits (hist[0] = first pass's digit
// counts, hist[1..] zeros, sc->sweep_tile zeros). Returns the buffer pair
// (0/1) holding the result.
void launch_emit_keys(const int2* bins, const int* pair_offsets, int n, int tiles_x, const Scalars* sc,
                      int64_t capacity, int* keys, int* ids, int* hist0, unsigned long long* status0,
                      cudaStream_t st);
int launch_radix_sort_onesweep(int* keys0, int* ids0, int* keys1, int* ids1, const int* count, Scalars* sc,
                               int* hist, unsigned long long* status0, unsigned long long* status1,
                               int total_bits, cudaStream_t st);
// The look-back's bounded wait (gs_test_set_sort_wait): spin_limit <= 0 is
// the default; blind reads every earlier status word as unpublished.
void set_sort_wait(int spin_limit, int blind);
// Pre-sort path: (depth key, index) of every Gaussian with pairs, index
// order; clears the per-block pair counts of the depth sort's output.
void launch_compact_visible(const int2* bins, int n, const int* vis_offsets, int* dkeys, int* dids,
                            int* sorted_counts, cudaStream_t st);
// (tile, Gaussian) pairs in the order of the depth-sorted Gaussians `order`,
// from the per-block pair counts of that order (scanned into offsets).
void launch_emit_sorted(const int2* bins, const int* order, int n, const Scalars* sc,
                        const int* sorted_counts, int* offsets, int tiles_x, int64_t capacity, int* keys,
                        int* ids, cudaStream_t st);
// Stable LSD sort of the *count (key, id) pairs in (keys0, ids0) by the low
// total_bits of the key, three launches per pass. counts: kRadix x max_tiles
// ints of scratch, totals: kRadix x passes. With bins and sorted_counts, the
// last pass also sums the pair counts of each 256-id block of its output.
// Returns the buffer pair (0/1) holding the result.
int launch_radix_sort(int* keys0, int* ids0, int* keys1, int* ids1, const int* count, int max_tiles,
                      int* counts, int* totals, int total_bits, const int2* bins, int* sorted_counts,
                      const char* name, cudaStream_t st);
// searchsorted(sorted_keys >> shift, arange(T+1)), side='left'.
void launch_tile_ranges_from_keys(const int* sorted_keys, int shift, const Scalars* sc, int num_tiles,
                                  int64_t capacity, int* ranges, cudaStream_t st);
void launch_tile_ranges_from_ids(const int* sorted_tile_ids, int64_t n_sorted, int num_tiles,
                                 int* ranges, cudaStream_t st);
// The reference's padded outputs: tile ids (key >> shift; T past the end) and Gaussian ids.
void launch_export_interactions(const int* keys, int shift, const int* ids, const Scalars* sc,
                                int64_t capacity, int num_tiles, int* out_tiles, int* out_ids, int* out_count,
                                cudaStream_t st);

// gs_raster.cu
// Work items (tile, 256-splat batch) per tile and the tile-count statistics.
// sort_timeouts (nullable, device): nonzero empties every range and is
// reported in extras->device_timeouts.
// tile_order (nullable): the tiles by pair count, most first (the forward's CTA order).
void launch_tile_items(int* ranges, int num_tiles, int* tile_items, Scalars* sc,
                       GsExtras* extras, const int* sort_timeouts, int* tile_order, cudaStream_t st);
void launch_raster_fwd(const Splat* splats, const int* ids, const int* ranges,
                       const int* tile_items, int n, const float* bg, int width, int height,
                       int tiles_x, int num_tiles, float* image, float* img_copy, float* pix_T,
                       float4* ckpt, int* item_info, int* item_cost, const int* tile_order, cudaStream_t st);
// The backward takes the forward's work items longest first (item_cost, the
// splat steps the forward ran per item, ordered into item_order by a small
// counting-sort kernel), so that the persistent grid ends with short items.
void launch_raster_bwd(const Splat* splats, const int* ids, const int* ranges, int n, int width,
                       int height, int tiles_x, int num_tiles, const float* grad_image,
                       const float* img, const float4* ckpt, const int* item_info, const int* item_cost,
                       int* item_order, Scalars* sc, SplatGrad* grads, const float* pix_T, float* grad_bg,
                       cudaStream_t st);

// gs_loss.cu: (1 - lambda) L1 + lambda D-SSIM and its image gradient.
size_t l1_dssim_workspace_bytes(int h, int w, int c);
void launch_l1_dssim(const float* pred, const float* target, int h, int w, int c, float lambda,
                     float* l1_out, float* dssim_out, float* ssim_out, float* loss_out, float* grad, void* ws,
                     cudaStream_t st);

// gs_density.cu: densify_and_prune / reset_opacities on the flat buffers.
size_t density_workspace_bytes(int n);
void launch_densify_and_prune(float* params, float* mu, float* nu, int n, int sh_k, uint8_t* active,
                              float* grad_accum, int* denom, const float* max_radii, const float* noise,
                              int enabled, float grad_threshold, float min_opacity, float extent,
                              float max_screen_size, void* ws, int* info, cudaStream_t st);
void launch_reset_opacities(float* params, int n, const uint8_t* active, float reset_val, cudaStream_t st);

// gs_2dgs.cu: the 2DGS surfel renderer, regularisers and flat Adam.
size_t splat2_bytes();
size_t splat2_grad_bytes();
void launch_pre2d_fwd(const float* means, const float* scales, const float* quats, const float* opac,
                      const float* sh, int n, int sh_k, const float* w2c, const CamParams& cp, void* splats,
                      int2* bins, int* block_counts, float* radii, uint8_t* valid, GsExtras* extras, cudaStream_t st);
void launch_raster2d_fwd(const void* splats, const int* ids, const int* ranges, int n, const float* bg, int width,
                         int height, int tiles_x, int num_tiles, float* image, float* depth, float* depth_sq,
                         float* normals, float* accum, float* pix_T, cudaStream_t st);
void launch_raster2d_bwd(const void* splats, const int* ids, const int* ranges, int n, int width, int height,
                         int tiles_x, int num_tiles, const float* image, const float* depth, const float* depth_sq,
                         const float* normals, const float* accum, const float* pix_T, const float* g_image,
                         const float* g_depth, const float* g_depth_sq, const float* g_normals,
                         const float* g_accum, void* grads, cudaStream_t st);
void launch_pre2d_bwd(const float* means, const float* scales, const float* quats, const float* opac,
                      const float* sh, int n, int sh_k, const float* w2c, const CamParams& cp, const void* grads,
                      float* g_means, float* g_scales, float* g_quats, float* g_opac, float* g_sh, cudaStream_t st);
size_t reg2d_workspace_bytes();
void launch_reg2d(const float* depth, const float* depth_sq, const float* normals, const float* accum, int h, int w,
                  float lam_dist, float lam_normal, float* dist_out, float* normal_out, float* g_depth,
                  float* g_depth_sq, float* g_normals, void* ws, cudaStream_t st);
// state (nullable): device [optax count before the update, CTA ticket];
// with it the bias corrections come from state[0] and the call advances it.
void launch_adam_flat(float* p, const float* g, float* m, float* v, int count, float lr, float b1, float b2,
                      float omb1, float omb2, float inv_bc1, float inv_bc2, float eps, int* state, cudaStream_t st);

// gs_train.cu
void launch_l1_loss(const float* pred, const float* target, int64_t count, float scale,
                    float* loss, float* grad, float* partials, Scalars* sc, cudaStream_t st);
void launch_mse_loss(const float* pred, const float* target, int64_t count, float scale,
                     float* loss, float* grad, float* partials, Scalars* sc, cudaStream_t st);
void launch_adam(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                 const uint8_t* active, const float lrs[5], float bc1, float bc2, float b1,
                 float b2, float omb1, float omb2, float eps, int* state, const float* sched_lr,
                 const float* sched_decay, const float* sched_steps, cudaStream_t st);
void launch_grad2d(const float* grad_means, const float* means, const float* w2c, int n, float fx,
                   float fy, int width, int height, float* out, cudaStream_t st);
void launch_step_metrics(const float* tail, const GsExtras* ex, float lambda, const int* wait_status, float* out,
                         cudaStream_t st);
void launch_step_stats(const float* grad_means, const float* means, const float* w2c, int n, float fx, float fy,
                       int width, int height, const float* radii, const uint8_t* valid, const uint8_t* active,
                       float* grad_accum, int32_t* denom, float* max_radii, float* grad2d, cudaStream_t st);
void launch_density_stats(const float* grad2d, const float* radii, const uint8_t* valid,
                          const uint8_t* radii_valid, const uint8_t* active, int n,
                          float* grad_accum, int32_t* denom, float* max_radii, cudaStream_t st);

// gs_ssim.cu
size_t dssim_workspace_bytes(int h, int w, int c);
// Zero the ticket block of a D-SSIM workspace (before every launch_dssim).
cudaError_t clear_dssim_ticket(void* ws, int h, int w, int c, cudaStream_t st);
void launch_dssim(const float* pred, const float* target, int h, int w, int c, float scale,
                  float* loss, float* ssim_out, float* grad, void* ws, cudaStream_t st);

constexpr int kLossGrid = 296;

}  // namespace gs
