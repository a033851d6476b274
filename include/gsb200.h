/*
 * gsb200.h -- C ABI of the B200 (sm_100a) differentiable tiled Gaussian-splat
 * renderer that stands in for jax-gs's `jax_gs.renderer` package.
 *
 * Conventions
 *  - Every pointer argument is a DEVICE pointer unless its comment says "host".
 *  - All arrays are fp32 / int32 / uint8, C-contiguous, row-major, with the
 *    shapes of the reference arrays they replace (N = static capacity).
 *  - No entry point allocates device memory, synchronises the stream or keeps
 *    global mutable state: scratch comes from a caller-owned `workspace` of at
 *    least gs_workspace_bytes(...) bytes, and all work is ordered on `stream`.
 *    The exceptions are named where they are declared: gs_dssim_loss_noalloc
 *    (its scratch is one array compiled into the library, shared by every
 *    call), gs_check_extras (synchronises the stream to read the health
 *    block), the kernel-timing aids gs_timing_* (process-global event
 *    records) and the test aid gs_test_set_sort_wait (a process-global
 *    setting of the sort's bounded wait).
 *  - Every entry point returns GS_OK (0) or a status code; gs_status_string()
 *    names it. Argument errors are detected on the host before any launch.
 *    Conditions that only the device can see (interaction capacity overflow, a
 *    bounded wait that gave up) are written to the device-side GsExtras block
 *    (or the caller's status word) and never cause an out-of-bounds access;
 *    gs_check_extras turns them into a status on the host.
 *
 * The reference functions each entry point replaces are cited as
 * file:line inside the jax-gs project.
 */
#ifndef GSB200_H_
#define GSB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported symbols keep default visibility (the library builds with
 * -fvisibility=hidden). */
#if defined(__GNUC__)
#define GS_API __attribute__((visibility("default")))
#else
#define GS_API
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* gs_stream_t;

/* Renderer constants, jax_gs/renderer/rasterizer.py:6-10 (same names/values). */
#define GS_TILE_SIZE 16
#define GS_OFFSET_SIZE 16
#define GS_BLOCK_SIZE 512
#define GS_MAX_TILE_CHUNKS 8
#define GS_MAX_TILE_INTERACTIONS (GS_BLOCK_SIZE * GS_MAX_TILE_CHUNKS)
/* Depth bits of the packed (tile << 13 | depth) key, rasterizer.py:84. */
#define GS_DEPTH_BITS 13

/* Status codes. */
#define GS_OK 0
#define GS_ERR_INVALID_ARGUMENT 1
#define GS_ERR_CAPACITY 2
#define GS_ERR_DEVICE_TIMEOUT 3
#define GS_ERR_CUDA 4
#define GS_ERR_WORKSPACE_TOO_SMALL 5
#define GS_ERR_TOO_LARGE 6

/*
 * Health counters of one render, jax_gs/renderer/renderer.py:79-90, written on
 * the device by gs_render_forward. 64 bytes, naturally aligned.
 */
typedef struct GsExtras {
  int32_t n_interactions;            /* valid (Gaussian, tile) pairs         */
  float mean_interactions_per_tile;  /* n_interactions / num_tiles           */
  int32_t max_interactions_per_tile; /* max over tiles of the pair count     */
  int32_t overflow_tiles;            /* tiles with > BLOCK_SIZE pairs        */
  int32_t overflow_interactions;     /* sum of max(count - BLOCK_SIZE, 0)    */
  int32_t truncated_tiles;           /* tiles with > MAX_TILE_INTERACTIONS   */
  int32_t truncated_interactions;    /* sum of max(count - MAX_TILE_..., 0)  */
  int32_t radius_cap_violations;     /* valid on-screen splats spanning > 16 tiles */
  int32_t capacity_overflow;         /* pairs that did not fit `capacity` (0 = none) */
  int32_t num_tiles;                 /* tiles_x * tiles_y                    */
  int32_t device_timeouts;           /* bounded device waits that gave up (the
                                        direct-path sort's look-back); 0 in a
                                        healthy run. Nonzero: the pair order is
                                        unknown, so every tile range is emptied
                                        and the image holds the background only
                                        -- the outputs are not the render. */
  int32_t reserved[5];
} GsExtras;

/* ---- housekeeping ------------------------------------------------------ */

GS_API const char* gs_status_string(int status);
/* Library ABI version, (major << 16) | minor. */
GS_API int gs_version(void);
/* Number of (Gaussian, tile) slots the reference materialises: n * OFFSET_SIZE^2
 * (rasterizer.py:56-77). With this capacity an overflow cannot happen. */
GS_API int64_t gs_default_capacity(int n);
/* Bytes of scratch that every entry point below needs for this problem size. */
GS_API size_t gs_workspace_bytes(int n, int width, int height, int64_t capacity);

/*
 * The device-side conditions of one render as a host status (no reference
 * counterpart: under XLA a failed custom call returns ffi::Error). Waits for
 * `stream`, reads the GsExtras block `extras` (device) and returns
 * GS_ERR_DEVICE_TIMEOUT if a bounded device wait gave up (the outputs are not
 * the render), GS_ERR_CAPACITY if pairs did not fit the capacity (the outputs
 * lack those pairs), else GS_OK. It synchronises the stream: call it where the
 * caller reads results back anyway, or when debugging.
 */
GS_API int gs_check_extras(const GsExtras* extras, gs_stream_t stream);

/* ---- stage entry points (one per reference function) ------------------- */

/*
 * project_gaussians, jax_gs/renderer/projection.py:6-79 (with
 * get_covariance_3d, jax_gs/core/gaussians.py:58-93).
 * means/scales (N,3), quats (N,4) wxyz, mask (N,) or NULL, w2c (4,4).
 * Outputs: means2d (N,2), cov2d (N,2,2), radii (N,), valid (N,), depths (N,).
 */
GS_API int gs_project_gaussians(const float* means, const float* scales, const float* quats, int n,
                         const uint8_t* mask, const float* w2c, int width, int height,
                         float fx, float fy, float cx, float cy, float* means2d, float* cov2d,
                         float* radii, uint8_t* valid, float* depths, gs_stream_t stream);

/*
 * get_covariance_3d, jax_gs/core/gaussians.py:58-93: Sigma = M M^T with
 * M = R(q / |q|) diag(exp(scales)), for scales (N,3) and quats (N,4) wxyz;
 * cov3d (N,3,3) row-major. The arithmetic (and so every bit) is the one
 * gs_project_gaussians uses for the same Gaussians.
 */
GS_API int gs_covariance_3d(const float* scales, const float* quats, int n, float* cov3d, gs_stream_t stream);

/*
 * eval_sh, jax_gs/renderer/sh.py:25-74. sh (N,K,3), view_dirs (N,3) -> out (N,3).
 */
GS_API int gs_eval_sh(int sh_degree, const float* sh, int n, int sh_k, const float* view_dirs,
               float* out, gs_stream_t stream);

/*
 * get_tile_interactions, jax_gs/renderer/rasterizer.py:12-116, followed by the
 * tile-range search of rasterizer.py:158-160 / renderer.py:57-61.
 * Writes the VALID interactions only, sorted by (tile, 13-bit depth key) with
 * ties in Gaussian order -- the reference's stable lax.sort_key_val order with
 * its sentinel and behind-camera entries removed. Slots [n_interactions,
 * capacity) are filled with tile id = num_tiles and Gaussian id 0, as the
 * reference pads. tile_ranges (num_tiles+1,) = searchsorted(tiles, arange(T+1)).
 * n_interactions is a device int32 scalar.
 */
GS_API int gs_get_tile_interactions(const float* means2d, const float* radii, const uint8_t* valid,
                             const float* depths, int n, int height, int width,
                             int64_t capacity, void* workspace, size_t workspace_bytes,
                             int32_t* sorted_tile_ids, int32_t* sorted_gaussian_ids,
                             int32_t* n_interactions, int32_t* tile_ranges,
                             gs_stream_t stream);

/*
 * render_tiles, jax_gs/renderer/rasterizer.py:119-248 (and the equivalent
 * render_tiles_tpu, rasterizer_tpu.py:13-135). sorted_tile_ids /
 * sorted_gaussian_ids are any (n_sorted,) arrays in the reference's sorted
 * layout (tile ids may include -1 and the num_tiles sentinel).
 * opacities are the raw logits (N,1); background (3,) or NULL for zeros.
 * image (H,W,3).
 */
GS_API int gs_render_tiles(const float* means2d, const float* cov2d, const float* opacities,
                    const float* colors, int n, const int32_t* sorted_tile_ids,
                    const int32_t* sorted_gaussian_ids, int64_t n_sorted, int height, int width,
                    const float* background, void* workspace, size_t workspace_bytes,
                    float* image, gs_stream_t stream);

/*
 * Vector-Jacobian product of render_tiles with respect to means2d, cov2d,
 * opacities (raw logits) and colors, given grad_image (H,W,3). Any output
 * pointer may be NULL. This is what jax.vjp of rasterizer.py:119-248 returns.
 */
GS_API int gs_render_tiles_backward(const float* means2d, const float* cov2d, const float* opacities,
                             const float* colors, int n, const int32_t* sorted_tile_ids,
                             const int32_t* sorted_gaussian_ids, int64_t n_sorted, int height,
                             int width, const float* background, const float* grad_image,
                             void* workspace, size_t workspace_bytes, float* grad_means2d,
                             float* grad_cov2d, float* grad_opacities, float* grad_colors,
                             gs_stream_t stream);

/* ---- fused renderer (the production path) ----------------------------- */

/*
 * render, jax_gs/renderer/renderer.py:15-107: projection + SH colour + tile
 * keys + device radix sort + tile ranges + front-to-back compositor, in one
 * stream-ordered call. Inputs are the Gaussians fields (means (N,3), scales
 * (N,3), quats (N,4), opacities (N,1), sh (N,K,3)), the optional active mask,
 * the device W2C (4,4) and background (3,) (NULL = zeros) and the static
 * camera scalars. Outputs: image (H,W,3), radii (N,), valid_mask (N,) and the
 * GsExtras block (device). The workspace keeps the residuals that
 * gs_render_backward reads; pass the same workspace, unmodified, to it.
 */
GS_API int gs_render_forward(const float* means, const float* scales, const float* quats,
                      const float* opacities, const float* sh, int n, int sh_k,
                      const uint8_t* mask, const float* w2c, int width, int height, float fx,
                      float fy, float cx, float cy, const float* background, int sh_degree,
                      int64_t capacity, void* workspace, size_t workspace_bytes, float* image,
                      float* radii, uint8_t* valid_mask, GsExtras* extras, gs_stream_t stream);

/*
 * gs_render_forward without the residuals of the backward (no per-batch
 * checkpoints, work items, final transmittance or image copy): the same
 * image, radii, valid_mask and extras, for render() calls that take no
 * gradient (jax_gs/renderer/renderer.py:15-107 as called by
 * animate_ply.py:134,141 and evaluation). Same arguments and workspace size;
 * gs_render_backward must not be called on this workspace afterwards.
 */
GS_API int gs_render_image(const float* means, const float* scales, const float* quats,
                    const float* opacities, const float* sh, int n, int sh_k,
                    const uint8_t* mask, const float* w2c, int width, int height, float fx,
                    float fy, float cx, float cy, const float* background, int sh_degree,
                    int64_t capacity, void* workspace, size_t workspace_bytes, float* image,
                    float* radii, uint8_t* valid_mask, GsExtras* extras, gs_stream_t stream);

/*
 * Backward of gs_render_forward (what jax.value_and_grad of render gives for
 * the Gaussians fields, trainer.py:66/137). grad_image (H,W,3) is dL/dimage.
 * Writes every element of grad_means (N,3), grad_scales (N,3), grad_quats
 * (N,4), grad_opacities (N,1), grad_sh (N,K,3); Gaussians without a pair get
 * exact zeros. grad_background (3,) may be NULL. touched (N,) may be NULL
 * (no reference counterpart; an output for the data-parallel update): 1
 * where Gaussian i received a nonzero compositor gradient, 0 where its whole
 * gradient row was written as exact +0, so gs_dp_update need not read it.
 */
GS_API int gs_render_backward(const float* means, const float* scales, const float* quats,
                       const float* opacities, const float* sh, int n, int sh_k,
                       const uint8_t* mask, const float* w2c, int width, int height, float fx,
                       float fy, float cx, float cy, const float* background, int sh_degree,
                       int64_t capacity, void* workspace, size_t workspace_bytes,
                       const float* grad_image, float* grad_means, float* grad_scales,
                       float* grad_quats, float* grad_opacities, float* grad_sh,
                       float* grad_background, uint8_t* touched, gs_stream_t stream);

/* ---- training-step kernels around the renderer ------------------------- */

/*
 * l1_loss, jax_gs/training/losses.py:4-8: loss = mean(|pred - target|) over
 * `count` elements, written to the device scalar `loss`; grad_pred (count,)
 * = sign(pred - target) * scale / count if not NULL (scale multiplies the
 * gradient, e.g. the 0.8 of trainer.py:26). Deterministic reduction.
 */
GS_API int gs_l1_loss(const float* pred, const float* target, int64_t count, float scale, float* loss,
               float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream);

/*
 * mse_loss, jax_gs/training/losses.py:10-14: loss = mean((pred - target)^2)
 * over `count` elements; grad_pred (count,) = 2 (pred - target) scale / count
 * if not NULL. Arguments and workspace as gs_l1_loss.
 */
GS_API int gs_mse_loss(const float* pred, const float* target, int64_t count, float scale, float* loss,
                float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream);

/*
 * d_ssim_loss, jax_gs/training/losses.py:16-75 (11-tap separable Gaussian
 * window, sigma 1.5, SAME zero padding, C1 = 0.01^2, C2 = 0.03^2):
 * loss = max(0, (1 - mean(ssim_map)) / 2) for (H,W,C) images.
 * grad_pred (H,W,C) += scale * dloss/dpred if not NULL (accumulates, so the
 * L1 gradient can be written first). ssim_out (device scalar) may be NULL.
 */
GS_API int gs_dssim_loss(const float* pred, const float* target, int height, int width, int channels,
                  float scale, float* loss, float* ssim_out, float* grad_pred, void* workspace,
                  size_t workspace_bytes, gs_stream_t stream);
GS_API size_t gs_dssim_workspace_bytes(int height, int width, int channels);

/*
 * The loss of the reference's training step, trainer.py:18-26:
 * loss = (1 - lambda_dssim) * l1_loss + lambda_dssim * d_ssim_loss
 * (losses.py:4-8, :71-75; lambda_dssim = 0.2 there), for (H,W,C) images,
 * C <= 3, in two kernels. Device scalars written when not NULL: l1, dssim,
 * ssim_out (mean SSIM map), loss. grad_pred (H,W,C), if not NULL, is
 * written (not accumulated) with dloss/dpred. Deterministic reductions.
 * Workspace: gs_l1_dssim_workspace_bytes(H, W, C) bytes, 256-byte aligned.
 */
GS_API int gs_l1_dssim_loss(const float* pred, const float* target, int height, int width, int channels,
                     float lambda_dssim, float* l1, float* dssim, float* ssim_out, float* loss,
                     float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream);
GS_API size_t gs_l1_dssim_workspace_bytes(int height, int width, int channels);

/*
 * One optax.adam step per parameter group (optax.multi_transform of
 * train.py:129-156 / train_parallel.py:142-170) followed by the active-mask
 * update masking of trainer.py:44-53/73-77. params/grads/mu/nu are flat fp32
 * buffers holding [means (N,3) | scales (N,3) | quats (N,4) | opacities (N,1)
 * | sh (N,K,3)] back to back. lrs (host, 5 floats) are the per-group learning
 * rates for this step; step is optax's count after the increment (1 for the
 * first update). Updates of inactive Gaussians are zeroed; mu/nu of every
 * element are updated exactly as optax does. b1, b2, eps are the Python-float
 * hyper-parameters: 1 - b is formed in double and rounded once, as JAX does
 * with weakly typed constants, and the bias corrections are 1 - f32(b)^step.
 */
GS_API int gs_adam_step(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                 const uint8_t* active_mask, const float* lrs, int step, double b1, double b2,
                 double eps, gs_stream_t stream);

/*
 * The same Adam step with the hyper-parameters evaluated on the device, so a
 * captured CUDA graph can replay it: state (device int32[2]) holds optax's
 * count before the step and a ticket the kernel uses internally; the call
 * reads the count, uses learning rate lr_init[g] * decay_rate[g] ^
 * (count / transition_steps[g]) for group g (optax.exponential_decay;
 * decay_rate 1 = constant) and bias corrections 1 - b^(count+1), and
 * leaves count + 1 in state[0]. schedule is read on the host at call time.
 */
typedef struct GsAdamSchedule {
  float lr_init[5];
  float decay_rate[5];
  float transition_steps[5];
  double b1, b2, eps;
} GsAdamSchedule;
GS_API int gs_adam_step_scheduled(float* params, const float* grads, float* mu, float* nu, int n,
                                  int sh_k, const uint8_t* active_mask,
                                  const GsAdamSchedule* schedule, int32_t* state,
                                  gs_stream_t stream);

/*
 * Data-parallel step tail over NVLink peer memory, replacing the pmean /
 * pmax all-reduces of trainer.py:69-71, :97, :108-111 followed by the optax
 * update (:73-77) and the statistics (:99-113). Rank r of R owns the stripes
 * of GS_DP_STRIPE consecutive Gaussians whose stripe index is r modulo R
 * (Gaussian i belongs to rank (i / GS_DP_STRIPE) % R): it reads those
 * Gaussians' entries of every rank's gradient buffer through peer pointers,
 * averages them (fixed rank order), runs the masked Adam step on them with
 * its own mu / nu (so each rank keeps the moments of its stripes only), and
 * writes the updated parameters and statistics into every rank's buffers,
 * leaving all parameter replicas bitwise identical. The caller orders the
 * ranks around the call (all gradients final before it, all peer writes
 * done before the next step), e.g. with gs_dp_barrier on each side.
 * All pointers in GsPeerSet are device pointers valid in the calling process
 * (peers through CUDA IPC). Buffers use the flat layout of gs_adam_step;
 * grads carries tail_len extra floats (loss and metrics), averaged into
 * tail_out. denom uses each rank's own valid mask; max_radii the max over
 * ranks of valid-masked radii, as the reference does.
 * barrier_status (device int32, nullable) is the status word of this rank's
 * gs_dp_barrier calls: when it is nonzero (a rendezvous gave up, so a peer
 * may be absent or gone) the kernels touch no peer memory at all and leave
 * this rank's parameters, moments, statistics and tail_out unchanged; the
 * optax count is not advanced. The caller reads the word on the host
 * (gs_train_step_metrics reports it) and stops the run.
 * touched_in[r] (all NULL, or all set) is rank r's inbox of touched flags:
 * GS_MAX_RANKS rows of n bytes, row q holding rank q's touched flags
 * (gs_render_backward) for the Gaussians rank r owns, written by
 * gs_dp_publish_barrier. With them, rank r reads rank q's gradient row of a
 * Gaussian over NVLink only where q's flag is 1 (a 0 row is exact +0, and
 * adding +0 changes no sum the update uses); NULL: every row is read.
 */
#define GS_MAX_RANKS 8
#define GS_DP_STRIPE 32
typedef struct GsPeerSet {
  int32_t world, rank;
  float* params[GS_MAX_RANKS];
  const float* grads[GS_MAX_RANKS];
  const float* radii[GS_MAX_RANKS];
  const uint8_t* valid[GS_MAX_RANKS];
  const float* w2c[GS_MAX_RANKS];
  float* grad_accum[GS_MAX_RANKS];
  int32_t* denom[GS_MAX_RANKS];
  float* max_radii[GS_MAX_RANKS];
  int32_t* flags[GS_MAX_RANKS]; /* each rank's GS_MAX_RANKS rendezvous words (gs_dp_barrier), zeroed once */
  uint8_t* touched_in[GS_MAX_RANKS];
  /* each rank's GsExtras as int32 words (nullable): when set, tail_out[3..11]
   * average the render counters read from there (words 0..7, word 1 a float,
   * then device_timeouts) instead of those tail floats of the gradients */
  const int32_t* extras[GS_MAX_RANKS];
} GsPeerSet;
GS_API int gs_dp_update(const GsPeerSet* peers, float* mu, float* nu, int n, int sh_k,
                        const uint8_t* active_mask, const GsAdamSchedule* schedule,
                        int32_t* adam_state, float fx, float fy, int width, int height,
                        int tail_len, float* tail_out, const int32_t* barrier_status,
                        gs_stream_t stream);

/*
 * Stream-ordered rendezvous of the ranks of a GsPeerSet over peer memory (no
 * reference counterpart: it stands in for the one-element all-reduce that
 * orders pmap's collectives): one small kernel raises this rank's word in
 * every rank's flags array to the next epoch (*epoch, a device counter of
 * this rank, advanced by the call) after a system-scope fence, then waits
 * until every rank's word in its own array reached that epoch. The wait is
 * bounded (about a second of polling): on expiry it adds 1 to *status
 * (device) and returns, so a missing rank never hangs the GPU. Ranks must be
 * on distinct GPUs and call it the same number of times.
 */
GS_API int gs_dp_barrier(const GsPeerSet* peers, int32_t* epoch, int32_t* status, gs_stream_t stream);

/*
 * gs_dp_barrier preceded by the publication of this rank's touched flags
 * (gs_render_backward's output, n bytes) into row `rank` of every owner's
 * touched_in inbox, so that gs_dp_update reads only the gradient rows that
 * may be nonzero (no reference counterpart: it saves NVLink bytes of the
 * reference's gradient pmean, trainer.py:69-71, without changing it). epoch
 * is a device int32[2] here: [0] the epoch counter, [1] a ticket word zeroed
 * once by the caller (the kernel leaves it zero). Same bounded wait and
 * status word as gs_dp_barrier; all touched_in entries must be set.
 */
GS_API int gs_dp_publish_barrier(const GsPeerSet* peers, const uint8_t* touched, int n, int32_t* epoch,
                                 int32_t* status, gs_stream_t stream);

/*
 * Peer mappings for GsPeerSet (no reference counterpart: XLA's pmean owns its
 * buffers). gs_ipc_open maps another process's device allocation, named by
 * its 64-byte cudaIpcMemHandle_t (host bytes), into the current device's
 * context and returns its base address; gs_ipc_close unmaps it. Setup-time
 * calls, not for the step itself.
 */
GS_API int gs_ipc_open(const void* handle64, void** base_out);
GS_API int gs_ipc_close(void* base);

/*
 * Densification statistics of trainer.py:143-159 (single device) /
 * trainer.py:79-113 (data parallel, after the caller's all-reduces):
 * grad2d[i] = |grad_means[i]| * max(z_i, 0.01) / ((fx+fy)/2) * W*H*3 where z is
 * the camera depth of means under w2c.  Written to grad2d (N,).
 */
GS_API int gs_grad2d_magnitude(const float* grad_means, const float* means, const float* w2c, int n,
                        float fx, float fy, int width, int height, float* grad2d,
                        gs_stream_t stream);
/*
 * grad_accum += grad2d; denom += (valid & active); max_radii =
 * radii_valid ? max(max_radii, radii) : max_radii (trainer.py:100-113/152-159).
 * Single device: radii_valid = valid (or NULL). Data parallel: valid is this
 * rank's own projection mask (the reference's denom uses it) while radii /
 * radii_valid are the max over ranks of the masked radii and of valid.
 */
GS_API int gs_accumulate_density_stats(const float* grad2d, const float* radii, const uint8_t* valid,
                                       const uint8_t* radii_valid, const uint8_t* active, int n,
                                       float* grad_accum, int32_t* denom, float* max_radii,
                                       gs_stream_t stream);

/*
 * The single-device densification statistics of trainer.py:143-159 in one
 * kernel: grad_2d_mag of grad_means and the pre-update means (as
 * gs_grad2d_magnitude; also written to grad2d (N,) when it is not NULL),
 * accumulated as gs_accumulate_density_stats does with radii_valid = valid.
 * The same results as those two calls in a row, one launch and no grad2d
 * round trip through memory.
 */
GS_API int gs_density_step_stats(const float* grad_means, const float* means, const float* w2c, int n, float fx,
                                 float fy, int width, int height, const float* radii, const uint8_t* valid,
                                 const uint8_t* active, float* grad_accum, int32_t* denom, float* max_radii,
                                 float* grad2d, gs_stream_t stream);

/*
 * The train step's returned loss and metrics (trainer.py:18-26 and the
 * metrics dict of train_step_internal) packed by one small kernel: from
 * tail = [l1, d_ssim, ...] writes out[0] = (1 - lambda) l1 + lambda d_ssim,
 * out[1] = l1, out[2] = 1 - 2 d_ssim (ssim), out[3 .. 10] = the eight health
 * counters of GsExtras as floats -- from `extras` when set, else from
 * tail[3 .. 10] (already floats, e.g. averaged over ranks) -- and out[11] =
 * the bounded device waits that gave up: extras->device_timeouts (else
 * tail[11]) plus *wait_status (the data-parallel rendezvous word; nullable).
 * out[11] != 0 means the step's results are not valid.
 */
GS_API int gs_train_step_metrics(const float* tail, const GsExtras* extras, float lambda_dssim,
                                 const int32_t* wait_status, float* out, gs_stream_t stream);

/* ---- 2DGS surfel renderer (jax_2dgs) ----------------------------------- */

/*
 * render, jax_2dgs/renderer/renderer.py:7-47: 2D Gaussian disks (means (N,3),
 * scales (N,2) log, quaternions (N,4), opacities (N,1), sh (N,K,3) of which
 * only the DC coefficient is used) projected by projection_2d.py:6-87 (no
 * active mask; valid = z > 0.01), the tile pairs of gs_get_tile_interactions,
 * and the compositor of rasterizer_2d.py:6-131: the first 512 sorted splats
 * of each tile, giving image (H,W,3) = C + T bg, depth (H,W,1),
 * depth_sq (H,W,1), normals (H,W,3, camera space) and accum_weight (H,W,1)
 * = 1 - T. radii / valid_mask (N,) and GsExtras as gs_render_forward.
 * Workspace: gs_render2d_workspace_bytes(N, W, H, capacity).
 */
GS_API int gs_render2d_forward(const float* means, const float* scales, const float* quats,
                        const float* opacities, const float* sh, int n, int sh_k, const float* w2c,
                        int width, int height, float fx, float fy, float cx, float cy,
                        const float* background, int64_t capacity, void* workspace,
                        size_t workspace_bytes, float* image, float* depth, float* depth_sq,
                        float* normals, float* accum_weight, float* radii, uint8_t* valid_mask,
                        GsExtras* extras, gs_stream_t stream);
GS_API size_t gs_render2d_workspace_bytes(int n, int width, int height, int64_t capacity);

/*
 * Backward of gs_render2d_forward on its workspace, given the forward's five
 * outputs and their gradients (grad_depth, grad_depth_sq, grad_normals,
 * grad_accum_weight may be NULL = 0). Writes every element of grad_means
 * (N,3), grad_scales (N,2), grad_quats (N,4), grad_opacities (N,1), grad_sh
 * (N,K,3) (non-DC coefficients 0).
 */
GS_API int gs_render2d_backward(const float* means, const float* scales, const float* quats,
                         const float* opacities, const float* sh, int n, int sh_k, const float* w2c,
                         int width, int height, float fx, float fy, float cx, float cy,
                         int64_t capacity, void* workspace, size_t workspace_bytes,
                         const float* image, const float* depth, const float* depth_sq,
                         const float* normals, const float* accum_weight, const float* grad_image,
                         const float* grad_depth, const float* grad_depth_sq,
                         const float* grad_normals, const float* grad_accum_weight, float* grad_means,
                         float* grad_scales, float* grad_quats, float* grad_opacities, float* grad_sh,
                         gs_stream_t stream);

/*
 * depth_distortion_loss and normal_consistency_loss,
 * jax_2dgs/training/losses.py:4-78 (means over H x W; accum_weight and the
 * normal loss's weight carry no gradient, as there). dist_loss / normal_loss
 * (device scalars, nullable) receive the losses; if grad_* are set they are
 * written with d(lambda_distortion dist + lambda_normal normal) / d map.
 */
GS_API int gs_2dgs_regularizers(const float* depth, const float* depth_sq, const float* normals,
                         const float* accum_weight, int height, int width, float lambda_distortion,
                         float lambda_normal, float* dist_loss, float* normal_loss, float* grad_depth,
                         float* grad_depth_sq, float* grad_normals, void* workspace,
                         size_t workspace_bytes, gs_stream_t stream);
GS_API size_t gs_2dgs_regularizers_workspace_bytes(void);

/*
 * optax.adam(lr) on a flat float32 buffer of `count` elements, step >= 1 the
 * optax count after this update (the 2DGS trainer's optimizer,
 * tests/test_benchmark_3dgs_vs_2dgs.py:58 / jax_2dgs/training/trainer.py:70).
 */
GS_API int gs_adam_step_flat(float* params, const float* grads, float* mu, float* nu, int64_t count,
                      float lr, int step, double b1, double b2, double eps, gs_stream_t stream);
/*
 * The same with the optax count on the device: state = [count before this
 * update, internal ticket] (int32, zeroed at start); the call leaves count + 1
 * in state[0], so a captured CUDA graph replays successive steps.
 */
GS_API int gs_adam_step_flat_device(float* params, const float* grads, float* mu, float* nu, int64_t count,
                                    float lr, double b1, double b2, double eps, int32_t* state,
                                    gs_stream_t stream);

/* ---- density control ------------------------------------------------ */

/*
 * densify_and_prune, jax_gs/training/density.py:98-211, on the flat training
 * buffers (params, mu, nu: [means | scales | quats | opacities | sh], the
 * layout of gs_adam_step). Prunes active Gaussians with sigmoid(opacity) <
 * min_opacity, max(exp(scales)) > 0.1 extent or max_radii > max_screen_size;
 * marks kept ones whose grad_accum / denom >= grad_threshold for a split
 * (max(exp(scales)) > 0.01 extent) or a clone; if densify_enabled and the new
 * Gaussians fit in the empty slots, the k-th empty slot (index order)
 * receives the k-th clone, then the k-th split (parameter row and both Adam
 * moments, density.py:171-181), and every split source and copy gets scales
 * -= log(1.6) and means += noise[row] * exp(scales) (density.py:183-190).
 * noise (N,3) holds standard normal samples: the reference's
 * jax.random.normal(rng_key, (N, 3)). active_mask is updated; grad_accum and
 * denom are reset to 0; max_radii is unchanged (as in the reference).
 * info (device int32[4]) receives [pruned, clones, splits, applied].
 * Workspace: gs_density_workspace_bytes(N) bytes, 256-byte aligned.
 */
GS_API int gs_densify_and_prune(float* params, float* mu, float* nu, int n, int sh_k, uint8_t* active_mask,
                         float* grad_accum, int32_t* denom, const float* max_radii, const float* noise,
                         int densify_enabled, float grad_threshold, float min_opacity, float extent,
                         float max_screen_size, void* workspace, size_t workspace_bytes, int32_t* info,
                         gs_stream_t stream);
GS_API size_t gs_density_workspace_bytes(int n);

/*
 * reset_opacities, density.py:76-96: the opacities of active Gaussians are
 * set to log(reset_val / (1 - reset_val)) (float32); moments unchanged.
 */
GS_API int gs_reset_opacities(float* params, int n, const uint8_t* active_mask, float reset_val,
                       gs_stream_t stream);

/*
 * D-SSIM loss for callers that cannot allocate device memory. No reference
 * counterpart: jax-gs always lets XLA allocate. Same inputs, outputs and
 * results as gs_dssim_loss, but the scratch (three H*W*C coefficient maps,
 * per-CTA partial sums, a completion ticket) lives in one fixed-size array
 * compiled into this library, so no workspace is passed and nothing is
 * allocated. For code that runs where allocation is not allowed or not
 * possible: inside an XLA FFI handler or another framework's stream capture,
 * or under a host whose device allocator belongs to someone else.
 *  - Limit: height * width * channels <= GS_NOALLOC_DSSIM_MAX_ELEMENTS
 *    (512 * 512 * 3); larger images return GS_ERR_TOO_LARGE.
 *  - The array costs about 9.3 MB on every GPU that loads the library, held
 *    until the process exits.
 *  - The first call on a device looks up the array's device address (once
 *    per device, with that device current); make that first call before any
 *    stream capture.
 *  - Every call shares the one array: calls that overlap on the GPU (other
 *    streams, other host threads) race and corrupt each other's results.
 */
#define GS_NOALLOC_DSSIM_MAX_ELEMENTS 786432
GS_API int gs_dssim_loss_noalloc(const float* pred, const float* target, int height, int width,
                                 int channels, float scale, float* loss, float* ssim_out,
                                 float* grad_pred, gs_stream_t stream);

/* ---- test aid ---------------------------------------------------------- */

/*
 * No reference counterpart. Sets, for this process, the bounded wait of the
 * direct-path sort's look-back: a waiting CTA gives up after spin_limit
 * polling rounds (spin_limit <= 0 restores the default, about a second), and
 * with ignore_published != 0 it treats every earlier key tile's status word
 * as not yet published, so each wait runs out after spin_limit rounds. That
 * lets a test drive the give-up path (GsExtras.device_timeouts, emptied tile
 * ranges) without stalling a GPU. Takes effect for launches issued after the
 * call; not thread-safe; leave it at the default outside tests.
 */
GS_API int gs_test_set_sort_wait(int spin_limit, int ignore_published);

/* ---- kernel timing (benchmarking aid) ---------------------------------- */

/*
 * No reference counterpart (the reference times whole jitted blocks on the
 * host, train.py:220-230). When enabled, every kernel launch of this library
 * is bracketed by two CUDA events on its stream, for at most max_records
 * launches; gs_timing_collect() waits for them and aggregates device time per
 * kernel name, returning the number of kernel names (or -status), and
 * gs_timing_get() reads entry `index`. Process-global, not thread-safe.
 */
GS_API int gs_timing_enable(int max_records);
GS_API int gs_timing_disable(void);
GS_API int gs_timing_reset(void);
GS_API int gs_timing_collect(void);
GS_API int gs_timing_get(int index, char* name, int name_len, double* total_ms, int* count);

#ifdef __cplusplus
}
#endif

#endif /* GSB200_H_ */
