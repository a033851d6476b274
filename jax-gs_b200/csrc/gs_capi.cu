// extern "C" entry points of libgsb200.so (declared in include/gsb200.h).
//
// Host side only: argument validation, the workspace layout and the launch
// sequence of each entry point. No allocation, no synchronisation.
#include <algorithm>
#include <cstring>

#include "gs_kernels.cuh"

namespace gs {

static inline size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

// surfels: the 2DGS layout (64-byte records, no per-batch checkpoints: its
// backward replays each tile from the start).
static Layout make_layout(int n, int width, int height, int64_t capacity, bool surfels = false) {
  Layout L;
  L.n = n;
  L.width = width;
  L.height = height;
  L.tiles_x = (width + kTile - 1) / kTile;
  L.tiles_y = (height + kTile - 1) / kTile;
  L.num_tiles = L.tiles_x * L.tiles_y;
  L.n_blocks = (n + 255) / 256;
  L.capacity = capacity;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align_up(bytes);
    return o;
  };
  const size_t cap = (size_t)(capacity > 0 ? capacity : 0);
  const size_t pix = (size_t)width * (size_t)height;
  L.scalars = take(sizeof(Scalars));
  L.loss_partials = take(sizeof(float) * kLossGrid);
  L.splats = take((surfels ? splat2_bytes() : sizeof(Splat)) * (size_t)n);
  L.grads = take((surfels ? splat2_grad_bytes() : sizeof(SplatGrad)) * (size_t)n);
  L.bins = take(sizeof(int2) * (size_t)n);
  L.block_counts = take(sizeof(int) * 2 * (size_t)L.n_blocks);  // [pairs | visible] per block
  L.block_offsets = take(sizeof(int) * (size_t)L.n_blocks);      // pair offsets (direct path)
  L.vis_offsets = take(sizeof(int) * (size_t)L.n_blocks);        // compaction offsets (pre-sort path)
  L.hist = take(sizeof(int) * kRadix * 2 * kMaxSortPasses);      // digit totals [tile | depth]
  L.presort = n >= kPresortMinN;
  const size_t key_tiles = std::max<size_t>(1, (cap + kSortTileKeys - 1) / kSortTileKeys);
  L.sort_tiles = (int)key_tiles;
  L.depth_tiles = std::max(1, (n + kSortTileKeys - 1) / kSortTileKeys);
  L.status0 = L.status1 = L.tcounts = L.dcounts = L.dkeys0 = L.dids0 = L.dkeys1 = L.dids1 = 0;
  L.sorted_counts = L.emit_offsets = 0;
  if (!L.presort) {
    // look-back status words of the single-pass radix sort, two passes' worth
    const size_t os_tiles = std::max<size_t>(1, (cap + kOsTileKeys - 1) / kOsTileKeys);
    L.status0 = take(sizeof(unsigned long long) * kRadix * os_tiles);
    L.status1 = take(sizeof(unsigned long long) * kRadix * os_tiles);
  } else {
    // per-tile digit counts [digit][tile] and the depth sort's buffers
    L.tcounts = take(sizeof(int) * kRadix * key_tiles);
    L.dcounts = take(sizeof(int) * kRadix * (size_t)L.depth_tiles);
    L.dkeys0 = take(sizeof(int) * (size_t)n);
    L.dids0 = take(sizeof(int) * (size_t)n);
    L.dkeys1 = take(sizeof(int) * (size_t)n);
    L.dids1 = take(sizeof(int) * (size_t)n);
    L.sorted_counts = take(sizeof(int) * (size_t)std::max(1, L.n_blocks));
    L.emit_offsets = take(sizeof(int) * (size_t)std::max(1, L.n_blocks));
  }
  L.ranges = take(sizeof(int) * (size_t)(L.num_tiles + 1));
  L.tile_items = take(sizeof(int) * (size_t)(L.num_tiles + 1));
  L.tile_order = take(sizeof(int) * (size_t)L.num_tiles);  // the forward's CTA order
  // (tile, batch) work items: at most 4096 / batch per tile and at most one
  // per `batch` pairs plus one partial batch per tile.
  const int batch = compositor_batch(L.num_tiles);
  L.max_items = surfels ? 0
                        : std::min<int64_t>((int64_t)(kMaxTileInteractions / batch) * L.num_tiles,
                                            ((int64_t)cap + batch - 1) / batch + L.num_tiles);
  L.item_info = take(sizeof(int) * (size_t)L.max_items);
  L.item_cost = take(sizeof(int) * (size_t)L.max_items);   // splat steps the forward ran per item
  L.item_order = take(sizeof(int) * (size_t)L.max_items);  // the backward's item order (longest first)
  L.ckpt = take(sizeof(float4) * kTilePixels * (size_t)L.max_items);
  L.pix_T = take(sizeof(float) * pix);
  L.img = take(sizeof(float) * 3 * pix);
  L.keys0 = take(sizeof(int) * cap);
  L.ids0 = take(sizeof(int) * cap);
  L.keys1 = take(sizeof(int) * cap);
  L.ids1 = take(sizeof(int) * cap);
  L.total = off;
  return L;
}

template <typename T>
static inline T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

// Largest supported sizes: keys are (tile << 13 | depth) in 31 bits and the
// reference's N * 256 candidate count must fit int32.
constexpr int kMaxN = (1 << 23) - 1;
constexpr int kMaxTiles = (1 << 18) - 1;

static int check_image(int width, int height) {
  if (width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  long long tx = (width + kTile - 1) / kTile, ty = (height + kTile - 1) / kTile;
  if (tx * ty > kMaxTiles || tx > 0xFFFF || ty > 0x7FFF) return GS_ERR_INVALID_ARGUMENT;
  return GS_OK;
}

static int check_common(int n, int width, int height, int64_t capacity, void* ws, size_t ws_bytes) {
  if (n < 0 || n > kMaxN) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_image(width, height)) return s;
  if (capacity < 0 || capacity > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, capacity);
  if (ws == nullptr || ws_bytes < L.total) return GS_ERR_WORKSPACE_TOO_SMALL;
  if (((uintptr_t)ws) & 255) return GS_ERR_INVALID_ARGUMENT;
  return GS_OK;
}

static int check_sh(int sh_degree, int sh_k) {
  if (sh_degree < 0 || sh_degree > 3) return GS_ERR_INVALID_ARGUMENT;
  if (sh_k < (sh_degree + 1) * (sh_degree + 1) || sh_k > 16) return GS_ERR_INVALID_ARGUMENT;
  return GS_OK;
}

static int last_error() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

static int tile_bits(int num_tiles) {
  int tb = 0;
  while ((1 << tb) < num_tiles) ++tb;
  return tb;
}

// Radix bits of the pair sort: (tile << 13 | depth) on the direct path, the
// tile id alone after the depth pre-sort.
static int pair_sort_bits(const Layout& L) { return tile_bits(L.num_tiles) + (L.presort ? 0 : kDepthBits); }

// Shift from a sorted pair key to its tile id.
static int key_shift(const Layout& L) { return L.presort ? 0 : kDepthBits; }

// Which buffer pair (0/1) holds the sorted pairs after bin_and_sort.
static int sorted_buffer(const Layout& L) { return ((pair_sort_bits(L) + kRadixBits - 1) / kRadixBits) & 1; }

static CamParams cam_params(const Layout& L, float fx, float fy, float cx, float cy) {
  CamParams cp;
  cp.fx = fx; cp.fy = fy; cp.cx = cx; cp.cy = cy;
  cp.width = L.width; cp.height = L.height; cp.tiles_x = L.tiles_x; cp.tiles_y = L.tiles_y;
  return cp;
}

// Pair emission, sort (direct or depth pre-sort path, by n), ranges and work
// items, on bins and block counts already in the workspace. Returns the index
// (0/1) of the buffer pair that holds the sorted result.
static int bin_and_sort(const Layout& L, void* ws, GsExtras* extras, cudaStream_t st) {
  Scalars* sc = at<Scalars>(ws, L.scalars);
  int* thist = at<int>(ws, L.hist);
  int* dhist = thist + kRadix * kMaxSortPasses;
  launch_scan_block_counts(at<int>(ws, L.block_counts), L.n_blocks, at<int>(ws, L.block_offsets),
                           at<int>(ws, L.vis_offsets), sc, L.capacity, L.num_tiles, extras, st);
  // the sort's give-up count (both paths; only the direct path waits) and the
  // single-pass sweep counters
  cudaMemsetAsync(&sc->sort_timeouts, 0, sizeof(sc->sort_timeouts) + sizeof(sc->sweep_tile), st);
  int cur;
  if (!L.presort) {
    cudaMemsetAsync(thist, 0, sizeof(int) * kRadix * kMaxSortPasses, st);

    launch_emit_keys(at<int2>(ws, L.bins), at<int>(ws, L.block_offsets), L.n, L.tiles_x, sc, L.capacity,
                     at<int>(ws, L.keys0), at<int>(ws, L.ids0), thist, at<unsigned long long>(ws, L.status0), st);
    cur = launch_radix_sort_onesweep(at<int>(ws, L.keys0), at<int>(ws, L.ids0), at<int>(ws, L.keys1),
                                     at<int>(ws, L.ids1), &sc->n_emit, sc, thist,
                                     at<unsigned long long>(ws, L.status0), at<unsigned long long>(ws, L.status1),
                                     pair_sort_bits(L), st);
  } else {
    launch_compact_visible(at<int2>(ws, L.bins), L.n, at<int>(ws, L.vis_offsets), at<int>(ws, L.dkeys0),
                           at<int>(ws, L.dids0), at<int>(ws, L.sorted_counts), st);
    const int dcur = launch_radix_sort(at<int>(ws, L.dkeys0), at<int>(ws, L.dids0), at<int>(ws, L.dkeys1),
                                       at<int>(ws, L.dids1), &sc->n_vis, L.depth_tiles, at<int>(ws, L.dcounts),
                                       dhist, kDepthBits, at<int2>(ws, L.bins), at<int>(ws, L.sorted_counts),
                                       "sort_depth", st);
    launch_emit_sorted(at<int2>(ws, L.bins), at<int>(ws, dcur ? L.dids1 : L.dids0), L.n, sc,
                       at<int>(ws, L.sorted_counts), at<int>(ws, L.emit_offsets), L.tiles_x, L.capacity,
                       at<int>(ws, L.keys0), at<int>(ws, L.ids0), st);
    cur = launch_radix_sort(at<int>(ws, L.keys0), at<int>(ws, L.ids0), at<int>(ws, L.keys1), at<int>(ws, L.ids1),
                            &sc->n_emit, L.sort_tiles, at<int>(ws, L.tcounts), thist, pair_sort_bits(L), nullptr,
                            nullptr, "sort_tile", st);
  }
  launch_tile_ranges_from_keys(at<int>(ws, cur ? L.keys1 : L.keys0), key_shift(L), sc, L.num_tiles, L.capacity,
                               at<int>(ws, L.ranges), st);
  launch_tile_items(at<int>(ws, L.ranges), L.num_tiles, at<int>(ws, L.tile_items), sc, extras, &sc->sort_timeouts,
                    at<int>(ws, L.tile_order), st);
  return cur;
}

// Forward compositor on the workspace's splats / ranges / work items.
// residuals = false: no checkpoints, work items, final T or image copy (no
// backward will read this workspace).
static void composite(const Layout& L, void* ws, const int* ids, int n, const float* bg,
                      float* image, float* img_copy, cudaStream_t st, bool residuals = true) {
  launch_raster_fwd(at<Splat>(ws, L.splats), ids, at<int>(ws, L.ranges), at<int>(ws, L.tile_items), n, bg,
                    L.width, L.height, L.tiles_x, L.num_tiles, image, residuals ? img_copy : nullptr,
                    residuals ? at<float>(ws, L.pix_T) : nullptr,
                    residuals ? at<float4>(ws, L.ckpt) : nullptr,
                    residuals ? at<int>(ws, L.item_info) : nullptr,
                    residuals ? at<int>(ws, L.item_cost) : nullptr, at<int>(ws, L.tile_order), st);
}

// Backward compositor into the workspace's SplatGrad accumulators.
static void composite_backward(const Layout& L, void* ws, const int* ids, int n,
                               const float* grad_image, float* grad_bg, cudaStream_t st) {
  SplatGrad* grads = at<SplatGrad>(ws, L.grads);
  cudaMemsetAsync(grads, 0, sizeof(SplatGrad) * (size_t)n, st);
  if (grad_bg) cudaMemsetAsync(grad_bg, 0, 3 * sizeof(float), st);
  launch_raster_bwd(at<Splat>(ws, L.splats), ids, at<int>(ws, L.ranges), n, L.width, L.height, L.tiles_x,
                    L.num_tiles, grad_image, at<float>(ws, L.img), at<float4>(ws, L.ckpt),
                    at<int>(ws, L.item_info), at<int>(ws, L.item_cost), at<int>(ws, L.item_order),
                    at<Scalars>(ws, L.scalars), grads, at<float>(ws, L.pix_T),
                    grad_bg, st);
}

}  // namespace gs

using namespace gs;

extern "C" {

const char* gs_status_string(int status) {
  switch (status) {
    case GS_OK: return "ok";
    case GS_ERR_INVALID_ARGUMENT: return "invalid argument (shape, size or pointer)";
    case GS_ERR_CAPACITY: return "interaction capacity exceeded";
    case GS_ERR_DEVICE_TIMEOUT: return "bounded device wait expired";
    case GS_ERR_CUDA: return "CUDA launch error";
    case GS_ERR_WORKSPACE_TOO_SMALL: return "workspace too small or missing";
    case GS_ERR_TOO_LARGE: return "problem larger than the fixed scratch of this entry point";
    default: return "unknown status";
  }
}

int gs_version(void) { return (1 << 16) | 0; }

int64_t gs_default_capacity(int n) { return (int64_t)(n > 0 ? n : 0) * kOffset * kOffset; }

size_t gs_workspace_bytes(int n, int width, int height, int64_t capacity) {
  if (n < 0 || width <= 0 || height <= 0 || capacity < 0) return 0;
  return make_layout(n, width, height, capacity).total;
}

int gs_project_gaussians(const float* means, const float* scales, const float* quats, int n,
                         const uint8_t* mask, const float* w2c, int width, int height, float fx,
                         float fy, float cx, float cy, float* means2d, float* cov2d, float* radii,
                         uint8_t* valid, float* depths, gs_stream_t stream) {
  if (n < 0 || n > kMaxN) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_image(width, height)) return s;
  if (n > 0 && (!means || !scales || !quats || !w2c || !means2d || !cov2d || !radii || !valid || !depths))
    return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(0, width, height, 0);
  launch_project(means, scales, quats, n, mask, w2c, cam_params(L, fx, fy, cx, cy), means2d, cov2d,
                 radii, valid, depths, stream);
  return last_error();
}

int gs_covariance_3d(const float* scales, const float* quats, int n, float* cov3d, gs_stream_t stream) {
  if (n < 0 || n > kMaxN) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!scales || !quats || !cov3d)) return GS_ERR_INVALID_ARGUMENT;
  launch_covariance_3d(scales, quats, n, cov3d, stream);
  return last_error();
}

int gs_eval_sh(int sh_degree, const float* sh, int n, int sh_k, const float* view_dirs, float* out,
               gs_stream_t stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_sh(sh_degree, sh_k)) return s;
  if (n > 0 && (!sh || !view_dirs || !out)) return GS_ERR_INVALID_ARGUMENT;
  launch_eval_sh(sh_degree, sh, n, sh_k, view_dirs, out, stream);
  return last_error();
}

int gs_get_tile_interactions(const float* means2d, const float* radii, const uint8_t* valid,
                             const float* depths, int n, int height, int width, int64_t capacity,
                             void* workspace, size_t workspace_bytes, int32_t* sorted_tile_ids,
                             int32_t* sorted_gaussian_ids, int32_t* n_interactions,
                             int32_t* tile_ranges, gs_stream_t stream) {
  if (int s = check_common(n, width, height, capacity, workspace, workspace_bytes)) return s;
  if (n > 0 && (!means2d || !radii || !valid || !depths)) return GS_ERR_INVALID_ARGUMENT;
  if (capacity > 0 && (!sorted_tile_ids || !sorted_gaussian_ids)) return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, capacity);
  cudaMemsetAsync(at<char>(workspace, L.scalars), 0, sizeof(Scalars), stream);
  launch_bin_prep(means2d, radii, valid, depths, n, width, height, at<int2>(workspace, L.bins),
                  at<int>(workspace, L.block_counts), stream);
  int cur = bin_and_sort(L, workspace, nullptr, stream);
  const Scalars* sc = at<Scalars>(workspace, L.scalars);
  launch_export_interactions(at<int>(workspace, cur ? L.keys1 : L.keys0), key_shift(L),
                             at<int>(workspace, cur ? L.ids1 : L.ids0), sc, capacity, L.num_tiles,
                             sorted_tile_ids, sorted_gaussian_ids, n_interactions, stream);
  if (tile_ranges)
    cudaMemcpyAsync(tile_ranges, at<int>(workspace, L.ranges), sizeof(int) * (L.num_tiles + 1),
                    cudaMemcpyDeviceToDevice, stream);
  return last_error();
}

int gs_render_tiles(const float* means2d, const float* cov2d, const float* opacities,
                    const float* colors, int n, const int32_t* sorted_tile_ids,
                    const int32_t* sorted_gaussian_ids, int64_t n_sorted, int height, int width,
                    const float* background, void* workspace, size_t workspace_bytes, float* image,
                    gs_stream_t stream) {
  if (n_sorted < 0 || n_sorted > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_common(n, width, height, n_sorted, workspace, workspace_bytes)) return s;
  if (!image || (n > 0 && (!means2d || !cov2d || !opacities || !colors))) return GS_ERR_INVALID_ARGUMENT;
  if (n_sorted > 0 && (!sorted_tile_ids || !sorted_gaussian_ids || n == 0)) return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, n_sorted);
  cudaMemsetAsync(at<char>(workspace, L.scalars), 0, sizeof(Scalars), stream);
  launch_pack_splats(means2d, cov2d, opacities, colors, n, at<Splat>(workspace, L.splats), stream);
  int* ranges = at<int>(workspace, L.ranges);
  cudaMemsetAsync(ranges, 0, sizeof(int) * (L.num_tiles + 1), stream);
  launch_tile_ranges_from_ids(sorted_tile_ids, n_sorted, L.num_tiles, ranges, stream);
  launch_tile_items(ranges, L.num_tiles, at<int>(workspace, L.tile_items), at<Scalars>(workspace, L.scalars),
                    nullptr, nullptr, at<int>(workspace, L.tile_order), stream);
  composite(L, workspace, sorted_gaussian_ids, n, background, image, nullptr, stream);
  return last_error();
}

int gs_render_tiles_backward(const float* means2d, const float* cov2d, const float* opacities,
                             const float* colors, int n, const int32_t* sorted_tile_ids,
                             const int32_t* sorted_gaussian_ids, int64_t n_sorted, int height,
                             int width, const float* background, const float* grad_image,
                             void* workspace, size_t workspace_bytes, float* grad_means2d,
                             float* grad_cov2d, float* grad_opacities, float* grad_colors,
                             gs_stream_t stream) {
  if (n_sorted < 0 || n_sorted > 0x7FFFFFFFll || !grad_image) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_common(n, width, height, n_sorted, workspace, workspace_bytes)) return s;
  if (n > 0 && (!means2d || !cov2d || !opacities || !colors)) return GS_ERR_INVALID_ARGUMENT;
  if (n_sorted > 0 && (!sorted_tile_ids || !sorted_gaussian_ids || n == 0)) return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, n_sorted);
  cudaMemsetAsync(at<char>(workspace, L.scalars), 0, sizeof(Scalars), stream);
  launch_pack_splats(means2d, cov2d, opacities, colors, n, at<Splat>(workspace, L.splats), stream);
  int* ranges = at<int>(workspace, L.ranges);
  cudaMemsetAsync(ranges, 0, sizeof(int) * (L.num_tiles + 1), stream);
  launch_tile_ranges_from_ids(sorted_tile_ids, n_sorted, L.num_tiles, ranges, stream);
  launch_tile_items(ranges, L.num_tiles, at<int>(workspace, L.tile_items), at<Scalars>(workspace, L.scalars),
                    nullptr, nullptr, at<int>(workspace, L.tile_order), stream);
  // forward replay: residuals (checkpoints, image) into the workspace
  composite(L, workspace, sorted_gaussian_ids, n, background, at<float>(workspace, L.img), nullptr, stream);
  composite_backward(L, workspace, sorted_gaussian_ids, n, grad_image, nullptr, stream);
  launch_splat_grads_to_inputs(cov2d, opacities, at<SplatGrad>(workspace, L.grads), n, grad_means2d,
                               grad_cov2d, grad_opacities, grad_colors, stream);
  return last_error();
}

static int render_forward(const float* means, const float* scales, const float* quats,
                          const float* opacities, const float* sh, int n, int sh_k, const uint8_t* mask,
                          const float* w2c, int width, int height, float fx, float fy, float cx, float cy,
                          const float* background, int sh_degree, int64_t capacity, void* workspace,
                          size_t workspace_bytes, float* image, float* radii, uint8_t* valid_mask,
                          GsExtras* extras, cudaStream_t stream, bool residuals) {
  if (int s = check_common(n, width, height, capacity, workspace, workspace_bytes)) return s;
  if (int s = check_sh(sh_degree, sh_k)) return s;
  if (!w2c || !image || !radii || !valid_mask || !extras) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!means || !scales || !quats || !opacities || !sh)) return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, capacity);
  cudaMemsetAsync(extras, 0, sizeof(GsExtras), stream);
  cudaMemsetAsync(at<char>(workspace, L.scalars), 0, sizeof(Scalars), stream);
  launch_preprocess_fwd(means, scales, quats, opacities, sh, n, sh_k, sh_degree, mask, w2c,
                        cam_params(L, fx, fy, cx, cy), at<Splat>(workspace, L.splats),
                        at<int2>(workspace, L.bins), at<int>(workspace, L.block_counts), radii,
                        valid_mask, extras, stream);
  int cur = bin_and_sort(L, workspace, extras, stream);
  composite(L, workspace, at<int>(workspace, cur ? L.ids1 : L.ids0), n, background, image,
            at<float>(workspace, L.img), stream, residuals);
  return last_error();
}

int gs_render_forward(const float* means, const float* scales, const float* quats,
                      const float* opacities, const float* sh, int n, int sh_k, const uint8_t* mask,
                      const float* w2c, int width, int height, float fx, float fy, float cx, float cy,
                      const float* background, int sh_degree, int64_t capacity, void* workspace,
                      size_t workspace_bytes, float* image, float* radii, uint8_t* valid_mask,
                      GsExtras* extras, gs_stream_t stream) {
  return render_forward(means, scales, quats, opacities, sh, n, sh_k, mask, w2c, width, height, fx, fy,
                        cx, cy, background, sh_degree, capacity, workspace, workspace_bytes, image, radii,
                        valid_mask, extras, (cudaStream_t)stream, true);
}

int gs_render_image(const float* means, const float* scales, const float* quats,
                    const float* opacities, const float* sh, int n, int sh_k, const uint8_t* mask,
                    const float* w2c, int width, int height, float fx, float fy, float cx, float cy,
                    const float* background, int sh_degree, int64_t capacity, void* workspace,
                    size_t workspace_bytes, float* image, float* radii, uint8_t* valid_mask,
                    GsExtras* extras, gs_stream_t stream) {
  return render_forward(means, scales, quats, opacities, sh, n, sh_k, mask, w2c, width, height, fx, fy,
                        cx, cy, background, sh_degree, capacity, workspace, workspace_bytes, image, radii,
                        valid_mask, extras, (cudaStream_t)stream, false);
}

int gs_render_backward(const float* means, const float* scales, const float* quats,
                       const float* opacities, const float* sh, int n, int sh_k,
                       const uint8_t* mask, const float* w2c, int width, int height, float fx,
                       float fy, float cx, float cy, const float* background, int sh_degree,
                       int64_t capacity, void* workspace, size_t workspace_bytes,
                       const float* grad_image, float* grad_means, float* grad_scales,
                       float* grad_quats, float* grad_opacities, float* grad_sh,
                       float* grad_background, uint8_t* touched, gs_stream_t stream) {
  (void)mask;
  if (int s = check_common(n, width, height, capacity, workspace, workspace_bytes)) return s;
  if (int s = check_sh(sh_degree, sh_k)) return s;
  if (!w2c || !grad_image) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!means || !scales || !quats || !opacities || !sh || !grad_means || !grad_scales ||
                !grad_quats || !grad_opacities || !grad_sh))
    return GS_ERR_INVALID_ARGUMENT;
  Layout L = make_layout(n, width, height, capacity);
  (void)background;
  const int cur = sorted_buffer(L);
  composite_backward(L, workspace, at<int>(workspace, cur ? L.ids1 : L.ids0), n, grad_image,
                     grad_background, stream);
  launch_preprocess_bwd(means, scales, quats, opacities, sh, n, sh_k, sh_degree, w2c,
                        cam_params(L, fx, fy, cx, cy), at<SplatGrad>(workspace, L.grads), grad_means,
                        grad_scales, grad_quats, grad_opacities, grad_sh, touched, stream);
  return last_error();
}

int gs_l1_loss(const float* pred, const float* target, int64_t count, float scale, float* loss,
               float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream) {
  if (count < 0 || !loss || (count > 0 && (!pred || !target))) return GS_ERR_INVALID_ARGUMENT;
  const size_t need = align_up(sizeof(Scalars)) + align_up(sizeof(float) * kLossGrid);
  if (!workspace || workspace_bytes < need || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  Scalars* sc = at<Scalars>(workspace, 0);
  float* partials = at<float>(workspace, align_up(sizeof(Scalars)));
  cudaMemsetAsync(sc, 0, sizeof(Scalars), stream);
  launch_l1_loss(pred, target, count, scale, loss, grad_pred, partials, sc, stream);
  return last_error();
}

int gs_mse_loss(const float* pred, const float* target, int64_t count, float scale, float* loss,
                float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream) {
  if (count < 0 || !loss || (count > 0 && (!pred || !target))) return GS_ERR_INVALID_ARGUMENT;
  const size_t need = align_up(sizeof(Scalars)) + align_up(sizeof(float) * kLossGrid);
  if (!workspace || workspace_bytes < need || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  Scalars* sc = at<Scalars>(workspace, 0);
  float* partials = at<float>(workspace, align_up(sizeof(Scalars)));
  cudaMemsetAsync(sc, 0, sizeof(Scalars), stream);
  launch_mse_loss(pred, target, count, scale, loss, grad_pred, partials, sc, stream);
  return last_error();
}

size_t gs_dssim_workspace_bytes(int height, int width, int channels) {
  if (height <= 0 || width <= 0 || channels <= 0) return 0;
  return dssim_workspace_bytes(height, width, channels);
}

int gs_dssim_loss(const float* pred, const float* target, int height, int width, int channels,
                  float scale, float* loss, float* ssim_out, float* grad_pred, void* workspace,
                  size_t workspace_bytes, gs_stream_t stream) {
  if (height <= 0 || width <= 0 || channels <= 0 || !pred || !target) return GS_ERR_INVALID_ARGUMENT;
  size_t need = dssim_workspace_bytes(height, width, channels);
  if (!workspace || workspace_bytes < need || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  // zero the ticket / factor block at the end of the workspace
  if (clear_dssim_ticket(workspace, height, width, channels, stream) != cudaSuccess) {
    cudaGetLastError();
    return GS_ERR_CUDA;
  }
  launch_dssim(pred, target, height, width, channels, scale, loss, ssim_out, grad_pred, workspace,
               stream);
  return last_error();
}

size_t gs_l1_dssim_workspace_bytes(int height, int width, int channels) {
  if (height <= 0 || width <= 0 || channels <= 0) return 0;
  return l1_dssim_workspace_bytes(height, width, channels);
}

int gs_l1_dssim_loss(const float* pred, const float* target, int height, int width, int channels,
                     float lambda_dssim, float* l1, float* dssim, float* ssim_out, float* loss,
                     float* grad_pred, void* workspace, size_t workspace_bytes, gs_stream_t stream) {
  if (height <= 0 || width <= 0 || channels <= 0 || channels > 3 || !pred || !target)
    return GS_ERR_INVALID_ARGUMENT;
  if (!(lambda_dssim >= 0.f && lambda_dssim <= 1.f)) return GS_ERR_INVALID_ARGUMENT;
  if ((long long)height * width * channels > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  const size_t need = l1_dssim_workspace_bytes(height, width, channels);
  if (!workspace || workspace_bytes < need || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  launch_l1_dssim(pred, target, height, width, channels, lambda_dssim, l1, dssim, ssim_out, loss, grad_pred,
                  workspace, (cudaStream_t)stream);
  return last_error();
}

// ---- 2DGS ---------------------------------------------------------------
size_t gs_render2d_workspace_bytes(int n, int width, int height, int64_t capacity) {
  if (n < 0 || width <= 0 || height <= 0 || capacity < 0) return 0;
  return make_layout(n, width, height, capacity, true).total;
}

static int check2d(int n, int sh_k, int width, int height, int64_t capacity, void* ws, size_t ws_bytes) {
  if (n < 0 || n > kMaxN || sh_k < 1 || sh_k > 16) return GS_ERR_INVALID_ARGUMENT;
  if (int s = check_image(width, height)) return s;
  if (capacity < 0 || capacity > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (!ws || ws_bytes < make_layout(n, width, height, capacity, true).total || (((uintptr_t)ws) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  return GS_OK;
}

int gs_render2d_forward(const float* means, const float* scales, const float* quats, const float* opacities,
                        const float* sh, int n, int sh_k, const float* w2c, int width, int height, float fx,
                        float fy, float cx, float cy, const float* background, int64_t capacity, void* workspace,
                        size_t workspace_bytes, float* image, float* depth, float* depth_sq, float* normals,
                        float* accum_weight, float* radii, uint8_t* valid_mask, GsExtras* extras,
                        gs_stream_t stream) {
  if (int s = check2d(n, sh_k, width, height, capacity, workspace, workspace_bytes)) return s;
  if (!w2c || !image || !depth || !depth_sq || !normals || !accum_weight || !radii || !valid_mask || !extras)
    return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!means || !scales || !quats || !opacities || !sh)) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  Layout L = make_layout(n, width, height, capacity, true);
  cudaMemsetAsync(extras, 0, sizeof(GsExtras), st);
  cudaMemsetAsync(at<char>(workspace, L.scalars), 0, sizeof(Scalars), st);
  launch_pre2d_fwd(means, scales, quats, opacities, sh, n, sh_k, w2c, cam_params(L, fx, fy, cx, cy),
                   at<void>(workspace, L.splats), at<int2>(workspace, L.bins), at<int>(workspace, L.block_counts),
                   radii, valid_mask, extras, st);
  const int cur = bin_and_sort(L, workspace, extras, st);
  launch_raster2d_fwd(at<void>(workspace, L.splats), at<int>(workspace, cur ? L.ids1 : L.ids0),
                      at<int>(workspace, L.ranges), n, background, width, height, L.tiles_x, L.num_tiles, image,
                      depth, depth_sq, normals, accum_weight, at<float>(workspace, L.pix_T), st);
  return last_error();
}

int gs_render2d_backward(const float* means, const float* scales, const float* quats, const float* opacities,
                         const float* sh, int n, int sh_k, const float* w2c, int width, int height, float fx,
                         float fy, float cx, float cy, int64_t capacity, void* workspace, size_t workspace_bytes,
                         const float* image, const float* depth, const float* depth_sq, const float* normals,
                         const float* accum_weight, const float* grad_image, const float* grad_depth,
                         const float* grad_depth_sq, const float* grad_normals, const float* grad_accum_weight,
                         float* grad_means, float* grad_scales, float* grad_quats, float* grad_opacities,
                         float* grad_sh, gs_stream_t stream) {
  if (int s = check2d(n, sh_k, width, height, capacity, workspace, workspace_bytes)) return s;
  if (!w2c || !image || !depth || !depth_sq || !normals || !accum_weight || !grad_image)
    return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!means || !scales || !quats || !opacities || !sh || !grad_means || !grad_scales ||
                !grad_quats || !grad_opacities || !grad_sh))
    return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  Layout L = make_layout(n, width, height, capacity, true);
  const int cur = sorted_buffer(L);
  launch_raster2d_bwd(at<void>(workspace, L.splats), at<int>(workspace, cur ? L.ids1 : L.ids0),
                      at<int>(workspace, L.ranges), n, width, height, L.tiles_x, L.num_tiles, image, depth, depth_sq,
                      normals, accum_weight, at<float>(workspace, L.pix_T), grad_image, grad_depth, grad_depth_sq,
                      grad_normals, grad_accum_weight, at<void>(workspace, L.grads), st);
  launch_pre2d_bwd(means, scales, quats, opacities, sh, n, sh_k, w2c, cam_params(L, fx, fy, cx, cy),
                   at<void>(workspace, L.grads), grad_means, grad_scales, grad_quats, grad_opacities, grad_sh, st);
  return last_error();
}

size_t gs_2dgs_regularizers_workspace_bytes(void) { return reg2d_workspace_bytes(); }

int gs_2dgs_regularizers(const float* depth, const float* depth_sq, const float* normals,
                         const float* accum_weight, int height, int width, float lambda_distortion,
                         float lambda_normal, float* dist_loss, float* normal_loss, float* grad_depth,
                         float* grad_depth_sq, float* grad_normals, void* workspace, size_t workspace_bytes,
                         gs_stream_t stream) {
  if (height <= 0 || width <= 0 || (long long)height * width > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (!depth || !depth_sq || !normals || !accum_weight) return GS_ERR_INVALID_ARGUMENT;
  if ((grad_depth || grad_depth_sq || grad_normals) && !(grad_depth && grad_depth_sq && grad_normals))
    return GS_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < reg2d_workspace_bytes() || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  launch_reg2d(depth, depth_sq, normals, accum_weight, height, width, lambda_distortion, lambda_normal, dist_loss,
               normal_loss, grad_depth, grad_depth_sq, grad_normals, workspace, (cudaStream_t)stream);
  return last_error();
}

int gs_adam_step_flat(float* params, const float* grads, float* mu, float* nu, int64_t count, float lr, int step,
                      double b1, double b2, double eps, gs_stream_t stream) {
  if (count < 0 || count > 0x7FFFFFFFll || step < 1) return GS_ERR_INVALID_ARGUMENT;
  if (count > 0 && (!params || !grads || !mu || !nu)) return GS_ERR_INVALID_ARGUMENT;
  const float b1f = (float)b1, b2f = (float)b2;
  const float bc1 = 1.f - (float)pow((double)b1f, (double)step);
  const float bc2 = 1.f - (float)pow((double)b2f, (double)step);
  launch_adam_flat(params, grads, mu, nu, (int)count, lr, b1f, b2f, (float)(1.0 - b1), (float)(1.0 - b2), 1.f / bc1,
                   1.f / bc2, (float)eps, nullptr, (cudaStream_t)stream);
  return last_error();
}

int gs_adam_step_flat_device(float* params, const float* grads, float* mu, float* nu, int64_t count, float lr,
                             double b1, double b2, double eps, int32_t* state, gs_stream_t stream) {
  if (count < 0 || count > 0x7FFFFFFFll || !state) return GS_ERR_INVALID_ARGUMENT;
  if (count > 0 && (!params || !grads || !mu || !nu)) return GS_ERR_INVALID_ARGUMENT;
  launch_adam_flat(params, grads, mu, nu, (int)count, lr, (float)b1, (float)b2, (float)(1.0 - b1), (float)(1.0 - b2),
                   1.f, 1.f, (float)eps, state, (cudaStream_t)stream);
  return last_error();
}

size_t gs_density_workspace_bytes(int n) { return n < 0 ? 0 : density_workspace_bytes(n); }

int gs_densify_and_prune(float* params, float* mu, float* nu, int n, int sh_k, uint8_t* active_mask,
                         float* grad_accum, int32_t* denom, const float* max_radii, const float* noise,
                         int densify_enabled, float grad_threshold, float min_opacity, float extent,
                         float max_screen_size, void* workspace, size_t workspace_bytes, int32_t* info,
                         gs_stream_t stream) {
  if (n < 0 || sh_k < 1 || sh_k > 16 || !info) return GS_ERR_INVALID_ARGUMENT;
  if ((long long)n * (11 + 3 * sh_k) > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!params || !mu || !nu || !active_mask || !grad_accum || !denom || !max_radii || !noise))
    return GS_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < density_workspace_bytes(n) || (((uintptr_t)workspace) & 255))
    return GS_ERR_WORKSPACE_TOO_SMALL;
  launch_densify_and_prune(params, mu, nu, n, sh_k, active_mask, grad_accum, denom, max_radii, noise,
                           densify_enabled, grad_threshold, min_opacity, extent, max_screen_size, workspace,
                           info, (cudaStream_t)stream);
  return last_error();
}

int gs_reset_opacities(float* params, int n, const uint8_t* active_mask, float reset_val, gs_stream_t stream) {
  if (n < 0 || (n > 0 && (!params || !active_mask))) return GS_ERR_INVALID_ARGUMENT;
  if (!(reset_val > 0.f && reset_val < 1.f)) return GS_ERR_INVALID_ARGUMENT;
  launch_reset_opacities(params, n, active_mask, reset_val, (cudaStream_t)stream);
  return last_error();
}

int gs_adam_step(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                 const uint8_t* active_mask, const float* lrs, int step, double b1, double b2,
                 double eps, gs_stream_t stream) {
  if (n < 0 || sh_k < 1 || sh_k > 16 || step < 1 || !lrs) return GS_ERR_INVALID_ARGUMENT;
  if ((long long)n * (11 + 3 * sh_k) > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!params || !grads || !mu || !nu)) return GS_ERR_INVALID_ARGUMENT;
  // optax bias_correction: 1 - decay ** count with a float32 decay.
  const float b1f = (float)b1, b2f = (float)b2;
  const float bc1 = 1.f - (float)pow((double)b1f, (double)step);
  const float bc2 = 1.f - (float)pow((double)b2f, (double)step);
  launch_adam(params, grads, mu, nu, n, sh_k, active_mask, lrs, bc1, bc2, b1f, b2f, (float)(1.0 - b1),
              (float)(1.0 - b2), (float)eps, nullptr, nullptr, nullptr, nullptr, stream);
  return last_error();
}

int gs_adam_step_scheduled(float* params, const float* grads, float* mu, float* nu, int n, int sh_k,
                           const uint8_t* active_mask, const GsAdamSchedule* schedule, int32_t* state,
                           gs_stream_t stream) {
  if (n < 0 || sh_k < 1 || sh_k > 16 || !schedule || !state) return GS_ERR_INVALID_ARGUMENT;
  if ((long long)n * (11 + 3 * sh_k) > 0x7FFFFFFFll) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!params || !grads || !mu || !nu)) return GS_ERR_INVALID_ARGUMENT;
  for (int g = 0; g < 5; ++g)
    if (!(schedule->transition_steps[g] > 0.f)) return GS_ERR_INVALID_ARGUMENT;
  const float zeros[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  launch_adam(params, grads, mu, nu, n, sh_k, active_mask, zeros, 1.f, 1.f, (float)schedule->b1,
              (float)schedule->b2, (float)(1.0 - schedule->b1), (float)(1.0 - schedule->b2),
              (float)schedule->eps, state, schedule->lr_init, schedule->decay_rate,
              schedule->transition_steps, stream);
  return last_error();
}

int gs_grad2d_magnitude(const float* grad_means, const float* means, const float* w2c, int n,
                        float fx, float fy, int width, int height, float* grad2d,
                        gs_stream_t stream) {
  if (n < 0 || width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!grad_means || !means || !w2c || !grad2d)) return GS_ERR_INVALID_ARGUMENT;
  launch_grad2d(grad_means, means, w2c, n, fx, fy, width, height, grad2d, stream);
  return last_error();
}

int gs_train_step_metrics(const float* tail, const GsExtras* extras, float lambda_dssim,
                          const int32_t* wait_status, float* out, gs_stream_t stream) {
  if (!tail || !out) return GS_ERR_INVALID_ARGUMENT;
  launch_step_metrics(tail, extras, lambda_dssim, wait_status, out, (cudaStream_t)stream);
  return last_error();
}

int gs_check_extras(const GsExtras* extras, gs_stream_t stream) {
  if (!extras) return GS_ERR_INVALID_ARGUMENT;
  GsExtras h;
  if (cudaMemcpyAsync(&h, extras, sizeof(h), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess ||
      cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) {
    cudaGetLastError();
    return GS_ERR_CUDA;
  }
  if (h.device_timeouts != 0) return GS_ERR_DEVICE_TIMEOUT;
  if (h.capacity_overflow != 0) return GS_ERR_CAPACITY;
  return GS_OK;
}

int gs_test_set_sort_wait(int spin_limit, int ignore_published) {
  set_sort_wait(spin_limit, ignore_published);
  return GS_OK;
}

int gs_density_step_stats(const float* grad_means, const float* means, const float* w2c, int n, float fx,
                          float fy, int width, int height, const float* radii, const uint8_t* valid,
                          const uint8_t* active, float* grad_accum, int32_t* denom, float* max_radii,
                          float* grad2d, gs_stream_t stream) {
  if (n < 0 || width <= 0 || height <= 0) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!grad_means || !means || !w2c || !radii || !valid || !grad_accum || !denom || !max_radii))
    return GS_ERR_INVALID_ARGUMENT;
  launch_step_stats(grad_means, means, w2c, n, fx, fy, width, height, radii, valid, active, grad_accum, denom,
                    max_radii, grad2d, (cudaStream_t)stream);
  return last_error();
}

int gs_accumulate_density_stats(const float* grad2d, const float* radii, const uint8_t* valid,
                                const uint8_t* radii_valid, const uint8_t* active, int n,
                                float* grad_accum, int32_t* denom, float* max_radii,
                                gs_stream_t stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!grad2d || !radii || !valid || !grad_accum || !denom || !max_radii))
    return GS_ERR_INVALID_ARGUMENT;
  launch_density_stats(grad2d, radii, valid, radii_valid ? radii_valid : valid, active, n, grad_accum,
                       denom, max_radii, stream);
  return last_error();
}

}  // extern "C"
