// XLA typed-FFI handlers that put libgsb200.so behind jax-gs's render()
// (jax_gs/renderer/renderer.py:15-107) as jax.ffi.ffi_call targets:
//   GsRenderFwd   -> gs_render_forward   (image, radii, valid, extras, residual workspace)
//   GsRenderBwd   -> gs_render_backward  (the five Gaussians gradients and the background's)
//   GsRenderImage -> gs_render_image     (the forward without the backward's residuals)
// The Python side (jax_shim.py) wraps the first two in a jax.custom_vjp.
//
// Static camera scalars, sh_degree and the pair capacity are FFI attributes;
// W2C, background and the active mask are buffers. The workspace is a u8
// result buffer of gs_workspace_bytes(...) + 256 bytes: XLA does not promise
// 256-byte alignment, so both handlers use the first 256-byte boundary inside
// it (the same offset, since the backward receives the forward's buffer).
//
// Build: jax-gs_b200/xla/build_ffi.py (needs jax.ffi.include_dir()).
#include <cstdint>
#include <cuda_runtime_api.h>

#include "gsb200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

// The 256-byte aligned part of an XLA-owned workspace buffer.
struct Aligned {
  void* ptr;
  size_t bytes;
};

Aligned align_workspace(void* base, size_t bytes) {
  const uintptr_t p = reinterpret_cast<uintptr_t>(base);
  const uintptr_t a = (p + 255) & ~static_cast<uintptr_t>(255);
  const size_t skip = static_cast<size_t>(a - p);
  return {reinterpret_cast<void*>(a), bytes > skip ? bytes - skip : 0};
}

ffi::Error status_error(int status) {
  if (status == GS_OK) return ffi::Error::Success();
  return ffi::Error(ffi::ErrorCode::kInternal, gs_status_string(status));
}

int sh_coeffs(const ffi::Buffer<ffi::F32>& sh) {
  const auto d = sh.dimensions();
  return d.size() >= 2 ? static_cast<int>(d[1]) : 1;
}

ffi::Error RenderForwardImpl(bool residuals, cudaStream_t stream, ffi::Buffer<ffi::F32> means,
                             ffi::Buffer<ffi::F32> scales, ffi::Buffer<ffi::F32> quats,
                             ffi::Buffer<ffi::F32> opacities, ffi::Buffer<ffi::F32> sh,
                             ffi::Buffer<ffi::PRED> mask, ffi::Buffer<ffi::F32> w2c, ffi::Buffer<ffi::F32> bg,
                             int32_t W, int32_t H, float fx, float fy, float cx, float cy, int32_t sh_degree,
                             int64_t capacity, ffi::ResultBuffer<ffi::F32> image,
                             ffi::ResultBuffer<ffi::F32> radii, ffi::ResultBuffer<ffi::PRED> valid,
                             ffi::ResultBuffer<ffi::S32> extras, ffi::ResultBuffer<ffi::U8> workspace) {
  const int n = static_cast<int>(means.dimensions()[0]);
  if (extras->element_count() * sizeof(int32_t) < sizeof(GsExtras))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "extras must hold 16 int32");
  const Aligned ws = align_workspace(workspace->untyped_data(), workspace->size_bytes());
  auto fn = residuals ? gs_render_forward : gs_render_image;
  return status_error(fn(means.typed_data(), scales.typed_data(), quats.typed_data(), opacities.typed_data(),
                         sh.typed_data(), n, sh_coeffs(sh), reinterpret_cast<const uint8_t*>(mask.typed_data()),
                         w2c.typed_data(), W, H, fx, fy, cx, cy, bg.typed_data(), sh_degree, capacity, ws.ptr,
                         ws.bytes, image->typed_data(), radii->typed_data(),
                         reinterpret_cast<uint8_t*>(valid->typed_data()),
                         reinterpret_cast<GsExtras*>(extras->typed_data()), reinterpret_cast<gs_stream_t>(stream)));
}

ffi::Error RenderFwd(cudaStream_t stream, ffi::Buffer<ffi::F32> means, ffi::Buffer<ffi::F32> scales,
                     ffi::Buffer<ffi::F32> quats, ffi::Buffer<ffi::F32> opacities, ffi::Buffer<ffi::F32> sh,
                     ffi::Buffer<ffi::PRED> mask, ffi::Buffer<ffi::F32> w2c, ffi::Buffer<ffi::F32> bg, int32_t W,
                     int32_t H, float fx, float fy, float cx, float cy, int32_t sh_degree, int64_t capacity,
                     ffi::ResultBuffer<ffi::F32> image, ffi::ResultBuffer<ffi::F32> radii,
                     ffi::ResultBuffer<ffi::PRED> valid, ffi::ResultBuffer<ffi::S32> extras,
                     ffi::ResultBuffer<ffi::U8> workspace) {
  return RenderForwardImpl(true, stream, means, scales, quats, opacities, sh, mask, w2c, bg, W, H, fx, fy, cx, cy,
                           sh_degree, capacity, image, radii, valid, extras, workspace);
}

ffi::Error RenderImage(cudaStream_t stream, ffi::Buffer<ffi::F32> means, ffi::Buffer<ffi::F32> scales,
                       ffi::Buffer<ffi::F32> quats, ffi::Buffer<ffi::F32> opacities, ffi::Buffer<ffi::F32> sh,
                       ffi::Buffer<ffi::PRED> mask, ffi::Buffer<ffi::F32> w2c, ffi::Buffer<ffi::F32> bg,
                       int32_t W, int32_t H, float fx, float fy, float cx, float cy, int32_t sh_degree,
                       int64_t capacity, ffi::ResultBuffer<ffi::F32> image, ffi::ResultBuffer<ffi::F32> radii,
                       ffi::ResultBuffer<ffi::PRED> valid, ffi::ResultBuffer<ffi::S32> extras,
                       ffi::ResultBuffer<ffi::U8> workspace) {
  return RenderForwardImpl(false, stream, means, scales, quats, opacities, sh, mask, w2c, bg, W, H, fx, fy, cx, cy,
                           sh_degree, capacity, image, radii, valid, extras, workspace);
}

ffi::Error RenderBwd(cudaStream_t stream, ffi::Buffer<ffi::F32> means, ffi::Buffer<ffi::F32> scales,
                     ffi::Buffer<ffi::F32> quats, ffi::Buffer<ffi::F32> opacities, ffi::Buffer<ffi::F32> sh,
                     ffi::Buffer<ffi::PRED> mask, ffi::Buffer<ffi::F32> w2c, ffi::Buffer<ffi::F32> bg,
                     ffi::Buffer<ffi::U8> workspace, ffi::Buffer<ffi::F32> grad_image, int32_t W, int32_t H,
                     float fx, float fy, float cx, float cy, int32_t sh_degree, int64_t capacity,
                     ffi::ResultBuffer<ffi::F32> g_means, ffi::ResultBuffer<ffi::F32> g_scales,
                     ffi::ResultBuffer<ffi::F32> g_quats, ffi::ResultBuffer<ffi::F32> g_opacities,
                     ffi::ResultBuffer<ffi::F32> g_sh, ffi::ResultBuffer<ffi::F32> g_bg,
                     ffi::ResultBuffer<ffi::U8> workspace_out) {
  const int n = static_cast<int>(means.dimensions()[0]);
  // gs_render_backward reads the forward's residuals from the workspace and
  // also writes into it (gradient accumulators, work-item order): the Python
  // side aliases the workspace operand to this last result
  // (input_output_aliases), so the writes are XLA's to expect.
  (void)workspace;
  const Aligned ws = align_workspace(workspace_out->untyped_data(), workspace_out->size_bytes());
  return status_error(gs_render_backward(
      means.typed_data(), scales.typed_data(), quats.typed_data(), opacities.typed_data(), sh.typed_data(), n,
      sh_coeffs(sh), reinterpret_cast<const uint8_t*>(mask.typed_data()), w2c.typed_data(), W, H, fx, fy, cx, cy,
      bg.typed_data(), sh_degree, capacity, ws.ptr, ws.bytes, grad_image.typed_data(), g_means->typed_data(),
      g_scales->typed_data(), g_quats->typed_data(), g_opacities->typed_data(), g_sh->typed_data(),
      g_bg->typed_data(), /*touched=*/nullptr, reinterpret_cast<gs_stream_t>(stream)));
}

}  // namespace

#define GS_FORWARD_BINDING                                                                                  \
  ffi::Ffi::Bind()                                                                                          \
      .Ctx<ffi::PlatformStream<cudaStream_t>>()                                                             \
      .Arg<ffi::Buffer<ffi::F32>>() /* means (N,3) */                                                       \
      .Arg<ffi::Buffer<ffi::F32>>() /* scales (N,3) */                                                      \
      .Arg<ffi::Buffer<ffi::F32>>() /* quaternions (N,4) */                                                 \
      .Arg<ffi::Buffer<ffi::F32>>() /* opacities (N,1) */                                                   \
      .Arg<ffi::Buffer<ffi::F32>>() /* sh (N,K,3) */                                                        \
      .Arg<ffi::Buffer<ffi::PRED>>() /* active mask (N,) */                                                 \
      .Arg<ffi::Buffer<ffi::F32>>() /* W2C (4,4) */                                                         \
      .Arg<ffi::Buffer<ffi::F32>>() /* background (3,) */                                                   \
      .Attr<int32_t>("W")                                                                                   \
      .Attr<int32_t>("H")                                                                                   \
      .Attr<float>("fx")                                                                                    \
      .Attr<float>("fy")                                                                                    \
      .Attr<float>("cx")                                                                                    \
      .Attr<float>("cy")                                                                                    \
      .Attr<int32_t>("sh_degree")                                                                           \
      .Attr<int64_t>("capacity")                                                                            \
      .Ret<ffi::Buffer<ffi::F32>>() /* image (H,W,3) */                                                     \
      .Ret<ffi::Buffer<ffi::F32>>() /* radii (N,) */                                                        \
      .Ret<ffi::Buffer<ffi::PRED>>() /* valid (N,) */                                                       \
      .Ret<ffi::Buffer<ffi::S32>>() /* GsExtras as int32[16] */                                             \
      .Ret<ffi::Buffer<ffi::U8>>() /* workspace: gs_workspace_bytes + 256 */

XLA_FFI_DEFINE_HANDLER_SYMBOL(GsRenderFwd, RenderFwd, GS_FORWARD_BINDING);
XLA_FFI_DEFINE_HANDLER_SYMBOL(GsRenderImage, RenderImage, GS_FORWARD_BINDING);

XLA_FFI_DEFINE_HANDLER_SYMBOL(GsRenderBwd, RenderBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()  // means
                                  .Arg<ffi::Buffer<ffi::F32>>()  // scales
                                  .Arg<ffi::Buffer<ffi::F32>>()  // quaternions
                                  .Arg<ffi::Buffer<ffi::F32>>()  // opacities
                                  .Arg<ffi::Buffer<ffi::F32>>()  // sh
                                  .Arg<ffi::Buffer<ffi::PRED>>()  // active mask
                                  .Arg<ffi::Buffer<ffi::F32>>()  // W2C
                                  .Arg<ffi::Buffer<ffi::F32>>()  // background
                                  .Arg<ffi::Buffer<ffi::U8>>()   // the forward's workspace
                                  .Arg<ffi::Buffer<ffi::F32>>()  // dL/dimage (H,W,3)
                                  .Attr<int32_t>("W")
                                  .Attr<int32_t>("H")
                                  .Attr<float>("fx")
                                  .Attr<float>("fy")
                                  .Attr<float>("cx")
                                  .Attr<float>("cy")
                                  .Attr<int32_t>("sh_degree")
                                  .Attr<int64_t>("capacity")
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d means
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d scales
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d quaternions
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d opacities
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d sh
                                  .Ret<ffi::Buffer<ffi::F32>>()  // d background (3,)
                                  .Ret<ffi::Buffer<ffi::U8>>());  // the workspace, aliased to operand 8
