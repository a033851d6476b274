// gs_dssim_loss_noalloc: the D-SSIM loss with its scratch in a fixed array
// compiled into the library, for callers that cannot allocate device memory
// (see the declaration in include/gsb200.h for the contract).
#include <mutex>

#include "gs_kernels.cuh"

namespace gs {

constexpr size_t kNoAllocMaxElements = GS_NOALLOC_DSSIM_MAX_ELEMENTS;
// three coefficient maps + up to 65536 per-CTA partial sums + the ticket block
constexpr size_t kNoAllocBytes = 3 * kNoAllocMaxElements * sizeof(float) + 65536 * sizeof(float) + 256;

// The scratch itself. In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_dssim_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_scratch_mutex;
static void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per
// device (with that device current) and cached.
static void* scratch_on_current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = GS_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dssim_scratch) != cudaSuccess || p == nullptr) {
      *status = GS_ERR_CUDA;
      return nullptr;
    }
    g_scratch_addr[dev] = p;
  }
  *status = GS_OK;
  return g_scratch_addr[dev];
}

}  // namespace gs

using namespace gs;

extern "C" int gs_dssim_loss_noalloc(const float* pred, const float* target, int height, int width,
                                     int channels, float scale, float* loss, float* ssim_out,
                                     float* grad_pred, gs_stream_t stream) {
  if (height <= 0 || width <= 0 || channels <= 0 || !pred || !target) return GS_ERR_INVALID_ARGUMENT;
  if ((size_t)height * (size_t)width * (size_t)channels > kNoAllocMaxElements) return GS_ERR_TOO_LARGE;
  const size_t need = dssim_workspace_bytes(height, width, channels);
  if (need > kNoAllocBytes) return GS_ERR_TOO_LARGE;
  int status = GS_OK;
  void* ws = scratch_on_current_device(&status);
  if (!ws) return status;
  // the array keeps the previous call's contents: its completion ticket
  // must start at zero (the block gs_dssim_loss clears in its workspace)
  if (clear_dssim_ticket(ws, height, width, channels, stream) != cudaSuccess) {
    cudaGetLastError();
    return GS_ERR_CUDA;
  }
  launch_dssim(pred, target, height, width, channels, scale, loss, ssim_out, grad_pred, ws, stream);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}
