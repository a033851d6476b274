// Per-kernel CUDA-event timing hook (see gs_timing.cuh) and its C ABI.
#include <cstring>
#include <string>
#include <vector>

#include "gs_kernels.cuh"
#include "gs_timing.cuh"

namespace gs {

static bool g_enabled = false;
static int g_cap = 0;
static int g_used = 0;
static std::vector<cudaEvent_t> g_events;
static std::vector<const char*> g_names;
static std::vector<std::string> g_agg_names;
static std::vector<double> g_agg_ms;
static std::vector<int> g_agg_count;

int timer_begin(const char* name, cudaStream_t st) {
  if (!g_enabled || g_used >= g_cap) return -1;
  int s = g_used++;
  g_names[s] = name;
  cudaEventRecord(g_events[2 * s], st);
  return s;
}

void timer_end(int slot, cudaStream_t st) { cudaEventRecord(g_events[2 * slot + 1], st); }

static void destroy_events() {
  for (cudaEvent_t e : g_events) cudaEventDestroy(e);
  g_events.clear();
  g_names.clear();
  g_cap = 0;
  g_used = 0;
}

}  // namespace gs

using namespace gs;

extern "C" {

int gs_timing_enable(int max_records) {
  if (max_records <= 0 || max_records > (1 << 20)) return GS_ERR_INVALID_ARGUMENT;
  destroy_events();
  g_events.resize(2 * (size_t)max_records);
  for (auto& e : g_events) {
    if (cudaEventCreate(&e) != cudaSuccess) {
      destroy_events();
      return GS_ERR_CUDA;
    }
  }
  g_names.assign(max_records, nullptr);
  g_cap = max_records;
  g_used = 0;
  g_enabled = true;
  return GS_OK;
}

int gs_timing_disable(void) {
  g_enabled = false;
  destroy_events();
  return GS_OK;
}

int gs_timing_reset(void) {
  g_used = 0;
  return GS_OK;
}

int gs_timing_collect(void) {
  g_agg_names.clear();
  g_agg_ms.clear();
  g_agg_count.clear();
  for (int s = 0; s < g_used; ++s) {
    if (cudaEventSynchronize(g_events[2 * s + 1]) != cudaSuccess) return -GS_ERR_CUDA;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, g_events[2 * s], g_events[2 * s + 1]) != cudaSuccess) return -GS_ERR_CUDA;
    size_t k = 0;
    while (k < g_agg_names.size() && g_agg_names[k] != g_names[s]) ++k;
    if (k == g_agg_names.size()) {
      g_agg_names.emplace_back(g_names[s]);
      g_agg_ms.push_back(0.0);
      g_agg_count.push_back(0);
    }
    g_agg_ms[k] += ms;
    g_agg_count[k] += 1;
  }
  return (int)g_agg_names.size();
}

int gs_timing_get(int index, char* name, int name_len, double* total_ms, int* count) {
  if (index < 0 || index >= (int)g_agg_names.size() || !name || name_len <= 0 || !total_ms || !count)
    return GS_ERR_INVALID_ARGUMENT;
  std::strncpy(name, g_agg_names[index].c_str(), name_len - 1);
  name[name_len - 1] = 0;
  *total_ms = g_agg_ms[index];
  *count = g_agg_count[index];
  return GS_OK;
}

}  // extern "C"
