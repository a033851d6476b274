// Optional per-kernel timing for benchmarking: when enabled through
// gs_timing_enable(), every kernel launch of the library is bracketed by a
// pair of CUDA events recorded on the launching stream, and
// gs_timing_collect() / gs_timing_get() report the total device time and the
// launch count per kernel. Disabled (the default) it costs one branch per
// launch. Process-global and not thread-safe: a profiling aid only.
#pragma once

#include <cuda_runtime.h>

namespace gs {

int timer_begin(const char* name, cudaStream_t st);  // returns a slot or -1
void timer_end(int slot, cudaStream_t st);

struct TimerScope {
  int slot;
  cudaStream_t st;
  TimerScope(const char* name, cudaStream_t s) : slot(timer_begin(name, s)), st(s) {}
  ~TimerScope() {
    if (slot >= 0) timer_end(slot, st);
  }
};

}  // namespace gs

#define GS_TIMED_CAT2(a, b) a##b
#define GS_TIMED_CAT(a, b) GS_TIMED_CAT2(a, b)
#define GS_TIMED(name, st) ::gs::TimerScope GS_TIMED_CAT(gs_timer_scope_, __LINE__)(name, st)
