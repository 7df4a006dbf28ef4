// tl_trace.cuh -- RAII bracket that times one kernel launch when tracing is on.
#pragma once
#include "tl_common.cuh"

namespace tl {
bool trace_on();
// No kernel is timed while suspended (launches recorded into a CUDA graph).
void trace_suspend(bool on);
class TraceScope {
 public:
  TraceScope(DeviceCtx *c, const char *name);
  ~TraceScope();
  TraceScope(const TraceScope &) = delete;
  TraceScope &operator=(const TraceScope &) = delete;

 private:
  DeviceCtx *c_ = nullptr;
  const char *name_ = nullptr;
  cudaEvent_t a_ = nullptr;
  bool nvtx_ = false;
};
}  // namespace tl
