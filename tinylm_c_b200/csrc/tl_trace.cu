// tl_trace.cu -- per-kernel device timing with CUDA events on the library stream.
//
// The reference's tracing is wall-clock only (wtime, tinylm.c:139-145).  Here,
// when tracing is on, every kernel the library launches is bracketed by two
// events on the stream it is launched on; tl_trace_get folds the finished pairs
// into a per-name total and count.  Off by default; when off it costs one
// branch per launch.  With TL_NVTX=1 every launch is also an NVTX range of the
// same name.
#include <cstdlib>
#include <cstring>
#include <nvtx3/nvToolsExt.h>
#include <string>
#include <unordered_map>
#include <vector>
#include "tl_common.cuh"
#include "tl_trace.cuh"

namespace tl {

struct Pending {
  std::string name;
  cudaEvent_t a, b;
};
struct Stat {
  double ms = 0.0;
  long long count = 0;
};

static bool g_on = false;
static std::vector<Pending> g_pending;
static std::vector<cudaEvent_t> g_free;
static std::unordered_map<std::string, Stat> g_stats;
static std::vector<std::string> g_order;

static cudaEvent_t get_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

static thread_local bool g_suspended = false;   // while a CUDA graph is being captured

// NVTX ranges named after each launch, for profiler timelines (TL_NVTX=1).
static bool nvtx_on() {
  static const bool on = [] {
    const char *e = getenv("TL_NVTX");
    return e && *e && *e != '0';
  }();
  return on;
}

bool trace_on() { return g_on && !g_suspended; }
void trace_suspend(bool on) { g_suspended = on; }

TraceScope::TraceScope(DeviceCtx *c, const char *name) : c_(c), name_(name) {
  if (nvtx_on()) {
    nvtxRangePushA(name);
    nvtx_ = true;
  }
  if (!g_on || g_suspended || !c) return;
  a_ = get_event();
  cudaEventRecord(a_, c->stream);
}

TraceScope::~TraceScope() {
  if (nvtx_) nvtxRangePop();
  if (!a_) return;
  cudaEvent_t b = get_event();
  cudaEventRecord(b, c_->stream);
  g_pending.push_back({name_, a_, b});
}

static int fold() {
  for (auto &p : g_pending) {
    cudaError_t e = cudaEventSynchronize(p.b);
    if (e != cudaSuccess) return cuda_check(e, "cudaEventSynchronize(trace)");
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, p.a, p.b);
    auto it = g_stats.find(p.name);
    if (it == g_stats.end()) {
      g_order.push_back(p.name);
      it = g_stats.emplace(p.name, Stat{}).first;
    }
    it->second.ms += ms;
    it->second.count += 1;
    g_free.push_back(p.a);
    g_free.push_back(p.b);
  }
  g_pending.clear();
  return TL_OK;
}

}  // namespace tl

using namespace tl;

TL_API int tl_trace_enable(int on) {
  g_on = on != 0;
  return TL_OK;
}

TL_API int tl_trace_reset(void) {
  int rc = fold();
  g_stats.clear();
  g_order.clear();
  return rc;
}

TL_API int tl_trace_get(const char *name, double *total_ms, long long *count) {
  int rc = fold();
  if (rc) return rc;
  if (!name) return set_error(TL_EINVAL, "name is NULL");
  auto it = g_stats.find(name);
  if (total_ms) *total_ms = it == g_stats.end() ? 0.0 : it->second.ms;
  if (count) *count = it == g_stats.end() ? 0 : it->second.count;
  return TL_OK;
}

TL_API int tl_trace_names(char *buf, size_t len) {
  int rc = fold();
  if (rc) return rc;
  std::string s;
  for (auto &n : g_order) {
    if (!s.empty()) s += ",";
    s += n;
  }
  if (!buf || len == 0) return set_error(TL_EINVAL, "buffer is empty");
  strncpy(buf, s.c_str(), len - 1);
  buf[len - 1] = 0;
  return TL_OK;
}
