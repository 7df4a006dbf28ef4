// tl_common.cuh -- shared state and error plumbing of libtinylm_cuda.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include "../../include/tinylm_cuda.h"

#define TL_API extern "C" __attribute__((visibility("default")))

namespace tl {

constexpr int kMaxDevices = 16;
// Norm reduction: partial sums per block, fixed count so the reduction order
// (and so the result) does not depend on the launch.
constexpr int kNormBlocks = 1184;  // 148 SMs x 8
constexpr int kNormThreads = 256;

struct DeviceCtx {
  bool ready = false;
  int device = -1;
  int num_sms = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;       // stream used for launches
  double *norm_partials = nullptr;     // [kNormBlocks] persistent workspace
  unsigned int *norm_ticket = nullptr; // last-block-done counter
  double *sumsq = nullptr;             // [1] scratch for tl_grad_norm
  float *scalars = nullptr;            // [4] scratch: norm, gscale
  int *err_flag = nullptr;             // device error word set by bounded waits
  float *gemm_ws = nullptr;            // split-K partial outputs
  size_t gemm_ws_floats = 0;
  unsigned *gemm_amax = nullptr;       // [8] operand max |x| (float bits) for the fp16-split GEMM
  bool host_buffers = false;           // tl_set_host_buffers: compute calls may take host memory
  char *host_arena = nullptr;          // staging copies of host operands (grown on demand)
  size_t host_arena_bytes = 0;
};
constexpr size_t kGemmWorkspaceFloats = 16u << 20;  // 64 MiB

DeviceCtx *ctx();                          // context of the current device, or null
int set_error(int code, const char *fmt, ...);
int cuda_check(cudaError_t e, const char *what);
int check_device_ptr(const void *p, const char *name);  // TL_EPTR for host memory
bool is_host_ptr(const void *p);                        // pageable or pinned host memory

// Host-buffer mode (tl_host.cu): the compute entry points with host operands,
// staged through the context's arena; synchronous.
enum class GemmOp;
int host_gemm(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N);
int host_grad_norm(DeviceCtx *c, const float *G, size_t n, float *norm_out);
int host_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr, float b1, float b2,
               float wd, int t, float gscale);

}  // namespace tl

#define TL_TRY_CUDA(call)                                  \
  do {                                                     \
    cudaError_t _e = (call);                               \
    if (_e != cudaSuccess) return tl::cuda_check(_e, #call); \
  } while (0)

#define TL_REQUIRE_CTX(c)                                                        \
  tl::DeviceCtx *c = tl::ctx();                                                  \
  if (!c) return tl::set_error(TL_ENOINIT, "tl_init() not called for this device")
