// tl_runtime.cu -- device contexts, streams, memory and errors of libtinylm_cuda.
#include <cstdarg>
#include <cstring>
#include "tl_common.cuh"

namespace tl {

void p2p_mark_aborted(int device, int code);   // tl_p2p.cu

static DeviceCtx g_ctx[kMaxDevices];
static thread_local char g_err[512] = "";

DeviceCtx *ctx() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return g_ctx[dev].ready ? &g_ctx[dev] : nullptr;
}

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return TL_OK;
  if (e == cudaErrorMemoryAllocation)
    return set_error(TL_ENOMEM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(TL_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

int check_device_ptr(const void *p, const char *name) {
  if (!p) return set_error(TL_EINVAL, "%s is NULL", name);
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(TL_EPTR, "%s: not a CUDA pointer (%s)", name, cudaGetErrorString(e));
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return TL_OK;
  return set_error(TL_EPTR, "%s is a host pointer; the library computes on device memory only", name);
}

}  // namespace tl

using namespace tl;

TL_API const char *tl_last_error(void) { return g_err; }
TL_API const char *tl_version(void) { return "libtinylm_cuda 0.1 sm_100a"; }

TL_API int tl_init(int device) {
  if (device < 0 || device >= kMaxDevices) return set_error(TL_EINVAL, "device %d out of range", device);
  int ndev = 0;
  TL_TRY_CUDA(cudaGetDeviceCount(&ndev));
  if (device >= ndev) return set_error(TL_EINVAL, "device %d but only %d visible", device, ndev);
  TL_TRY_CUDA(cudaSetDevice(device));
  DeviceCtx &c = g_ctx[device];
  if (c.ready) return TL_OK;
  cudaDeviceProp prop;
  TL_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return set_error(TL_EINVAL, "device %d is sm_%d%d; this library is built for sm_100a only",
                     device, prop.major, prop.minor);
  c.device = device;
  c.num_sms = prop.multiProcessorCount;
  TL_TRY_CUDA(cudaStreamCreateWithFlags(&c.own_stream, cudaStreamNonBlocking));
  c.stream = c.own_stream;
  TL_TRY_CUDA(cudaMalloc(&c.norm_partials, sizeof(double) * kNormBlocks));
  TL_TRY_CUDA(cudaMalloc(&c.norm_ticket, sizeof(unsigned int)));
  TL_TRY_CUDA(cudaMemset(c.norm_ticket, 0, sizeof(unsigned int)));
  TL_TRY_CUDA(cudaMalloc(&c.sumsq, sizeof(double) * 2));
  TL_TRY_CUDA(cudaMalloc(&c.scalars, sizeof(float) * 4));
  TL_TRY_CUDA(cudaMalloc(&c.err_flag, sizeof(int)));
  TL_TRY_CUDA(cudaMemset(c.err_flag, 0, sizeof(int)));
  TL_TRY_CUDA(cudaMalloc(&c.gemm_ws, sizeof(float) * kGemmWorkspaceFloats));
  c.gemm_ws_floats = kGemmWorkspaceFloats;
  TL_TRY_CUDA(cudaMalloc(&c.gemm_amax, sizeof(unsigned) * 8));
  TL_TRY_CUDA(cudaDeviceSynchronize());
  c.ready = true;
  return TL_OK;
}

TL_API int tl_set_stream(void *stream) {
  TL_REQUIRE_CTX(c);
  c->stream = (cudaStream_t)stream;  // NULL is the CUDA legacy default stream
  return TL_OK;
}

TL_API void *tl_get_stream(void) {
  DeviceCtx *c = ctx();
  return c ? (void *)c->stream : nullptr;
}

TL_API int tl_alloc(void **ptr, size_t bytes) {
  if (!ptr) return set_error(TL_EINVAL, "ptr is NULL");
  *ptr = nullptr;
  TL_REQUIRE_CTX(c);
  (void)c;
  TL_TRY_CUDA(cudaMalloc(ptr, bytes ? bytes : 16));
  return TL_OK;
}

TL_API int tl_free(void *ptr) {
  if (!ptr) return TL_OK;
  TL_TRY_CUDA(cudaFree(ptr));
  return TL_OK;
}

TL_API int tl_memcpy_h2d(void *dst, const void *src, size_t bytes) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream));
  return TL_OK;
}

TL_API int tl_memcpy_d2h(void *dst, const void *src, size_t bytes) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream));
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  return TL_OK;
}

TL_API int tl_memset(void *dst, int value, size_t bytes) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaMemsetAsync(dst, value, bytes, c->stream));
  return TL_OK;
}

TL_API int tl_sync(void) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  return TL_OK;
}

TL_API int tl_device_status(void) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  int code = 0;
  TL_TRY_CUDA(cudaMemcpy(&code, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) {
    TL_TRY_CUDA(cudaMemset(c->err_flag, 0, sizeof(int)));
    if (code >= 100)
      return set_error(TL_EINVAL, "a device-side input check failed (code %d: token id outside [0, V))", code);
    p2p_mark_aborted(c->device, code);
    return set_error(TL_ETIMEOUT, "a bounded device-side wait expired (site %d); the kernel returned early", code);
  }
  return TL_OK;
}
