// tl_noalloc.cu -- a gradient-norm entry point that allocates no device memory.
//
// tl_grad_norm (tl_optim.cu) keeps its partial sums in a workspace that tl_init
// obtains with cudaMalloc.  Some callers cannot allocate device memory at the
// point where they need the norm: a host framework whose allocator owns the
// whole device (so a stray cudaMalloc fails or fragments its pool), a runtime
// that fixes its memory budget at start-up and forbids allocation afterwards,
// or code that must not call into the allocator at all.  For them this file
// provides tl_grad_norm_noalloc, which computes the same norm using only the
// caller's input and output and a scratch array compiled into the library.
//
// The scratch is a file-scope __device__ array of fixed, modest size: one
// double per chunk of TL_NOALLOC_CHUNK elements, at most TL_NOALLOC_MAX_PARTIALS
// chunks (128 KiB), plus a completion counter.  Every GPU that loads the
// library holds this array until the process exits.  In host code the array's
// name is only a host-side stand-in, so the device address is looked up with
// cudaGetSymbolAddress, once per device, on the first call made with that
// device current; that first call should come before any stream capture.
// All calls share the one array: calls that overlap on the GPU (two streams,
// or two host threads on one device) race on it and must be serialised by the
// caller.
#include <atomic>
#include "tl_common.cuh"

#define TL_NOALLOC_CHUNK 65536u
#define TL_NOALLOC_MAX_PARTIALS 16384u

namespace tl {
namespace noalloc {

struct Scratch {
  double partials[TL_NOALLOC_MAX_PARTIALS];
  unsigned int ticket;
};

static __device__ __align__(256) Scratch g_scratch;

// Device address of g_scratch per device, looked up on first use.  Atomic:
// two host threads making their first call on one device may both look it up
// (they store the same value).
static std::atomic<Scratch *> g_scratch_addr[kMaxDevices] = {};

// Block b sums squares of its chunk [b*CHUNK, min(n, (b+1)*CHUNK)) in double;
// the last block to finish adds the partials in index order, writes the norm
// (and the sum of squares when asked) and re-arms the counter.
__global__ void __launch_bounds__(256)
chunk_sumsq_kernel(const float *__restrict__ G, size_t n, Scratch *__restrict__ sc,
                   float *__restrict__ norm_out, double *__restrict__ sumsq_out) {
  __shared__ double red[8];
  __shared__ bool is_last;
  const size_t lo = (size_t)blockIdx.x * TL_NOALLOC_CHUNK;
  const size_t hi = lo + TL_NOALLOC_CHUNK < n ? lo + TL_NOALLOC_CHUNK : n;
  double acc = 0.0;
  const bool vec = ((reinterpret_cast<uintptr_t>(G) & 15) == 0);
  if (vec) {
    const float4 *G4 = reinterpret_cast<const float4 *>(G + lo);
    const size_t n4 = (hi - lo) / 4;
    for (size_t i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 a = __ldg(G4 + i);
      acc += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w;
    }
    for (size_t i = lo + n4 * 4 + threadIdx.x; i < hi; i += blockDim.x) acc += (double)G[i] * G[i];
  } else {
    for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += (double)G[i] * G[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
    sc->partials[blockIdx.x] = s;
    __threadfence();
    is_last = atomicAdd(&sc->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (unsigned b = 0; b < gridDim.x; b++) s += __ldcg(&sc->partials[b]);
    if (sumsq_out) *sumsq_out = s;
    *norm_out = (float)sqrt(s);
    sc->ticket = 0u;
  }
}

static int scratch_for_current_device(Scratch **out) {
  int dev = -1;
  TL_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(TL_EINVAL, "device %d out of range", dev);
  Scratch *addr = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!addr) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) return cuda_check(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(no-alloc scratch)");
    addr = static_cast<Scratch *>(p);
    g_scratch_addr[dev].store(addr, std::memory_order_release);
  }
  *out = addr;
  return TL_OK;
}

}  // namespace noalloc
}  // namespace tl

using namespace tl;

// The norm tl_grad_norm computes (sqrt of a double sum of squares, rounded to
// float), up to summation order -- 64 Ki-element chunks here, a fixed
// 1184-block grid there, so the two may differ in the last bit -- without any
// device allocation.  norm_dev: device float; stream: a
// cudaStream_t (NULL = legacy default stream).  n is limited to
// TL_NOALLOC_MAX_PARTIALS * TL_NOALLOC_CHUNK = 2^30 elements.  Needs no tl_init.
TL_API int tl_grad_norm_noalloc(const float *G, size_t n, float *norm_dev, void *stream) {
  const size_t max_n = (size_t)TL_NOALLOC_MAX_PARTIALS * TL_NOALLOC_CHUNK;
  if (n > max_n)
    return set_error(TL_EINVAL, "tl_grad_norm_noalloc: n = %zu exceeds the fixed scratch limit of %zu elements "
                     "(use tl_grad_norm)", n, max_n);
  int rc;
  if ((rc = check_device_ptr(norm_dev, "norm_dev"))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    TL_TRY_CUDA(cudaMemsetAsync(norm_dev, 0, sizeof(float), st));
    return TL_OK;
  }
  if ((rc = check_device_ptr(G, "G"))) return rc;
  noalloc::Scratch *sc = nullptr;
  if ((rc = noalloc::scratch_for_current_device(&sc))) return rc;
  // The counter must start at zero; it is re-armed by every completed call,
  // and cleared here so that a call interrupted earlier cannot poison this one.
  TL_TRY_CUDA(cudaMemsetAsync(&sc->ticket, 0, sizeof(unsigned int), st));
  const unsigned blocks = (unsigned)((n + TL_NOALLOC_CHUNK - 1) / TL_NOALLOC_CHUNK);
  noalloc::chunk_sumsq_kernel<<<blocks, 256, 0, st>>>(G, n, sc, norm_dev, nullptr);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}
