// tl_optim.cuh -- AdamW element update and block reductions shared by the
// single-GPU optimizer kernels and the peer-memory ZeRO-1 step.
#pragma once
#include <cmath>
#include "tl_common.cuh"

namespace tl {

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum in a fixed order (result valid in thread 0).
__device__ __forceinline__ double block_sum(double v, double *smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = (threadIdx.x < nw) ? smem[threadIdx.x] : 0.0;
  if (warp == 0) v = warp_sum(v);
  return v;
}

struct AdamArgs {
  float lr, b1, b2, omb1, omb2, wd, bc1, bc2, gscale;
  const float *gscale_ptr;
  // When set, lr, bc1, bc2 are read from device memory (hyper[0..2]) instead
  // of the values above: a captured CUDA graph replays with the step's own
  // learning rate and bias corrections, written there before each launch.
  const float *hyper;
};

// The arguments in effect inside a kernel (device scalars applied).
__device__ __forceinline__ AdamArgs adam_live(const AdamArgs &a) {
  AdamArgs e = a;
  if (a.hyper) {
    e.lr = __ldg(a.hyper);
    e.bc1 = __ldg(a.hyper + 1);
    e.bc2 = __ldg(a.hyper + 2);
  }
  return e;
}

__device__ __forceinline__ void adam_elem(float &p, float g, float &m, float &v,
                                          const AdamArgs &a, float gs) {
  g = g * gs;
  m = a.b1 * m + a.omb1 * g;
  v = a.b2 * v + a.omb2 * g * g;
  const float mh = m / a.bc1, vh = v / a.bc2;
  p -= a.lr * (mh / (sqrtf(vh) + 1e-8f) + a.wd * p);
}

inline AdamArgs make_adam_args(float lr, float b1, float b2, float wd, int t, float gscale,
                               const float *gscale_dev) {
  AdamArgs a;
  a.lr = lr; a.b1 = b1; a.b2 = b2; a.wd = wd;
  a.omb1 = 1.0f - b1; a.omb2 = 1.0f - b2;
  // Bias corrections in fp32 with powf, as tinylm.c:1161.
  a.bc1 = 1.0f - powf(b1, (float)t);
  a.bc2 = 1.0f - powf(b2, (float)t);
  a.gscale = gscale;
  a.gscale_ptr = gscale_dev;
  a.hyper = nullptr;
  return a;
}

}  // namespace tl
