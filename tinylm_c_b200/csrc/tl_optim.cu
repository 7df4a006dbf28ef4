// tl_optim.cu -- global grad norm, clip scale and fused AdamW (sm_100a).
//
// K1 sumsq/norm: tinylm.c:1171-1176 (global_gradnorm), double accumulation.
// K2 AdamW:      tinylm.c:1159-1170 (adamw), clip scale folded in.
//
// Both are HBM-bound streams.  Algorithmic bytes: the norm reads G once
// (4 B/elem); AdamW reads P,G,M,V and writes P,M,V (28 B/elem).
#include <cmath>
#include "tl_optim.cuh"
#include "tl_trace.cuh"

namespace tl {

// Two-stage deterministic sum of squares.  Stage 1: each of the gridDim.x
// blocks reduces a fixed strided subset of G into partials[block].  Stage 2:
// the last block to finish (ticket) reduces the partials in index order and
// writes sumsq (double), and optionally norm = (float)sqrt(sumsq) and the clip
// scale.  The ticket is reset for the next launch.
__global__ void __launch_bounds__(kNormThreads)
sumsq_kernel(const float *__restrict__ G, size_t n, double *__restrict__ partials,
             unsigned int *__restrict__ ticket, double *__restrict__ sumsq_out,
             float *__restrict__ norm_out, float *__restrict__ gscale_out, float max_norm) {
  __shared__ double smem[32];
  __shared__ bool is_last;
  // Split into a scalar head (to reach 16-byte alignment), a float4 body and a
  // scalar tail.
  const uintptr_t addr = reinterpret_cast<uintptr_t>(G);
  size_t head = ((16 - (addr & 15)) & 15) / 4;
  if (head > n) head = n;
  const size_t n4 = (n - head) / 4;
  const size_t tail_start = head + n4 * 4;
  const float4 *G4 = reinterpret_cast<const float4 *>(G + head);

  double acc = 0.0;
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = tid;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 a = ld_stream(G4 + i), b = ld_stream(G4 + i + stride);
    float4 c = ld_stream(G4 + i + 2 * stride), d = ld_stream(G4 + i + 3 * stride);
    acc += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w;
    acc += (double)b.x * b.x + (double)b.y * b.y + (double)b.z * b.z + (double)b.w * b.w;
    acc += (double)c.x * c.x + (double)c.y * c.y + (double)c.z * c.z + (double)c.w * c.w;
    acc += (double)d.x * d.x + (double)d.y * d.y + (double)d.z * d.z + (double)d.w * d.w;
  }
  for (; i < n4; i += stride) {
    float4 a = ld_stream(G4 + i);
    acc += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w;
  }
  if (blockIdx.x == 0) {
    if (threadIdx.x < head) acc += (double)G[threadIdx.x] * G[threadIdx.x];
    if (tail_start + threadIdx.x < n) {
      const float g = G[tail_start + threadIdx.x];
      acc += (double)g * g;
    }
  }
  double bsum = block_sum(acc, smem);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = bsum;
    __threadfence();
    const unsigned int t = atomicAdd(ticket, 1u);
    is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  double s = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) s += __ldcg(partials + b);
  __syncthreads();
  s = block_sum(s, smem);
  if (threadIdx.x == 0) {
    if (sumsq_out) *sumsq_out = s;
    const float norm = (float)sqrt(s);
    if (norm_out) *norm_out = norm;
    if (gscale_out) *gscale_out = norm > max_norm ? max_norm / norm : 1.0f;
    *ticket = 0u;
  }
}

__global__ void clip_scale_kernel(const double *__restrict__ sumsq, float max_norm,
                                  float *__restrict__ norm_out, float *__restrict__ gscale_out) {
  const float norm = (float)sqrt(*sumsq);
  if (norm_out) *norm_out = norm;
  if (gscale_out) *gscale_out = norm > max_norm ? max_norm / norm : 1.0f;
}

// Vector body: one float4 of each of P,G,M,V per thread per step, two steps
// unrolled so eight 16-byte loads are in flight per thread.
__global__ void __launch_bounds__(256)
adamw_vec_kernel(float4 *__restrict__ P, const float4 *__restrict__ G, float4 *__restrict__ M,
                 float4 *__restrict__ V, size_t n4, AdamArgs a0) {
  const AdamArgs a = adam_live(a0);
  const float gs = a.gscale_ptr ? __ldg(a.gscale_ptr) : a.gscale;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    float4 p0 = __ldcs(P + i), m0 = __ldcs(M + i), v0 = __ldcs(V + i);
    float4 g0 = ld_stream(G + i);
    float4 p1 = __ldcs(P + i + stride), m1 = __ldcs(M + i + stride), v1 = __ldcs(V + i + stride);
    float4 g1 = ld_stream(G + i + stride);
    adam_elem(p0.x, g0.x, m0.x, v0.x, a, gs); adam_elem(p0.y, g0.y, m0.y, v0.y, a, gs);
    adam_elem(p0.z, g0.z, m0.z, v0.z, a, gs); adam_elem(p0.w, g0.w, m0.w, v0.w, a, gs);
    adam_elem(p1.x, g1.x, m1.x, v1.x, a, gs); adam_elem(p1.y, g1.y, m1.y, v1.y, a, gs);
    adam_elem(p1.z, g1.z, m1.z, v1.z, a, gs); adam_elem(p1.w, g1.w, m1.w, v1.w, a, gs);
    __stcs(P + i, p0); __stcs(M + i, m0); __stcs(V + i, v0);
    __stcs(P + i + stride, p1); __stcs(M + i + stride, m1); __stcs(V + i + stride, v1);
  }
  if (i < n4) {
    float4 p0 = __ldcs(P + i), m0 = __ldcs(M + i), v0 = __ldcs(V + i);
    float4 g0 = ld_stream(G + i);
    adam_elem(p0.x, g0.x, m0.x, v0.x, a, gs); adam_elem(p0.y, g0.y, m0.y, v0.y, a, gs);
    adam_elem(p0.z, g0.z, m0.z, v0.z, a, gs); adam_elem(p0.w, g0.w, m0.w, v0.w, a, gs);
    __stcs(P + i, p0); __stcs(M + i, m0); __stcs(V + i, v0);
  }
}

// Scalar path: unaligned buffers and the tail of the vector body.
__global__ void adamw_scalar_kernel(float *__restrict__ P, const float *__restrict__ G,
                                    float *__restrict__ M, float *__restrict__ V, size_t n,
                                    AdamArgs a0) {
  const AdamArgs a = adam_live(a0);
  const float gs = a.gscale_ptr ? __ldg(a.gscale_ptr) : a.gscale;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float p = P[i], m = M[i], v = V[i];
    adam_elem(p, G[i], m, v, a, gs);
    P[i] = p; M[i] = m; V[i] = v;
  }
}

int launch_sumsq(DeviceCtx *c, const float *G, size_t n, double *sumsq_out, float *norm_out,
                 float *gscale_out, float max_norm) {
  TraceScope ts(c, "sumsq");
  sumsq_kernel<<<kNormBlocks, kNormThreads, 0, c->stream>>>(G, n, c->norm_partials, c->norm_ticket,
                                                            sumsq_out, norm_out, gscale_out, max_norm);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

int launch_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr,
                 float b1, float b2, float wd, int t, float gscale, const float *gscale_dev,
                 const float *hyper = nullptr) {
  if (n == 0) return TL_OK;
  AdamArgs a = make_adam_args(lr, b1, b2, wd, t, gscale, gscale_dev);
  a.hyper = hyper;
  const bool aligned = ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(G) |
                         reinterpret_cast<uintptr_t>(M) | reinterpret_cast<uintptr_t>(V)) & 15) == 0;
  size_t done = 0;
  if (aligned && n >= 4) {
    const size_t n4 = n / 4;
    // Enough threads for two float4 per thread, capped at 32 resident waves.
    size_t blocks = (n4 + 511) / 512;
    const size_t cap = (size_t)c->num_sms * 8 * 32;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    TraceScope ts(c, "adamw_vec");
    adamw_vec_kernel<<<(unsigned)blocks, 256, 0, c->stream>>>(
        reinterpret_cast<float4 *>(P), reinterpret_cast<const float4 *>(G),
        reinterpret_cast<float4 *>(M), reinterpret_cast<float4 *>(V), n4, a);
    TL_TRY_CUDA(cudaGetLastError());
    done = n4 * 4;
  }
  if (done < n) {
    const size_t rem = n - done;
    size_t blocks = (rem + 255) / 256;
    const size_t cap = (size_t)c->num_sms * 8;
    if (blocks > cap) blocks = cap;
    TraceScope ts(c, "adamw_scalar");
    adamw_scalar_kernel<<<(unsigned)blocks, 256, 0, c->stream>>>(P + done, G + done, M + done,
                                                                  V + done, rem, a);
    TL_TRY_CUDA(cudaGetLastError());
  }
  return TL_OK;
}

static int check_adam_ptrs(float *P, const float *G, float *M, float *V) {
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) ||
      (rc = check_device_ptr(M, "M")) || (rc = check_device_ptr(V, "V")))
    return rc;
  return TL_OK;
}

}  // namespace tl

using namespace tl;

TL_API int tl_grad_sumsq(const float *G, size_t n, double *sumsq_dev) {
  TL_REQUIRE_CTX(c);
  int rc;
  if (n && (rc = check_device_ptr(G, "G"))) return rc;
  if ((rc = check_device_ptr(sumsq_dev, "sumsq_dev"))) return rc;
  return launch_sumsq(c, G, n, sumsq_dev, nullptr, nullptr, 1.0f);
}

TL_API int tl_clip_scale(const double *sumsq_dev, float max_norm, float *norm_dev, float *gscale_dev) {
  TL_REQUIRE_CTX(c);
  int rc;
  if ((rc = check_device_ptr(sumsq_dev, "sumsq_dev"))) return rc;
  if (!(max_norm > 0.0f)) return set_error(TL_EINVAL, "max_norm must be > 0");
  TraceScope ts(c, "clip_scale");
  clip_scale_kernel<<<1, 1, 0, c->stream>>>(sumsq_dev, max_norm, norm_dev, gscale_dev);
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

TL_API int tl_grad_norm(const float *G, size_t n, float *norm_out) {
  TL_REQUIRE_CTX(c);
  int rc;
  if (!norm_out) return set_error(TL_EINVAL, "norm_out is NULL");
  if (c->host_buffers && n && is_host_ptr(G)) return host_grad_norm(c, G, n, norm_out);
  if (n && (rc = check_device_ptr(G, "G"))) return rc;
  cudaPointerAttributes at;
  bool host_out = cudaPointerGetAttributes(&at, norm_out) != cudaSuccess ||
                  (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged);
  cudaGetLastError();
  float *dst = host_out ? c->scalars : norm_out;
  if ((rc = launch_sumsq(c, G, n, c->sumsq, dst, nullptr, 1.0f))) return rc;
  if (host_out) {
    TL_TRY_CUDA(cudaMemcpyAsync(norm_out, c->scalars, sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  }
  return TL_OK;
}

TL_API int tl_adamw_step(float *P, const float *G, float *M, float *V, size_t n, float lr, float b1,
                         float b2, float wd, int t, float gscale) {
  TL_REQUIRE_CTX(c);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (n == 0) return TL_OK;
  int rc;
  if (c->host_buffers && (is_host_ptr(P) || is_host_ptr(G) || is_host_ptr(M) || is_host_ptr(V)))
    return host_adamw(c, P, G, M, V, n, lr, b1, b2, wd, t, gscale);
  if ((rc = check_adam_ptrs(P, G, M, V))) return rc;
  return launch_adamw(c, P, G, M, V, n, lr, b1, b2, wd, t, gscale, nullptr);
}

TL_API int tl_adamw_step_dev(float *P, const float *G, float *M, float *V, size_t n, float lr,
                             float b1, float b2, float wd, int t, const float *gscale_dev) {
  TL_REQUIRE_CTX(c);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (n == 0) return TL_OK;
  int rc;
  if ((rc = check_adam_ptrs(P, G, M, V))) return rc;
  if (gscale_dev && (rc = check_device_ptr(gscale_dev, "gscale_dev"))) return rc;
  return launch_adamw(c, P, G, M, V, n, lr, b1, b2, wd, t, 1.0f, gscale_dev);
}

TL_API int tl_clip_adamw_step(float *P, const float *G, float *M, float *V, size_t n, float lr,
                              float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  TL_REQUIRE_CTX(c);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (!(max_norm > 0.0f)) return set_error(TL_EINVAL, "max_norm must be > 0");
  if (n == 0) return TL_OK;
  int rc;
  if ((rc = check_adam_ptrs(P, G, M, V))) return rc;
  if (norm_dev && (rc = check_device_ptr(norm_dev, "norm_dev"))) return rc;
  float *gscale = c->scalars + 1;
  if ((rc = launch_sumsq(c, G, n, c->sumsq, norm_dev, gscale, max_norm))) return rc;
  return launch_adamw(c, P, G, M, V, n, lr, b1, b2, wd, t, 1.0f, gscale);
}
