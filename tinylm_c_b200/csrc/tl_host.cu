// tl_host.cu -- host-buffer mode: the five reference-facing compute calls on
// an unchanged host program's own memory.
//
// tinylm.c keeps every buffer in host memory from fz() (calloc, tinylm.c:137)
// and reads results right after each primitive returns (e.g. forward() runs
// rmsnorm on the output of the previous mm).  A build that swaps only the
// primitives' bodies for calls into this library therefore
// needs calls that take host pointers and return with the result in host
// memory.  With tl_set_host_buffers(1) the GEMMs, the grad norm and AdamW
// copy each host operand into a per-device staging arena, run the same device
// code as for device pointers, copy the outputs back and wait.  Device
// pointers in the same call are used in place.  The arena grows to the
// largest call seen and is kept until exit.
#include "tl_gemm.cuh"

namespace tl {

int launch_sumsq(DeviceCtx *c, const float *G, size_t n, double *sumsq_out, float *norm_out,
                 float *gscale_out, float max_norm);
int launch_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr,
                 float b1, float b2, float wd, int t, float gscale, const float *gscale_dev,
                 const float *hyper);

bool is_host_ptr(const void *p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged;
}

namespace {

constexpr size_t kAlign = 256;

size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Make the arena at least `bytes` long (grown by at least half again so a
// sequence of slightly larger calls does not reallocate every time).
int arena_reserve(DeviceCtx *c, size_t bytes) {
  if (bytes <= c->host_arena_bytes) return TL_OK;
  size_t want = c->host_arena_bytes + c->host_arena_bytes / 2;
  if (want < bytes) want = bytes;
  want = round_up(want);
  if (c->host_arena) {
    TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
    TL_TRY_CUDA(cudaFree(c->host_arena));
    c->host_arena = nullptr;
    c->host_arena_bytes = 0;
  }
  TL_TRY_CUDA(cudaMalloc(&c->host_arena, want));
  c->host_arena_bytes = want;
  return TL_OK;
}

// One operand of a staged call: where the caller's data is, where the kernel
// reads it, its size and whether it moves in, out or both ways.
struct Slot {
  const float *user;
  float *dev;
  size_t floats;
  bool in, out, host;
};

// Assign arena space to the host slots, copy the inputs in.
int stage_in(DeviceCtx *c, Slot *s, int ns) {
  size_t need = 0;
  for (int i = 0; i < ns; i++) {
    s[i].host = is_host_ptr(s[i].user);
    if (s[i].host) need += round_up(sizeof(float) * s[i].floats);
  }
  int rc;
  if ((rc = arena_reserve(c, need))) return rc;
  size_t off = 0;
  for (int i = 0; i < ns; i++) {
    if (!s[i].host) {
      s[i].dev = const_cast<float *>(s[i].user);
      continue;
    }
    s[i].dev = reinterpret_cast<float *>(c->host_arena + off);
    off += round_up(sizeof(float) * s[i].floats);
    if (s[i].in && s[i].floats)
      TL_TRY_CUDA(cudaMemcpyAsync(s[i].dev, s[i].user, sizeof(float) * s[i].floats, cudaMemcpyHostToDevice,
                                  c->stream));
  }
  return TL_OK;
}

// Copy the host outputs back and wait for them.
int stage_out(DeviceCtx *c, const Slot *s, int ns) {
  for (int i = 0; i < ns; i++)
    if (s[i].host && s[i].out && s[i].floats)
      TL_TRY_CUDA(cudaMemcpyAsync(const_cast<float *>(s[i].user), s[i].dev, sizeof(float) * s[i].floats,
                                  cudaMemcpyDeviceToHost, c->stream));
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  return TL_OK;
}

}  // namespace

int host_gemm(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N) {
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  // Operand extents: NN A = X[M,K], B = W[K,N]; NT A = dY[M,N], B = W[K,N];
  // TN A = X[M,K], B = dY[M,N].  The accumulating forms read C as well.
  const size_t a_fl = op == GemmOp::NT ? (size_t)M * N : (size_t)M * K;
  const size_t b_fl = op == GemmOp::TN ? (size_t)M * N : (size_t)K * N;
  Slot s[3] = {{C, nullptr, (size_t)I * J, op != GemmOp::NN, true, false},
               {A, nullptr, R > 0 ? a_fl : 0, true, false, false},
               {B, nullptr, R > 0 ? b_fl : 0, true, false, false}};
  int rc;
  if ((rc = stage_in(c, s, 3))) return rc;
  if ((rc = gemm_run(c, op, s[0].dev, s[1].dev, s[2].dev, M, K, N))) return rc;
  return stage_out(c, s, 3);
}

int host_grad_norm(DeviceCtx *c, const float *G, size_t n, float *norm_out) {
  Slot s[1] = {{G, nullptr, n, true, false, false}};
  int rc;
  if ((rc = stage_in(c, s, 1))) return rc;
  if ((rc = launch_sumsq(c, s[0].dev, n, c->sumsq, c->scalars, nullptr, 1.0f))) return rc;
  const bool host_out = is_host_ptr(norm_out);
  TL_TRY_CUDA(cudaMemcpyAsync(norm_out, c->scalars, sizeof(float),
                              host_out ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, c->stream));
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  return TL_OK;
}

int host_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr, float b1, float b2,
               float wd, int t, float gscale) {
  Slot s[4] = {{P, nullptr, n, true, true, false},
               {G, nullptr, n, true, false, false},
               {M, nullptr, n, true, true, false},
               {V, nullptr, n, true, true, false}};
  int rc;
  if ((rc = stage_in(c, s, 4))) return rc;
  if ((rc = launch_adamw(c, s[0].dev, s[1].dev, s[2].dev, s[3].dev, n, lr, b1, b2, wd, t, gscale, nullptr,
                         nullptr)))
    return rc;
  return stage_out(c, s, 4);
}

}  // namespace tl

using namespace tl;

TL_API int tl_set_host_buffers(int on) {
  TL_REQUIRE_CTX(c);
  c->host_buffers = on != 0;
  return TL_OK;
}
