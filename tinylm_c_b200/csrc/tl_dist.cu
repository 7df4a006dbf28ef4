// tl_dist.cu -- data parallelism with a ZeRO-1 sharded optimizer step (NCCL).
//
// The reference has no distributed code; this is the multi-GPU form of its
// optimizer step (tinylm.c:2630-2633): the gradient is reduce-scattered with
// averaging, each rank takes the sum of squares of its shard, one 8-byte
// all-reduce gives every rank the same global norm and clip scale, AdamW runs
// on the rank's shard of P/M/V, and P is all-gathered.
//
// Failure handling: the communicator is non-blocking, every NCCL call is
// followed by a bounded poll of ncclCommGetAsyncError, and tl_dist_sync waits
// for the stream with a host-side deadline.  A peer that never arrives turns
// into TL_ETIMEOUT (the communicator is aborted) instead of a hang.
#include <nccl.h>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include "tl_common.cuh"

namespace tl {
int launch_sumsq(DeviceCtx *c, const float *G, size_t n, double *sumsq_out, float *norm_out,
                 float *gscale_out, float max_norm);
int launch_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr,
                 float b1, float b2, float wd, int t, float gscale, const float *gscale_dev);
__global__ void clip_scale_kernel(const double *sumsq, float max_norm, float *norm_out, float *gscale_out);
void p2p_release_device(int device);

struct DistCtx {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = -1;
  bool ready = false;
};
static DistCtx g_dist[kMaxDevices];

static int timeout_ms() {
  const char *e = getenv("TL_DIST_TIMEOUT_MS");
  int v = e ? atoi(e) : 0;
  return v > 0 ? v : 120000;
}

static int nccl_fail(DistCtx &d, ncclResult_t r, const char *what) {
  set_error(TL_ENCCL, "%s: %s", what, ncclGetErrorString(r));
  if (d.comm) { ncclCommAbort(d.comm); d.comm = nullptr; }
  d.ready = false;
  return TL_ENCCL;
}

// Poll the communicator until the last call has been accepted or failed.
static int nccl_settle(DistCtx &d, ncclResult_t r, const char *what) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(d, r, what);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms());
  ncclResult_t st = ncclInProgress;
  while (true) {
    ncclResult_t q = ncclCommGetAsyncError(d.comm, &st);
    if (q != ncclSuccess) return nccl_fail(d, q, what);
    if (st == ncclSuccess) return TL_OK;
    if (st != ncclInProgress) return nccl_fail(d, st, what);
    if (std::chrono::steady_clock::now() > deadline) {
      set_error(TL_ETIMEOUT, "%s: no progress within %d ms", what, timeout_ms());
      ncclCommAbort(d.comm);
      d.comm = nullptr;
      d.ready = false;
      return TL_ETIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static DistCtx *dist() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return g_dist[dev].ready ? &g_dist[dev] : nullptr;
}

// This device's rank and world size (false without a communicator).
bool dist_rank_world(int *rank, int *world) {
  DistCtx *d = dist();
  if (!d) return false;
  *rank = d->rank;
  *world = d->world;
  return true;
}

// All-gather `bytes` bytes per rank between device buffers on the library
// stream, then wait for it with the host deadline.
int dist_allgather_bytes(const void *send_dev, void *recv_dev, size_t bytes) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  ncclResult_t r = ncclAllGather(send_dev, recv_dev, bytes, ncclInt8, d->comm, c->stream);
  int rc = nccl_settle(*d, r, "ncclAllGather(bytes)");
  if (rc) return rc;
  return tl_dist_sync(0);
}

}  // namespace tl

using namespace tl;

TL_API size_t tl_zero1_padded(size_t n, int world) {
  if (world < 1) world = 1;
  const size_t q = (size_t)world * TL_ZERO1_ALIGN;
  return (n + q - 1) / q * q;
}

TL_API int tl_dist_unique_id(void *uid128) {
  if (!uid128) return set_error(TL_EINVAL, "uid buffer is NULL");
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(TL_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(uid128, &id, sizeof id);
  return TL_OK;
}

TL_API int tl_dist_init(int rank, int world, const void *uid128) {
  TL_REQUIRE_CTX(c);
  if (world < 1 || rank < 0 || rank >= world) return set_error(TL_EINVAL, "rank %d / world %d", rank, world);
  if (!uid128) return set_error(TL_EINVAL, "uid is NULL");
  DistCtx &d = g_dist[c->device];
  if (d.ready) {
    if (d.rank == rank && d.world == world) return TL_OK;
    return set_error(TL_EINVAL, "communicator already initialised as rank %d / %d", d.rank, d.world);
  }
  ncclUniqueId id;
  memcpy(&id, uid128, sizeof id);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  d.rank = rank; d.world = world; d.device = c->device;
  ncclResult_t r = ncclCommInitRankConfig(&d.comm, world, id, rank, &cfg);
  int rc = nccl_settle(d, r, "ncclCommInitRankConfig");
  if (rc) return rc;
  d.ready = true;
  return TL_OK;
}

TL_API int tl_dist_finalize(void) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TL_OK;
  p2p_release_device(dev);
  DistCtx &d = g_dist[dev];
  if (d.comm) {
    ncclCommFinalize(d.comm);
    ncclResult_t st = ncclInProgress;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms());
    while (ncclCommGetAsyncError(d.comm, &st) == ncclSuccess && st == ncclInProgress &&
           std::chrono::steady_clock::now() < deadline)
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    if (st == ncclSuccess) ncclCommDestroy(d.comm); else ncclCommAbort(d.comm);
    d.comm = nullptr;
  }
  d.ready = false;
  return TL_OK;
}

TL_API int tl_dist_allreduce_f32(float *buf, size_t count, int average) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat, average ? ncclAvg : ncclSum, d->comm, c->stream);
  return nccl_settle(*d, r, "ncclAllReduce(f32)");
}

TL_API int tl_dist_allreduce_f64(double *buf, size_t count) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  ncclResult_t r = ncclAllReduce(buf, buf, count, ncclDouble, ncclSum, d->comm, c->stream);
  return nccl_settle(*d, r, "ncclAllReduce(f64)");
}

// Wait for the library stream with a host deadline; a communicator error or a
// timeout aborts the communicator and returns an error status.
TL_API int tl_dist_sync(int timeout_ms_arg) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  const int lim = timeout_ms_arg > 0 ? timeout_ms_arg : timeout_ms();
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(lim);
  while (true) {
    cudaError_t e = cudaStreamQuery(c->stream);
    if (e == cudaSuccess) return TL_OK;
    if (e != cudaErrorNotReady) return cuda_check(e, "cudaStreamQuery");
    if (d) {
      ncclResult_t st = ncclSuccess;
      ncclResult_t q = ncclCommGetAsyncError(d->comm, &st);
      if (q != ncclSuccess) return nccl_fail(*d, q, "ncclCommGetAsyncError");
      if (st != ncclSuccess && st != ncclInProgress) return nccl_fail(*d, st, "communicator");
    }
    if (std::chrono::steady_clock::now() > deadline) {
      if (d && d->comm) { ncclCommAbort(d->comm); d->comm = nullptr; d->ready = false; }
      return set_error(TL_ETIMEOUT, "stream did not drain within %d ms", lim);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

TL_API int tl_zero1_step(float *P, float *G, float *M_shard, float *V_shard, size_t n, float lr,
                         float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (!(max_norm > 0.0f)) return set_error(TL_EINVAL, "max_norm must be > 0");
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) ||
      (rc = check_device_ptr(M_shard, "M_shard")) || (rc = check_device_ptr(V_shard, "V_shard")))
    return rc;
  const size_t n_pad = tl_zero1_padded(n, d->world);
  const size_t shard = n_pad / d->world;
  float *Gs = G + (size_t)d->rank * shard;
  float *Ps = P + (size_t)d->rank * shard;
  // 1. gradient average, this rank's shard lands in place
  ncclResult_t r = ncclReduceScatter(G, Gs, shard, ncclFloat, ncclAvg, d->comm, c->stream);
  if ((rc = nccl_settle(*d, r, "ncclReduceScatter(G)"))) return rc;
  // 2. shard sum of squares -> 3. global sum -> clip scale
  if ((rc = launch_sumsq(c, Gs, shard, c->sumsq, nullptr, nullptr, max_norm))) return rc;
  r = ncclAllReduce(c->sumsq, c->sumsq, 1, ncclDouble, ncclSum, d->comm, c->stream);
  if ((rc = nccl_settle(*d, r, "ncclAllReduce(sumsq)"))) return rc;
  float *gscale = c->scalars + 1;
  clip_scale_kernel<<<1, 1, 0, c->stream>>>(c->sumsq, max_norm, norm_dev, gscale);
  TL_TRY_CUDA(cudaGetLastError());
  // 4. AdamW on the owned shard
  if ((rc = launch_adamw(c, Ps, Gs, M_shard, V_shard, shard, lr, b1, b2, wd, t, 1.0f, gscale))) return rc;
  // 5. every rank receives the updated parameters
  r = ncclAllGather(Ps, P, shard, ncclFloat, d->comm, c->stream);
  return nccl_settle(*d, r, "ncclAllGather(P)");
}
