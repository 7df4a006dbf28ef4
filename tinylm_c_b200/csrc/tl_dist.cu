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
#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include "tl_common.cuh"
#include "tl_dist.cuh"
#include "tl_trace.cuh"

namespace tl {
int launch_sumsq(DeviceCtx *c, const float *G, size_t n, double *sumsq_out, float *norm_out,
                 float *gscale_out, float max_norm);
int launch_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr,
                 float b1, float b2, float wd, int t, float gscale, const float *gscale_dev,
                 const float *hyper = nullptr);
__global__ void clip_scale_kernel(const double *sumsq, float max_norm, float *norm_out, float *gscale_out);
void p2p_release_device(int device);

struct DistCtx {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = -1;
  bool ready = false;
  cudaStream_t side = nullptr;            // overlapped shard reductions
  cudaEvent_t ev[kMaxShards + 1] = {};
};
static DistCtx g_dist[kMaxDevices];

static int timeout_ms() {
  const char *e = getenv("TL_DIST_TIMEOUT_MS");
  int v = e ? atoi(e) : 0;
  return v > 0 ? v : 120000;
}
// Communicator creation (bootstrap, topology and channel set-up) can take
// seconds on a cold node, whatever bound the steps use: its own limit,
// TL_DIST_INIT_TIMEOUT_MS, at least the step bound, default 120 s.
static int init_timeout_ms() {
  const char *e = getenv("TL_DIST_INIT_TIMEOUT_MS");
  const int v = e ? atoi(e) : 0;
  return std::max(v > 0 ? v : 120000, timeout_ms());
}

static int nccl_fail(DistCtx &d, ncclResult_t r, const char *what) {
  set_error(TL_ENCCL, "%s: %s", what, ncclGetErrorString(r));
  if (d.comm) { ncclCommAbort(d.comm); d.comm = nullptr; }
  d.ready = false;
  return TL_ENCCL;
}

// Poll the communicator until the last call has been accepted or failed
// (limit_ms: the bound, default the step bound).
static int nccl_settle(DistCtx &d, ncclResult_t r, const char *what, int limit_ms = 0) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(d, r, what);
  const int lim = limit_ms > 0 ? limit_ms : timeout_ms();
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(lim);
  ncclResult_t st = ncclInProgress;
  while (true) {
    ncclResult_t q = ncclCommGetAsyncError(d.comm, &st);
    if (q != ncclSuccess) return nccl_fail(d, q, what);
    if (st == ncclSuccess) return TL_OK;
    if (st != ncclInProgress) return nccl_fail(d, st, what);
    if (std::chrono::steady_clock::now() > deadline) {
      set_error(TL_ETIMEOUT, "%s: no progress within %d ms", what, lim);
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
// stream, then wait for it with the host deadline.  Used for set-up exchanges
// (peer-memory registration), so it is bounded like communicator creation
// (TL_DIST_INIT_TIMEOUT_MS): the first collective on a communicator also
// builds its connections, which can take seconds on a cold node.
int dist_allgather_bytes(const void *send_dev, void *recv_dev, size_t bytes) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  ncclResult_t r = ncclAllGather(send_dev, recv_dev, bytes, ncclInt8, d->comm, c->stream);
  int rc = nccl_settle(*d, r, "ncclAllGather(bytes)", init_timeout_ms());
  if (rc) return rc;
  return tl_dist_sync(init_timeout_ms());
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
  int rc = nccl_settle(d, r, "ncclCommInitRankConfig", init_timeout_ms());
  if (rc) return rc;
  d.ready = true;
  return TL_OK;
}

TL_API int tl_dist_finalize(void) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TL_OK;
  p2p_release_device(dev);
  DistCtx &d = g_dist[dev];
  if (d.side) {
    cudaStreamSynchronize(d.side);
    for (auto &e : d.ev) if (e) { cudaEventDestroy(e); e = nullptr; }
    cudaStreamDestroy(d.side);
    d.side = nullptr;
  }
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

namespace tl {

// Steps 2-5 of the ZeRO-1 step, once this rank's shard of G holds the
// averaged gradient: shard sum of squares -> all-reduce -> clip scale ->
// AdamW on the shard -> all-gather of P.
static int zero1_tail(DeviceCtx *c, DistCtx *d, float *P, float *G, float *M_shard, float *V_shard, size_t shard,
                      float lr, float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  int rc;
  float *Gs = G + (size_t)d->rank * shard;
  float *Ps = P + (size_t)d->rank * shard;
  if ((rc = launch_sumsq(c, Gs, shard, c->sumsq, nullptr, nullptr, max_norm))) return rc;
  ncclResult_t r = ncclAllReduce(c->sumsq, c->sumsq, 1, ncclDouble, ncclSum, d->comm, c->stream);
  if ((rc = nccl_settle(*d, r, "ncclAllReduce(sumsq)"))) return rc;
  float *gscale = c->scalars + 1;
  {
    TraceScope ts(c, "clip_scale");
    clip_scale_kernel<<<1, 1, 0, c->stream>>>(c->sumsq, max_norm, norm_dev, gscale);
    TL_TRY_CUDA(cudaGetLastError());
  }
  if ((rc = launch_adamw(c, Ps, Gs, M_shard, V_shard, shard, lr, b1, b2, wd, t, 1.0f, gscale))) return rc;
  r = ncclAllGather(Ps, P, shard, ncclFloat, d->comm, c->stream);
  return nccl_settle(*d, r, "ncclAllGather(P)");
}

static int zero1_args(DeviceCtx *c, DistCtx *d, float *P, float *G, float *M_shard, float *V_shard, int t,
                      float max_norm) {
  (void)c;
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (!(max_norm > 0.0f)) return set_error(TL_EINVAL, "max_norm must be > 0");
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) ||
      (rc = check_device_ptr(M_shard, "M_shard")) || (rc = check_device_ptr(V_shard, "V_shard")))
    return rc;
  return TL_OK;
}

// ------------------------------------------------ reduction overlapped with backward
// The shards double as buckets: shard j is reduced (average) onto its owner
// rank j with one ncclReduce as soon as the backward pass has finished every
// gradient inside it.  The backward fills the flat G from the end (MTP heads,
// final norm, last layer ...) towards the embedding at offset 0, so the high
// shards go out while the early layers are still being differentiated.  The
// reductions run on a side stream ordered by events; every rank issues them
// in the same order (shard R-1 down to 0), so the communicator sees one
// sequence.  At the end the library stream waits for the side stream.
int overlap_begin(DeviceCtx *c, float *G, size_t n, OverlapState *o) {
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  if (!d->side) {
    TL_TRY_CUDA(cudaStreamCreateWithFlags(&d->side, cudaStreamNonBlocking));
    for (int i = 0; i < kMaxShards + 1; i++) TL_TRY_CUDA(cudaEventCreateWithFlags(&d->ev[i], cudaEventDisableTiming));
  }
  if (d->world > kMaxShards) return set_error(TL_EINVAL, "overlapped reduction supports up to %d ranks", kMaxShards);
  o->G = G;
  o->n_pad = tl_zero1_padded(n, d->world);
  o->shard = o->n_pad / d->world;
  o->next = d->world - 1;   // highest shard not issued yet
  o->events = 0;
  return TL_OK;
}

// G[done_from, n_pad) is final: reduce every remaining shard inside it.
int overlap_ready(DeviceCtx *c, OverlapState *o, size_t done_from) {
  DistCtx *d = dist();
  if (!d) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  if (o->next < 0 || (size_t)o->next * o->shard < done_from) return TL_OK;
  cudaEvent_t ev = d->ev[o->events++];
  TL_TRY_CUDA(cudaEventRecord(ev, c->stream));
  TL_TRY_CUDA(cudaStreamWaitEvent(d->side, ev, 0));
  while (o->next >= 0 && (size_t)o->next * o->shard >= done_from) {
    float *Gj = o->G + (size_t)o->next * o->shard;
    ncclResult_t r = ncclReduce(Gj, Gj, o->shard, ncclFloat, ncclAvg, o->next, d->comm, d->side);
    int rc = nccl_settle(*d, r, "ncclReduce(G shard)");
    if (rc) return rc;
    o->next--;
  }
  return TL_OK;
}

// Reduce what is left and join the side stream into the library stream.
int overlap_finish(DeviceCtx *c, OverlapState *o) {
  int rc = overlap_ready(c, o, 0);
  if (rc) return rc;
  DistCtx *d = dist();
  cudaEvent_t ev = d->ev[kMaxShards];
  TL_TRY_CUDA(cudaEventRecord(ev, d->side));
  TL_TRY_CUDA(cudaStreamWaitEvent(c->stream, ev, 0));
  return TL_OK;
}

int zero1_finish_after_overlap(DeviceCtx *c, float *P, float *G, float *M_shard, float *V_shard, size_t n,
                               float lr, float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  DistCtx *d = dist();
  int rc = zero1_args(c, d, P, G, M_shard, V_shard, t, max_norm);
  if (rc) return rc;
  const size_t shard = tl_zero1_padded(n, d->world) / d->world;
  return zero1_tail(c, d, P, G, M_shard, V_shard, shard, lr, b1, b2, wd, t, max_norm, norm_dev);
}

}  // namespace tl

TL_API int tl_zero1_step(float *P, float *G, float *M_shard, float *V_shard, size_t n, float lr,
                         float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  TL_REQUIRE_CTX(c);
  DistCtx *d = dist();
  int rc = zero1_args(c, d, P, G, M_shard, V_shard, t, max_norm);
  if (rc) return rc;
  const size_t n_pad = tl_zero1_padded(n, d->world);
  const size_t shard = n_pad / d->world;
  float *Gs = G + (size_t)d->rank * shard;
  // 1. gradient average, this rank's shard lands in place
  ncclResult_t r = ncclReduceScatter(G, Gs, shard, ncclFloat, ncclAvg, d->comm, c->stream);
  if ((rc = nccl_settle(*d, r, "ncclReduceScatter(G)"))) return rc;
  return zero1_tail(c, d, P, G, M_shard, V_shard, shard, lr, b1, b2, wd, t, max_norm, norm_dev);
}
