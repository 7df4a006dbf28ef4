// tl_p2p.cu -- ZeRO-1 optimizer step over peer memory (one node, NVLink).
//
// The same step as tl_zero1_step (tinylm.c:2630-2633 on a sharded optimizer),
// with the exchanges done by this library's own kernels instead of NCCL
// collectives:
//
//   1. signal/wait GRAD   every rank's backward has finished writing its G
//   2. rs_sumsq           this rank's shard of the averaged gradient, summed
//                         straight from every rank's G (plain peer loads, rank
//                         order 0..R-1), written in place into the own G, fused
//                         with the shard's sum of squares; the shard total is
//                         stored into every rank's mailbox (+ SUMSQ flag)
//   3. clip               wait for all SUMSQ flags, total in rank order, norm
//                         and clip scale
//   4. adamw              AdamW on the shard; the new parameters are stored into
//                         every rank's P (the all-gather, fused)
//   5. signal/wait PARAM  every rank's P is complete before the next forward
//
// The reduce-scatter and the norm read G once instead of twice, and the
// all-gather costs no extra pass over P.  Peers' P and G are mapped with CUDA
// IPC at registration; the mailboxes (flags and shard sums) are library
// buffers.  Flags carry the step epoch, so nothing is reset between steps.
// Every wait is bounded (TL_DIST_TIMEOUT_MS, %globaltimer): on expiry the rank
// records a device error code (tl_device_status -> TL_ETIMEOUT) and sets its
// abort word.  From then on every kernel of this and later steps returns at
// once, touching no peer memory, and records error 23 again, so each later
// step is reported too; once tl_device_status has seen one of these codes the
// host refuses further steps (TL_ETIMEOUT) until the caller releases the
// peer set and registers again.
// No TMA and no multicast: peer memory is touched only by plain loads/stores.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include <vector>
#include "tl_optim.cuh"
#include "tl_trace.cuh"

namespace tl {

bool dist_rank_world(int *rank, int *world);
int dist_allgather_bytes(const void *send_dev, void *recv_dev, size_t bytes);

constexpr int kMaxRanks = 8;
enum { FLAG_GRAD = 0, FLAG_SUMSQ = 1, FLAG_PARAM = 2, NFLAGS = 3 };
constexpr int ERR_WAIT_GRAD = 20, ERR_WAIT_SUMSQ = 21, ERR_WAIT_PARAM = 22, ERR_ABORTED = 23;

// One per rank in its own device memory, written by every peer.
struct Mailbox {
  unsigned long long flag[NFLAGS][kMaxRanks];  // [kind][writer rank] = epoch
  double sumsq[kMaxRanks];                     // [writer rank] shard sum of squares
  int abort;                                   // a wait of this rank expired
};

struct PeerSet {
  float *P[kMaxRanks];
  float *G[kMaxRanks];
  Mailbox *mb[kMaxRanks];
};

struct P2PCtx {
  bool ready = false;
  int rank = 0, world = 1;
  size_t n = 0, n_pad = 0, shard = 0;
  float *P = nullptr, *G = nullptr;
  Mailbox *own = nullptr;
  PeerSet peers{};
  unsigned long long epoch = 0;
  bool aborted = false;   // tl_device_status saw an expired wait of this rank
  std::vector<void *> opened;
};
static P2PCtx g_p2p[kMaxDevices];

static unsigned long long wait_limit_ns() {
  const char *e = getenv("TL_DIST_TIMEOUT_MS");
  long long v = e ? atoll(e) : 0;
  if (v <= 0) v = 120000;
  return (unsigned long long)v * 1000000ull;
}

// ---------------------------------------------------------------- kernels
// True (and error 23 recorded) when an earlier wait of this rank expired.
__device__ __forceinline__ bool p2p_aborted(const Mailbox *own, int *err) {
  if (!*(volatile const int *)&own->abort) return false;
  if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, ERR_ABORTED);
  return true;
}

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Signal `kind` for this epoch to every rank, then wait until every rank has
// signalled it here.  One warp; lane j talks to rank j.
__global__ void p2p_signal_wait_kernel(PeerSet ps, Mailbox *own, int rank, int world, int kind,
                                       unsigned long long epoch, unsigned long long limit_ns, int *err,
                                       int code) {
  const int lane = threadIdx.x;
  if (p2p_aborted(own, err)) return;
  __threadfence_system();
  if (lane < world) st_release_sys(&ps.mb[lane]->flag[kind][rank], epoch);
  bool ok = true;
  if (lane < world) {
    const unsigned long long t0 = gtime();
    while (ld_acquire_sys(&own->flag[kind][lane]) < epoch) {
      if (gtime() - t0 > limit_ns) { ok = false; break; }
    }
  }
  if (!__all_sync(0xffffffffu, ok) && lane == 0) {
    own->abort = 1;
    atomicExch(err, code);
  }
}

// Averaged gradient of this rank's shard, from every rank's G in rank order,
// in place into the own G; two-stage deterministic sum of squares whose last
// block publishes the shard total to every mailbox.
__global__ void __launch_bounds__(kNormThreads)
p2p_rs_sumsq_kernel(PeerSet ps, Mailbox *own, int rank, int world, size_t shard, double *partials,
                    unsigned int *ticket, unsigned long long epoch, int *err) {
  __shared__ double smem[32];
  __shared__ bool is_last;
  if (p2p_aborted(own, err)) return;
  const size_t off = (size_t)rank * shard;
  const size_t n4 = shard / 4;
  float4 *Gme = reinterpret_cast<float4 *>(ps.G[rank] + off);
  const float fw = (float)world;
  double acc = 0.0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 s = __ldcg(reinterpret_cast<const float4 *>(ps.G[0] + off) + i);
    for (int j = 1; j < world; j++) {
      const float4 x = __ldcg(reinterpret_cast<const float4 *>(ps.G[j] + off) + i);
      s.x += x.x; s.y += x.y; s.z += x.z; s.w += x.w;
    }
    s.x /= fw; s.y /= fw; s.z /= fw; s.w /= fw;
    Gme[i] = s;
    acc += (double)s.x * s.x + (double)s.y * s.y + (double)s.z * s.z + (double)s.w * s.w;
  }
  const double bsum = block_sum(acc, smem);
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
    *ticket = 0u;
    for (int j = 0; j < world; j++) ps.mb[j]->sumsq[rank] = s;
    __threadfence_system();
    for (int j = 0; j < world; j++) st_release_sys(&ps.mb[j]->flag[FLAG_SUMSQ][rank], epoch);
  }
}

// Wait for every rank's shard sum, add them in rank order, norm and clip scale.
__global__ void p2p_clip_kernel(Mailbox *own, int world, unsigned long long epoch, float max_norm,
                                float *norm_out, float *gscale_out, unsigned long long limit_ns, int *err) {
  const int lane = threadIdx.x;
  if (p2p_aborted(own, err)) return;
  bool ok = true;
  double mine = 0.0;
  if (lane < world) {
    const unsigned long long t0 = gtime();
    while (ld_acquire_sys(&own->flag[FLAG_SUMSQ][lane]) < epoch) {
      if (gtime() - t0 > limit_ns) { ok = false; break; }
    }
    if (ok) mine = *(volatile double *)&own->sumsq[lane];
  }
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) { own->abort = 1; atomicExch(err, ERR_WAIT_SUMSQ); }
    return;
  }
  double total = 0.0;
  for (int j = 0; j < world; j++) total += __shfl_sync(0xffffffffu, mine, j);
  if (lane == 0) {
    const float norm = (float)sqrt(total);
    if (norm_out) *norm_out = norm;
    *gscale_out = norm > max_norm ? max_norm / norm : 1.0f;
  }
}

// AdamW on this rank's shard; the updated parameters go to every rank's P.
__global__ void __launch_bounds__(256)
p2p_adamw_kernel(PeerSet ps, Mailbox *own, int rank, int world, size_t shard, float4 *__restrict__ M,
                 float4 *__restrict__ V, AdamArgs a, int *err) {
  if (p2p_aborted(own, err)) return;
  const float gs = __ldg(a.gscale_ptr);
  const size_t off = (size_t)rank * shard;
  const size_t n4 = shard / 4;
  const float4 *P4 = reinterpret_cast<const float4 *>(ps.P[rank] + off);
  const float4 *G4 = reinterpret_cast<const float4 *>(ps.G[rank] + off);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 p = P4[i], m = __ldcs(M + i), v = __ldcs(V + i);
    const float4 g = __ldcs(G4 + i);
    adam_elem(p.x, g.x, m.x, v.x, a, gs); adam_elem(p.y, g.y, m.y, v.y, a, gs);
    adam_elem(p.z, g.z, m.z, v.z, a, gs); adam_elem(p.w, g.w, m.w, v.w, a, gs);
    __stcs(M + i, m);
    __stcs(V + i, v);
    for (int j = 0; j < world; j++) reinterpret_cast<float4 *>(ps.P[j] + off)[i] = p;
  }
  __threadfence_system();
}

// ------------------------------------------------------------------- host
struct Exchange {
  cudaIpcMemHandle_t hP, hG, hMb;
  unsigned long long baseP, baseG, offP, offG;
};

static PFN_cuMemGetAddressRange_v3020 g_range = nullptr;

static int alloc_base(const void *p, unsigned long long *base) {
  if (!g_range) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(TL_ECUDA, "cuMemGetAddressRange not available from the driver");
    g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  if (g_range(&b, &sz, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
    return set_error(TL_EPTR, "cannot find the allocation of a registered buffer");
  *base = (unsigned long long)b;
  return TL_OK;
}

static void release(P2PCtx &x) {
  for (void *p : x.opened) cudaIpcCloseMemHandle(p);
  x.opened.clear();
  x.aborted = false;
  if (x.own) cudaFree(x.own);
  x.own = nullptr;
  x.ready = false;
}

// tl_device_status found a peer-wait code (20-23) on `device`.
void p2p_mark_aborted(int device, int code) {
  if (device >= 0 && device < kMaxDevices && g_p2p[device].ready && code >= ERR_WAIT_GRAD && code <= ERR_ABORTED)
    g_p2p[device].aborted = true;
}

void p2p_release_device(int device) {
  if (device >= 0 && device < kMaxDevices && (g_p2p[device].ready || g_p2p[device].own)) {
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    release(g_p2p[device]);
    cudaSetDevice(cur);
  }
}

}  // namespace tl

using namespace tl;

TL_API int tl_zero1_p2p_register(float *P, float *G, size_t n) {
  TL_REQUIRE_CTX(c);
  int rank, world;
  if (!dist_rank_world(&rank, &world)) return set_error(TL_ENOINIT, "tl_dist_init() not called for this device");
  if (world > kMaxRanks) return set_error(TL_EINVAL, "peer-memory step supports up to %d ranks (got %d)", kMaxRanks, world);
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G"))) return rc;
  if (((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(G)) & 15) != 0)
    return set_error(TL_EALIGN, "P and G must be 16-byte aligned");
  P2PCtx &x = g_p2p[c->device];
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  release(x);
  x.rank = rank; x.world = world; x.n = n;
  x.n_pad = tl_zero1_padded(n, world);
  x.shard = x.n_pad / world;
  x.P = P; x.G = G;
  x.epoch = 0;
  TL_TRY_CUDA(cudaMalloc(&x.own, sizeof(Mailbox)));
  TL_TRY_CUDA(cudaMemset(x.own, 0, sizeof(Mailbox)));
  TL_TRY_CUDA(cudaDeviceSynchronize());

  Exchange mine{};
  if ((rc = alloc_base(P, &mine.baseP)) || (rc = alloc_base(G, &mine.baseG))) { release(x); return rc; }
  mine.offP = reinterpret_cast<unsigned long long>(P) - mine.baseP;
  mine.offG = reinterpret_cast<unsigned long long>(G) - mine.baseG;
  cudaError_t e1 = cudaIpcGetMemHandle(&mine.hP, reinterpret_cast<void *>(mine.baseP));
  cudaError_t e2 = cudaIpcGetMemHandle(&mine.hG, reinterpret_cast<void *>(mine.baseG));
  cudaError_t e3 = cudaIpcGetMemHandle(&mine.hMb, x.own);
  if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) {
    cudaGetLastError();
    release(x);
    return set_error(TL_EINVAL, "P/G cannot be shared over CUDA IPC (%s); use tl_zero1_step",
                     cudaGetErrorString(e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3)));
  }
  // Exchange the records through the communicator.
  void *dbuf = nullptr;
  TL_TRY_CUDA(cudaMalloc(&dbuf, sizeof(Exchange) * (world + 1)));
  std::vector<Exchange> all(world);
  Exchange *dsend = reinterpret_cast<Exchange *>(dbuf) + world;
  rc = cuda_check(cudaMemcpy(dsend, &mine, sizeof mine, cudaMemcpyHostToDevice), "cudaMemcpy");
  if (!rc) rc = dist_allgather_bytes(dsend, dbuf, sizeof(Exchange));
  if (!rc) rc = cuda_check(cudaMemcpy(all.data(), dbuf, sizeof(Exchange) * world, cudaMemcpyDeviceToHost), "cudaMemcpy");
  cudaFree(dbuf);
  if (rc) { release(x); return rc; }
  for (int j = 0; j < world; j++) {
    if (j == rank) {
      x.peers.P[j] = P; x.peers.G[j] = G; x.peers.mb[j] = x.own;
      continue;
    }
    void *mb = nullptr, *bp = nullptr, *bg = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&mb, all[j].hMb, cudaIpcMemLazyEnablePeerAccess);
    if (e == cudaSuccess) { x.opened.push_back(mb); e = cudaIpcOpenMemHandle(&bp, all[j].hP, cudaIpcMemLazyEnablePeerAccess); }
    if (e == cudaSuccess) {
      x.opened.push_back(bp);
      if (all[j].baseG == all[j].baseP) {
        bg = bp;  // P and G in one allocation of that rank: one mapping
      } else {
        e = cudaIpcOpenMemHandle(&bg, all[j].hG, cudaIpcMemLazyEnablePeerAccess);
        if (e == cudaSuccess) x.opened.push_back(bg);
      }
    }
    if (e != cudaSuccess) {
      cudaGetLastError();
      release(x);
      return set_error(TL_ECUDA, "cudaIpcOpenMemHandle for rank %d: %s", j, cudaGetErrorString(e));
    }
    x.peers.mb[j] = reinterpret_cast<Mailbox *>(mb);
    x.peers.P[j] = reinterpret_cast<float *>(reinterpret_cast<char *>(bp) + all[j].offP);
    x.peers.G[j] = reinterpret_cast<float *>(reinterpret_cast<char *>(bg) + all[j].offG);
  }
  // Every rank has mapped every peer before anyone signals.
  void *z = nullptr;
  TL_TRY_CUDA(cudaMalloc(&z, 8 * (world + 1)));
  rc = dist_allgather_bytes(reinterpret_cast<char *>(z) + 8 * world, z, 8);
  cudaFree(z);
  if (rc) { release(x); return rc; }
  x.ready = true;
  return TL_OK;
}

TL_API int tl_zero1_p2p_release(void) {
  TL_REQUIRE_CTX(c);
  TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
  release(g_p2p[c->device]);
  return TL_OK;
}

TL_API int tl_zero1_step_p2p(float *P, float *G, float *M_shard, float *V_shard, size_t n, float lr,
                             float b1, float b2, float wd, int t, float max_norm, float *norm_dev) {
  TL_REQUIRE_CTX(c);
  P2PCtx &x = g_p2p[c->device];
  if (!x.ready) return set_error(TL_ENOINIT, "tl_zero1_p2p_register() not called for this device");
  if (P != x.P || G != x.G || n != x.n)
    return set_error(TL_EINVAL, "P, G and n must be the buffers registered with tl_zero1_p2p_register");
  if (x.aborted)
    return set_error(TL_ETIMEOUT, "an earlier peer wait of this rank expired; release the peer set "
                                  "(tl_zero1_p2p_release) and register again");
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (!(max_norm > 0.0f)) return set_error(TL_EINVAL, "max_norm must be > 0");
  int rc;
  if ((rc = check_device_ptr(M_shard, "M_shard")) || (rc = check_device_ptr(V_shard, "V_shard"))) return rc;
  if (((reinterpret_cast<uintptr_t>(M_shard) | reinterpret_cast<uintptr_t>(V_shard)) & 15) != 0)
    return set_error(TL_EALIGN, "M_shard and V_shard must be 16-byte aligned");
  const unsigned long long ep = ++x.epoch;
  const unsigned long long lim = wait_limit_ns();
  {
    TraceScope ts(c, "p2p_wait");
    p2p_signal_wait_kernel<<<1, 32, 0, c->stream>>>(x.peers, x.own, x.rank, x.world, FLAG_GRAD, ep, lim,
                                                    c->err_flag, ERR_WAIT_GRAD);
    TL_TRY_CUDA(cudaGetLastError());
  }
  {
    TraceScope ts(c, "p2p_rs_sumsq");
    p2p_rs_sumsq_kernel<<<kNormBlocks, kNormThreads, 0, c->stream>>>(x.peers, x.own, x.rank, x.world, x.shard,
                                                                     c->norm_partials, c->norm_ticket, ep,
                                                                     c->err_flag);
    TL_TRY_CUDA(cudaGetLastError());
  }
  float *gscale = c->scalars + 1;
  {
    TraceScope ts(c, "p2p_clip");
    p2p_clip_kernel<<<1, 32, 0, c->stream>>>(x.own, x.world, ep, max_norm, norm_dev, gscale, lim, c->err_flag);
    TL_TRY_CUDA(cudaGetLastError());
  }
  {
    TraceScope ts(c, "p2p_adamw");
    const AdamArgs a = make_adam_args(lr, b1, b2, wd, t, 1.0f, gscale);
    size_t blocks = (x.shard / 4 + 255) / 256;
    const size_t cap = (size_t)c->num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    p2p_adamw_kernel<<<(unsigned)blocks, 256, 0, c->stream>>>(x.peers, x.own, x.rank, x.world, x.shard,
                                                               reinterpret_cast<float4 *>(M_shard),
                                                               reinterpret_cast<float4 *>(V_shard), a,
                                                               c->err_flag);
    TL_TRY_CUDA(cudaGetLastError());
  }
  {
    TraceScope ts(c, "p2p_wait");
    p2p_signal_wait_kernel<<<1, 32, 0, c->stream>>>(x.peers, x.own, x.rank, x.world, FLAG_PARAM, ep, lim,
                                                    c->err_flag, ERR_WAIT_PARAM);
    TL_TRY_CUDA(cudaGetLastError());
  }
  return TL_OK;
}
