/* tinylm_cuda.h -- C ABI of libtinylm_cuda, the B200 (sm_100a) implementation of
 * tinylm-c's training-step hot path.
 *
 * Drop-in boundary.  Each compute entry point replaces one CPU primitive of the
 * reference (tinylm.c) one for one, with the same argument order and meaning, so
 * a call site changes only by name:
 *
 *   reference (tinylm.c)                          this library
 *   mm(Y,X,W,M,K,N)              439-478   ->     tl_matmul(Y,X,W,M,K,N)
 *   mm_bt(dX,dY,W,M,K,N)         480-508   ->     tl_matmul_bt(dX,dY,W,M,K,N)
 *   mm_atb(dW,X,dY,M,K,N)        510-537   ->     tl_matmul_at(dW,X,dY,M,K,N)
 *   global_gradnorm(G,n)        1171-1176  ->     tl_grad_norm(G,n,&norm)
 *   adamw(P,G,M,V,n,lr,b1,b2,wd,t,gscale)
 *                               1159-1170  ->     tl_adamw_step(...same...)
 *   gnm>1 ? 1/gnm : 1      2630-2631, 4739 ->     tl_clip_adamw_step (norm+clip+AdamW,
 *                                                  no host round trip)
 *
 * Conventions
 *  - All matrices are fp32, row-major, densely packed (leading dimension = the
 *    row length), exactly as the reference stores them.
 *  - Every float pointer passed to a compute call is a DEVICE pointer (from
 *    tl_alloc, cudaMalloc, or a framework allocator).  There is no CPU fallback:
 *    a host pointer is rejected with TL_EPTR, unless host-buffer mode
 *    (tl_set_host_buffers) stages it through device memory for the five
 *    reference-facing calls.
 *  - Calls are asynchronous and ordered on the library stream of the current
 *    device (tl_set_stream); tl_sync() is the only call that blocks, except the
 *    few documented to read a result back into host memory.
 *  - Every call returns TL_OK (0) or a negative TL_E* code and never exits the
 *    process; tl_last_error() returns the message of the last failure on the
 *    calling thread.  The reference had no error codes and called exit(1).
 *  - One host thread drives one device; the library is not re-entrant across
 *    threads sharing a device.
 */
#ifndef TINYLM_CUDA_H
#define TINYLM_CUDA_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TL_OK        0
#define TL_EINVAL   -1   /* bad shape, size or argument                       */
#define TL_EALIGN   -2   /* pointer not aligned as the call requires          */
#define TL_ECUDA    -3   /* CUDA runtime or driver error                      */
#define TL_ENCCL    -4   /* NCCL error                                        */
#define TL_ETIMEOUT -5   /* a bounded wait ran out                            */
#define TL_ENOINIT  -6   /* tl_init / tl_dist_init not called for this device */
#define TL_EPTR     -7   /* host pointer where a device pointer is required   */
#define TL_ENOMEM   -8   /* device allocation failed                          */

/* ---------------------------------------------------------------- runtime */
/* Select `device`, create its library stream and its persistent workspace
 * (norm partials).  Idempotent per device.  Replaces nothing in the reference
 * (its buffers are host callocs, fz() tinylm.c:137). */
int tl_init(int device);
/* Use `stream` (a cudaStream_t) for all later calls on the current device.
 * NULL selects the CUDA legacy default stream (the stream torch uses unless
 * told otherwise).  Until the first call the library uses its own
 * non-blocking stream, created by tl_init. */
int tl_set_stream(void *stream);
void *tl_get_stream(void);
const char *tl_last_error(void);
const char *tl_version(void);
int tl_alloc(void **ptr, size_t bytes);
int tl_free(void *ptr);
int tl_memcpy_h2d(void *dst_dev, const void *src_host, size_t bytes);
int tl_memcpy_d2h(void *dst_host, const void *src_dev, size_t bytes);
int tl_memset(void *dst_dev, int value, size_t bytes);
int tl_sync(void);
/* Host-buffer mode, for a host program that keeps its buffers in ordinary
 * host memory and reads each result as soon as the call returns -- tinylm.c
 * itself, whose buffers are fz() callocs (tinylm.c:137) and whose mm, mm_bt,
 * mm_atb, adamw and global_gradnorm (439-537, 1159-1176) are the call sites
 * this library replaces.  When on (for the current device), tl_matmul,
 * tl_matmul_bt, tl_matmul_at, tl_grad_norm and tl_adamw_step also accept
 * host pointers: each host operand is copied into a staging arena on the
 * device (grown to the largest call, kept until exit), the device code runs
 * as for device pointers, outputs are copied back and the call returns once
 * they are in host memory.  Device pointers in the same call are used in
 * place.  Off by default: a host pointer is then TL_EPTR.  The reference has
 * no counterpart (its primitives always run on the host). */
int tl_set_host_buffers(int on);
/* Wait for the stream, then report (and clear) the device error word that
 * bounded waits inside library kernels set when they give up: TL_ETIMEOUT if
 * any kernel since the last call returned early, else TL_OK. */
int tl_device_status(void);

/* Kernel tracing: when on, every library kernel launch is bracketed by CUDA
 * events on its stream; tl_trace_get returns the summed device time (ms) and
 * launch count per kernel name (it waits for pending events).  Names in
 * launch order: tl_trace_names (comma separated).  The reference only has
 * wall-clock timing (wtime, tinylm.c:139-145). */
int tl_trace_enable(int on);
int tl_trace_reset(void);
int tl_trace_get(const char *name, double *total_ms, long long *count);
int tl_trace_names(char *buf, size_t len);

/* ------------------------------------------------------------------ GEMMs */
/* Y[M,N] = X[M,K] @ W[K,N]  (overwrite, beta = 0).  tinylm.c:439-478 (mm). */
int tl_matmul(float *Y, const float *X, const float *W, int M, int K, int N);
/* dX[M,K] += dY[M,N] @ W[K,N]^T  (accumulate, beta = 1).  tinylm.c:480-508 (mm_bt). */
int tl_matmul_bt(float *dX, const float *dY, const float *W, int M, int K, int N);
/* dW[K,N] += X[M,K]^T @ dY[M,N]  (accumulate, beta = 1).  tinylm.c:510-537 (mm_atb). */
int tl_matmul_at(float *dW, const float *X, const float *dY, int M, int K, int N);

/* dX[M,K] = sum over t < nprod of dY[t][M,N[t]] @ W[t][K,N[t]]^T (overwrite),
 * 1 <= nprod <= 3; dY and W are host arrays of device pointers.  Where the
 * CTA-pair tensor-core kernel takes every product this is one launch whose
 * reduction runs through the products in turn; otherwise one mm_bt per
 * product.  Replaces the reference's memset followed by consecutive mm_bt
 * calls into one gradient: tinylm.c:1135-1138 (dq, dk, dv into the attention
 * norm's gradient) and 1113-1115 (the two FFN input projections). */
int tl_matmul_bt_sum(float *dX, int nprod, const float *const *dY, const float *const *W, const int *N, int M,
                     int K);

/* GEMM engine selection, for tests and benchmarks: 0 = automatic (tensor
 * cores where the shape allows, else CUDA-core fp32; the CTA pair uses the
 * tf32 split for these calls and the hybrid split for the GEMMs of the device
 * training step, tl_model_*), 1 = CUDA-core fp32 only, 2 = tensor-core 3xTF32,
 * one CTA per 128 x 128 tile, 3 = tensor-core 3xTF32, a CTA pair (two SMs,
 * cta_group::2) per 256 x 256 tile, 4 = the CTA pair with each operand scaled
 * by a power of two and split into fp16 hi + lo (fp16 MMAs at twice the tf32
 * rate, at least the same accuracy), 5 = the CTA pair with the hybrid split:
 * one tf32 MMA for hi*hi and the two cross terms as one bf16 chain over
 * [hi | lo] x [lo | hi] (no scaling; within the same 1e-4 bound)
 * (2-5: TL_EINVAL where the shape does not allow the tensor-core engine).
 * No counterpart in the reference (its only engine switch is USE_BLAS,
 * tinylm.c:29-31). */
int tl_set_gemm_engine(int engine);
/* Engine the last GEMM call on this thread ran on (1 to 5), 0 if none. */
int tl_last_gemm_engine(void);

/* -------------------------------------------------------------- optimizer */
/* norm = sqrt(sum_i (double)G[i]^2), rounded to float.  tinylm.c:1171-1176.
 * `norm_out` may be a device or a host pointer; a host pointer makes the call
 * synchronous (it waits for the result). */
int tl_grad_norm(const float *G, size_t n, float *norm_out);
/* The same norm (up to summation order: the two may differ in the last bit)
 * for callers that cannot allocate device memory (a framework
 * whose allocator owns the whole GPU, a runtime with a fixed memory budget):
 * no cudaMalloc, no tl_init needed.  No counterpart in the reference.  Uses a
 * scratch array compiled into the library (128 KiB per device that loads it,
 * held until exit), so n <= 2^30 elements; larger n returns TL_EINVAL.
 * norm_dev is a device float; stream a cudaStream_t (NULL = legacy default).
 * The first call on a device looks up the scratch address, so make it before
 * any stream capture.  Calls share the scratch: calls that overlap on the GPU
 * race and must be serialised by the caller. */
int tl_grad_norm_noalloc(const float *G, size_t n, float *norm_dev, void *stream);
/* sumsq_dev[0] = sum_i (double)G[i]^2 (device double) -- the per-shard half of
 * global_gradnorm, for sharded (ZeRO-1) norms. */
int tl_grad_sumsq(const float *G, size_t n, double *sumsq_dev);
/* From a device sum of squares: norm = sqrt(sumsq), gscale = norm > max_norm ?
 * max_norm / norm : 1 (tinylm.c:2631 with the clip of 1.0 made a parameter).
 * Either output pointer may be NULL. */
int tl_clip_scale(const double *sumsq_dev, float max_norm, float *norm_dev, float *gscale_dev);

/* AdamW with clip scale folded in; G is not modified.  tinylm.c:1159-1170.
 * bc1 = 1-b1^t, bc2 = 1-b2^t in fp32; eps = 1e-8 added to sqrt(vhat);
 * decoupled weight decay wd*P on every parameter. */
int tl_adamw_step(float *P, const float *G, float *M, float *V, size_t n,
                  float lr, float b1, float b2, float wd, int t, float gscale);
/* Same, with the clip scale read from device memory (NULL = 1.0): no host sync. */
int tl_adamw_step_dev(float *P, const float *G, float *M, float *V, size_t n,
                      float lr, float b1, float b2, float wd, int t,
                      const float *gscale_dev);
/* The whole optimizer step of train_loop (tinylm.c:2630-2633) on the device:
 * norm -> clip scale (max_norm; the reference hard-codes 1.0) -> AdamW.
 * norm_dev (device, may be NULL) receives the pre-clip norm. */
int tl_clip_adamw_step(float *P, const float *G, float *M, float *V, size_t n,
                       float lr, float b1, float b2, float wd, int t,
                       float max_norm, float *norm_dev);

/* ------------------------------------------------ device training step */
/* The reference's whole step -- forward (tinylm.c:968-1029), backward
 * (1072-1154, MTP heads 1036-1069), norm, clip, AdamW (2628-2633) -- on the
 * device, for dense configurations (no MoE, no QK-norm; T <= 256, head_dim <=
 * 64).  P/G/M/V use the reference's flat layout (map_weights, 361-393).
 * cfg8 = {V, D, L, H, KV, F, T, n_mtp}.  Activations are allocated once, for
 * `micro_batch` sequences; a batch B (a multiple of it) runs as consecutive
 * micro-batches accumulating into G, every logits gradient scaled by 1/(B*T).
 * Token arrays are device int32: tok/tgt [B*T], tgt_mtp [n_mtp][B*T]. */
int tl_model_create(const int *cfg8, int micro_batch, void **handle);
size_t tl_model_nparams(void *handle);
int tl_model_destroy(void *handle);
/* param_count (tinylm.c:345-358) of a dense configuration (0 if invalid). */
size_t tl_model_param_count(const int *cfg8);
/* init_params (tinylm.c:395-419) into a HOST buffer of tl_model_param_count
 * floats, reference generator seeded as TINYLM_SEED does (tinylm.c:4809-4811).
 * rng_out (may be NULL) gets the generator state after the draws, where the
 * reference's batch sampling continues.  Host only (no GPU needed). */
int tl_model_init_params(const int *cfg8, float *P_host, unsigned long long seed, unsigned long long *rng_out);
/* Loss only (mean cross-entropy, as forward() returns). */
int tl_model_forward(void *handle, const float *P, const int *tok, const int *tgt, int B, float *loss_dev);
/* G += gradients of the batch; loss_dev (may be NULL) = mean loss. */
int tl_model_forward_backward(void *handle, const float *P, float *G, const int *tok, const int *tgt,
                              const int *tgt_mtp, int B, float *loss_dev);
/* memset(G) -> forward/backward -> norm -> clip(max_norm) -> AdamW(lr, 0.9,
 * 0.95, 0.1, t): one step of train_loop / cmd_bench (tinylm.c:2627-2633). */
int tl_model_step(void *handle, float *P, float *G, float *M, float *V, const int *tok, const int *tgt,
                  const int *tgt_mtp, int B, float lr, int t, float max_norm, float *loss_dev, float *norm_dev);
/* tl_model_step as one CUDA graph: captured on the first call (and again when
 * a buffer, B or max_norm changes) and replayed with a single launch; lr and
 * the bias corrections of step t are copied to the device before each replay.
 * Same results as tl_model_step, bit for bit.  The buffers must stay where
 * they were at capture. */
/* Attention engine (forward and backward), for tests and benchmarks:
 * 0 = automatic (tensor cores -- tcgen05, 3xTF32 -- where T = 256 and
 * head_dim = 64, else CUDA cores), 1 = CUDA cores only, 2 = tensor cores
 * only for the forward (TL_EINVAL from the model calls when the shape does
 * not allow it; the backward follows the automatic choice). */
int tl_set_attn_engine(int engine);
int tl_model_graph_step(void *handle, float *P, float *G, float *M, float *V, const int *tok, const int *tgt,
                        const int *tgt_mtp, int B, float lr, int t, float max_norm, float *loss_dev,
                        float *norm_dev);
/* The data-parallel step (after tl_dist_init): this rank's batch of B
 * sequences through forward/backward, the ZeRO-1 update of tl_zero1_step on
 * the padded buffers (P, G: n_pad floats; M_shard, V_shard: this rank's shard;
 * n_pad = tl_zero1_padded(nparams, world)), with the gradient reduction
 * overlapped with the backward pass: each rank's shard of G is reduced
 * (average) onto its owner as soon as the backward has finished every
 * gradient inside it.  Same result as tl_model_forward_backward +
 * tl_zero1_step (bit for bit at 2 ranks).  loss_dev is this rank's own
 * mean loss. */
int tl_model_step_zero1(void *handle, float *P, float *G, float *M_shard, float *V_shard, const int *tok,
                        const int *tgt, const int *tgt_mtp, int B, float lr, int t, float max_norm,
                        float *loss_dev, float *norm_dev);

/* ------------------------------------- training loop: host-side pieces */
/* Checkpoints in the reference's formats.  Buffers may be host or device
 * memory (device data is staged through the host).
 * TLM4 bundle, model_save_bundle (tinylm.c:1895-1914): hdr11 =
 * {V,D,L,H,KV,F,T,eot,tmpl,n_mtp,n_exp}, then n fp32 parameters, then the
 * tokenizer blob. */
int tl_ckpt_save_bundle(const char *path, const int *hdr11, const float *P, size_t n, const void *tok_blob,
                        int tok_len);
/* model_load (tinylm.c:1915-1938) for TLM1-TLM4: header into hdr11 (missing
 * fields 0); when P is not NULL, n_expected parameters into P (TL_EINVAL if
 * the file is shorter).  *n_in_file (may be NULL) = 4-byte words after the
 * header (parameters + tokenizer length + tokenizer blob): an upper bound on
 * the parameter count, not the count. */
int tl_ckpt_load_bundle(const char *path, int *hdr11, float *P, size_t n_expected, size_t *n_in_file);
/* TOPT sidecar, opt_save / opt_load (tinylm.c:2526-2539): "TOPT", iter, M[n],
 * V[n].  Create the file once, then write / read any range of M and V -- each
 * ZeRO-1 rank stores and restores its own shard, no gather needed. */
int tl_ckpt_opt_create(const char *path, int iter, size_t n);
int tl_ckpt_opt_write(const char *path, size_t n, size_t offset, const float *M, const float *V, size_t count);
int tl_ckpt_opt_read(const char *path, size_t n, size_t offset, float *M, float *V, size_t count, int *iter_out);
/* LR at iteration it: linear warm-up, then cosine to 0.1*lr (train_loop,
 * tinylm.c:2587-2590). */
float tl_lr_at(int it, float lr, int iters, float warmup);
/* B windows of a uint16 token stream drawn with the reference's generator
 * (*rng is advanced): training (val=0, tinylm.c:2623-2626) or validation
 * batches (val=1, 2596-2597).  Outputs are host int32 arrays: tok/tgt [B*T],
 * tgt_mtp [n_mtp][B*T] (training only). */
int tl_sample_windows(unsigned long long *rng, const unsigned short *stream, size_t n, int B, int T, int n_mtp,
                      int val, int *tok, int *tgt, int *tgt_mtp);

/* ------------------------------------------- data parallel + ZeRO-1 (NCCL) */
/* No counterpart in the reference (it has no distributed code); this is the
 * multi-GPU form of the optimizer step above.
 *
 * Shard layout: the flat buffer of n floats is padded to n_pad, a multiple of
 * world*4096 (TL_ZERO1_ALIGN); rank r owns [r*n_pad/world, (r+1)*n_pad/world).
 * Buffers given to tl_zero1_step hold n_pad floats for P and G (the pad is kept
 * zero) and n_pad/world floats for M and V (this rank's shard). */
#define TL_ZERO1_ALIGN 4096
size_t tl_zero1_padded(size_t n, int world);
/* 128-byte NCCL unique id; rank 0 creates it and the caller ships it to the
 * other ranks (e.g. over torch.distributed or a file). */
int tl_dist_unique_id(void *uid128);
/* Blocking communicator set-up for this process's current device, bounded by
 * TL_DIST_INIT_TIMEOUT_MS (default 120000, never below TL_DIST_TIMEOUT_MS);
 * TL_ETIMEOUT when a rank never joins. */
int tl_dist_init(int rank, int world, const void *uid128);
int tl_dist_finalize(void);
/* One ZeRO-1 optimizer step over the padded flat buffers:
 *   ReduceScatter(G, avg) -> shard sum of squares -> AllReduce(sum) -> clip ->
 *   AdamW on this rank's shard of P/M/V -> AllGather(P).
 * Averaging, not summing, because each rank's loss is its local mean
 * (tinylm.c:1079 scales dlogits by 1/N_local).  G's own shard is overwritten
 * with the averaged gradient; the rest of G is left as is. */
int tl_zero1_step(float *P, float *G, float *M_shard, float *V_shard, size_t n,
                  float lr, float b1, float b2, float wd, int t, float max_norm,
                  float *norm_dev);
/* The same ZeRO-1 step with the exchanges done by this library's kernels over
 * peer memory (one node, every GPU reachable over NVLink) instead of NCCL
 * collectives: the averaged gradient of this rank's shard is summed straight
 * from every rank's G (rank order 0..R-1) fused with the shard's sum of
 * squares; shard sums are exchanged through peer stores; AdamW on the shard
 * stores the updated parameters into every rank's P.  Same results as
 * tl_zero1_step (bit for bit at R = 2; at larger R the gradient sums may
 * differ in the last bit, rank order here against NCCL's algorithm order).
 * Before the first step every rank
 * registers its own P and G (n_pad floats each, 16-byte aligned, cudaMalloc
 * memory that CUDA IPC can share) -- a collective call; tl_zero1_step_p2p must
 * then be given exactly those buffers.  Device waits are bounded by
 * TL_DIST_TIMEOUT_MS: on expiry the step records an error that
 * tl_device_status() returns as TL_ETIMEOUT, and from then on no kernel of
 * this or any later step touches peer memory (each later step records the
 * error again); once tl_device_status has reported it, tl_zero1_step_p2p
 * returns TL_ETIMEOUT without launching until tl_zero1_p2p_release and a new
 * tl_zero1_p2p_register.  Up to 8 ranks.  No counterpart in the reference. */
int tl_zero1_p2p_register(float *P, float *G, size_t n);
int tl_zero1_step_p2p(float *P, float *G, float *M_shard, float *V_shard, size_t n,
                      float lr, float b1, float b2, float wd, int t, float max_norm,
                      float *norm_dev);
/* Unmap the peers' buffers (after every rank's last step has completed). */
int tl_zero1_p2p_release(void);
/* Plain collectives on the library communicator (fp32, in place / out of place). */
int tl_dist_allreduce_f32(float *buf, size_t count, int average);
int tl_dist_allreduce_f64(double *buf, size_t count);
/* Wait for the library stream with a host-side deadline (timeout_ms <= 0: the
 * TL_DIST_TIMEOUT_MS environment value, default 120000).  A communicator error
 * or an expired deadline aborts the communicator and returns TL_ENCCL /
 * TL_ETIMEOUT instead of hanging. */
int tl_dist_sync(int timeout_ms);

#ifdef __cplusplus
}
#endif
#endif /* TINYLM_CUDA_H */
