// tl_gemm.cu -- C-ABI entry points of the three GEMM primitives and engine choice.
#include "tl_gemm.cuh"

namespace tl {

// 0 auto, 1 CUDA-core, 2 tensor-core, 3 tensor-core pair (tf32 split),
// 4 tensor-core pair (fp16 split), 5 tensor-core pair (hybrid split)
static thread_local int g_engine_pref = 0;
static thread_local int g_engine_last = 0;
static thread_local int g_sustained = 0;   // open gemm_sustained_scope()s

void gemm_sustained_scope(bool enter) { g_sustained += enter ? 1 : -1; }

// The split the pair kernel gets: the forced engine's, else the hybrid inside
// a sustained scope and the tf32 split outside one.  In single calls at full
// clock the tf32 split is the faster (config-3 shapes); over a training step
// under the power cap the hybrid's bf16 MMAs draw less power and the step
// runs at a higher clock (config 5: 816.5 against 854.4 ms on one box).
static GemmSplit pair_split() {
  if (g_engine_pref == 4) return GemmSplit::F16;
  if (g_engine_pref == 5) return GemmSplit::HYB;
  if (g_engine_pref == 3) return GemmSplit::TF32;
  return g_sustained > 0 ? GemmSplit::HYB : GemmSplit::TF32;
}
static int engine_id(bool pair, GemmSplit split) {
  return !pair ? 2 : split == GemmSplit::F16 ? 4 : split == GemmSplit::HYB ? 5 : 3;
}

static int gemm_entry(GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
                      const char *names) {
  TL_REQUIRE_CTX(c);
  if (M < 0 || K < 0 || N < 0) return set_error(TL_EINVAL, "negative GEMM dimension (M=%d K=%d N=%d)", M, K, N);
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  if (I == 0 || J == 0) return TL_OK;
  int rc;
  if (c->host_buffers && (is_host_ptr(C) || (R > 0 && (is_host_ptr(A) || is_host_ptr(B)))))
    return host_gemm(c, op, C, A, B, M, K, N);
  if ((rc = check_device_ptr(C, "output"))) return rc;
  if (R > 0) {
    if ((rc = check_device_ptr(A, "first operand"))) return rc;
    if ((rc = check_device_ptr(B, "second operand"))) return rc;
  }
  (void)names;
  if (R == 0) {  // empty reduction: mm writes zeros, the accumulating forms do nothing
    g_engine_last = 1;
    if (op == GemmOp::NN) TL_TRY_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * (size_t)I * J, c->stream));
    return TL_OK;
  }
  return gemm_run(c, op, C, A, B, M, K, N);
}

}  // namespace tl

// Engine choice without argument checks, for callers inside the library that
// have validated their buffers once (the device training step).
int tl::gemm_run(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N) {
  return gemm_run_add(c, op, C, A, B, M, K, N, op == GemmOp::NN ? nullptr : C);
}

int tl::gemm_run_add(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
                     const float *add) {
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  if (I == 0 || J == 0) return TL_OK;
  if (R == 0) {
    const size_t bytes = sizeof(float) * (size_t)I * J;
    if (!add) TL_TRY_CUDA(cudaMemsetAsync(C, 0, bytes, c->stream));
    else if (add != C) TL_TRY_CUDA(cudaMemcpyAsync(C, add, bytes, cudaMemcpyDeviceToDevice, c->stream));
    return TL_OK;
  }
  const bool tc_ok = gemm_tc_supported(op, C, A, B, M, K, N);
  if (g_engine_pref >= 2 && !tc_ok)
    return set_error(TL_EINVAL, "tensor-core engine forced but shape/alignment unsupported (M=%d K=%d N=%d)", M, K, N);
  if (tc_ok && g_engine_pref != 1) {
    const bool pair = g_engine_pref >= 3 || (g_engine_pref == 0 && gemm_tc_prefer_pair(I, J, R));
    const GemmSplit split = pair ? pair_split() : GemmSplit::TF32;
    g_engine_last = engine_id(pair, split);
    return gemm_tc(c, op, C, A, B, M, K, N, pair, add, split);
  }
  g_engine_last = 1;
  return gemm_simt(c, op, C, A, B, M, K, N, add);
}

bool tl::gemm_try_rope(DeviceCtx *c, float *C, const float *A, const float *B, int M, int K, int N,
                       const GemmRope &rope, int *rc) {
  if (M <= 0 || K <= 0 || N <= 0 || N % 64 || rope.T <= 0 || g_engine_pref == 1 || g_engine_pref == 2) return false;
  if (((reinterpret_cast<uintptr_t>(rope.cosT) | reinterpret_cast<uintptr_t>(rope.sinT)) & 15) != 0) return false;
  if (!gemm_tc_supported(GemmOp::NN, C, A, B, M, K, N)) return false;
  if (g_engine_pref == 0 && !gemm_tc_prefer_pair(M, N, K)) return false;
  const GemmSplit split = pair_split();
  g_engine_last = engine_id(true, split);
  *rc = gemm_tc(c, GemmOp::NN, C, A, B, M, K, N, true, nullptr, split, &rope);
  return true;
}

int tl::gemm_run_nt_sum(DeviceCtx *c, float *C, int nprod, const float *const *A, const float *const *B,
                        const int *N, int M, int K) {
  bool fused = nprod >= 1 && nprod <= 3 && M > 0 && K > 0 && (g_engine_pref == 0 || g_engine_pref >= 3);
  for (int t = 0; fused && t < nprod; t++)
    fused = N[t] > 0 && gemm_tc_supported(GemmOp::NT, C, A[t], B[t], M, K, N[t]) &&
            (g_engine_pref >= 3 || gemm_tc_prefer_pair(M, K, N[t]));
  if (fused) {
    const GemmSplit split = pair_split();
    g_engine_last = engine_id(true, split);
    return gemm_tc_nt_sum(c, C, nprod, A, B, N, M, K, split);
  }
  for (int t = 0; t < nprod; t++) {
    const int rc = gemm_run_add(c, GemmOp::NT, C, A[t], B[t], M, K, N[t], t == 0 ? nullptr : C);
    if (rc) return rc;
  }
  return TL_OK;
}

using namespace tl;

TL_API int tl_matmul(float *Y, const float *X, const float *W, int M, int K, int N) {
  return gemm_entry(GemmOp::NN, Y, X, W, M, K, N, "Y,X,W");
}
TL_API int tl_matmul_bt(float *dX, const float *dY, const float *W, int M, int K, int N) {
  return gemm_entry(GemmOp::NT, dX, dY, W, M, K, N, "dX,dY,W");
}
TL_API int tl_matmul_at(float *dW, const float *X, const float *dY, int M, int K, int N) {
  return gemm_entry(GemmOp::TN, dW, X, dY, M, K, N, "dW,X,dY");
}
TL_API int tl_matmul_bt_sum(float *dX, int nprod, const float *const *dY, const float *const *W, const int *N, int M,
                            int K) {
  TL_REQUIRE_CTX(c);
  if (nprod < 1 || nprod > 3) return set_error(TL_EINVAL, "nprod must be 1, 2 or 3, not %d", nprod);
  if (!dY || !W || !N) return set_error(TL_EINVAL, "null operand array");
  if (M < 0 || K < 0) return set_error(TL_EINVAL, "negative GEMM dimension (M=%d K=%d)", M, K);
  for (int t = 0; t < nprod; t++)
    if (N[t] < 0) return set_error(TL_EINVAL, "negative GEMM dimension (N[%d]=%d)", t, N[t]);
  if (M == 0 || K == 0) return TL_OK;
  int rc;
  if ((rc = check_device_ptr(dX, "output"))) return rc;
  for (int t = 0; t < nprod; t++) {
    if (N[t] == 0) continue;
    if ((rc = check_device_ptr(dY[t], "first operand"))) return rc;
    if ((rc = check_device_ptr(W[t], "second operand"))) return rc;
  }
  // Products with an empty reduction add nothing.
  const float *As[3], *Bs[3];
  int Ns[3], n = 0;
  for (int t = 0; t < nprod; t++)
    if (N[t] > 0) { As[n] = dY[t]; Bs[n] = W[t]; Ns[n] = N[t]; n++; }
  if (n == 0) {
    g_engine_last = 1;
    TL_TRY_CUDA(cudaMemsetAsync(dX, 0, sizeof(float) * (size_t)M * K, c->stream));
    return TL_OK;
  }
  return gemm_run_nt_sum(c, dX, n, As, Bs, Ns, M, K);
}
TL_API int tl_set_gemm_engine(int engine) {
  if (engine < 0 || engine > 5) return set_error(TL_EINVAL, "engine must be 0, 1, 2, 3, 4 or 5");
  g_engine_pref = engine;
  return TL_OK;
}
TL_API int tl_last_gemm_engine(void) { return g_engine_last; }
