// tl_gemm.cuh -- shared declarations of the GEMM engines.
#pragma once
#include "tl_common.cuh"

namespace tl {

// The three reference primitives as one C[I,J] (=|+=) sum_r A(i,r) B(r,j).
enum class GemmOp {
  NN,  // mm     (tinylm.c:439-478):  Y[M,N]  = X[M,K]   @ W[K,N]
  NT,  // mm_bt  (tinylm.c:480-508):  dX[M,K] += dY[M,N] @ W[K,N]^T
  TN,  // mm_atb (tinylm.c:510-537):  dW[K,N] += X[M,K]^T @ dY[M,N]
};

inline void gemm_dims(GemmOp op, int M, int K, int N, int *I, int *J, int *R) {
  switch (op) {
    case GemmOp::NN: *I = M; *J = N; *R = K; break;
    case GemmOp::NT: *I = M; *J = K; *R = N; break;
    case GemmOp::TN: *I = K; *J = N; *R = M; break;
  }
}

// The reference semantics: mm overwrites C, mm_bt / mm_atb accumulate into C.
int gemm_run(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N);
// C = op(A, B) + add, where add is nullptr (overwrite), C itself (accumulate)
// or another I x J array with C's row stride (a residual).  Each element is
// the fp32 sum of the rounded product and the addend, exactly what a GEMM
// followed by an element-wise add produces.
int gemm_run_add(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
                 const float *add);
int gemm_simt(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
              const float *add);
// Returns TL_EINVAL (without launching) when the shape or alignment is not
// supported by the tensor-core engine.
bool gemm_tc_supported(GemmOp op, const float *C, const float *A, const float *B, int M, int K, int N);
// Automatic choice between the two tensor-core kernels for an I x J output
// with reduction length R.
bool gemm_tc_prefer_pair(int I, int J, int R);
// Host-side set-up of every tensor-core kernel (before a CUDA graph capture).
int gemm_tc_prepare(DeviceCtx *c);
// RoPE applied to a product's rows in the pair kernel's epilogue: heads of 64
// columns, row i at sequence position i % T, tables [T][32].
struct GemmRope {
  const float *cosT, *sinT;
  int T;
};
// How the CTA-pair kernel splits each fp32 product: tf32 hi/lo (three tf32
// MMAs), scaled fp16 hi/lo (three fp16 MMAs, specialised warps), or the
// hybrid (one tf32 hi*hi MMA and the two cross terms as one bf16 chain).
enum class GemmSplit { TF32 = 0, F16 = 1, HYB = 2 };
// pair: the CTA-pair kernel (256 x 256 tiles over two SMs) instead of the
// one-CTA kernel (128 x 128 tiles); split (pair only): see GemmSplit; rope
// (pair only): RoPE on the output rows (no split-K then).
int gemm_tc(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N, bool pair,
            const float *add, GemmSplit split, const GemmRope *rope = nullptr);
// The automatic engine choice gives the pair kernel the hybrid split while a
// scope is open on this thread (the device training step's GEMMs: long runs
// under the power cap, where its bf16 MMAs let the clock rise), else the tf32
// split.  Scopes nest.
void gemm_sustained_scope(bool enter);
// C[M,N] = A[M,K] B[K,N] with RoPE on C's rows, in one pair-kernel launch;
// false (nothing launched) where the engine choice would not give the pair
// kernel this shape, or N is not whole heads of 64.
bool gemm_try_rope(DeviceCtx *c, float *C, const float *A, const float *B, int M, int K, int N, const GemmRope &rope,
                   int *rc);

// C[M,K] = sum over t < nprod (<= 3) of A_t[M,N_t] @ B_t[K,N_t]^T, one
// CTA-pair launch whose reduction walks the products' k-blocks in turn
// (overwrites C).
int gemm_tc_nt_sum(DeviceCtx *c, float *C, int nprod, const float *const *A, const float *const *B, const int *N,
                   int M, int K, GemmSplit split);
// The same sum through the engine choice: one launch when the pair kernel
// would take every product, else one NT GEMM per product accumulating in turn.
int gemm_run_nt_sum(DeviceCtx *c, float *C, int nprod, const float *const *A, const float *const *B, const int *N,
                    int M, int K);

}  // namespace tl
