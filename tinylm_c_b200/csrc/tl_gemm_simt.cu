// tl_gemm_simt.cu -- CUDA-core fp32 GEMM for the three reference layouts.
//
// The engine for shapes the tensor-core path cannot take (row strides that are
// not a multiple of 16 bytes, e.g. the reference selftest's K=131), and the
// exact-fp32 yardstick the tensor-core engine is tested against.  Plain FFMA,
// fp32 accumulation, like the reference's portable kernels (tinylm.c:452-537).
//
// One generic form covers all three primitives:
//   C[i,j] (=|+=) sum_r A(i,r) * B(r,j)
//   mm     (tinylm.c:439):  I=M J=N R=K, A=X  (r contiguous),  B=W  (j contiguous)
//   mm_bt  (tinylm.c:480):  I=M J=K R=N, A=dY (r contiguous),  B=W^T(r contiguous)
//   mm_atb (tinylm.c:510):  I=K J=N R=M, A=X^T(i contiguous),  B=dY (j contiguous)
// and C = product + add (add: nullptr, C itself, or a residual).
#include "tl_common.cuh"
#include "tl_gemm.cuh"
#include "tl_trace.cuh"

namespace tl {

constexpr int SB_M = 128, SB_N = 128, SB_K = 16, S_THREADS = 256;

// A_RC: A(i,r) = A[i*lda + r] (reduction-contiguous) else A[r*lda + i].
// B_RC: B(r,j) = B[j*ldb + r] (reduction-contiguous) else B[r*ldb + j].
template <bool A_RC, bool B_RC>
__global__ void __launch_bounds__(S_THREADS)
gemm_simt_kernel(float *__restrict__ C, const float *__restrict__ A, const float *__restrict__ B,
                 int I, int J, int R, int lda, int ldb, int ldc, const float *__restrict__ add) {
  __shared__ float As[SB_K][SB_M + 4];
  __shared__ float Bs[SB_K][SB_N + 4];
  const int tid = threadIdx.x;
  const int i0 = blockIdx.y * SB_M, j0 = blockIdx.x * SB_N;
  const int ti = (tid / 16) * 8, tj = (tid % 16) * 8;
  float acc[8][8];
#pragma unroll
  for (int a = 0; a < 8; a++)
#pragma unroll
    for (int b = 0; b < 8; b++) acc[a][b] = 0.0f;

  for (int r0 = 0; r0 < R; r0 += SB_K) {
    // 2048 elements of each tile, 8 per thread, index order chosen so that
    // consecutive threads touch consecutive addresses.
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int idx = e * S_THREADS + tid;
      int ii, rr;
      if (A_RC) { rr = idx % SB_K; ii = idx / SB_K; } else { ii = idx % SB_M; rr = idx / SB_M; }
      const int gi = i0 + ii, gr = r0 + rr;
      float v = 0.0f;
      if (gi < I && gr < R) v = A_RC ? A[(size_t)gi * lda + gr] : A[(size_t)gr * lda + gi];
      As[rr][ii] = v;
      int jj;
      if (B_RC) { rr = idx % SB_K; jj = idx / SB_K; } else { jj = idx % SB_N; rr = idx / SB_N; }
      const int gj = j0 + jj;
      const int gr2 = r0 + rr;
      float w = 0.0f;
      if (gj < J && gr2 < R) w = B_RC ? B[(size_t)gj * ldb + gr2] : B[(size_t)gr2 * ldb + gj];
      Bs[rr][jj] = w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SB_K; k++) {
      float a[8], b[8];
#pragma unroll
      for (int x = 0; x < 8; x++) { a[x] = As[k][ti + x]; b[x] = Bs[k][tj + x]; }
#pragma unroll
      for (int x = 0; x < 8; x++)
#pragma unroll
        for (int y = 0; y < 8; y++) acc[x][y] = fmaf(a[x], b[y], acc[x][y]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 8; x++) {
    const int gi = i0 + ti + x;
    if (gi >= I) continue;
#pragma unroll
    for (int y = 0; y < 8; y++) {
      const int gj = j0 + tj + y;
      if (gj >= J) continue;
      const size_t o = (size_t)gi * ldc + gj;
      C[o] = add ? add[o] + acc[x][y] : acc[x][y];
    }
  }
}

int gemm_simt(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
              const float *add) {
  int I, J, R;
  gemm_dims(op, M, K, N, &I, &J, &R);
  if (I == 0 || J == 0) return TL_OK;
  dim3 grid((J + SB_N - 1) / SB_N, (I + SB_M - 1) / SB_M);
  if (grid.y > 65535) return set_error(TL_EINVAL, "GEMM too tall for the CUDA-core engine (%d rows)", I);
  TraceScope ts(c, "gemm_simt");
  switch (op) {
    case GemmOp::NN:  // mm: A=X[M,K] lda=K, B=W[K,N] ldb=N (j contiguous), C ldc=N
      gemm_simt_kernel<true, false><<<grid, S_THREADS, 0, c->stream>>>(C, A, B, I, J, R, K, N, N, add);
      break;
    case GemmOp::NT:  // mm_bt: A=dY[M,N] lda=N, B(r=n,j=k)=W[k*N+n] ldb=N, C ldc=K
      gemm_simt_kernel<true, true><<<grid, S_THREADS, 0, c->stream>>>(C, A, B, I, J, R, N, N, K, add);
      break;
    case GemmOp::TN:  // mm_atb: A(i=k,r=m)=X[m*K+k] lda=K, B=dY[M,N] ldb=N, C ldc=N
      gemm_simt_kernel<false, false><<<grid, S_THREADS, 0, c->stream>>>(C, A, B, I, J, R, K, N, N, add);
      break;
  }
  TL_TRY_CUDA(cudaGetLastError());
  return TL_OK;
}

}  // namespace tl
