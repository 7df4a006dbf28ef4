// tl_model_kernels.cu -- device versions of the non-GEMM ops of tinylm-c's
// training step (forward tinylm.c:968-1029, backward 1072-1154, mtp_grad
// 1036-1069), all fp32.
//
// Embedding gather/scatter, RMSNorm fwd/bwd (eps 1e-5, 539-588), RoPE fwd and
// transpose (608-651), causal GQA attention fwd/bwd (698-783), SwiGLU fwd/bwd
// (1005-1006, 1105-1112), softmax + cross-entropy fused with the logits
// gradient (1019-1028 with 1076-1082; MTP heads 1050-1057), residual adds.
// Reductions that feed parameters (RMSNorm gains) and the loss use a fixed
// order, so they do not depend on scheduling.
#include "tl_model.cuh"
#include "tl_trace.cuh"

namespace tl {
namespace mk {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float siluf(float z) { return z / (1.0f + expf(-z)); }

// ------------------------------------------------------------- embedding
// a_in[n, :] = emb[tok[n], :]   (tinylm.c:971-976)
__global__ void embed_fwd_kernel(const float *__restrict__ emb, const int *__restrict__ tok,
                                 float *__restrict__ out, int N, int D, int V, int *err) {
  const int n = blockIdx.x;
  if (n >= N) return;
  int t = tok[n];
  if (t < 0 || t >= V) {  // out-of-range token: record and use row 0
    if (threadIdx.x == 0) atomicExch(err, 100);
    t = 0;
  }
  const float *src = emb + (size_t)t * D;
  float *dst = out + (size_t)n * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) dst[d] = src[d];
}

// dEmb[tok[n], :] += dout[n, :]   (tinylm.c:1148-1153)
// gemb[v] += dout[n] for every n with tok[n] == v, in increasing n, starting
// from the gradient already in gemb: the reference's single-threaded scatter
// order (tinylm.c:1148-1153), so the result is deterministic and the same
// bits as that loop (no atomics).  One warp per vocabulary row scans the
// batch's tokens 32 at a time (ballot) and adds the matching rows; columns go
// in chunks of 32*EMB_CHUNK so the sums stay in registers (one scan of the
// tokens per row up to D = 1024).  Rows of tokens outside [0, V) are never
// added (embed_fwd reports them).
constexpr int EMB_CHUNK = 32;
__global__ void __launch_bounds__(256)
embed_bwd_kernel(float *__restrict__ gemb, const int *__restrict__ tok, const float *__restrict__ dout, int N,
                 int D, int V) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int v = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; v < V; v += nwarps) {
    float *row = gemb + (size_t)v * D;
    for (int c0 = 0; c0 < D; c0 += 32 * EMB_CHUNK) {
      float acc[EMB_CHUNK];
      bool any = false;
      for (int base = 0; base < N; base += 32) {
        const int n = base + lane;
        const int t = n < N ? __ldg(tok + n) : -1;
        unsigned mask = __ballot_sync(0xffffffffu, t == v);
        if (mask && !any) {
#pragma unroll
          for (int e = 0; e < EMB_CHUNK; e++) {
            const int d = c0 + e * 32 + lane;
            acc[e] = d < D ? row[d] : 0.0f;
          }
          any = true;
        }
        while (mask) {
          const int j = __ffs(mask) - 1;
          mask &= mask - 1;
          const float *src = dout + (size_t)(base + j) * D;
#pragma unroll
          for (int e = 0; e < EMB_CHUNK; e++) {
            const int d = c0 + e * 32 + lane;
            if (d < D) acc[e] += src[d];
          }
        }
      }
      if (any) {
#pragma unroll
        for (int e = 0; e < EMB_CHUNK; e++) {
          const int d = c0 + e * 32 + lane;
          if (d < D) row[d] = acc[e];
        }
      }
    }
  }
}

// The same sums without scanning every token per vocabulary row: the
// positions of each row's tokens are gathered first.  cnt[v] counts the
// tokens equal to v (atomic counts: order-free), off[v] is their exclusive
// prefix sum, cur[v] a cursor from off[v] that places each position into
// list (in any order), and each bucket is then written to sorted in
// increasing position order (a position's rank is the number of smaller
// ones in its bucket; positions are distinct).  The sum over a row then runs
// over its bucket in that order: the same bits as embed_bwd_kernel.
__global__ void emb_count_kernel(const int *__restrict__ tok, int N, int V, int *__restrict__ cnt) {
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    const int t = tok[n];
    if (t >= 0 && t < V) atomicAdd(cnt + t, 1);
  }
}

// One block of 1024 threads: each takes a contiguous run of entries.
__global__ void __launch_bounds__(1024)
emb_scan_kernel(const int *__restrict__ cnt, int V, int *__restrict__ off, int *__restrict__ cur) {
  __shared__ int wsum[32];
  const int per = (V + 1023) / 1024, v0 = threadIdx.x * per, v1 = min(V, v0 + per);
  int s = 0;
  for (int v = v0; v < v1; v++) s += cnt[v];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = s;                                 // inclusive scan over the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    int y = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int z = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) y += z;
    }
    wsum[lane] = y;                          // inclusive over warps
  }
  __syncthreads();
  int run = x - s + (w > 0 ? wsum[w - 1] : 0);   // exclusive start of this thread's run
  for (int v = v0; v < v1; v++) {
    off[v] = run;
    cur[v] = run;
    run += cnt[v];
  }
}

__global__ void emb_place_kernel(const int *__restrict__ tok, int N, int V, int *__restrict__ cur,
                                 int *__restrict__ list) {
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    const int t = tok[n];
    if (t >= 0 && t < V) list[atomicAdd(cur + t, 1)] = n;
  }
}

__global__ void __launch_bounds__(256)
embed_bwd_sorted_kernel(float *__restrict__ gemb, const float *__restrict__ dout, const int *__restrict__ cnt,
                        const int *__restrict__ off, const int *__restrict__ list, int *__restrict__ sorted, int D,
                        int V) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int v = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; v < V; v += nwarps) {
    const int c = cnt[v];
    if (c == 0) continue;
    const int o = off[v];
    for (int i = lane; i < c; i += 32) {
      const int x = list[o + i];
      int r = 0;
      for (int j = 0; j < c; j++) r += list[o + j] < x ? 1 : 0;
      sorted[o + r] = x;
    }
    __syncwarp();
    float *row = gemb + (size_t)v * D;
    for (int c0 = 0; c0 < D; c0 += 32 * EMB_CHUNK) {
      float acc[EMB_CHUNK];
#pragma unroll
      for (int e = 0; e < EMB_CHUNK; e++) {
        const int d = c0 + e * 32 + lane;
        acc[e] = d < D ? row[d] : 0.0f;
      }
      for (int i = 0; i < c; i++) {
        const float *src = dout + (size_t)sorted[o + i] * D;
#pragma unroll
        for (int e = 0; e < EMB_CHUNK; e++) {
          const int d = c0 + e * 32 + lane;
          if (d < D) acc[e] += src[d];
        }
      }
#pragma unroll
      for (int e = 0; e < EMB_CHUNK; e++) {
        const int d = c0 + e * 32 + lane;
        if (d < D) row[d] = acc[e];
      }
    }
  }
}

// ---------------------------------------------------------------- RMSNorm
// out = x * s * g, s = 1/sqrt(mean(x^2) + 1e-5); one warp per row.  (539-566)
__global__ void rmsnorm_fwd_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                   float *__restrict__ out, float *__restrict__ rinv, int rows, int D) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *xr = x + (size_t)warp * D;
  float ms = 0.0f;
  for (int i = lane; i < D; i += 32) ms += xr[i] * xr[i];
  ms = warp_sum_f(ms);
  const float s = 1.0f / sqrtf(ms / D + 1e-5f);
  if (lane == 0) rinv[warp] = s;
  float *orow = out + (size_t)warp * D;
  for (int i = lane; i < D; i += 32) orow[i] = xr[i] * s * g[i];
}

// The same with the row held in registers: D = 128 * NV, float4 loads, x read
// once (one warp per row).
template <int NV>
__global__ void __launch_bounds__(256)
rmsnorm_fwd_reg_kernel(const float4 *__restrict__ x, const float4 *__restrict__ g, float4 *__restrict__ out,
                       float *__restrict__ rinv, int rows) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  constexpr int D = 128 * NV;
  const float4 *xr = x + (size_t)warp * (D / 4);
  float4 v[NV];
  float ms = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; k++) {
    v[k] = __ldg(xr + k * 32 + lane);
    ms += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
  }
  ms = warp_sum_f(ms);
  const float s = 1.0f / sqrtf(ms / D + 1e-5f);
  if (lane == 0) rinv[warp] = s;
  float4 *orow = out + (size_t)warp * (D / 4);
#pragma unroll
  for (int k = 0; k < NV; k++) {
    const float4 gg = __ldg(g + k * 32 + lane);
    orow[k * 32 + lane] = make_float4(v[k].x * s * gg.x, v[k].y * s * gg.y, v[k].z * s * gg.z, v[k].w * s * gg.w);
  }
}

// dx += s*g*dy - (s^3/D * sum(x*g*dy)) * x ; per-block partial of dg = sum_rows x*s*dy.
// (tinylm.c:568-588; the per-thread buffers + critical section become a fixed-
// order two-stage reduction.)  Block b handles rows b*8+w, stepping gridDim*8.
// dx = dres + (RMSNorm backward of dy); dres may be dx itself (accumulate) or
// nullptr (dx overwritten).
__global__ void rmsnorm_bwd_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                   const float *__restrict__ rinv, const float *__restrict__ dy,
                                   const float *dres, float *dx, float *__restrict__ dg_part, int rows, int D) {
  extern __shared__ float sm[];  // [8][D]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) sm[i] = 0.0f;
  __syncthreads();
  float *my = sm + w * D;
  for (int r = blockIdx.x * 8 + w; r < rows; r += gridDim.x * 8) {
    const float *xr = x + (size_t)r * D, *dyr = dy + (size_t)r * D;
    float *dxr = dx + (size_t)r * D;
    const float *drr = dres ? dres + (size_t)r * D : nullptr;
    const float s = rinv[r];
    float c = 0.0f;
    for (int i = lane; i < D; i += 32) c += xr[i] * g[i] * dyr[i];
    c = warp_sum_f(c);
    const float coef = s * s * s / D * c;
    for (int i = lane; i < D; i += 32) {
      const float t = s * g[i] * dyr[i] - coef * xr[i];
      dxr[i] = drr ? drr[i] + t : t;
      my[i] += (xr[i] * s) * dyr[i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float acc = 0.0f;
#pragma unroll
    for (int ww = 0; ww < 8; ww++) acc += sm[ww * D + i];
    dg_part[(size_t)blockIdx.x * D + i] = acc;
  }
}

// The same with float4 accesses (D % 4 == 0, 16-byte aligned rows).
__global__ void rmsnorm_bwd4_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                    const float *__restrict__ rinv, const float *__restrict__ dy,
                                    const float *dres, float *dx, float *__restrict__ dg_part, int rows, int D) {
  extern __shared__ float sm[];  // [8][D]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) sm[i] = 0.0f;
  __syncthreads();
  float4 *my = reinterpret_cast<float4 *>(sm + w * D);
  const int nv = D / 4;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  for (int r = blockIdx.x * 8 + w; r < rows; r += gridDim.x * 8) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * D);
    const float4 *dyr = reinterpret_cast<const float4 *>(dy + (size_t)r * D);
    float4 *dxr = reinterpret_cast<float4 *>(dx + (size_t)r * D);
    const float4 *drr = dres ? reinterpret_cast<const float4 *>(dres + (size_t)r * D) : nullptr;
    const float s = rinv[r];
    float c = 0.0f;
    for (int v = lane; v < nv; v += 32) {
      const float4 a = xr[v], b = __ldg(g4 + v), d = dyr[v];
      c += a.x * b.x * d.x + a.y * b.y * d.y + a.z * b.z * d.z + a.w * b.w * d.w;
    }
    c = warp_sum_f(c);
    const float coef = s * s * s / D * c;
    for (int v = lane; v < nv; v += 32) {
      const float4 a = xr[v], b = __ldg(g4 + v), d = dyr[v];
      float4 t;
      t.x = s * b.x * d.x - coef * a.x; t.y = s * b.y * d.y - coef * a.y;
      t.z = s * b.z * d.z - coef * a.z; t.w = s * b.w * d.w - coef * a.w;
      if (drr) {
        const float4 o = drr[v];
        t.x = o.x + t.x; t.y = o.y + t.y; t.z = o.z + t.z; t.w = o.w + t.w;
      }
      dxr[v] = t;
      float4 m = my[v];
      m.x += (a.x * s) * d.x; m.y += (a.y * s) * d.y; m.z += (a.z * s) * d.z; m.w += (a.w * s) * d.w;
      my[v] = m;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float acc = 0.0f;
#pragma unroll
    for (int ww = 0; ww < 8; ww++) acc += sm[ww * D + i];
    dg_part[(size_t)blockIdx.x * D + i] = acc;
  }
}

// dg[i] += sum over blocks of dg_part[b][i].  Block per 32 columns, lane =
// column (coalesced rows); warp w sums parts w, w+8, ... and the eight warp
// sums are added in warp order: a fixed order, so the result is deterministic.
__global__ void __launch_bounds__(256)
colsum_add_kernel(const float *__restrict__ part, int nparts, int D, float *__restrict__ dg) {
  __shared__ float ws[8][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 32 + lane;
  float acc = 0.0f;
  if (i < D)
    for (int b = w; b < nparts; b += 8) acc += part[(size_t)b * D + i];
  ws[w][lane] = acc;
  __syncthreads();
  if (w == 0 && i < D) {
    float t = ws[0][lane];
#pragma unroll
    for (int k = 1; k < 8; k++) t += ws[k][lane];
    dg[i] += t;
  }
}

// The gain gradient's column sums in two fixed-order levels: block (cx, cy)
// sums partial rows [cy * per, (cy + 1) * per) of columns cx * 32 .. + 31
// into tmp[cy]; colsum_final_kernel adds the COLSUM_SPLIT sums in cy order
// into dg.  (The one-level kernel above runs only D / 32 blocks.)
constexpr int COLSUM_SPLIT = 8;
__global__ void __launch_bounds__(256)
colsum_split_kernel(const float *__restrict__ part, int nparts, int D, float *__restrict__ tmp) {
  __shared__ float ws[8][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 32 + lane;
  const int per = (nparts + COLSUM_SPLIT - 1) / COLSUM_SPLIT;
  const int r0 = blockIdx.y * per, r1 = min(nparts, r0 + per);
  float acc = 0.0f;
  if (i < D)
    for (int b = r0 + w; b < r1; b += 8) acc += part[(size_t)b * D + i];
  ws[w][lane] = acc;
  __syncthreads();
  if (w == 0 && i < D) {
    float t = ws[0][lane];
#pragma unroll
    for (int k = 1; k < 8; k++) t += ws[k][lane];
    tmp[(size_t)blockIdx.y * D + i] = t;
  }
}
__global__ void colsum_final_kernel(const float *__restrict__ tmp, int D, float *__restrict__ dg) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= D) return;
  float t = tmp[i];
#pragma unroll
  for (int k = 1; k < COLSUM_SPLIT; k++) t += tmp[(size_t)k * D + i];
  dg[i] += t;
}

// ------------------------------------------------------------------- RoPE
// buf[rows][nh*hd]; position of row r = r % T.  back=1 applies the transpose.
__global__ void rope_kernel(float *__restrict__ buf, const float *__restrict__ cosT, const float *__restrict__ sinT,
                            int rows, int nh, int hd, int T, int back) {
  const int half = hd / 2;
  const size_t total = (size_t)rows * nh * half;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const size_t rh = idx / half;
    const int h = (int)(rh % nh);
    const int r = (int)(rh / nh);
    const int t = r % T;
    float *v = buf + (size_t)r * nh * hd + (size_t)h * hd;
    const float c = cosT[t * half + i], s = sinT[t * half + i];
    const float a = v[i], b = v[i + half];
    if (!back) { v[i] = a * c - b * s; v[i + half] = b * c + a * s; }
    else       { v[i] = a * c + b * s; v[i + half] = -a * s + b * c; }
  }
}

// The same, four rotation pairs (i..i+3 with i+half..i+half+3) per thread,
// for half % 4 == 0.
__global__ void rope4_kernel(float *__restrict__ buf, const float *__restrict__ cosT, const float *__restrict__ sinT,
                             int rows, int nh, int hd, int T, int back) {
  const int half = hd / 2, q4 = half / 4;
  const size_t total = (size_t)rows * nh * q4;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % q4) * 4;
    const size_t rh = idx / q4;
    const int t = (int)((rh / nh) % T);
    float *v = buf + rh * hd;
    const float4 c = *reinterpret_cast<const float4 *>(cosT + (size_t)t * half + i);
    const float4 sn = *reinterpret_cast<const float4 *>(sinT + (size_t)t * half + i);
    const float4 a = *reinterpret_cast<const float4 *>(v + i), b = *reinterpret_cast<const float4 *>(v + i + half);
    float4 oa, ob;
    if (!back) {
      oa.x = a.x * c.x - b.x * sn.x; ob.x = b.x * c.x + a.x * sn.x;
      oa.y = a.y * c.y - b.y * sn.y; ob.y = b.y * c.y + a.y * sn.y;
      oa.z = a.z * c.z - b.z * sn.z; ob.z = b.z * c.z + a.z * sn.z;
      oa.w = a.w * c.w - b.w * sn.w; ob.w = b.w * c.w + a.w * sn.w;
    } else {
      oa.x = a.x * c.x + b.x * sn.x; ob.x = -a.x * sn.x + b.x * c.x;
      oa.y = a.y * c.y + b.y * sn.y; ob.y = -a.y * sn.y + b.y * c.y;
      oa.z = a.z * c.z + b.z * sn.z; ob.z = -a.z * sn.z + b.z * c.z;
      oa.w = a.w * c.w + b.w * sn.w; ob.w = -a.w * sn.w + b.w * c.w;
    }
    *reinterpret_cast<float4 *>(v + i) = oa;
    *reinterpret_cast<float4 *>(v + i + half) = ob;
  }
}

// --------------------------------------------------------------- elementwise
// The element-wise kernels below run a float4 body over the first n & ~3
// elements (all buffers are 256-byte aligned arena slices) and a scalar tail.
__global__ void add_inplace_kernel(float *__restrict__ y, const float *__restrict__ x, size_t n) {
  const size_t n4 = n / 4, stride = (size_t)gridDim.x * blockDim.x;
  float4 *y4 = reinterpret_cast<float4 *>(y);
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 a = y4[i];
    const float4 b = __ldcs(x4 + i);
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    y4[i] = a;
  }
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) y[i] += x[i];
}
// act = silu(g) * u   (tinylm.c:1005-1006)
__global__ void swiglu_fwd_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                  float *__restrict__ act, size_t n) {
  const size_t n4 = n / 4, stride = (size_t)gridDim.x * blockDim.x;
  const float4 *g4 = reinterpret_cast<const float4 *>(g), *u4 = reinterpret_cast<const float4 *>(u);
  float4 *a4 = reinterpret_cast<float4 *>(act);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 z = __ldcs(g4 + i), v = __ldcs(u4 + i);
    a4[i] = make_float4(siluf(z.x) * v.x, siluf(z.y) * v.y, siluf(z.z) * v.z, siluf(z.w) * v.w);
  }
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    act[i] = siluf(g[i]) * u[i];
}
// dg = dact*u*dsilu(g), du = dact*silu(g)   (tinylm.c:1106-1112)
__device__ __forceinline__ void swiglu_bwd_elem(float z, float uu, float da, float &dg, float &du) {
  const float sig = 1.0f / (1.0f + expf(-z));
  const float silu = z * sig;
  const float dsilu = sig + z * sig * (1.0f - sig);
  dg = da * uu * dsilu;
  du = da * silu;
}
__global__ void swiglu_bwd_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                  const float *__restrict__ dact, float *__restrict__ dg,
                                  float *__restrict__ du, size_t n) {
  const size_t n4 = n / 4, stride = (size_t)gridDim.x * blockDim.x;
  const float4 *g4 = reinterpret_cast<const float4 *>(g), *u4 = reinterpret_cast<const float4 *>(u);
  const float4 *d4 = reinterpret_cast<const float4 *>(dact);
  float4 *dg4 = reinterpret_cast<float4 *>(dg), *du4 = reinterpret_cast<float4 *>(du);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 z = __ldcs(g4 + i), v = __ldcs(u4 + i), a = __ldcs(d4 + i);
    float4 og, ou;
    swiglu_bwd_elem(z.x, v.x, a.x, og.x, ou.x);
    swiglu_bwd_elem(z.y, v.y, a.y, og.y, ou.y);
    swiglu_bwd_elem(z.z, v.z, a.z, og.z, ou.z);
    swiglu_bwd_elem(z.w, v.w, a.w, og.w, ou.w);
    dg4[i] = og;
    du4[i] = ou;
  }
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    swiglu_bwd_elem(g[i], u[i], dact[i], dg[i], du[i]);
}
// hk = fn + silu(t1)   (tinylm.c:1046-1047)
__global__ void mtp_hk_kernel(const float *__restrict__ fn, const float *__restrict__ t1,
                              float *__restrict__ hk, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    hk[i] = fn[i] + siluf(t1[i]);
}
// dfn += dhk; dt1 = dhk * dsilu(t1)   (tinylm.c:1062-1065)
__global__ void mtp_bwd_kernel(const float *__restrict__ t1, const float *__restrict__ dhk,
                               float *__restrict__ dfn, float *__restrict__ dt1, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float z = t1[i];
    const float sig = 1.0f / (1.0f + expf(-z));
    dfn[i] += dhk[i];
    dt1[i] = dhk[i] * (sig + z * sig * (1.0f - sig));
  }
}

// ---------------------------------------------------- softmax + cross-entropy
// One block per row of V logits.  Writes the logits gradient in place:
//   d[i] = softmax(l)[i] * scale, d[tgt] -= scale
// and, when loss_rows is given, -log(p[tgt] + 1e-12) in double for the row.
// (forward 1019-1028 + backward 1076-1082; MTP heads 1050-1057)
__global__ void softmax_ce_kernel(float *__restrict__ logits, const int *__restrict__ tgt, int V, float scale,
                                  double *__restrict__ loss_rows) {
  __shared__ float red[32];
  __shared__ float bcast;
  const int n = blockIdx.x;
  float *l = logits + (size_t)n * V;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float mx = -1e30f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, l[i]);
  mx = warp_max_f(mx);
  if (lane == 0) red[w] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int i = 1; i < nw; i++) m = fmaxf(m, red[i]);
    bcast = m;
  }
  __syncthreads();
  mx = bcast;
  float sum = 0.0f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float e = expf(l[i] - mx);
    l[i] = e;
    sum += e;
  }
  sum = warp_sum_f(sum);
  __syncthreads();
  if (lane == 0) red[w] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    bcast = s;
  }
  __syncthreads();
  const float inv = 1.0f / bcast;
  const int t = tgt[n];
  if (threadIdx.x == 0 && loss_rows) {
    const float pt = (t >= 0 && t < V) ? l[t] * inv : 0.0f;
    loss_rows[n] = -log((double)pt + 1e-12);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += blockDim.x) l[i] = l[i] * inv * scale;
  __syncthreads();
  if (threadIdx.x == 0 && t >= 0 && t < V) l[t] -= scale;
}

// The same row operation with the row held in registers: NV4 float4 per
// thread, V = 1024 * NV4, so the row is read once and written once.  Per
// element the arithmetic is the kernel above's; the sums run over a fixed
// partition (thread, then warp, then the block's warps in order), so the
// result is deterministic.
template <int NV4>
__global__ void __launch_bounds__(256)
softmax_ce_reg_kernel(float *__restrict__ logits, const int *__restrict__ tgt, float scale,
                      double *__restrict__ loss_rows) {
  constexpr int V = 1024 * NV4;
  __shared__ float red[8];
  const int n = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float4 *l4 = reinterpret_cast<float4 *>(logits + (size_t)n * V);
  float4 x[NV4];
  float mx = -1e30f;
#pragma unroll
  for (int k = 0; k < NV4; k++) {
    x[k] = l4[threadIdx.x + 256 * k];
    mx = fmaxf(mx, fmaxf(fmaxf(x[k].x, x[k].y), fmaxf(x[k].z, x[k].w)));
  }
  mx = warp_max_f(mx);
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int i = 1; i < 8; i++) mx = fmaxf(mx, red[i]);
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < NV4; k++) {
    x[k].x = expf(x[k].x - mx); x[k].y = expf(x[k].y - mx);
    x[k].z = expf(x[k].z - mx); x[k].w = expf(x[k].w - mx);
    sum += x[k].x; sum += x[k].y; sum += x[k].z; sum += x[k].w;
  }
  sum = warp_sum_f(sum);
  __syncthreads();                       // every thread has read red[] as maxima
  if (lane == 0) red[w] = sum;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) tot += red[i];
  const float inv = 1.0f / tot;
  const int t = tgt[n];
  const int tq = (t >= 0 && t < V) ? t >> 2 : -1;    // the float4 holding the target
#pragma unroll
  for (int k = 0; k < NV4; k++) {
    const int q = threadIdx.x + 256 * k;
    float4 o;
    o.x = x[k].x * inv * scale; o.y = x[k].y * inv * scale;
    o.z = x[k].z * inv * scale; o.w = x[k].w * inv * scale;
    if (q == tq) {
      const int c = t & 3;
      const float e = c == 0 ? x[k].x : c == 1 ? x[k].y : c == 2 ? x[k].z : x[k].w;
      if (loss_rows) loss_rows[n] = -log((double)(e * inv) + 1e-12);
      if (c == 0) o.x -= scale; else if (c == 1) o.y -= scale; else if (c == 2) o.z -= scale; else o.w -= scale;
    }
    l4[q] = o;
  }
  if (loss_rows && threadIdx.x == 0 && tq < 0) loss_rows[n] = -log(1e-12);
}

// acc[0] += sum(loss_rows[0..N)) in index order (one block).
__global__ void loss_sum_kernel(const double *__restrict__ rows, int N, double *__restrict__ acc) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < N; i += blockDim.x) s += rows[i];
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    acc[0] += t;
  }
}
__global__ void loss_final_kernel(const double *__restrict__ acc, double denom, float *__restrict__ out) {
  *out = (float)(acc[0] / denom);
}

// ---------------------------------------------------------------- attention
// Causal GQA attention in 64x64 tiles, fp32 on the CUDA cores with register
// tiling (FlashAttention-style: online softmax forward, recomputed scores in
// the backward).  Layout as the reference: q/out [B*T][H*hd], k/v
// [B*T][KV*hd]; query head h reads kv head h / (H/KV); softmax of scale*q.k
// over keys s <= t (tinylm.c:698-783).  Requires T % 64 == 0, hd <= 64 and
// hd % 4 == 0; head dims below 64 are zero-padded in shared memory.
//
// 256 threads as a 16x16 grid; thread (ty, tx) owns rows ty*4..ty*4+3 and
// columns tx*4..tx*4+3 of every 64x64 tile.  A 16-thread row group lives in
// one half-warp, so row reductions are 4 xor-shuffles.
constexpr int AT = 64;        // tile edge
constexpr int ALD = 68;       // padded row stride of shared tiles (16-byte aligned)
constexpr int ATILE = AT * ALD;

// acc[i][j] += sum_k A^T[k][ty*4+i] * B[k][tx*4+j]   (A^T and B in shared memory)
__device__ __forceinline__ void mm64(float acc[4][4], const float *__restrict__ At, const float *__restrict__ Bm,
                                     int kd, int ty, int tx) {
#pragma unroll 8
  for (int k = 0; k < kd; k++) {
    const float4 a = *reinterpret_cast<const float4 *>(At + k * ALD + ty * 4);
    const float4 b = *reinterpret_cast<const float4 *>(Bm + k * ALD + tx * 4);
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}
// Two products sharing the k loop: acc1 += A1^T B1, acc2 += A2^T B2.
__device__ __forceinline__ void mm64x2(float c1[4][4], float c2[4][4], const float *__restrict__ A1,
                                       const float *__restrict__ B1, const float *__restrict__ A2,
                                       const float *__restrict__ B2, int kd, int ty, int tx) {
#pragma unroll 4
  for (int k = 0; k < kd; k++) {
    const float4 a = *reinterpret_cast<const float4 *>(A1 + k * ALD + ty * 4);
    const float4 b = *reinterpret_cast<const float4 *>(B1 + k * ALD + tx * 4);
    const float4 e = *reinterpret_cast<const float4 *>(A2 + k * ALD + ty * 4);
    const float4 f = *reinterpret_cast<const float4 *>(B2 + k * ALD + tx * 4);
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    const float ev[4] = {e.x, e.y, e.z, e.w}, fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        c1[i][j] = fmaf(av[i], bv[j], c1[i][j]);
        c2[i][j] = fmaf(ev[i], fv[j], c2[i][j]);
      }
  }
}
__device__ __forceinline__ void zero44(float a[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) a[i][j] = 0.0f;
}
// 64 rows x hd columns of a [rows][ld] global array (row r0, column c0) into
// shared memory, row-major (dst[r][c]) or transposed (dst[c][r]); columns
// hd..63 are zero.
__device__ __forceinline__ void load_tile(float *__restrict__ dst, const float *__restrict__ src, size_t ld,
                                          int hd, bool transpose) {
  const int nq = AT * (AT / 4);  // float4 slots of a 64x64 tile
  for (int idx = threadIdx.x; idx < nq; idx += blockDim.x) {
    const int r = idx / (AT / 4), c4 = (idx % (AT / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c4 < hd) v = *reinterpret_cast<const float4 *>(src + (size_t)r * ld + c4);
    if (!transpose) {
      *reinterpret_cast<float4 *>(dst + r * ALD + c4) = v;
    } else {
      dst[(c4 + 0) * ALD + r] = v.x; dst[(c4 + 1) * ALD + r] = v.y;
      dst[(c4 + 2) * ALD + r] = v.z; dst[(c4 + 3) * ALD + r] = v.w;
    }
  }
}
__device__ __forceinline__ float hsum16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float hmax16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Forward: CTA per (b, h, 64-row query tile); online softmax over key tiles
// 0..qt.  Writes out and the row log-sum-exp.
__global__ void __launch_bounds__(256)
attn_fwd_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                float *__restrict__ out, float *__restrict__ lse, int T, int H, int KV, int hd, float scale) {
  extern __shared__ float sm[];
  float *Qt = sm, *Kt = Qt + ATILE, *Vr = Kt + ATILE, *Pt = Vr + ATILE;
  const int nqt = T / AT;
  const int qt = blockIdx.x % nqt, bh = blockIdx.x / nqt, b = bh / H, h = bh % H, kvh = h / (H / KV);
  const int D = H * hd, KD = KV * hd;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const size_t qrow0 = (size_t)b * T + qt * AT;
  load_tile(Qt, q + qrow0 * D + (size_t)h * hd, D, hd, true);
  float m[4], l[4], o[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++) { m[i] = -1e30f; l[i] = 0.0f; }
  zero44(o);
  for (int kt = 0; kt <= qt; kt++) {
    const size_t krow0 = (size_t)b * T + kt * AT;
    __syncthreads();
    load_tile(Kt, k + krow0 * KD + (size_t)kvh * hd, KD, hd, true);
    load_tile(Vr, v + krow0 * KD + (size_t)kvh * hd, KD, hd, false);
    __syncthreads();
    float s[4][4];
    zero44(s);
    mm64(s, Qt, Kt, hd, ty, tx);
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qi = qt * AT + ty * 4 + i;
      float mx = m[i];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kj = kt * AT + tx * 4 + j;
        s[i][j] = (kj <= qi) ? s[i][j] * scale : -1e30f;
        mx = fmaxf(mx, s[i][j]);
      }
      mx = hmax16(mx);
      const float corr = expf(m[i] - mx);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int kj = kt * AT + tx * 4 + j;
        p[i][j] = (kj <= qi) ? expf(s[i][j] - mx) : 0.0f;
        rs += p[i][j];
      }
      rs = hsum16(rs);
      l[i] = l[i] * corr + rs;
#pragma unroll
      for (int j = 0; j < 4; j++) o[i][j] *= corr;
      m[i] = mx;
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) Pt[(tx * 4 + j) * ALD + ty * 4 + i] = p[i][j];
    __syncthreads();
    mm64(o, Pt, Vr, AT, ty, tx);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int r = ty * 4 + i;
    const float inv = 1.0f / l[i];
    float *orow = out + (qrow0 + r) * D + (size_t)h * hd;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int d = tx * 4 + j;
      if (d < hd) orow[d] = o[i][j] * inv;
    }
    if (tx == 0) lse[(size_t)bh * T + qt * AT + r] = m[i] + logf(l[i]);
  }
}

// Per-row D = dO . out (softmax backward identity sum_s p_s dp_s = dO . out).
__global__ void attn_rowdot_kernel(const float *__restrict__ dout, const float *__restrict__ out,
                                   float *__restrict__ Drow, int B, int T, int H, int hd) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int rows = B * H * T;
  if (warp >= rows) return;
  const int bh = warp / T, t = warp % T, b = bh / H, h = bh % H;
  const size_t o = ((size_t)b * T + t) * H * hd + (size_t)h * hd;
  float acc = 0.0f;
  // float2 per lane (hd % 4 == 0 and rows start at multiples of hd floats)
  for (int d = 2 * lane; d < hd; d += 64) {
    const float2 a = *reinterpret_cast<const float2 *>(dout + o + d);
    const float2 b = *reinterpret_cast<const float2 *>(out + o + d);
    acc += a.x * b.x + a.y * b.y;
  }
  acc = warp_sum_f(acc);
  if (lane == 0) Drow[warp] = acc;
}

// The same row dot for head_dim 64 and up to 16 heads: a warp per token row
// covers all H heads with float4 loads (16 lanes per head, two heads per
// 32-lane pass), all passes' loads issued before the reductions, so a warp
// has the whole row (2 x 4 KB at H = 16) in flight instead of 2 x 256 B.
__global__ void __launch_bounds__(256)
attn_rowdot64_kernel(const float4 *__restrict__ dout, const float4 *__restrict__ out, float *__restrict__ Drow,
                     int B, int T, int H) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= B * T) return;
  const int b = row / T, t = row % T;
  const int n4 = H * 16;                       // float4 per token row (<= 256)
  const size_t o = (size_t)row * n4;
  float part[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const int i = k * 32 + lane;
    part[k] = 0.0f;
    if (i < n4) {
      const float4 x = __ldg(dout + o + i), y = __ldg(out + o + i);
      part[k] = x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; k++) {
    float acc = part[k];
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    const int h = 2 * k + (lane >> 4);
    if ((lane & 15) == 0 && h < H) Drow[((size_t)b * H + h) * T + t] = acc;
  }
}

// Backward, key side: CTA per (b, kv head, key tile); loops over the group's
// query heads and the query tiles at or after the key tile:
//   S^T = K Q^T and dP^T = V dO^T in one k loop, P^T, dS^T as above,
//   dV += P^T dO, dK += dS^T Q.  Writes dk, dv (overwrite) and dS^T of every
//   causal tile pair to dsT[b][h][key][q] for the query-side product.
// P^T and dS^T reuse the shared tiles of Q^T and dO^T (no longer read once
// S^T and dP^T are in registers): six tiles, two CTAs per SM.
__global__ void __launch_bounds__(256, 2)
attn_bwd_dkdv_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                     const float *__restrict__ dout, const float *__restrict__ lse, const float *__restrict__ Drow,
                     float *__restrict__ dk, float *__restrict__ dv, float *__restrict__ dsT, int T, int H, int KV,
                     int hd, float scale) {
  extern __shared__ float sm[];
  float *Kt = sm, *Vt = Kt + ATILE, *Qt = Vt + ATILE, *Ot = Qt + ATILE, *Qr = Ot + ATILE, *Or = Qr + ATILE;
  float *Ps = Qt, *Ss = Ot;
  float *Ls = Or + ATILE, *Ds = Ls + AT;
  const int nkt = T / AT;
  const int kt = blockIdx.x % nkt, bk = blockIdx.x / nkt, b = bk / KV, kvh = bk % KV, grp = H / KV;
  const int D = H * hd, KD = KV * hd;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const size_t krow0 = (size_t)b * T + kt * AT;
  load_tile(Kt, k + krow0 * KD + (size_t)kvh * hd, KD, hd, true);
  load_tile(Vt, v + krow0 * KD + (size_t)kvh * hd, KD, hd, true);
  float gk[4][4], gv[4][4];
  zero44(gk);
  zero44(gv);
  for (int hh = 0; hh < grp; hh++) {
    const int h = kvh * grp + hh, bh = b * H + h;
    for (int qt = kt; qt < T / AT; qt++) {
      const size_t qrow0 = (size_t)b * T + qt * AT;
      __syncthreads();
      load_tile(Qt, q + qrow0 * D + (size_t)h * hd, D, hd, true);
      load_tile(Ot, dout + qrow0 * D + (size_t)h * hd, D, hd, true);
      load_tile(Qr, q + qrow0 * D + (size_t)h * hd, D, hd, false);
      load_tile(Or, dout + qrow0 * D + (size_t)h * hd, D, hd, false);
      if (tid < AT) {
        Ls[tid] = lse[(size_t)bh * T + qt * AT + tid];
        Ds[tid] = Drow[(size_t)bh * T + qt * AT + tid];
      }
      __syncthreads();
      float st[4][4], dpt[4][4];   // rows = keys (ty), cols = queries (tx)
      zero44(st);
      zero44(dpt);
      mm64x2(st, dpt, Kt, Qt, Vt, Ot, hd, ty, tx);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int kj = kt * AT + ty * 4 + i;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int qi = qt * AT + tx * 4 + j;
          const int ql = tx * 4 + j;
          const float pr = (kj <= qi) ? expf(st[i][j] * scale - Ls[ql]) : 0.0f;
          st[i][j] = pr;
          dpt[i][j] = pr * (dpt[i][j] - Ds[ql]) * scale;
        }
      }
      __syncthreads();             // every thread is done reading Q^T and dO^T
#pragma unroll
      for (int i = 0; i < 4; i++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          Ps[(tx * 4 + j) * ALD + ty * 4 + i] = st[i][j];
          Ss[(tx * 4 + j) * ALD + ty * 4 + i] = dpt[i][j];
        }
        float *row = dsT + ((size_t)bh * T + kt * AT + ty * 4 + i) * T + qt * AT + tx * 4;
        *reinterpret_cast<float4 *>(row) = make_float4(dpt[i][0], dpt[i][1], dpt[i][2], dpt[i][3]);
      }
      __syncthreads();
      mm64(gv, Ps, Or, AT, ty, tx);
      mm64(gk, Ss, Qr, AT, ty, tx);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const size_t o = (krow0 + ty * 4 + i) * KD + (size_t)kvh * hd;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int d = tx * 4 + j;
      if (d < hd) { dk[o + d] = gk[i][j]; dv[o + d] = gv[i][j]; }
    }
  }
}

// Backward, query side: CTA per (b, h, query tile); dQ = sum over key tiles
// 0..qt of dS (read back as dS^T[key][q] from the key-side kernel) times K.
// Key tiles and the k loop run in the same order as a recomputing kernel
// would, so dQ is the same to the bit.
__global__ void __launch_bounds__(256)
attn_bwd_dq_kernel(const float *__restrict__ k, const float *__restrict__ dsT, float *__restrict__ dq, int T,
                   int H, int KV, int hd) {
  extern __shared__ float sm[];
  float *St = sm, *Kr = St + ATILE;
  const int nqt = T / AT;
  const int qt = blockIdx.x % nqt, bh = blockIdx.x / nqt, b = bh / H, h = bh % H, kvh = h / (H / KV);
  const int D = H * hd, KD = KV * hd;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const size_t qrow0 = (size_t)b * T + qt * AT;
  float g[4][4];
  zero44(g);
  for (int kt = 0; kt <= qt; kt++) {
    const size_t krow0 = (size_t)b * T + kt * AT;
    __syncthreads();
    load_tile(St, dsT + ((size_t)bh * T + kt * AT) * T + qt * AT, T, AT, false);
    load_tile(Kr, k + krow0 * KD + (size_t)kvh * hd, KD, hd, false);
    __syncthreads();
    mm64(g, St, Kr, AT, ty, tx);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float *row = dq + (qrow0 + ty * 4 + i) * D + (size_t)h * hd;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int d = tx * 4 + j;
      if (d < hd) row[d] = g[i][j];
    }
  }
}

}  // namespace mk

// ------------------------------------------------------------ launchers
static inline unsigned grid_for(size_t n, int threads, int cap_waves_sm, int num_sms) {
  size_t b = (n + threads - 1) / threads;
  const size_t cap = (size_t)num_sms * cap_waves_sm;
  if (b > cap) b = cap;
  return (unsigned)(b ? b : 1);
}

size_t attn_smem_fwd() { return sizeof(float) * 4 * mk::ATILE; }
size_t attn_smem_dq() { return sizeof(float) * 2 * mk::ATILE; }
size_t attn_smem_dkdv() { return sizeof(float) * (6 * mk::ATILE + 2 * mk::AT); }

int attn_tc_prepare(DeviceCtx *c);

int mk_setup(int device) {
  static bool done[kMaxDevices] = {};
  if (done[device]) return TL_OK;
  {
    DeviceCtx *c = ctx();
    int rc = c ? attn_tc_prepare(c) : TL_OK;
    if (rc) return rc;
  }
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_fwd()));
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_dq()));
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_dkdv()));
  done[device] = true;
  return TL_OK;
}

#define MK_LAUNCH_CHECK() TL_TRY_CUDA(cudaGetLastError())

int k_embed_fwd(DeviceCtx *c, const float *emb, const int *tok, float *out, int N, int D, int V) {
  TraceScope ts(c, "k_embed_fwd");
  mk::embed_fwd_kernel<<<N, 128, 0, c->stream>>>(emb, tok, out, N, D, V, c->err_flag);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_embed_bwd(DeviceCtx *c, float *gemb, const int *tok, const float *dout, int N, int D, int V, int *scratch) {
  TraceScope ts(c, "k_embed_bwd");
  if (!scratch) {
    mk::embed_bwd_kernel<<<(unsigned)((V + 7) / 8), 256, 0, c->stream>>>(gemb, tok, dout, N, D, V);
    MK_LAUNCH_CHECK();
    return TL_OK;
  }
  if (N <= 0 || V <= 0) return TL_OK;   // no tokens: the gradient is unchanged
  // scratch: cnt[V], off[V], cur[V], list[N], sorted[N]
  int *cnt = scratch, *off = cnt + V, *cur = off + V, *list = cur + V, *sorted = list + N;
  const unsigned g = (unsigned)std::min((N + 255) / 256, 4 * c->num_sms);
  TL_TRY_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int) * V, c->stream));
  mk::emb_count_kernel<<<g, 256, 0, c->stream>>>(tok, N, V, cnt);
  mk::emb_scan_kernel<<<1, 1024, 0, c->stream>>>(cnt, V, off, cur);
  mk::emb_place_kernel<<<g, 256, 0, c->stream>>>(tok, N, V, cur, list);
  mk::embed_bwd_sorted_kernel<<<(unsigned)((V + 7) / 8), 256, 0, c->stream>>>(gemb, dout, cnt, off, list, sorted,
                                                                               D, V);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rmsnorm_fwd(DeviceCtx *c, const float *x, const float *g, float *out, float *rinv, int rows, int D) {
  TraceScope ts(c, "k_rmsnorm_fwd");
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) |
                    reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const float4 *x4 = reinterpret_cast<const float4 *>(x), *g4 = reinterpret_cast<const float4 *>(g);
  float4 *o4 = reinterpret_cast<float4 *>(out);
  if (al && D == 1024) mk::rmsnorm_fwd_reg_kernel<8><<<grid, 256, 0, c->stream>>>(x4, g4, o4, rinv, rows);
  else if (al && D == 512) mk::rmsnorm_fwd_reg_kernel<4><<<grid, 256, 0, c->stream>>>(x4, g4, o4, rinv, rows);
  else if (al && D == 256) mk::rmsnorm_fwd_reg_kernel<2><<<grid, 256, 0, c->stream>>>(x4, g4, o4, rinv, rows);
  else if (al && D == 128) mk::rmsnorm_fwd_reg_kernel<1><<<grid, 256, 0, c->stream>>>(x4, g4, o4, rinv, rows);
  else mk::rmsnorm_fwd_kernel<<<grid, 256, 0, c->stream>>>(x, g, out, rinv, rows, D);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rmsnorm_bwd(DeviceCtx *c, const float *x, const float *g, const float *rinv, const float *dy,
                  const float *dres, float *dx, float *dg, float *part, int part_rows, int rows, int D, float *tmp) {
  int nb = (rows + 7) / 8;
  if (nb > part_rows) nb = part_rows;
  const bool vec = D % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(dy) |
                     reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dres)) & 15) == 0;
  {
    TraceScope ts(c, "k_rmsnorm_bwd");
    if (vec)
      mk::rmsnorm_bwd4_kernel<<<nb, 256, sizeof(float) * 8 * D, c->stream>>>(x, g, rinv, dy, dres, dx, part, rows, D);
    else
      mk::rmsnorm_bwd_kernel<<<nb, 256, sizeof(float) * 8 * D, c->stream>>>(x, g, rinv, dy, dres, dx, part, rows, D);
    MK_LAUNCH_CHECK();
  }
  TraceScope ts(c, "k_colsum_add");
  if (tmp && nb >= 8 * mk::COLSUM_SPLIT) {
    mk::colsum_split_kernel<<<dim3((D + 31) / 32, mk::COLSUM_SPLIT), 256, 0, c->stream>>>(part, nb, D, tmp);
    MK_LAUNCH_CHECK();
    mk::colsum_final_kernel<<<(D + 255) / 256, 256, 0, c->stream>>>(tmp, D, dg);
  } else {
    mk::colsum_add_kernel<<<(D + 31) / 32, 256, 0, c->stream>>>(part, nb, D, dg);
  }
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rope(DeviceCtx *c, float *buf, const float *cosT, const float *sinT, int rows, int nh, int hd, int T, int back) {
  TraceScope ts(c, "k_rope");
  const int half = hd / 2;
  if (half % 4 == 0 && ((reinterpret_cast<uintptr_t>(buf) | reinterpret_cast<uintptr_t>(cosT) |
                         reinterpret_cast<uintptr_t>(sinT)) & 15) == 0) {
    const size_t n4 = (size_t)rows * nh * (half / 4);
    mk::rope4_kernel<<<grid_for(n4, 256, 16, c->num_sms), 256, 0, c->stream>>>(buf, cosT, sinT, rows, nh, hd, T, back);
    MK_LAUNCH_CHECK();
    return TL_OK;
  }
  const size_t n = (size_t)rows * nh * half;
  mk::rope_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(buf, cosT, sinT, rows, nh, hd, T, back);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_add(DeviceCtx *c, float *y, const float *x, size_t n) {
  TraceScope ts(c, "k_add");
  mk::add_inplace_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(y, x, n);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_swiglu_fwd(DeviceCtx *c, const float *g, const float *u, float *act, size_t n) {
  TraceScope ts(c, "k_swiglu_fwd");
  mk::swiglu_fwd_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(g, u, act, n);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_swiglu_bwd(DeviceCtx *c, const float *g, const float *u, const float *dact, float *dg, float *du, size_t n) {
  TraceScope ts(c, "k_swiglu_bwd");
  mk::swiglu_bwd_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(g, u, dact, dg, du, n);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_mtp_hk(DeviceCtx *c, const float *fn, const float *t1, float *hk, size_t n) {
  TraceScope ts(c, "k_mtp_hk");
  mk::mtp_hk_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(fn, t1, hk, n);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_mtp_bwd(DeviceCtx *c, const float *t1, const float *dhk, float *dfn, float *dt1, size_t n) {
  TraceScope ts(c, "k_mtp_bwd");
  mk::mtp_bwd_kernel<<<grid_for(n, 256, 16, c->num_sms), 256, 0, c->stream>>>(t1, dhk, dfn, dt1, n);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_softmax_ce(DeviceCtx *c, float *logits, const int *tgt, int N, int V, float scale, double *loss_rows) {
  TraceScope ts(c, "k_softmax_ce");
  const bool al = (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (al && V == 8192)
    mk::softmax_ce_reg_kernel<8><<<N, 256, 0, c->stream>>>(logits, tgt, scale, loss_rows);
  else if (al && V == 4096)
    mk::softmax_ce_reg_kernel<4><<<N, 256, 0, c->stream>>>(logits, tgt, scale, loss_rows);
  else if (al && V == 2048)
    mk::softmax_ce_reg_kernel<2><<<N, 256, 0, c->stream>>>(logits, tgt, scale, loss_rows);
  else
    mk::softmax_ce_kernel<<<N, 256, 0, c->stream>>>(logits, tgt, V, scale, loss_rows);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_loss_sum(DeviceCtx *c, const double *rows, int N, double *acc) {
  TraceScope ts(c, "k_loss_sum");
  mk::loss_sum_kernel<<<1, 1024, 0, c->stream>>>(rows, N, acc);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_loss_final(DeviceCtx *c, const double *acc, double denom, float *out) {
  TraceScope ts(c, "k_loss_final");
  mk::loss_final_kernel<<<1, 1, 0, c->stream>>>(acc, denom, out);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
bool attn_fwd_tc_supported(const float *q, const float *k, const float *v, int T, int hd, int H, int KV);
int attn_fwd_tc(DeviceCtx *c, const float *q, const float *k, const float *v, float *out, float *lse, int B, int T,
                int H, int KV, int hd);
bool attn_bwd_dq_tc_supported(const float *dsT, const float *k, const float *dq, int T, int hd, int H, int KV);
int attn_bwd_dq_tc(DeviceCtx *c, const float *dsT, const float *k, float *dq, int B, int H, int KV, const float *cosT,
                   const float *sinT);
bool attn_bwd_dkdv_tc_supported(const float *const *ptrs, int nptr, int T, int hd, int H, int KV);
int attn_bwd_dkdv_tc(DeviceCtx *c, const float *q, const float *k, const float *v, const float *dout,
                     const float *lse, const float *Drow, float *dsT, float *dk, float *dv, int B, int H, int KV,
                     const float *cosT, const float *sinT);
static thread_local int g_attn_engine = 0;   // 0 automatic, 1 CUDA cores, 2 tensor cores

int k_attn_fwd(DeviceCtx *c, const float *q, const float *k, const float *v, float *out, float *lse, int B, int T,
               int H, int KV, int hd) {
  if (g_attn_engine != 1 && attn_fwd_tc_supported(q, k, v, T, hd, H, KV))
    return attn_fwd_tc(c, q, k, v, out, lse, B, T, H, KV, hd);
  if (g_attn_engine == 2) return set_error(TL_EINVAL, "tensor-core attention needs T = 256 and head_dim 64");
  TraceScope ts(c, "k_attn_fwd");
  const float scale = 1.0f / sqrtf((float)hd);
  mk::attn_fwd_kernel<<<B * H * (T / mk::AT), 256, attn_smem_fwd(), c->stream>>>(q, k, v, out, lse, T, H, KV, hd,
                                                                                  scale);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_attn_bwd(DeviceCtx *c, const float *q, const float *k, const float *v, const float *out, const float *dout,
               const float *lse, float *Drow, float *dsT, float *dq, float *dk, float *dv, int B, int T, int H,
               int KV, int hd, const float *cosT, const float *sinT) {
  const float scale = 1.0f / sqrtf((float)hd);
  const int rows = B * H * T;
  {
    TraceScope ts(c, "k_attn_rowdot");
    if (hd == 64 && H <= 16 && ((reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(out)) & 15) == 0)
      mk::attn_rowdot64_kernel<<<(B * T + 7) / 8, 256, 0, c->stream>>>(
          reinterpret_cast<const float4 *>(dout), reinterpret_cast<const float4 *>(out), Drow, B, T, H);
    else
      mk::attn_rowdot_kernel<<<(rows + 7) / 8, 256, 0, c->stream>>>(dout, out, Drow, B, T, H, hd);
    MK_LAUNCH_CHECK();
  }
  // The tensor-core kernels apply RoPE's backward to dK / dQ as they store
  // them; after the CUDA-core kernels it is a separate pass.
  const float *ptrs[9] = {q, k, v, dout, lse, Drow, dsT, dk, dv};
  bool dk_rotated = false, dq_rotated = false;
  if (g_attn_engine != 1 && attn_bwd_dkdv_tc_supported(ptrs, 9, T, hd, H, KV)) {
    const int rc = attn_bwd_dkdv_tc(c, q, k, v, dout, lse, Drow, dsT, dk, dv, B, H, KV, cosT, sinT);
    if (rc) return rc;
    dk_rotated = true;
  } else {
    TraceScope ts(c, "k_attn_bwd_dkdv");
    mk::attn_bwd_dkdv_kernel<<<B * KV * (T / mk::AT), 256, attn_smem_dkdv(), c->stream>>>(
        q, k, v, dout, lse, Drow, dk, dv, dsT, T, H, KV, hd, scale);
    MK_LAUNCH_CHECK();
  }
  if (g_attn_engine != 1 && attn_bwd_dq_tc_supported(dsT, k, dq, T, hd, H, KV)) {
    const int rc = attn_bwd_dq_tc(c, dsT, k, dq, B, H, KV, cosT, sinT);
    if (rc) return rc;
    dq_rotated = true;
  } else {
    TraceScope ts(c, "k_attn_bwd_dq");
    mk::attn_bwd_dq_kernel<<<B * H * (T / mk::AT), 256, attn_smem_dq(), c->stream>>>(k, dsT, dq, T, H, KV, hd);
    MK_LAUNCH_CHECK();
  }
  int rc;
  if (!dq_rotated && (rc = k_rope(c, dq, cosT, sinT, B * T, H, hd, T, 1))) return rc;
  if (!dk_rotated && (rc = k_rope(c, dk, cosT, sinT, B * T, KV, hd, T, 1))) return rc;
  return TL_OK;
}

}  // namespace tl

TL_API int tl_set_attn_engine(int engine) {
  if (engine < 0 || engine > 2) return tl::set_error(TL_EINVAL, "engine must be 0, 1 or 2");
  tl::g_attn_engine = engine;
  return TL_OK;
}
