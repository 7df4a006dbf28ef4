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
__global__ void embed_bwd_kernel(float *__restrict__ gemb, const int *__restrict__ tok,
                                 const float *__restrict__ dout, int N, int D, int V) {
  const int n = blockIdx.x;
  if (n >= N) return;
  const int t = tok[n];
  if (t < 0 || t >= V) return;
  float *dst = gemb + (size_t)t * D;
  const float *src = dout + (size_t)n * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) atomicAdd(dst + d, src[d]);
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

// dx += s*g*dy - (s^3/D * sum(x*g*dy)) * x ; per-block partial of dg = sum_rows x*s*dy.
// (tinylm.c:568-588; the per-thread buffers + critical section become a fixed-
// order two-stage reduction.)  Block b handles rows b*8+w, stepping gridDim*8.
__global__ void rmsnorm_bwd_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                   const float *__restrict__ rinv, const float *__restrict__ dy,
                                   float *__restrict__ dx, float *__restrict__ dg_part, int rows, int D) {
  extern __shared__ float sm[];  // [8][D]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) sm[i] = 0.0f;
  __syncthreads();
  float *my = sm + w * D;
  for (int r = blockIdx.x * 8 + w; r < rows; r += gridDim.x * 8) {
    const float *xr = x + (size_t)r * D, *dyr = dy + (size_t)r * D;
    float *dxr = dx + (size_t)r * D;
    const float s = rinv[r];
    float c = 0.0f;
    for (int i = lane; i < D; i += 32) c += xr[i] * g[i] * dyr[i];
    c = warp_sum_f(c);
    const float coef = s * s * s / D * c;
    for (int i = lane; i < D; i += 32) {
      dxr[i] += s * g[i] * dyr[i] - coef * xr[i];
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

// dg[i] += sum over blocks of dg_part[b][i], in block order.
__global__ void colsum_add_kernel(const float *__restrict__ part, int nparts, int D, float *__restrict__ dg) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= D) return;
  float acc = 0.0f;
  for (int b = 0; b < nparts; b++) acc += part[(size_t)b * D + i];
  dg[i] += acc;
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

// --------------------------------------------------------------- elementwise
__global__ void add_inplace_kernel(float *__restrict__ y, const float *__restrict__ x, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] += x[i];
}
// act = silu(g) * u   (tinylm.c:1005-1006)
__global__ void swiglu_fwd_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                  float *__restrict__ act, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    act[i] = siluf(g[i]) * u[i];
}
// dg = dact*u*dsilu(g), du = dact*silu(g)   (tinylm.c:1106-1112)
__global__ void swiglu_bwd_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                  const float *__restrict__ dact, float *__restrict__ dg,
                                  float *__restrict__ du, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float z = g[i];
    const float sig = 1.0f / (1.0f + expf(-z));
    const float silu = z * sig;
    const float dsilu = sig + z * sig * (1.0f - sig);
    dg[i] = dact[i] * u[i] * dsilu;
    du[i] = dact[i] * silu;
  }
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
// Causal GQA attention, T <= ATT_TMAX, head_dim <= ATT_HDMAX.  Layout as the
// reference: q/out [B*T][H*hd], k/v [B*T][KV*hd]; query head h reads kv head
// h / (H/KV).  Softmax of scale*q.k over keys s <= t.

// Forward: one CTA per (b, h), 16 warps, a warp per query row (interleaved
// rows for causal balance).  K is held transposed in shared memory so lanes
// (over keys) read it without bank conflicts; V row-major for lanes over d.
// Also stores the row log-sum-exp for the backward pass.
__global__ void __launch_bounds__(512)
attn_fwd_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                float *__restrict__ out, float *__restrict__ lse, int T, int H, int KV, int hd, float scale) {
  extern __shared__ float sm[];
  const int TP = T + 1;
  float *Kt = sm;                     // [hd][T+1]
  float *Vs = Kt + hd * TP;           // [T][hd]
  float *qb = Vs + T * hd;            // [16][hd]
  float *pb = qb + 16 * hd;           // [16][T]
  const int bh = blockIdx.x, b = bh / H, h = bh % H, kvh = h / (H / KV);
  const int D = H * hd, KD = KV * hd;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int idx = threadIdx.x; idx < T * hd; idx += blockDim.x) {
    const int s = idx / hd, d = idx % hd;
    const size_t g = (size_t)(b * T + s) * KD + (size_t)kvh * hd + d;
    Kt[d * TP + s] = k[g];
    Vs[s * hd + d] = v[g];
  }
  __syncthreads();
  float *myq = qb + w * hd, *myp = pb + w * T;
  for (int t = w; t < T; t += 16) {
    const float *qr = q + (size_t)(b * T + t) * D + (size_t)h * hd;
    for (int d = lane; d < hd; d += 32) myq[d] = qr[d];
    __syncwarp();
    float mx = -1e30f;
    for (int s = lane; s <= t; s += 32) {
      float dot = 0.0f;
      for (int d = 0; d < hd; d++) dot += myq[d] * Kt[d * TP + s];
      dot *= scale;
      myp[s] = dot;
      mx = fmaxf(mx, dot);
    }
    mx = warp_max_f(mx);
    float sum = 0.0f;
    for (int s = lane; s <= t; s += 32) {
      const float e = expf(myp[s] - mx);
      myp[s] = e;
      sum += e;
    }
    sum = warp_sum_f(sum);
    const float inv = 1.0f / sum;
    if (lane == 0) lse[(size_t)bh * T + t] = mx + logf(sum);
    __syncwarp();
    float *orow = out + (size_t)(b * T + t) * D + (size_t)h * hd;
    for (int d = lane; d < hd; d += 32) {
      float acc = 0.0f;
      for (int s = 0; s <= t; s++) acc += (myp[s] * inv) * Vs[s * hd + d];
      orow[d] = acc;
    }
    __syncwarp();
  }
}

// Backward, query side: one CTA per (b, h), 8 warps, a warp per query row.
//   p = exp(scale q.k - lse), dp_s = dO.v_s, Drow = dO.out,
//   ds = p (dp - Drow) scale, dq = sum_s ds k_s.
// Writes dq (overwrite) and Drow for the key-side kernel.
__global__ void __launch_bounds__(256)
attn_bwd_dq_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                   const float *__restrict__ out, const float *__restrict__ dout, const float *__restrict__ lse,
                   float *__restrict__ dq, float *__restrict__ Drow, int T, int H, int KV, int hd, float scale) {
  extern __shared__ float sm[];
  const int TP = T + 1;
  float *Kt = sm;                 // [hd][T+1]
  float *Ks = Kt + hd * TP;       // [T][hd]
  float *Vt = Ks + T * hd;        // [hd][T+1]
  float *qb = Vt + hd * TP;       // [8][hd]
  float *ob = qb + 8 * hd;        // [8][hd]
  float *pb = ob + 8 * hd;        // [8][T]
  const int bh = blockIdx.x, b = bh / H, h = bh % H, kvh = h / (H / KV);
  const int D = H * hd, KD = KV * hd;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int idx = threadIdx.x; idx < T * hd; idx += blockDim.x) {
    const int s = idx / hd, d = idx % hd;
    const size_t g = (size_t)(b * T + s) * KD + (size_t)kvh * hd + d;
    const float kv = k[g];
    Kt[d * TP + s] = kv;
    Ks[s * hd + d] = kv;
    Vt[d * TP + s] = v[g];
  }
  __syncthreads();
  float *myq = qb + w * hd, *myo = ob + w * hd, *myp = pb + w * T;
  for (int t = w; t < T; t += 8) {
    const size_t ro = (size_t)(b * T + t) * D + (size_t)h * hd;
    float dd = 0.0f;
    for (int d = lane; d < hd; d += 32) {
      myq[d] = q[ro + d];
      const float g = dout[ro + d];
      myo[d] = g;
      dd += g * out[ro + d];
    }
    dd = warp_sum_f(dd);
    if (lane == 0) Drow[(size_t)bh * T + t] = dd;
    __syncwarp();
    const float L = lse[(size_t)bh * T + t];
    for (int s = lane; s <= t; s += 32) {
      float dot = 0.0f, dp = 0.0f;
      for (int d = 0; d < hd; d++) {
        dot += myq[d] * Kt[d * TP + s];
        dp += myo[d] * Vt[d * TP + s];
      }
      const float p = expf(dot * scale - L);
      myp[s] = p * (dp - dd) * scale;
    }
    __syncwarp();
    for (int d = lane; d < hd; d += 32) {
      float acc = 0.0f;
      for (int s = 0; s <= t; s++) acc += myp[s] * Ks[s * hd + d];
      dq[ro + d] = acc;
    }
    __syncwarp();
  }
}

// Backward, key side: one CTA per (b, kv head), 16 warps, a warp per key.
// Loops over the H/KV query heads of the group: Q and dO of the head are held
// transposed in shared memory (lanes over queries, then lanes over d).
//   dv_s += sum_{t>=s} p_ts dO_t,  dk_s += sum_{t>=s} ds_ts q_t.
// Writes dk, dv (overwrite).  Keys per warp: T/16 <= 16.
__global__ void __launch_bounds__(512)
attn_bwd_dkdv_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                     const float *__restrict__ dout, const float *__restrict__ lse, const float *__restrict__ Drow,
                     float *__restrict__ dk, float *__restrict__ dv, int T, int H, int KV, int hd, float scale) {
  extern __shared__ float sm[];
  const int TP = T + 1;
  float *Qt = sm;                 // [hd][T+1]
  float *Ot = Qt + hd * TP;       // [hd][T+1]  (dO transposed)
  float *Lh = Ot + hd * TP;       // [T]
  float *Dh = Lh + T;             // [T]
  float *kb = Dh + T;             // [16][hd]
  float *vb = kb + 16 * hd;       // [16][hd]
  float *pb = vb + 16 * hd;       // [16][T]
  float *sb = pb + 16 * T;        // [16][T]
  const int bk = blockIdx.x, b = bk / KV, kvh = bk % KV, grp = H / KV;
  const int D = H * hd, KD = KV * hd;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int KPW = ATT_TMAX / 16;  // keys per warp (max)
  float dka[KPW][2], dva[KPW][2];
#pragma unroll
  for (int j = 0; j < KPW; j++) { dka[j][0] = dka[j][1] = dva[j][0] = dva[j][1] = 0.0f; }
  float *myk = kb + w * hd, *myv = vb + w * hd, *myp = pb + w * T, *mys = sb + w * T;
  for (int hh = 0; hh < grp; hh++) {
    const int h = kvh * grp + hh;
    const int bh = b * H + h;
    __syncthreads();
    for (int idx = threadIdx.x; idx < T * hd; idx += blockDim.x) {
      const int t = idx / hd, d = idx % hd;
      const size_t g = (size_t)(b * T + t) * D + (size_t)h * hd + d;
      Qt[d * TP + t] = q[g];
      Ot[d * TP + t] = dout[g];
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      Lh[t] = lse[(size_t)bh * T + t];
      Dh[t] = Drow[(size_t)bh * T + t];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < KPW; j++) {
      const int s = w + 16 * j;
      if (s >= T) break;
      const size_t gk = (size_t)(b * T + s) * KD + (size_t)kvh * hd;
      for (int d = lane; d < hd; d += 32) { myk[d] = k[gk + d]; myv[d] = v[gk + d]; }
      __syncwarp();
      for (int t = s + lane; t < T; t += 32) {
        float dot = 0.0f, dp = 0.0f;
        for (int d = 0; d < hd; d++) {
          dot += Qt[d * TP + t] * myk[d];
          dp += Ot[d * TP + t] * myv[d];
        }
        const float p = expf(dot * scale - Lh[t]);
        myp[t] = p;
        mys[t] = p * (dp - Dh[t]) * scale;
      }
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const int d = lane + 32 * c;
        if (d < hd) {
          float av = 0.0f, ak = 0.0f;
          for (int t = s; t < T; t++) {
            av += myp[t] * Ot[d * TP + t];
            ak += mys[t] * Qt[d * TP + t];
          }
          dva[j][c] += av;
          dka[j][c] += ak;
        }
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int j = 0; j < KPW; j++) {
    const int s = w + 16 * j;
    if (s >= T) break;
    const size_t gk = (size_t)(b * T + s) * KD + (size_t)kvh * hd;
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const int d = lane + 32 * c;
      if (d < hd) { dk[gk + d] = dka[j][c]; dv[gk + d] = dva[j][c]; }
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

size_t attn_smem_fwd(int T, int hd) { return sizeof(float) * ((size_t)hd * (T + 1) + (size_t)T * hd + 16 * hd + 16 * T); }
size_t attn_smem_dq(int T, int hd) {
  return sizeof(float) * (2 * (size_t)hd * (T + 1) + (size_t)T * hd + 16 * hd + 8 * T);
}
size_t attn_smem_dkdv(int T, int hd) {
  return sizeof(float) * (2 * (size_t)hd * (T + 1) + 2 * T + 32 * hd + 32 * T);
}

int mk_setup(int device) {
  static bool done[kMaxDevices] = {};
  if (done[device]) return TL_OK;
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_fwd(ATT_TMAX, ATT_HDMAX)));
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_dq(ATT_TMAX, ATT_HDMAX)));
  TL_TRY_CUDA(cudaFuncSetAttribute(mk::attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)attn_smem_dkdv(ATT_TMAX, ATT_HDMAX)));
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
int k_embed_bwd(DeviceCtx *c, float *gemb, const int *tok, const float *dout, int N, int D, int V) {
  TraceScope ts(c, "k_embed_bwd");
  mk::embed_bwd_kernel<<<N, 128, 0, c->stream>>>(gemb, tok, dout, N, D, V);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rmsnorm_fwd(DeviceCtx *c, const float *x, const float *g, float *out, float *rinv, int rows, int D) {
  TraceScope ts(c, "k_rmsnorm_fwd");
  mk::rmsnorm_fwd_kernel<<<(rows + 7) / 8, 256, 0, c->stream>>>(x, g, out, rinv, rows, D);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rmsnorm_bwd(DeviceCtx *c, const float *x, const float *g, const float *rinv, const float *dy, float *dx,
                  float *dg, float *part, int part_rows, int rows, int D) {
  TraceScope ts(c, "k_rmsnorm_bwd");
  int nb = (rows + 7) / 8;
  if (nb > part_rows) nb = part_rows;
  mk::rmsnorm_bwd_kernel<<<nb, 256, sizeof(float) * 8 * D, c->stream>>>(x, g, rinv, dy, dx, part, rows, D);
  MK_LAUNCH_CHECK();
  mk::colsum_add_kernel<<<(D + 255) / 256, 256, 0, c->stream>>>(part, nb, D, dg);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_rope(DeviceCtx *c, float *buf, const float *cosT, const float *sinT, int rows, int nh, int hd, int T, int back) {
  TraceScope ts(c, "k_rope");
  const size_t n = (size_t)rows * nh * (hd / 2);
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
int k_attn_fwd(DeviceCtx *c, const float *q, const float *k, const float *v, float *out, float *lse, int B, int T,
               int H, int KV, int hd) {
  TraceScope ts(c, "k_attn_fwd");
  const float scale = 1.0f / sqrtf((float)hd);
  mk::attn_fwd_kernel<<<B * H, 512, attn_smem_fwd(T, hd), c->stream>>>(q, k, v, out, lse, T, H, KV, hd, scale);
  MK_LAUNCH_CHECK();
  return TL_OK;
}
int k_attn_bwd(DeviceCtx *c, const float *q, const float *k, const float *v, const float *out, const float *dout,
               const float *lse, float *Drow, float *dq, float *dk, float *dv, int B, int T, int H, int KV, int hd) {
  TraceScope ts(c, "k_attn_bwd");
  const float scale = 1.0f / sqrtf((float)hd);
  mk::attn_bwd_dq_kernel<<<B * H, 256, attn_smem_dq(T, hd), c->stream>>>(q, k, v, out, dout, lse, dq, Drow, T, H,
                                                                         KV, hd, scale);
  MK_LAUNCH_CHECK();
  mk::attn_bwd_dkdv_kernel<<<B * KV, 512, attn_smem_dkdv(T, hd), c->stream>>>(q, k, v, dout, lse, Drow, dk, dv, T,
                                                                             H, KV, hd, scale);
  MK_LAUNCH_CHECK();
  return TL_OK;
}

}  // namespace tl
