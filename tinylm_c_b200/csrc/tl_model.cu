// tl_model.cu -- the whole training step of tinylm-c on the device.
//
// The reference runs forward (tinylm.c:968-1029), backward (1072-1154, MTP
// heads 1036-1069), the grad norm and AdamW on host buffers.  Here the same
// graph runs on the GPU over device-resident P/G/M/V: the GEMMs go through the
// library's tensor-core engine, everything else through tl_model_kernels.cu.
// The flat parameter layout is the reference's map_weights order (361-393), so
// P is byte-compatible with its checkpoints.
//
// Memory: activations are allocated once for a micro-batch of `mb` sequences.
// A larger local batch is processed as consecutive micro-batches whose
// gradients accumulate into G; every logits gradient is scaled by
// 1/(B*T) of the whole local batch, exactly the reference's 1/N (1079), so only
// the order of floating-point sums changes.
#include <cmath>
#include <cstring>
#include <vector>
#include "tl_gemm.cuh"
#include "tl_model.cuh"
#include "tl_dist.cuh"
#include "tl_trace.cuh"

namespace tl {
int launch_sumsq(DeviceCtx *c, const float *G, size_t n, double *sumsq_out, float *norm_out,
                 float *gscale_out, float max_norm);
int launch_adamw(DeviceCtx *c, float *P, const float *G, float *M, float *V, size_t n, float lr,
                 float b1, float b2, float wd, int t, float gscale, const float *gscale_dev,
                 const float *hyper = nullptr);

constexpr int RMS_PART_ROWS = 1184;

struct Model {
  int V, D, L, H, KV, F, T, n_mtp, hd, KD, half, mb, N;  // N = mb*T rows per micro-batch
  size_t np;
  size_t o_emb, o_nf;
  std::vector<size_t> o_an1, o_wq, o_wk, o_wv, o_wo, o_an2, o_w1, o_w3, o_w2, o_mtp;
  int device;
  void *arena = nullptr;
  float *rope_cos, *rope_sin;
  std::vector<float *> a_in, a_norm, rinv1, q, k, v, att, lse, f_in, f_norm, rinv2, g, u, act;
  float *x_final, *fn, *fn_rinv, *logits;
  float *dact, *dgb, *du, *dout, *dfnorm, *dfin, *datt, *dq, *dnorm, *dain, *dfn, *dk, *dv, *Drow, *dsT;
  float *t1, *hk, *dhk, *dt1;
  float *rms_part, *rms_tmp;   // gain-gradient partial rows and their middle level
  float *emb_idx;              // embedding backward: token positions by vocabulary row (ints)
  double *loss_rows, *loss_acc;
  // CUDA graph of one whole training step (tl_model_graph_step): the buffers
  // it was captured with, and the per-step scalars it reads on the device
  // (lr, AdamW bias corrections 1-b1^t, 1-b2^t).
  cudaGraphExec_t gexec = nullptr;
  cudaStream_t gstream = nullptr;
  float *hyper = nullptr;
  std::vector<uintptr_t> gkey;
};

// Offsets of every tensor in the flat buffer -- map_weights, tinylm.c:361-393
// (dense FFN, no QK-norm, no router: the configurations this path serves).
static void layout(Model &m) {
  size_t p = 0;
  m.o_emb = p; p += (size_t)m.V * m.D;
  for (int l = 0; l < m.L; l++) {
    m.o_an1.push_back(p); p += m.D;
    m.o_wq.push_back(p); p += (size_t)m.D * m.D;
    m.o_wk.push_back(p); p += (size_t)m.D * m.KD;
    m.o_wv.push_back(p); p += (size_t)m.D * m.KD;
    m.o_wo.push_back(p); p += (size_t)m.D * m.D;
    m.o_an2.push_back(p); p += m.D;
    m.o_w1.push_back(p); p += (size_t)m.D * m.F;
    m.o_w3.push_back(p); p += (size_t)m.D * m.F;
    m.o_w2.push_back(p); p += (size_t)m.F * m.D;
  }
  m.o_nf = p; p += m.D;
  for (int k = 0; k < m.n_mtp; k++) { m.o_mtp.push_back(p); p += (size_t)m.D * m.D; }
  m.np = p;
}

// The reference's generator (xorshift64 + Box-Muller, tinylm.c:127-134).
struct Rng {
  uint64_t s;
  uint64_t next() { uint64_t x = s; x ^= x << 13; x ^= x >> 7; x ^= x << 17; s = x; return x; }
  float uniform() { return (float)(next() >> 11) * (1.0f / 9007199254740992.0f); }
  float normal() {
    float u1 = uniform();
    if (u1 < 1e-9f) u1 = 1e-9f;
    const float u2 = uniform();
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
  }
};

#define TRY(x) do { int _rc = (x); if (_rc) return _rc; } while (0)

static int gemm(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N) {
  return gemm_run(c, op, C, A, B, M, K, N);
}
// C = A @ W, then RoPE on C's rows (nh heads): in the GEMM's epilogue where
// the pair kernel takes it (head_dim 64), else as a separate pass.
static int gemm_rope(DeviceCtx *c, const Model &m, float *C, const float *A, const float *W, int M, int K, int N,
                     int nh) {
  int rc = TL_OK;
  if (m.hd == 64 && gemm_try_rope(c, C, A, W, M, K, N, GemmRope{m.rope_cos, m.rope_sin, m.T}, &rc)) return rc;
  if ((rc = gemm_run(c, GemmOp::NN, C, A, W, M, K, N))) return rc;
  return k_rope(c, C, m.rope_cos, m.rope_sin, M, nh, m.hd, m.T, 0);
}
// C = op(A, B) + add (add: nullptr to overwrite, or a residual); replaces the
// reference's memset-then-accumulate and GEMM-then-add pairs with one pass.
static int gemm_add(DeviceCtx *c, GemmOp op, float *C, const float *A, const float *B, int M, int K, int N,
                    const float *add) {
  return gemm_run_add(c, op, C, A, B, M, K, N, add);
}

// One micro-batch: forward + backward, gradients accumulated into G.
// ov (data-parallel step only, last micro-batch): told after each layer which
// tail of G is final, so shard reductions start during the backward pass.
static int micro_step(DeviceCtx *c, Model &m, const float *P, float *G, const int *tok, const int *tgt,
                      const int *const *tgt_mtp, float scale, bool backward, OverlapState *ov = nullptr) {
  const int N = m.N, D = m.D, F = m.F, KD = m.KD, V = m.V;
  const size_t ND = (size_t)N * D, NF = (size_t)N * F;
  const float *emb = P + m.o_emb;
  // ---------------- forward (tinylm.c:968-1029)
  TRY(k_embed_fwd(c, emb, tok, m.a_in[0], N, D, V));
  for (int l = 0; l < m.L; l++) {
    float *xin = m.a_in[l];
    TRY(k_rmsnorm_fwd(c, xin, P + m.o_an1[l], m.a_norm[l], m.rinv1[l], N, D));
    // q and k with RoPE, v (tinylm.c:981-989)
    TRY(gemm_rope(c, m, m.q[l], m.a_norm[l], P + m.o_wq[l], N, D, D, m.H));
    TRY(gemm_rope(c, m, m.k[l], m.a_norm[l], P + m.o_wk[l], N, D, KD, m.KV));
    TRY(gemm(c, GemmOp::NN, m.v[l], m.a_norm[l], P + m.o_wv[l], N, D, KD));
    TRY(k_attn_fwd(c, m.q[l], m.k[l], m.v[l], m.att[l], m.lse[l], m.mb, m.T, m.H, m.KV, m.hd));
    TRY(gemm_add(c, GemmOp::NN, m.f_in[l], m.att[l], P + m.o_wo[l], N, D, D, xin));   // + residual
    TRY(k_rmsnorm_fwd(c, m.f_in[l], P + m.o_an2[l], m.f_norm[l], m.rinv2[l], N, D));
    float *out = (l + 1 < m.L) ? m.a_in[l + 1] : m.x_final;
    TRY(gemm(c, GemmOp::NN, m.g[l], m.f_norm[l], P + m.o_w1[l], N, D, F));
    TRY(gemm(c, GemmOp::NN, m.u[l], m.f_norm[l], P + m.o_w3[l], N, D, F));
    TRY(k_swiglu_fwd(c, m.g[l], m.u[l], m.act[l], NF));
    TRY(gemm_add(c, GemmOp::NN, out, m.act[l], P + m.o_w2[l], N, F, D, m.f_in[l]));   // + residual
  }
  TRY(k_rmsnorm_fwd(c, m.x_final, P + m.o_nf, m.fn, m.fn_rinv, N, D));
  // tied head: logits = fn @ emb^T  (memset + mm_bt, 1015-1016, as one overwrite)
  TRY(gemm_add(c, GemmOp::NT, m.logits, m.fn, emb, N, V, D, nullptr));
  // softmax + CE, logits gradient written in place (1019-1028, 1076-1082)
  TRY(k_softmax_ce(c, m.logits, tgt, N, V, scale, m.loss_rows));
  TRY(k_loss_sum(c, m.loss_rows, N, m.loss_acc));
  if (!backward) return TL_OK;

  // ---------------- backward (tinylm.c:1072-1154)
  float *gemb = G + m.o_emb;
  TRY(gemm(c, GemmOp::NN, m.dfn, m.logits, emb, N, V, D));       // dfn = dlogits @ emb
  TRY(gemm(c, GemmOp::TN, gemb, m.logits, m.fn, N, V, D));        // dEmb += dlogits^T @ fn
  // MTP heads (1036-1069): hk = fn + silu(fn@Wk), tied logits, weight 0.2*0.8^k
  for (int kh = 0; kh < m.n_mtp; kh++) {
    const float wk = 0.2f * powf(0.8f, (float)kh);
    const float *Wk = P + m.o_mtp[kh];
    TRY(gemm(c, GemmOp::NN, m.t1, m.fn, Wk, N, D, D));
    TRY(k_mtp_hk(c, m.fn, m.t1, m.hk, ND));
    TRY(gemm_add(c, GemmOp::NT, m.logits, m.hk, emb, N, V, D, nullptr));
    TRY(k_softmax_ce(c, m.logits, tgt_mtp[kh], N, V, wk * scale, nullptr));
    TRY(gemm(c, GemmOp::TN, gemb, m.logits, m.hk, N, V, D));       // dEmb += dl^T @ hk
    TRY(gemm(c, GemmOp::NN, m.dhk, m.logits, emb, N, V, D));       // dhk = dl @ emb
    TRY(k_mtp_bwd(c, m.t1, m.dhk, m.dfn, m.dt1, ND));              // dfn += dhk; dt1
    TRY(gemm(c, GemmOp::TN, G + m.o_mtp[kh], m.fn, m.dt1, N, D, D));
    TRY(gemm(c, GemmOp::NT, m.dfn, m.dt1, Wk, N, D, D));
  }
  TRY(k_rmsnorm_bwd(c, m.x_final, P + m.o_nf, m.fn_rinv, m.dfn, nullptr, m.dout, G + m.o_nf, m.rms_part,
                    RMS_PART_ROWS, N, D, m.rms_tmp));
  if (ov) TRY(overlap_ready(c, ov, m.o_nf));            // final norm and MTP heads are done
  for (int l = m.L - 1; l >= 0; l--) {
    // FFN
    TRY(gemm(c, GemmOp::TN, G + m.o_w2[l], m.act[l], m.dout, N, F, D));
    TRY(gemm_add(c, GemmOp::NT, m.dact, m.dout, P + m.o_w2[l], N, F, D, nullptr));
    TRY(k_swiglu_bwd(c, m.g[l], m.u[l], m.dact, m.dgb, m.du, NF));
    {  // dfnorm = dgb @ W1^T + du @ W3^T
      const float *As[2] = {m.dgb, m.du}, *Bs[2] = {P + m.o_w1[l], P + m.o_w3[l]};
      const int Ns[2] = {F, F};
      TRY(gemm_run_nt_sum(c, m.dfnorm, 2, As, Bs, Ns, N, D));
    }
    TRY(gemm(c, GemmOp::TN, G + m.o_w1[l], m.f_norm[l], m.dgb, N, D, F));
    TRY(gemm(c, GemmOp::TN, G + m.o_w3[l], m.f_norm[l], m.du, N, D, F));
    // dfin = dout + rmsnorm2 backward
    TRY(k_rmsnorm_bwd(c, m.f_in[l], P + m.o_an2[l], m.rinv2[l], m.dfnorm, m.dout, m.dfin, G + m.o_an2[l],
                      m.rms_part, RMS_PART_ROWS, N, D, m.rms_tmp));
    // attention output projection
    TRY(gemm_add(c, GemmOp::NT, m.datt, m.dfin, P + m.o_wo[l], N, D, D, nullptr));
    TRY(gemm(c, GemmOp::TN, G + m.o_wo[l], m.att[l], m.dfin, N, D, D));
    // attention and RoPE's backward (tinylm.c:1130-1133)
    TRY(k_attn_bwd(c, m.q[l], m.k[l], m.v[l], m.att[l], m.datt, m.lse[l], m.Drow, m.dsT, m.dq, m.dk, m.dv, m.mb, m.T, m.H,
                   m.KV, m.hd, m.rope_cos, m.rope_sin));
    {  // dnorm = dq @ Wq^T + dk @ Wk^T + dv @ Wv^T
      const float *As[3] = {m.dq, m.dk, m.dv}, *Bs[3] = {P + m.o_wq[l], P + m.o_wk[l], P + m.o_wv[l]};
      const int Ns[3] = {D, KD, KD};
      TRY(gemm_run_nt_sum(c, m.dnorm, 3, As, Bs, Ns, N, D));
    }
    TRY(gemm(c, GemmOp::TN, G + m.o_wq[l], m.a_norm[l], m.dq, N, D, D));
    TRY(gemm(c, GemmOp::TN, G + m.o_wk[l], m.a_norm[l], m.dk, N, D, KD));
    TRY(gemm(c, GemmOp::TN, G + m.o_wv[l], m.a_norm[l], m.dv, N, D, KD));
    // dain = dfin + rmsnorm1 backward; becomes the next layer's dout
    TRY(k_rmsnorm_bwd(c, m.a_in[l], P + m.o_an1[l], m.rinv1[l], m.dnorm, m.dfin, m.dain, G + m.o_an1[l],
                      m.rms_part, RMS_PART_ROWS, N, D, m.rms_tmp));
    std::swap(m.dout, m.dain);
    if (ov) TRY(overlap_ready(c, ov, m.o_an1[l]));       // layers l..L-1 are done
  }
  TRY(k_embed_bwd(c, gemb, tok, m.dout, N, D, V, reinterpret_cast<int *>(m.emb_idx)));
  return TL_OK;
}

// The step's GEMMs run as one long sequence under the power cap: the
// automatic engine choice gives them the hybrid split (gemm_sustained_scope).
struct SustainedGemms {
  SustainedGemms() { gemm_sustained_scope(true); }
  ~SustainedGemms() { gemm_sustained_scope(false); }
};

static int run_batch(DeviceCtx *c, Model &m, const float *P, float *G, const int *tok, const int *tgt,
                     const int *tgt_mtp, int B, float *loss_dev, bool backward, OverlapState *ov = nullptr) {
  SustainedGemms sustained;
  if (B < 1 || B % m.mb) return set_error(TL_EINVAL, "batch %d must be a positive multiple of the micro-batch %d", B, m.mb);
  const size_t Ntot = (size_t)B * m.T;
  const float scale = 1.0f / (float)Ntot;
  TL_TRY_CUDA(cudaMemsetAsync(m.loss_acc, 0, sizeof(double), c->stream));
  std::vector<const int *> mt(m.n_mtp > 0 ? m.n_mtp : 1, nullptr);
  for (int i = 0; i < B / m.mb; i++) {
    const size_t off = (size_t)i * m.N;
    for (int kh = 0; kh < m.n_mtp; kh++) mt[kh] = tgt_mtp + (size_t)kh * Ntot + off;
    TRY(micro_step(c, m, P, G, tok + off, tgt + off, mt.data(), scale, backward,
                   i == B / m.mb - 1 ? ov : nullptr));
  }
  if (loss_dev) TRY(k_loss_final(c, m.loss_acc, (double)Ntot, loss_dev));
  return TL_OK;
}

static int alloc_model(Model &m) {
  const size_t N = m.N, D = m.D, F = m.F, KD = m.KD, V = m.V, L = m.L;
  const size_t att_rows = (size_t)m.mb * m.H * m.T;
  size_t floats = 0;
  auto take = [&](size_t n) { size_t o = floats; floats += (n + 63) / 64 * 64; return o; };
  std::vector<std::pair<float **, size_t>> slots;
  m.a_in.resize(L); m.a_norm.resize(L); m.rinv1.resize(L); m.q.resize(L); m.k.resize(L); m.v.resize(L);
  m.att.resize(L); m.lse.resize(L); m.f_in.resize(L); m.f_norm.resize(L); m.rinv2.resize(L); m.g.resize(L);
  m.u.resize(L); m.act.resize(L);
  slots.push_back({&m.rope_cos, take((size_t)m.T * m.half)});
  slots.push_back({&m.rope_sin, take((size_t)m.T * m.half)});
  for (size_t l = 0; l < L; l++) {
    slots.push_back({&m.a_in[l], take(N * D)});
    slots.push_back({&m.a_norm[l], take(N * D)});
    slots.push_back({&m.rinv1[l], take(N)});
    slots.push_back({&m.q[l], take(N * D)});
    slots.push_back({&m.k[l], take(N * KD)});
    slots.push_back({&m.v[l], take(N * KD)});
    slots.push_back({&m.att[l], take(N * D)});
    slots.push_back({&m.lse[l], take(att_rows)});
    slots.push_back({&m.f_in[l], take(N * D)});
    slots.push_back({&m.f_norm[l], take(N * D)});
    slots.push_back({&m.rinv2[l], take(N)});
    slots.push_back({&m.g[l], take(N * F)});
    slots.push_back({&m.u[l], take(N * F)});
    slots.push_back({&m.act[l], take(N * F)});   // kept for the backward (no recompute)
  }
  for (float **p : {&m.x_final, &m.fn, &m.dout, &m.dfnorm, &m.dfin, &m.datt, &m.dq, &m.dnorm, &m.dain, &m.dfn,
                    &m.t1, &m.hk, &m.dhk, &m.dt1})
    slots.push_back({p, take(N * D)});
  slots.push_back({&m.fn_rinv, take(N)});
  slots.push_back({&m.logits, take(N * V)});
  for (float **p : {&m.dact, &m.dgb, &m.du}) slots.push_back({p, take(N * F)});
  slots.push_back({&m.dk, take(N * KD)});
  slots.push_back({&m.dv, take(N * KD)});
  slots.push_back({&m.Drow, take(att_rows)});
  slots.push_back({&m.dsT, take(att_rows * m.T)});
  slots.push_back({&m.rms_part, take((size_t)RMS_PART_ROWS * D)});
  slots.push_back({&m.rms_tmp, take(8 * D)});
  slots.push_back({&m.emb_idx, take(3 * (size_t)V + 2 * (size_t)N)});
  const size_t o_loss = take(2 * N + 2);  // doubles: N rows + accumulator
  TL_TRY_CUDA(cudaMalloc(&m.arena, floats * sizeof(float)));
  float *base = static_cast<float *>(m.arena);
  for (auto &s : slots) *s.first = base + s.second;
  // The attention backward writes dS^T only for key tiles at or below the
  // query tile; the rest is read as zeros by the tensor-core dQ product.
  TL_TRY_CUDA(cudaMemset(m.dsT, 0, sizeof(float) * att_rows * m.T));
  m.loss_rows = reinterpret_cast<double *>(base + o_loss);
  m.loss_acc = m.loss_rows + N;
  // RoPE table in fp32 exactly as rope_init (tinylm.c:613-623)
  std::vector<float> cs((size_t)m.T * m.half), sn((size_t)m.T * m.half);
  for (int t = 0; t < m.T; t++)
    for (int i = 0; i < m.half; i++) {
      const float inv = powf(10000.0f, -(2.0f * i) / m.hd);
      const float a = t * inv;
      cs[(size_t)t * m.half + i] = cosf(a);
      sn[(size_t)t * m.half + i] = sinf(a);
    }
  TL_TRY_CUDA(cudaMemcpy(m.rope_cos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
  TL_TRY_CUDA(cudaMemcpy(m.rope_sin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
  return TL_OK;
}

}  // namespace tl

using namespace tl;

static int cfg_model(const int *cfg8, Model &m);

TL_API int tl_model_create(const int *cfg8, int micro_batch, void **handle) {
  if (!handle || !cfg8) return set_error(TL_EINVAL, "NULL argument");
  *handle = nullptr;
  TL_REQUIRE_CTX(c);
  Model *m = new Model();
  int rc0 = cfg_model(cfg8, *m);
  if (rc0) {
    delete m;
    return rc0;
  }
  if (m->T > ATT_TMAX || m->T % 64 || m->hd > ATT_HDMAX || m->hd % 4) {
    delete m;
    return set_error(TL_EINVAL, "attention supports T <= %d (a multiple of 64) and head_dim <= %d (a multiple of 4)",
                     ATT_TMAX, ATT_HDMAX);
  }
  m->mb = micro_batch > 0 ? micro_batch : 1;
  m->N = m->mb * m->T;
  m->device = c->device;
  int rc = mk_setup(c->device);
  if (!rc) rc = alloc_model(*m);
  if (rc) {
    if (m->arena) cudaFree(m->arena);
    delete m;
    return rc;
  }
  *handle = m;
  return TL_OK;
}

TL_API size_t tl_model_nparams(void *h) { return h ? static_cast<Model *>(h)->np : 0; }

TL_API int tl_model_destroy(void *h) {
  Model *m = static_cast<Model *>(h);
  if (!m) return TL_OK;
  if (m->gexec) cudaGraphExecDestroy(m->gexec);
  if (m->gstream) cudaStreamDestroy(m->gstream);
  if (m->hyper) cudaFree(m->hyper);
  if (m->arena) cudaFree(m->arena);
  delete m;
  return TL_OK;
}

static int cfg_model(const int *cfg8, Model &m) {
  m.V = cfg8[0]; m.D = cfg8[1]; m.L = cfg8[2]; m.H = cfg8[3]; m.KV = cfg8[4]; m.F = cfg8[5];
  m.T = cfg8[6] > 0 ? cfg8[6] : 256; m.n_mtp = cfg8[7];
  if (m.V < 1 || m.D < 1 || m.L < 1 || m.H < 1 || m.KV < 1 || m.F < 1 || m.n_mtp < 0 || m.D % m.H || m.H % m.KV)
    return set_error(TL_EINVAL, "bad model configuration");
  m.hd = m.D / m.H; m.KD = m.KV * m.hd; m.half = m.hd / 2;
  layout(m);
  return TL_OK;
}

// param_count (tinylm.c:345-358) for a dense configuration.
TL_API size_t tl_model_param_count(const int *cfg8) {
  Model m;
  if (!cfg8 || cfg_model(cfg8, m)) return 0;
  return m.np;
}

// init_params (tinylm.c:395-419) into a host buffer of tl_model_param_count
// floats, with the reference generator seeded as TINYLM_SEED does (seed | 1).
// rng_out (may be NULL) receives the generator state after the draws, where
// train_loop's batch sampling continues.  Host only: needs no GPU.
TL_API int tl_model_init_params(const int *cfg8, float *P_host, unsigned long long seed, unsigned long long *rng_out) {
  if (!cfg8 || !P_host) return set_error(TL_EINVAL, "NULL argument");
  Model mm;
  int rc = cfg_model(cfg8, mm);
  if (rc) return rc;
  Model *m = &mm;
  Rng r{(uint64_t)seed | 1ULL};
  const size_t D = m->D, KD = m->KD, F = m->F;
  float *p = P_host;
  for (size_t i = 0; i < (size_t)m->V * D; i++) p[m->o_emb + i] = 0.02f * r.normal();
  const float scaled = 0.02f / sqrtf(2.0f * m->L);
  for (int l = 0; l < m->L; l++) {
    for (size_t i = 0; i < D; i++) { p[m->o_an1[l] + i] = 1.0f; p[m->o_an2[l] + i] = 1.0f; }
    for (size_t i = 0; i < D * D; i++) p[m->o_wq[l] + i] = 0.02f * r.normal();
    for (size_t i = 0; i < D * KD; i++) p[m->o_wk[l] + i] = 0.02f * r.normal();
    for (size_t i = 0; i < D * KD; i++) p[m->o_wv[l] + i] = 0.02f * r.normal();
    for (size_t i = 0; i < D * D; i++) p[m->o_wo[l] + i] = scaled * r.normal();
    for (size_t i = 0; i < D * F; i++) p[m->o_w1[l] + i] = 0.02f * r.normal();
    for (size_t i = 0; i < D * F; i++) p[m->o_w3[l] + i] = 0.02f * r.normal();
    for (size_t i = 0; i < F * D; i++) p[m->o_w2[l] + i] = scaled * r.normal();
  }
  for (size_t i = 0; i < D; i++) p[m->o_nf + i] = 1.0f;
  for (int k = 0; k < m->n_mtp; k++)
    for (size_t i = 0; i < D * D; i++) p[m->o_mtp[k] + i] = 0.0f;
  if (rng_out) *rng_out = r.s;  // the generator continues into batch sampling
  return TL_OK;
}

TL_API int tl_model_forward(void *h, const float *P, const int *tok, const int *tgt, int B, float *loss_dev) {
  Model *m = static_cast<Model *>(h);
  if (!m) return set_error(TL_EINVAL, "NULL model");
  TL_REQUIRE_CTX(c);
  if (c->device != m->device) return set_error(TL_EINVAL, "model belongs to device %d", m->device);
  return run_batch(c, *m, P, nullptr, tok, tgt, nullptr, B, loss_dev, false);
}

TL_API int tl_model_forward_backward(void *h, const float *P, float *G, const int *tok, const int *tgt,
                                     const int *tgt_mtp, int B, float *loss_dev) {
  Model *m = static_cast<Model *>(h);
  if (!m) return set_error(TL_EINVAL, "NULL model");
  TL_REQUIRE_CTX(c);
  if (c->device != m->device) return set_error(TL_EINVAL, "model belongs to device %d", m->device);
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) || (rc = check_device_ptr(tok, "tok")) ||
      (rc = check_device_ptr(tgt, "tgt")))
    return rc;
  if (m->n_mtp > 0 && (rc = check_device_ptr(tgt_mtp, "tgt_mtp"))) return rc;
  return run_batch(c, *m, P, G, tok, tgt, tgt_mtp, B, loss_dev, true);
}

TL_API int tl_model_step(void *h, float *P, float *G, float *M, float *V, const int *tok, const int *tgt,
                         const int *tgt_mtp, int B, float lr, int t, float max_norm, float *loss_dev,
                         float *norm_dev) {
  Model *m = static_cast<Model *>(h);
  if (!m) return set_error(TL_EINVAL, "NULL model");
  TL_REQUIRE_CTX(c);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  int rc;
  if ((rc = check_device_ptr(M, "M")) || (rc = check_device_ptr(V, "V"))) return rc;
  TL_TRY_CUDA(cudaMemsetAsync(G, 0, sizeof(float) * m->np, c->stream));       // memset(G) 2628
  if ((rc = tl_model_forward_backward(h, P, G, tok, tgt, tgt_mtp, B, loss_dev))) return rc;
  float *gscale = c->scalars + 1;                                              // 2630-2631
  if ((rc = launch_sumsq(c, G, m->np, c->sumsq, norm_dev, gscale, max_norm))) return rc;
  return launch_adamw(c, P, G, M, V, m->np, lr, 0.9f, 0.95f, 0.1f, t, 1.0f, gscale);  // 2633
}


// One training step as a CUDA graph: captured on the first call (and again
// whenever a buffer, the batch or max_norm changes), then replayed with one
// launch.  The step's learning rate and bias corrections (1 - b^t in fp32
// with powf, as the eager step computes them) are copied to the device before
// each replay, where the captured AdamW kernel reads them; everything else is
// identical to tl_model_step, to the bit.
TL_API int tl_model_graph_step(void *h, float *P, float *G, float *M, float *V, const int *tok, const int *tgt,
                               const int *tgt_mtp, int B, float lr, int t, float max_norm, float *loss_dev,
                               float *norm_dev) {
  Model *m = static_cast<Model *>(h);
  if (!m) return set_error(TL_EINVAL, "NULL model");
  TL_REQUIRE_CTX(c);
  if (c->device != m->device) return set_error(TL_EINVAL, "model belongs to device %d", m->device);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  if (B < 1 || B % m->mb) return set_error(TL_EINVAL, "batch %d must be a positive multiple of the micro-batch %d", B, m->mb);
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) || (rc = check_device_ptr(M, "M")) ||
      (rc = check_device_ptr(V, "V")) || (rc = check_device_ptr(tok, "tok")) || (rc = check_device_ptr(tgt, "tgt")))
    return rc;
  if (m->n_mtp > 0 && (rc = check_device_ptr(tgt_mtp, "tgt_mtp"))) return rc;
  if (!m->hyper) TL_TRY_CUDA(cudaMalloc(&m->hyper, 4 * sizeof(float)));
  if (!m->gstream) TL_TRY_CUDA(cudaStreamCreateWithFlags(&m->gstream, cudaStreamNonBlocking));
  uint32_t mn_bits;
  memcpy(&mn_bits, &max_norm, 4);
  const std::vector<uintptr_t> key = {(uintptr_t)P, (uintptr_t)G, (uintptr_t)M, (uintptr_t)V, (uintptr_t)tok,
                                      (uintptr_t)tgt, (uintptr_t)tgt_mtp, (uintptr_t)B, (uintptr_t)mn_bits,
                                      (uintptr_t)loss_dev, (uintptr_t)norm_dev};
  if (!m->gexec || key != m->gkey) {
    if (m->gexec) { cudaGraphExecDestroy(m->gexec); m->gexec = nullptr; }
    if ((rc = gemm_tc_prepare(c))) return rc;
    TL_TRY_CUDA(cudaStreamSynchronize(c->stream));
    const cudaStream_t lib_stream = c->stream;
    TL_TRY_CUDA(cudaStreamBeginCapture(m->gstream, cudaStreamCaptureModeRelaxed));
    c->stream = m->gstream;
    trace_suspend(true);
    float *gscale = c->scalars + 1;
    rc = cuda_check(cudaMemsetAsync(G, 0, sizeof(float) * m->np, c->stream), "cudaMemsetAsync(G)");
    if (!rc) rc = run_batch(c, *m, P, G, tok, tgt, tgt_mtp, B, loss_dev, true);
    if (!rc) rc = launch_sumsq(c, G, m->np, c->sumsq, norm_dev, gscale, max_norm);
    if (!rc) rc = launch_adamw(c, P, G, M, V, m->np, lr, 0.9f, 0.95f, 0.1f, t, 1.0f, gscale, m->hyper);
    trace_suspend(false);
    c->stream = lib_stream;
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(m->gstream, &graph);
    if (rc) { if (graph) cudaGraphDestroy(graph); return rc; }
    if (ec != cudaSuccess) return cuda_check(ec, "cudaStreamEndCapture");
    const cudaError_t ei = cudaGraphInstantiate(&m->gexec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) { m->gexec = nullptr; return cuda_check(ei, "cudaGraphInstantiate"); }
    m->gkey = key;
  }
  const float hy[4] = {lr, 1.0f - powf(0.9f, (float)t), 1.0f - powf(0.95f, (float)t), 0.0f};
  TL_TRY_CUDA(cudaMemcpyAsync(m->hyper, hy, sizeof hy, cudaMemcpyHostToDevice, c->stream));
  TraceScope ts(c, "graph_step");
  TL_TRY_CUDA(cudaGraphLaunch(m->gexec, c->stream));
  return TL_OK;
}

TL_API int tl_model_step_zero1(void *h, float *P, float *G, float *M_shard, float *V_shard, const int *tok,
                               const int *tgt, const int *tgt_mtp, int B, float lr, int t, float max_norm,
                               float *loss_dev, float *norm_dev) {
  Model *m = static_cast<Model *>(h);
  if (!m) return set_error(TL_EINVAL, "NULL model");
  TL_REQUIRE_CTX(c);
  if (c->device != m->device) return set_error(TL_EINVAL, "model belongs to device %d", m->device);
  if (t < 1) return set_error(TL_EINVAL, "step t must be >= 1 (got %d)", t);
  int rc;
  if ((rc = check_device_ptr(P, "P")) || (rc = check_device_ptr(G, "G")) || (rc = check_device_ptr(tok, "tok")) ||
      (rc = check_device_ptr(tgt, "tgt")) || (rc = check_device_ptr(M_shard, "M_shard")) ||
      (rc = check_device_ptr(V_shard, "V_shard")))
    return rc;
  if (m->n_mtp > 0 && (rc = check_device_ptr(tgt_mtp, "tgt_mtp"))) return rc;
  OverlapState ov;
  if ((rc = overlap_begin(c, G, m->np, &ov))) return rc;
  TL_TRY_CUDA(cudaMemsetAsync(G, 0, sizeof(float) * ov.n_pad, c->stream));
  if ((rc = run_batch(c, *m, P, G, tok, tgt, tgt_mtp, B, loss_dev, true, &ov))) return rc;
  if ((rc = overlap_finish(c, &ov))) return rc;
  return zero1_finish_after_overlap(c, P, G, M_shard, V_shard, m->np, lr, 0.9f, 0.95f, 0.1f, t, max_norm,
                                    norm_dev);
}