// tl_model.cuh -- declarations shared by the device training step.
#pragma once
#include "tl_common.cuh"

namespace tl {

constexpr int ATT_TMAX = 256;   // the reference's context (tinylm.c:111)
constexpr int ATT_HDMAX = 64;

int mk_setup(int device);
int k_embed_fwd(DeviceCtx *c, const float *emb, const int *tok, float *out, int N, int D, int V);
// scratch: 3 * V + 2 * N ints (nullptr: the token-scanning kernel)
int k_embed_bwd(DeviceCtx *c, float *gemb, const int *tok, const float *dout, int N, int D, int V, int *scratch);
int k_rmsnorm_fwd(DeviceCtx *c, const float *x, const float *g, float *out, float *rinv, int rows, int D);
// dx = dres + RMSNorm backward of dy (dres: nullptr, dx itself, or another
// array); dg += the gain gradient (fixed-order reduction of per-block partial
// rows `part`; tmp, 8 x D floats or nullptr, holds its middle level).
int k_rmsnorm_bwd(DeviceCtx *c, const float *x, const float *g, const float *rinv, const float *dy,
                  const float *dres, float *dx, float *dg, float *part, int part_rows, int rows, int D, float *tmp);
int k_rope(DeviceCtx *c, float *buf, const float *cosT, const float *sinT, int rows, int nh, int hd, int T, int back);
int k_add(DeviceCtx *c, float *y, const float *x, size_t n);
int k_swiglu_fwd(DeviceCtx *c, const float *g, const float *u, float *act, size_t n);
int k_swiglu_bwd(DeviceCtx *c, const float *g, const float *u, const float *dact, float *dg, float *du, size_t n);
int k_mtp_hk(DeviceCtx *c, const float *fn, const float *t1, float *hk, size_t n);
int k_mtp_bwd(DeviceCtx *c, const float *t1, const float *dhk, float *dfn, float *dt1, size_t n);
int k_softmax_ce(DeviceCtx *c, float *logits, const int *tgt, int N, int V, float scale, double *loss_rows);
int k_loss_sum(DeviceCtx *c, const double *rows, int N, double *acc);
int k_loss_final(DeviceCtx *c, const double *acc, double denom, float *out);
int k_attn_fwd(DeviceCtx *c, const float *q, const float *k, const float *v, float *out, float *lse, int B, int T,
               int H, int KV, int hd);
// dsT: scratch of B*H*T*T floats (dS^T of the causal tile pairs, written by the
// key-side kernel and read by the query-side one).
// Also applies RoPE's backward (tables cosT / sinT) to dQ and dK.
int k_attn_bwd(DeviceCtx *c, const float *q, const float *k, const float *v, const float *out, const float *dout,
               const float *lse, float *Drow, float *dsT, float *dq, float *dk, float *dv, int B, int T, int H,
               int KV, int hd, const float *cosT, const float *sinT);

}  // namespace tl
