/* ref_harness.c -- TEST INFRASTRUCTURE ONLY (the parity oracle's reference leg).
 *
 * Compiles the reference's own tinylm.c (unmodified, read where it lies via -I)
 * into oracle/_ref/libtlref.so and exports thin extern "C" wrappers around its
 * static functions, so tests and bench.py's CPU-baseline leg can call the
 * reference arithmetic directly through ctypes.  Nothing in the product path
 * links or loads this library.
 *
 * Wrapped reference functions (tinylm.c line numbers):
 *   mm 439-478, mm_bt 480-508, mm_atb 510-537, adamw 1159-1170,
 *   global_gradnorm 1171-1176, forward 968-1029, backward 1072-1154,
 *   init_params 395-419, param_count 345-358, preset 109-124, rng 126-134,
 *   set_ftz 4790-4804, step order of cmd_bench 4734-4741, train_loop 2562-2654,
 *   model_load 1915-1938, opt_load 2533-2539.
 */
#define main tinylm_main
#include "tinylm.c"
#undef main

#define TLREF_API __attribute__((visibility("default")))

/* ---- process set-up (mirrors main() 4809-4826 without the CLI) ---------- */
TLREF_API void tlref_init(int nthreads, unsigned long long seed)
{
    g_rng = (uint64_t)seed | 1ULL;               /* TINYLM_SEED semantics, 4809-4811 */
    set_ftz();
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
    #pragma omp parallel
    { set_ftz(); }
#else
    (void)nthreads;
#endif
}
TLREF_API int tlref_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
TLREF_API void tlref_seed(unsigned long long seed) { g_rng = (uint64_t)seed | 1ULL; }
TLREF_API unsigned long long tlref_xorshift(void) { return xorshift(); }
TLREF_API void tlref_fill_normal(float *dst, size_t n, float scale)
{ for (size_t i = 0; i < n; i++) dst[i] = scale * rnd_normal(); }

/* ---- the hot-path primitives ------------------------------------------- */
TLREF_API void tlref_mm(float *Y, const float *X, const float *W, int M, int K, int N)
{ mm(Y, X, W, M, K, N); }
TLREF_API void tlref_mm_bt(float *dX, const float *dY, const float *W, int M, int K, int N)
{ mm_bt(dX, dY, W, M, K, N); }
TLREF_API void tlref_mm_atb(float *dW, const float *X, const float *dY, int M, int K, int N)
{ mm_atb(dW, X, dY, M, K, N); }
TLREF_API void tlref_adamw(float *P, float *G, float *M, float *V, size_t n, float lr,
                           float b1, float b2, float wd, int t, float gscale)
{ adamw(P, G, M, V, n, lr, b1, b2, wd, t, gscale); }
TLREF_API float tlref_gradnorm(const float *G, size_t n) { return global_gradnorm(G, n); }
TLREF_API int tlref_selftest(void) { return cmd_selftest(0, 0); }

/* ---- a whole training step, for loss parity and the step CPU baseline --- */
typedef struct {
    Cfg c; size_t np; int B, N;
    float *P, *G, *M, *V;
    Weights w, gr; Acts *a;
    int *tok, *tgt, **tgt_mtp;
} RefModel;

/* cfg: V,D,L,H,KV,F,T (T<=0 -> 256).  Draw order follows cmd_bench 4718-4724:
 * init_params normals, then tok/tgt interleaved, then each MTP target row. */
TLREF_API void *tlref_model_new(const int *cfg7, int n_mtp, int B, unsigned long long seed)
{
    RefModel *r = (RefModel *)calloc(1, sizeof(RefModel));
    Cfg *c = &r->c;
    memset(c, 0, sizeof(*c));
    c->V = cfg7[0]; c->D = cfg7[1]; c->L = cfg7[2]; c->H = cfg7[3]; c->KV = cfg7[4];
    c->F = cfg7[5]; c->T = cfg7[6] > 0 ? cfg7[6] : 256; c->rope_base = 10000.0f;
    c->n_mtp = n_mtp;
    cfg_derive(c);
    g_rng = (uint64_t)seed | 1ULL;
    /* rope_init caches its table by position count only (tinylm.c:615), so a
     * second model with another head size in the same process would index a
     * stale table; drop it first (a CLI process only ever builds one model). */
    free(rope_cos); free(rope_sin); rope_cos = rope_sin = NULL; rope_max = 0;
    rope_init(c, c->T);
    r->np = param_count(c);
    r->P = fz(r->np); r->G = fz(r->np); r->M = fz(r->np); r->V = fz(r->np);
    map_weights(c, r->P, &r->w); map_weights(c, r->G, &r->gr);
    memset(&r->w.ng, 0, sizeof(r->w.ng)); memset(&r->gr.ng, 0, sizeof(r->gr.ng));
    init_params(c, &r->w);
    r->B = B; r->N = B * c->T;
    r->a = acts_new(c, B);
    r->tok = (int *)malloc(sizeof(int) * r->N); r->tgt = (int *)malloc(sizeof(int) * r->N);
    for (int i = 0; i < r->N; i++) { r->tok[i] = (int)(xorshift() % c->V); r->tgt[i] = (int)(xorshift() % c->V); }
    r->tgt_mtp = n_mtp > 0 ? (int **)malloc(sizeof(int *) * n_mtp) : NULL;
    for (int k = 0; k < n_mtp; k++) {
        r->tgt_mtp[k] = (int *)malloc(sizeof(int) * r->N);
        for (int i = 0; i < r->N; i++) r->tgt_mtp[k][i] = (int)(xorshift() % c->V);
    }
    return r;
}
TLREF_API size_t tlref_model_nparams(void *h) { return ((RefModel *)h)->np; }
TLREF_API float *tlref_model_buf(void *h, int which)
{
    RefModel *r = (RefModel *)h;
    return which == 0 ? r->P : which == 1 ? r->G : which == 2 ? r->M : r->V;
}
TLREF_API int *tlref_model_tokens(void *h, int which)
{
    RefModel *r = (RefModel *)h;
    if (which == 0) return r->tok;
    if (which == 1) return r->tgt;
    return r->tgt_mtp ? r->tgt_mtp[which - 2] : NULL;
}
TLREF_API float *tlref_model_logits(void *h) { return ((RefModel *)h)->a->logits; }
/* forward only (loss with targets) */
TLREF_API float tlref_model_forward(void *h)
{
    RefModel *r = (RefModel *)h;
    return forward(&r->c, &r->w, r->a, r->tok, r->tgt);
}
/* forward + memset(G) + backward only (the gradient stays in G); returns the loss. */
TLREF_API float tlref_model_fwd_bwd(void *h)
{
    RefModel *r = (RefModel *)h;
    float loss = forward(&r->c, &r->w, r->a, r->tok, r->tgt);
    memset(r->G, 0, sizeof(float) * r->np);
    backward(&r->c, &r->w, &r->gr, r->a, r->tok, r->tgt, r->tgt_mtp);
    return loss;
}
/* One step exactly as cmd_bench 4736-4740; returns the loss, writes the grad norm. */
TLREF_API float tlref_model_step(void *h, float lr, int t, float *gnorm_out)
{
    RefModel *r = (RefModel *)h;
    float loss = forward(&r->c, &r->w, r->a, r->tok, r->tgt);
    memset(r->G, 0, sizeof(float) * r->np);
    backward(&r->c, &r->w, &r->gr, r->a, r->tok, r->tgt, r->tgt_mtp);
    float gnm = global_gradnorm(r->G, r->np);
    float gs = gnm > 1.0f ? 1.0f / gnm : 1.0f;
    adamw(r->P, r->G, r->M, r->V, r->np, lr, 0.9f, 0.95f, 0.1f, t, gs);
    if (gnorm_out) *gnorm_out = gnm;
    return loss;
}
TLREF_API void tlref_model_free(void *h)
{
    RefModel *r = (RefModel *)h;
    if (!r) return;
    free(r->P); free(r->G); free(r->M); free(r->V);
    free(r->tok); free(r->tgt);
    for (int k = 0; k < r->c.n_mtp; k++) free(r->tgt_mtp[k]);
    free(r->tgt_mtp);
    free(r);   /* Acts and weight-pointer tables are leaked as the reference does */
}

/* ---- the reference's whole training loop, for trainer / checkpoint parity --
 * Runs train_loop (tinylm.c:2562-2654) on a fresh model (init_params seeded
 * as TINYLM_SEED) or, when resume_bundle is given, on the parameters of that
 * TLM bundle and the AdamW state of resume_opt (model_load + opt_load, the
 * resume path of cmd_train 2742-2743; the generator restarts from the seed).
 * tr/vl are uint16 token streams.  Writes `out` (TLM4) and `optpath` (TOPT)
 * as train_loop does; its progress lines go to stdout. */
TLREF_API int tlref_train(const int *cfg7, int n_mtp, int B, int iters, float lr, unsigned long long seed,
                          const uint16_t *tr, size_t ntr, const uint16_t *vl, size_t nvl,
                          const char *out, const char *optpath, const uint8_t *tok_blob, int tok_len,
                          const char *resume_bundle, const char *resume_opt)
{
    Cfg c; memset(&c, 0, sizeof(c));
    int start_iter = 0;
    float *loaded = NULL;
    if (resume_bundle) {
        loaded = model_load(resume_bundle, &c);
    } else {
        c.V = cfg7[0]; c.D = cfg7[1]; c.L = cfg7[2]; c.H = cfg7[3]; c.KV = cfg7[4];
        c.F = cfg7[5]; c.T = cfg7[6] > 0 ? cfg7[6] : 256; c.rope_base = 10000.0f;
        c.n_mtp = n_mtp;
        cfg_derive(&c);
    }
    g_rng = (uint64_t)seed | 1ULL;
    free(rope_cos); free(rope_sin); rope_cos = rope_sin = NULL; rope_max = 0;
    rope_init(&c, c.T);
    size_t np = param_count(&c);
    float *P = fz(np), *G = fz(np), *M = fz(np), *Vv = fz(np);
    Weights w, gr; map_weights(&c, P, &w); map_weights(&c, G, &gr);
    memset(&w.ng, 0, sizeof(w.ng)); memset(&gr.ng, 0, sizeof(gr.ng));
    if (loaded) {
        memcpy(P, loaded, sizeof(float) * np); free(loaded);
        start_iter = opt_load(resume_opt, M, Vv, np);
    } else {
        init_params(&c, &w);
    }
    fflush(stdout);
    train_loop(&c, &w, &gr, P, G, M, Vv, np, tr, ntr, vl, nvl, B, iters, lr, start_iter,
               out, optpath, tok_blob, tok_len);
    fflush(stdout);
    free(P); free(G); free(M); free(Vv);
    return start_iter;
}
/* model_load (tinylm.c:1915-1938) of a bundle: fills cfg11 with the header
 * fields V,D,L,H,KV,F,T,eot,tmpl,n_mtp,n_exp and returns the parameter count;
 * copies the parameters to P when P is not NULL. */
TLREF_API size_t tlref_model_load(const char *path, int *cfg11, float *P, size_t cap)
{
    Cfg c; memset(&c, 0, sizeof(c));
    float *p = model_load(path, &c);
    size_t np = param_count(&c);
    int h[11] = {c.V, c.D, c.L, c.H, c.KV, c.F, c.T, c.eot, c.tmpl, c.n_mtp, c.n_exp};
    memcpy(cfg11, h, sizeof(h));
    if (P && cap >= np) memcpy(P, p, sizeof(float) * np);
    free(p);
    return np;
}
