/* tl_oracle.c -- TEST INFRASTRUCTURE ONLY: a plain-C restatement of the
 * reference's hot-path arithmetic, used as the parity checker for the CUDA
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg load it, and only to check or time against; the product never calls it.
 *
 * Pinned against the compiled reference (oracle/_ref/libtlref.so, built from
 * the reference's own tinylm.c by oracle/Makefile) through the golden fixtures
 * in tests/golden/, see tests/test_oracle.py.
 *
 * Each function names the reference lines it restates (tinylm.c).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define TLO_API __attribute__((visibility("default")))

/* AdamW with the clip scale folded in -- tinylm.c:1159-1170.
 * bias corrections with powf in fp32, eps 1e-8 added to sqrt(vhat), decoupled
 * weight decay on the pre-update parameter, G left untouched. */
TLO_API void tlo_adamw(float *P, const float *G, float *M, float *V, size_t n,
                       float lr, float b1, float b2, float wd, int t, float gscale)
{
    const float bc1 = 1.0f - powf(b1, (float)t);
    const float bc2 = 1.0f - powf(b2, (float)t);
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) {
        const float g = G[i] * gscale;
        const float m = b1 * M[i] + (1.0f - b1) * g;
        const float v = b2 * V[i] + (1.0f - b2) * g * g;
        M[i] = m;
        V[i] = v;
        const float mhat = m / bc1, vhat = v / bc2;
        P[i] -= lr * (mhat / (sqrtf(vhat) + 1e-8f) + wd * P[i]);
    }
}

/* Global L2 norm with a double accumulator -- tinylm.c:1171-1176. */
TLO_API float tlo_grad_norm(const float *G, size_t n)
{
    double s = 0.0;
    #pragma omp parallel for reduction(+ : s) schedule(static)
    for (long long i = 0; i < (long long)n; i++) s += (double)G[i] * (double)G[i];
    return (float)sqrt(s);
}

/* Sum of squares only (double), for sharded norms: the global norm is
 * sqrt(sum over shards), the ZeRO-1 decomposition of tinylm.c:1171-1176. */
TLO_API double tlo_sumsq(const float *G, size_t n)
{
    double s = 0.0;
    #pragma omp parallel for reduction(+ : s) schedule(static)
    for (long long i = 0; i < (long long)n; i++) s += (double)G[i] * (double)G[i];
    return s;
}

/* Clip rule with max-norm 1.0 -- tinylm.c:2630-2631 (train_loop), 4739 (bench). */
TLO_API float tlo_clip_scale(float gnorm) { return gnorm > 1.0f ? 1.0f / gnorm : 1.0f; }

/* Y[M,N] = X[M,K] @ W[K,N], overwrite -- tinylm.c:439-478 (semantics of mm).
 * acc64 != 0 accumulates in double (the selftest's reference, 4764). */
TLO_API void tlo_mm(float *Y, const float *X, const float *W, int M, int K, int N, int acc64)
{
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float *x = X + (size_t)m * K;
        float *y = Y + (size_t)m * N;
        for (int n = 0; n < N; n++) {
            if (acc64) {
                double s = 0.0;
                for (int k = 0; k < K; k++) s += (double)x[k] * (double)W[(size_t)k * N + n];
                y[n] = (float)s;
            } else {
                float s = 0.0f;
                for (int k = 0; k < K; k++) s += x[k] * W[(size_t)k * N + n];
                y[n] = s;
            }
        }
    }
}

/* dX[M,K] += dY[M,N] @ W[K,N]^T, accumulate -- tinylm.c:480-508 (mm_bt). */
TLO_API void tlo_mm_bt(float *dX, const float *dY, const float *W, int M, int K, int N, int acc64)
{
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float *dy = dY + (size_t)m * N;
        float *dx = dX + (size_t)m * K;
        for (int k = 0; k < K; k++) {
            const float *w = W + (size_t)k * N;
            if (acc64) {
                double s = 0.0;
                for (int n = 0; n < N; n++) s += (double)dy[n] * (double)w[n];
                dx[k] = (float)((double)dx[k] + s);
            } else {
                float s = 0.0f;
                for (int n = 0; n < N; n++) s += dy[n] * w[n];
                dx[k] += s;
            }
        }
    }
}

/* dW[K,N] += X[M,K]^T @ dY[M,N], accumulate -- tinylm.c:510-537 (mm_atb). */
TLO_API void tlo_mm_atb(float *dW, const float *X, const float *dY, int M, int K, int N, int acc64)
{
    #pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++) {
        float *dw = dW + (size_t)k * N;
        for (int n = 0; n < N; n++) {
            if (acc64) {
                double s = 0.0;
                for (int m = 0; m < M; m++) s += (double)X[(size_t)m * K + k] * (double)dY[(size_t)m * N + n];
                dw[n] = (float)((double)dw[n] + s);
            } else {
                float s = 0.0f;
                for (int m = 0; m < M; m++) s += X[(size_t)m * K + k] * dY[(size_t)m * N + n];
                dw[n] += s;
            }
        }
    }
}

/* The selftest's error metric -- tinylm.c:4778-4784: max|err| / mean|ref|. */
TLO_API double tlo_rel_err(const float *got, const float *ref, size_t n, double *max_abs_out)
{
    double e = 0.0, s = 0.0;
    for (size_t i = 0; i < n; i++) {
        double d = fabs((double)got[i] - (double)ref[i]);
        if (d > e || d != d) e = d;
        s += fabs((double)ref[i]);
    }
    if (max_abs_out) *max_abs_out = e;
    return n ? e / (s / (double)n) : 0.0;
}

/* xorshift64 + Box-Muller normals with the reference's exact draw recipe --
 * tinylm.c:127-134 -- so fixtures can be regenerated without the reference. */
static uint64_t tlo_rng = 1;
TLO_API void tlo_seed(unsigned long long seed) { tlo_rng = (uint64_t)seed | 1ULL; }
TLO_API unsigned long long tlo_xorshift(void)
{
    uint64_t x = tlo_rng;
    x ^= x << 13; x ^= x >> 7; x ^= x << 17;
    tlo_rng = x;
    return x;
}
static float tlo_uniform(void) { return (float)(tlo_xorshift() >> 11) * (1.0f / 9007199254740992.0f); }
TLO_API void tlo_fill_normal(float *dst, size_t n, float scale)
{
    for (size_t i = 0; i < n; i++) {
        float u1 = tlo_uniform();
        if (u1 < 1e-9f) u1 = 1e-9f;
        float u2 = tlo_uniform();
        dst[i] = scale * (sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2));
    }
}

/* Learning-rate schedule of train_loop -- tinylm.c:2587-2590: linear warm-up
 * over `warmup` iterations, then cosine from lr to 0.1*lr. */
TLO_API float tlo_lr_at(int it, float lr, int iters, float warmup)
{
    if (it < warmup) return lr * (it + 1) / warmup;
    float r = (it - warmup) / (float)(iters > warmup ? iters - warmup : 1);
    if (r > 1) r = 1;
    return 0.1f * lr + 0.5f * (1 + cosf(3.14159265f * r)) * (lr - 0.1f * lr);
}
