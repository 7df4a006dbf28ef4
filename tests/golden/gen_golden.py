"""Generate the golden fixtures in tests/golden/ from the reference itself.

    make -C oracle && python tests/golden/gen_golden.py

Every output here is computed by the reference's own tinylm.c (compiled
unmodified into oracle/_ref/libtlref.so by oracle/Makefile with the reference
CI's flags, OMP threads = 8).  Inputs are either drawn with the reference's own
xorshift64/Box-Muller generator (tinylm.c:127-134; regenerated bit-exactly by
the restatement, so only their hash is stored) or with numpy default_rng
(stored).  Runs only where the reference sources exist; the fixtures are
committed and read by tests/ on any machine.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

LR, B1, B2, WD = 3e-4, 0.9, 0.95, 0.1


def sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def ref_normals(R, n, scale=1.0):
    a = np.empty(n, np.float32)
    R.tlref_fill_normal(oracle.fptr(a), n, scale)
    return a


def gen_gemm(R, name, M, K, N, seed, init_nonzero):
    """Inputs drawn with the reference rng: X(MK), W(KN), dY(MN)[, dX0(MK), dW0(KN)]."""
    R.tlref_seed(seed)
    X = ref_normals(R, M * K)
    W = ref_normals(R, K * N)
    dY = ref_normals(R, M * N)
    if init_nonzero:
        dX0 = ref_normals(R, M * K)
        dW0 = ref_normals(R, K * N)
    else:
        dX0 = np.zeros(M * K, np.float32)
        dW0 = np.zeros(K * N, np.float32)
    Y = np.full(M * N, np.nan, np.float32)  # mm overwrites: NaN must vanish
    dX = dX0.copy()
    dW = dW0.copy()
    R.tlref_mm(oracle.fptr(Y), oracle.fptr(X), oracle.fptr(W), M, K, N)
    R.tlref_mm_bt(oracle.fptr(dX), oracle.fptr(dY), oracle.fptr(W), M, K, N)
    R.tlref_mm_atb(oracle.fptr(dW), oracle.fptr(X), oracle.fptr(dY), M, K, N)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), Y=Y, dX=dX, dW=dW,
                        shape=np.array([M, K, N]), seed=np.array([seed]),
                        init_nonzero=np.array([int(init_nonzero)]),
                        input_sha=np.array([sha(X, W, dY, dX0, dW0)]))


def gen_adamw(R):
    """n = 4099 (not a multiple of 4); config-2 distributions, plus a large-g case
    whose norm > 1 exercises the clip.  Clip scale from the reference's own
    global_gradnorm and the gnm>1 rule of cmd_bench (tinylm.c:4739)."""
    n = 4099
    out = {}
    for case, (gsd, t) in {"t1": (1e-3, 1), "t100": (1e-3, 100), "clip": (0.05, 7)}.items():
        rng = np.random.default_rng({"t1": 11, "t100": 12, "clip": 13}[case])
        p = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))
        g = (rng.standard_normal(n, dtype=np.float32) * np.float32(gsd))
        m = (rng.standard_normal(n, dtype=np.float32) * np.float32(1e-4))
        v = np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(1e-6))
        gn = R.tlref_gradnorm(oracle.fptr(g), n)
        gs = np.float32(1.0) / np.float32(gn) if gn > 1.0 else np.float32(1.0)
        P, G, M_, V = p.copy(), g.copy(), m.copy(), v.copy()
        R.tlref_adamw(oracle.fptr(P), oracle.fptr(G), oracle.fptr(M_), oracle.fptr(V), n,
                      LR, B1, B2, WD, t, float(gs))
        assert np.array_equal(G, g), "reference adamw must not modify G"
        for k, a in dict(p=p, g=g, m=m, v=v, P=P, M=M_, V=V).items():
            out[f"{case}_{k}"] = a
        out[f"{case}_t"] = np.array([t])
        out[f"{case}_gnorm"] = np.array([gn], np.float32)
        out[f"{case}_gscale"] = np.array([gs], np.float32)
    np.savez_compressed(os.path.join(HERE, "adamw.npz"), **out)


def gen_gradnorm(R):
    """Norms of vectors of ragged sizes and scales (including empty and 1)."""
    rng = np.random.default_rng(21)
    sizes = [0, 1, 3, 4, 5, 31, 1000, 4099, 65537, 1 << 20]
    scales = [1.0, 1e-3, 1.0, 2.0, 1e-6, 1e3, 0.5, 1e-3, 1.0, 1e-2]
    vecs, norms = {}, []
    for i, (n, s) in enumerate(zip(sizes, scales)):
        g = (rng.standard_normal(n, dtype=np.float32) * np.float32(s))
        norms.append(R.tlref_gradnorm(oracle.fptr(g), n) if n else 0.0)
        if n <= 65537:
            vecs[f"g{i}"] = g
    np.savez_compressed(os.path.join(HERE, "gradnorm.npz"), sizes=np.array(sizes),
                        scales=np.array(scales), norms=np.array(norms, np.float32),
                        rng_seed=np.array([21]), **vecs)


def gen_train(R, name, cfg7, n_mtp, B, steps, seed=0):
    """Loss and grad norm per step of the reference's cmd_bench loop
    (tinylm.c:4734-4741, t = it+1, lr 3e-4), seed recipe of tinylm.c:4809-4811."""
    h = R.tlref_model_new((oracle._i * 7)(*cfg7), n_mtp, B, seed)
    np_ = R.tlref_model_nparams(h)
    P = np.ctypeslib.as_array(R.tlref_model_buf(h, 0), shape=(np_,))
    p0_sha = sha(P)
    N = B * (cfg7[6] if cfg7[6] > 0 else 256)
    tok = np.ctypeslib.as_array(R.tlref_model_tokens(h, 0), shape=(N,)).copy()
    tgt = np.ctypeslib.as_array(R.tlref_model_tokens(h, 1), shape=(N,)).copy()
    mtp = [np.ctypeslib.as_array(R.tlref_model_tokens(h, 2 + k), shape=(N,)).copy() for k in range(n_mtp)]
    losses, gnorms, psum = [], [], []
    gn = oracle._f(0.0)
    for it in range(steps):
        loss = R.tlref_model_step(h, LR, it + 1, oracle.ctypes.byref(gn))
        losses.append(loss)
        gnorms.append(gn.value)
        psum.append(float(P.astype(np.float64).sum()))
    P_final_head = P[:4096].copy()
    R.tlref_model_free(h)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), cfg=np.array(cfg7), n_mtp=np.array([n_mtp]),
                        B=np.array([B]), seed=np.array([seed]), nparams=np.array([np_]),
                        losses=np.array(losses, np.float32), gnorms=np.array(gnorms, np.float32),
                        psum=np.array(psum), P_final_head=P_final_head,
                        tok=tok.astype(np.int32), tgt=tgt.astype(np.int32),
                        mtp=np.array(mtp, np.int32).reshape(n_mtp, N), p0_sha=np.array([p0_sha]))
    return losses


def main():
    R = oracle.ref()
    R.tlref_init(8, 0)
    gen_gemm(R, "gemm_selftest", 201, 131, 259, seed=0, init_nonzero=False)  # cmd_selftest shape
    gen_gemm(R, "gemm_accum", 37, 20, 44, seed=5, init_nonzero=True)
    gen_gemm(R, "gemm_aligned", 256, 128, 96, seed=7, init_nonzero=True)
    gen_adamw(R)
    gen_gradnorm(R)
    # m1 preset (tinylm.c:114) with n_mtp=2, batch 8
    l1 = gen_train(R, "train_m1", [2048, 128, 4, 4, 1, 336, 256], 2, 8, 10)
    # nano preset (tinylm.c:112), batch 2: a small fast case with KV=2
    l2 = gen_train(R, "train_nano", [512, 64, 4, 4, 2, 176, 256], 0, 2, 10)
    meta = {"generator": "tests/golden/gen_golden.py", "omp_threads": 8,
            "ref_flags": "-O3 -mavx2 -mfma -ffast-math -funroll-loops -fopenmp (oracle/Makefile)",
            "train_m1_losses": [float(x) for x in l1], "train_nano_losses": [float(x) for x in l2]}
    with open(os.path.join(HERE, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(json.dumps(meta, indent=1))


if __name__ == "__main__":
    main()
