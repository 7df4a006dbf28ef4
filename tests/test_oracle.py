"""The oracle itself, pinned against fixtures made by the reference's own code
(tests/golden/gen_golden.py).  CPU only."""
import numpy as np
import pytest

import oracle
from helpers import ADAMW_RTOL, assert_adamw_close, gemm_rel
from tests.golden.gen_golden import sha


def regen_gemm_inputs(z):
    M, K, N = (int(x) for x in z["shape"])
    oracle.port().tlo_seed(int(z["seed"][0]))
    X = oracle.fill_normal(M * K, 1.0)
    W = oracle.fill_normal(K * N, 1.0)
    dY = oracle.fill_normal(M * N, 1.0)
    if int(z["init_nonzero"][0]):
        dX0 = oracle.fill_normal(M * K, 1.0)
        dW0 = oracle.fill_normal(K * N, 1.0)
    else:
        dX0 = np.zeros(M * K, np.float32)
        dW0 = np.zeros(K * N, np.float32)
    assert sha(X, W, dY, dX0, dW0) == str(z["input_sha"][0]), "restated rng drifted from the reference's"
    return M, K, N, X, W, dY, dX0, dW0


@pytest.mark.parametrize("name", ["gemm_selftest", "gemm_accum", "gemm_aligned"])
def test_port_gemm_matches_reference(golden, name):
    z = golden(name)
    M, K, N, X, W, dY, dX0, dW0 = regen_gemm_inputs(z)
    Y = np.full(M * N, np.nan, np.float32)
    oracle.mm(Y, X, W, M, K, N)
    dX = dX0.copy(); oracle.mm_bt(dX, dY, W, M, K, N)
    dW = dW0.copy(); oracle.mm_atb(dW, X, dY, M, K, N)
    # fp32 restatement vs the reference's register-blocked fp32 loops
    assert gemm_rel(Y, z["Y"]) < 1e-5
    assert gemm_rel(dX, z["dX"]) < 1e-5
    assert gemm_rel(dW, z["dW"]) < 1e-5
    # and the double-accumulated truth is within the selftest's bound of both
    Y64 = np.empty_like(Y); oracle.mm(Y64, X, W, M, K, N, acc64=True)
    assert gemm_rel(z["Y"], Y64) < 1e-5


@pytest.mark.parametrize("case", ["t1", "t100", "clip"])
def test_port_adamw_matches_reference(golden, case):
    z = golden("adamw")
    p, g, m, v = (z[f"{case}_{k}"].copy() for k in "pgmv")
    gn = oracle.grad_norm(g)
    assert gn == pytest.approx(float(z[f"{case}_gnorm"][0]), rel=2.5e-7)
    gs = oracle.clip_scale(gn)
    assert gs == pytest.approx(float(z[f"{case}_gscale"][0]), rel=2.5e-7)
    g0 = g.copy()
    oracle.adamw(p, g, m, v, 3e-4, 0.9, 0.95, 0.1, int(z[f"{case}_t"][0]), gs)
    assert np.array_equal(g, g0)
    assert_adamw_close(p, z[f"{case}_P"], z[f"{case}_p"], "P")
    assert_adamw_close(m, z[f"{case}_M"], z[f"{case}_m"], "M")
    assert_adamw_close(v, z[f"{case}_V"], z[f"{case}_v"], "V")
    if case == "clip":
        assert float(z["clip_gscale"][0]) < 1.0, "clip fixture must exercise the clip"
    assert ADAMW_RTOL == 1e-6


def test_port_gradnorm_matches_reference(golden):
    z = golden("gradnorm")
    for i, n in enumerate(z["sizes"]):
        if f"g{i}" not in z:
            continue
        g = z[f"g{i}"]
        assert g.size == n
        assert oracle.grad_norm(g) == pytest.approx(float(z["norms"][i]), rel=2.5e-7, abs=0)


@pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")
def test_reference_leg_reproduces_fixtures(golden):
    """Re-running the compiled reference gives the committed numbers (determinism
    of the reference build, OMP threads = 8)."""
    R = oracle.ref()
    R.tlref_init(8, 0)
    z = golden("train_nano")
    cfg = [int(x) for x in z["cfg"]]
    h = R.tlref_model_new((oracle._i * 7)(*cfg), int(z["n_mtp"][0]), int(z["B"][0]), int(z["seed"][0]))
    try:
        gn = oracle._f(0.0)
        for it in range(3):
            loss = R.tlref_model_step(h, 3e-4, it + 1, oracle.ctypes.byref(gn))
            assert loss == pytest.approx(float(z["losses"][it]), rel=1e-5)
    finally:
        R.tlref_model_free(h)


def test_fixture_train_m1_is_config1(golden):
    z = golden("train_m1")
    assert list(z["cfg"]) == [2048, 128, 4, 4, 1, 336, 256]
    assert int(z["n_mtp"][0]) == 2 and int(z["B"][0]) == 8
    assert int(z["nparams"][0]) == 976000
    # loss at step 4 recorded by the survey's determinism probe
    assert float(z["losses"][3]) == pytest.approx(7.407012, abs=2e-6)
