"""Shared checks for the parity tests (tolerances are stated here, once)."""
import numpy as np

# AdamW: parameters within 1e-6 relative after one step (north star).  The scale
# of an element is max(|ref|, |input|) so that elements the update drives through
# zero are judged against the magnitude that was updated.
ADAMW_RTOL = 1e-6
# GEMM: the reference selftest's metric max|err| / mean|ref| (tinylm.c:4778-4784)
# within 1e-4 (north star).
GEMM_REL_TOL = 1e-4
# Grad norm: a float rounded from a double sum; summation order may move it by
# at most one float ulp.
NORM_RTOL = 2.5e-7


def assert_adamw_close(got, ref, inp, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), np.abs(np.asarray(inp, np.float64)))
    err = np.abs(got - ref)
    bad = err > ADAMW_RTOL * scale + 1e-30
    assert not bad.any(), (f"{what}: {bad.sum()} elements outside {ADAMW_RTOL} relative; "
                           f"worst err {err.max():.3e} at {int(np.argmax(err - ADAMW_RTOL * scale))}")


def gemm_rel(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    if ref.size == 0:
        return 0.0
    return np.abs(got - ref).max() / max(np.abs(ref).mean(), 1e-30)
