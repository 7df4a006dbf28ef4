"""Host side of the device training step: parameter count and initialisation
against the reference (CPU only, no GPU call)."""
import numpy as np
import pytest

import oracle
from tinylm_c_b200 import model


@pytest.mark.parametrize("preset,n_mtp,want", [("m1", 2, 976000), ("nano", 0, 217664), ("m8", 0, 7562016),
                                               ("scaled", 0, 188777472)])
def test_param_count_matches_reference(preset, n_mtp, want):
    """param_count (tinylm.c:345-358); the survey's figures for the BASELINE configs."""
    assert model.param_count(model.cfg8(preset, n_mtp)) == want


@pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")
@pytest.mark.parametrize("preset,n_mtp", [("nano", 0), ("m1", 2)])
def test_init_params_matches_reference(preset, n_mtp):
    """init_params (tinylm.c:395-419) with the reference generator: bit-identical
    for the 0.02-scaled tensors and norms; the residual projections (wo, w2,
    scaled by 0.02/sqrt(2L)) within two float ulps, because the reference is
    built with -ffast-math, which re-associates that product."""
    R = oracle.ref()
    cfg = list(model.PRESETS[preset])
    h = R.tlref_model_new((oracle._i * 7)(*cfg), n_mtp, 1, 0)
    try:
        n = R.tlref_model_nparams(h)
        Pr = np.ctypeslib.as_array(R.tlref_model_buf(h, 0), shape=(n,)).copy()
    finally:
        R.tlref_model_free(h)
    P = model.init_params(model.cfg8(preset, n_mtp), 0).numpy()
    assert P.shape == Pr.shape
    V, D = cfg[0], cfg[1]
    assert np.array_equal(P[:V * D], Pr[:V * D]), "embedding must be bit-identical"
    ulp = np.spacing(np.abs(Pr).astype(np.float32))
    assert (np.abs(P - Pr) <= 2 * ulp).all()
