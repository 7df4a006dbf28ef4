"""The drop-in proof: the reference's own tinylm.c with libtinylm_cuda at its
five seams (oracle/dropin_patch.py -- the patch INTEGRATION.md documents,
applied to a build-time copy), its GEMMs, grad norm and AdamW running on the
GPU over the reference's own host buffers (host-buffer mode).  The
reference's CLI runs its own selftest (tinylm.c:4753-4788) and bench
(4705-4748), and its training step reproduces the reference's 10-step losses
of BASELINE config 1 (tests/golden/train_m1.npz) within 1e-4."""
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import oracle

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.has_dropin(), reason="drop-in build not present")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LOSS_ATOL = 1e-4
GNORM_RTOL = 1e-4


def run_cli(*args, env=None):
    e = dict(os.environ, **(env or {}))
    r = subprocess.run([oracle.DROPIN_EXE, *args], capture_output=True, text=True, timeout=600, env=e)
    return r.returncode, r.stdout.replace("\r", "\n"), r.stderr


def test_reference_selftest_passes_through_the_library():
    rc, out, err = run_cli("selftest")
    assert rc == 0, (out, err)
    assert "PASS" in out, out
    rels = [float(x) for x in re.findall(r"rel=([0-9.eE+-]+)", out)]
    assert len(rels) == 3 and max(rels) <= 1e-4, out     # north star: 1e-4 (the selftest itself allows 1e-2)


def test_reference_bench_runs_through_the_library():
    rc, out, err = run_cli("bench", "m1", "3", "8", env={"TINYLM_SEED": "0", "TINYLM_NMTP": "2"})
    assert rc == 0, (out, err)
    m = re.search(r"([0-9.]+) tok/s", out)
    assert m and float(m.group(1)) > 0, out


def test_reference_step_matches_reference_losses(golden):
    """BASELINE config 1 (m1, n_mtp=2, B=8, seed 0): the patched reference's
    ten steps against the unpatched reference's committed losses."""
    z = golden("train_m1")
    cfg = ",".join(str(int(x)) for x in z["cfg"])
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "dropin_steps.py"), cfg, str(int(z["n_mtp"][0])),
                        str(int(z["B"][0])), "10", str(int(z["seed"][0]))],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    res = json.loads(r.stdout.strip().splitlines()[-1])
    np.testing.assert_allclose(res["losses"], z["losses"], rtol=0, atol=LOSS_ATOL)
    np.testing.assert_allclose(res["gnorms"], z["gnorms"], rtol=GNORM_RTOL)
