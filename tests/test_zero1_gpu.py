"""ZeRO-1 optimizer step through the C ABI on one GPU (a 1-rank NCCL
communicator): must equal the fused single-GPU step, which is itself pinned to
the reference.  The 2..8-GPU form runs in tests/zero1_multi.py under torchrun
when more GPUs are visible."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
from helpers import NORM_RTOL, assert_adamw_close
from tinylm_c_b200 import ops
from tinylm_c_b200.zero1 import Zero1, zero1_layout

pytestmark = pytest.mark.gpu
LR, B1, B2, WD = 3e-4, 0.9, 0.95, 0.1


def test_zero1_single_rank_matches_fused_step(cuda):
    n = 50021
    p, g, m, v = oracle.adamw_inputs(n, seed=17)
    g *= np.float32(30.0)                      # clip active
    z = Zero1(n, 0, 1, 0)
    n_pad, shard = zero1_layout(n, 1)
    P = torch.zeros(n_pad, device=cuda); P[:n] = torch.from_numpy(p)
    G = torch.zeros(n_pad, device=cuda); G[:n] = torch.from_numpy(g)
    M = torch.zeros(shard, device=cuda); M[:n] = torch.from_numpy(m)
    V = torch.zeros(shard, device=cuda); V[:n] = torch.from_numpy(v)
    norm = torch.zeros(1, device=cuda)
    z.step(P, G, M, V, LR, B1, B2, WD, 5, 1.0, norm)
    z.sync(30000)
    gn = oracle.grad_norm(g)
    assert norm.item() == pytest.approx(gn, rel=NORM_RTOL)
    ref = [x.copy() for x in (p, g, m, v)]
    oracle.adamw(*ref, LR, B1, B2, WD, 5, oracle.clip_scale(gn))
    assert_adamw_close(P[:n].cpu().numpy(), ref[0], p, "P")
    assert_adamw_close(M[:n].cpu().numpy(), ref[2], m, "M")
    assert_adamw_close(V[:n].cpu().numpy(), ref[3], v, "V")
    assert torch.all(P[n:] == 0), "padding must stay zero"
    z.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero1_two_ranks_matches_single_rank_oracle(cuda, tmp_path):
    script = os.path.join(os.path.dirname(__file__), "zero1_multi.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
                        "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
                        script, str(tmp_path)], capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ZERO1_OK" in r.stdout


def test_dist_init_reports_timeout_when_peer_never_joins(cuda):
    """A 2-rank communicator whose second rank never arrives: tl_dist_init must
    come back with TL_ETIMEOUT after the configured deadline (host-side failure
    injection; no kernel is in flight)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import ctypes, sys\n"
        f"sys.path.insert(0, {root!r})\n"
        "from tinylm_c_b200 import _lib, ops\n"
        "ops.init(0)\n"
        "L = _lib.lib()\n"
        "uid = (ctypes.c_char * 128)()\n"
        "assert L.tl_dist_unique_id(ctypes.addressof(uid)) == 0\n"
        "rc = L.tl_dist_init(0, 2, ctypes.addressof(uid))\n"
        "print('RC', rc, L.tl_last_error().decode())\n"
    )
    env = dict(os.environ, TL_DIST_TIMEOUT_MS="3000", NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", code],
                       capture_output=True, text=True, env=env)
    assert "RC -5" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
