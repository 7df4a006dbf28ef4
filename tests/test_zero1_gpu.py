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
from tinylm_c_b200 import _lib, ops
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


def test_zero1_p2p_single_rank_matches_fused_step(cuda):
    """The peer-memory step on a one-rank communicator (no peers mapped):
    same result as the collective step, bit for bit."""
    n = 50021
    p, g, m, v = oracle.adamw_inputs(n, seed=23)
    g *= np.float32(30.0)
    out = {}
    for exchange in ("nccl", "p2p"):
        z = Zero1(n, 0, 1, 0, exchange=exchange)
        n_pad, shard = zero1_layout(n, 1)
        P = torch.zeros(n_pad, device=cuda); P[:n] = torch.from_numpy(p)
        G = torch.zeros(n_pad, device=cuda); G[:n] = torch.from_numpy(g)
        M = torch.zeros(shard, device=cuda); M[:n] = torch.from_numpy(m)
        V = torch.zeros(shard, device=cuda); V[:n] = torch.from_numpy(v)
        norm = torch.zeros(1, device=cuda)
        for t in (5, 6):
            z.step(P, G, M, V, LR, B1, B2, WD, t, 1.0, norm)
        z.sync(30000)
        _lib.check(_lib.lib().tl_device_status())
        out[exchange] = [x.cpu() for x in (P, M, V, norm)]
        z.close()
    for a, b in zip(out["nccl"], out["p2p"]):
        assert torch.equal(a, b)


def _torchrun2(script, args, port, env_extra=None, limit=300):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", **(env_extra or {}))
    return subprocess.run(["timeout", "-k", "30", str(limit), sys.executable, "-m", "torch.distributed.run",
                           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
                           os.path.join(os.path.dirname(__file__), script)] + args,
                          capture_output=True, text=True, env=env)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,port", [("nccl", 29531), ("p2p", 29533)])
def test_zero1_two_ranks_matches_single_rank_oracle(cuda, tmp_path, exchange, port):
    """Two ranks, each with its own gradient: the averaged-gradient step equals
    the oracle; the peer-memory step also equals the collective one bit for
    bit and runs a second epoch on the same registration."""
    r = _torchrun2("zero1_multi.py", [str(tmp_path), exchange], port)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"ZERO1_OK {exchange}" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero1_p2p_wait_expires_when_a_rank_does_not_join(cuda):
    """Host-side failure injection: rank 1 never calls the step.  Rank 0's
    bounded device wait must expire (TL_DIST_TIMEOUT_MS=1500) and report
    TL_ETIMEOUT through tl_device_status, with P untouched."""
    r = _torchrun2("zero1_p2p_timeout.py", [], 29535, {"TL_DIST_TIMEOUT_MS": "1500"}, limit=180)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TIMEOUT_OK" in r.stdout, r.stdout[-3000:]


def test_dist_init_reports_timeout_when_peer_never_joins(cuda):
    """A 2-rank communicator whose second rank never arrives: tl_dist_init must
    come back with TL_ETIMEOUT after the configured set-up deadline
    (TL_DIST_INIT_TIMEOUT_MS; host-side failure injection, no kernel in
    flight)."""
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
    env = dict(os.environ, TL_DIST_TIMEOUT_MS="3000", TL_DIST_INIT_TIMEOUT_MS="3000", NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", code],
                       capture_output=True, text=True, env=env)
    assert "RC -5" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
