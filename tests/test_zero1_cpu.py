"""Host-side logic of the ZeRO-1 step on CPU ranks (gloo, world_size 2 and 4):
the shard layout (the library's own tl_zero1_padded), averaging of per-rank
gradients, the norm assembled from shard sums of squares, AdamW on shards and
the gather of P must reproduce the single-process optimizer step on the mean
gradient.  Arithmetic is the oracle's (CPU), the layout the library's."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

LR, B1, B2, WD = 3e-4, 0.9, 0.95, 0.1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import oracle
    from tinylm_c_b200 import _lib
    from tinylm_c_b200.zero1 import shard_range, zero1_layout
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        n_pad, shard = zero1_layout(n, world)
        assert _lib.lib().tl_zero1_padded(n, world) == n_pad
        lo, hi = shard_range(n, world, rank)
        p, _, m, v = oracle.adamw_inputs(n, seed=3)
        g_local = oracle.adamw_inputs(n, seed=50 + rank)[1] * np.float32(25.0)
        P = np.zeros(n_pad, np.float32); P[:n] = p
        G = torch.zeros(n_pad); G[:n] = torch.from_numpy(g_local)
        # ReduceScatter(avg): gloo has no reduce_scatter, so all_reduce then keep the shard
        dist.all_reduce(G)
        G /= world
        Gs = np.ascontiguousarray(G.numpy()[lo:hi])
        ss = torch.tensor([oracle.sumsq(Gs)], dtype=torch.float64)
        dist.all_reduce(ss)
        gn = np.float32(np.sqrt(ss.item()))
        gs = oracle.clip_scale(gn)
        Ms = np.zeros(n_pad, np.float32); Ms[:n] = m
        Vs = np.zeros(n_pad, np.float32); Vs[:n] = v
        Ps, Ms, Vs = (np.ascontiguousarray(x[lo:hi]) for x in (P, Ms, Vs))
        oracle.adamw(Ps, Gs, Ms, Vs, LR, B1, B2, WD, 4, gs)
        out = [torch.zeros(shard) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(Ps))
        Pfull = torch.cat(out).numpy()
        if rank == 0:
            q.put((Pfull[:n].copy(), float(gn), bool((Pfull[n:] == 0).all())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_zero1_host_logic_matches_single_process(world):
    n = 2 * 4096 * world + 1234
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    Pfull, gn, pad_zero = q.get(timeout=120)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    import oracle
    p, _, m, v = oracle.adamw_inputs(n, seed=3)
    grads = [oracle.adamw_inputs(n, seed=50 + r)[1] * np.float32(25.0) for r in range(world)]
    gavg = (np.sum(np.stack(grads), axis=0, dtype=np.float32) / np.float32(world)).astype(np.float32)
    want_gn = oracle.grad_norm(gavg)
    assert gn == pytest.approx(want_gn, rel=1e-6)
    oracle.adamw(p, gavg, m, v, LR, B1, B2, WD, 4, oracle.clip_scale(want_gn))
    assert pad_zero
    np.testing.assert_allclose(Pfull, p, rtol=1e-6, atol=1e-9)


def _never_joins_worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        return                      # this rank exits without ever joining
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:         # the survivor learns of it on the host, by timeout
        q.put(type(e).__name__)


def test_peer_that_never_joins_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_never_joins_worker, args=(r, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = q.get(timeout=60)
    for pr in procs:
        pr.join(timeout=30)
    assert res != "joined"
