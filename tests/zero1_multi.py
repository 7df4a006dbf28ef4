"""Worker for the multi-GPU ZeRO-1 parity test (run by torchrun, one rank per
GPU).  Each rank holds its own local gradient; after one tl_zero1_step every
rank's full P must equal the single-rank oracle applied to the averaged
gradient (the reference semantics of one big batch, tinylm.c:1079)."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))
import oracle  # noqa: E402
from helpers import assert_adamw_close  # noqa: E402
from tinylm_c_b200.zero1 import Zero1, zero1_layout  # noqa: E402

LR, B1, B2, WD = 3e-4, 0.9, 0.95, 0.1


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    n = 3 * 4096 * world + 777                     # ragged: needs padding
    p, _, m, v = oracle.adamw_inputs(n, seed=1)
    grads = [oracle.adamw_inputs(n, seed=100 + r)[1] * np.float32(40.0) for r in range(world)]
    gavg = (np.sum(np.stack(grads).astype(np.float64), axis=0) / world).astype(np.float32)
    exchange = sys.argv[2] if len(sys.argv) > 2 else "nccl"
    z = Zero1(n, rank, world, local, exchange=exchange)
    n_pad, shard = zero1_layout(n, world)
    lo = rank * shard
    mp = np.zeros(n_pad, np.float32); mp[:n] = m
    vp = np.zeros(n_pad, np.float32); vp[:n] = v

    def run(zz):
        P = torch.zeros(n_pad, device=dev); P[:n] = torch.from_numpy(p)
        G = torch.zeros(n_pad, device=dev); G[:n] = torch.from_numpy(grads[rank])
        M = torch.from_numpy(mp[lo:lo + shard].copy()).to(dev)
        V = torch.from_numpy(vp[lo:lo + shard].copy()).to(dev)
        norm = torch.zeros(1, device=dev)
        zz.step(P, G, M, V, LR, B1, B2, WD, 2, 1.0, norm)
        zz.sync(60000)
        return P, G, M, V, norm

    P, G, M, V, norm = run(z)
    P1, M1, norm1 = P.clone(), M.clone(), norm.clone()
    if exchange == "p2p":
        # the collective path on the same inputs: identical bits
        z.exchange = "nccl"
        Pn, Gn, Mn, Vn, normn = run(z)
        z.exchange = "p2p"
        if world == 2:   # a + b does not depend on the order: identical bits
            assert torch.equal(P, Pn) and torch.equal(M, Mn) and torch.equal(V, Vn), "p2p != nccl"
            assert torch.equal(G[lo:lo + shard], Gn[lo:lo + shard]) and torch.equal(norm, normn)
        else:            # sums in another order: within the oracle tolerance below
            assert torch.allclose(P, Pn, rtol=0, atol=1e-6 * float(P.abs().max()))
        # a second p2p step on the same registered buffers (epoch 2)
        z.step(P, G, M, V, LR, B1, B2, WD, 3, 1.0, norm)
        z.sync(60000)
        assert torch.isfinite(P).all()
        from tinylm_c_b200 import _lib
        _lib.check(_lib.lib().tl_device_status())
    P, M, norm = P1, M1, norm1
    gn = oracle.grad_norm(gavg)
    assert abs(norm.item() - gn) <= 1e-6 * gn, (norm.item(), gn)
    ref = [p.copy(), gavg.copy(), m.copy(), v.copy()]
    oracle.adamw(*ref, LR, B1, B2, WD, 2, oracle.clip_scale(gn))
    # averaging in fp32 across ranks may differ from the float64 mean by an ulp of g
    Pg = P[:n].cpu().numpy()
    err = np.abs(Pg.astype(np.float64) - ref[0])
    assert err.max() <= 1e-6 * np.maximum(np.abs(ref[0]), np.abs(p)).max(), err.max()
    hi = min(lo + shard, n)
    if hi > lo:
        assert_adamw_close(M[:hi - lo].cpu().numpy(), ref[2][lo:hi], m[lo:hi], "M shard")
    z.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("ZERO1_OK", exchange)


if __name__ == "__main__":
    main()
