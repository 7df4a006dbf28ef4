"""Worker for the peer-memory step's failure test (torchrun, 2 ranks, one GPU
each).  Both ranks register; then rank 1 never calls the step (a rank that
does not join, injected on the host).  Rank 0's step must come back on its
own: its bounded device wait expires after TL_DIST_TIMEOUT_MS and
tl_device_status() reports TL_ETIMEOUT; a second step is then refused with
TL_ETIMEOUT.  Rank 1 touches nothing on the device
meanwhile and both leave through a host barrier."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from tinylm_c_b200 import _lib  # noqa: E402
from tinylm_c_b200.zero1 import Zero1, zero1_layout  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    n = 4096 * world * 3
    z = Zero1(n, rank, world, local, exchange="p2p")
    n_pad, shard = zero1_layout(n, world)
    P = torch.zeros(n_pad, device=dev)
    G = torch.ones(n_pad, device=dev)
    M = torch.zeros(shard, device=dev)
    V = torch.zeros(shard, device=dev)
    z.register(P, G)
    dist.barrier()
    if rank == 0:
        z.step(P, G, M, V, 1e-3, 0.9, 0.95, 0.1, 1, 1.0, None)
        torch.cuda.synchronize(dev)
        rc = _lib.lib().tl_device_status()
        print("STATUS", rc, _lib.lib().tl_last_error().decode(), flush=True)
        ok = rc == _lib.TL_ETIMEOUT and torch.all(P == 0).item()
        # A later step is refused (nothing launched) until release + register.
        try:
            z.step(P, G, M, V, 1e-3, 0.9, 0.95, 0.1, 2, 1.0, None)
            again = None
        except _lib.TLError as e:
            again = e.code
        print("SECOND STEP", again, flush=True)
        ok = ok and again == _lib.TL_ETIMEOUT and torch.all(P == 0).item()
    dist.barrier()                      # rank 1 waited here, idle
    z.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and ok:
        print("TIMEOUT_OK")


if __name__ == "__main__":
    main()
