"""Worker for the multi-GPU trainer test (run by torchrun, one rank per GPU).

Usage: trainer_multi.py OUTDIR fresh|resume|overlap
  fresh:  train the nano preset for 6 iterations at global batch 4 from seed 0
          and write OUTDIR/w2.bin + OUTDIR/w2.opt
  resume: resume OUTDIR/w2r.bin + OUTDIR/w2r.opt (copies of files written by a
          one-rank run at iteration 3) to iteration 6
  overlap: 3 iterations with the gradient reduction overlapped with the
          backward pass (tl_model_step_zero1) and 3 without it, from the same
          start: parameters and optimizer shards must be identical bits
Rank 0 prints the validation lines prefixed with VAL and finally TRAINER_OK.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from tinylm_c_b200 import _lib, model, trainer  # noqa: E402

LR = 6e-4


def streams():
    rng = np.random.default_rng(0)
    return rng.integers(0, 512, 20000).astype(np.uint16), rng.integers(0, 512, 5000).astype(np.uint16)


def main():
    out, mode = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    tr, vl = streams()
    if mode == "overlap":
        res = []
        for ov in (True, False):
            t = trainer.Trainer(model.cfg8("nano", 0), 4, micro_batch=1, device=local, rank=rank, world=world,
                                overlap=ov)
            t.run(tr, vl, 3, LR, seed=0, log=lambda *_: None)
            _lib.check(_lib.lib().tl_device_status())
            res.append([x.cpu().clone() for x in (t.P, t.M, t.V)])
            t.close()
        for a, b in zip(*res):
            assert torch.equal(a, b), "overlapped step differs"
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            print("TRAINER_OK")
        return
    t = trainer.Trainer(model.cfg8("nano", 0), 4, device=local, rank=rank, world=world)
    lines = []
    if mode == "fresh":
        files = (os.path.join(out, "w2.bin"), os.path.join(out, "w2.opt"))
        t.run(tr, vl, 6, LR, seed=0, out=files[0], optpath=files[1], log=lines.append)
    else:
        files = (os.path.join(out, "w2r.bin"), os.path.join(out, "w2r.opt"))
        t.run(tr, vl, 6, LR, seed=0, out=files[0], optpath=files[1], resume=True, log=lines.append)
    _lib.check(_lib.lib().tl_device_status())
    t.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        for ln in lines:
            print("VAL", ln)
        print("TRAINER_OK")


if __name__ == "__main__":
    main()
