"""Worker for the drop-in test (own process: the patched reference's seams
turn on the library's host-buffer mode for the device).  Runs the
reference's own training step (cmd_bench order, tinylm.c:4734-4741) from the
harness built over the patched tinylm.c, so its GEMMs, grad norm and AdamW
are libtinylm_cuda calls on the reference's calloc'd buffers, and prints one
JSON line with the losses and grad norms.

    python tests/dropin_steps.py <preset V,D,L,H,KV,F,T> <n_mtp> <B> <steps> <seed>
"""
import ctypes
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402


def main():
    cfg7 = [int(x) for x in sys.argv[1].split(",")]
    n_mtp, B, steps, seed = (int(x) for x in sys.argv[2:6])
    R = oracle.ref_cuda()
    R.tlref_init(len(os.sched_getaffinity(0)), seed)
    h = R.tlref_model_new((oracle._i * 7)(*cfg7), n_mtp, B, seed)
    losses, norms = [], []
    gn = oracle._f(0.0)
    for it in range(steps):
        losses.append(R.tlref_model_step(h, 3e-4, it + 1, ctypes.byref(gn)))
        norms.append(gn.value)
    R.tlref_model_free(h)
    sys.stdout.flush()
    print(json.dumps({"losses": losses, "gnorms": norms}), flush=True)


if __name__ == "__main__":
    main()
