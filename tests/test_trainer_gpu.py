"""The training loop on the GPU (tinylm_c_b200.trainer) against the
reference's own train_loop (tinylm.c:2562-2654) run live on the same data:
validation losses, the final TLM4 bundle and TOPT sidecar, and resuming from
files the reference wrote."""
import os
import re
import shutil

import numpy as np
import pytest
import torch

import oracle
from tinylm_c_b200 import _lib, model, trainer

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")]
CFG7 = [512, 64, 4, 4, 2, 176, 256]      # nano preset (tinylm.c:112)
LR = 6e-4                                 # default_lr_for a D=64 model (tinylm.c:2546)
VAL_RE = re.compile(r"iter\s+(\d+) .*\| val ([0-9.]+)")


def streams():
    rng = np.random.default_rng(0)
    return rng.integers(0, 512, 20000).astype(np.uint16), rng.integers(0, 512, 5000).astype(np.uint16)


def vals(lines):
    return [(int(m.group(1)), float(m.group(2))) for m in map(VAL_RE.search, lines) if m]


def read_opt(path, n):
    raw = open(path, "rb").read()
    it = int(np.frombuffer(raw[4:8], np.int32)[0])
    body = np.frombuffer(raw[8:], np.float32)
    return it, body[:n].astype(np.float64), body[n:2 * n].astype(np.float64)


def read_bundle(path, n):
    raw = open(path, "rb").read()
    return raw[:48], np.frombuffer(raw[48:48 + 4 * n], np.float32).astype(np.float64)


def rel(a, b):
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def compare_runs(mine, ref, P0, n):
    hm, Pm = read_bundle(mine[0], n)
    hr, Pr = read_bundle(ref[0], n)
    assert hm == hr, "bundle headers differ"
    assert rel(Pm - P0, Pr - P0) <= 1e-3, "parameter update differs"
    itm, Mm, Vm = read_opt(mine[1], n)
    itr, Mr, Vr = read_opt(ref[1], n)
    assert itm == itr
    assert rel(Mm, Mr) <= 1e-4 and rel(Vm, Vr) <= 1e-4


def test_fresh_run_matches_reference_train_loop(cuda, tmp_path):
    tr, vl = streams()
    oracle.ref().tlref_init(8, 0)
    ref = (str(tmp_path / "r.bin"), str(tmp_path / "r.opt"))
    ref_lines = oracle.ref_train(CFG7, 0, 2, 6, LR, 0, tr, vl, ref[0], ref[1])
    cfg = model.cfg8("nano", 0)
    t = trainer.Trainer(cfg, 2, device=0)
    mine = (str(tmp_path / "m.bin"), str(tmp_path / "m.opt"))
    lines = []
    t.run(tr, vl, 6, LR, seed=0, out=mine[0], optpath=mine[1], log=lines.append)
    _lib.check(_lib.lib().tl_device_status())
    t.close()
    vr, vm = vals(ref_lines), vals(lines)
    assert [i for i, _ in vr] == [i for i, _ in vm] == [0, 6]
    for (_, a), (_, b) in zip(vm, vr):
        assert abs(a - b) <= 2e-4, (vm, vr)            # the reference prints 4 decimals
    P0 = model.init_params(cfg, 0).numpy().astype(np.float64)
    compare_runs(mine, ref, P0, t.n)


def test_resume_from_reference_files_matches_reference_resume(cuda, tmp_path):
    """The reference trains 3 iterations and writes its files; the reference and
    this trainer each resume from those files to iteration 6."""
    tr, vl = streams()
    R = oracle.ref()
    R.tlref_init(8, 0)
    a = (str(tmp_path / "a.bin"), str(tmp_path / "a.opt"))
    oracle.ref_train(CFG7, 0, 2, 3, LR, 0, tr, vl, a[0], a[1])
    ref = (str(tmp_path / "r.bin"), str(tmp_path / "r.opt"))
    shutil.copy(a[0], ref[0]); shutil.copy(a[1], ref[1])
    ref_lines = oracle.ref_train(CFG7, 0, 2, 6, LR, 0, tr, vl, ref[0], ref[1], resume=ref)
    mine = (str(tmp_path / "m.bin"), str(tmp_path / "m.opt"))
    shutil.copy(a[0], mine[0]); shutil.copy(a[1], mine[1])
    cfg = model.cfg8("nano", 0)
    t = trainer.Trainer(cfg, 2, device=0)
    lines = []
    t.run(tr, vl, 6, LR, seed=0, out=mine[0], optpath=mine[1], resume=True, log=lines.append)
    _lib.check(_lib.lib().tl_device_status())
    t.close()
    vr, vm = vals(ref_lines), vals(lines)
    assert [i for i, _ in vr] == [i for i, _ in vm] == [3, 6]
    for (_, x), (_, y) in zip(vm, vr):
        assert abs(x - y) <= 2e-4, (vm, vr)
    _, P3 = read_bundle(a[0], t.n)
    compare_runs(mine, ref, P3, t.n)


def test_micro_batched_trainer_matches_whole_batch(cuda, tmp_path):
    """Same run with the batch as one micro-batch or as two: same validation
    losses and parameters up to rounding."""
    tr, vl = streams()
    cfg = model.cfg8("nano", 0)
    out = []
    for mb in (4, 2):
        t = trainer.Trainer(cfg, 4, micro_batch=mb, device=0)
        h = t.run(tr, vl, 3, LR, seed=1, log=lambda *_: None)
        out.append(([v for k, _, v in h if k == "val"], t.P[: t.n].cpu().numpy().astype(np.float64)))
        t.close()
    assert np.allclose(out[0][0], out[1][0], atol=1e-5)
    assert np.max(np.abs(out[0][1] - out[1][1])) < 1e-6


def _torchrun(script_args, port):
    script = os.path.join(os.path.dirname(__file__), "trainer_multi.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    import subprocess
    import sys
    r = subprocess.run(["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
                        "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
                        script] + script_args, capture_output=True, text=True, env=env)
    assert r.returncode == 0 and "TRAINER_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
    return [ln[4:] for ln in r.stdout.splitlines() if ln.startswith("VAL ")]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_trainer_matches_one_rank(cuda, tmp_path):
    """Data parallel over 2 GPUs (each rank half of the global batch, ZeRO-1
    step, shard-wise TOPT writes) against the one-rank trainer on the same
    global batch: same validation losses, parameters and optimizer state up
    to the rounding of the cross-rank gradient average.  Then both resume
    from one-rank files written at iteration 3."""
    tr, vl = streams()
    cfg = model.cfg8("nano", 0)
    one = (str(tmp_path / "w1.bin"), str(tmp_path / "w1.opt"))
    t = trainer.Trainer(cfg, 4, device=0)
    lines1 = []
    t.run(tr, vl, 6, LR, seed=0, out=one[0], optpath=one[1], log=lines1.append)
    n = t.n
    t.close()
    lines2 = _torchrun([str(tmp_path), "fresh"], 29541)
    v1, v2 = vals(lines1), vals(lines2)
    assert [i for i, _ in v1] == [i for i, _ in v2] == [0, 6]
    for (_, a), (_, b) in zip(v1, v2):
        assert abs(a - b) <= 2e-4, (v1, v2)
    P0 = model.init_params(cfg, 0).numpy().astype(np.float64)
    compare_runs((str(tmp_path / "w2.bin"), str(tmp_path / "w2.opt")), one, P0, n)

    # resume: one-rank files at iteration 3, continued by 1 and by 2 ranks
    a = (str(tmp_path / "a.bin"), str(tmp_path / "a.opt"))
    t = trainer.Trainer(cfg, 4, device=0)
    t.run(tr, vl, 3, LR, seed=0, out=a[0], optpath=a[1], log=lambda *_: None)
    t.close()
    r1 = (str(tmp_path / "r1.bin"), str(tmp_path / "r1.opt"))
    for dst in (r1, (str(tmp_path / "w2r.bin"), str(tmp_path / "w2r.opt"))):
        shutil.copy(a[0], dst[0]); shutil.copy(a[1], dst[1])
    t = trainer.Trainer(cfg, 4, device=0)
    lines1 = []
    t.run(tr, vl, 6, LR, seed=0, out=r1[0], optpath=r1[1], resume=True, log=lines1.append)
    t.close()
    lines2 = _torchrun([str(tmp_path), "resume"], 29543)
    v1, v2 = vals(lines1), vals(lines2)
    assert [i for i, _ in v1] == [i for i, _ in v2] == [3, 6]
    for (_, x), (_, y) in zip(v1, v2):
        assert abs(x - y) <= 2e-4, (v1, v2)
    _, P3 = read_bundle(a[0], n)
    compare_runs((str(tmp_path / "w2r.bin"), str(tmp_path / "w2r.opt")), r1, P3, n)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_overlapped_reduction_is_bit_identical(cuda, tmp_path):
    """tl_model_step_zero1 (shard reductions issued during the backward pass,
    two micro-batches per rank) against forward_backward + tl_zero1_step: at
    two ranks every sum has two terms, so the results are the same bits."""
    _torchrun([str(tmp_path), "overlap"], 29545)
