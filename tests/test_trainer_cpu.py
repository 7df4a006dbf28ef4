"""Host-side pieces of the training loop against the reference (CPU only):
the learning-rate schedule, the batch sampler, and the TLM4 / TOPT checkpoint
formats read and written both ways."""
import ctypes
import os

import numpy as np
import pytest

import oracle
from tinylm_c_b200 import _lib, model, trainer

L = _lib.lib()


@pytest.mark.parametrize("iters,warmup", [(1000, 200.0), (150, 200.0), (5, 1.0), (200, 200.0)])
def test_lr_schedule_matches_reference(iters, warmup):
    """train_loop's schedule (tinylm.c:2587-2590), every iteration, within one
    float ulp (the builds differ in fused multiply-add contraction)."""
    P = oracle.port()
    for it in range(iters + 1):
        a = np.float32(L.tl_lr_at(it, 3e-4, iters, warmup))
        b = np.float32(P.tlo_lr_at(it, 3e-4, iters, warmup))
        assert abs(a - b) <= np.spacing(b), (it, a, b)


def _xorshift(s):
    M = (1 << 64) - 1
    s ^= (s << 13) & M
    s ^= s >> 7
    s ^= (s << 17) & M
    return s


@pytest.mark.parametrize("val,n_mtp", [(0, 0), (0, 2), (1, 0)])
def test_sampler_matches_reference_recipe(val, n_mtp):
    """Windows of train_loop (tinylm.c:2596-2597 validation, 2623-2626
    training), drawn with the reference generator."""
    rng = np.random.default_rng(4)
    stream = rng.integers(0, 2048, 5000).astype(np.uint16)
    B, T = 3, 256
    st = ctypes.c_ulonglong(12345)
    tok = np.empty(B * T, np.int32); tgt = np.empty(B * T, np.int32); mtp = np.empty(max(n_mtp, 1) * B * T, np.int32)
    _lib.check(L.tl_sample_windows(ctypes.byref(st), stream.ctypes.data, stream.size, B, T, n_mtp, val,
                                   tok.ctypes.data, tgt.ctypes.data, mtp.ctypes.data))
    s = 12345
    span = T + 1 if val else T + n_mtp + 2
    for i in range(B):
        s = _xorshift(s)
        start = s % (stream.size - span)
        assert (tok[i * T:(i + 1) * T] == stream[start:start + T]).all()
        assert (tgt[i * T:(i + 1) * T] == stream[start + 1:start + T + 1]).all()
        if not val:
            for k in range(n_mtp):
                assert (mtp[k * B * T + i * T:k * B * T + (i + 1) * T] == stream[start + 2 + k:start + 2 + k + T]).all()
    assert st.value == s


def test_bundle_round_trip_and_reference_reads_it(tmp_path):
    import torch
    cfg = model.cfg8("nano", 0)
    P = model.init_params(cfg, 3)
    path = str(tmp_path / "m.bin")
    trainer.save_bundle(path, cfg, P, P.numel(), eot=7, tmpl=1, tok_blob=b"TLTKxyz")
    data = open(path, "rb").read()
    hdr = np.frombuffer(data[4:48], np.int32)
    assert data[:4] == b"TLM4" and list(hdr) == [512, 64, 4, 4, 2, 176, 256, 7, 1, 0, 0]
    assert np.array_equal(np.frombuffer(data[48:48 + 4 * P.numel()], np.float32), P.numpy())
    assert data[48 + 4 * P.numel():] == np.int32(7).tobytes() + b"TLTKxyz"
    Q = torch.zeros_like(P)
    h = trainer.load_bundle(path, Q)
    assert h["eot"] == 7 and h["tmpl"] == 1 and torch.equal(P, Q)
    if oracle.has_ref():      # the reference's own model_load (tinylm.c:1915-1938)
        R = oracle.ref()
        c11 = (ctypes.c_int * 11)()
        Pr = np.empty(P.numel(), np.float32)
        n = R.tlref_model_load(path.encode(), c11, oracle.fptr(Pr), Pr.size)
        assert n == P.numel() and list(c11) == [512, 64, 4, 4, 2, 176, 256, 7, 1, 0, 0]
        assert np.array_equal(Pr, P.numpy())


def test_opt_sidecar_by_shards_equals_one_write(tmp_path):
    n = 10007
    rng = np.random.default_rng(1)
    M = rng.standard_normal(n, dtype=np.float32)
    V = rng.standard_normal(n, dtype=np.float32)
    one, two = str(tmp_path / "a.opt"), str(tmp_path / "b.opt")
    _lib.check(L.tl_ckpt_opt_create(one.encode(), 42, n))
    _lib.check(L.tl_ckpt_opt_write(one.encode(), n, 0, M.ctypes.data, V.ctypes.data, n))
    _lib.check(L.tl_ckpt_opt_create(two.encode(), 42, n))
    shard = 4096                       # ZeRO-1 style ranges, last one ragged
    for lo in range(0, n, shard):
        cnt = min(shard, n - lo)
        _lib.check(L.tl_ckpt_opt_write(two.encode(), n, lo, M[lo:].ctypes.data, V[lo:].ctypes.data, cnt))
    a, b = open(one, "rb").read(), open(two, "rb").read()
    assert a == b == b"TOPT" + np.int32(42).tobytes() + M.tobytes() + V.tobytes()
    Mr = np.empty(100, np.float32); Vr = np.empty(100, np.float32); it = ctypes.c_int(0)
    _lib.check(L.tl_ckpt_opt_read(two.encode(), n, 9000, Mr.ctypes.data, Vr.ctypes.data, 100, ctypes.byref(it)))
    assert it.value == 42 and np.array_equal(Mr, M[9000:9100]) and np.array_equal(Vr, V[9000:9100])
    assert L.tl_ckpt_opt_write(two.encode(), n, n - 5, M.ctypes.data, V.ctypes.data, 6) == _lib.TL_EINVAL


@pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")
def test_reference_written_checkpoint_reads_back(tmp_path):
    """Files written by the reference's own train_loop load through the
    library: header, parameters and the TOPT iteration / moments."""
    rng = np.random.default_rng(0)
    tr = rng.integers(0, 512, 20000).astype(np.uint16)
    vl = rng.integers(0, 512, 5000).astype(np.uint16)
    out, opt = str(tmp_path / "r.bin"), str(tmp_path / "r.opt")
    oracle.ref().tlref_init(8, 0)
    oracle.ref_train([512, 64, 4, 4, 2, 176, 256], 0, 2, 2, 6e-4, 0, tr, vl, out, opt)
    import torch
    n = model.param_count(model.cfg8("nano", 0))
    P = torch.zeros(n)
    h = trainer.load_bundle(out, P)
    assert [h[k] for k in ("V", "D", "L", "H", "KV", "F", "T")] == [512, 64, 4, 4, 2, 176, 256]
    raw = open(out, "rb").read()
    assert np.array_equal(np.frombuffer(raw[48:48 + 4 * n], np.float32), P.numpy())
    M = np.empty(n, np.float32); V = np.empty(n, np.float32); it = ctypes.c_int(0)
    _lib.check(L.tl_ckpt_opt_read(opt.encode(), n, 0, M.ctypes.data, V.ctypes.data, n, ctypes.byref(it)))
    raw = open(opt, "rb").read()
    assert it.value == 2 and np.array_equal(M, np.frombuffer(raw[8:8 + 4 * n], np.float32))
