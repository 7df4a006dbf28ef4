"""Parity of the three GEMM primitives (CUDA, through the C ABI) against the
reference's own outputs and a double-accumulated oracle.  Metric and bound:
max|err| / mean|ref| <= 1e-4 (the reference selftest's metric, tinylm.c:4778)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import GEMM_REL_TOL, gemm_rel
from test_oracle import regen_gemm_inputs
from tinylm_c_b200 import TLError, _lib, ops

pytestmark = pytest.mark.gpu
ENGINES = {"auto": 0, "cuda_core": 1}


def device_ok():
    """No bounded device-side wait expired in any kernel since the last check."""
    _lib.check(_lib.lib().tl_device_status())


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.fixture(params=list(ENGINES))
def engine(request, cuda):
    ops.set_gemm_engine(ENGINES[request.param])
    yield request.param
    ops.set_gemm_engine(0)


@pytest.mark.parametrize("name", ["gemm_selftest", "gemm_accum", "gemm_aligned"])
def test_gemms_match_reference_fixture(cuda, golden, engine, name):
    z = golden(name)
    M, K, N, X, W, dY, dX0, dW0 = regen_gemm_inputs(z)
    tX, tW, tdY = dev(X, cuda), dev(W, cuda), dev(dY, cuda)
    Y = torch.full((M * N,), float("nan"), device=cuda)
    dX, dW = dev(dX0, cuda), dev(dW0, cuda)
    ops.mm(Y, tX, tW, M, K, N)
    ops.mm_bt(dX, tdY, tW, M, K, N)
    ops.mm_atb(dW, tX, tdY, M, K, N)
    torch.cuda.synchronize()
    device_ok()
    # truth: double accumulation
    Y64 = np.empty(M * N, np.float32); oracle.mm(Y64, X, W, M, K, N, acc64=True)
    dX64 = dX0.copy(); oracle.mm_bt(dX64, dY, W, M, K, N, acc64=True)
    dW64 = dW0.copy(); oracle.mm_atb(dW64, X, dY, M, K, N, acc64=True)
    for got, fix, truth in ((Y, z["Y"], Y64), (dX, z["dX"], dX64), (dW, z["dW"], dW64)):
        g = got.cpu().numpy()
        assert np.isfinite(g).all()
        assert gemm_rel(g, fix) <= GEMM_REL_TOL
        assert gemm_rel(g, truth) <= GEMM_REL_TOL


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (5, 3, 2), (128, 64, 96), (130, 68, 100), (1000, 36, 72),
                                   (64, 2816, 32), (300, 256, 2048)])
def test_gemm_shapes_vs_oracle(cuda, engine, M, K, N):
    rng = np.random.default_rng(M * 31 + K * 7 + N)
    X = rng.standard_normal(M * K, dtype=np.float32)
    W = rng.standard_normal(K * N, dtype=np.float32) * np.float32(0.02)
    dY = rng.standard_normal(M * N, dtype=np.float32)
    dX0 = rng.standard_normal(M * K, dtype=np.float32)
    dW0 = rng.standard_normal(K * N, dtype=np.float32)
    Y = torch.empty(M * N, device=cuda)
    dX, dW = dev(dX0, cuda), dev(dW0, cuda)
    ops.mm(Y, dev(X, cuda), dev(W, cuda), M, K, N)
    ops.mm_bt(dX, dev(dY, cuda), dev(W, cuda), M, K, N)
    ops.mm_atb(dW, dev(X, cuda), dev(dY, cuda), M, K, N)
    torch.cuda.synchronize()
    device_ok()
    Y64 = np.empty(M * N, np.float32); oracle.mm(Y64, X, W, M, K, N, acc64=True)
    dX64 = dX0.copy(); oracle.mm_bt(dX64, dY, W, M, K, N, acc64=True)
    dW64 = dW0.copy(); oracle.mm_atb(dW64, X, dY, M, K, N, acc64=True)
    assert gemm_rel(Y.cpu().numpy(), Y64) <= GEMM_REL_TOL
    assert gemm_rel(dX.cpu().numpy(), dX64) <= GEMM_REL_TOL
    assert gemm_rel(dW.cpu().numpy(), dW64) <= GEMM_REL_TOL


def test_gemm_empty_dims(cuda):
    Y = torch.full((12,), 5.0, device=cuda)
    z = torch.zeros(16, device=cuda)
    ops.mm(Y, z, z, 3, 0, 4)            # empty reduction: mm overwrites with zeros
    dX = torch.full((12,), 5.0, device=cuda)
    ops.mm_bt(dX, z, z, 3, 4, 0)        # accumulate forms leave the output alone
    ops.mm_atb(dX, z, z, 0, 3, 4)
    ops.mm(z, z, z, 0, 4, 4)            # no rows: nothing to do
    torch.cuda.synchronize()
    assert torch.all(Y == 0) and torch.all(dX == 5)


def test_gemm_rejects_host_memory(cuda):
    Y = torch.zeros(4)
    with pytest.raises(ValueError):
        ops.mm(Y, Y, Y, 2, 2, 2)
    with pytest.raises(TLError):
        X = np.zeros(4, np.float32)
        ops.mm(torch.zeros(4, device=cuda), X.ctypes.data, X.ctypes.data, 2, 2, 2)


TC_ENGINES = {"tc_1cta": 2, "tc_pair": 3, "tc_pair_f16": 4, "tc_pair_hyb": 5}


@pytest.mark.parametrize("tc_engine", list(TC_ENGINES))
@pytest.mark.parametrize("M,K,N", [(128, 32, 128), (256, 64, 256), (130, 68, 100), (1000, 36, 72), (257, 1024, 2816),
                                   (384, 8, 520), (100, 4096, 260)])
def test_tensor_core_engine_forced(cuda, tc_engine, M, K, N):
    """Each tcgen05 3xTF32 kernel alone (engine 2: one CTA per 128 x 128
    tile; engine 3: a CTA pair per 256 x 256 tile) on aligned shapes,
    including partial tiles in every dimension, a pair whose second CTA has
    no rows (M=100) and split-K (K=4096 with few tiles)."""
    eng = TC_ENGINES[tc_engine]
    ops.set_gemm_engine(eng)
    try:
        rng = np.random.default_rng(M + K + N)
        X = rng.standard_normal(M * K, dtype=np.float32)
        W = rng.standard_normal(K * N, dtype=np.float32) * np.float32(0.02)
        dY = rng.standard_normal(M * N, dtype=np.float32)
        dX0 = rng.standard_normal(M * K, dtype=np.float32)
        dW0 = rng.standard_normal(K * N, dtype=np.float32)
        Y = torch.full((M * N,), float("nan"), device=cuda)
        dX, dW = dev(dX0, cuda), dev(dW0, cuda)
        ops.mm(Y, dev(X, cuda), dev(W, cuda), M, K, N)
        assert ops.last_gemm_engine() == eng
        ops.mm_bt(dX, dev(dY, cuda), dev(W, cuda), M, K, N)
        assert ops.last_gemm_engine() == eng
        ops.mm_atb(dW, dev(X, cuda), dev(dY, cuda), M, K, N)
        assert ops.last_gemm_engine() == eng
        torch.cuda.synchronize()
        device_ok()
    finally:
        ops.set_gemm_engine(0)
    Xd, Wd, dYd = (a.astype(np.float64) for a in (X, W, dY))
    Y64 = (Xd.reshape(M, K) @ Wd.reshape(K, N)).ravel()
    dX64 = dX0 + (dYd.reshape(M, N) @ Wd.reshape(K, N).T).ravel()
    dW64 = dW0 + (Xd.reshape(M, K).T @ dYd.reshape(M, N)).ravel()
    assert gemm_rel(Y.cpu().numpy(), Y64) <= GEMM_REL_TOL
    assert gemm_rel(dX.cpu().numpy(), dX64) <= GEMM_REL_TOL
    assert gemm_rel(dW.cpu().numpy(), dW64) <= GEMM_REL_TOL


@pytest.mark.parametrize("eng", [0, 1, 3, 4, 5])
@pytest.mark.parametrize("M,K,Ns", [(512, 384, (96, 40, 72)), (300, 260, (256, 512)), (256, 256, (2048, 1024, 1024)),
                                    (100, 64, (64, 64, 64)), (384, 256, (64, 0, 32)), (257, 1024, (2816,))])
def test_mm_bt_sum(cuda, eng, M, K, Ns):
    """dX = sum_t dY_t @ W_t^T as one pair launch walking the products'
    k-blocks (engine 3, and auto where the pair kernel takes the shape), or
    consecutive mm_bt: reductions that end inside a k-block (N=40, 72), a
    product with no columns, partial tiles and split-K (few output tiles,
    long reduction)."""
    rng = np.random.default_rng(M + K + sum(Ns))
    dYs = [rng.standard_normal(M * n, dtype=np.float32) for n in Ns]
    Ws = [rng.standard_normal(K * n, dtype=np.float32) * np.float32(0.02) for n in Ns]
    dX = torch.full((M * K,), float("nan"), device=cuda)
    ops.set_gemm_engine(eng)
    try:
        ops.mm_bt_sum(dX, [dev(a, cuda) for a in dYs], [dev(w, cuda) for w in Ws], list(Ns), M, K)
        last = ops.last_gemm_engine()
        torch.cuda.synchronize()
        device_ok()
    finally:
        ops.set_gemm_engine(0)
    if eng in (3, 4, 5):
        assert last == eng
    elif eng == 0 and M > 128 and K > 128:
        assert last == 3
    want = np.zeros((M, K))
    for a, w, n in zip(dYs, Ws, Ns):
        want += a.astype(np.float64).reshape(M, n) @ w.astype(np.float64).reshape(K, n).T
    assert gemm_rel(dX.cpu().numpy(), want.ravel()) <= GEMM_REL_TOL


@pytest.mark.parametrize("eng", [4, 5])
@pytest.mark.parametrize("sa,sb", [(1e5, 1e-7), (1e-20, 1e15), (3e4, 3e4), (0.0, 1.0)])
def test_f16_split_operand_scales(cuda, eng, sa, sb):
    """The fp16-split pair kernel (engine 4) scales each operand by a power of
    two from its max |x|; the hybrid split (engine 5) keeps fp32's exponent
    range in bf16.  Operands far outside fp16's range, tiny ones, a product
    whose scales differ by 2^90, and an all-zero operand keep the 1e-4
    bound, on all three primitives and on a summed mm_bt whose products have
    different magnitudes."""
    M, K, N = 384, 320, 288
    rng = np.random.default_rng(7)
    X = (rng.standard_normal(M * K) * sa).astype(np.float32)
    W = (rng.standard_normal(K * N) * sb).astype(np.float32)
    dY = (rng.standard_normal(M * N) * sb).astype(np.float32)
    Y = torch.full((M * N,), float("nan"), device=cuda)
    dX, dW = torch.zeros(M * K, device=cuda), torch.zeros(K * N, device=cuda)
    W2 = (rng.standard_normal(K * 64) * sa).astype(np.float32)
    dY2 = (rng.standard_normal(M * 64)).astype(np.float32)
    dXs = torch.full((M * K,), float("nan"), device=cuda)
    ops.set_gemm_engine(eng)
    try:
        ops.mm(Y, dev(X, cuda), dev(W, cuda), M, K, N)
        ops.mm_bt(dX, dev(dY, cuda), dev(W, cuda), M, K, N)
        ops.mm_atb(dW, dev(X, cuda), dev(dY, cuda), M, K, N)
        ops.mm_bt_sum(dXs, [dev(dY, cuda), dev(dY2, cuda)], [dev(W, cuda), dev(W2, cuda)], [N, 64], M, K)
        torch.cuda.synchronize()
        device_ok()
    finally:
        ops.set_gemm_engine(0)
    Xd, Wd, dYd = (a.astype(np.float64) for a in (X, W, dY))
    checks = [(Y, (Xd.reshape(M, K) @ Wd.reshape(K, N)).ravel()),
              (dX, (dYd.reshape(M, N) @ Wd.reshape(K, N).T).ravel()),
              (dW, (Xd.reshape(M, K).T @ dYd.reshape(M, N)).ravel()),
              (dXs, (dYd.reshape(M, N) @ Wd.reshape(K, N).T
                     + dY2.astype(np.float64).reshape(M, 64) @ W2.astype(np.float64).reshape(K, 64).T).ravel())]
    for got, want in checks:
        g = got.cpu().numpy()
        assert np.isfinite(g).all()
        if not np.any(want):
            assert not np.any(g)
        else:
            assert gemm_rel(g, want) <= GEMM_REL_TOL


@pytest.mark.parametrize("eng", [0, 4, 5])
@pytest.mark.parametrize("M,K,Ns,accumulate", [(16384, 1024, (1024, 256, 256), False), (16384, 1024, (2816, 2816), False),
                                               (16384, 1024, (1024,), True), (65536, 256, (256,), True),
                                               (16128, 1000, (512,), False)])
def test_tail_split_tiles(cuda, eng, M, K, Ns, accumulate):
    """Outputs of 256 (or 252) pair tiles fill three waves of resident CTA
    pairs and leave a partial one: the last tiles run as two pairs over half
    the reduction each, summed by the tail pass.  The config-5 attention and
    FFN input-norm gradients (summed products), an accumulating mm_bt, and
    ragged edges (16128 x 1000), against float64 on sampled rows."""
    g = torch.Generator(device=cuda).manual_seed(M + K + sum(Ns))
    dYs = [torch.randn(M * n, device=cuda, generator=g) for n in Ns]
    Ws = [torch.randn(K * n, device=cuda, generator=g) * 0.02 for n in Ns]
    dX0 = torch.randn(M * K, device=cuda, generator=g) * 0.1
    dX = dX0.clone()
    ops.set_gemm_engine(eng)
    try:
        if accumulate:
            ops.mm_bt(dX, dYs[0], Ws[0], M, K, Ns[0])
        else:
            ops.mm_bt_sum(dX, dYs, Ws, list(Ns), M, K)
        torch.cuda.synchronize()
        device_ok()
    finally:
        ops.set_gemm_engine(0)
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(K))[:256].sort().values.to(cuda)
    want = dX0.view(M, K)[rows].double() if accumulate else torch.zeros(256, K, device=cuda, dtype=torch.float64)
    for a, w, n in zip(dYs, Ws, Ns):
        want += a.view(M, n)[rows].double() @ w.view(K, n).double().T
    assert gemm_rel(dX.view(M, K)[rows].cpu().numpy(), want.cpu().numpy()) <= GEMM_REL_TOL
    # rows of the last tiles (the tail) too
    tail = dX.view(M, K)[-256:].double()
    want_t = dX0.view(M, K)[-256:].double() if accumulate else torch.zeros(256, K, device=cuda, dtype=torch.float64)
    for a, w, n in zip(dYs, Ws, Ns):
        want_t += a.view(M, n)[-256:].double() @ w.view(K, n).double().T
    assert gemm_rel(tail.cpu().numpy(), want_t.cpu().numpy()) <= GEMM_REL_TOL


def test_mm_bt_sum_rejects_bad_args(cuda):
    z = torch.zeros(64, device=cuda)
    with pytest.raises(TLError):
        ops.mm_bt_sum(z, [z] * 4, [z] * 4, [4] * 4, 4, 4)   # at most three products
    with pytest.raises(TLError):
        ops.mm_bt_sum(z, [z], [z], [-1], 4, 4)


@pytest.mark.parametrize("tc_engine", list(TC_ENGINES))
def test_tensor_core_engine_rejects_unaligned(cuda, tc_engine):
    ops.set_gemm_engine(TC_ENGINES[tc_engine])
    try:
        z = torch.zeros(201 * 259, device=cuda)
        with pytest.raises(TLError):
            ops.mm(z, z, z, 201, 131, 259)      # K=131: rows not 16-byte multiples
    finally:
        ops.set_gemm_engine(0)


@pytest.mark.parametrize("tc_engine", list(TC_ENGINES))
@pytest.mark.parametrize("M,K,N", [(16384, 1024, 1024), (16384, 256, 2816), (65536, 512, 256)])
def test_gemm_sweep_shapes_sampled(cuda, tc_engine, M, K, N):
    """BASELINE config-3 shapes at full size on each tensor-core kernel,
    checked on sampled rows/columns against float64 (rows of Y and dX,
    columns of dW, are independent)."""
    ops.set_gemm_engine(TC_ENGINES[tc_engine])
    try:
        _sweep_shape_sampled(cuda, M, K, N)
    finally:
        ops.set_gemm_engine(0)


SWEEP = [(M, K, N) for M in (16384, 65536) for K in (256, 512, 1024, 2816) for N in (256, 512, 1024, 2816)]


@pytest.mark.parametrize("M,K,N", SWEEP)
def test_gemm_sweep_every_shape_default_engine(cuda, M, K, N):
    """All 32 (M, K, N) shapes of BASELINE config 3 x the three primitives on
    the engine the library picks by itself, at full size, against float64
    products of sampled rows (Y, dX) and columns (dW) computed on the device."""
    # Independent draws for X, W and dY (equal seeds would make mm_atb a Gram
    # matrix whose diagonal dwarfs the mean the metric divides by).
    base = 3 * M + 5 * K + 7 * N
    X = torch.randn(M * K, device=cuda, generator=torch.Generator(device=cuda).manual_seed(base))
    W = torch.randn(K * N, device=cuda, generator=torch.Generator(device=cuda).manual_seed(base + 1)) * 0.02
    dY = torch.randn(M * N, device=cuda, generator=torch.Generator(device=cuda).manual_seed(base + 2))
    Y = torch.empty(M * N, device=cuda)
    dX = torch.randn(M * K, device=cuda, generator=torch.Generator(device=cuda).manual_seed(7)) * 0.1
    dW = torch.randn(K * N, device=cuda, generator=torch.Generator(device=cuda).manual_seed(8)) * 0.1
    dX0, dW0 = dX.double(), dW.double()          # the accumulate primitives add to what is there
    ops.mm(Y, X, W, M, K, N)
    ops.mm_bt(dX, dY, W, M, K, N)
    ops.mm_atb(dW, X, dY, M, K, N)
    torch.cuda.synchronize()
    device_ok()
    g = torch.Generator(device="cpu").manual_seed(M * 7 + K * 3 + N)
    rows = torch.randperm(M, generator=g)[:128].sort().values.to(cuda)
    cols = torch.randperm(N, generator=g)[:32].sort().values.to(cuda)
    Xd, Wd, dYd = X.view(M, K).double(), W.view(K, N).double(), dY.view(M, N).double()
    want_y = Xd[rows] @ Wd
    want_dx = dX0.view(M, K)[rows] + dYd[rows] @ Wd.T
    want_dw = dW0.view(K, N)[:, cols] + Xd.T @ dYd[:, cols]
    for got, want in ((Y.view(M, N)[rows], want_y), (dX.view(M, K)[rows], want_dx), (dW.view(K, N)[:, cols], want_dw)):
        assert torch.isfinite(got).all()
        assert gemm_rel(got.cpu().numpy(), want.cpu().numpy()) <= GEMM_REL_TOL


def _sweep_shape_sampled(cuda, M, K, N):
    rng = np.random.default_rng(3)
    X = torch.randn(M * K, device=cuda, generator=torch.Generator(device=cuda).manual_seed(1))
    W = torch.randn(K * N, device=cuda, generator=torch.Generator(device=cuda).manual_seed(2)) * 0.02
    dY = torch.randn(M * N, device=cuda, generator=torch.Generator(device=cuda).manual_seed(3))
    Y = torch.empty(M * N, device=cuda)
    dX = torch.zeros(M * K, device=cuda)
    dW = torch.zeros(K * N, device=cuda)
    ops.mm(Y, X, W, M, K, N)
    ops.mm_bt(dX, dY, W, M, K, N)
    ops.mm_atb(dW, X, dY, M, K, N)
    torch.cuda.synchronize()
    device_ok()
    rows = np.sort(rng.choice(M, 64, replace=False))
    cols = np.sort(rng.choice(N, 16, replace=False))
    Xh = X.view(M, K).double().cpu().numpy()
    Wh = W.view(K, N).double().cpu().numpy()
    dYh = dY.view(M, N).double().cpu().numpy()
    assert gemm_rel(Y.view(M, N)[rows].cpu().numpy(), Xh[rows] @ Wh) <= GEMM_REL_TOL
    assert gemm_rel(dX.view(M, K)[rows].cpu().numpy(), dYh[rows] @ Wh.T) <= GEMM_REL_TOL
    assert gemm_rel(dW.view(K, N)[:, cols].cpu().numpy(), Xh.T @ dYh[:, cols]) <= GEMM_REL_TOL
