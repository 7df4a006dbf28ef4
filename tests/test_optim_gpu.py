"""Parity of the fused AdamW + clip and the grad norm (CUDA, through the C ABI)
against the reference's own outputs (golden fixtures) and the oracle."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import NORM_RTOL, assert_adamw_close
from tinylm_c_b200 import TLError, ops
from tinylm_c_b200 import _lib

pytestmark = pytest.mark.gpu
LR, B1, B2, WD = 3e-4, 0.9, 0.95, 0.1


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("case", ["t1", "t100", "clip"])
def test_adamw_matches_reference_fixture(cuda, golden, case):
    z = golden("adamw")
    p, g, m, v = (dev(z[f"{case}_{k}"], cuda) for k in "pgmv")
    g0 = g.clone()
    n = p.numel()
    ops.adamw(p, g, m, v, n, LR, B1, B2, WD, int(z[f"{case}_t"][0]), float(z[f"{case}_gscale"][0]))
    torch.cuda.synchronize()
    assert torch.equal(g, g0), "AdamW must not modify G"
    assert_adamw_close(p.cpu().numpy(), z[f"{case}_P"], z[f"{case}_p"], "P")
    assert_adamw_close(m.cpu().numpy(), z[f"{case}_M"], z[f"{case}_m"], "M")
    assert_adamw_close(v.cpu().numpy(), z[f"{case}_V"], z[f"{case}_v"], "V")


@pytest.mark.parametrize("case", ["t1", "clip"])
def test_clip_adamw_on_device_matches_reference_fixture(cuda, golden, case):
    """norm -> clip -> AdamW with no host round trip (train_loop 2630-2633)."""
    z = golden("adamw")
    p, g, m, v = (dev(z[f"{case}_{k}"], cuda) for k in "pgmv")
    norm = torch.zeros(1, device=cuda)
    ops.clip_adamw(p, g, m, v, p.numel(), LR, B1, B2, WD, int(z[f"{case}_t"][0]), 1.0, norm)
    torch.cuda.synchronize()
    assert norm.item() == pytest.approx(float(z[f"{case}_gnorm"][0]), rel=NORM_RTOL)
    assert_adamw_close(p.cpu().numpy(), z[f"{case}_P"], z[f"{case}_p"], "P")
    assert_adamw_close(m.cpu().numpy(), z[f"{case}_M"], z[f"{case}_m"], "M")
    assert_adamw_close(v.cpu().numpy(), z[f"{case}_V"], z[f"{case}_v"], "V")


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 7, 8, 9, 31, 1023, 4097])
@pytest.mark.parametrize("offset", [0, 1, 2, 3])
def test_adamw_ragged_and_unaligned(cuda, n, offset):
    """Tails that are not a multiple of 4 and buffers that do not start on a
    16-byte boundary take the scalar path; results equal the oracle's."""
    p, g, m, v = oracle.adamw_inputs(n + offset, seed=n * 7 + offset)
    ref = [x[offset:].copy() for x in (p, g, m, v)]
    oracle.adamw(*ref, LR, B1, B2, WD, 3, 0.75)
    tp, tg, tm, tv = (dev(x, cuda) for x in (p, g, m, v))
    ops.adamw(tp[offset:], tg[offset:], tm[offset:], tv[offset:], n, LR, B1, B2, WD, 3, 0.75)
    torch.cuda.synchronize()
    assert_adamw_close(tp[offset:].cpu().numpy(), ref[0], p[offset:], "P")
    assert_adamw_close(tm[offset:].cpu().numpy(), ref[2], m[offset:], "M")
    assert_adamw_close(tv[offset:].cpu().numpy(), ref[3], v[offset:], "V")
    # the element in front of the view is untouched
    if offset:
        assert tp[offset - 1].item() == p[offset - 1]


def test_adamw_empty_and_bad_arguments(cuda):
    t = torch.zeros(8, device=cuda)
    ops.adamw(t, t, t, t, 0, LR, B1, B2, WD, 1, 1.0)          # n = 0: no-op
    with pytest.raises(TLError) as e:
        ops.adamw(t, t, t, t, 8, LR, B1, B2, WD, 0, 1.0)      # t must be >= 1
    assert e.value.code == _lib.TL_EINVAL
    host = np.zeros(8, np.float32)
    rc = _lib.lib().tl_adamw_step(host.ctypes.data, t.data_ptr(), t.data_ptr(), t.data_ptr(), 8,
                                  LR, B1, B2, WD, 1, 1.0)
    assert rc == _lib.TL_EPTR                                # no CPU fallback


def test_gradnorm_matches_reference_fixture(cuda, golden):
    z = golden("gradnorm")
    for i, n in enumerate(z["sizes"]):
        n = int(n)
        if f"g{i}" in z:
            g = z[f"g{i}"]
        else:  # the 2^20 vector is regenerated from the fixture's rng stream
            continue
        t = dev(g, cuda) if n else torch.zeros(1, device=cuda)
        got = ops.global_gradnorm(t, n)
        assert got == pytest.approx(float(z["norms"][i]), rel=NORM_RTOL, abs=0), (i, n)


@pytest.mark.parametrize("offset", [0, 1, 3])
def test_gradnorm_unaligned_and_deterministic(cuda, offset):
    rng = np.random.default_rng(5)
    g = rng.standard_normal((1 << 20) + 5, dtype=np.float32)
    t = dev(g, cuda)[offset:]
    want = oracle.grad_norm(np.ascontiguousarray(g[offset:]))
    a = ops.global_gradnorm(t, t.numel())
    b = ops.global_gradnorm(t, t.numel())
    assert a == b, "fixed-order reduction must be deterministic"
    assert a == pytest.approx(want, rel=NORM_RTOL)


def test_sumsq_and_clip_scale(cuda):
    rng = np.random.default_rng(9)
    g = rng.standard_normal(100003, dtype=np.float32) * np.float32(0.01)
    t = dev(g, cuda)
    s = torch.zeros(1, dtype=torch.float64, device=cuda)
    _lib.check(_lib.lib().tl_grad_sumsq(t.data_ptr(), t.numel(), s.data_ptr()))
    nrm = torch.zeros(1, device=cuda)
    gs = torch.zeros(1, device=cuda)
    _lib.check(_lib.lib().tl_clip_scale(s.data_ptr(), 1.0, nrm.data_ptr(), gs.data_ptr()))
    torch.cuda.synchronize()
    want = oracle.sumsq(g)
    assert s.item() == pytest.approx(want, rel=1e-12)
    assert nrm.item() == pytest.approx(oracle.grad_norm(g), rel=NORM_RTOL)
    assert gs.item() == pytest.approx(oracle.clip_scale(nrm.item()), rel=1e-7)
    assert gs.item() < 1.0   # norm ~3.2 -> clipped


def test_config2_full_size_properties(cuda):
    """BASELINE config 2 at its full size (2^28 fp32 each): the fused norm ->
    clip -> AdamW against the oracle on a strided sample (AdamW is elementwise,
    so the sample is exact), and the norm against a float64 numpy sum."""
    n = 1 << 28
    free, _ = torch.cuda.mem_get_info()
    if free < 6 * n * 4:
        pytest.skip("needs ~6.5 GB free")
    p, g, m, v = oracle.adamw_inputs(n, seed=0)
    want_norm = float(np.sqrt(np.sum(np.square(g, dtype=np.float64))))
    tp, tg, tm, tv = (dev(x, cuda) for x in (p, g, m, v))
    norm = torch.zeros(1, device=cuda)
    ops.clip_adamw(tp, tg, tm, tv, n, LR, B1, B2, WD, 100, 1.0, norm)
    torch.cuda.synchronize()
    assert norm.item() == pytest.approx(want_norm, rel=1e-6)
    gs = oracle.clip_scale(np.float32(norm.item()))
    idx = np.arange(0, n, 9973)
    sp, sg, sm, sv = (np.ascontiguousarray(x[idx]) for x in (p, g, m, v))
    P0 = sp.copy()
    oracle.adamw(sp, sg, sm, sv, LR, B1, B2, WD, 100, gs)
    ii = torch.from_numpy(idx).to(cuda)
    assert_adamw_close(tp[ii].cpu().numpy(), sp, P0, "P(sample)")
    assert_adamw_close(tm[ii].cpu().numpy(), sm, m[idx], "M(sample)")
    assert_adamw_close(tv[ii].cpu().numpy(), sv, v[idx], "V(sample)")
