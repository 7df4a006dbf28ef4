"""tl_grad_norm_noalloc: the gradient norm for callers that cannot allocate
device memory (a host framework whose allocator owns the whole GPU, or a
runtime that fixes its memory budget at start-up).  It must give the same norm
as tl_grad_norm and as the oracle, through the C ABI, on two calls in a row that share its fixed
scratch array, and refuse sizes beyond that array's limit.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process (the
no-alloc call is made first, before anything calls tl_init)."""
import ctypes

import pytest
import torch

import oracle
from helpers import NORM_RTOL
from tinylm_c_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_noalloc_norm_matches_grad_norm_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L = _lib.lib()
    gen = torch.Generator(device=dev).manual_seed(123)
    # two calls in a row: an aligned buffer spanning 17 chunks, then an
    # unaligned, ragged one spanning 4 chunks (leftover partials from the
    # first call must not leak into the second)
    cases = [((1 << 20) + 7, 0, 1e-3), (3 * 65536 + 5, 1, 2.0)]
    got = []
    for n, offset, scale in cases:
        g = (torch.randn(n + offset, generator=gen, device=dev) * scale)[offset:]
        out = torch.full((1,), -1.0, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(L.tl_grad_norm_noalloc(g.data_ptr(), n, out.data_ptr(), stream))
        got.append((g, n, out))
    torch.cuda.synchronize()
    ops.init(0)  # the existing entry point needs its context
    for g, n, out in got:
        ref = torch.zeros(1, device=dev)
        _lib.check(L.tl_grad_norm(g.data_ptr(), n, ref.data_ptr()))
        torch.cuda.synchronize()
        assert out.item() == pytest.approx(ref.item(), rel=NORM_RTOL), (n, out.item(), ref.item())
        # and against the oracle's norm of the same values (double sum, one rounding)
        want = oracle.grad_norm(g.cpu().numpy())
        assert out.item() == pytest.approx(want, rel=NORM_RTOL), (n, out.item(), want)
        assert out.item() > 0


def test_noalloc_norm_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    L = _lib.lib()
    out = torch.zeros(1, device="cuda:0")
    rc = L.tl_grad_norm_noalloc(out.data_ptr(), (1 << 30) + 1, out.data_ptr(), None)
    assert rc == _lib.TL_EINVAL
    assert b"limit" in L.tl_last_error()
