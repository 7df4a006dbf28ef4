"""Host-side mirror of the reference's hot-path primitives, on CUDA tensors.

Same names, argument order and meaning as tinylm.c's static functions, so a
test or a driver reads like the reference's own code:

    mm(Y, X, W, M, K, N)                          tinylm.c:439-478
    mm_bt(dX, dY, W, M, K, N)                     tinylm.c:480-508
    mm_atb(dW, X, dY, M, K, N)                    tinylm.c:510-537
    global_gradnorm(G, n) -> float                tinylm.c:1171-1176
    adamw(P, G, M, V, n, lr, b1, b2, wd, t, gscale)   tinylm.c:1159-1170

Buffers are torch CUDA float32 tensors (torch supplies device memory and the
stream; every byte of arithmetic runs in libtinylm_cuda).  A CPU tensor raises:
there is no CPU fallback.  Errors raise TLError instead of the reference's
exit(1).
"""
import ctypes

import torch

from ._lib import check, lib

_inited = set()
_stream_set = {}


def init(device=0):
    """tl_init for `device` and bind the library to torch's current stream there."""
    device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with torch.cuda.device(idx):
        if idx not in _inited:
            check(lib().tl_init(idx))
            _inited.add(idx)
        _bind_stream(idx)
    return idx


def _bind_stream(idx):
    s = torch.cuda.current_stream(idx).cuda_stream
    if _stream_set.get(idx) != s:
        check(lib().tl_set_stream(s))
        _stream_set[idx] = s


def _ptr(t, name, numel=None):
    if isinstance(t, int):
        return t
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a CUDA tensor or a device pointer")
    if not t.is_cuda:
        raise ValueError(f"{name}: CPU tensor given; libtinylm_cuda computes on the GPU only")
    if t.dtype != torch.float32:
        raise TypeError(f"{name}: expected float32, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name}: has {t.numel()} elements, call needs {numel}")
    return t.data_ptr()


def _prep(t):
    if isinstance(t, torch.Tensor) and not t.is_cuda:
        raise ValueError("CPU tensor given; libtinylm_cuda computes on the GPU only")
    idx = t.device.index if isinstance(t, torch.Tensor) else torch.cuda.current_device()
    if idx not in _inited:
        init(idx)
    else:
        _bind_stream(idx)


def mm(Y, X, W, M, K, N):
    """Y[M,N] = X[M,K] @ W[K,N] (overwrite)."""
    _prep(Y)
    check(lib().tl_matmul(_ptr(Y, "Y", M * N), _ptr(X, "X", M * K), _ptr(W, "W", K * N), M, K, N))


def mm_bt(dX, dY, W, M, K, N):
    """dX[M,K] += dY[M,N] @ W[K,N]^T (accumulate)."""
    _prep(dX)
    check(lib().tl_matmul_bt(_ptr(dX, "dX", M * K), _ptr(dY, "dY", M * N), _ptr(W, "W", K * N), M, K, N))


def mm_bt_sum(dX, dYs, Ws, Ns, M, K):
    """dX[M,K] = sum_t dYs[t][M,Ns[t]] @ Ws[t][K,Ns[t]]^T (overwrite), 1 to 3 products."""
    _prep(dX)
    n = len(Ns)
    if not (len(dYs) == len(Ws) == n):
        raise ValueError("dYs, Ws and Ns must have the same length")
    arr = ctypes.c_void_p * max(n, 1)
    a = arr(*[_ptr(x, "dY", M * nt) for x, nt in zip(dYs, Ns)])
    b = arr(*[_ptr(w, "W", K * nt) for w, nt in zip(Ws, Ns)])
    nn = (ctypes.c_int * max(n, 1))(*Ns)
    check(lib().tl_matmul_bt_sum(_ptr(dX, "dX", M * K), n, a, b, nn, M, K))


def mm_atb(dW, X, dY, M, K, N):
    """dW[K,N] += X[M,K]^T @ dY[M,N] (accumulate)."""
    _prep(dW)
    check(lib().tl_matmul_at(_ptr(dW, "dW", K * N), _ptr(X, "X", M * K), _ptr(dY, "dY", M * N), M, K, N))


def set_gemm_engine(engine):
    """0 automatic, 1 CUDA-core fp32, 2 tensor-core 3xTF32 (one CTA per
    128 x 128 tile), 3 tensor-core 3xTF32 (CTA pair per 256 x 256 tile),
    4 tensor-core CTA pair with scaled fp16 hi/lo operands (3 fp16 MMAs),
    5 tensor-core CTA pair with the hybrid split (tf32 hi*hi + bf16 cross
    terms)."""
    check(lib().tl_set_gemm_engine(int(engine)))


def set_attn_engine(engine):
    """Attention forward and backward: 0 automatic, 1 CUDA cores, 2 tensor
    cores (T=256, hd=64)."""
    check(lib().tl_set_attn_engine(int(engine)))


def last_gemm_engine():
    return lib().tl_last_gemm_engine()


def global_gradnorm(G, n):
    """sqrt(sum (double)G^2) as float; waits for the result like the reference."""
    _prep(G)
    out = ctypes.c_float(0.0)
    check(lib().tl_grad_norm(_ptr(G, "G", n), n, ctypes.addressof(out)))
    return out.value


def grad_norm_dev(G, n, out):
    """Device-side norm into out[0] (float32 CUDA tensor); no host sync."""
    _prep(G)
    check(lib().tl_grad_norm(_ptr(G, "G", n), n, _ptr(out, "out", 1)))


def adamw(P, G, M, V, n, lr, b1, b2, wd, t, gscale):
    """AdamW with the clip scale folded in (host scalar gscale)."""
    _prep(P)
    check(lib().tl_adamw_step(_ptr(P, "P", n), _ptr(G, "G", n), _ptr(M, "M", n), _ptr(V, "V", n), n,
                              lr, b1, b2, wd, int(t), gscale))


def adamw_dev(P, G, M, V, n, lr, b1, b2, wd, t, gscale_dev=None):
    """AdamW reading the clip scale from device memory (None = 1.0)."""
    _prep(P)
    gp = None if gscale_dev is None else _ptr(gscale_dev, "gscale_dev", 1)
    check(lib().tl_adamw_step_dev(_ptr(P, "P", n), _ptr(G, "G", n), _ptr(M, "M", n), _ptr(V, "V", n),
                                  n, lr, b1, b2, wd, int(t), gp))


def clip_adamw(P, G, M, V, n, lr, b1, b2, wd, t, max_norm=1.0, norm_out=None):
    """norm -> clip scale -> AdamW, all on the device (train_loop tinylm.c:2630-2633)."""
    _prep(P)
    no = None if norm_out is None else _ptr(norm_out, "norm_out", 1)
    check(lib().tl_clip_adamw_step(_ptr(P, "P", n), _ptr(G, "G", n), _ptr(M, "M", n), _ptr(V, "V", n),
                                   n, lr, b1, b2, wd, int(t), max_norm, no))


def sync():
    check(lib().tl_sync())
