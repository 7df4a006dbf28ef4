"""TEST INFRASTRUCTURE ONLY -- the parity oracle.

Two CPU legs, loaded with ctypes:
  port() -> oracle/libtl_oracle.so   my C restatement of the reference's hot-path
                                     arithmetic (oracle/tl_oracle.c)
  ref()  -> oracle/_ref/libtlref.so  the reference's own tinylm.c compiled
                                     unmodified (oracle/Makefile, ref_harness.c)
and the drop-in proof (oracle/dropin_patch.py, `make dropin`): the reference
with libtinylm_cuda at its five seams, as the CLI oracle/_ref/tinylm_cuda and
the harness oracle/_ref/libtlref_cuda.so (DROPIN_* paths below).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this package, and only as the checker or the timed CPU baseline; the product
(tinylm_c_b200/) never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(HERE, "libtl_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libtlref.so")
DROPIN_EXE = os.path.join(HERE, "_ref", "tinylm_cuda")
DROPIN_LIB = os.path.join(HERE, "_ref", "libtlref_cuda.so")
# Where the reference sources are read at build time (overridable, like the
# Makefile's REF_DIR).  Machines without them use the prebuilt _ref files.
REF_DIR = os.environ.get("TL_REF_DIR", "/root/reference")
REF_SRC = os.path.join(REF_DIR, "tinylm.c")

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)
_f, _i, _sz, _u64, _d = ctypes.c_float, ctypes.c_int, ctypes.c_size_t, ctypes.c_ulonglong, ctypes.c_double


def build(ref=True):
    """Compile the restatement and, when the reference sources are present, the
    reference leg and the drop-in build (which links the in-tree
    libtinylm_cuda.so, so build that first).  On a machine without the sources
    the prebuilt _ref files are used."""
    targets = ["port"]
    if ref and os.path.exists(REF_SRC):
        targets += ["ref", "dropin"]
    subprocess.run(["make", "-s", "-C", HERE, "REF_DIR=" + REF_DIR] + targets, check=True)


def fptr(a):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


_port = None
_ref = None


def port():
    global _port
    if _port is None:
        if not os.path.exists(PORT_PATH):
            build(ref=False)
        L = ctypes.CDLL(PORT_PATH)
        L.tlo_adamw.argtypes = [_fp, _fp, _fp, _fp, _sz, _f, _f, _f, _f, _i, _f]
        L.tlo_grad_norm.argtypes = [_fp, _sz]
        L.tlo_grad_norm.restype = _f
        L.tlo_sumsq.argtypes = [_fp, _sz]
        L.tlo_sumsq.restype = _d
        L.tlo_clip_scale.argtypes = [_f]
        L.tlo_clip_scale.restype = _f
        for nm in ("tlo_mm", "tlo_mm_bt", "tlo_mm_atb"):
            getattr(L, nm).argtypes = [_fp, _fp, _fp, _i, _i, _i, _i]
        L.tlo_rel_err.argtypes = [_fp, _fp, _sz, ctypes.POINTER(_d)]
        L.tlo_rel_err.restype = _d
        L.tlo_seed.argtypes = [_u64]
        L.tlo_xorshift.restype = _u64
        L.tlo_fill_normal.argtypes = [_fp, _sz, _f]
        L.tlo_lr_at.argtypes = [_i, _f, _i, _f]
        L.tlo_lr_at.restype = _f
        _port = L
    return _port


def has_ref():
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            raise FileNotFoundError(f"{REF_PATH} not built (needs the reference sources)")
        _ref = _bind_ref(ctypes.CDLL(REF_PATH))
    return _ref


def has_dropin():
    return os.path.exists(DROPIN_EXE) and os.path.exists(DROPIN_LIB)


def ref_cuda():
    """The drop-in harness: the reference's step with its GEMMs, norm and AdamW
    in libtinylm_cuda (host-buffer mode).  Load it in a process of its own:
    its seams switch the library's host-buffer mode on for the device."""
    if not os.path.exists(DROPIN_LIB):
        raise FileNotFoundError(f"{DROPIN_LIB} not built (make -C oracle dropin)")
    return _bind_ref(ctypes.CDLL(DROPIN_LIB))


def _bind_ref(L):
    """ctypes signatures of the harness exports (ref_harness.c)."""
    L.tlref_init.argtypes = [_i, _u64]
    L.tlref_seed.argtypes = [_u64]
    L.tlref_xorshift.restype = _u64
    L.tlref_fill_normal.argtypes = [_fp, _sz, _f]
    for nm in ("tlref_mm", "tlref_mm_bt", "tlref_mm_atb"):
        getattr(L, nm).argtypes = [_fp, _fp, _fp, _i, _i, _i]
    L.tlref_adamw.argtypes = [_fp, _fp, _fp, _fp, _sz, _f, _f, _f, _f, _i, _f]
    L.tlref_gradnorm.argtypes = [_fp, _sz]
    L.tlref_gradnorm.restype = _f
    L.tlref_model_new.argtypes = [_ip, _i, _i, _u64]
    L.tlref_model_new.restype = ctypes.c_void_p
    L.tlref_model_nparams.argtypes = [ctypes.c_void_p]
    L.tlref_model_nparams.restype = _sz
    L.tlref_model_buf.argtypes = [ctypes.c_void_p, _i]
    L.tlref_model_buf.restype = _fp
    L.tlref_model_tokens.argtypes = [ctypes.c_void_p, _i]
    L.tlref_model_tokens.restype = _ip
    L.tlref_model_logits.argtypes = [ctypes.c_void_p]
    L.tlref_model_logits.restype = _fp
    L.tlref_model_forward.argtypes = [ctypes.c_void_p]
    L.tlref_model_forward.restype = _f
    L.tlref_model_fwd_bwd.argtypes = [ctypes.c_void_p]
    L.tlref_model_fwd_bwd.restype = _f
    L.tlref_model_step.argtypes = [ctypes.c_void_p, _f, _i, ctypes.POINTER(_f)]
    L.tlref_model_step.restype = _f
    L.tlref_model_free.argtypes = [ctypes.c_void_p]
    L.tlref_max_threads.restype = _i
    _u16p = ctypes.POINTER(ctypes.c_uint16)
    L.tlref_train.argtypes = [_ip, _i, _i, _i, _f, _u64, _u16p, _sz, _u16p, _sz, ctypes.c_char_p,
                              ctypes.c_char_p, ctypes.c_char_p, _i, ctypes.c_char_p, ctypes.c_char_p]
    L.tlref_train.restype = _i
    L.tlref_model_load.argtypes = [ctypes.c_char_p, _ip, _fp, _sz]
    L.tlref_model_load.restype = _sz
    return L


# ---- numpy-level helpers (restatement leg) ---------------------------------
def adamw(P, G, M, V, lr, b1, b2, wd, t, gscale):
    port().tlo_adamw(fptr(P), fptr(G), fptr(M), fptr(V), P.size, lr, b1, b2, wd, int(t), gscale)


def grad_norm(G):
    return port().tlo_grad_norm(fptr(G), G.size)


def sumsq(G):
    return port().tlo_sumsq(fptr(G), G.size)


def clip_scale(gnorm):
    return port().tlo_clip_scale(gnorm)


def mm(Y, X, W, M, K, N, acc64=False):
    port().tlo_mm(fptr(Y), fptr(X), fptr(W), M, K, N, int(acc64))


def mm_bt(dX, dY, W, M, K, N, acc64=False):
    port().tlo_mm_bt(fptr(dX), fptr(dY), fptr(W), M, K, N, int(acc64))


def mm_atb(dW, X, dY, M, K, N, acc64=False):
    port().tlo_mm_atb(fptr(dW), fptr(X), fptr(dY), M, K, N, int(acc64))


def rel_err(got, ref_):
    """The reference selftest's metric (tinylm.c:4778-4784): max|err| / mean|ref|."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    ref_ = np.ascontiguousarray(ref_, dtype=np.float32)
    mx = _d(0.0)
    r = port().tlo_rel_err(fptr(got), fptr(ref_), got.size, ctypes.byref(mx))
    return r, mx.value


def fill_normal(n, scale, seed=None):
    """Normals with the reference's xorshift64 + Box-Muller recipe (tinylm.c:127-134)."""
    if seed is not None:
        port().tlo_seed(seed)
    a = np.empty(n, dtype=np.float32)
    port().tlo_fill_normal(fptr(a), n, scale)
    return a


def adamw_inputs(n, seed=0):
    """Config-2 inputs: p~N(0,0.02), g~N(0,1e-3), m~N(0,1e-4), v=|N(0,1e-6)|,
    numpy default_rng(seed), drawn in the order p, g, m, v."""
    rng = np.random.default_rng(seed)
    p = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))
    g = (rng.standard_normal(n, dtype=np.float32) * np.float32(1e-3))
    m = (rng.standard_normal(n, dtype=np.float32) * np.float32(1e-4))
    v = np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(1e-6))
    return p, g, m, v


def ref_train(cfg7, n_mtp, B, iters, lr, seed, tr, vl, out, optpath, tok_blob=b"", resume=None):
    """Run the reference's train_loop (tinylm.c:2562-2654) on uint16 streams tr/vl;
    returns its stdout lines.  resume = (bundle, opt) continues from files."""
    import tempfile
    R = ref()
    tr = np.ascontiguousarray(tr, dtype=np.uint16)
    vl = np.ascontiguousarray(vl, dtype=np.uint16)
    u16 = ctypes.POINTER(ctypes.c_uint16)
    cap = tempfile.TemporaryFile(mode="w+b")
    import sys
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(cap.fileno(), 1)
    try:
        R.tlref_train((_i * 7)(*cfg7), n_mtp, B, iters, lr, seed, tr.ctypes.data_as(u16), tr.size,
                      vl.ctypes.data_as(u16), vl.size, out.encode(), optpath.encode(), tok_blob, len(tok_blob),
                      resume[0].encode() if resume else None, resume[1].encode() if resume else None)
    finally:
        os.dup2(saved, 1)
        os.close(saved)
    cap.seek(0)
    return cap.read().decode(errors="replace").replace("\r", "\n").splitlines()
