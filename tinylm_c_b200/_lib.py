"""ctypes binding of libtinylm_cuda.so (the C ABI declared in include/tinylm_cuda.h).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtinylm_cuda.so")

TL_OK = 0
TL_EINVAL = -1
TL_EALIGN = -2
TL_ECUDA = -3
TL_ENCCL = -4
TL_ETIMEOUT = -5
TL_ENOINIT = -6
TL_EPTR = -7
TL_ENOMEM = -8
TL_ZERO1_ALIGN = 4096

_c_int, _c_size, _c_float, _c_void_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); pointers are passed as integers (void*).
SIGNATURES = {
    "tl_init": (_c_int, [_c_int]),
    "tl_set_stream": (_c_int, [_c_void_p]),
    "tl_get_stream": (_c_void_p, []),
    "tl_last_error": (ctypes.c_char_p, []),
    "tl_version": (ctypes.c_char_p, []),
    "tl_alloc": (_c_int, [ctypes.POINTER(_c_void_p), _c_size]),
    "tl_free": (_c_int, [_c_void_p]),
    "tl_memcpy_h2d": (_c_int, [_c_void_p, _c_void_p, _c_size]),
    "tl_memcpy_d2h": (_c_int, [_c_void_p, _c_void_p, _c_size]),
    "tl_memset": (_c_int, [_c_void_p, _c_int, _c_size]),
    "tl_sync": (_c_int, []),
    "tl_device_status": (_c_int, []),
    "tl_set_host_buffers": (_c_int, [_c_int]),
    "tl_trace_enable": (_c_int, [_c_int]),
    "tl_trace_reset": (_c_int, []),
    "tl_trace_get": (_c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]),
    "tl_trace_names": (_c_int, [ctypes.c_char_p, _c_size]),
    "tl_matmul": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int]),
    "tl_matmul_bt": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int]),
    "tl_matmul_at": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int]),
    "tl_matmul_bt_sum": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int]),
    "tl_set_gemm_engine": (_c_int, [_c_int]),
    "tl_last_gemm_engine": (_c_int, []),
    "tl_grad_norm": (_c_int, [_c_void_p, _c_size, _c_void_p]),
    "tl_grad_sumsq": (_c_int, [_c_void_p, _c_size, _c_void_p]),
    "tl_grad_norm_noalloc": (_c_int, [_c_void_p, _c_size, _c_void_p, _c_void_p]),
    "tl_clip_scale": (_c_int, [_c_void_p, _c_float, _c_void_p, _c_void_p]),
    "tl_adamw_step": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size,
                               _c_float, _c_float, _c_float, _c_float, _c_int, _c_float]),
    "tl_adamw_step_dev": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size,
                                   _c_float, _c_float, _c_float, _c_float, _c_int, _c_void_p]),
    "tl_clip_adamw_step": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size,
                                    _c_float, _c_float, _c_float, _c_float, _c_int, _c_float,
                                    _c_void_p]),
    "tl_model_create": (_c_int, [ctypes.POINTER(_c_int), _c_int, ctypes.POINTER(_c_void_p)]),
    "tl_model_nparams": (_c_size, [_c_void_p]),
    "tl_model_destroy": (_c_int, [_c_void_p]),
    "tl_model_param_count": (_c_size, [ctypes.POINTER(_c_int)]),
    "tl_model_init_params": (_c_int, [ctypes.POINTER(_c_int), _c_void_p, ctypes.c_ulonglong,
                                      ctypes.POINTER(ctypes.c_ulonglong)]),
    "tl_ckpt_save_bundle": (_c_int, [ctypes.c_char_p, ctypes.POINTER(_c_int), _c_void_p, _c_size, _c_void_p, _c_int]),
    "tl_ckpt_load_bundle": (_c_int, [ctypes.c_char_p, ctypes.POINTER(_c_int), _c_void_p, _c_size,
                                     ctypes.POINTER(_c_size)]),
    "tl_ckpt_opt_create": (_c_int, [ctypes.c_char_p, _c_int, _c_size]),
    "tl_ckpt_opt_write": (_c_int, [ctypes.c_char_p, _c_size, _c_size, _c_void_p, _c_void_p, _c_size]),
    "tl_ckpt_opt_read": (_c_int, [ctypes.c_char_p, _c_size, _c_size, _c_void_p, _c_void_p, _c_size,
                                  ctypes.POINTER(_c_int)]),
    "tl_lr_at": (_c_float, [_c_int, _c_float, _c_int, _c_float]),
    "tl_sample_windows": (_c_int, [ctypes.POINTER(ctypes.c_ulonglong), _c_void_p, _c_size, _c_int, _c_int, _c_int,
                                   _c_int, _c_void_p, _c_void_p, _c_void_p]),
    "tl_model_forward": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "tl_model_forward_backward": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                           _c_int, _c_void_p]),
    "tl_model_step": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                               _c_void_p, _c_int, _c_float, _c_int, _c_float, _c_void_p, _c_void_p]),
    "tl_set_attn_engine": (_c_int, [_c_int]),
    "tl_model_graph_step": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                     _c_void_p, _c_int, _c_float, _c_int, _c_float, _c_void_p, _c_void_p]),
    "tl_model_step_zero1": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                     _c_void_p, _c_void_p, _c_int, _c_float, _c_int, _c_float, _c_void_p,
                                     _c_void_p]),
    "tl_zero1_padded": (_c_size, [_c_size, _c_int]),
    "tl_dist_unique_id": (_c_int, [_c_void_p]),
    "tl_dist_init": (_c_int, [_c_int, _c_int, _c_void_p]),
    "tl_dist_finalize": (_c_int, []),
    "tl_zero1_step": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size,
                               _c_float, _c_float, _c_float, _c_float, _c_int, _c_float,
                               _c_void_p]),
    "tl_zero1_p2p_register": (_c_int, [_c_void_p, _c_void_p, _c_size]),
    "tl_zero1_step_p2p": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size,
                                   _c_float, _c_float, _c_float, _c_float, _c_int, _c_float,
                                   _c_void_p]),
    "tl_zero1_p2p_release": (_c_int, []),
    "tl_dist_allreduce_f32": (_c_int, [_c_void_p, _c_size, _c_int]),
    "tl_dist_allreduce_f64": (_c_int, [_c_void_p, _c_size]),
    "tl_dist_sync": (_c_int, [_c_int]),
}


class TLError(RuntimeError):
    """A negative status from libtinylm_cuda, with the library's message."""

    def __init__(self, code, msg):
        super().__init__(f"libtinylm_cuda error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Load libtinylm_cuda.so once; raises ImportError if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m tinylm_c_b200.build` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != TL_OK:
        raise TLError(rc, (lib().tl_last_error() or b"").decode(errors="replace"))
    return rc
