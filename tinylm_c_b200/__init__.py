"""tinylm_c_b200: B200 (sm_100a) implementation of tinylm-c's training-step hot
path -- fused AdamW with global grad-norm clipping and the three fp32 GEMM
primitives -- behind the C ABI of libtinylm_cuda (include/tinylm_cuda.h), plus
data parallelism with a ZeRO-1 optimizer step over NCCL.

Modules: ops (the reference-named primitives), zero1 (multi-GPU step),
build (nvcc recipe), _lib (ctypes binding).
"""
from ._lib import LIB_PATH, TLError, lib  # noqa: F401

__all__ = ["LIB_PATH", "TLError", "lib"]
