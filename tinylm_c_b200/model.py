"""The reference's whole training step on the device (tl_model_* in the C ABI).

Configurations are the reference's presets (tinylm.c:109-124) plus the scaled
tiny Llama of BASELINE config 5; cfg8 = (V, D, L, H, KV, F, T, n_mtp).
"""
import ctypes

import torch

from ._lib import check, lib
from . import ops

PRESETS = {
    "nano": (512, 64, 4, 4, 2, 176, 256),
    "micro": (2048, 96, 4, 6, 2, 256, 256),
    "m1": (2048, 128, 4, 4, 1, 336, 256),
    "m3": (2048, 192, 6, 6, 2, 512, 256),
    "m6": (2048, 256, 8, 8, 2, 688, 256),
    "m8": (2048, 288, 8, 8, 2, 768, 256),
    "m16": (2048, 512, 5, 8, 2, 1408, 256),
    "m32": (2048, 512, 10, 8, 2, 1536, 256),
    "m70": (2048, 768, 11, 12, 2, 2048, 256),
    "scaled": (8192, 1024, 16, 16, 4, 2816, 256),
}


def cfg8(preset, n_mtp=0):
    return (ctypes.c_int * 8)(*PRESETS[preset], n_mtp) if isinstance(preset, str) else (ctypes.c_int * 8)(*preset)


def param_count(cfg):
    return lib().tl_model_param_count(cfg)


def init_params(cfg, seed, return_rng=False):
    """init_params (tinylm.c:395-419) on the host, reference generator seeded
    as TINYLM_SEED=seed does; returns a float32 CPU tensor (and, when asked,
    the generator state the reference's batch sampling continues from)."""
    n = param_count(cfg)
    P = torch.empty(n, dtype=torch.float32)
    st = ctypes.c_ulonglong(0)
    check(lib().tl_model_init_params(cfg, P.data_ptr(), seed, ctypes.byref(st)))
    return (P, st.value) if return_rng else P


def _iptr(t, name):
    if t is None:
        return None
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.int32 and t.is_contiguous()):
        raise TypeError(f"{name}: expected a contiguous int32 CUDA tensor")
    return t.data_ptr()


class Model:
    """Activation arena for `micro_batch` sequences on one device."""

    def __init__(self, cfg, micro_batch, device=0):
        self.cfg = cfg
        self.T = cfg[6] if cfg[6] > 0 else 256
        self.n_mtp = cfg[7]
        self.micro_batch = micro_batch
        self.device = ops.init(device)
        h = ctypes.c_void_p()
        check(lib().tl_model_create(cfg, micro_batch, ctypes.byref(h)))
        self.h = h
        self.nparams = lib().tl_model_nparams(h)

    def forward(self, P, tok, tgt, B, loss_out):
        ops._prep(P)
        check(lib().tl_model_forward(self.h, ops._ptr(P, "P", self.nparams), _iptr(tok, "tok"), _iptr(tgt, "tgt"),
                                     B, ops._ptr(loss_out, "loss_out", 1)))

    def forward_backward(self, P, G, tok, tgt, tgt_mtp, B, loss_out=None):
        ops._prep(P)
        check(lib().tl_model_forward_backward(
            self.h, ops._ptr(P, "P", self.nparams), ops._ptr(G, "G", self.nparams), _iptr(tok, "tok"),
            _iptr(tgt, "tgt"), _iptr(tgt_mtp, "tgt_mtp"), B,
            None if loss_out is None else ops._ptr(loss_out, "loss_out", 1)))

    def step(self, P, G, M, V, tok, tgt, tgt_mtp, B, lr, t, max_norm=1.0, loss_out=None, norm_out=None,
             graph=False):
        """One training step; graph=True replays it as a CUDA graph
        (tl_model_graph_step; buffers must not move between calls)."""
        ops._prep(P)
        n = self.nparams
        fn = lib().tl_model_graph_step if graph else lib().tl_model_step
        check(fn(
            self.h, ops._ptr(P, "P", n), ops._ptr(G, "G", n), ops._ptr(M, "M", n), ops._ptr(V, "V", n),
            _iptr(tok, "tok"), _iptr(tgt, "tgt"), _iptr(tgt_mtp, "tgt_mtp"), B, lr, int(t), max_norm,
            None if loss_out is None else ops._ptr(loss_out, "loss_out", 1),
            None if norm_out is None else ops._ptr(norm_out, "norm_out", 1)))

    def step_zero1(self, z, P, G, M_shard, V_shard, tok, tgt, tgt_mtp, B, lr, t, max_norm=1.0, loss_out=None,
                   norm_out=None):
        """Data-parallel step over the Zero1 communicator z (NCCL exchange),
        the gradient reduction overlapped with the backward pass."""
        ops._prep(P)
        check(lib().tl_model_step_zero1(
            self.h, ops._ptr(P, "P", z.n_pad), ops._ptr(G, "G", z.n_pad), ops._ptr(M_shard, "M_shard", z.shard),
            ops._ptr(V_shard, "V_shard", z.shard), _iptr(tok, "tok"), _iptr(tgt, "tgt"), _iptr(tgt_mtp, "tgt_mtp"),
            B, lr, int(t), max_norm, None if loss_out is None else ops._ptr(loss_out, "loss_out", 1),
            None if norm_out is None else ops._ptr(norm_out, "norm_out", 1)))

    def close(self):
        if self.h:
            lib().tl_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
