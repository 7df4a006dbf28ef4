"""Data parallelism with a ZeRO-1 sharded optimizer step, over libtinylm_cuda's
own NCCL communicator.

The reference has no distributed code; this is the multi-GPU form of its
optimizer step (tinylm.c:2630-2633).  torch.distributed is used only to ship
the 128-byte NCCL unique id from rank 0 to the others; every collective of the
step runs inside tl_zero1_step on the library stream.
"""
import ctypes

import torch

from ._lib import TL_ZERO1_ALIGN, check, lib
from . import ops


def zero1_layout(n, world):
    """(n_pad, shard): the flat buffer padded to a multiple of world*4096 floats
    and the per-rank shard length.  Mirrors tl_zero1_padded."""
    q = world * TL_ZERO1_ALIGN
    n_pad = (n + q - 1) // q * q
    return n_pad, n_pad // world


def shard_range(n, world, rank):
    n_pad, shard = zero1_layout(n, world)
    return rank * shard, (rank + 1) * shard


class Zero1:
    """Owns the communicator; buffers are caller-owned CUDA tensors:
    P and G of n_pad floats (pad kept zero), M and V of one shard each.

    exchange="nccl": reduce-scatter / all-reduce / all-gather collectives
    (tl_zero1_step); exchange="p2p": the library's peer-memory kernels
    (tl_zero1_step_p2p; P and G are registered on the first step)."""

    def __init__(self, n, rank, world, device, group=None, exchange="nccl"):
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', not {exchange!r}")
        self.exchange = exchange
        self._registered = None
        self.n, self.rank, self.world = n, rank, world
        self.n_pad, self.shard = zero1_layout(n, world)
        ops.init(device)
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            check(lib().tl_dist_unique_id(ctypes.addressof(uid)))
        if world > 1:
            import torch.distributed as dist
            obj = [bytes(uid) if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0, group=group)
            ctypes.memmove(uid, obj[0], 128)
        check(lib().tl_dist_init(rank, world, ctypes.addressof(uid)))

    def register(self, P, G):
        """Map every rank's P and G for the peer-memory step (collective)."""
        ops._prep(P)
        pp, gp = ops._ptr(P, "P", self.n_pad), ops._ptr(G, "G", self.n_pad)
        check(lib().tl_zero1_p2p_register(pp, gp, self.n))
        self._registered = (pp, gp)

    def step(self, P, G, M_shard, V_shard, lr, b1, b2, wd, t, max_norm=1.0, norm_out=None):
        ops._prep(P)
        no = 0 if norm_out is None else ops._ptr(norm_out, "norm_out", 1)
        pp, gp = ops._ptr(P, "P", self.n_pad), ops._ptr(G, "G", self.n_pad)
        fn = lib().tl_zero1_step
        if self.exchange == "p2p":
            if self._registered != (pp, gp):
                self.register(P, G)
            fn = lib().tl_zero1_step_p2p
        check(fn(pp, gp, ops._ptr(M_shard, "M_shard", self.shard), ops._ptr(V_shard, "V_shard", self.shard),
                 self.n, lr, b1, b2, wd, int(t), max_norm, no or None))

    def allreduce_(self, t, average=False):
        ops._prep(t)
        check(lib().tl_dist_allreduce_f32(ops._ptr(t, "buf"), t.numel(), 1 if average else 0))

    def sync(self, timeout_ms=0):
        check(lib().tl_dist_sync(int(timeout_ms)))

    def close(self):
        if self._registered is not None:
            check(lib().tl_zero1_p2p_release())
            self._registered = None
        check(lib().tl_dist_finalize())
