"""The reference's training loop on the device: train_loop (tinylm.c:2562-2654).

Per iteration, as the reference: learning rate from the warm-up + cosine
schedule (2587-2590); validation on `val_batches` windows of the validation
stream at the first and last iteration and every `val_sec` seconds
(2591-2609); B training windows drawn with the reference's generator
(2623-2626); one step -- zeroed G, forward, backward, global-norm clip, AdamW
with betas 0.9/0.95 and weight decay 0.1 (2627-2633); progress lines and
time-based checkpoints (2635-2649); a final TLM4 bundle and TOPT sidecar
(2651-2653).  A run is fresh (init_params from the seed; the generator then
continues into batch sampling) or resumed from a bundle + sidecar (the
generator restarts from the seed), as cmd_train does (2739-2743).

With world > 1 every rank draws the same global batch and trains on its
1/world slice; the optimizer step is ZeRO-1 (tl_zero1_step).  Each rank
writes and reads its own shard of M and V in the TOPT file; rank 0 writes
the bundle.  Host-side pieces (sampler, schedule, file formats) are the
library's C functions; every step runs on the GPU.
"""
import ctypes
import os
import time

import numpy as np
import torch

from ._lib import check, lib
from . import model as tlm
from . import ops

BETA1, BETA2, WD = 0.9, 0.95, 0.1


def _fmt_dur(sec):
    sec = int(sec)
    return f"{sec // 3600}h{(sec // 60) % 60:02d}m" if sec >= 3600 else (f"{sec // 60}m{sec % 60:02d}s" if sec >= 60 else f"{sec}s")


def save_bundle(path, cfg, P, n, eot=0, tmpl=0, tok_blob=b""):
    """TLM4 bundle (model_save_bundle, tinylm.c:1895-1914) from host or device P."""
    V, D, L, H, KV, F, T, n_mtp = list(cfg)
    hdr = (ctypes.c_int * 11)(V, D, L, H, KV, F, T, eot, tmpl, n_mtp, 0)
    blob = bytes(tok_blob or b"")
    check(lib().tl_ckpt_save_bundle(path.encode(), hdr, P.data_ptr(), n, blob if blob else None, len(blob)))


def load_bundle(path, P=None):
    """Header dict (and parameters into P, host or device tensor) of a TLM1-4 bundle."""
    hdr = (ctypes.c_int * 11)()
    nf = ctypes.c_size_t(0)
    check(lib().tl_ckpt_load_bundle(path.encode(), hdr, None if P is None else P.data_ptr(),
                                    0 if P is None else P.numel(), ctypes.byref(nf)))
    keys = ("V", "D", "L", "H", "KV", "F", "T", "eot", "tmpl", "n_mtp", "n_exp")
    return dict(zip(keys, list(hdr)))


class Trainer:
    def __init__(self, cfg, B, micro_batch=None, device=0, rank=0, world=1, exchange="nccl", overlap=True):
        self.cfg = cfg
        self.T = cfg[6] if cfg[6] > 0 else 256
        self.n_mtp = cfg[7]
        self.B, self.rank, self.world = B, rank, world
        # NCCL exchange: reduce gradient shards during the backward pass
        self.overlap = overlap and exchange == "nccl"
        if B % world:
            raise ValueError(f"batch {B} not divisible by {world} ranks")
        self.Bl = B // world
        mb = micro_batch or self.Bl
        if self.Bl % mb:
            raise ValueError(f"local batch {self.Bl} not a multiple of micro-batch {mb}")
        self.device = ops.init(device)
        self.dev = torch.device("cuda", self.device)
        self.model = tlm.Model(cfg, mb, self.device)
        self.n = self.model.nparams
        if world > 1:
            from .zero1 import Zero1
            self.z = Zero1(self.n, rank, world, self.device, exchange=exchange)
            self.n_pad, self.shard = self.z.n_pad, self.z.shard
        else:
            self.z = None
            self.n_pad, self.shard = self.n, self.n
        self.P = torch.zeros(self.n_pad, device=self.dev)
        self.G = torch.zeros(self.n_pad, device=self.dev)
        self.M = torch.zeros(self.shard, device=self.dev)
        self.V = torch.zeros(self.shard, device=self.dev)
        N = B * self.T
        self.h_tok = np.empty(N, np.int32)
        self.h_tgt = np.empty(N, np.int32)
        self.h_mtp = np.empty(max(self.n_mtp, 1) * N, np.int32)
        Nl = self.Bl * self.T
        self.d_tok = torch.empty(Nl, dtype=torch.int32, device=self.dev)
        self.d_tgt = torch.empty(Nl, dtype=torch.int32, device=self.dev)
        self.d_mtp = torch.empty((self.n_mtp, Nl), dtype=torch.int32, device=self.dev) if self.n_mtp else None
        self.loss = torch.zeros(1, device=self.dev)
        self.norm = torch.zeros(1, device=self.dev)

    # ---------------------------------------------------------------- state
    def init_fresh(self, seed):
        P0, st = tlm.init_params(self.cfg, seed, return_rng=True)
        self.P[: self.n].copy_(P0.to(self.dev))
        self.M.zero_()
        self.V.zero_()
        self.rng = ctypes.c_ulonglong(st)
        return 0

    def load(self, bundle, optpath, seed):
        hdr = load_bundle(bundle)
        mine = list(self.cfg)
        got = [hdr[k] for k in ("V", "D", "L", "H", "KV", "F", "T")] + [hdr["n_mtp"]]
        if got != mine:
            raise ValueError(f"{bundle}: configuration {got} does not match {mine}")
        load_bundle(bundle, self.P[: self.n])
        lo = self.rank * self.shard
        cnt = max(0, min(self.shard, self.n - lo))
        it = ctypes.c_int(0)
        check(lib().tl_ckpt_opt_read(optpath.encode(), self.n, min(lo, self.n), self.M.data_ptr(),
                                     self.V.data_ptr(), cnt, ctypes.byref(it)))
        self.rng = ctypes.c_ulonglong(seed | 1)
        return it.value

    def save(self, out, optpath, it, eot=0, tmpl=0, tok_blob=b""):
        torch.cuda.synchronize(self.dev)
        if self.rank == 0:
            save_bundle(out, self.cfg, self.P, self.n, eot, tmpl, tok_blob)
            check(lib().tl_ckpt_opt_create(optpath.encode(), int(it), self.n))
        self._barrier()
        lo = self.rank * self.shard
        cnt = max(0, min(self.shard, self.n - lo))
        if cnt:
            check(lib().tl_ckpt_opt_write(optpath.encode(), self.n, lo, self.M.data_ptr(), self.V.data_ptr(), cnt))
        self._barrier()

    def _barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    # ------------------------------------------------------------- batches
    def _sample(self, stream, val):
        N = self.B * self.T
        check(lib().tl_sample_windows(ctypes.byref(self.rng), stream.ctypes.data, stream.size, self.B, self.T,
                                      self.n_mtp, 1 if val else 0, self.h_tok.ctypes.data, self.h_tgt.ctypes.data,
                                      self.h_mtp.ctypes.data))
        Nl = self.Bl * self.T
        lo = self.rank * Nl
        self.d_tok.copy_(torch.from_numpy(self.h_tok[lo:lo + Nl]), non_blocking=False)
        self.d_tgt.copy_(torch.from_numpy(self.h_tgt[lo:lo + Nl]), non_blocking=False)
        if self.n_mtp and not val:
            m = self.h_mtp[: self.n_mtp * N].reshape(self.n_mtp, N)[:, lo:lo + Nl]
            self.d_mtp.copy_(torch.from_numpy(np.ascontiguousarray(m)))

    def _mean_over_ranks(self, t):
        if self.world > 1:
            self.z.allreduce_(t, average=True)
        return t.item()

    def val_loss(self, vl, batches):
        v = np.float32(0.0)
        for _ in range(batches):
            self._sample(vl, True)
            self.model.forward(self.P, self.d_tok, self.d_tgt, self.Bl, self.loss)
            v = np.float32(v + np.float32(self._mean_over_ranks(self.loss)))
        return float(np.float32(v / np.float32(batches)))

    def step(self, lr, t):
        if self.world == 1:
            self.model.step(self.P, self.G, self.M, self.V, self.d_tok, self.d_tgt, self.d_mtp, self.Bl, lr, t,
                            1.0, self.loss, self.norm)
        elif self.overlap:
            self.model.step_zero1(self.z, self.P, self.G, self.M, self.V, self.d_tok, self.d_tgt, self.d_mtp,
                                  self.Bl, lr, t, 1.0, self.loss, self.norm)
        else:
            self.G.zero_()
            self.model.forward_backward(self.P, self.G, self.d_tok, self.d_tgt, self.d_mtp, self.Bl, self.loss)
            self.z.step(self.P, self.G, self.M, self.V, lr, BETA1, BETA2, WD, t, 1.0, self.norm)

    # ---------------------------------------------------------------- loop
    def run(self, tr, vl, iters, lr, seed=0, out=None, optpath=None, resume=False, eot=0, tmpl=0, tok_blob=b"",
            warmup=200.0, val_batches=4, print_sec=15.0, val_sec=600.0, save_sec=300.0, max_seconds=0.0,
            log=print):
        tr = np.ascontiguousarray(tr, dtype=np.uint16)
        vl = np.ascontiguousarray(vl, dtype=np.uint16)
        if resume and out and optpath and os.path.exists(out) and os.path.exists(optpath):
            start = self.load(out, optpath, seed)
        else:
            start = self.init_fresh(seed)
        iters = max(iters, start)
        spe = max(1, tr.size // (self.B * self.T))
        history = []
        say = log if self.rank == 0 else (lambda *a, **k: None)
        wall0 = time.time()
        last_print = last_val = last_save = wall0
        timeup = False
        it = start
        while it <= iters:
            cur_lr = lib().tl_lr_at(it, lr, iters, warmup)
            wall = time.time()
            if it == start or it == iters or wall - last_val >= val_sec:
                v = self.val_loss(vl, val_batches)
                wall = time.time()
                say(f"iter {it:5d} (ep {it / spe:.2f}) | val {v:.4f} | lr {cur_lr:.2e} | {_fmt_dur(wall - wall0)}")
                history.append(("val", it, v))
                last_val = last_print = wall
            if it == iters:
                break
            if max_seconds > 0 and not timeup and time.time() - wall0 >= max_seconds:
                say(f"[train] max seconds reached at iter {it}")
                timeup, iters = True, it
                continue                     # re-enter with it == iters: final validation
            self._sample(tr, False)
            self.step(cur_lr, it + 1)
            loss = self.loss.item()
            history.append(("train", it, loss))
            wall = time.time()
            if it > start and wall - last_print >= print_sec:
                done = wall - wall0
                sps = done / (it - start)
                say(f"iter {it:5d} (ep {it / spe:.2f}) | loss {loss:.4f} | "
                    f"{self.B * self.T * (it - start) / done:.0f} tok/s | {100.0 * it / iters:.1f}% | "
                    f"{_fmt_dur(done)} | ETA {_fmt_dur((iters - it) * sps)}")
                last_print = wall
            if out and optpath and it > start and wall - last_save >= save_sec:
                self.save(out, optpath, it, eot, tmpl, tok_blob)
                say(f"[ckpt] saved {out} @ iter {it} (ep {it / spe:.2f})")
                last_save = time.time()
            it += 1
        if out and optpath:
            self.save(out, optpath, iters, eot, tmpl, tok_blob)
        return history

    def close(self):
        self.model.close()
        if self.z is not None:
            self.z.close()
