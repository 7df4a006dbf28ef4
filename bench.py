"""Benchmark of tinylm-c's training-step hot path on B200 (libtinylm_cuda).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload adamw|gemm]

Default workload: the fused AdamW + global-norm clip step
over flat fp32 buffers p, g, m, v of 2^28 elements each (p~N(0,0.02),
g~N(0,1e-3), m~N(0,1e-4), v=|N(0,1e-6)|, t counting up from 100, lr 3e-4,
betas 0.9/0.95, wd 0.1, clip 1.0).  One step = sum of squares of G -> clip scale
-> AdamW, 32 algorithmic bytes per element.  With N > 1 GPUs (torchrun, one
process per GPU) one step is the ZeRO-1 optimizer step over the same 2^28
buffer: ReduceScatter(G, avg) -> shard norm -> AllReduce -> AdamW on the 1/N
shard -> AllGather(P); total work is fixed, so scaling is "strong".

Rank 0 prints ONE JSON line.  `value` is device-timed with inputs resident in
HBM; `e2e` is the same metric through the C ABI with pinned host buffers and
the host<->device copies inside the timed region.  `--impl reference` times the
reference's own CPU implementation (tinylm.c adamw + global_gradnorm, compiled
by oracle/Makefile) on the host cores.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ELEMS = 1 << 28
LR, B1, B2, WD, MAX_NORM, T0 = 3e-4, 0.9, 0.95, 0.1, 1.0, 100
BYTES_PER_ELEM = 32          # norm reads G (4) + AdamW reads P,G,M,V and writes P,M,V (28)
ADAMW_BYTES_PER_ELEM = 28
NORM_BYTES_PER_ELEM = 4
METRIC = "fused AdamW+clip HBM GB/s (fp32, 2^28 params)"
GEMM_METRIC = "GEMM GFLOP/s (fp32 3xTF32)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["adamw", "gemm"], default="adamw")
    ap.add_argument("--n", type=int, default=N_ELEMS, help="elements per buffer (default 2^28)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def emit(obj):
    print(json.dumps(obj), flush=True)


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_uuid(torch, dev):
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return dev


# --------------------------------------------------------------------- peaks
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def committed_traffic(kernel, workload):
    """dram bytes per launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    e = d.get(f"{workload}:{kernel}")
    return e


# ----------------------------------------------------------- reference (CPU)
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference_adamw(n, steps, warmup):
    """The reference's own adamw + global_gradnorm (tinylm.c:1159-1176), compiled
    unmodified, on all host threads; one step = norm + clip + AdamW on n elements."""
    import numpy as np
    import oracle
    R = oracle.ref()
    threads = cpu_threads()
    R.tlref_init(threads, 0)
    p, g, m, v = oracle.adamw_inputs(n, seed=0)
    fp = oracle.fptr
    times = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        gn = R.tlref_gradnorm(fp(g), n)
        gs = 1.0 / gn if gn > 1.0 else 1.0
        R.tlref_adamw(fp(p), fp(g), fp(m), fp(v), n, LR, B1, B2, WD, T0 + it, gs)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    sec = statistics.median(times)
    return n * BYTES_PER_ELEM / sec / 1e9, sec, threads


def cpu_baseline_adamw(n_full):
    """Bounded sample for the GPU arm's line: the reference at the full n for a
    few steps (memory-bound; per-step cost does not depend on the step count)."""
    steps = int(os.environ.get("TL_CPU_BASELINE_STEPS", "5"))
    gbs, sec, threads = run_reference_adamw(n_full, steps, 1)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"tinylm.c adamw+global_gradnorm (oracle/_ref), n=2^{n_full.bit_length() - 1}, "
                      f"median of {steps} steps after 1 warm-up, OMP threads={threads}",
            "ms_per_step": round(sec * 1e3, 3)}


# ------------------------------------------------------------- our arm (GPU)
def run_ours_adamw(args, rank, world, local):
    import torch
    from tinylm_c_b200 import _lib, ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    ops.init(local)
    L = _lib.lib()
    n = args.n
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    stream = torch.cuda.current_stream(dev)

    if world == 1:
        p = torch.randn(n, device=dev, generator=gen) * 0.02
        g = torch.randn(n, device=dev, generator=gen) * 1e-3
        m = torch.randn(n, device=dev, generator=gen) * 1e-4
        v = (torch.randn(n, device=dev, generator=gen) * 1e-6).abs()
        norm = torch.zeros(1, device=dev)

        def step(t):
            ops.clip_adamw(p, g, m, v, n, LR, B1, B2, WD, t, MAX_NORM, norm)
        shard_n = n
    else:
        from tinylm_c_b200.zero1 import Zero1
        z = Zero1(n, rank, world, local)
        shard_n = z.shard
        p = torch.zeros(z.n_pad, device=dev)
        g = torch.zeros(z.n_pad, device=dev)
        p[:n] = torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(1234)) * 0.02
        g[:n] = torch.randn(n, device=dev, generator=gen) * 1e-3
        m = torch.randn(z.shard, device=dev, generator=gen) * 1e-4
        v = (torch.randn(z.shard, device=dev, generator=gen) * 1e-6).abs()
        norm = torch.zeros(1, device=dev)

        def step(t):
            z.step(p, g, m, v, LR, B1, B2, WD, t, MAX_NORM, norm)
    torch.cuda.synchronize()

    t = T0
    for _ in range(args.warmup):
        step(t)
        t += 1
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    L.tl_trace_reset()
    L.tl_trace_enable(1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid(torch, dev)) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step(t)
            t += 1
        e1.record(stream)
        barrier()
    L.tl_trace_enable(0)
    ms = e0.elapsed_time(e1)
    kernels = {}
    names = ctypes.create_string_buffer(4096)
    _lib.check(L.tl_trace_names(names, 4096))
    for nm in filter(None, names.value.decode().split(",")):
        tot, cnt = ctypes.c_double(0), ctypes.c_longlong(0)
        _lib.check(L.tl_trace_get(nm.encode(), ctypes.byref(tot), ctypes.byref(cnt)))
        kernels[nm] = {"ms_total": tot.value, "launches": cnt.value}
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = tt.item()
    ms_step = ms / args.steps
    value = n * BYTES_PER_ELEM / (ms_step * 1e-3) / 1e9

    # ---- end to end through the C ABI with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = e2e_adamw(args, torch, ops, dev, stream, world, rank, n, shard_n, p, g, m, v, norm, step, t)

    # ---- roofline of the dominant kernel
    peaks, peak_kind = measured_peaks()
    adam = kernels.get("adamw_vec", {"ms_total": 0, "launches": 0})
    adam_ms = adam["ms_total"] / max(1, adam["launches"])
    adam_elems = shard_n
    achieved = adam_elems * ADAMW_BYTES_PER_ELEM / (adam_ms * 1e-3) / 1e9 if adam_ms > 0 else None
    norm_k = kernels.get("sumsq", {"ms_total": 0, "launches": 0})
    norm_ms = norm_k["ms_total"] / max(1, norm_k["launches"])
    roofline = {"kernel": "adamw_vec", "bound": "hbm", "achieved": round(achieved, 1) if achieved else None,
                "peak": peaks["hbm_gbs"], "peak_source": peak_kind, "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4) if achieved else None,
                "traffic": None, "algorithmic_bytes": adam_elems * ADAMW_BYTES_PER_ELEM,
                "ms_per_launch": round(adam_ms, 4),
                "sumsq": {"achieved": round(shard_n * NORM_BYTES_PER_ELEM / (norm_ms * 1e-3) / 1e9, 1)
                          if norm_ms > 0 else None, "ms_per_launch": round(norm_ms, 4)}}
    tr = committed_traffic("adamw_vec", "adamw" if world == 1 else f"adamw_zero1_{world}")
    if tr:
        roofline["traffic"] = tr.get("bytes_per_launch")
        roofline["traffic_source"] = tr.get("source")

    launches = sum(k["launches"] for k in kernels.values())
    out = None
    if rank == 0:
        clocks = clk.summary()
        out = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
               "data": "synthetic (seeded normals with config-2 distributions)",
               "config": {"workload": "config2_fused_adamw_clip" if world == 1 else "config2_zero1_adamw",
                          "n_params": n, "bytes_per_param": BYTES_PER_ELEM, "t_start": T0,
                          "parallelism": "single" if world == 1 else f"zero1_dp{world}",
                          "l2": "inputs 4 GiB >> 126 MB L2 (no flush needed)"},
               "e2e": e2e, "roofline": roofline, "clocks": clocks, "gpu_launches": launches,
               "kernels": kernels}
    if world > 1:
        import torch.distributed as dist
        z.close()
        dist.barrier()
        dist.destroy_process_group()
    return out


def e2e_adamw(args, torch, ops, dev, stream, world, rank, n, shard_n, p, g, m, v, norm, step, t):
    """Same step through the C ABI with the step's input in host memory.

    Per step the input is the fresh gradient G (a training loop produces one per
    step) and the result is the global norm: G goes host->device from pinned
    memory, the optimizer step runs (tl_clip_adamw_step, or tl_zero1_step with
    N ranks), and the norm comes back.  P, M and V are optimizer state and stay
    resident, as they do in any GPU training run.  `all_host` repeats the
    measurement with P, M and V also copied in and out every step (the literal
    host-buffer form of the reference's adamw() call)."""
    steps = max(1, min(args.steps, int(os.environ.get("TL_E2E_STEPS", "5"))))
    hg = g.cpu().pin_memory()
    hnorm = torch.zeros(1).pin_memory()
    if world == 1:
        state = [(p, p.cpu().pin_memory()), (m, m.cpu().pin_memory()), (v, v.cpu().pin_memory())]
    else:
        lo = rank * shard_n
        ps = p[lo:lo + shard_n]
        state = [(ps, ps.cpu().pin_memory()), (m, m.cpu().pin_memory()), (v, v.cpu().pin_memory())]

    def timed(all_host):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(steps):
            g.copy_(hg, non_blocking=True)
            if all_host:
                for d, h in state:
                    d.copy_(h, non_blocking=True)
            step(t + i)
            if all_host:
                for d, h in state:
                    h.copy_(d, non_blocking=True)
            hnorm.copy_(norm, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            import torch.distributed as dist
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = tt.item()
        return ms / steps

    ms_g = timed(False)
    ms_all = timed(True)
    st_bytes = sum(d.numel() * 4 for d, _ in state)
    gb = lambda ms: round(n * BYTES_PER_ELEM / (ms * 1e-3) / 1e9, 3)
    return {"value": gb(ms_g), "unit": "GB/s", "h2d_bytes_per_step": g.numel() * 4, "d2h_bytes_per_step": 4,
            "steps": steps, "ms_per_step": round(ms_g, 3),
            "path": "pinned host G -> tl_clip_adamw_step / tl_zero1_step -> host norm; P,M,V resident",
            "all_host": {"value": gb(ms_all), "ms_per_step": round(ms_all, 3),
                         "h2d_bytes_per_step": g.numel() * 4 + st_bytes, "d2h_bytes_per_step": st_bytes + 4}}


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.workload != "adamw":
            emit({"impl": "reference", "unavailable": "reference arm implemented for the adamw workload only"})
            return 0
        import oracle
        if not oracle.has_ref():
            emit({"impl": "reference", "unavailable": "oracle/_ref/libtlref.so not built (needs the reference sources at build time)"})
            return 0
        gbs, sec, threads = run_reference_adamw(args.n, args.steps, args.warmup)
        emit({"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
              "data": "synthetic (numpy default_rng(0), config-2 distributions)",
              "config": {"workload": "config2_fused_adamw_clip", "n_params": args.n,
                         "bytes_per_param": BYTES_PER_ELEM, "t_start": T0, "parallelism": f"cpu_omp{threads}"},
              "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                               "sample": f"tinylm.c adamw+global_gradnorm on the full n, median of {args.steps} steps"},
              "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return 0

    out = run_ours_adamw(args, rank, world, local)
    if rank == 0 and out is not None:
        if world == 1 and not args.no_cpu_baseline:
            import torch
            torch.cuda.empty_cache()
            out["cpu_baseline"] = cpu_baseline_adamw(args.n)
        emit(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
