"""Benchmark of tinylm-c's training-step hot path on B200 (libtinylm_cuda).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload train|train_m1|train_m8|adamw]

Default workload: BASELINE config 5, the scaled tiny Llama (V 8192, D 1024,
16 layers, 16 heads / 4 KV heads, SwiGLU 2816, ctx 256, fp32, 188.8 M params)
trained on a global batch of 512x256 uniform random tokens: one step =
forward + backward + global-norm clip + AdamW, data parallel over N GPUs (one
process per GPU, torchrun) with a ZeRO-1 optimizer step (reduce-scatter of G,
sharded AdamW, all-gather of P over NCCL).  Global batch fixed across N:
scaling is "strong".  Metric: train tokens/s (whole job).  The same line
carries the second half of BASELINE's metric, the fused AdamW+clip HBM GB/s
(config 2: 2^28 fp32 params; at N=1 measured in the same run).

Other workloads: train_m1 (config 1: m1 preset, n_mtp=2, batch 8), train_m8
(config 4: m8, batch 64), adamw (config 2 alone; ZeRO-1 with N > 1).

Rank 0 prints ONE JSON line.  `value` is device-timed (CUDA events, max over
ranks) with inputs resident in HBM; `e2e` is the same metric through the
library's API with the step's input (tokens, or the gradient for adamw) copied
from pinned host memory and the result (loss / norm) read back every step.
`--impl reference` times the reference's own CPU implementation (tinylm.c
compiled unmodified by oracle/Makefile) on the host cores.
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
# NCCL's communicator set-up lines (rank count, transports, NVLS) go to the log;
# descriptor 1 is redirected to stderr for the run (run_as_script), so they
# cannot precede the JSON line.
# Set unconditionally: an NCCL_DEBUG=WARN inherited from the environment
# would hide the lines that show each communicator's rank count.
os.environ["NCCL_DEBUG"] = "INFO"
os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
_JSON_OUT = 1   # file descriptor the JSON line is written to (see the end of the file)

T_CTX = 256
LR, B1, B2, WD, MAX_NORM = 3e-4, 0.9, 0.95, 0.1, 1.0
ADAMW_N = 1 << 28
ADAMW_T0 = 100
BYTES_PER_PARAM = 32          # norm reads G (4) + AdamW reads P,G,M,V and writes P,M,V (28)
ADAMW_BYTES = 28
NORM_BYTES = 4
TRAIN_METRIC = "train tokens/s (fwd+bwd+AdamW)"
ADAMW_METRIC = "fused AdamW+clip HBM GB/s (fp32, 2^28 params)"

# name -> (preset, n_mtp, global batch, micro-batch cap, CPU-baseline batch, BASELINE config)
TRAIN = {
    "train": ("scaled", 0, 512, 64, 2, "config5_scaled_tiny_llama"),
    "train_m1": ("m1", 2, 8, 8, 8, "config1_m1_nmtp2_b8"),
    "train_m8": ("m8", 0, 64, 64, 8, "config4_m8_b64"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(TRAIN) + ["adamw", "gemm"], default="train")
    ap.add_argument("--n", type=int, default=ADAMW_N, help="adamw workload: elements per buffer")
    ap.add_argument("--batch", type=int, default=0, help="train workloads: global batch (0 = the config's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-adamw-line", action="store_true", help="train: skip the config-2 AdamW sub-measurement")
    ap.add_argument("--no-configs", action="store_true",
                    help="train at N=1: skip the sub-measurements of BASELINE configs 1-4 in the same line")
    ap.add_argument("--shape", default="", help="gemm workload: one M,K,N instead of the sweep")
    ap.add_argument("--op", default="all", choices=["all", "mm", "mm_bt", "mm_atb"], help="gemm workload: primitive")
    ap.add_argument("--zero1", default="nccl", choices=["nccl", "p2p"],
                    help="N>1: ZeRO-1 exchanges by NCCL collectives or by the library's peer-memory kernels")
    ap.add_argument("--no-graph", action="store_true",
                    help="train workloads at N=1: launch the step eagerly instead of replaying a CUDA graph")
    ap.add_argument("--no-overlap", action="store_true",
                    help="N>1, nccl exchange: reduce-scatter after the backward instead of per-shard reductions during it")
    ap.add_argument("--gemm-engine", type=int, default=0, choices=[0, 1, 2, 3, 4, 5],
                    help="GEMM engine: 0 automatic, 1 CUDA-core, 2 tensor-core one CTA, 3 tensor-core CTA pair, "
                         "4 CTA pair with the fp16 split, 5 CTA pair with the hybrid split")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def emit(obj):
    sys.stdout.flush()
    os.write(_JSON_OUT, (json.dumps(obj) + "\n").encode())


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
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def tf32_probe(n=8192, burst_iters=10, sustain_s=3.0):
    """The tf32 tensor-core rate of this GPU, measured with a cuBLAS fp32
    matmul that may use tf32 (n^3 products, 2n^3 flop): the best of
    `burst_iters` single calls, and the mean over back-to-back calls for
    `sustain_s` seconds.  A denominator only: the product never runs through
    cuBLAS.  3xTF32 needs three tf32 passes per fp32 product, so its ceiling
    is a third of this."""
    import torch
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("high")
    try:
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        c = torch.empty(n, n, device="cuda")
        flop = 2.0 * n ** 3
        for _ in range(3):
            torch.matmul(a, b, out=c)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(burst_iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(); torch.matmul(a, b, out=c); e1.record(); e1.synchronize()
            best = max(best, flop / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        calls, t0 = 0, time.time()
        e0.record()
        while time.time() - t0 < sustain_s:
            for _ in range(8):
                torch.matmul(a, b, out=c)
            calls += 8
            e1.record(); e1.synchronize()
        sustained = flop * calls / (e0.elapsed_time(e1) * 1e-3) / 1e12
        del a, b, c
        torch.cuda.empty_cache()
        return {"tf32_tflops": round(best, 1), "tf32_tflops_sustained": round(sustained, 1),
                "how": f"torch.matmul fp32 with tf32 allowed (cuBLAS), {n}^3: best of {burst_iters} calls and "
                       f"{calls} calls back to back ({sustain_s:g} s)"}
    finally:
        torch.set_float32_matmul_precision(prev)


_TF32_PROBE = None


def cached_tf32_probe():
    global _TF32_PROBE
    if _TF32_PROBE is None:
        _TF32_PROBE = tf32_probe()
    return _TF32_PROBE


def gemm_ceiling(engine, training=False):
    """Divisor of the bf16 peak giving the GEMM engine's fp32-product ceiling,
    the kernel's name and the reason.  `training`: the GEMMs of the device
    training step, which the automatic choice runs with the hybrid split."""
    if engine == 4:
        return 3.0, "gemm_tc (tcgen05 fp16 split)", "3 fp16 MMAs per fp32 product, fp16 = bf16 rate"
    if engine == 5 or (engine == 0 and training):
        return 4.0, "gemm_tc (tcgen05 hybrid split: tf32 hi*hi + bf16 cross terms)", \
            "one tf32 MMA (bf16/2 rate) + one bf16 MMA over twice the K per fp32 product"
    return 6.0, "gemm_tc (tcgen05 3xTF32)", "tf32 = bf16/2; 3 tf32 MMAs per fp32 product"


def committed_traffic(key):
    """dram bytes per launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(key)


def gemm_flops_per_token(cfg):
    """fp32 FLOPs of all GEMMs per token of one training step: 6 x the
    GEMM-held parameters (each weight: one forward and two backward GEMMs),
    plus the MTP heads (tinylm.c:1036-1069)."""
    V, D, L, H, KV, F, T, n_mtp = cfg
    KD = KV * (D // H)
    per = 6 * (L * (2 * D * D + 2 * D * KD + 3 * D * F) + D * V)
    per += n_mtp * (6 * D * D + 6 * D * V)
    return per


# ------------------------------------------------------------------ helpers
class Run:
    """Per-process GPU context: device, optional NCCL process group, library."""

    def __init__(self, rank, world, local):
        import torch
        from tinylm_c_b200 import _lib, ops
        self.torch, self.ops, self.L, self._lib = torch, ops, _lib.lib(), _lib
        self.rank, self.world, self.local = rank, world, local
        self.dev = torch.device("cuda", local)
        torch.cuda.set_device(self.dev)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=self.dev)
        ops.init(local)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x):
        if self.world == 1:
            return x
        import torch.distributed as dist
        t = self.torch.tensor([x], device=self.dev, dtype=self.torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def timed(self, step, steps, t0, trace=True):
        """K steps between barriers; device time from CUDA events on the
        launching stream, max over ranks; per-kernel times from the tracer
        (trace=False: no per-launch events inside the timed region)."""
        torch, L = self.torch, self.L
        L.tl_trace_reset()
        L.tl_trace_enable(1 if trace else 0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(gpu_uuid(torch, self.dev)) as clk:
            self.barrier()
            e0.record(self.stream)
            for i in range(steps):
                step(t0 + i)
            e1.record(self.stream)
            self.barrier()
        L.tl_trace_enable(0)
        ms = self.max_over_ranks(e0.elapsed_time(e1))
        return ms / steps, self.kernels(steps) if trace else {}, clk.summary()

    def kernels(self, steps):
        L, _lib = self.L, self._lib
        out = {}
        names = ctypes.create_string_buffer(8192)
        _lib.check(L.tl_trace_names(names, 8192))
        for nm in filter(None, names.value.decode().split(",")):
            tot, cnt = ctypes.c_double(0), ctypes.c_longlong(0)
            _lib.check(L.tl_trace_get(nm.encode(), ctypes.byref(tot), ctypes.byref(cnt)))
            out[nm] = {"ms_per_step": round(tot.value / steps, 4), "launches": cnt.value,
                       "ms_per_launch": round(tot.value / max(1, cnt.value), 5)}
        return out

    def status(self):
        self._lib.check(self.L.tl_device_status())

    def close(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------ reference CPU arm
def reference_train(wl, steps, warmup):
    """The reference's own forward/backward/norm/AdamW (tinylm.c:4736-4740),
    compiled unmodified, on all host threads, at a CPU-sized batch."""
    import oracle
    from tinylm_c_b200 import model
    preset, n_mtp, _, _, B, _ = TRAIN[wl]
    R = oracle.ref()
    threads = cpu_threads()
    R.tlref_init(threads, 0)
    cfg = list(model.PRESETS[preset])
    h = R.tlref_model_new((oracle._i * 7)(*cfg), n_mtp, B, 0)
    times = []
    gn = oracle._f(0.0)
    try:
        for it in range(warmup + steps):
            t0 = time.perf_counter()
            R.tlref_model_step(h, LR, it + 1, ctypes.byref(gn))
            dt = time.perf_counter() - t0
            if it >= warmup:
                times.append(dt)
    finally:
        R.tlref_model_free(h)
    sec = statistics.median(times)
    return B * T_CTX / sec, sec, threads, B


def reference_adamw(n, steps, warmup):
    """The reference's own adamw + global_gradnorm (tinylm.c:1159-1176)."""
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
        R.tlref_adamw(fp(p), fp(g), fp(m), fp(v), n, LR, B1, B2, WD, ADAMW_T0 + it, gs)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    sec = statistics.median(times)
    return n * BYTES_PER_PARAM / sec / 1e9, sec, threads


# ---------------------------------------------------------- train workloads
def run_train(args, rk):
    torch, ops = rk.torch, rk.ops
    from tinylm_c_b200 import model
    preset, n_mtp, B_glob, mb_cap, _, cfg_name = TRAIN[args.workload]
    if args.batch:
        B_glob = args.batch
    world, rank = rk.world, rk.rank
    if B_glob % world:
        raise SystemExit(f"global batch {B_glob} not divisible by {world} ranks")
    B = B_glob // world
    mb = min(B, mb_cap)
    while B % mb:
        mb -= 1
    cfg = model.cfg8(preset, n_mtp)
    m = model.Model(cfg, mb, rk.local)
    n = m.nparams
    P0 = model.init_params(cfg, 0)
    dev = rk.dev
    if world == 1:
        n_pad, shard = n, n
        P = P0.to(dev)
        G = torch.zeros(n, device=dev)
    else:
        from tinylm_c_b200.zero1 import Zero1
        z = Zero1(n, rank, world, rk.local, exchange=args.zero1)
        n_pad, shard = z.n_pad, z.shard
        P = torch.zeros(n_pad, device=dev)
        P[:n] = P0.to(dev)
        G = torch.zeros(n_pad, device=dev)
    del P0
    M = torch.zeros(shard, device=dev)
    V = torch.zeros(shard, device=dev)
    Vocab = cfg[0]
    N = B * T_CTX
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    tok = torch.randint(0, Vocab, (N,), generator=gen, device=dev, dtype=torch.int32)
    tgt = torch.randint(0, Vocab, (N,), generator=gen, device=dev, dtype=torch.int32)
    mtp = torch.randint(0, Vocab, (n_mtp, N), generator=gen, device=dev, dtype=torch.int32) if n_mtp else None
    loss = torch.zeros(1, device=dev)
    norm = torch.zeros(1, device=dev)

    use_graph = world == 1 and not args.no_graph
    if world == 1:
        def eager_step(t):
            m.step(P, G, M, V, tok, tgt, mtp, B, LR, t, MAX_NORM, loss, norm)

        def step(t):   # N=1: the whole step replayed as one CUDA graph (tl_model_graph_step)
            m.step(P, G, M, V, tok, tgt, mtp, B, LR, t, MAX_NORM, loss, norm, graph=use_graph)
    elif args.zero1 == "nccl" and not args.no_overlap:
        def step(t):   # tl_model_step_zero1: shard reductions overlap the backward pass
            m.step_zero1(z, P, G, M, V, tok, tgt, mtp, B, LR, t, MAX_NORM, loss, norm)
    else:
        def step(t):
            G.zero_()
            m.forward_backward(P, G, tok, tgt, mtp, B, loss)
            z.step(P, G, M, V, LR, B1, B2, WD, t, MAX_NORM, norm)

    for i in range(args.warmup):
        step(1 + i)
    rk.torch.cuda.synchronize()
    rk.status()
    t0 = 1 + args.warmup
    # The timed steps run without per-launch trace events (at N=1 the step is
    # one graph replay anyway); the per-kernel breakdown and the GEMM roofline
    # come from the same step run again, eagerly, with every launch traced.
    ms_step, _, clocks = rk.timed(step, args.steps, t0, trace=False)
    rk.status()
    value = B_glob * T_CTX / (ms_step * 1e-3)
    loss_val = loss.item()
    n_tr = max(1, min(args.steps, 2))
    eager_ms, kernels, _ = rk.timed(eager_step if world == 1 else step, n_tr, t0 + args.steps)
    rk.status()
    t0 += n_tr

    # ---- end to end: tokens from pinned host memory, loss read back, every step
    e2e = None
    if not args.no_e2e:
        steps = max(1, min(args.steps, 5))
        hs = [x.cpu().pin_memory() for x in (tok, tgt) + ((mtp,) if n_mtp else ())]
        ds = [tok, tgt] + ([mtp] if n_mtp else [])
        hloss = torch.zeros(1).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rk.barrier()
        e0.record(rk.stream)
        t1 = t0 + args.steps
        for i in range(steps):
            for d, h in zip(ds, hs):
                d.copy_(h, non_blocking=True)
            step(t1 + i)
            hloss.copy_(loss, non_blocking=True)
        e1.record(rk.stream)
        rk.barrier()
        ms = rk.max_over_ranks(e0.elapsed_time(e1)) / steps
        e2e = {"value": round(B_glob * T_CTX / (ms * 1e-3), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": sum(h.numel() * 4 for h in hs) * world, "d2h_bytes_per_step": 4,
               "steps": steps, "ms_per_step": round(ms, 3),
               "path": "pinned host tokens -> tl_model_step (N=1) / tl_model_step_zero1 (N>1) -> host loss"}

    # ---- roofline of the dominant kernel (the tensor-core GEMM)
    peaks, peak_kind = measured_peaks()
    gflop_tok = gemm_flops_per_token(tuple(cfg))
    gemm = gemm_kernels(kernels)
    flops_rank = gflop_tok * N
    achieved = flops_rank / (gemm["ms_per_step"] * 1e-3) / 1e12 if gemm["ms_per_step"] else None
    bf16 = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    div, kname, why = gemm_ceiling(args.gemm_engine, training=True)
    peak = bf16 / div
    roofline = {"kernel": kname, "bound": "tensor", "unit": "TFLOP/s",
                "achieved": round(achieved, 2) if achieved else None, "peak": round(peak, 1),
                "peak_source": f"{peak_kind} bf16 sustained {bf16} TFLOP/s / {div:g} ({why})",
                "frac": round(achieved / peak, 4) if achieved else None,
                # against the ceiling of the 3xTF32 algorithm (bf16 sustained / 6)
                "frac_of_3xtf32_ceiling": round(achieved * 6.0 / bf16, 4) if achieved else None,
                "traffic": None, "algorithmic_flops_per_step": flops_rank,
                "gemm_share_of_step": round(gemm["ms_per_step"] / (eager_ms or ms_step), 4) if ms_step else None}
    tr = committed_traffic(f"{args.workload}:gemm_tc")
    if tr:
        roofline["traffic"] = tr.get("bytes_per_step")
        roofline["traffic_source"] = tr.get("source")
    # the traced pass ran n_tr steps; the timed region ran the same kernels args.steps times
    launches = sum(k["launches"] for k in kernels.values()) * args.steps // n_tr

    adam_line = None
    if kernels.get("adamw_vec", {}).get("ms_per_launch"):
        a = kernels["adamw_vec"]["ms_per_launch"]
        adam_line = {"in_step_adamw_gbs": round(shard * ADAMW_BYTES / (a * 1e-3) / 1e9, 1),
                     "params_per_rank": shard}
    m.close()
    del P, G, M, V
    if world > 1:
        z.close()
    torch.cuda.empty_cache()
    if world == 1 and roofline.get("achieved"):
        # the tf32 rate probed on this GPU after the timed region: 3xTF32's
        # ceiling is a third of it (sustained: the step runs for seconds), the
        # mark the hybrid split is measured against too
        pr = cached_tf32_probe()
        roofline["tf32_probe"] = pr
        roofline["frac_of_probed_tf32"] = round(roofline["achieved"] / (pr["tf32_tflops_sustained"] / 3.0), 4)

    out = None
    if rank == 0:
        out = {"metric": TRAIN_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
               "data": "synthetic (uniform random token ids, seeded); weights from the reference's seeded init_params",
               "config": {"workload": cfg_name, "model": preset, "n_params": n, "n_mtp": n_mtp,
                          "global_batch": B_glob, "seq_len": T_CTX, "micro_batch": mb,
                          "parallelism": "single" if world == 1 else
                          f"dp{world}_zero1_{args.zero1}" + ("" if args.zero1 != "nccl" or args.no_overlap else "_overlap"),
                          "gemm_gflop_per_token": round(gflop_tok / 1e9, 4),
                          "launch": "cuda_graph" if use_graph else "eager",
                          "l2": "per-step working set >> 126 MB L2 (no flush needed)"},
               "e2e": e2e, "roofline": roofline, "clocks": clocks, "gpu_launches": launches,
               "loss": round(loss_val, 5), "kernels": kernels}
        out["traced_ms_per_step"] = round(eager_ms, 3)
        if adam_line:
            out["fused_adamw"] = adam_line
    return out


# --------------------------------------------------------------- adamw (cfg 2)
def run_adamw(args, rk, n):
    torch, ops = rk.torch, rk.ops
    world, rank, dev = rk.world, rk.rank, rk.dev
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    if world == 1:
        p = torch.randn(n, device=dev, generator=gen) * 0.02
        g = torch.randn(n, device=dev, generator=gen) * 1e-3
        m = torch.randn(n, device=dev, generator=gen) * 1e-4
        v = (torch.randn(n, device=dev, generator=gen) * 1e-6).abs()
        shard = n
        norm = torch.zeros(1, device=dev)

        def step(t):
            ops.clip_adamw(p, g, m, v, n, LR, B1, B2, WD, t, MAX_NORM, norm)
    else:
        from tinylm_c_b200.zero1 import Zero1
        z = Zero1(n, rank, world, rk.local, exchange=args.zero1)
        shard = z.shard
        p = torch.zeros(z.n_pad, device=dev)
        g = torch.zeros(z.n_pad, device=dev)
        p[:n] = torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(1234)) * 0.02
        g[:n] = torch.randn(n, device=dev, generator=gen) * 1e-3
        m = torch.randn(shard, device=dev, generator=gen) * 1e-4
        v = (torch.randn(shard, device=dev, generator=gen) * 1e-6).abs()
        norm = torch.zeros(1, device=dev)

        def step(t):
            z.step(p, g, m, v, LR, B1, B2, WD, t, MAX_NORM, norm)
    for i in range(args.warmup):
        step(ADAMW_T0 + i)
    torch.cuda.synchronize()
    t0 = ADAMW_T0 + args.warmup
    ms_step, kernels, clocks = rk.timed(step, args.steps, t0)
    rk.status()
    value = n * BYTES_PER_PARAM / (ms_step * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        steps = max(1, min(args.steps, 5))
        hg = g.cpu().pin_memory()
        hnorm = torch.zeros(1).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rk.barrier()
        e0.record(rk.stream)
        for i in range(steps):
            g.copy_(hg, non_blocking=True)
            step(t0 + args.steps + i)
            hnorm.copy_(norm, non_blocking=True)
        e1.record(rk.stream)
        rk.barrier()
        ms = rk.max_over_ranks(e0.elapsed_time(e1)) / steps
        e2e = {"value": round(n * BYTES_PER_PARAM / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": g.numel() * 4 * world, "d2h_bytes_per_step": 4, "steps": steps,
               "ms_per_step": round(ms, 3),
               "path": "pinned host G -> tl_clip_adamw_step / tl_zero1_step -> host norm; P,M,V resident"}

    peaks, peak_kind = measured_peaks()
    # The peer-memory step's AdamW kernel also stores the shard into the other
    # ranks' P (the fused all-gather); its algorithmic bytes here are the
    # local 28 B/elem, like adamw_vec's.
    kname = "p2p_adamw" if (world > 1 and args.zero1 == "p2p") else "adamw_vec"
    adam = kernels.get(kname, {"ms_per_launch": 0})
    a_ms = adam["ms_per_launch"]
    achieved = shard * ADAMW_BYTES / (a_ms * 1e-3) / 1e9 if a_ms else None
    nk = kernels.get("sumsq", {"ms_per_launch": 0})
    roofline = {"kernel": kname, "bound": "hbm", "unit": "GB/s",
                "achieved": round(achieved, 1) if achieved else None, "peak": peaks["hbm_gbs"],
                "peak_source": f"{peak_kind} HBM copy", "frac": round(achieved / peaks["hbm_gbs"], 4) if achieved else None,
                "traffic": None, "algorithmic_bytes": shard * ADAMW_BYTES,
                "sumsq_gbs": round(shard * NORM_BYTES / (nk["ms_per_launch"] * 1e-3) / 1e9, 1) if nk["ms_per_launch"] else None}
    tr = committed_traffic("adamw:adamw_vec" if world == 1 else f"adamw_zero1_{world}:adamw_vec")
    if tr:
        roofline["traffic"] = tr.get("bytes_per_launch")
        roofline["traffic_source"] = tr.get("source")
    launches = sum(k["launches"] for k in kernels.values())
    if world > 1:
        z.close()
    del p, g, m, v
    torch.cuda.empty_cache()
    return {"metric": ADAMW_METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded normals with config-2 distributions)",
            "config": {"workload": "config2_fused_adamw_clip" if world == 1 else "config2_zero1_adamw",
                       "n_params": n, "bytes_per_param": BYTES_PER_PARAM, "t_start": ADAMW_T0,
                       "parallelism": "single" if world == 1 else f"zero1_dp{world}_{args.zero1}",
                       "l2": "inputs 4 GiB >> 126 MB L2 (no flush needed)"},
            "e2e": e2e, "roofline": roofline, "clocks": clocks, "gpu_launches": launches, "kernels": kernels}


def gemm_kernels(kernels):
    """The tensor-core GEMM launches of a traced region, both kernels summed."""
    out = {"ms_per_step": 0.0, "launches": 0, "names": []}
    for name in ("gemm_tc", "gemm_tc_pair"):
        k = kernels.get(name)
        if k:
            out["ms_per_step"] += k["ms_per_step"]
            out["launches"] += k["launches"]
            out["names"].append(name)
    return out


# ------------------------------------------------------------- gemm (cfg 3)
GEMM_SWEEP_M = (16384, 65536)
GEMM_SWEEP_KN = (256, 512, 1024, 2816)
GEMM_METRIC = "GEMM fp32 TFLOP/s (3xTF32 tensor cores), BASELINE config-3 sweep"


def gemm_shapes(args):
    if args.shape:
        M, K, N = (int(x) for x in args.shape.split(","))
        return [(M, K, N)]
    return [(M, K, N) for M in GEMM_SWEEP_M for K in GEMM_SWEEP_KN for N in GEMM_SWEEP_KN]


def run_gemm(args, rk, shapes=None):
    """X@W, X@W^T, X^T@W over the config-3 sweep (X~N(0,1), W~N(0,0.02),
    dY~N(0,1)), or over `shapes`; per shape and primitive: warm-up, then K
    timed calls."""
    torch, ops = rk.torch, rk.ops
    dev = rk.dev
    ops_sel = ["mm", "mm_bt", "mm_atb"] if args.op == "all" else [args.op]
    results = []
    tot_flop = tot_ms = 0.0
    launches = 0
    clocks_all = []
    for (M, K, N) in (shapes or gemm_shapes(args)):
        g = torch.Generator(device=dev).manual_seed(M + K + N)
        X = torch.randn(M * K, device=dev, generator=g)
        W = torch.randn(K * N, device=dev, generator=g) * 0.02
        dY = torch.randn(M * N, device=dev, generator=g)
        out = {"mm": torch.empty(M * N, device=dev), "mm_bt": torch.zeros(M * K, device=dev),
               "mm_atb": torch.zeros(K * N, device=dev)}
        fns = {"mm": lambda: ops.mm(out["mm"], X, W, M, K, N),
               "mm_bt": lambda: ops.mm_bt(out["mm_bt"], dY, W, M, K, N),
               "mm_atb": lambda: ops.mm_atb(out["mm_atb"], X, dY, M, K, N)}
        for op in ops_sel:
            for _ in range(args.warmup):
                fns[op]()
            torch.cuda.synchronize()
            ms, kernels, clocks = rk.timed(lambda t, f=fns[op]: f(), args.steps, 0)
            rk.status()
            flop = 2.0 * M * K * N
            results.append({"op": op, "M": M, "K": K, "N": N, "ms": round(ms, 4),
                            "tflops": round(flop / (ms * 1e-3) / 1e12, 2),
                            "engine": ops.last_gemm_engine()})
            tot_flop += flop
            tot_ms += ms
            launches += sum(k["launches"] for k in kernels.values())
            if clocks.get("sm_mhz"):
                clocks_all.append(clocks)
        del X, W, dY, out
        torch.cuda.empty_cache()
    peaks, peak_kind = measured_peaks()
    bf16 = peaks.get("bf16_tflops", 0)
    div, kname, why = gemm_ceiling(args.gemm_engine)
    peak = bf16 / div
    agg = tot_flop / (tot_ms * 1e-3) / 1e12
    best = max(results, key=lambda r: r["tflops"])
    # the tf32 rate probed on this GPU (burst: the sweep's calls are short)
    probe = cached_tf32_probe() if rk.world == 1 and args.gemm_engine in (0, 2, 3) else None
    return {"metric": GEMM_METRIC, "value": round(agg, 2), "unit": "TFLOP/s", "n_gpus": rk.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_ms / max(1, len(results)), 4),
            "higher_is_better": True, "scaling": "replicas", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (X~N(0,1), W~N(0,0.02), dY~N(0,1), seeded)",
            "config": {"workload": ("config3_gemm_sample" if shapes else "config3_gemm_sweep") if not args.shape
                       else "config3_gemm_one",
                       "shapes": len(results), "value_is": "total FLOP / total time over the sweep",
                       "l2": "sample: >= 248 MB of operands per call (> 126 MB L2), no flush; full sweep: "
                             "the smallest shapes (16384 x 256 x 256: 33 MB) repeat from L2"},
            "roofline": {"kernel": kname, "bound": "tensor", "unit": "TFLOP/s",
                         "achieved": round(agg, 2), "best_shape": best, "peak": round(peak, 1),
                         "peak_source": f"{peak_kind} bf16 burst {bf16} TFLOP/s / {div:g} ({why})",
                         "frac": round(agg / peak, 4) if peak else None, "traffic": None,
                         "tf32_probe": probe,
                         "frac_of_probed_tf32": round(agg / (probe["tf32_tflops"] / 3.0), 4) if probe else None},
            "clocks": clocks_all[-1] if clocks_all else {}, "gpu_launches": launches, "sweep": results}


def reference_gemm(args, shapes=None):
    """The reference's mm/mm_bt/mm_atb (tinylm.c:439-537) on a row sample of
    the sweep or of `shapes` (M scaled down to 1024 rows; per-row work
    identical)."""
    import numpy as np
    import oracle
    R = oracle.ref()
    threads = cpu_threads()
    R.tlref_init(threads, 0)
    tot_flop = tot_s = 0.0
    shapes = shapes or gemm_shapes(args)
    for (M, K, N) in shapes[: (1 if args.shape else len(shapes))]:
        Ms = min(M, 1024)
        rng = np.random.default_rng(0)
        X = rng.standard_normal(Ms * K, dtype=np.float32)
        W = rng.standard_normal(K * N, dtype=np.float32) * np.float32(0.02)
        dY = rng.standard_normal(Ms * N, dtype=np.float32)
        Y = np.empty(Ms * N, np.float32); dX = np.zeros(Ms * K, np.float32); dW = np.zeros(K * N, np.float32)
        fp = oracle.fptr
        for fn in (lambda: R.tlref_mm(fp(Y), fp(X), fp(W), Ms, K, N),
                   lambda: R.tlref_mm_bt(fp(dX), fp(dY), fp(W), Ms, K, N),
                   lambda: R.tlref_mm_atb(fp(dW), fp(X), fp(dY), Ms, K, N)):
            t0 = time.perf_counter()
            fn()
            tot_s += time.perf_counter() - t0
            tot_flop += 2.0 * Ms * K * N
    return tot_flop / tot_s / 1e12, threads


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        import oracle
        if not oracle.has_ref():
            emit({"impl": "reference", "unavailable": "oracle/_ref/libtlref.so not built (needs the reference sources at build time)"})
            return 0
        if args.workload == "gemm":
            tf, threads = reference_gemm(args)
            emit({"impl": "reference", "metric": GEMM_METRIC, "value": round(tf, 4), "unit": "TFLOP/s",
                  "n_gpus": world, "steps": 1, "warmup": 0, "higher_is_better": True, "scaling": "replicas",
                  "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy default_rng(0))",
                  "config": {"workload": "config3_gemm_sweep", "parallelism": f"cpu_omp{threads}"},
                  "cpu_baseline": {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                                   "sample": "tinylm.c mm/mm_bt/mm_atb on every sweep shape with M cut to 1024 rows"},
                  "e2e": {"value": round(tf, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
            return 0
        if args.workload == "adamw":
            gbs, sec, threads = reference_adamw(args.n, args.steps, args.warmup)
            emit({"impl": "reference", "metric": ADAMW_METRIC, "value": round(gbs, 3), "unit": "GB/s",
                  "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
                  "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                  "data": "synthetic (numpy default_rng(0), config-2 distributions)",
                  "config": {"workload": "config2_fused_adamw_clip", "n_params": args.n,
                             "parallelism": f"cpu_omp{threads}"},
                  "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                                   "sample": f"tinylm.c adamw+global_gradnorm, n={args.n}, median of {args.steps} steps"},
                  "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
            return 0
        tps, sec, threads, B = reference_train(args.workload, args.steps, args.warmup)
        preset, n_mtp, B_glob, _, _, cfg_name = TRAIN[args.workload]
        emit({"impl": "reference", "metric": TRAIN_METRIC, "value": round(tps, 2), "unit": "tokens/s",
              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 2),
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
              "data": "synthetic (reference xorshift tokens, seed 0)",
              "config": {"workload": cfg_name, "model": preset, "n_mtp": n_mtp, "global_batch": B_glob,
                         "seq_len": T_CTX, "parallelism": f"cpu_omp{threads}"},
              "cpu_baseline": {"value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "reference",
                               "sample": f"tinylm.c forward+backward+gradnorm+adamw at batch {B}x{T_CTX} "
                                         f"(per-token work of the config), median of {args.steps} steps"},
              "e2e": {"value": round(tps, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return 0

    rk = Run(rank, world, local)
    if args.gemm_engine:
        rk.ops.set_gemm_engine(args.gemm_engine)
    if args.workload == "gemm":
        out = run_gemm(args, rk)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            tf, threads = reference_gemm(args)
            out["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                                   "sample": "tinylm.c mm/mm_bt/mm_atb with M cut to 1024 rows"}
    elif args.workload == "adamw":
        out = run_adamw(args, rk, args.n)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            steps = cpu_baseline_steps()
            gbs, sec, threads = reference_adamw(args.n, steps, 1)
            out["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                                   "sample": f"tinylm.c adamw+global_gradnorm (oracle/_ref), n={args.n}, median of {steps} steps"}
    else:
        out = run_train(args, rk)
        if world == 1 and not args.no_adamw_line:
            a = run_adamw(argparse.Namespace(warmup=3, steps=20, no_e2e=True), rk, ADAMW_N)
            if rank == 0:
                out.setdefault("fused_adamw", {}).update(
                    {"config2_gbs": a["value"], "config2_adamw_kernel_gbs": a["roofline"]["achieved"],
                     "config2_frac_of_hbm": a["roofline"]["frac"], "config2_ms_per_step": a["ms_per_step"],
                     "metric": ADAMW_METRIC})
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline_train(args.workload)
        if world == 1 and args.workload == "train" and not args.no_configs:
            configs = run_other_configs(args, rk)
            if rank == 0:
                out["configs"] = configs
    if rank == 0:
        emit(out)
    rk.close()
    return 0


def cpu_baseline_steps():
    """Timed reference steps per CPU baseline (median taken; at least 3)."""
    return max(3, int(os.environ.get("TL_CPU_BASELINE_STEPS", "3")))


def cpu_baseline_train(workload):
    steps = cpu_baseline_steps()
    tps, sec, threads, B = reference_train(workload, steps, 1)
    return {"value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"tinylm.c forward+backward+gradnorm+adamw at batch {B}x{T_CTX} (same per-token work), "
                      f"median of {steps} steps after 1 warm-up",
            "s_per_step": round(sec, 3)}


# The BASELINE configs other than the headline, measured in the same run (N=1):
# config 1 and 4 training steps, config 2 AdamW+clip with its own CPU baseline
# and end-to-end figure, and a sample of the config-3 GEMM sweep.
# Every sampled shape moves at least 248 MB of operands per call, about twice
# the 126 MB L2, so repeats start cold without a flush.
GEMM_SAMPLE = ((16384, 2816, 2816), (16384, 1024, 2816), (16384, 2816, 1024), (65536, 1024, 2816),
               (65536, 2816, 1024), (65536, 512, 512))


def _compact(line, keep=("metric", "value", "unit", "ms_per_step", "steps", "warmup", "config", "e2e", "roofline",
                         "cpu_baseline", "gpu_launches", "clocks", "loss", "traced_ms_per_step")):
    return {k: line[k] for k in keep if k in line}


def run_other_configs(args, rk):
    rank = rk.rank
    out = {}
    base = dict(vars(args), batch=0, no_e2e=False, no_graph=False, gemm_engine=args.gemm_engine)
    for wl, steps in (("train_m1", 30), ("train_m8", 20)):
        line = run_train(argparse.Namespace(**dict(base, workload=wl, steps=steps, warmup=3)), rk)
        if rank == 0:
            line = _compact(line)
            if not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline_train(wl)
            out[TRAIN[wl][5]] = line
    line = run_adamw(argparse.Namespace(**dict(base, workload="adamw", steps=20, warmup=3)), rk, ADAMW_N)
    if rank == 0:
        line = _compact(line)
        if not args.no_cpu_baseline:
            steps = cpu_baseline_steps()
            gbs, sec, threads = reference_adamw(ADAMW_N, steps, 1)
            line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                                    "sample": f"tinylm.c global_gradnorm + adamw at n=2^28, median of {steps} steps "
                                              "after 1 warm-up"}
        out["config2_fused_adamw_clip"] = line
    line = run_gemm(argparse.Namespace(**dict(base, workload="gemm", steps=10, warmup=3, op="all", shape="")), rk,
                    shapes=GEMM_SAMPLE)
    if rank == 0:
        line = _compact(line, keep=("metric", "value", "unit", "config", "roofline", "gpu_launches", "clocks",
                                    "sweep"))
        if not args.no_cpu_baseline:
            tf, threads = reference_gemm(args, shapes=GEMM_SAMPLE)
            line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                                    "sample": "tinylm.c mm/mm_bt/mm_atb on the sampled shapes with M cut to 1024 rows"}
        out["config3_gemm_sample"] = line
    return out


def run_as_script(entry=None):
    """Run `entry` (main) as the script does.  Rank 0's stdout must carry
    exactly one JSON line, but libraries write to file descriptor 1 on their
    own (NCCL prints its version banner there at the WARN level).  So
    descriptor 1 points at stderr for the whole run and the JSON line goes to
    a duplicate of the original stdout."""
    global _JSON_OUT
    _JSON_OUT = os.dup(1)
    os.dup2(2, 1)
    return (entry or main)()


if __name__ == "__main__":
    sys.exit(run_as_script())
