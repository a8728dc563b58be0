"""Benchmark of the K-quant decode GEMV (the hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload q6k-gemv|q4k-gemv] [--m M]

Workload (default): the Q6_K dequant-GEMV of a 14336 -> 4096 down-projection
(N = 4096 output rows, K = 14336, GGUF Q6_K, 48,168,960 weight bytes) at batch
M = 1, f32 activations.  One step = that GEMV over each of 8 distinct seeded
weights (385 MB in total, more than the 126 MB L2, so every step streams its
weights from HBM).  Data is synthetic: seeded random Q6_K superblocks with the
distribution the reference's benchmark names (int8 scales in [-32, 31], d =
f16(|N(0, 0.005)|)), x ~ N(0, 1).

Metric: GB/s of algorithmic bytes (weight bytes + M*K*4 + M*N*4 per GEMV).
* value    -- device-resident inputs, a step captured once into a CUDA graph and
              replayed; CUDA events on the launch stream; max over ranks.
* e2e      -- the same GEMVs through the C ABI with host buffers (pinned),
              host->device copy of x and device->host copy of y per call.
* roofline -- the GEMV kernel alone, bracketed by CUDA events inside the last
              replay of the timed region, against MEASURED_PEAKS.json's HBM
              copy bandwidth.
* cpu_baseline -- the reference's CPU algorithm (QuantizedLinear::forward over
              tile_dequant blocks, restated in oracle/kq_oracle.c) on the same
              shape, timed on this host.

Multi-GPU (torchrun): every rank runs its own 8 weights (the decode GEMVs of
independent layers shard with no exchange), "scaling": "weak"; the only
collectives are the barrier and the max-over-ranks of the timing.

--impl reference runs the reference's CPU path alone (rank 0; other ranks
exit 0) with the same metric, on a bounded sample of rows per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "Q4_K/Q6_K dequant-GEMV GB/s (% HBM peak); decode tok/s at 1/2/4/8 B200"
WORKLOADS = {
    # name: (gguf type, legacy type, N rows, K, description)
    "q6k-gemv": (14, 114, 4096, 14336, "Q6_K dequant+GEMV 4096x14336 (down-proj shape)"),
    "q4k-gemv": (12, 112, 4096, 4096, "Q4_K dequant+GEMV 4096x4096"),
}
PREFILL_METRIC = "Q4_K prefill dequant-GEMM TFLOP/s (% dense bf16 peak)"
PREFILL = {
    # name: (gguf type, legacy type, N rows, K, description); bf16 activations, M tokens
    "prefill-4096": (12, 112, 4096, 4096, "Q4_K dequant-GEMM 4096x4096, bf16 x"),
    "prefill-14336": (12, 112, 14336, 4096, "Q4_K dequant-GEMM 14336x4096, bf16 x"),
}
DECODE_METRIC = METRIC
DECODERS = {
    # name: (config name in pesti_b200.decoder, context length)
    "decode-llama8b": ("LLAMA3_8B", 2048),
    "decode-qwen05b": ("QWEN25_05B", 512),
}
L2_BYTES = 126 * 1024 * 1024  # B200 L2


def num_weights(wbytes):
    # distinct weights per step: at least 8 and at least 3x the L2 in bytes, so
    # every GEMV streams its weight from HBM
    return max(8, -(-3 * L2_BYTES // wbytes))
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(PREFILL) + sorted(DECODERS),
                   default="q6k-gemv")
    p.add_argument("--m", "--batch", dest="m", type=int, default=1,
                   help="tokens per call (decode batch); --batch is the form to use under torchrun")
    p.add_argument("--path", choices=["auto", "tcgen05", "mma", "dp4a", "imma"], default="auto",
                   help="kernel family for the GEMV (auto: dp4a m<=4, mma m<=64, tcgen05 above)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--prefetch", action="store_true",
                   help="each GEMV prefetches the next one's weight into L2 (kq_ctx_prefetch_next)")
    p.add_argument("--no-fuse", action="store_true",
                   help="decoders: separate RMSNorm / SwiGLU / add kernels at batch 1")
    return p.parse_args()


def kernel_path(name):
    from pesti_b200 import kq
    return {"auto": kq.KQ_PATH_AUTO, "tcgen05": kq.KQ_PATH_TCGEN05, "mma": kq.KQ_PATH_MMA,
            "dp4a": kq.KQ_PATH_DP4A, "imma": kq.KQ_PATH_IMMA}[name]


def algorithmic_bytes(qtype, n, k, m):
    wbytes = n * (k // 256) * (144 if qtype == 12 else 210)
    return wbytes, wbytes + m * k * 4 + m * n * 4


def peaks(key="hbm_gbs", fallback=None):
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return float(d[key]), "measured"
    except Exception:
        return (FALLBACK_HBM_GBS if fallback is None else fallback), "fallback"


def profiled_traffic(workload, m):
    """dram bytes per launch of the GEMV kernel from a committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"gemv_{workload}_m{m}.txt")
    try:
        with open(path) as fh:
            for line in fh:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].split()[0]))
    except OSError:
        pass
    return None


# ---- clocks during the timed region ------------------------------------------

class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks",
               0x1: "gpu_idle", 0x10: "sync_boost"}

    def __init__(self, device_index, period_s=0.01):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hi = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hi)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        h = hi
            self.h = h or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.period = period_s
            self.ok = True
        except Exception as e:  # no NVML: report that, do not guess
            self.err = str(e)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
                r = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons - {"gpu_idle"})}


# ---- CPU legs ------------------------------------------------------------------

class CpuReference:
    """The reference's algorithm -- QuantizedLinear::forward: full f32
    dequantization, then a sequential f32 dot per output, threads over batch
    rows only -- over the workload shape in the reference's own block layout
    (restated in oracle/kq_oracle.c)."""

    def __init__(self, workload, m, seed=0):
        import oracle
        from pesti_b200 import synthetic
        self.oracle = oracle
        self.qtype, self.legacy, self.n, self.k, _ = {**WORKLOADS, **PREFILL}[workload]
        self.m = m
        self.data = synthetic.legacy_weight(self.legacy, self.n, self.k, seed=seed)
        self.x = synthetic.activations(m, self.k, seed=seed + 1)

    def run(self, row0, rows):
        """Forward over rows [row0, row0+rows); returns (seconds, algorithmic bytes)."""
        sub = self.data[row0:row0 + rows]
        t0 = time.perf_counter()
        self.oracle.legacy_forward(self.legacy, sub, self.k, rows, self.x, self.m,
                                   nthreads=os.cpu_count() or 1, threads_over_batch=True)
        dt = time.perf_counter() - t0
        return dt, algorithmic_bytes(self.qtype, rows, self.k, self.m)[1]


def cpu_baseline(workload, m, budget_s=12.0):
    ref = CpuReference(workload, m)
    n, k = ref.n, ref.k
    total_t, total_b, passes = 0.0, 0, 0
    while total_t < budget_s and passes < 64:
        dt, alg = ref.run(0, n)
        total_t += dt
        total_b += alg
        passes += 1
    cores = min(m, os.cpu_count() or 1)
    return {"value": round(total_b / total_t / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{passes} full passes of QuantizedLinear::forward (full f32 dequant + sequential "
                      f"dot, threads over batch rows) over a {n}x{k} pesti-legacy weight at M={m}; "
                      f"bytes counted as the GGUF workload's",
            "host_cpus": os.cpu_count()}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    if args.workload in DECODERS:
        from pesti_b200 import decoder as dec
        cfg_name, ctx_len = DECODERS[args.workload]
        cfg = getattr(dec, cfg_name)
        base = cpu_decode_sample(cfg)
        print(json.dumps({"metric": DECODE_METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": world,
                          "steps": 1, "warmup": 0, "ms_per_step": round(1e3 / base["value"], 3),
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic", "impl": "reference",
                          "config": {"workload": f"{args.workload}: {cfg.name} decode, batch 1, context {ctx_len}",
                                     "parallelism": "cpu"},
                          "cpu_baseline": base,
                          "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    prefill = args.workload in PREFILL
    qtype, _, n, k, desc = {**WORKLOADS, **PREFILL}[args.workload]
    m = args.m if not prefill or args.m > 1 else 2048
    steps, warm = max(args.steps, 1), max(args.warmup, 0)
    ref = CpuReference(args.workload, m)
    # each step is a bounded sample of rows so the whole run stays ~2 minutes
    dt1, _ = ref.run(0, 256)
    per_row = dt1 / 256
    rows = int(max(16, min(n, 90.0 / ((steps + warm) * per_row))))
    starts = list(range(0, n - rows + 1, rows)) or [0]
    for i in range(warm):
        ref.run(starts[i % len(starts)], rows)
    tt, tb = 0.0, 0
    for i in range(steps):
        dt, alg = ref.run(starts[i % len(starts)], rows)
        tt += dt
        tb += alg
    value = tb / tt / 1e9
    unit, metric = "GB/s", METRIC
    if prefill:  # the same sampled work counted in FLOPs
        value = steps * 2.0 * m * rows * k / tt / 1e12
        unit, metric = "TFLOP/s", PREFILL_METRIC
    cores = min(m, os.cpu_count() or 1)
    line = {"metric": metric, "value": round(value, 6), "unit": unit, "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(tt / steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"{args.workload}: {desc}, M={m}, {rows} of {n} rows per step",
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": cores, "kind": "port",
                             "sample": f"{rows} of {n} rows per step of QuantizedLinear::forward restated "
                                       f"(oracle/kq_oracle.c) in the reference's block layout"},
            "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- our arm -------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from pesti_b200 import kq, synthetic

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    qtype, _, n, k, desc = WORKLOADS[args.workload]
    m = args.m
    wbytes, alg = algorithmic_bytes(qtype, n, k, m)
    NUM_WEIGHTS = num_weights(wbytes)

    ctx = kq.Context(local_rank)
    weights = [kq.Weight(ctx, qtype, synthetic.gguf_weight(qtype, n, k, seed=1000 * rank + i), n, k)
               for i in range(NUM_WEIGHTS)]
    x = torch.from_numpy(synthetic.activations(m, k, seed=7 + rank)).to(dev)
    ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _ in range(NUM_WEIGHTS)]
    ctx.set_path(kernel_path(args.path))
    ctx.reserve(weights[0], m)

    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)

    def step(prefetch=args.prefetch):
        # a stream of GEMVs as in a decode step: each call is told the weight
        # the next one reads (kq_ctx_prefetch_next), the last one the first
        for i, (w, y) in enumerate(zip(weights, ys)):
            ctx.prefetch_next(weights[(i + 1) % NUM_WEIGHTS] if prefetch else None)
            w.linear(x, m, y, device_ptrs=True)

    with torch.cuda.stream(stream):
        for _ in range(3):  # eager warm-up (module load, first launches)
            step()
    stream.synchronize()

    # Two CUDA graphs of one step each.  `plain` is what the step time is
    # measured on: the 8 GEMVs back to back, nothing between them.  `bracketed`
    # carries a CUDA-event pair around every GEMV's main kernel (event nodes
    # serialise the kernels, so it is only used for the per-kernel average).
    ctx.profile_begin(NUM_WEIGHTS)
    bracketed = torch.cuda.CUDAGraph()
    launches0 = ctx.launch_count
    with torch.cuda.graph(bracketed, stream=stream):
        step()
    launches_per_step = ctx.launch_count - launches0
    plain = torch.cuda.CUDAGraph()  # the bracket budget is used up: no events
    with torch.cuda.graph(plain, stream=stream):
        step()
    plain_np = torch.cuda.CUDAGraph()  # the same stream with the other prefetch setting
    with torch.cuda.graph(plain_np, stream=stream):
        step(prefetch=not args.prefetch)

    for _ in range(max(args.warmup, 3)):
        plain.replay()
        plain_np.replay()
        bracketed.replay()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            plain.replay()
        stop.record(stream)
    stop.synchronize()
    clocks.stop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(stop)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            plain_np.replay()
        stop.record(stream)
    stop.synchronize()
    ms_total_np = start.elapsed_time(stop)

    # per-kernel average over replays of the bracketed graph
    kernel_ms, kernel_n = 0.0, 0
    for _ in range(max(1, min(args.steps, 50))):
        with torch.cuda.stream(stream):
            bracketed.replay()
        ms, cnt = ctx.profile_read()
        kernel_ms += ms
        kernel_n += cnt
    ctx.profile_end()

    t = torch.tensor([ms_total, kernel_ms / max(kernel_n, 1), ms_total_np], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, kernel_ms_avg, ms_total_np = float(t[0]), float(t[1]), float(t[2])
    ms_per_step = ms_total / args.steps
    value = world * NUM_WEIGHTS * alg / (ms_per_step * 1e-3) / 1e9

    # e2e through the C ABI with pinned host buffers (copies inside the timed region)
    ctx.set_stream(None)
    xh = torch.empty((m, k), dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    yh = [torch.empty((m, n), dtype=torch.float32).pin_memory() for _ in range(NUM_WEIGHTS)]
    xn, yn = xh.numpy(), [y.numpy() for y in yh]

    def step_host():
        for w, y in zip(weights, yn):
            w.linear(xn, m, y)  # synchronous: H2D x, kernels, D2H y

    for _ in range(3):
        step_host()
    e2e_steps = max(1, min(args.steps, 400))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * NUM_WEIGHTS * alg * e2e_steps / float(te[0]) / 1e9

    if rank == 0:
        peak, peak_kind = peaks()
        # One kernel per GEMV (the single-token path): its launch duration in
        # the timed graph is the step time per GEMV (CUDA events on the launch
        # stream around the replays).  Otherwise (separate activation prep):
        # the event-bracketed main kernel, timed alone.
        one_kernel = launches_per_step == NUM_WEIGHTS
        kernel_us = ms_per_step * 1e3 / NUM_WEIGHTS if one_kernel else kernel_ms_avg * 1e3
        achieved = alg / (kernel_us * 1e-6) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random GGUF superblocks, x ~ N(0,1))",
            "config": {"workload": f"{args.workload}: {desc}, M={m}, {NUM_WEIGHTS} distinct weights per step",
                       "rows": n, "k": k, "m": m, "weights_per_step": NUM_WEIGHTS,
                       "weight_bytes_per_gemv": wbytes, "algorithmic_bytes_per_gemv": alg,
                       "l2": f"inputs larger than L2 ({NUM_WEIGHTS * wbytes / 1e6:.0f} MB of weights per step)",
                       "parallelism": f"replicas x{world} (independent weights per rank, no data-path collective)",
                       "prefetch": ("each GEMV prefetches the next one's weight into L2 (kq_ctx_prefetch_next)"
                                    if args.prefetch else "off")},
            ("without_prefetch" if args.prefetch else "with_prefetch"): {
                "value": round(world * NUM_WEIGHTS * alg / (ms_total_np / args.steps * 1e-3) / 1e9, 2),
                "ms_per_step": round(ms_total_np / args.steps, 5)},
            "gpu_launches": launches_per_step * args.steps,
            "pct_hbm_peak": round(100.0 * value / world / peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (hbm copy)",
                         "kernel": ("GEMV kernel: timed-graph duration per launch (one kernel per GEMV)"
                                    if one_kernel else
                                    "main GEMV kernel: CUDA events around each launch, averaged over replays"),
                         "kernel_us": round(kernel_us, 3),
                         "kernel_us_isolated": round(kernel_ms_avg * 1e3, 3),
                         "traffic": profiled_traffic(args.workload, m)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": NUM_WEIGHTS * m * k * 4,
                    "d2h_bytes_per_step": NUM_WEIGHTS * m * n * 4,
                    "api": "kq_linear_f32 with host pointers (pinned), synchronous per call"},
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.workload, m)
        print(json.dumps(line), flush=True)
    del plain, plain_np, bracketed
    for w in weights:
        w.free()
    ctx.close()
    return 0


def run_prefill(args, rank, world, local_rank):
    """Prefill dequant-GEMM: y[M][N] = x_bf16[M][K] . W_q4k[N][K] on tcgen05."""
    import torch
    import torch.distributed as dist
    from pesti_b200 import kq, synthetic

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    qtype, _, n, k, desc = PREFILL[args.workload]
    m = args.m if args.m > 1 else 2048
    flops = 2.0 * m * n * k
    wbytes = n * (k // 256) * 144
    xbytes = m * k * 2
    nw = max(4, -(-3 * L2_BYTES // (wbytes + xbytes)))
    ctx = kq.Context(local_rank)
    weights = [kq.Weight(ctx, qtype, synthetic.gguf_weight(qtype, n, k, seed=1000 * rank + i), n, k)
               for i in range(nw)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    xs = [torch.randn((m, k), generator=gen, device=dev).to(torch.bfloat16) for _ in range(nw)]
    ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _ in range(nw)]
    ctx.reserve(weights[0], m)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)

    def step():
        for w, x, y in zip(weights, xs, ys):
            w.linear_bf16(x, m, y, device_ptrs=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    stream.synchronize()
    ctx.profile_begin(nw)
    bracketed = torch.cuda.CUDAGraph()
    launches0 = ctx.launch_count
    with torch.cuda.graph(bracketed, stream=stream):
        step()
    launches_per_step = ctx.launch_count - launches0
    plain = torch.cuda.CUDAGraph()
    with torch.cuda.graph(plain, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            plain.replay()
            bracketed.replay()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            plain.replay()
        stop.record(stream)
    stop.synchronize()
    clocks.stop()
    ms_total = start.elapsed_time(stop)
    kernel_ms, kernel_n = 0.0, 0
    for _ in range(max(1, min(args.steps, 20))):
        with torch.cuda.stream(stream):
            bracketed.replay()
        ms, cnt = ctx.profile_read()
        kernel_ms += ms
        kernel_n += cnt
    ctx.profile_end()
    t = torch.tensor([ms_total, kernel_ms / max(kernel_n, 1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t[0]) / args.steps
    kernel_us = float(t[1]) * 1e3
    value = world * nw * flops / (ms_per_step * 1e-3) / 1e12

    # e2e: host bf16 x and host y through the C ABI (copies inside the timed region)
    ctx.set_stream(None)
    xh = xs[0].cpu().view(torch.int16).numpy().view(np.uint16)
    yh = np.empty((m, n), np.float32)
    e2e_steps = max(1, min(args.steps, 10))
    weights[0].linear_bf16(xh, m, yh)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        weights[0].linear_bf16(xh, m, yh)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * flops * e2e_steps / float(te[0]) / 1e12

    if rank == 0:
        peak, peak_kind = peaks("bf16_tflops", 1590.0)
        achieved = flops / (kernel_us * 1e-6) / 1e12
        line = {
            "metric": PREFILL_METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random GGUF Q4_K superblocks, x ~ N(0,1) in bf16)",
            "config": {"workload": f"{args.workload}: {desc}, M={m}, {nw} distinct weights and inputs per step",
                       "rows": n, "k": k, "m": m, "flops_per_gemm": flops,
                       "l2": f"inputs larger than L2 ({nw * (wbytes + xbytes) / 1e6:.0f} MB per step)",
                       "parallelism": f"replicas x{world}"},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (cuBLAS bf16 burst)",
                         "kernel": "tcgen05 dequant-GEMM kernel: CUDA events around each launch",
                         "kernel_us": round(kernel_us, 3), "traffic": None},
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": m * k * 2,
                    "d2h_bytes_per_step": m * n * 4,
                    "api": "kq_linear_bf16 with host pointers, synchronous per call"},
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    del plain, bracketed
    for w in weights:
        w.free()
    ctx.close()
    return 0


def cpu_decode_sample(cfg, budget_s=12.0):
    """The reference's CPU decode of this model shape, timed on a sample: the
    seven QuantizedLinear::forward calls of one layer (full f32 dequant +
    sequential dot, restated in oracle/kq_oracle.c, legacy block layout) on
    bounded row counts, scaled to a whole token (layers x per-layer time +
    head).  Attention and norms are omitted (under 1% of the CPU time)."""
    import oracle
    from pesti_b200 import synthetic
    D, F, hd = cfg.dim, cfg.ffn, cfg.head_dim
    Dp = -(-D // 256) * 256
    shapes = [(cfg.heads * hd, Dp), (cfg.kv_heads * hd, Dp), (cfg.kv_heads * hd, Dp), (D, Dp), (F, Dp), (F, Dp), (D, F)]
    per_layer = 0.0
    used = 0.0
    for n, k in shapes:
        rows = max(16, min(n, 64))
        data = synthetic.legacy_weight(112, rows, k, seed=1)
        x = synthetic.activations(1, k, seed=2)
        t0 = time.perf_counter()
        oracle.legacy_forward(112, data, k, rows, x, 1, nthreads=1, threads_over_batch=True)
        dt = time.perf_counter() - t0
        used += dt
        per_layer += dt * n / rows
    rows = 64
    data = synthetic.legacy_weight(112, rows, Dp, seed=3)
    x = synthetic.activations(1, Dp, seed=4)
    t0 = time.perf_counter()
    oracle.legacy_forward(112, data, Dp, rows, x, 1, nthreads=1, threads_over_batch=True)
    head = (time.perf_counter() - t0) * cfg.vocab / rows
    sec_per_token = cfg.layers * per_layer + head
    return {"value": round(1.0 / sec_per_token, 6), "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"QuantizedLinear::forward (oracle/kq_oracle.c, legacy blocks) on <=64 rows of each of the "
                      f"7 per-layer projections and the head of {cfg.name}, scaled to {cfg.layers} layers; "
                      f"batch 1, one core (the reference threads over batch rows only)",
            "host_cpus": os.cpu_count()}


def run_decoder(args, rank, world, local_rank):
    """Decode throughput of a synthetic decoder (one step = one token for each
    of `--m` sequences at the context length), tensor-parallel over the ranks."""
    import torch
    import torch.distributed as dist
    from pesti_b200 import decoder as dec, kq

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg_name, ctx_len = DECODERS[args.workload]
    cfg = getattr(dec, cfg_name)
    B = args.m
    ctx = kq.Context(local_rank)
    ctx.set_path(kernel_path(args.path))
    tp = None
    if world > 1:
        tp = kq.TensorParallel(ctx, world, rank, max_out_elems=dec.exchange_elems(cfg, B))
    model = dec.Decoder(cfg, ctx, B, ctx_len, max_new=2, world=world, rank=rank, tp=tp, seed=11,
                        fused=not args.no_fuse, prefetch=args.prefetch)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    model.tokens.copy_(torch.randint(0, cfg.vocab, (B,), generator=gen, device=dev, dtype=torch.int32))
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)
    pos = ctx_len
    with torch.cuda.stream(stream):
        model.step(pos)
    stream.synchronize()
    launches0 = ctx.launch_count
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        model.step(pos)
    launches_per_step = ctx.launch_count - launches0
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            graph.replay()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local_rank)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        stop.record(stream)
    stop.synchronize()
    clocks.stop()
    t = torch.tensor([start.elapsed_time(stop)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t[0]) / args.steps
    value = B / (ms_per_step * 1e-3)  # tokens per second for the whole group

    # e2e: token ids in from pinned host memory, logits out, per step
    tok_h = torch.empty(B, dtype=torch.int32).pin_memory()
    tok_h.copy_(model.tokens.cpu())
    logits_h = torch.empty((B, cfg.vocab), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.steps, 50))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(stream):
            model.tokens.copy_(tok_h, non_blocking=True)
            graph.replay()
            logits_h.copy_(model.logits, non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = B * e2e_steps / float(te[0])

    wb = torch.tensor([float(model.weight_bytes()), float(model.kv_bytes(pos))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(wb)
    step_bytes = float(wb[0] + wb[1])
    if rank == 0:
        peak, peak_kind = peaks()
        achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
        line = {
            "metric": DECODE_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random GGUF K-quant weights, random f16 KV cache, random token ids)",
            "config": {"workload": f"{args.workload}: {cfg.name} decode, batch {B}, context {ctx_len}",
                       "layers": cfg.layers, "dim": cfg.dim, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
                       "head_dim": cfg.head_dim, "ffn": cfg.ffn, "vocab": cfg.vocab, "batch": B,
                       "context": ctx_len, "weight_bytes": int(wb[0]), "kv_bytes_per_step": int(wb[1]),
                       "l2": "inputs larger than L2 (every step streams all weights and the KV cache)",
                       "parallelism": ((f"tensor parallel x{world}: heads, KV cache and FFN blocks split; output and "
                                        f"down projections column-split, their partial residual vectors exchanged "
                                        f"over NVLink peer memory from inside the GEMVs (2 exchanges per layer)")
                                       if model.col_split else
                                       (f"tensor parallel x{world}: heads, KV cache and row blocks sharded, "
                                        f"4 all-gathers per layer over NVLink peer memory")) if world > 1
                       else "single GPU",
                       "fused": ("RoPE + KV append + attention in one kernel; "
                                 + ("RMSNorm, SwiGLU and residual adds inside the single-token GEMVs"
                                    if model.fused else "separate RMSNorm / SwiGLU / add kernels")
                                 if model.fused_attention else "separate kernels"),
                       "prefetch": "next weight into L2 during each linear" if model.prefetch else "off"},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak * world, "unit": "GB/s",
                         "frac": round(achieved / (peak * world), 4),
                         "peak_source": f"{peak_kind} (hbm copy) x {world} GPUs",
                         "kernel": "whole decode step (graph replay): weight + KV bytes / step time",
                         "kernel_us": round(ms_per_step * 1e3, 3), "traffic": None},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": B * 4,
                    "d2h_bytes_per_step": B * cfg.vocab * 4,
                    "api": "graph replay with token ids copied in and logits copied out per step"},
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_decode_sample(cfg)
        print(json.dumps(line), flush=True)
    del graph
    model.close()
    if tp is not None:
        tp.close()
    ctx.close()
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload in PREFILL:
            return run_prefill(args, rank, world, local_rank)
        if args.workload in DECODERS:
            return run_decoder(args, rank, world, local_rank)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
