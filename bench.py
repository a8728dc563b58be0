"""Benchmark of the K-quant quantized-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--m M] [--no-extras]

Default workload: the Q6_K dequant-GEMV of a 14336 -> 4096 down-projection
(N = 4096 output rows, K = 14336, GGUF Q6_K, 48,168,960 weight bytes) at batch
M = 1, f32 activations.  One step = that GEMV over each of W distinct seeded
weights, W chosen so one rank streams more than 3x the 126 MB L2 per step (9
weights, 434 MB, on one GPU), so every GEMV reads its weight from HBM.  Data
is synthetic: seeded random Q6_K superblocks with the distribution the
benchmark names (int8 scales in [-32, 31], d = f16(|N(0, 0.005)|)), x ~ N(0, 1).

Metric: GB/s of algorithmic bytes (weight bytes + M*K*4 + M*N*4 per GEMV).
* value    -- device-resident inputs, a step captured once into a CUDA graph and
              replayed; CUDA events on the launch stream; max over ranks.
* e2e      -- the same GEMVs through the public API with host buffers (pinned):
              host->device copy of x and device->host copy of every y per step.
* roofline -- the GEMV kernel alone against MEASURED_PEAKS.json's HBM copy
              bandwidth.
* cpu_baseline -- the reference's CPU algorithm (QuantizedLinear::forward over
              tile_dequant blocks, restated in oracle/kq_oracle.c) on the same
              shape, timed on this host; plus the same algorithm threaded over
              output rows on every core.

Multi-GPU (torchrun, N > 1): strong scaling of the same GEMVs -- each weight's
rows are split over the N ranks and every call runs kq_tp_linear_f32 (this
rank's rows, then an all-gather of the output slices over NVLink peer memory
into the full y on every rank), all inside the timed region.

Sub-records of the default line (skipped with --no-extras):
* q4k_gemv -- the Q4_K 4096x4096 decode GEMV (M = 1), per call in a stream of
              distinct weights and timed alone;
* legacy_gemv -- (one GPU) the default line's GEMV over the reference's own
              42-byte Q6_K blocks;
* prefill  -- (one GPU) the Q4_K 14336x4096 bf16 prefill dequant-GEMM at M =
              4096 tokens, TFLOP/s against the sustained bf16 peak;
* decode   -- the Llama-3-8B-shaped Q4_K_M decode step (context 2048) at
              batch 1, 8 and 32, tokens/s over the N GPUs (tensor parallel).

Other workloads (--workload): q4k-gemv, prefill-4096 / prefill-14336 (--m
tokens), decode-llama8b / decode-qwen05b (--batch), and the single-op
profiling targets attention (--batch, --len) and norm-swiglu (--rows, --k).

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
    # the other K-quant types on the same 4096x4096 shape (their CPU legs run the
    # reference's Q5_K rows; Q2_K / Q3_K have no QuantizedLinear form there)
    "q5k-gemv": (13, 113, 4096, 4096, "Q5_K dequant+GEMV 4096x4096"),
    "q3k-gemv": (11, 113, 4096, 4096, "Q3_K dequant+GEMV 4096x4096"),
    "q2k-gemv": (10, 113, 4096, 4096, "Q2_K dequant+GEMV 4096x4096"),
}
# bytes per 256 weights (GGUF) or per 16 weights (the reference's legacy blocks)
BLOCK_BYTES = {10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
               112: (16, 28), 113: (16, 36), 114: (16, 42)}
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
OPS = ("attention", "norm-swiglu")
L2_BYTES = 126 * 1024 * 1024  # B200 L2
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_SUSTAINED = 1400.0


def num_weights(wbytes, world=1):
    """Distinct weights per step: at least 8, and enough that one rank streams
    more than 3x the L2 per step when each holds 1/world of every weight."""
    return max(8, -(-3 * L2_BYTES * world // wbytes))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(PREFILL) + sorted(DECODERS) + list(OPS),
                   default="q6k-gemv")
    p.add_argument("--m", "--batch", dest="m", type=int, default=1,
                   help="tokens per call (decode batch); --batch is the form to use under torchrun")
    p.add_argument("--path", choices=["auto", "tcgen05", "mma", "dp4a", "imma"], default="auto",
                   help="kernel family for the GEMV (auto: dp4a m=1, integer MMA / mma.sync m<=64, tcgen05 above)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--layout", choices=["gguf", "legacy"], default="gguf",
                   help="GEMV workloads: GGUF superblocks, or the reference's own 28 / 42-byte 16-weight blocks")
    p.add_argument("--no-extras", action="store_true", help="default line only, without its sub-records")
    p.add_argument("--prefetch", action="store_true",
                   help="each GEMV prefetches the next one's weight into L2 (kq_ctx_prefetch_next)")
    p.add_argument("--no-fuse", action="store_true",
                   help="decoders: separate RMSNorm / SwiGLU / add kernels at batch 1")
    p.add_argument("--step", action="store_true",
                   help="decoders at batch 1: the persistent step kernel instead of one kernel per operation")
    p.add_argument("--len", type=int, default=2049, help="attention: positions attended (the new one included)")
    p.add_argument("--rows", type=int, default=28672, help="norm-swiglu: weight rows ((gate, up) pairs)")
    p.add_argument("--k", type=int, default=4096, help="norm-swiglu: in_features")
    return p.parse_args()


def kernel_path(name):
    from pesti_b200 import kq
    return {"auto": kq.KQ_PATH_AUTO, "tcgen05": kq.KQ_PATH_TCGEN05, "mma": kq.KQ_PATH_MMA,
            "dp4a": kq.KQ_PATH_DP4A, "imma": kq.KQ_PATH_IMMA}[name]


def algorithmic_bytes(qtype, n, k, m):
    per, bs = BLOCK_BYTES[qtype]
    wbytes = n * ((k + per - 1) // per) * bs
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

    def __init__(self, device_index, period_s=0.005):
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

    def _sample(self):
        n = self.nvml
        try:
            self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
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


# ---- small helpers ---------------------------------------------------------------

def max_over_ranks(values, dev, world):
    """Element-wise max over the ranks of a list of floats (device all-reduce)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def timed_replays(graph, stream, steps, local_rank, world):
    """Replay `graph` `steps` times between CUDA events on `stream`, with a
    barrier and a synchronize on both sides and NVML clock samples during the
    timed region; returns (ms, clocks)."""
    import torch
    stream.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        stop.record(stream)
    stop.synchronize()
    clocks.stop()
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(stop), clocks.summary()


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

    def run(self, row0, rows, all_cores=False, legacy_bytes=False):
        """Forward over rows [row0, row0+rows); returns (seconds, algorithmic
        bytes: of the GGUF workload, or of the legacy blocks themselves).
        all_cores: the same algorithm threaded over output rows."""
        sub = self.data[row0:row0 + rows]
        t0 = time.perf_counter()
        self.oracle.legacy_forward(self.legacy, sub, self.k, rows, self.x, self.m,
                                   nthreads=os.cpu_count() or 1, threads_over_batch=not all_cores)
        dt = time.perf_counter() - t0
        return dt, algorithmic_bytes(self.legacy if legacy_bytes else self.qtype, rows, self.k, self.m)[1]


def cpu_baseline(workload, m, budget_s=12.0, legacy=False):
    ref = CpuReference(workload, m)
    n, k = ref.n, ref.k
    total_t, total_b, passes = 0.0, 0, 0
    while total_t < budget_s and passes < 64:
        dt, alg = ref.run(0, n, legacy_bytes=legacy)
        total_t += dt
        total_b += alg
        passes += 1
    # the same algorithm with its output rows spread over every core
    at, ab, ap = 0.0, 0, 0
    while at < budget_s / 4 and ap < 256:
        dt, alg = ref.run(0, n, all_cores=True, legacy_bytes=legacy)
        at += dt
        ab += alg
        ap += 1
    cores = min(m, os.cpu_count() or 1)
    return {"value": round(total_b / total_t / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{passes} full passes of QuantizedLinear::forward (full f32 dequant + sequential "
                      f"dot, threads over batch rows) over a {n}x{k} pesti-legacy weight at M={m}; "
                      f"bytes counted as the {'legacy blocks' if legacy else 'GGUF workload'}'s",
            "host_cpus": os.cpu_count(),
            "all_cores": {"value": round(ab / at / 1e9, 4), "unit": "GB/s", "cores": os.cpu_count() or 1,
                          "sample": f"{ap} passes of the same algorithm threaded over output rows"}}


def cpu_decode_sample(cfg, budget_rows=64):
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
    for n, k in shapes:
        rows = max(16, min(n, budget_rows))
        data = synthetic.legacy_weight(112, rows, k, seed=1)
        x = synthetic.activations(1, k, seed=2)
        t0 = time.perf_counter()
        oracle.legacy_forward(112, data, k, rows, x, 1, nthreads=1, threads_over_batch=True)
        dt = time.perf_counter() - t0
        per_layer += dt * n / rows
    rows = budget_rows
    data = synthetic.legacy_weight(112, rows, Dp, seed=3)
    x = synthetic.activations(1, Dp, seed=4)
    t0 = time.perf_counter()
    oracle.legacy_forward(112, data, Dp, rows, x, 1, nthreads=1, threads_over_batch=True)
    head = (time.perf_counter() - t0) * cfg.vocab / rows
    sec_per_token = cfg.layers * per_layer + head
    return {"value": round(1.0 / sec_per_token, 6), "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"QuantizedLinear::forward (oracle/kq_oracle.c, legacy blocks) on <={budget_rows} rows of "
                      f"each of the 7 per-layer projections and the head of {cfg.name}, scaled to {cfg.layers} "
                      f"layers; batch 1, one core (the reference threads over batch rows only)",
            "host_cpus": os.cpu_count()}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    if args.workload in OPS:
        print(json.dumps({"impl": "reference", "unavailable": f"{args.workload} is a single-op profiling target "
                                                              f"with no CPU counterpart timed here"}), flush=True)
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


# ---- decode GEMV ---------------------------------------------------------------

def measure_gemv(args, workload, m, rank, world, local_rank, steps, warmup):
    """A step of W distinct GEMVs of `workload` (rows split over the ranks at
    world > 1, each call all-gathering its output): device-resident timing,
    per-kernel timing and the host-buffer e2e.  Returns a dict (rank 0's view
    of the max over ranks)."""
    import torch
    from pesti_b200 import decoder as dec, kq, synthetic

    dev = torch.device("cuda", local_rank)
    qtype, legacy_type, n, k, desc = WORKLOADS[workload]
    legacy = getattr(args, "layout", "gguf") == "legacy"
    if legacy:
        if qtype not in (12, 14):
            raise SystemExit(f"{workload}: the reference's legacy blocks exist for Q4_K and Q6_K only")
        qtype = legacy_type
        desc = desc.replace("Q6_K", "Q6_K (reference 42-byte blocks)").replace("Q4_K", "Q4_K (reference 28-byte blocks)")
    wbytes, alg = algorithmic_bytes(qtype, n, k, m)
    nw = num_weights(wbytes, world)
    r0, r1 = kq.shard_rows(n, world, rank)
    ctx = kq.Context(local_rank)
    tp = kq.TensorParallel(ctx, world, rank, max_out_elems=m * n) if world > 1 else None
    weights = []
    for i in range(nw):  # the same seeded weights on every rank; each keeps its rows
        if legacy:
            full = torch.from_numpy(synthetic.legacy_weight(qtype, n, k, seed=1000 + i)).to(dev)
        elif qtype in (12, 14):
            full = dec.gguf_weight_device(qtype, n, k, seed=1000 + i, device=dev)
        else:
            full = torch.from_numpy(synthetic.gguf_weight(qtype, n, k, seed=1000 + i)).to(dev)
        weights.append(kq.Weight(ctx, qtype, full[r0:r1].contiguous(), r1 - r0, k))
        del full
    x = torch.from_numpy(synthetic.activations(m, k, seed=7)).to(dev)
    ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _ in range(nw)]
    ctx.set_path(kernel_path(args.path))
    ctx.reserve(weights[0], m)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)

    def step(prefetch=args.prefetch):
        # a stream of GEMVs as in a decode step: each call may be told the
        # weight the next one reads (kq_ctx_prefetch_next)
        for i, (w, y) in enumerate(zip(weights, ys)):
            ctx.prefetch_next(weights[(i + 1) % nw] if prefetch else None)
            if tp is None:
                w.linear(x, m, y, device_ptrs=True)
            else:
                tp.linear(w, r0, n, x, m, y)

    with torch.cuda.stream(stream):
        for _ in range(3):  # eager warm-up (module load, first launches)
            step()
    stream.synchronize()

    # `plain` is what the step time is measured on: the GEMVs back to back.
    # `bracketed` carries a CUDA-event pair around every GEMV's main kernel
    # (event nodes serialise the kernels: the per-call time of a GEMV alone).
    ctx.profile_begin(nw)
    bracketed = torch.cuda.CUDAGraph()
    launches0 = ctx.launch_count
    with torch.cuda.graph(bracketed, stream=stream):
        step()
    launches_per_step = ctx.launch_count - launches0
    plain = torch.cuda.CUDAGraph()  # the bracket budget is used up: no events
    with torch.cuda.graph(plain, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            plain.replay()
            bracketed.replay()
    ms_total, clocks = timed_replays(plain, stream, steps, local_rank, world)

    kernel_ms, kernel_n = 0.0, 0
    for _ in range(max(1, min(steps, 50))):
        with torch.cuda.stream(stream):
            bracketed.replay()
        ms, cnt = ctx.profile_read()
        kernel_ms += ms
        kernel_n += cnt
    ctx.profile_end()
    stream.synchronize()
    barrier(world)

    # e2e through the public API with pinned host buffers (copies inside the timed region)
    xh = torch.empty((m, k), dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    yh = [torch.empty((m, n), dtype=torch.float32).pin_memory() for _ in range(nw)]
    if tp is None:
        ctx.set_stream(None)
        xn, yn = xh.numpy(), [y.numpy() for y in yh]

        def step_host():
            # every call queues H2D x, its kernels and D2H y (KQ_ASYNC); one wait per step
            for w, y in zip(weights, yn):
                w.linear(xn, m, y, queue=True)
            ctx.synchronize()
        api = ("kq_linear_f32 with host pointers (pinned): each call queues its H2D copy of x, kernels and D2H "
               "copy of y (KQ_ASYNC), one kq_ctx_synchronize per step")
    else:
        xd = torch.empty_like(x)

        def step_host():
            with torch.cuda.stream(stream):
                xd.copy_(xh, non_blocking=True)
                for w, yd, y in zip(weights, ys, yh):
                    tp.linear(w, r0, n, xd, m, yd)
                    y.copy_(yd, non_blocking=True)
            stream.synchronize()
        api = "x copied in from pinned host memory, kq_tp_linear_f32 per weight, every y copied out, per step"
    for _ in range(3):
        step_host()
    e2e_steps = max(1, min(steps, 400))
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_host()
    e2e_s = time.perf_counter() - t0

    ms_total, kernel_ms_avg, e2e_s = max_over_ranks([ms_total, kernel_ms / max(kernel_n, 1), e2e_s], dev, world)
    ms_per_step = ms_total / steps
    res = {
        "workload": workload, "desc": desc, "n": n, "k": k, "m": m, "qtype": qtype, "weights": nw,
        "wbytes": wbytes, "alg": alg, "ms_per_step": ms_per_step,
        "value": nw * alg / (ms_per_step * 1e-3) / 1e9,
        "launches_per_step": launches_per_step, "kernel_us_isolated": kernel_ms_avg * 1e3,
        # one kernel per GEMV (the single-token path on one GPU): the timed
        # graph's duration per launch is the kernel's streaming time
        "one_kernel": launches_per_step == nw,
        "e2e": nw * alg * e2e_steps / e2e_s / 1e9, "e2e_api": api,
        "h2d": m * k * 4 if tp is not None else nw * m * k * 4, "d2h": nw * m * n * 4, "clocks": clocks,
        "rows_per_rank": r1 - r0, "legacy": legacy,
    }
    del plain, bracketed
    for w in weights:
        w.free()
    if tp is not None:
        tp.close()
    ctx.close()
    return res


def gemv_roofline(res, world):
    peak, peak_kind = peaks()
    rank_alg = res["wbytes"] * res["rows_per_rank"] / res["n"] + res["m"] * res["k"] * 4 + \
        res["m"] * res["rows_per_rank"] * 4
    if res["one_kernel"]:
        kernel_us = res["ms_per_step"] * 1e3 / res["weights"]
        how = "GEMV kernel: timed-graph duration per launch (one kernel per GEMV)"
    else:
        kernel_us = res["kernel_us_isolated"]
        how = "main GEMV kernel: CUDA events around each launch, averaged over replays"
    achieved = rank_alg / (kernel_us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (hbm copy)", "kernel": how,
            "kernel_us": round(kernel_us, 3), "kernel_us_isolated": round(res["kernel_us_isolated"], 3),
            "frac_isolated": round(rank_alg / (res["kernel_us_isolated"] * 1e-6) / 1e9 / peak, 4),
            "algorithmic_bytes_per_launch": int(rank_alg),
            "traffic": profiled_traffic(res["workload"], res["m"]) if world == 1 and not res["legacy"] else None}


def run_gemv(args, rank, world, local_rank):
    res = measure_gemv(args, args.workload, args.m, rank, world, local_rank, args.steps, args.warmup)
    extras = {}
    if args.workload == "q6k-gemv" and args.m == 1 and args.layout == "gguf" and not args.no_extras:
        extras = measure_extras(args, rank, world, local_rank)
    if rank != 0:
        return 0
    peak, _ = peaks()
    m, nw = res["m"], res["weights"]
    if world > 1:
        par = (f"row-sharded x{world}: each weight's rows split over the ranks ({res['rows_per_rank']} rows per "
               f"rank), kq_tp_linear_f32 all-gathers every output over NVLink peer memory inside the timed region")
    else:
        par = "single GPU"
    line = {
        "metric": METRIC, "value": round(res["value"], 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 5),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random GGUF superblocks, x ~ N(0,1))",
        "config": {"workload": f"{args.workload}: {res['desc']}, M={m}, {nw} distinct weights per step",
                   "layout": args.layout,
                   "rows": res["n"], "k": res["k"], "m": m, "weights_per_step": nw,
                   "weight_bytes_per_gemv": res["wbytes"], "algorithmic_bytes_per_gemv": res["alg"],
                   "l2": f"inputs larger than L2 ({nw * res['wbytes'] / world / 1e6:.0f} MB of weights per rank "
                         f"per step)",
                   "parallelism": par,
                   "prefetch": ("each GEMV prefetches the next one's weight into L2 (kq_ctx_prefetch_next)"
                                if args.prefetch else "off")},
        "gpu_launches": res["launches_per_step"] * args.steps,
        "pct_hbm_peak": round(100.0 * res["value"] / world / peak, 2),
        "roofline": gemv_roofline(res, world),
        "e2e": {"value": round(res["e2e"], 2), "unit": "GB/s", "h2d_bytes_per_step": res["h2d"],
                "d2h_bytes_per_step": res["d2h"], "api": res["e2e_api"]},
        "clocks": res["clocks"],
    }
    line.update(extras)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, m, legacy=args.layout == "legacy")
    print(json.dumps(line), flush=True)
    return 0


def measure_extras(args, rank, world, local_rank):
    """The sub-records of the default line (see the module docstring)."""
    from pesti_b200 import decoder as dec
    out = {}
    steps = max(args.steps, 10)
    q4 = measure_gemv(args, "q4k-gemv", 1, rank, world, local_rank, steps, args.warmup)
    rl = gemv_roofline(q4, world)
    out["q4k_gemv"] = {"workload": "Q4_K dequant+GEMV 4096x4096, M=1" + (f", rows split x{world}" if world > 1
                                                                          else ""),
                       "weights_per_step": q4["weights"], "value": round(q4["value"], 2), "unit": "GB/s",
                       "us_per_call": round(q4["ms_per_step"] * 1e3 / q4["weights"], 3),
                       "roofline": rl, "e2e": round(q4["e2e"], 2), "clocks": q4["clocks"]}
    if world == 1:
        # the same GEMV over the reference's own 42-byte blocks (the layout its
        # QuantizedLinear holds today), bytes counted as those blocks
        import copy
        la = copy.copy(args)
        la.layout = "legacy"
        lg = measure_gemv(la, "q6k-gemv", 1, rank, world, local_rank, steps, args.warmup)
        rl = gemv_roofline(lg, world)
        out["legacy_gemv"] = {"workload": "Q6_K dequant+GEMV 4096x14336, M=1, the reference's 42-byte blocks",
                              "weights_per_step": lg["weights"], "value": round(lg["value"], 2), "unit": "GB/s",
                              "us_per_call": round(lg["ms_per_step"] * 1e3 / lg["weights"], 3), "roofline": rl,
                              "e2e": round(lg["e2e"], 2), "clocks": lg["clocks"]}
        p = measure_prefill(args, "prefill-14336", 4096, rank, world, local_rank, min(steps, 20), args.warmup)
        sus, sus_kind = peaks("bf16_tflops_sustained", FALLBACK_BF16_SUSTAINED)
        out["prefill"] = {"workload": "Q4_K dequant-GEMM 14336x4096, bf16 x, M=4096 tokens, f32 accumulate",
                          "value": round(p["value"], 2), "unit": "TFLOP/s",
                          "kernel_us": round(p["kernel_us"], 2),
                          "achieved": round(p["achieved"], 2), "peak_sustained": sus,
                          "frac": round(p["achieved"] / sus, 4),
                          "peak_source": f"{sus_kind} (cuBLAS bf16, sustained: the kernel runs inside a long "
                                         f"timed region)", "clocks": p["clocks"]}
    decode = {}
    for batch in (1, 8, 32):
        d = measure_decoder(args, "decode-llama8b", batch, rank, world, local_rank, min(steps, 50), args.warmup)
        peak, _ = peaks()
        decode[f"batch{batch}"] = {"value": round(d["value"], 2), "unit": "tok/s", "ms_per_step": round(
            d["ms_per_step"], 4), "frac": round(d["achieved"] / (peak * world), 4),
            "step_bytes": int(d["step_bytes"]), "e2e": round(d["e2e"], 2), "parallelism": d["parallelism"],
            "gpu_launches_per_step": d["launches_per_step"], "clocks": d["clocks"]}
    out["decode"] = {"workload": "Llama-3-8B-shaped Q4_K_M decode step, context 2048 (weight + KV bytes / step "
                                 "time against N x the measured HBM copy peak)", **decode}
    if world == 1 and not args.no_cpu_baseline:
        out["decode"]["cpu_baseline"] = cpu_decode_sample(dec.LLAMA3_8B, budget_rows=32)
    return out


# ---- prefill -------------------------------------------------------------------

def measure_prefill(args, workload, m, rank, world, local_rank, steps, warmup):
    """Prefill dequant-GEMM: y[M][N] = x_bf16[M][K] . W_q4k[N][K] on tcgen05."""
    import torch
    from pesti_b200 import decoder as dec, kq

    dev = torch.device("cuda", local_rank)
    qtype, _, n, k, desc = PREFILL[workload]
    flops = 2.0 * m * n * k
    wbytes = n * (k // 256) * 144
    xbytes = m * k * 2
    nw = max(4, -(-3 * L2_BYTES // (wbytes + xbytes)))
    ctx = kq.Context(local_rank)
    weights = [kq.Weight(ctx, qtype, dec.gguf_weight_device(qtype, n, k, seed=1000 * rank + i, device=dev), n, k)
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
        for _ in range(max(warmup, 3)):
            plain.replay()
            bracketed.replay()
    ms_total, clocks = timed_replays(plain, stream, steps, local_rank, world)
    kernel_ms, kernel_n = 0.0, 0
    for _ in range(max(1, min(steps, 20))):
        with torch.cuda.stream(stream):
            bracketed.replay()
        ms, cnt = ctx.profile_read()
        kernel_ms += ms
        kernel_n += cnt
    ctx.profile_end()

    # e2e: host bf16 x and host y through the C ABI (copies inside the timed region)
    ctx.set_stream(None)
    xh = xs[0].cpu().view(torch.int16).numpy().view(np.uint16)
    yh = np.empty((m, n), np.float32)
    e2e_steps = max(1, min(steps, 10))
    weights[0].linear_bf16(xh, m, yh)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        weights[0].linear_bf16(xh, m, yh)
    e2e_s = time.perf_counter() - t0
    ms_total, kernel_ms_avg, e2e_s = max_over_ranks([ms_total, kernel_ms / max(kernel_n, 1), e2e_s], dev, world)
    ms_per_step = ms_total / steps
    res = {"desc": desc, "n": n, "k": k, "m": m, "flops": flops, "weights": nw, "ms_per_step": ms_per_step,
           "value": world * nw * flops / (ms_per_step * 1e-3) / 1e12, "kernel_us": kernel_ms_avg * 1e3,
           "achieved": flops / (kernel_ms_avg * 1e-3) / 1e12, "launches_per_step": launches_per_step,
           "e2e": world * flops * e2e_steps / e2e_s / 1e12, "clocks": clocks,
           "l2": f"inputs larger than L2 ({nw * (wbytes + xbytes) / 1e6:.0f} MB per step)"}
    del plain, bracketed
    for w in weights:
        w.free()
    ctx.close()
    return res


def run_prefill(args, rank, world, local_rank):
    m = args.m if args.m > 1 else 2048
    r = measure_prefill(args, args.workload, m, rank, world, local_rank, args.steps, args.warmup)
    if rank != 0:
        return 0
    peak, peak_kind = peaks("bf16_tflops", FALLBACK_BF16_TFLOPS)
    sus, _ = peaks("bf16_tflops_sustained", FALLBACK_BF16_SUSTAINED)
    line = {
        "metric": PREFILL_METRIC, "value": round(r["value"], 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random GGUF Q4_K superblocks, x ~ N(0,1) in bf16)",
        "config": {"workload": f"{args.workload}: {r['desc']}, M={m}, {r['weights']} distinct weights and inputs "
                               f"per step", "rows": r["n"], "k": r["k"], "m": m, "flops_per_gemm": r["flops"],
                   "l2": r["l2"], "parallelism": f"replicas x{world}"},
        "gpu_launches": r["launches_per_step"] * args.steps,
        "roofline": {"bound": "tensor", "achieved": round(r["achieved"], 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(r["achieved"] / peak, 4), "peak_source": f"{peak_kind} (cuBLAS bf16 burst)",
                     "frac_sustained": round(r["achieved"] / sus, 4),
                     "kernel": "tcgen05 dequant-GEMM kernel: CUDA events around each launch",
                     "kernel_us": round(r["kernel_us"], 3), "traffic": None},
        "e2e": {"value": round(r["e2e"], 2), "unit": "TFLOP/s", "h2d_bytes_per_step": m * r["k"] * 2,
                "d2h_bytes_per_step": m * r["n"] * 4, "api": "kq_linear_bf16 with host pointers, synchronous per call"},
        "clocks": r["clocks"],
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- decoder -------------------------------------------------------------------

def measure_decoder(args, workload, batch, rank, world, local_rank, steps, warmup):
    """Decode throughput of a synthetic decoder (one step = one token for each
    of `batch` sequences at the context length), tensor-parallel over the ranks."""
    import torch
    from pesti_b200 import decoder as dec, kq

    dev = torch.device("cuda", local_rank)
    cfg_name, ctx_len = DECODERS[workload]
    cfg = getattr(dec, cfg_name)
    B = batch
    ctx = kq.Context(local_rank)
    ctx.set_path(kernel_path(args.path))
    tp = kq.TensorParallel(ctx, world, rank, max_out_elems=dec.exchange_elems(cfg, B)) if world > 1 else None
    model = dec.Decoder(cfg, ctx, B, ctx_len, max_new=2, world=world, rank=rank, tp=tp, seed=11,
                        fused=not args.no_fuse, prefetch=args.prefetch, step_kernel=args.step)
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
        for _ in range(max(warmup, 3)):
            graph.replay()
    ms_total, clocks = timed_replays(graph, stream, steps, local_rank, world)

    # e2e: token ids in from pinned host memory, logits out, per step
    tok_h = torch.empty(B, dtype=torch.int32).pin_memory()
    tok_h.copy_(model.tokens.cpu())
    logits_h = torch.empty((B, cfg.vocab), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(steps, 50))
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(stream):
            model.tokens.copy_(tok_h, non_blocking=True)
            graph.replay()
            logits_h.copy_(model.logits, non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    ms_total, e2e_s = max_over_ranks([ms_total, e2e_s], dev, world)
    wb = torch.tensor([float(model.weight_bytes()), float(model.kv_bytes(pos))], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(wb)
    ms_per_step = ms_total / steps
    step_bytes = float(wb[0] + wb[1])
    if world == 1:
        par = "single GPU"
    elif model.col_batch:
        par = (f"tensor parallel x{world}: heads, KV cache and FFN blocks split; output and down projections "
               f"column-split, each partial residual block all-reduced over NVLink peer memory (2 exchanges per "
               f"layer)")
    elif model.col_split:
        par = (f"tensor parallel x{world}: heads, KV cache and FFN blocks split; output and down projections "
               f"column-split, their partial residual vectors exchanged over NVLink peer memory from inside the "
               f"GEMVs (2 exchanges per layer)")
    else:
        par = (f"tensor parallel x{world}: heads, KV cache and row blocks sharded, 4 all-gathers per layer over "
               f"NVLink peer memory")
    if model.step_kernel:
        par += "; the step (all layers and the head) is one persistent kernel launch"
    res = {"cfg": cfg, "ctx_len": ctx_len, "batch": B, "ms_per_step": ms_per_step, "value": B / (ms_per_step * 1e-3),
           "e2e": B * e2e_steps / e2e_s, "launches_per_step": launches_per_step, "clocks": clocks,
           "weight_bytes": int(wb[0]), "kv_bytes": int(wb[1]), "step_bytes": step_bytes,
           "achieved": step_bytes / (ms_per_step * 1e-3) / 1e9, "parallelism": par,
           "fused": ("RoPE + KV append + attention in one kernel; "
                     + ("RMSNorm, SwiGLU and residual adds inside the single-token GEMVs"
                        if model.fused else "separate RMSNorm / SwiGLU / add kernels")
                     if model.fused_attention else "separate kernels"),
           "prefetch": "next weight into L2 during each linear" if model.prefetch else "off"}
    del graph
    model.close()
    if tp is not None:
        tp.close()
    ctx.close()
    torch.cuda.empty_cache()
    return res


def run_decoder(args, rank, world, local_rank):
    r = measure_decoder(args, args.workload, args.m, rank, world, local_rank, args.steps, args.warmup)
    if rank != 0:
        return 0
    cfg, B = r["cfg"], r["batch"]
    peak, peak_kind = peaks()
    line = {
        "metric": DECODE_METRIC, "value": round(r["value"], 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random GGUF K-quant weights, random f16 KV cache, random token ids)",
        "config": {"workload": f"{args.workload}: {cfg.name} decode, batch {B}, context {r['ctx_len']}",
                   "layers": cfg.layers, "dim": cfg.dim, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
                   "head_dim": cfg.head_dim, "ffn": cfg.ffn, "vocab": cfg.vocab, "batch": B,
                   "context": r["ctx_len"], "weight_bytes": r["weight_bytes"], "kv_bytes_per_step": r["kv_bytes"],
                   "l2": "inputs larger than L2 (every step streams all weights and the KV cache)",
                   "parallelism": r["parallelism"], "fused": r["fused"], "prefetch": r["prefetch"]},
        "gpu_launches": r["launches_per_step"] * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(r["achieved"], 2), "peak": peak * world, "unit": "GB/s",
                     "frac": round(r["achieved"] / (peak * world), 4),
                     "peak_source": f"{peak_kind} (hbm copy) x {world} GPUs",
                     "kernel": "whole decode step (graph replay): weight + KV bytes / step time",
                     "kernel_us": round(r["ms_per_step"] * 1e3, 3), "traffic": None},
        "e2e": {"value": round(r["e2e"], 2), "unit": "tok/s", "h2d_bytes_per_step": B * 4,
                "d2h_bytes_per_step": B * cfg.vocab * 4,
                "api": "graph replay with token ids copied in and logits copied out per step"},
        "clocks": r["clocks"],
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_sample(cfg)
    print(json.dumps(line), flush=True)
    return 0


# ---- single-op profiling targets -------------------------------------------------

def run_op(args, rank, world, local_rank):
    """One device op of the decode path run repeatedly (what an ncu capture of
    one kernel needs): `attention` is RoPE + KV append + GQA attention of the
    Llama-3-8B-shaped step (--batch, --len positions); `norm-swiglu` the fused
    RMSNorm + (gate, up) GEMV + SwiGLU (--rows, --k).  Seeded random inputs;
    GB/s of the bytes the op must read."""
    import ctypes

    import torch
    from pesti_b200 import decoder as dec, kq

    if world > 1 and rank != 0:
        return 0
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    dev = torch.device("cuda", local_rank)
    ctx = kq.Context(local_rank)
    lib = dec._bind(ctx.lib)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    if args.workload == "attention":
        B, hq, hkv, hd = args.m, 32, 8, 128
        max_seq = args.len + 1
        ld = (hq + 2 * hkv) * hd
        qkv = torch.randn((B, ld), generator=gen, device=dev)
        kc = torch.randn((B, hkv, max_seq, hd), generator=gen, device=dev).half()
        vc = torch.randn((B, hkv, max_seq, hd), generator=gen, device=dev).half()
        out = torch.empty((B, hq * hd), device=dev)
        sbytes = lib.kq_dec_attention_scratch(ctx.handle, B, hq, hkv, hd, max_seq)
        scratch = torch.zeros(max(sbytes // 4, 1), device=dev)
        pos = args.len - 1

        def call():
            ctx.check(lib.kq_dec_rope_attention(ctx.handle, ptr(qkv), ld, ptr(kc), ptr(vc), ptr(out), hq * hd, B, hq,
                                                hkv, hd, pos, max_seq, 5e5, ptr(scratch), sbytes),
                      "kq_dec_rope_attention")
        what = f"rope+attention batch {B}, {args.len} positions, {hq}/{hkv} heads of {hd}"
        nbytes = 2 * B * hkv * args.len * hd * 2
    else:
        qt = kq.KQ_GGUF_Q4_K
        w = kq.Weight(ctx, qt, dec.gguf_weight_device(qt, args.rows, args.k, 5, dev), args.rows, args.k)
        x = torch.randn((1, args.k), generator=gen, device=dev)
        nw = 1.0 + 0.1 * torch.randn(args.k, generator=gen, device=dev)
        y = torch.empty((1, args.rows // 2), device=dev)

        def call():
            ctx.check(lib.kq_dec_norm_linear(ctx.handle, w.handle, ptr(x), ptr(nw), args.k, 1e-5, 0, None, ptr(y), 0),
                      "kq_dec_norm_linear")
        what = f"RMSNorm + Q4_K {args.rows}x{args.k} (gate, up) pairs + SwiGLU, one token"
        nbytes = w.device_bytes
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            call()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"metric": f"{args.workload} op GB/s", "value": round(nbytes / us / 1e3, 2), "unit": "GB/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": {"workload": what + " (same inputs each call)"},
                      "gpu_launches": args.steps}), flush=True)
    ctx.set_stream(None)
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
    else:
        import torch
        torch.cuda.set_device(local_rank)
    try:
        if args.workload in PREFILL:
            return run_prefill(args, rank, world, local_rank)
        if args.workload in DECODERS:
            return run_decoder(args, rank, world, local_rank)
        if args.workload in OPS:
            return run_op(args, rank, world, local_rank)
        return run_gemv(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
