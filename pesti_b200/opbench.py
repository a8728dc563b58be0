"""Run one device op of the decode path repeatedly: a timing and profiling
harness for single kernels (what an ncu capture of one kernel needs: a
small program that launches it a few times on realistic shapes).

    python -m pesti_b200.opbench attention --batch 32 --len 2049
    python -m pesti_b200.opbench norm-swiglu --rows 28672 --k 4096
    python -m pesti_b200.opbench linear --type q6k --rows 4096 --k 14336

Inputs are seeded random tensors of the given shapes (GGUF superblocks as in
pesti_b200.decoder.gguf_weight_device).  Prints the mean time per call
measured with CUDA events on the context stream.
"""
from __future__ import annotations

import argparse
import ctypes

from . import decoder as dec
from . import kq

_TYPES = {"q4k": kq.KQ_GGUF_Q4_K, "q6k": kq.KQ_GGUF_Q6_K}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def main(argv=None) -> int:
    import torch
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("op", choices=["attention", "norm-swiglu", "linear"])
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--len", type=int, default=2049, help="attention: positions attended (the new one included)")
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--type", choices=sorted(_TYPES), default="q4k")
    p.add_argument("--rows", type=int, default=28672)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--calls", type=int, default=20)
    a = p.parse_args(argv)

    ctx = kq.Context(0)
    lib = dec._bind(ctx.lib)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    ctx.set_stream(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)

    if a.op == "attention":
        B, hq, hkv, hd = a.batch, a.heads, a.kv_heads, a.head_dim
        max_seq = a.len + 1
        ld = (hq + 2 * hkv) * hd
        qkv = torch.randn((B, ld), generator=gen, device=dev)
        kc = torch.randn((B, hkv, max_seq, hd), generator=gen, device=dev).half()
        vc = torch.randn((B, hkv, max_seq, hd), generator=gen, device=dev).half()
        out = torch.empty((B, hq * hd), device=dev)
        sbytes = lib.kq_dec_attention_scratch(ctx.handle, B, hq, hkv, hd, max_seq)
        scratch = torch.zeros(max(sbytes // 4, 1), device=dev)
        pos = a.len - 1

        def call():
            ctx.check(lib.kq_dec_rope_attention(ctx.handle, _ptr(qkv), ld, _ptr(kc), _ptr(vc), _ptr(out), hq * hd,
                                                B, hq, hkv, hd, pos, max_seq, 5e5, _ptr(scratch), sbytes),
                      "kq_dec_rope_attention")
        what = f"rope+attention batch {B}, {a.len} positions, {hq}/{hkv} heads of {hd}"
        nbytes = 2 * B * hkv * a.len * hd * 2
    else:
        qt = _TYPES[a.type]
        w = kq.Weight(ctx, qt, dec.gguf_weight_device(qt, a.rows, a.k, 5, dev), a.rows, a.k)
        x = torch.randn((1, a.k), generator=gen, device=dev)
        nw = 1.0 + 0.1 * torch.randn(a.k, generator=gen, device=dev)
        if a.op == "norm-swiglu":
            y = torch.empty((1, a.rows // 2), device=dev)

            def call():
                ctx.check(lib.kq_dec_norm_linear(ctx.handle, w.handle, _ptr(x), _ptr(nw), a.k, 1e-5, 0, None, _ptr(y),
                                                 0), "kq_dec_norm_linear")
            what = f"RMSNorm + {a.type} {a.rows}x{a.k} (gate, up) pairs + SwiGLU, one token"
        else:
            y = torch.empty((1, a.rows), device=dev)

            def call():
                w.linear(x, 1, y, device_ptrs=True)
            what = f"{a.type} {a.rows}x{a.k} GEMV, one token"
        nbytes = w.device_bytes

    with torch.cuda.stream(stream):
        for _ in range(3):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.calls):
            call()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.calls
    print(f"{what}: {us:.2f} us per call, {nbytes / us / 1e3:.0f} GB/s (same inputs each call)")
    ctx.set_stream(None)
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
