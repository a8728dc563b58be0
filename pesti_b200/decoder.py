"""Decode step of a Llama-style decoder on the quantized linears.

The device form of pesti-runner's CPU decode step (transformer/model.rs:961-1075,
layer.rs:169-244,266-274,344-372): embedding lookup, per layer RMSNorm ->
Q/K/V projections -> rotary embedding + KV-cache append -> attention over the
cache -> output projection + residual -> RMSNorm -> gate/up projections ->
SwiGLU -> down projection + residual, then the optional final norm and the
output head.  Every projection is a GGUF K-quant weight resident in HBM and
runs through ``kq_linear_f32``; the small ops are the kernels of
``include/pesti_decoder.h``.  Activations are f32, the KV cache f16.

Tensor parallelism (``world > 1``, one process per GPU): heads are split across
ranks -- rank r owns query heads and KV heads [r*h/world, (r+1)*h/world), its
slice of the fused Q|K|V rows, its KV cache, a contiguous block of the head
rows and of the gate|up rows.  Up to 16 tokens (heads and FFN blocks on
superblock edges) the output and down projections are column-split -- rank r
holds the columns of its heads / FFN block -- and each one's partial residual
block is summed over the ranks into the residual (at one token inside the
GEMVs through exchange words, above it by ``kq_tp_allreduce_f32``): two
exchanges per layer.  Otherwise those projections are row-split and four
all-gathers per layer move activations over NVLink peer memory
(``kq_tp_allgather_f32``): the attention output, the output projection (added
into the residual), the SwiGLU output and the down projection (added into the
residual).  One more gathers the logits.

Weights are synthetic (no checkpoints): random GGUF superblocks generated on
the GPU from a seed per tensor, the same bytes on every rank, so a model
sharded over any number of GPUs computes the same function.
"""
from __future__ import annotations

import ctypes
import zlib
from dataclasses import dataclass
from typing import Optional

from . import kq

SWIGLU_REFERENCE = 0  # pesti's swiglu (layer.rs:16-29): negative gates use g / (1 + e^g)
SWIGLU_SILU = 1


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    layers: int
    dim: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float
    theta: float
    final_norm: bool
    linear_type: int = kq.KQ_GGUF_Q4_K
    down_type: int = kq.KQ_GGUF_Q6_K
    head_type: int = kq.KQ_GGUF_Q6_K


# Qwen2.5-0.5B-shaped: 896-wide activations are fed to K-quant rows as 1024
# (zero activations in the padded superblock).  Qwen models carry a final norm
# (model.rs:290-293).
QWEN25_05B = DecoderConfig("qwen2.5-0.5b-shaped", 24, 896, 14, 2, 64, 4864, 151936, 1e-6, 1e6, True)
# Llama-3-8B-shaped.  pesti's Llama path applies no final norm (model.rs:290-293).
LLAMA3_8B = DecoderConfig("llama-3-8b-shaped", 32, 4096, 32, 8, 128, 14336, 128256, 1e-5, 500000.0, False)


def round_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def _bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    P, I, I64, F, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    sig = {
        "kq_dec_rmsnorm": [P, P, I64, P, P, I64, I64, I64, F],
        "kq_dec_rope_append": [P, P, I64, P, P, I64, I, I, I, I64, I64, F],
        "kq_dec_attention": [P, P, I64, P, P, P, I64, I64, I, I, I, I64, I64, P, Z],
        "kq_dec_swiglu": [P, P, P, I64, I64, I],
        "kq_dec_add": [P, P, I64, P, I64, I64, I64],
        "kq_dec_embed": [P, P, P, P, I64, I64, I64],
        "kq_dec_norm_linear": [P, P, P, P, I64, F, I, P, P, I],
        "kq_dec_swiglu_linear": [P, P, P, I, P, P, I],
        "kq_dec_residual_linear": [P, P, P, P, I],
        "kq_dec_norm_linear_batch": [P, P, P, I64, I64, P, I64, F, P, I],
        "kq_dec_residual_linear_batch": [P, P, P, I64, P, I],
        "kq_dec_rope_attention": [P, P, I64, P, P, P, I64, I64, I, I, I, I64, I64, F, P, Z],
        "kq_dec_tp_partial_linear": [P, P, P, I, I],
        "kq_dec_tp_reduce_linear": [P, P, P, P, P, I64, F, I, P, I],
        "kq_step_linear": [P, P, I, P, P, I64, F, P, I, P, I],
        "kq_step_attention": [P, P, P, P, P, I, I, I, I64, F],
        "kq_step_run": [P, I64, I],
        "kq_step_trace": [P, P, Z],
        "kq_step_destroy": [P],
    }
    for name, args in sig.items():
        getattr(lib, name).argtypes = args
        getattr(lib, name).restype = I
    lib.kq_dec_attention_scratch.argtypes = [P, I64, I, I, I, I64]
    lib.kq_dec_attention_scratch.restype = Z
    lib.kq_step_create.argtypes = [P, P, ctypes.POINTER(P)]
    lib.kq_step_create.restype = I
    return lib


# kq_step_linear modes (include/pesti_decoder.h)
STEP_IN_PLAIN, STEP_IN_NORM, STEP_IN_RESIDUAL, STEP_IN_RESIDUAL_NORM = 0, 1, 2, 3
STEP_OUT_STORE, STEP_OUT_SWIGLU, STEP_OUT_PARTIAL = 0, 1, 2


def gguf_weight_device(qtype: int, n: int, k: int, seed: int, device):
    """Seeded random GGUF superblocks [n][k/256][bytes] as a uint8 CUDA tensor,
    with the distributions of pesti_b200.synthetic: Q4_K d, dmin = f16(|N(0,
    0.02)|); Q6_K int8 scales in [-32, 31], d = f16(|N(0, 0.005)|)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    sb = k // 256
    if qtype == kq.KQ_GGUF_Q4_K:
        raw = torch.randint(0, 256, (n, sb, 144), dtype=torch.uint8, device=device, generator=gen)
        dd = (torch.randn((n, sb, 2), generator=gen, device=device) * 0.02).abs().to(torch.float16)
        raw[:, :, 0:4] = dd.view(torch.uint8).view(n, sb, 4)
    elif qtype == kq.KQ_GGUF_Q6_K:
        raw = torch.randint(0, 256, (n, sb, 210), dtype=torch.uint8, device=device, generator=gen)
        sc = torch.randint(-32, 32, (n, sb, 16), dtype=torch.int8, device=device, generator=gen)
        raw[:, :, 192:208] = sc.view(torch.uint8)
        d = (torch.randn((n, sb, 1), generator=gen, device=device) * 0.005).abs().to(torch.float16)
        raw[:, :, 208:210] = d.view(torch.uint8).view(n, sb, 2)
    else:
        raise ValueError(f"type {qtype}")
    return raw.view(n, -1)


def exchange_elems(cfg: DecoderConfig, batch: int, world: int = 8) -> int:
    """Words one slot of the tensor-parallel exchange buffer needs for this
    model: the widest all-gathered activation (logits, SwiGLU output, residual
    stream) or one partial residual block per rank (the column split)."""
    return max(batch * max(cfg.vocab, cfg.ffn, cfg.dim, cfg.heads * cfg.head_dim), world * batch * cfg.dim)


def column_block(raw, k: int, c0: int, c1: int):
    """Columns [c0, c1) (multiples of 256) of a GGUF weight held as [n][k/256 *
    bytes]: the superblocks of that range in every row."""
    n = raw.shape[0]
    sb = k // 256
    return raw.view(n, sb, -1)[:, c0 // 256:c1 // 256].contiguous().view(n, -1)


class Decoder:
    """One model replica (or one rank of a tensor-parallel group) with its KV
    cache, able to run decode steps for `batch` sequences.  ``step`` queues one
    step on the context stream (capturable into a CUDA graph)."""

    def __init__(self, cfg: DecoderConfig, ctx: "kq.Context", batch: int, context_len: int, max_new: int = 8,
                 world: int = 1, rank: int = 0, tp: Optional["kq.TensorParallel"] = None, seed: int = 0,
                 swiglu_mode: int = SWIGLU_REFERENCE, kv_scale: float = 1.0, keep_raw: bool = False,
                 fused: bool = True, prefetch: bool = False, step_kernel: bool = False):
        import torch
        if cfg.heads % world or cfg.kv_heads % world:
            raise ValueError(f"{cfg.name}: {cfg.heads} query / {cfg.kv_heads} KV heads do not split over {world}")
        if world > 1 and tp is None:
            raise ValueError("world > 1 needs a TensorParallel group")
        self.cfg, self.ctx, self.batch, self.world, self.rank, self.tp = cfg, ctx, batch, world, rank, tp
        self.swiglu_mode = swiglu_mode
        # fused: RoPE + KV append + attention in one kernel, and at batch 1
        # RMSNorm, SwiGLU and the residual adds inside the single-token GEMVs;
        # prefetch: each linear pulls the next one's weight into L2
        self.fused_attention, self.fused, self.prefetch = fused, fused and batch == 1, prefetch
        # batch > 1: RMSNorm inside the integer-MMA linears' activation
        # preparation and the residual adds in their epilogue, where that
        # kernel serves the weight at this batch (the calls report
        # unsupported otherwise and the separate kernels run)
        self.fuse_batch = fused and batch > 1
        # column split (batch 1, tensor parallel): the output and down
        # projections hold W[:, this rank's heads / FFN block] and exchange
        # partial residual vectors (2 exchanges per layer) instead of
        # all-gathering row blocks (4); needs both blocks on superblock edges
        aligned = (cfg.heads // world * cfg.head_dim) % 256 == 0 and cfg.ffn % (256 * world) == 0
        self.col_split = world > 1 and self.fused and aligned
        # the same column split at 2..16 tokens: each projection's partial
        # residual block [batch][dim] is all-reduced into the residual
        # (kq_tp_allreduce_f32), 2 exchanges per layer instead of 4 all-gathers
        # (above 16 tokens the all-gathers move fewer bytes)
        self.col_batch = world > 1 and self.fuse_batch and aligned and batch <= 16
        # gate/up as (gate, up) row pairs with the SwiGLU in the GEMV epilogue: the
        # paths that run it (one GPU or the column split at batch 1); otherwise
        # [gate block | up block] for the separate SwiGLU kernel
        self.pairs = self.fused and (world == 1 or self.col_split)
        # batch 1, opt-in: the whole step as one persistent kernel (kq_step_*),
        # on one GPU or with the column split; otherwise one kernel per
        # operation (measured faster: the per-operation kernels overlap each
        # launch's start-up with the previous kernel's tail)
        self.step_kernel = step_kernel and self.fused and (world == 1 or self.col_split)
        self._step = None
        self.lib = _bind(ctx.lib)
        dev = torch.device("cuda", ctx.device)
        self.device = dev
        D, hd, F = cfg.dim, cfg.head_dim, cfg.ffn
        self.Dp = round_up(D, 256)                 # K of projections fed by the residual stream
        self.Ap = round_up(cfg.heads * hd, 256)    # K of the output projection
        self.hq, self.hkv = cfg.heads // world, cfg.kv_heads // world
        self.max_seq = context_len + max_new
        self.context_len = context_len
        B = batch

        def slot(i, name):  # one seed per tensor, the same in every process
            return (seed * 1000003 + i * 1009 + zlib.crc32(name.encode())) % (1 << 62)

        # keep_raw: host copies of the full tensors (small test models only)
        self.raw = {} if keep_raw else None

        def keep(key, t):
            if self.raw is not None:
                self.raw[key] = t.cpu().numpy()

        def upload(raw, qtype, n, k):
            return kq.Weight(ctx, qtype, raw, n, k)

        hq0, hkv0 = self.hq * rank, self.hkv * rank
        self.o_rows = kq.shard_rows(D, world, rank)
        self.f_rows = kq.shard_rows(F, world, rank)
        self.v_rows = kq.shard_rows(cfg.vocab, world, rank)
        self.layers = []
        for li in range(cfg.layers):
            L = {}
            wq = gguf_weight_device(cfg.linear_type, cfg.heads * hd, self.Dp, slot(li, "q"), dev)
            wk = gguf_weight_device(cfg.linear_type, cfg.kv_heads * hd, self.Dp, slot(li, "k"), dev)
            wv = gguf_weight_device(cfg.linear_type, cfg.kv_heads * hd, self.Dp, slot(li, "v"), dev)
            keep((li, "q"), wq)
            keep((li, "k"), wk)
            keep((li, "v"), wv)
            qkv = torch.cat([wq[hq0 * hd:(hq0 + self.hq) * hd], wk[hkv0 * hd:(hkv0 + self.hkv) * hd],
                             wv[hkv0 * hd:(hkv0 + self.hkv) * hd]]).contiguous()
            L["qkv"] = upload(qkv, cfg.linear_type, qkv.shape[0], self.Dp)
            del wq, wk, wv, qkv
            wo = gguf_weight_device(cfg.linear_type, D, self.Ap, slot(li, "o"), dev)
            keep((li, "o"), wo)
            r0, r1 = self.o_rows
            if self.col_split or self.col_batch:
                a0, a1 = hq0 * hd, (hq0 + self.hq) * hd
                L["o"] = upload(column_block(wo, self.Ap, a0, a1), cfg.linear_type, D, a1 - a0)
            else:
                L["o"] = upload(wo[r0:r1].contiguous(), cfg.linear_type, r1 - r0, self.Ap)
            wg = gguf_weight_device(cfg.linear_type, F, self.Dp, slot(li, "gate"), dev)
            wu = gguf_weight_device(cfg.linear_type, F, self.Dp, slot(li, "up"), dev)
            keep((li, "gate"), wg)
            keep((li, "up"), wu)
            f0, f1 = self.f_rows
            if self.pairs:  # (gate, up) row pairs: the GEMV applies the SwiGLU itself
                gu = torch.stack([wg[f0:f1], wu[f0:f1]], dim=1).reshape(2 * (f1 - f0), -1).contiguous()
            else:
                gu = torch.cat([wg[f0:f1], wu[f0:f1]]).contiguous()
            L["gu"] = upload(gu, cfg.linear_type, 2 * (f1 - f0), self.Dp)
            del wg, wu, gu
            wd = gguf_weight_device(cfg.down_type, D, F, slot(li, "down"), dev)
            keep((li, "down"), wd)
            if self.col_split or self.col_batch:
                L["down"] = upload(column_block(wd, F, f0, f1), cfg.down_type, D, f1 - f0)
            else:
                L["down"] = upload(wd[r0:r1].contiguous(), cfg.down_type, r1 - r0, F)
            del wd
            g = torch.Generator(device=dev)
            g.manual_seed(slot(li, "norms"))
            L["attn_norm"] = 1.0 + 0.1 * torch.randn(D, generator=g, device=dev)
            L["ffn_norm"] = 1.0 + 0.1 * torch.randn(D, generator=g, device=dev)
            keep((li, "attn_norm"), L["attn_norm"])
            keep((li, "ffn_norm"), L["ffn_norm"])
            # KV cache: this rank's heads, a random N(0, kv_scale) prefix of context_len positions
            kvshape = (B, cfg.kv_heads, self.max_seq, hd)
            g.manual_seed(slot(li, "kv"))
            kc = (kv_scale * torch.randn(kvshape, generator=g, device=dev)).to(torch.float16)
            vc = (kv_scale * torch.randn(kvshape, generator=g, device=dev)).to(torch.float16)
            L["k"] = kc[:, hkv0:hkv0 + self.hkv].contiguous()
            L["v"] = vc[:, hkv0:hkv0 + self.hkv].contiguous()
            keep((li, "kcache"), kc)
            keep((li, "vcache"), vc)
            del kc, vc
            self.layers.append(L)
        wh = gguf_weight_device(cfg.head_type, cfg.vocab, self.Dp, slot(cfg.layers, "head"), dev)
        keep("head", wh)
        v0, v1 = self.v_rows
        self.head = upload(wh[v0:v1].contiguous(), cfg.head_type, v1 - v0, self.Dp)
        del wh
        g = torch.Generator(device=dev)
        g.manual_seed(slot(cfg.layers, "embed"))
        self.embed = 0.5 * torch.randn((cfg.vocab, D), generator=g, device=dev)
        self.final_norm = 1.0 + 0.1 * torch.randn(D, generator=g, device=dev) if cfg.final_norm else None
        keep("embed", self.embed)
        if self.final_norm is not None:
            keep("final_norm", self.final_norm)

        # activations (padded columns stay zero)
        z = lambda *s: torch.zeros(s, device=dev)  # noqa: E731
        self.h, self.a = z(B, self.Dp), z(B, self.Dp)
        self.h2 = z(B, self.Dp) if self.col_split else None  # the other residual buffer
        self.qkv_ld = (self.hq + 2 * self.hkv) * hd
        self.qkv = z(B, self.qkv_ld)
        self.attn = z(B, self.Ap)
        self.attn_r = z(B, self.hq * hd)
        self.o = z(B, r1 - r0)
        self.gu = z(B, 2 * (f1 - f0))
        self.s_r = z(B, f1 - f0)
        self.s = z(B, F)
        self.dn = z(B, r1 - r0)
        self.logits_r = z(B, v1 - v0)
        self.logits = z(B, cfg.vocab)
        self.part = z(B, D) if self.col_batch else None  # this rank's partial residual block
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        sbytes = self.lib.kq_dec_attention_scratch(ctx.handle, B, self.hq, self.hkv, hd, self.max_seq)
        self.att_scratch = torch.zeros(max(sbytes // 4, 1), device=dev)  # counters start at zero
        self.att_scratch_bytes = sbytes
        for L in self.layers:
            for key in ("qkv", "o", "gu", "down"):
                ctx.reserve(L[key], B)
        ctx.reserve(self.head, B)
        # the weights in the order a step reads them; _next[id] is the one after
        order = [L[key] for L in self.layers for key in ("qkv", "o", "gu", "down")] + [self.head]
        self._next = {id(a): b for a, b in zip(order, order[1:] + [None])}
        torch.cuda.synchronize(dev)

    # ---- one decode step ------------------------------------------------------------
    def _check(self, rc, what):
        self.ctx.check(rc, what)

    def _gather(self, src, cols, row0, rows, dst, ld, accumulate):
        self.tp.allgather(src, self.batch, row0, rows, cols, dst, y_ld=ld, accumulate=accumulate)

    def _hint(self, w) -> None:
        """Tell the next linear call on the context which weight follows `w`."""
        if self.prefetch:
            self.ctx.prefetch_next(self._next[id(w)])

    def _norm_linear(self, w, norm, y, act: int = -1) -> None:
        """y = rmsnorm(h; norm) . W^T (token 0 only when fused; act >= 0: SwiGLU
        of (gate, up) row pairs)."""
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        c, cfg = self.ctx.handle, self.cfg
        self._hint(w)
        if self.fused:
            self._check(self.lib.kq_dec_norm_linear(c, w.handle, ptr(self.h), ptr(norm), cfg.dim, cfg.eps, act, None,
                                                    ptr(y), 0), "norm_linear")
            return
        if self.fuse_batch:
            rc = self.lib.kq_dec_norm_linear_batch(c, w.handle, ptr(self.h), self.Dp, self.batch, ptr(norm), cfg.dim,
                                                   cfg.eps, ptr(y), 0)
            if rc != kq.KQ_ERR_UNSUPPORTED:
                self._check(rc, "norm_linear_batch")
                return
        self._check(self.lib.kq_dec_rmsnorm(c, ptr(self.h), self.Dp, ptr(norm), ptr(self.a), self.Dp, self.batch,
                                            cfg.dim, cfg.eps), "rmsnorm")
        w.linear(self.a, self.batch, y, device_ptrs=True)

    def _residual_batch(self, w, x) -> bool:
        """h += x . W^T in the linear's epilogue (batch > 1, one GPU, residual
        rows not padded); False when the caller must queue linear + add."""
        if not self.fuse_batch or self.world > 1 or self.Dp != self.cfg.dim:
            return False
        rc = self.lib.kq_dec_residual_linear_batch(self.ctx.handle, w.handle, ctypes.c_void_p(x.data_ptr()),
                                                   self.batch, ctypes.c_void_p(self.h.data_ptr()), 0)
        if rc == kq.KQ_ERR_UNSUPPORTED:
            return False
        self._check(rc, "residual_linear_batch")
        return True

    def step(self, pos: int) -> None:
        """Queue one decode step for the tokens in ``self.tokens`` at position
        ``pos`` (the cache holds positions [0, pos)); logits land in
        ``self.logits``."""
        cfg, lib, c, B = self.cfg, self.lib, self.ctx.handle, self.batch
        D, hd, F = cfg.dim, cfg.head_dim, cfg.ffn
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        if not 0 <= pos < self.max_seq:
            raise ValueError(f"position {pos} outside the cache ({self.max_seq})")
        if self.step_kernel:
            self._step_persistent(pos)
            return
        if self.col_split:
            self._step_col_split(pos)
            return
        r0, r1 = self.o_rows
        f0, f1 = self.f_rows
        tp = self.world > 1
        self._check(lib.kq_dec_embed(c, ptr(self.embed), ptr(self.tokens), ptr(self.h), self.Dp, B, D), "embed")
        for L in self.layers:
            self._norm_linear(L["qkv"], L["attn_norm"], self.qkv)
            out, out_ld = (self.attn_r, self.hq * hd) if tp else (self.attn, self.Ap)
            if self.fused_attention:
                self._check(lib.kq_dec_rope_attention(c, ptr(self.qkv), self.qkv_ld, ptr(L["k"]), ptr(L["v"]),
                                                      ptr(out), out_ld, B, self.hq, self.hkv, hd, pos, self.max_seq,
                                                      cfg.theta, ptr(self.att_scratch), self.att_scratch_bytes),
                            "rope_attention")
            else:
                self._check(lib.kq_dec_rope_append(c, ptr(self.qkv), self.qkv_ld, ptr(L["k"]), ptr(L["v"]), B,
                                                   self.hq, self.hkv, hd, pos, self.max_seq, cfg.theta), "rope")
                self._check(lib.kq_dec_attention(c, ptr(self.qkv), self.qkv_ld, ptr(L["k"]), ptr(L["v"]), ptr(out),
                                                 out_ld, B, self.hq, self.hkv, hd, pos + 1, self.max_seq,
                                                 ptr(self.att_scratch), self.att_scratch_bytes), "attention")
            if tp and not self.col_batch:
                self._gather(self.attn_r, cfg.heads * hd, self.rank * self.hq * hd, self.hq * hd, self.attn, self.Ap,
                             False)
            self._hint(L["o"])
            if self.col_batch:  # W_o[:, this rank's heads] . attn_r, summed over the ranks into h
                L["o"].linear(self.attn_r, B, self.part, device_ptrs=True)
                self.tp.allreduce(self.part, B, D, self.h, y_ld=self.Dp, accumulate=True)
            elif tp:
                L["o"].linear(self.attn, B, self.o, device_ptrs=True)
                self._gather(self.o, D, r0, r1 - r0, self.h, self.Dp, True)
            elif self.fused:
                self._check(lib.kq_dec_residual_linear(c, L["o"].handle, ptr(self.attn), ptr(self.h), 0), "o")
            elif not self._residual_batch(L["o"], self.attn):
                L["o"].linear(self.attn, B, self.o, device_ptrs=True)
                self._check(lib.kq_dec_add(c, ptr(self.h), self.Dp, ptr(self.o), D, B, D), "add")
            if self.fused and not tp:
                # gate/up pairs + SwiGLU in one GEMV, then the down projection's residual update
                self._norm_linear(L["gu"], L["ffn_norm"], self.s, act=self.swiglu_mode)
                self._hint(L["down"])
                self._check(lib.kq_dec_residual_linear(c, L["down"].handle, ptr(self.s), ptr(self.h), 0), "down")
                continue
            self._norm_linear(L["gu"], L["ffn_norm"], self.gu)
            self._hint(L["down"])
            self._check(lib.kq_dec_swiglu(c, ptr(self.gu), ptr(self.s_r if tp else self.s), B, f1 - f0,
                                          self.swiglu_mode), "swiglu")
            if self.col_batch:  # W_down[:, this rank's FFN block] . s_r, summed over the ranks into h
                L["down"].linear(self.s_r, B, self.part, device_ptrs=True)
                self.tp.allreduce(self.part, B, D, self.h, y_ld=self.Dp, accumulate=True)
            elif tp:
                self._gather(self.s_r, F, f0, f1 - f0, self.s, F, False)
                L["down"].linear(self.s, B, self.dn, device_ptrs=True)
                self._gather(self.dn, D, r0, r1 - r0, self.h, self.Dp, True)
            elif not self._residual_batch(L["down"], self.s):
                L["down"].linear(self.s, B, self.dn, device_ptrs=True)
                self._check(lib.kq_dec_add(c, ptr(self.h), self.Dp, ptr(self.dn), D, B, D), "add")
        v0, v1 = self.v_rows
        logits = self.logits_r if tp else self.logits
        if self.final_norm is not None:
            self._norm_linear(self.head, self.final_norm, logits)
        else:
            self._hint(self.head)
            self.head.linear(self.h, B, logits, device_ptrs=True)
        if tp:
            self._gather(self.logits_r, cfg.vocab, v0, v1 - v0, self.logits, cfg.vocab, False)

    def _step_col_split(self, pos: int) -> None:
        """Batch-1 tensor-parallel step with column-split output / down
        projections: per layer two exchanges of partial residual vectors, each
        sent from inside the producing GEMV and summed (with the residual and
        the next RMSNorm) inside the consuming GEMV's activation staging."""
        cfg, lib, c = self.cfg, self.lib, self.ctx.handle
        D, hd = cfg.dim, cfg.head_dim
        tph = self.tp.handle
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        cur, nxt = self.h, self.h2
        self._check(lib.kq_dec_embed(c, ptr(self.embed), ptr(self.tokens), ptr(cur), self.Dp, 1, D), "embed")
        pending = False  # an exchange of partials waits to be added to `cur`

        def reduce_linear(w, norm, y, act=-1):
            nonlocal cur, nxt
            self._hint(w)
            if not pending:
                self._check(lib.kq_dec_norm_linear(c, w.handle, ptr(cur), ptr(norm), D, cfg.eps, act, None, ptr(y),
                                                   0), "norm_linear")
                return
            self._check(lib.kq_dec_tp_reduce_linear(tph, w.handle, ptr(cur), ptr(nxt),
                                                    ptr(norm) if norm is not None else None, D, cfg.eps, act, ptr(y),
                                                    0), "tp_reduce_linear")
            cur, nxt = nxt, cur

        for L in self.layers:
            reduce_linear(L["qkv"], L["attn_norm"], self.qkv)
            self._check(lib.kq_dec_rope_attention(c, ptr(self.qkv), self.qkv_ld, ptr(L["k"]), ptr(L["v"]),
                                                  ptr(self.attn_r), self.hq * hd, 1, self.hq, self.hkv, hd, pos,
                                                  self.max_seq, cfg.theta, ptr(self.att_scratch),
                                                  self.att_scratch_bytes), "rope_attention")
            self._hint(L["o"])
            self._check(lib.kq_dec_tp_partial_linear(tph, L["o"].handle, ptr(self.attn_r), -1, 0), "o partial")
            pending = True
            reduce_linear(L["gu"], L["ffn_norm"], self.s_r, act=self.swiglu_mode)
            self._hint(L["down"])
            self._check(lib.kq_dec_tp_partial_linear(tph, L["down"].handle, ptr(self.s_r), -1, 0), "down partial")
            pending = True
        v0, v1 = self.v_rows
        self._hint(self.head)
        if self.final_norm is not None or pending:
            reduce_linear(self.head, self.final_norm, self.logits_r)
        else:
            self.head.linear(cur, 1, self.logits_r, device_ptrs=True)
        self._gather(self.logits_r, cfg.vocab, v0, v1 - v0, self.logits, cfg.vocab, False)

    def _build_step(self) -> None:
        """The step program of the persistent kernel (kq_step_*): per layer
        RMSNorm + q|k|v, attention, the output projection as a partial residual
        update, residual + RMSNorm + gate/up + SwiGLU, the down projection as a
        partial; then the residual, the final norm and the head.  On one GPU the
        output and down projections are whole weights whose 'partial' is the full
        update; with the column split each rank holds W[:, its heads / FFN block]."""
        import torch
        cfg, lib = self.cfg, self.lib
        D, hd = cfg.dim, cfg.head_dim
        ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        h = ctypes.c_void_p()
        self.ctx.check(lib.kq_step_create(self.ctx.handle, self.tp.handle if self.tp is not None else None,
                                          ctypes.byref(h)), "kq_step_create")
        self._step = h
        if self.h2 is None:
            self.h2 = torch.zeros_like(self.h)
        # the residual alternates between two buffers: a RESIDUAL stage writes the
        # new residual to the other one, the next PARTIAL stage updates it
        cur, nxt = self.h, self.h2
        pending = False
        c = lambda rc, what: self.ctx.check(rc, what)  # noqa: E731
        for L in self.layers:
            if pending:
                c(lib.kq_step_linear(h, L["qkv"].handle, STEP_IN_RESIDUAL_NORM, None, ptr(L["attn_norm"]), D,
                                     cfg.eps, ptr(nxt), STEP_OUT_STORE, ptr(self.qkv), 0), "step qkv")
                cur, nxt = nxt, cur
            else:
                c(lib.kq_step_linear(h, L["qkv"].handle, STEP_IN_NORM, ptr(cur), ptr(L["attn_norm"]), D, cfg.eps,
                                     None, STEP_OUT_STORE, ptr(self.qkv), 0), "step qkv")
            out = self.attn_r if self.col_split else self.attn
            c(lib.kq_step_attention(h, ptr(self.qkv), ptr(L["k"]), ptr(L["v"]), ptr(out), self.hq, self.hkv, hd,
                                    self.max_seq, cfg.theta), "step attention")
            c(lib.kq_step_linear(h, L["o"].handle, STEP_IN_PLAIN, ptr(out), None, 0, 0.0, ptr(cur), STEP_OUT_PARTIAL,
                                 None, 0), "step o")
            c(lib.kq_step_linear(h, L["gu"].handle, STEP_IN_RESIDUAL_NORM, None, ptr(L["ffn_norm"]), D, cfg.eps,
                                 ptr(nxt), STEP_OUT_SWIGLU, ptr(self.s_r if self.col_split else self.s),
                                 self.swiglu_mode), "step gate/up")
            cur, nxt = nxt, cur
            c(lib.kq_step_linear(h, L["down"].handle, STEP_IN_PLAIN, ptr(self.s_r if self.col_split else self.s),
                                 None, 0, 0.0, ptr(cur), STEP_OUT_PARTIAL, None, 0), "step down")
            pending = True
        logits = self.logits_r if self.world > 1 else self.logits
        mode = STEP_IN_RESIDUAL_NORM if self.final_norm is not None else STEP_IN_RESIDUAL
        c(lib.kq_step_linear(h, self.head.handle, mode, None, ptr(self.final_norm), D, cfg.eps, ptr(nxt),
                             STEP_OUT_STORE, ptr(logits), 0), "step head")
        self._step_in = self.h  # the embedding goes here; the residual ends in `nxt`

    def _step_persistent(self, pos: int) -> None:
        """Batch-1 step: embedding lookup, the persistent step kernel, and (tensor
        parallel) the all-gather of the logits slices."""
        cfg, lib, c = self.cfg, self.lib, self.ctx.handle
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        if self._step is None:
            self._build_step()
        self._check(lib.kq_dec_embed(c, ptr(self.embed), ptr(self.tokens), ptr(self._step_in), self.Dp, 1, cfg.dim),
                    "embed")
        self._check(lib.kq_step_run(self._step, pos, 0), "kq_step_run")
        if self.world > 1:
            v0, v1 = self.v_rows
            self._gather(self.logits_r, cfg.vocab, v0, v1 - v0, self.logits, cfg.vocab, False)

    def weight_bytes(self) -> int:
        """HBM bytes of this rank's quantized weights."""
        total = self.head.device_bytes
        for L in self.layers:
            total += sum(L[key].device_bytes for key in ("qkv", "o", "gu", "down"))
        return total

    def kv_bytes(self, pos: int) -> int:
        """KV-cache bytes one step at `pos` reads on this rank."""
        return self.cfg.layers * 2 * self.batch * self.hkv * (pos + 1) * self.cfg.head_dim * 2

    def close(self) -> None:
        if self._step is not None:
            self.lib.kq_step_destroy(self._step)
            self._step = None
        for L in self.layers:
            for key in ("qkv", "o", "gu", "down"):
                L[key].free()
        self.head.free()
        self.layers = []
