"""CPU restatement of pesti-runner's decode step -- test infrastructure only
(tests/ use it as the checker of pesti_b200.decoder; nothing ships it).

Follows, in numpy f32 (f64 for the long dot products):
  Model::embed                       transformer/model.rs:966-984
  RmsNorm::forward                   transformer/rms_norm.rs:24-43  (x / rms * w)
  RopeConfig::apply_single           transformer/rope.rs:36-77      (pairs i, i + hd/2;
                                                                     freq = base^(-i/half), angle = pos*freq, f32)
  LayerKvCache::append / k_head       transformer/kv_cache.rs:57-80  (kept in f16 here, as the device cache)
  Attention::forward_with_cache      transformer/layer.rs:169-244
  swiglu                             transformer/layer.rs:16-29     (mode 0 mirrors its negative-gate branch)
  TransformerLayer::forward_with_cache transformer/layer.rs:344-372
  forward_layers_with_cache + head    transformer/model.rs:1025-1061, 987-996
The linear layers use the GGUF-spec dequantization of oracle.gguf_dequant_rows.
Padded inputs: K-quant rows of width round_up(dim, 256) see zero activations
beyond dim, so only the first dim columns of each weight matter.
"""
import numpy as np

from . import gguf_dequant_rows, GGUF_Q4_K, GGUF_Q6_K

_TYPES = {12: GGUF_Q4_K, 14: GGUF_Q6_K}


def dequant(raw, qtype, n, k):
    return gguf_dequant_rows(_TYPES[qtype], np.ascontiguousarray(raw).reshape(-1), n, k).reshape(n, k)


def rmsnorm(x, w, eps):
    x = x.astype(np.float32)
    var = np.float32((x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True) / x.shape[-1])
    rms = np.sqrt(var + np.float32(eps)).astype(np.float32)
    return (x / rms * w).astype(np.float32)


def rope(x, heads, hd, pos, theta):
    """x [B][heads*hd] -> rotated copy."""
    half = hd // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.power(np.float32(theta), -i / np.float32(half)).astype(np.float32)
    angle = (np.float32(pos) * freq).astype(np.float32)
    c, s = np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)
    y = x.reshape(x.shape[0], heads, hd).astype(np.float32).copy()
    a, b = y[..., :half].copy(), y[..., half:].copy()
    y[..., :half] = a * c - b * s
    y[..., half:] = a * s + b * c
    return y.reshape(x.shape[0], heads * hd)


def swiglu(g, u, mode):
    g = g.astype(np.float32)
    with np.errstate(over="ignore"):  # both branches are evaluated; the unused one may overflow
        sig = np.where((g >= 0) | (mode == 1), 1.0 / (1.0 + np.exp(-g)), g / (1.0 + np.exp(g))).astype(np.float32)
    return (sig * g * u).astype(np.float32)


def attention(q, kc, vc, length, heads, kv_heads, hd):
    """softmax(q . k^T / sqrt(hd)) . v over positions [0, length) with grouped
    query heads (Attention::forward_with_cache, layer.rs:197-239).
    q [B][heads*hd]; kc, vc [B][kv_heads][max_seq][hd] -> [B][heads*hd]."""
    B = q.shape[0]
    group = heads // kv_heads
    out = np.zeros((B, heads * hd), np.float32)
    scale = 1.0 / np.sqrt(hd)
    for b in range(B):
        for hh in range(heads):
            g = hh // group
            qh = q[b, hh * hd:(hh + 1) * hd].astype(np.float64)
            scores = (kc[b, g, :length].astype(np.float64) @ qh) * scale
            e = np.exp(scores - scores.max())
            out[b, hh * hd:(hh + 1) * hd] = (e / e.sum()) @ vc[b, g, :length].astype(np.float64)
    return out


def decode_step(cfg, raw, tokens, pos, kcache, vcache, swiglu_mode=0):
    """One step for tokens [B] at position pos.  raw: the decoder's host
    copies of the full tensors; kcache / vcache: per layer f32 arrays
    [B][kv_heads][max_seq][hd] (modified: position pos is written).
    Returns logits [B][vocab]."""
    D, hd, F, V = cfg.dim, cfg.head_dim, cfg.ffn, cfg.vocab
    Dp = -(-D // 256) * 256
    Ap = -(-(cfg.heads * hd) // 256) * 256
    B = len(tokens)
    h = raw["embed"][np.asarray(tokens)].astype(np.float32)
    for li in range(cfg.layers):
        def W(name, qt, n, k, cols):
            return dequant(raw[(li, name)], qt, n, k)[:, :cols].astype(np.float64)
        a = rmsnorm(h, raw[(li, "attn_norm")], cfg.eps)
        q = (a @ W("q", cfg.linear_type, cfg.heads * hd, Dp, D).T).astype(np.float32)
        k = (a @ W("k", cfg.linear_type, cfg.kv_heads * hd, Dp, D).T).astype(np.float32)
        v = (a @ W("v", cfg.linear_type, cfg.kv_heads * hd, Dp, D).T).astype(np.float32)
        q = rope(q, cfg.heads, hd, pos, cfg.theta)
        k = rope(k, cfg.kv_heads, hd, pos, cfg.theta)
        kc, vc = kcache[li], vcache[li]
        kc[:, :, pos, :] = k.reshape(B, cfg.kv_heads, hd).astype(np.float16).astype(np.float32)
        vc[:, :, pos, :] = v.reshape(B, cfg.kv_heads, hd).astype(np.float16).astype(np.float32)
        attn = attention(q, kc, vc, pos + 1, cfg.heads, cfg.kv_heads, hd)
        o = (attn.astype(np.float64) @ W("o", cfg.linear_type, D, Ap, cfg.heads * hd).T).astype(np.float32)
        h = (h + o).astype(np.float32)
        a2 = rmsnorm(h, raw[(li, "ffn_norm")], cfg.eps)
        gt = (a2 @ W("gate", cfg.linear_type, F, Dp, D).T).astype(np.float32)
        up = (a2 @ W("up", cfg.linear_type, F, Dp, D).T).astype(np.float32)
        s = swiglu(gt, up, swiglu_mode)
        dn = (s.astype(np.float64) @ W("down", cfg.down_type, D, F, F).T).astype(np.float32)
        h = (h + dn).astype(np.float32)
    if cfg.final_norm:
        h = rmsnorm(h, raw["final_norm"], cfg.eps)
    head = dequant(raw["head"], cfg.head_type, V, Dp)[:, :D].astype(np.float64)
    return (h.astype(np.float64) @ head.T).astype(np.float32)
