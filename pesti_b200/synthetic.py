"""Seeded synthetic K-quant weights and activations.

The reference publishes no dataset or model for this path; its benchmark
shapes are stand-ins for real GGUF tensors.  These generators reproduce those
shapes and value distributions from a seed (numpy ``default_rng``), one stream
per tensor:

* GGUF Q4_K (144 B / 256 weights): scale/min bytes (4..15) and quant bytes
  (16..143) uniform random; ``d`` and ``dmin`` are f16(|N(0, 0.02)|).
* GGUF Q6_K (210 B / 256 weights): ``ql``/``qh`` uniform random; the 16 int8
  sub-block scales uniform in [-32, 31]; ``d`` is f16(|N(0, 0.005)|).
* GGUF Q2_K (84 B), Q3_K (110 B) and Q5_K (176 B): every packed byte uniform
  random; the f16 fields (Q2_K / Q5_K d and dmin, Q3_K d) are f16(|N(0, 0.02)|).
* pesti-legacy blocks (28 B / 42 B per 16 weights, the layout that
  pesti-runner/src/tile_dequant.rs decodes): every byte the decoder reads is
  seeded; unused bytes are random too, so a decoder that reads them is caught.
  Legacy Q5_K rows are 36 B per 16 weights whose leading 28 B per 16 hold
  Q4_K tiles (what QuantizedLinear decodes them with).
"""
from __future__ import annotations

import numpy as np

QK_K = 256
Q4_K_BYTES = 144
Q6_K_BYTES = 210

GGUF_Q2_K = 10
GGUF_Q3_K = 11
GGUF_Q4_K = 12
GGUF_Q5_K = 13
GGUF_Q6_K = 14
PESTI_Q4_K_LEGACY = 112
PESTI_Q5_K_LEGACY = 113
PESTI_Q6_K_LEGACY = 114
#: bytes per superblock and the offsets of its f16 scale fields
_OTHER_K = {GGUF_Q2_K: (84, (80, 82)), GGUF_Q3_K: (110, (108,)), GGUF_Q5_K: (176, (0, 2))}


def _f16_abs_normal(rng, size, sigma):
    return np.abs(rng.normal(0.0, sigma, size)).astype(np.float16)


def q4_k_weight(n: int, k: int, seed: int = 0) -> np.ndarray:
    """Random GGUF Q4_K weight, uint8 [n, k/256*144] (row-major superblocks)."""
    if k % QK_K:
        raise ValueError("Q4_K rows must hold a whole number of 256-weight superblocks")
    rng = np.random.default_rng(seed)
    nb = n * (k // QK_K)
    blk = rng.integers(0, 256, size=(nb, Q4_K_BYTES), dtype=np.uint8)
    blk[:, 0:2] = _f16_abs_normal(rng, nb, 0.02).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = _f16_abs_normal(rng, nb, 0.02).view(np.uint8).reshape(nb, 2)
    return blk.reshape(n, -1)


def q6_k_weight(n: int, k: int, seed: int = 0) -> np.ndarray:
    """Random GGUF Q6_K weight, uint8 [n, k/256*210]."""
    if k % QK_K:
        raise ValueError("Q6_K rows must hold a whole number of 256-weight superblocks")
    rng = np.random.default_rng(seed)
    nb = n * (k // QK_K)
    blk = rng.integers(0, 256, size=(nb, Q6_K_BYTES), dtype=np.uint8)
    blk[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
    blk[:, 208:210] = _f16_abs_normal(rng, nb, 0.005).view(np.uint8).reshape(nb, 2)
    return blk.reshape(n, -1)


def other_k_weight(qtype: int, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Random GGUF Q2_K / Q3_K / Q5_K weight, uint8 [n, k/256*bytes]."""
    if k % QK_K:
        raise ValueError("K-quant rows must hold a whole number of 256-weight superblocks")
    bs, f16_at = _OTHER_K[qtype]
    rng = np.random.default_rng(seed)
    nb = n * (k // QK_K)
    blk = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    for off in f16_at:
        blk[:, off:off + 2] = _f16_abs_normal(rng, nb, 0.02).view(np.uint8).reshape(nb, 2)
    return blk.reshape(n, -1)


def gguf_weight(qtype: int, n: int, k: int, seed: int = 0) -> np.ndarray:
    if qtype == GGUF_Q4_K:
        return q4_k_weight(n, k, seed)
    if qtype == GGUF_Q6_K:
        return q6_k_weight(n, k, seed)
    if qtype in _OTHER_K:
        return other_k_weight(qtype, n, k, seed)
    raise ValueError(f"unsupported GGUF type {qtype}")


def legacy_row_bytes(qtype: int, k: int) -> int:
    """QuantizedLinear::row_bytes (pesti-runner/src/quantized_linear.rs:86-95)."""
    if qtype == PESTI_Q4_K_LEGACY:
        return ((k + 15) // 16) * 28
    if qtype == PESTI_Q5_K_LEGACY:
        return ((k + 15) // 16) * 36
    if qtype == PESTI_Q6_K_LEGACY:
        return ((k + 15) // 16) * 42
    raise ValueError(f"unsupported legacy type {qtype}")


def legacy_weight(qtype: int, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Random pesti-legacy weight, uint8 [n, row_bytes]: rows at the stride
    QuantizedLinear uses, each holding ceil(k/16) 28- or 42-byte blocks."""
    if qtype == PESTI_Q5_K_LEGACY:
        # Q4_K tiles packed at the start of each 36-byte-per-16 row, random slack after them
        rng = np.random.default_rng(seed + 1)
        nblk = (k + 15) // 16
        rows = rng.integers(0, 256, size=(n, legacy_row_bytes(qtype, k)), dtype=np.uint8)
        rows[:, :28 * nblk] = legacy_weight(PESTI_Q4_K_LEGACY, n, k, seed)
        return rows
    rng = np.random.default_rng(seed)
    rb = legacy_row_bytes(qtype, k)
    nblk = (k + 15) // 16
    bs = 28 if qtype == PESTI_Q4_K_LEGACY else 42
    data = rng.integers(0, 256, size=(n, nblk, bs), dtype=np.uint8)
    if qtype == PESTI_Q4_K_LEGACY:
        data[:, :, 0:2] = rng.normal(0.0, 0.02, (n, nblk)).astype(np.float16).view(np.uint8).reshape(n, nblk, 2)
        data[:, :, 2:4] = rng.normal(0.0, 0.1, (n, nblk)).astype(np.float16).view(np.uint8).reshape(n, nblk, 2)
        hs = rng.normal(0.0, 1.0, (n, nblk, 2)).astype(np.float16)
        data[:, :, 12:16] = hs.view(np.uint8).reshape(n, nblk, 4)
    else:
        data[:, :, 0:2] = np.abs(rng.normal(0.0, 0.01, (n, nblk))).astype(np.float16).view(np.uint8).reshape(n, nblk, 2)
        sc = rng.normal(0.0, 1.0, (n, nblk, 4)).astype(np.float16)
        data[:, :, 2:10] = sc.view(np.uint8).reshape(n, nblk, 8)
    return data.reshape(n, rb)


def activations(m: int, k: int, seed: int = 1, dtype=np.float32) -> np.ndarray:
    """x ~ N(0, 1), shape [m, k]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    return x.astype(dtype) if dtype is not np.float32 else x
