"""Generate the GGUF K-quant golden fixtures from gguf-py.

The reference has no GGUF-correct Q4_K/Q6_K decoder of its own (its
tile_dequant.rs decodes an invented 16-element layout); the format's arithmetic
lives in llama.cpp, which the reference links through llama-cpp-sys-2 0.1.146
and does not vendor.  gguf-py 0.19.0 (installed in the build image) implements
the same published format in numpy; this script uses it as the independent
source of expected values and writes small fixtures that travel with the repo:

  tests/golden/gguf_kquant_golden.npz
    q4k_raw  uint8 [n, 144]   superblocks (edge cases first, then random)
    q4k_bits uint32 [n, 256]  gguf-py dequantized values as f32 bit patterns
    q6k_raw  uint8 [n, 210]
    q6k_bits uint32 [n, 256]
    lin_*    a small Q4_K and Q6_K linear: raw weight, x, and y computed in f64
             from the gguf-py dequantized weight
  tests/golden/gguf_kquant_more_golden.npz
    the same for Q2_K (84 B), Q3_K (110 B) and Q5_K (176 B): q2k_raw /
    q2k_bits, q3k_*, q5k_*, and lin_q2k_*, lin_q3k_*, lin_q5k_*

It also cross-checks the C oracle (oracle/kq_oracle.c) against gguf-py on
1,000,000 random superblocks of each of the five types and refuses to write
fixtures if a single bit differs.

Run from the repo root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import gguf  # noqa: E402
from gguf import GGMLQuantizationType as QT  # noqa: E402

import oracle  # noqa: E402

F16_SPECIALS = np.array([
    0x0000, 0x8000,          # +-0
    0x0001, 0x03FF,          # smallest / largest subnormal
    0x0400, 0x3C00, 0xBC00,  # smallest normal, +-1
    0x7BFF, 0xFBFF,          # +-max finite
    0x7C00, 0xFC00,          # +-inf
    0x7E00,                  # nan
    0x2E66, 0x1400,          # 0.1, 2^-10
], dtype=np.uint16)


def _edge_q4k(rng):
    rows = []
    for d in F16_SPECIALS:
        for dmin in (0x0000, 0x3C00, int(d), 0x7BFF):
            for pattern in ("zeros", "ones", "random"):
                b = np.zeros(144, np.uint8)
                b[0:2] = np.array([d], np.uint16).view(np.uint8)
                b[2:4] = np.array([dmin], np.uint16).view(np.uint8)
                if pattern == "ones":
                    b[4:] = 0xFF
                elif pattern == "random":
                    b[4:] = rng.integers(0, 256, 140, dtype=np.uint8)
                rows.append(b)
    return np.stack(rows)


def _edge_q6k(rng):
    rows = []
    for d in F16_SPECIALS:
        for sc in ("min", "max", "zero", "random"):
            for pattern in ("zeros", "ones", "random"):
                b = np.zeros(210, np.uint8)
                if pattern == "ones":
                    b[0:192] = 0xFF
                elif pattern == "random":
                    b[0:192] = rng.integers(0, 256, 192, dtype=np.uint8)
                s = {"min": np.full(16, -128, np.int8), "max": np.full(16, 127, np.int8),
                     "zero": np.zeros(16, np.int8),
                     "random": rng.integers(-128, 128, 16, dtype=np.int8)}[sc]
                b[192:208] = s.view(np.uint8)
                b[208:210] = np.array([d], np.uint16).view(np.uint8)
                rows.append(b)
    return np.stack(rows)


# (block bytes, offset of d, offset of dmin or None) of the other K-quants
_MORE = {"q2k": (QT.Q2_K, 84, 80, 82, oracle.GGUF_Q2_K), "q3k": (QT.Q3_K, 110, 108, None, oracle.GGUF_Q3_K),
         "q5k": (QT.Q5_K, 176, 0, 2, oracle.GGUF_Q5_K)}


def _edge_generic(rng, bs, d_off, dmin_off):
    """Every special f16 as d (and a few dmin values), with all-zero, all-one
    and random payload bytes."""
    rows = []
    for d in F16_SPECIALS:
        for dmin in ((0x0000, 0x3C00, int(d), 0x7BFF) if dmin_off is not None else (None,)):
            for pattern in ("zeros", "ones", "random"):
                b = np.zeros(bs, np.uint8)
                if pattern == "ones":
                    b[:] = 0xFF
                elif pattern == "random":
                    b[:] = rng.integers(0, 256, bs, dtype=np.uint8)
                b[d_off:d_off + 2] = np.array([d], np.uint16).view(np.uint8)
                if dmin_off is not None:
                    b[dmin_off:dmin_off + 2] = np.array([dmin], np.uint16).view(np.uint8)
                rows.append(b)
    return np.stack(rows)


def _ref_dequant(raw, qt):
    with np.errstate(all="ignore"):
        return gguf.quants.dequantize(raw, qt).reshape(raw.shape[0], 256).astype(np.float32)


def _same_bits(a, b):
    ab, bb = a.view(np.uint32), b.view(np.uint32)
    both_nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((ab == bb) | both_nan))


def cross_check(n_blocks=1_000_000, chunk=100_000, seed=1234):
    rng = np.random.default_rng(seed)
    # (name, type, block bytes, oracle type, high bytes of the f16 fields)
    for name, qt, bs, otype, f16_hi in (("Q4_K", QT.Q4_K, 144, oracle.GGUF_Q4_K, (1, 3)),
                                        ("Q6_K", QT.Q6_K, 210, oracle.GGUF_Q6_K, (209,)),
                                        ("Q2_K", QT.Q2_K, 84, oracle.GGUF_Q2_K, (81, 83)),
                                        ("Q3_K", QT.Q3_K, 110, oracle.GGUF_Q3_K, (109,)),
                                        ("Q5_K", QT.Q5_K, 176, oracle.GGUF_Q5_K, (1, 3))):
        done = 0
        while done < n_blocks:
            raw = rng.integers(0, 256, (chunk, bs), dtype=np.uint8)
            # keep the f16 scales finite so the sweep exercises arithmetic, not
            # nan propagation (the edge-case fixture covers specials)
            for hb in f16_hi:
                raw[:, hb] &= 0x7B
            want = _ref_dequant(raw, qt)
            got = oracle.dequant_blocks(otype, raw).reshape(chunk, 256)
            if not _same_bits(got, want):
                bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))[0]
                raise SystemExit(f"{name}: oracle differs from gguf-py at block {done + bad[0]} elem {bad[1]}")
            done += chunk
        print(f"{name}: C oracle == gguf-py bit-for-bit on {done} random superblocks")


def main():
    cross_check()
    rng = np.random.default_rng(20261201)
    q4 = np.concatenate([_edge_q4k(rng), rng.integers(0, 256, (256, 144), dtype=np.uint8)])
    q6 = np.concatenate([_edge_q6k(rng), rng.integers(0, 256, (256, 210), dtype=np.uint8)])
    q4_vals = _ref_dequant(q4, QT.Q4_K)
    q6_vals = _ref_dequant(q6, QT.Q6_K)
    assert _same_bits(oracle.dequant_blocks(oracle.GGUF_Q4_K, q4).reshape(-1, 256), q4_vals)
    assert _same_bits(oracle.dequant_blocks(oracle.GGUF_Q6_K, q6).reshape(-1, 256), q6_vals)

    # small linears: y computed in f64 from gguf-py's dequantized weight
    from pesti_b200 import synthetic
    lin = {}
    for tag, qt, qtype, n, k in (("q4k", QT.Q4_K, synthetic.GGUF_Q4_K, 48, 768),
                                 ("q6k", QT.Q6_K, synthetic.GGUF_Q6_K, 40, 512)):
        w = synthetic.gguf_weight(qtype, n, k, seed=7)
        x = synthetic.activations(3, k, seed=8)
        wf = gguf.quants.dequantize(w, qt).reshape(n, k).astype(np.float64)
        lin[f"lin_{tag}_w"] = w
        lin[f"lin_{tag}_x"] = x
        lin[f"lin_{tag}_y64"] = x.astype(np.float64) @ wf.T
    out = os.path.join(HERE, "gguf_kquant_golden.npz")
    np.savez_compressed(out, q4k_raw=q4, q4k_bits=q4_vals.view(np.uint32),
                        q6k_raw=q6, q6k_bits=q6_vals.view(np.uint32),
                        gguf_py_version=np.array(["0.19.0"]), **lin)
    print(f"wrote {out}: {q4.shape[0]} Q4_K and {q6.shape[0]} Q6_K superblocks")

    # Q2_K, Q3_K and Q5_K: edge cases and random superblocks, and a small linear each
    rng = np.random.default_rng(20261202)
    more = {}
    for tag, (qt, bs, d_off, dmin_off, otype) in _MORE.items():
        raw = np.concatenate([_edge_generic(rng, bs, d_off, dmin_off),
                              rng.integers(0, 256, (128, bs), dtype=np.uint8)])
        vals = _ref_dequant(raw, qt)
        assert _same_bits(oracle.dequant_blocks(otype, raw).reshape(-1, 256), vals)
        more[f"{tag}_raw"] = raw
        more[f"{tag}_bits"] = vals.view(np.uint32)
        n, k = 24, 512
        w = synthetic.gguf_weight(otype, n, k, seed=9)
        x = synthetic.activations(3, k, seed=10)
        wf = gguf.quants.dequantize(w, qt).reshape(n, k).astype(np.float64)
        more[f"lin_{tag}_w"] = w
        more[f"lin_{tag}_x"] = x
        more[f"lin_{tag}_y64"] = x.astype(np.float64) @ wf.T
    out = os.path.join(HERE, "gguf_kquant_more_golden.npz")
    np.savez_compressed(out, gguf_py_version=np.array(["0.19.0"]), **more)
    print(f"wrote {out}: " + ", ".join(f"{more[t + '_raw'].shape[0]} {t}" for t in _MORE))


if __name__ == "__main__":
    main()
