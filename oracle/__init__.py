"""CPU oracle for the K-quant linear path -- TEST INFRASTRUCTURE ONLY.

This package is the checker: tests, the smoke check and the CPU-baseline leg of
bench.py call it to produce expected values.  The product (pesti_b200) never
imports it.

Two restatements are exposed (both compiled from oracle/kq_oracle.c):

* O1 "GGUF-spec" -- GGUF Q4_K / Q6_K superblock decode and an f32 linear with
  a sequential per-output sum.  The reference only reaches GGUF-correct K-quant
  arithmetic through the un-vendored llama.cpp (llama-cpp-sys-2 0.1.146,
  pesti-runner/Cargo.toml:61-62); O1 restates the published format and is
  pinned bit-for-bit against gguf-py 0.19.0 by the fixtures in tests/golden/.
* O2 "pesti-legacy" -- the reference's own CPU path:
  QuantizedLinear::forward (pesti-runner/src/quantized_linear.rs:101-183) over
  tile_dequant's 16-element blocks (pesti-runner/src/tile_dequant.rs:223-293,
  333-379), pinned by the reference's known-answer tests
  (tile_dequant.rs:450-539).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

GGUF_Q2_K = 10
GGUF_Q3_K = 11
GGUF_Q4_K = 12
GGUF_Q5_K = 13
GGUF_Q6_K = 14
PESTI_Q4_K_LEGACY = 112
PESTI_Q5_K_LEGACY = 113
PESTI_Q6_K_LEGACY = 114
#: bytes of one 256-weight GGUF superblock
GGUF_BLOCK_BYTES = {GGUF_Q2_K: 84, GGUF_Q3_K: 110, GGUF_Q4_K: 144, GGUF_Q5_K: 176, GGUF_Q6_K: 210}

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None
_lock = threading.Lock()


class OracleError(RuntimeError):
    pass


def build(force: bool = False) -> str:
    """Compile liboracle.so from kq_oracle.c with the Makefile beside it."""
    src = os.path.join(_HERE, "kq_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            build()
            lib = ctypes.CDLL(_LIB_PATH)
            P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
            lib.kqo_f16_to_f32.argtypes = [ctypes.c_uint16]
            lib.kqo_f16_to_f32.restype = ctypes.c_float
            lib.kqo_gguf_row_bytes.argtypes = [I, I64]
            lib.kqo_gguf_row_bytes.restype = I64
            for name in ("kqo_dequant_q2_k", "kqo_dequant_q3_k", "kqo_dequant_q4_k", "kqo_dequant_q5_k",
                         "kqo_dequant_q6_k"):
                getattr(lib, name).argtypes = [P, I64, P]
                getattr(lib, name).restype = I
            lib.kqo_dequant_blocks.argtypes = [I, P, I64, P]
            lib.kqo_dequant_blocks.restype = I
            lib.kqo_gguf_dequant_rows.argtypes = [I, P, I64, I64, I64, I64, P]
            lib.kqo_gguf_linear.argtypes = [I, P, I64, I64, P, I64, P, P, I]
            lib.kqo_legacy_row_bytes.argtypes = [I, I64]
            lib.kqo_legacy_row_bytes.restype = I64
            lib.kqo_legacy_dequant_q4_k_tile.argtypes = [P, I64, I64, P]
            lib.kqo_legacy_dequant_q6_k_tile.argtypes = [P, I64, I64, P]
            lib.kqo_legacy_dequant_rows.argtypes = [I, P, I64, I64, I64, I64, P]
            lib.kqo_legacy_forward.argtypes = [I, P, I64, I64, I64, P, I64, P, P, I, I]
            for name in ("kqo_dequant_q4_k", "kqo_dequant_q6_k", "kqo_gguf_dequant_rows",
                         "kqo_gguf_linear", "kqo_legacy_dequant_q4_k_tile",
                         "kqo_legacy_dequant_q6_k_tile", "kqo_legacy_dequant_rows",
                         "kqo_legacy_forward"):
                getattr(lib, name).restype = I
            _lib = lib
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _check(rc, what):
    if rc != 0:
        raise OracleError(f"{what} failed with status {rc}")


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def f16_to_f32(bits: int) -> float:
    return _load().kqo_f16_to_f32(bits)


def gguf_row_bytes(qtype: int, k: int) -> int:
    return int(_load().kqo_gguf_row_bytes(qtype, k))


def legacy_row_bytes(qtype: int, k: int) -> int:
    return int(_load().kqo_legacy_row_bytes(qtype, k))


def dequant_blocks(qtype: int, raw) -> np.ndarray:
    """Decode whole GGUF superblocks (raw bytes, any shape) to f32 [nblocks*256]."""
    raw = _u8(raw)
    bs = GGUF_BLOCK_BYTES.get(qtype)
    if bs is None:
        raise OracleError(f"type {qtype} is not a GGUF K-quant")
    if raw.size % bs:
        raise OracleError("byte count is not a whole number of superblocks")
    nb = raw.size // bs
    out = np.empty(nb * 256, np.float32)
    _check(_load().kqo_dequant_blocks(qtype, _ptr(raw), nb, _ptr(out)), "dequant")
    return out


def gguf_dequant_rows(qtype: int, w, n: int, k: int, row0: int = 0, nrows: int | None = None) -> np.ndarray:
    w = _u8(w)
    nrows = n - row0 if nrows is None else nrows
    out = np.empty((nrows, k), np.float32)
    _check(_load().kqo_gguf_dequant_rows(qtype, _ptr(w), n, k, row0, nrows, _ptr(out)), "gguf_dequant_rows")
    return out


def gguf_linear(qtype: int, w, n: int, k: int, x, bias=None, nthreads: int | None = None) -> np.ndarray:
    """y[m, n] = x[m, :] . W[n, :] (+bias) with a sequential f32 sum per output."""
    w = _u8(w)
    x = _f32(x).reshape(-1, k)
    bias = _f32(bias)
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    nt = nthreads or (os.cpu_count() or 1)
    _check(_load().kqo_gguf_linear(qtype, _ptr(w), n, k, _ptr(x), m, _ptr(bias), _ptr(y), nt), "gguf_linear")
    return y


def legacy_dequant_tile(qtype: int, data, tile_size: int) -> np.ndarray:
    data = _u8(data)
    out = np.empty(tile_size, np.float32)
    fn = (_load().kqo_legacy_dequant_q4_k_tile if qtype in (PESTI_Q4_K_LEGACY, PESTI_Q5_K_LEGACY)
          else _load().kqo_legacy_dequant_q6_k_tile)
    _check(fn(_ptr(data), data.size, tile_size, _ptr(out)), "legacy_dequant_tile")
    return out


def legacy_dequant_rows(qtype: int, data, k: int, row0: int, nrows: int) -> np.ndarray:
    data = _u8(data)
    out = np.empty((nrows, k), np.float32)
    _check(_load().kqo_legacy_dequant_rows(qtype, _ptr(data), data.size, k, row0, nrows, _ptr(out)),
           "legacy_dequant_rows")
    return out


def legacy_forward(qtype: int, data, in_features: int, out_features: int, x, batch: int,
                   bias=None, nthreads: int = 1, threads_over_batch: bool = True) -> np.ndarray:
    """QuantizedLinear::forward restated; returns y [batch, out_features]."""
    data = _u8(data)
    x = _f32(x).reshape(-1)
    bias = _f32(bias)
    y = np.empty((batch, out_features), np.float32)
    _check(_load().kqo_legacy_forward(qtype, _ptr(data), data.size, in_features, out_features,
                                      _ptr(x), batch, _ptr(bias), _ptr(y), nthreads,
                                      1 if threads_over_batch else 0), "legacy_forward")
    return y
