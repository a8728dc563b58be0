"""CPU checks of the C ABI: the library builds for sm_100a, loads, exports
every entry point include/pesti_kq.h declares, and rejects bad arguments with
status codes (these paths run before any device work, so no GPU is needed)."""
import ctypes
import os
import re

import numpy as np
import pytest

from pesti_b200 import build, kq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            with open(os.path.join(ROOT, "include", fn)) as fh:
                text = fh.read()
            names |= set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(kq_\w+)\s*\(", text, re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    build.build()
    return kq.load_library()


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 15
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(kq.EXPORTED_SYMBOLS) <= names


def test_abi_version(lib):
    assert lib.kq_abi_version() == 1


def test_status_strings(lib):
    for st in range(8):
        assert kq.status_string(st)
    assert kq.status_string(0) == "ok"
    assert kq.status_string(4) == "buffer too short"


def test_row_bytes(lib):
    assert kq.row_bytes(kq.KQ_GGUF_Q4_K, 4096) == 2304
    assert kq.row_bytes(kq.KQ_GGUF_Q6_K, 14336) == 11760
    # QuantizedLinear::row_bytes (quantized_linear.rs:91,93)
    assert kq.row_bytes(kq.KQ_PESTI_Q4_K_LEGACY, 300) == 19 * 28
    assert kq.row_bytes(kq.KQ_PESTI_Q6_K_LEGACY, 16) == 42
    with pytest.raises(kq.KqError) as e:
        kq.row_bytes(kq.KQ_GGUF_Q4_K, 300)
    assert e.value.status == kq.KQ_ERR_UNSUPPORTED
    with pytest.raises(kq.KqError):
        kq.row_bytes(99, 256)


def test_null_arguments_are_rejected(lib):
    assert lib.kq_ctx_create(0, None) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_ctx_destroy(None) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_weight_free(None) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_linear_f32(None, None, None, 1, None, None, 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dequant_f32(None, None, 0, 1, None, 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_last_error(None) == b"no context"
    assert lib.kq_ctx_launch_count(None) == -1


def test_context_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    h = ctypes.c_void_p()
    rc = lib.kq_ctx_create(0, ctypes.byref(h))
    assert rc in (kq.KQ_ERR_CUDA, kq.KQ_ERR_INVALID_ARG)
    assert not h.value


def test_unknown_dtype_raises_before_touching_a_device():
    # QuantizedLinear::from_quantized returns Err for unknown names (quantized_linear.rs:58-63)
    with pytest.raises(kq.KqError) as e:
        kq.QuantizedLinear.from_quantized(np.zeros(18, np.uint8), "Q4_0", 32, 1)
    assert e.value.status == kq.KQ_ERR_UNSUPPORTED
    with pytest.raises(kq.KqError):
        kq.QuantizedLinear(np.zeros(144, np.uint8), "Q4_K", 256, 1, layout="ggml-f16")


def test_library_is_built_for_sm100a():
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert os.path.exists(build.LIB)
