"""Python binding of libpesti_kq.so and the QuantizedLinear drop-in.

``QuantizedLinear`` mirrors pesti-runner's quantized-matmul entry point
(pesti-runner/src/quantized_linear.rs:12-183): the same constructor names and
argument meaning (``new``, ``from_quantized``), ``forward(x, batch_size)``
returning a fresh f32 vector of ``batch_size * out_features`` values, and the
memory accounting helpers.  The weight bytes are uploaded once and stay
resident in HBM; ``forward`` runs the sm_100a kernels through the C ABI
(include/pesti_kq.h).  There is no CPU path: if the library cannot be loaded or
no GPU is present, construction raises.

Error behaviour follows the reference:
* ``from_quantized`` with an unknown dtype name raises (reference: Err).
* a weight whose bytes are too short for its shape does not fail at
  construction; ``forward`` prints the decode error to stderr and returns
  zeros, as ``QuantizedLinear::forward`` does (quantized_linear.rs:108-114).
"""
from __future__ import annotations

import ctypes
import os
import sys
import threading
from typing import Optional

import numpy as np

from . import build as _build

KQ_OK = 0
KQ_ERR_INVALID_ARG = 1
KQ_ERR_UNSUPPORTED = 2
KQ_ERR_CUDA = 3
KQ_ERR_SHORT_BUFFER = 4
KQ_ERR_NCCL = 5
KQ_ERR_STATE = 6
KQ_ERR_NOMEM = 7
KQ_ERR_FORMAT = 8

KQ_GGUF_Q2_K = 10
KQ_GGUF_Q3_K = 11
KQ_GGUF_Q4_K = 12
KQ_GGUF_Q5_K = 13
KQ_GGUF_Q6_K = 14
KQ_PESTI_Q4_K_LEGACY = 112
KQ_PESTI_Q5_K_LEGACY = 113
KQ_PESTI_Q6_K_LEGACY = 114

KQ_HOST_PTRS = 0
KQ_DEVICE_PTRS = 1
KQ_SYNC = 2
KQ_ACCUMULATE = 4
KQ_ASYNC = 8

KQ_PATH_AUTO = 0
KQ_PATH_TCGEN05 = 1
KQ_PATH_MMA = 2
KQ_PATH_DP4A = 3
KQ_PATH_IMMA = 4

#: every symbol include/pesti_kq.h declares
EXPORTED_SYMBOLS = (
    "kq_abi_version", "kq_status_string", "kq_last_error",
    "kq_ctx_create", "kq_ctx_destroy", "kq_ctx_set_stream", "kq_ctx_synchronize",
    "kq_ctx_set_path", "kq_ctx_reserve", "kq_ctx_prefetch_next", "kq_ctx_launch_count", "kq_ctx_profile_begin",
    "kq_ctx_profile_end", "kq_ctx_profile_read", "kq_row_bytes", "kq_weight_upload", "kq_weight_free", "kq_weight_info",
    "kq_linear_f32", "kq_linear_bf16", "kq_linear_f32_static", "kq_dequant_f32",
    "kq_tp_create", "kq_tp_handle", "kq_tp_open", "kq_tp_linear_f32", "kq_tp_allgather_f32",
    "kq_tp_allreduce_f32",
    "kq_tp_destroy", "kq_dec_rmsnorm", "kq_dec_rope_append", "kq_dec_attention_scratch", "kq_dec_attention",
    "kq_dec_swiglu", "kq_dec_add", "kq_dec_embed", "kq_dec_norm_linear", "kq_dec_swiglu_linear",
    "kq_dec_residual_linear", "kq_dec_norm_linear_batch", "kq_dec_residual_linear_batch", "kq_dec_rope_attention",
    "kq_dec_tp_partial_linear", "kq_dec_tp_reduce_linear",
    "kq_step_create", "kq_step_linear", "kq_step_attention", "kq_step_run", "kq_step_trace", "kq_step_destroy",
    "kq_gguf_open", "kq_gguf_close", "kq_gguf_tensor_count", "kq_gguf_find_tensor", "kq_gguf_tensor_info",
    "kq_gguf_read_tensor", "kq_gguf_upload", "kq_gguf_meta_count", "kq_gguf_find_meta", "kq_gguf_meta_info",
    "kq_gguf_meta_int", "kq_gguf_meta_float", "kq_gguf_meta_string", "kq_gguf_meta_array",
)


class KqError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


_lib = None
_lib_lock = threading.Lock()


def library_path() -> str:
    return _build.LIB


def load_library(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libpesti_kq.so (building it in-tree first if it is absent)."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if not os.path.exists(path):
            if not build_if_missing:
                raise KqError(KQ_ERR_STATE, f"{path} is missing; build it with python -m pesti_b200.build")
            _build.build()
        lib = ctypes.CDLL(path)
        P, I, I64, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
        PP = ctypes.POINTER(ctypes.c_void_p)
        sig = {
            "kq_abi_version": ([], I),
            "kq_status_string": ([I], ctypes.c_char_p),
            "kq_last_error": ([P], ctypes.c_char_p),
            "kq_ctx_create": ([I, PP], I),
            "kq_ctx_destroy": ([P], I),
            "kq_ctx_set_stream": ([P, P], I),
            "kq_ctx_synchronize": ([P], I),
            "kq_ctx_set_path": ([P, I], I),
            "kq_ctx_reserve": ([P, P, I64], I),
            "kq_ctx_prefetch_next": ([P, P], I),
            "kq_ctx_launch_count": ([P], I64),
            "kq_ctx_profile_begin": ([P, I], I),
            "kq_ctx_profile_end": ([P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(I64)], I),
            "kq_ctx_profile_read": ([P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(I64)], I),
            "kq_row_bytes": ([I, I64, ctypes.POINTER(I64)], I),
            "kq_weight_upload": ([P, I, P, Z, I64, I64, PP], I),
            "kq_weight_free": ([P], I),
            "kq_weight_info": ([P, ctypes.POINTER(I), ctypes.POINTER(I64), ctypes.POINTER(I64),
                                ctypes.POINTER(I64)], I),
            "kq_linear_f32": ([P, P, P, I64, P, P, I], I),
            "kq_linear_bf16": ([P, P, P, I64, P, P, I], I),
            "kq_linear_f32_static": ([P, P, P, I64, P, P, I], I),
            "kq_dequant_f32": ([P, P, I64, I64, P, I], I),
            "kq_tp_create": ([P, I, I, I64, PP], I),
            "kq_tp_handle": ([P, P, ctypes.POINTER(Z)], I),
            "kq_tp_open": ([P, P, Z], I),
            "kq_tp_linear_f32": ([P, P, I64, I64, P, I64, P, P, I], I),
            "kq_tp_allgather_f32": ([P, P, I64, I64, I64, I64, P, I64, I], I),
            "kq_tp_allreduce_f32": ([P, P, I64, I64, P, I64, I], I),
            "kq_tp_destroy": ([P], I),
            "kq_gguf_open": ([ctypes.c_char_p, PP, ctypes.c_char_p, Z], I),
            "kq_gguf_close": ([P], None),
            "kq_gguf_tensor_count": ([P], I64),
            "kq_gguf_find_tensor": ([P, ctypes.c_char_p], I64),
            "kq_gguf_tensor_info": ([P, I64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I), ctypes.POINTER(I),
                                     ctypes.POINTER(I64), ctypes.POINTER(ctypes.c_uint64),
                                     ctypes.POINTER(ctypes.c_uint64)], I),
            "kq_gguf_read_tensor": ([P, I64, P, ctypes.c_uint64], I),
            "kq_gguf_upload": ([P, P, I64, PP], I),
            "kq_gguf_meta_count": ([P], I64),
            "kq_gguf_find_meta": ([P, ctypes.c_char_p], I64),
            "kq_gguf_meta_info": ([P, I64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I), ctypes.POINTER(I),
                                   ctypes.POINTER(ctypes.c_uint64)], I),
            "kq_gguf_meta_int": ([P, I64, ctypes.POINTER(I64)], I),
            "kq_gguf_meta_float": ([P, I64, ctypes.POINTER(ctypes.c_double)], I),
            "kq_gguf_meta_string": ([P, I64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
                                     ctypes.POINTER(ctypes.c_uint64)], I),
            "kq_gguf_meta_array": ([P, I64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_uint64)], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load_library().kq_status_string(status).decode()


def row_bytes(kq_type: int, in_features: int) -> int:
    out = ctypes.c_int64()
    rc = load_library().kq_row_bytes(kq_type, in_features, ctypes.byref(out))
    if rc:
        raise KqError(rc, f"kq_row_bytes({kq_type}, {in_features}): {status_string(rc)}")
    return out.value


def _ptr(a) -> Optional[int]:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return int(a.data_ptr())  # torch tensor


class Context:
    """One device and one stream (include/pesti_kq.h kq_ctx)."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        h = ctypes.c_void_p()
        rc = self.lib.kq_ctx_create(device, ctypes.byref(h))
        if rc:
            raise KqError(rc, f"kq_ctx_create(device={device}) failed: {status_string(rc)}")
        self.handle = h
        self.device = device

    def check(self, rc: int, what: str) -> None:
        if rc:
            msg = self.lib.kq_last_error(self.handle).decode()
            raise KqError(rc, f"{what}: {msg or status_string(rc)}")

    def set_stream(self, stream) -> None:
        """Install a cudaStream_t (int handle, torch.cuda.Stream, or None)."""
        if stream is not None and hasattr(stream, "cuda_stream"):
            stream = stream.cuda_stream
        handle = ctypes.c_void_p(int(stream)) if stream else None
        self.check(self.lib.kq_ctx_set_stream(self.handle, handle), "kq_ctx_set_stream")

    def synchronize(self) -> None:
        self.check(self.lib.kq_ctx_synchronize(self.handle), "kq_ctx_synchronize")

    def set_path(self, path: int) -> None:
        """KQ_PATH_AUTO / KQ_PATH_TCGEN05 / KQ_PATH_MMA / KQ_PATH_DP4A for GGUF weights."""
        self.check(self.lib.kq_ctx_set_path(self.handle, path), "kq_ctx_set_path")

    def reserve(self, weight: "Weight", m: int) -> None:
        """Allocate the scratch calls on `weight` with up to m rows need."""
        self.check(self.lib.kq_ctx_reserve(self.handle, weight.handle, m), "kq_ctx_reserve")

    def prefetch_next(self, weight: Optional["Weight"]) -> None:
        """The next linear call prefetches `weight` into L2 (one-shot hint; None clears)."""
        self.check(self.lib.kq_ctx_prefetch_next(self.handle, weight.handle if weight is not None else None),
                   "kq_ctx_prefetch_next")

    @property
    def launch_count(self) -> int:
        return int(self.lib.kq_ctx_launch_count(self.handle))

    def profile_begin(self, max_calls: int) -> None:
        """Bracket the main kernel of the next max_calls compute calls with CUDA events."""
        self.check(self.lib.kq_ctx_profile_begin(self.handle, max_calls), "kq_ctx_profile_begin")

    def profile_end(self):
        """-> (summed main-kernel milliseconds, number of bracketed calls)."""
        ms, n = ctypes.c_double(), ctypes.c_int64()
        self.check(self.lib.kq_ctx_profile_end(self.handle, ctypes.byref(ms), ctypes.byref(n)),
                   "kq_ctx_profile_end")
        return ms.value, n.value

    def profile_read(self):
        """-> (summed main-kernel milliseconds, count) as last recorded, session kept open."""
        ms, n = ctypes.c_double(), ctypes.c_int64()
        self.check(self.lib.kq_ctx_profile_read(self.handle, ctypes.byref(ms), ctypes.byref(n)),
                   "kq_ctx_profile_read")
        return ms.value, n.value

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.kq_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx = {}


def default_context(device: int = 0) -> Context:
    ctx = _default_ctx.get(device)
    if ctx is None:
        ctx = _default_ctx[device] = Context(device)
    return ctx


class Weight:
    """A device-resident K-quant weight (kq_weight)."""

    def __init__(self, ctx: Context, kq_type: int, data, out_features: int, in_features: int):
        self.ctx = ctx
        if getattr(data, "is_cuda", False):  # a CUDA tensor: uploaded device to device
            t = data.contiguous()
            ptr, size = (t.data_ptr() if t.numel() else None), t.numel() * t.element_size()
        else:
            raw = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray))
                                       else np.asarray(data, dtype=np.uint8)).reshape(-1)
            ptr, size = (raw.ctypes.data if raw.size else None), raw.size
        h = ctypes.c_void_p()
        rc = ctx.lib.kq_weight_upload(ctx.handle, kq_type, ptr, size, out_features, in_features, ctypes.byref(h))
        ctx.check(rc, "kq_weight_upload")
        self.handle = h
        self.kq_type = kq_type
        self.out_features = out_features
        self.in_features = in_features
        dev_bytes = ctypes.c_int64()
        ctx.lib.kq_weight_info(h, None, None, None, ctypes.byref(dev_bytes))
        self.device_bytes = dev_bytes.value

    @classmethod
    def _adopt(cls, ctx: Context, handle: ctypes.c_void_p) -> "Weight":
        """Wrap a kq_weight the library created (e.g. kq_gguf_upload)."""
        w = cls.__new__(cls)
        w.ctx = ctx
        w.handle = handle
        kt, n, k, dev_bytes = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        ctx.lib.kq_weight_info(handle, ctypes.byref(kt), ctypes.byref(n), ctypes.byref(k), ctypes.byref(dev_bytes))
        w.kq_type, w.out_features, w.in_features, w.device_bytes = kt.value, n.value, k.value, dev_bytes.value
        return w

    def linear(self, x, m: int, y, bias=None, device_ptrs: bool = False, sync: bool = False,
               queue: bool = False) -> None:
        """y = x . W^T (+bias).  Host arrays are copied in and out synchronously,
        unless queue=True (KQ_ASYNC): then the call only queues its copies and
        kernels, and x, bias and y must stay alive until Context.synchronize()."""
        flags = (KQ_DEVICE_PTRS if device_ptrs else KQ_HOST_PTRS) | (KQ_SYNC if sync else 0) | (KQ_ASYNC if queue else 0)
        rc = self.ctx.lib.kq_linear_f32(self.ctx.handle, self.handle, _ptr(x), m, _ptr(bias), _ptr(y), flags)
        self.ctx.check(rc, "kq_linear_f32")

    def linear_bf16(self, x, m: int, y, bias=None, device_ptrs: bool = False, sync: bool = False) -> None:
        """x holds bf16 bit patterns (uint16 numpy array or bf16 torch tensor)."""
        flags = (KQ_DEVICE_PTRS if device_ptrs else KQ_HOST_PTRS) | (KQ_SYNC if sync else 0)
        rc = self.ctx.lib.kq_linear_bf16(self.ctx.handle, self.handle, _ptr(x), m, _ptr(bias), _ptr(y), flags)
        self.ctx.check(rc, "kq_linear_bf16")

    def linear_static(self, x, m: int, y, bias=None, sync: bool = False) -> None:
        """kq_linear_f32_static: device tensors only, scratch from the fixed device array."""
        flags = KQ_DEVICE_PTRS | (KQ_SYNC if sync else 0)
        rc = self.ctx.lib.kq_linear_f32_static(self.ctx.handle, self.handle, _ptr(x), m, _ptr(bias), _ptr(y), flags)
        self.ctx.check(rc, "kq_linear_f32_static")

    def dequant(self, row0: int = 0, nrows: Optional[int] = None, out=None, device_ptrs: bool = False):
        nrows = self.out_features - row0 if nrows is None else nrows
        if out is None:
            out = np.empty((nrows, self.in_features), np.float32)
        flags = KQ_DEVICE_PTRS | KQ_SYNC if device_ptrs else KQ_HOST_PTRS
        rc = self.ctx.lib.kq_dequant_f32(self.ctx.handle, self.handle, row0, nrows, _ptr(out), flags)
        self.ctx.check(rc, "kq_dequant_f32")
        return out

    def free(self) -> None:
        if getattr(self, "handle", None):
            self.ctx.lib.kq_weight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def shard_rows(n: int, world: int, rank: int):
    """Contiguous, balanced row block [r0, r1) of an n-row weight for `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    return n * rank // world, n * (rank + 1) // world


def torch_exchange(blob: bytes, group=None):
    """All ranks' blobs in rank order, over torch.distributed (any backend)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, blob, group=group)
    return out


class TensorParallel:
    """One rank of a row-sharded linear group (kq_tp_*): each rank holds rows
    [r0, r1) of a weight; ``linear`` returns the full output on every rank,
    all-gathered over NVLink peer memory.  ``exchange(blob) -> [blob per rank]``
    moves the IPC handles between ranks (torch.distributed by default)."""

    def __init__(self, ctx: "Context", world: int, rank: int, max_out_elems: int, exchange=None):
        self.ctx, self.world, self.rank = ctx, world, rank
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.kq_tp_create(ctx.handle, world, rank, max_out_elems, ctypes.byref(h)), "kq_tp_create")
        self.handle = h
        size = ctypes.c_size_t(0)
        ctx.check(ctx.lib.kq_tp_handle(self.handle, None, ctypes.byref(size)), "kq_tp_handle")
        buf = ctypes.create_string_buffer(size.value)
        ctx.check(ctx.lib.kq_tp_handle(self.handle, buf, ctypes.byref(size)), "kq_tp_handle")
        blobs = (exchange or torch_exchange)(buf.raw[:size.value])
        if len(blobs) != world or any(len(b) != size.value for b in blobs):
            raise KqError(KQ_ERR_INVALID_ARG, "handle exchange returned the wrong blobs")
        joined = b"".join(blobs)
        ctx.check(ctx.lib.kq_tp_open(self.handle, joined, len(joined)), "kq_tp_open")

    def linear(self, shard: "Weight", row0: int, n_total: int, x, m: int, y, bias=None, sync: bool = False):
        flags = KQ_DEVICE_PTRS | (KQ_SYNC if sync else 0)
        rc = self.ctx.lib.kq_tp_linear_f32(self.handle, shard.handle, row0, n_total, _ptr(x), m, _ptr(bias),
                                           _ptr(y), flags)
        self.ctx.check(rc, "kq_tp_linear_f32")

    def allgather(self, y_local, m: int, row0: int, rows: int, n_total: int, y, y_ld: Optional[int] = None,
                  accumulate: bool = False, sync: bool = False):
        flags = KQ_DEVICE_PTRS | (KQ_SYNC if sync else 0) | (KQ_ACCUMULATE if accumulate else 0)
        rc = self.ctx.lib.kq_tp_allgather_f32(self.handle, _ptr(y_local), m, row0, rows, n_total, _ptr(y),
                                              n_total if y_ld is None else y_ld, flags)
        self.ctx.check(rc, "kq_tp_allgather_f32")

    def allreduce(self, partial, m: int, n: int, y, y_ld: Optional[int] = None, accumulate: bool = False,
                  sync: bool = False):
        """y (+)= the sum over the ranks of each rank's partial[m][n], in rank order."""
        flags = KQ_DEVICE_PTRS | (KQ_SYNC if sync else 0) | (KQ_ACCUMULATE if accumulate else 0)
        rc = self.ctx.lib.kq_tp_allreduce_f32(self.handle, _ptr(partial), m, n, _ptr(y), n if y_ld is None else y_ld,
                                              flags)
        self.ctx.check(rc, "kq_tp_allreduce_f32")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx.lib.kq_tp_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QuantDtype:
    """pesti-runner/src/tile_dequant.rs:394-402 (the K-quant members: Q4_K,
    Q5_K, Q6_K), plus the GGUF Q2_K and Q3_K superblock types, which the
    reference's loader decodes (gguf_weight_loader.rs:334-477) but its
    QuantizedLinear does not hold."""
    Q2_K = "Q2_K"
    Q3_K = "Q3_K"
    Q4_K = "Q4_K"
    Q5_K = "Q5_K"
    Q6_K = "Q6_K"


# quantized_linear.rs:51-57 (the K-quant names), plus the Q2_K / Q3_K names
_DTYPE_NAMES = {
    "Q4_K": QuantDtype.Q4_K, "Q4_K_M": QuantDtype.Q4_K, "Q4_K_S": QuantDtype.Q4_K,
    "Q5_K": QuantDtype.Q5_K, "Q5_K_M": QuantDtype.Q5_K, "Q5_K_S": QuantDtype.Q5_K,
    "Q6_K": QuantDtype.Q6_K, "Q6_K_S": QuantDtype.Q6_K,
    "Q2_K": QuantDtype.Q2_K, "Q2_K_S": QuantDtype.Q2_K,
    "Q3_K": QuantDtype.Q3_K, "Q3_K_S": QuantDtype.Q3_K, "Q3_K_M": QuantDtype.Q3_K, "Q3_K_L": QuantDtype.Q3_K,
}

_LAYOUTS = {
    ("gguf", QuantDtype.Q2_K): KQ_GGUF_Q2_K,
    ("gguf", QuantDtype.Q3_K): KQ_GGUF_Q3_K,
    ("gguf", QuantDtype.Q4_K): KQ_GGUF_Q4_K,
    ("gguf", QuantDtype.Q5_K): KQ_GGUF_Q5_K,
    ("gguf", QuantDtype.Q6_K): KQ_GGUF_Q6_K,
    ("pesti-legacy", QuantDtype.Q4_K): KQ_PESTI_Q4_K_LEGACY,
    ("pesti-legacy", QuantDtype.Q5_K): KQ_PESTI_Q5_K_LEGACY,
    ("pesti-legacy", QuantDtype.Q6_K): KQ_PESTI_Q6_K_LEGACY,
}


class QuantizedLinear:
    """Drop-in for pesti-runner's ``QuantizedLinear`` on a B200.

    ``layout="gguf"`` (default) reads GGUF superblocks (Q4_K 144 B / Q6_K
    210 B per 256 weights).  ``layout="pesti-legacy"`` reads the reference's
    own 28 B / 42 B per 16-weight blocks (tile_dequant.rs) so its CPU forward
    can be reproduced byte for byte.
    """

    def __init__(self, data, dtype: str, in_features: int, out_features: int,
                 bias=None, layout: str = "gguf", device: int = 0, ctx: Optional[Context] = None):
        if (layout, dtype) not in _LAYOUTS:
            raise KqError(KQ_ERR_UNSUPPORTED, f"unsupported layout/dtype {layout}/{dtype}")
        self.dtype = dtype
        self.layout = layout
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.kq_type = _LAYOUTS[(layout, dtype)]
        self.data = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray))
                                         else np.asarray(data, dtype=np.uint8)).reshape(-1)
        self.bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        self.ctx = ctx or default_context(device)
        self._decode_error = None
        self.weight = None
        try:
            self.weight = Weight(self.ctx, self.kq_type, self.data, self.out_features, self.in_features)
        except KqError as e:
            if e.status != KQ_ERR_SHORT_BUFFER:
                raise
            self._decode_error = str(e)

    # quantized_linear.rs:27-41
    @classmethod
    def new(cls, data, dtype: str, in_features: int, out_features: int, bias=None, **kw):
        return cls(data, dtype, in_features, out_features, bias, **kw)

    # quantized_linear.rs:44-67
    @classmethod
    def from_quantized(cls, data, gguf_dtype: str, in_features: int, out_features: int, bias=None, **kw):
        dtype = _DTYPE_NAMES.get(gguf_dtype)
        if dtype is None:
            raise KqError(KQ_ERR_UNSUPPORTED, f"Unsupported quantization type for QuantizedLinear: {gguf_dtype}")
        return cls(data, dtype, in_features, out_features, bias, **kw)

    @classmethod
    def from_gguf(cls, gguf_file, name: str, bias=None, **kw):
        """The layer of a 2-D Q4_K / Q6_K tensor of a GGUF file (a path or a
        GgufFile): its stored bytes, in_features = the row length."""
        if not isinstance(gguf_file, GgufFile):
            with GgufFile(gguf_file) as f:  # opened here, so closed here
                return cls.from_gguf(f, name, bias, **kw)
        f = gguf_file
        t = f.tensors[name]
        dtype = {KQ_GGUF_Q2_K: "Q2_K", KQ_GGUF_Q3_K: "Q3_K", KQ_GGUF_Q4_K: "Q4_K", KQ_GGUF_Q5_K: "Q5_K",
                 KQ_GGUF_Q6_K: "Q6_K"}.get(t.ggml_type)
        if dtype is None or len(t.dims) != 2:
            raise KqError(KQ_ERR_UNSUPPORTED, f"{name}: not a 2-D K-quant tensor (type {t.ggml_type})")
        return cls(f.read(name), dtype, t.dims[0], t.dims[1], bias, **kw)

    # quantized_linear.rs:70-83
    def memory_bytes(self) -> int:
        return int(self.data.size + (0 if self.bias is None else self.bias.size * 4))

    def f32_memory_bytes(self) -> int:
        return self.in_features * self.out_features * 4 + (0 if self.bias is None else self.bias.size * 4)

    def memory_savings(self) -> float:
        return self.f32_memory_bytes() / self.memory_bytes()

    def forward(self, x, batch_size: int) -> np.ndarray:
        """y = x @ W^T + bias for x of batch_size * in_features f32 values
        (quantized_linear.rs:101-143); returns batch_size * out_features f32."""
        m, k, n = int(batch_size), self.in_features, self.out_features
        y = np.zeros(m * n, np.float32)
        if self._decode_error is not None:
            print(f"dequantize_full_row_range error: {self._decode_error}", file=sys.stderr)
            return y
        xa = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        if xa.size < m * k:
            raise KqError(KQ_ERR_INVALID_ARG, f"x has {xa.size} values, batch {m} x {k} needs {m * k}")
        self.weight.linear(xa, m, y, self.bias)
        return y

    def forward_device(self, x, bias=None, out=None):
        """Device path: x is a CUDA torch tensor [m, in_features] f32 on this
        context's device; runs on torch's current stream and returns y
        [m, out_features] (no host round trip)."""
        import torch
        if self._decode_error is not None:
            raise KqError(KQ_ERR_SHORT_BUFFER, self._decode_error)
        if not (x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()):
            raise KqError(KQ_ERR_INVALID_ARG, "x must be a contiguous CUDA float32 tensor")
        m = x.numel() // self.in_features
        if out is None:
            out = torch.empty((m, self.out_features), dtype=torch.float32, device=x.device)
        self.ctx.set_stream(torch.cuda.current_stream(x.device).cuda_stream)
        self.weight.linear(x, m, out, bias, device_ptrs=True)
        return out


# ---- GGUF files ---------------------------------------------------------------

#: GGUF metadata value types
GGUF_STRING, GGUF_ARRAY = 8, 9
_GGUF_NUMPY = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32, 6: np.float32,
               7: np.uint8, 10: np.uint64, 11: np.int64, 12: np.float64}


class GgufTensor:
    """One entry of a GGUF tensor directory.  ``shape`` is in row-major order
    (the file's ne reversed: [..., rows, row length])."""

    def __init__(self, index, name, ggml_type, dims, offset, nbytes):
        self.index, self.name, self.ggml_type = index, name, ggml_type
        self.dims, self.offset, self.nbytes = tuple(dims), offset, nbytes
        self.shape = tuple(reversed(self.dims))

    def __repr__(self):
        return f"GgufTensor({self.name!r}, type={self.ggml_type}, shape={self.shape})"


class GgufFile:
    """A GGUF file opened through the library's reader (kq_gguf_*): the
    tensor directory and metadata, the raw bytes of any tensor, and Q4_K /
    Q6_K tensors uploaded as device-resident weights -- the path the
    reference takes through pesti-gguf's extract_tensor_bytes_from_path
    (gguf_weight_loader.rs:79-81) without its f32 copies."""

    def __init__(self, path: str):
        self.lib = load_library()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = self.lib.kq_gguf_open(os.fsencode(path), ctypes.byref(h), err, len(err))
        if rc != KQ_OK:
            raise KqError(rc, f"kq_gguf_open: {err.value.decode(errors='replace')}")
        self.handle = h
        self.path = path
        self.tensors = {}
        for i in range(self.lib.kq_gguf_tensor_count(h)):
            name, t, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
            dims, off, nb = (ctypes.c_int64 * 4)(), ctypes.c_uint64(), ctypes.c_uint64()
            self._check(self.lib.kq_gguf_tensor_info(h, i, ctypes.byref(name), ctypes.byref(t), ctypes.byref(nd), dims,
                                                     ctypes.byref(off), ctypes.byref(nb)), "kq_gguf_tensor_info")
            nm = self._name(name.value, "tensor name")
            self.tensors[nm] = GgufTensor(i, nm, t.value, list(dims)[:nd.value], off.value, nb.value)
        self.metadata = {}
        for i in range(self.lib.kq_gguf_meta_count(h)):
            key, vt, et, cnt = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
            self._check(self.lib.kq_gguf_meta_info(h, i, ctypes.byref(key), ctypes.byref(vt), ctypes.byref(et),
                                                   ctypes.byref(cnt)), "kq_gguf_meta_info")
            self.metadata[self._name(key.value, "metadata key")] = self._value(i, vt.value, et.value, cnt.value)

    def _name(self, raw: bytes, what: str) -> str:
        # GGUF names are UTF-8; anything else is a malformed file, not a Python decode error
        try:
            return raw.decode("utf-8", errors="strict")
        except UnicodeDecodeError as e:
            self.close()
            raise KqError(KQ_ERR_FORMAT, f"{self.path}: {what} is not UTF-8 ({e})") from None

    def _check(self, rc, what):
        if rc != KQ_OK:
            raise KqError(rc, f"{what} failed on {self.path}")

    def _string(self, i, j):
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        self._check(self.lib.kq_gguf_meta_string(self.handle, i, j, ctypes.byref(p), ctypes.byref(n)),
                    "kq_gguf_meta_string")
        return ctypes.string_at(p, n.value).decode(errors="replace")

    def _value(self, i, vt, et, count):
        if vt == GGUF_STRING:
            return self._string(i, 0)
        if vt == GGUF_ARRAY:
            if et == GGUF_STRING:
                return [self._string(i, j) for j in range(count)]
            if et == GGUF_ARRAY:
                return None  # nested arrays are listed, not kept
            p, eb = ctypes.c_void_p(), ctypes.c_uint64()
            self._check(self.lib.kq_gguf_meta_array(self.handle, i, ctypes.byref(p), ctypes.byref(eb)),
                        "kq_gguf_meta_array")
            raw = ctypes.string_at(p, count * eb.value) if count else b""
            arr = np.frombuffer(raw, dtype=_GGUF_NUMPY[et]).copy()
            return arr.astype(bool) if et == 7 else arr
        if vt in (6, 12):
            v = ctypes.c_double()
            self._check(self.lib.kq_gguf_meta_float(self.handle, i, ctypes.byref(v)), "kq_gguf_meta_float")
            return v.value
        v = ctypes.c_int64()
        self._check(self.lib.kq_gguf_meta_int(self.handle, i, ctypes.byref(v)), "kq_gguf_meta_int")
        return bool(v.value) if vt == 7 else v.value

    def read(self, name: str) -> np.ndarray:
        """The tensor's stored bytes (uint8)."""
        t = self.tensors[name]
        out = np.empty(t.nbytes, np.uint8)
        self._check(self.lib.kq_gguf_read_tensor(self.handle, t.index, out.ctypes.data if t.nbytes else None,
                                                 t.nbytes), "kq_gguf_read_tensor")
        return out

    def upload(self, ctx: Context, name: str) -> Weight:
        """A 2-D Q4_K / Q6_K tensor as a device-resident Weight."""
        t = self.tensors[name]
        h = ctypes.c_void_p()
        ctx.check(self.lib.kq_gguf_upload(ctx.handle, self.handle, t.index, ctypes.byref(h)), "kq_gguf_upload")
        return Weight._adopt(ctx, h)

    def close(self) -> None:
        if self.handle:
            self.lib.kq_gguf_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
