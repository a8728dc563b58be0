"""GPU parity: the sm_100a kernels, called through the C ABI, against the oracle.

Bars (stated here, applied below):
* dequantized values: bit-exact (NaN compared as NaN);
* f32 linear: max|y - y_ref| / max|y_ref| <= 1e-3, y_ref = the oracle's
  sequential f32 sum (the f64 error is also checked, to the same bar).
"""
import os

import numpy as np
import pytest

import oracle
from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def same_bits(a, b):
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


GGUF = {"Q4_K": (kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K), "Q6_K": (kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K)}
LEGACY = {"Q4_K": (kq.KQ_PESTI_Q4_K_LEGACY, oracle.PESTI_Q4_K_LEGACY),
          "Q6_K": (kq.KQ_PESTI_Q6_K_LEGACY, oracle.PESTI_Q6_K_LEGACY)}


# ---- dequantization: bit-exact -------------------------------------------

@pytest.mark.parametrize("tag,dt", [("q4k", "Q4_K"), ("q6k", "Q6_K")])
def test_dequant_golden_blocks_bit_exact(gpu_ctx, tag, dt):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "gguf_kquant_golden.npz"))
    raw = g[f"{tag}_raw"]
    w = kq.Weight(gpu_ctx, GGUF[dt][0], raw, raw.shape[0], 256)
    got = w.dequant()
    assert same_bits(got, g[f"{tag}_bits"].view(np.float32))


@pytest.mark.parametrize("dt,n,k", [("Q4_K", 4096, 4096), ("Q6_K", 4096, 14336), ("Q6_K", 7, 4864)])
def test_dequant_random_bit_exact(gpu_ctx, dt, n, k):
    kt, ot = GGUF[dt]
    raw = synthetic.gguf_weight(kt, n, k, seed=11)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    for r0, nr in ((0, min(n, 48)), (max(0, n - 5), min(n, 5))):
        assert same_bits(w.dequant(r0, nr), oracle.gguf_dequant_rows(ot, raw, n, k, r0, nr))


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("k", [16, 20, 50, 300, 4096])
def test_dequant_legacy_bit_exact(gpu_ctx, dt, k):
    kt, ot = LEGACY[dt]
    n = 9
    raw = synthetic.legacy_weight(kt, n, k, seed=k)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    assert same_bits(w.dequant(), oracle.legacy_dequant_rows(ot, raw, k, 0, n))


# ---- linear: tolerance against the oracle ---------------------------------

CASES = [
    ("Q4_K", 4096, 4096, 1),   # decode GEMV, the Q4_K benchmark shape
    ("Q4_K", 13, 256, 1),      # one superblock per row, odd row count
    ("Q4_K", 257, 512, 3),
    ("Q4_K", 64, 1024, 31),    # m not a multiple of the m-tile
    ("Q6_K", 4096, 14336, 1),  # decode GEMV, the Q6_K benchmark shape
    ("Q6_K", 4096, 14336, 8),
    ("Q6_K", 4096, 14336, 32),
    ("Q6_K", 33, 4864, 2),     # 19 superblocks per row
    ("Q6_K", 1, 256, 5),
    ("Q4_K", 100, 2048, 12),   # m > 8: hi-only fragments, 2 n-tiles
    ("Q6_K", 48, 1536, 20),    # 3 n-tiles
    ("Q4_K", 40, 768, 40),     # m > 32: two chunks
    ("Q4_K", 4096, 4096, 8),   # batched decode shapes (integer MMA: split-K over 32 row tiles)
    ("Q4_K", 4096, 4096, 32),
    ("Q4_K", 300, 14336, 5),   # rows not a multiple of the 128-row tile, 56 superblocks
    ("Q6_K", 4096, 4096, 8),
    ("Q6_K", 1024, 14336, 32),
    ("Q6_K", 300, 14336, 5),
    ("Q4_K", 9600, 512, 40),   # 75 row tiles: the 32-token chunk runs unsplit, the 8-token tail split in two
]


PATHS = {"tcgen05": kq.KQ_PATH_TCGEN05, "mma": kq.KQ_PATH_MMA, "dp4a": kq.KQ_PATH_DP4A, "imma": kq.KQ_PATH_IMMA}
DP4A_MAX_M = 4  # the integer dot-product family serves 1..4 tokens


@pytest.fixture(params=sorted(PATHS))
def path_ctx(gpu_ctx, request):
    gpu_ctx.set_path(PATHS[request.param])
    gpu_ctx.path_name = request.param
    yield gpu_ctx
    gpu_ctx.set_path(kq.KQ_PATH_AUTO)


def test_tcgen05_single_tile_first(gpu_ctx):
    # the smallest tensor-core case (one CTA, one superblock) before anything larger
    gpu_ctx.set_path(kq.KQ_PATH_TCGEN05)
    try:
        for kt, ot in GGUF.values():
            raw = synthetic.gguf_weight(kt, 128, 256, seed=1)
            x = synthetic.activations(1, 256, seed=2)
            w = kq.Weight(gpu_ctx, kt, raw, 128, 256)
            y = np.empty((1, 128), np.float32)
            w.linear(x, 1, y)
            assert rel_err(y, oracle.gguf_linear(ot, raw, 128, 256, x)) <= TOL
    finally:
        gpu_ctx.set_path(kq.KQ_PATH_AUTO)


@pytest.mark.parametrize("dt,n,k,m", CASES)
def test_linear_matches_oracle(path_ctx, dt, n, k, m):
    if path_ctx.path_name == "dp4a" and m > DP4A_MAX_M:
        pytest.skip("larger batches leave the dp4a family")
    kt, ot = GGUF[dt]
    raw = synthetic.gguf_weight(kt, n, k, seed=n + k)
    x = synthetic.activations(m, k, seed=m)
    bias = np.random.default_rng(3).standard_normal(n).astype(np.float32)
    w = kq.Weight(path_ctx, kt, raw, n, k)
    y = np.empty((m, n), np.float32)
    w.linear(x, m, y, bias)
    ref = oracle.gguf_linear(ot, raw, n, k, x, bias)
    assert rel_err(y, ref) <= TOL
    wf = oracle.gguf_dequant_rows(ot, raw, n, k).astype(np.float64)
    ref64 = x.astype(np.float64) @ wf.T + bias
    assert rel_err(y, ref64) <= TOL


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
def test_activation_outliers(path_ctx, dt):
    # one large activation per token and a superblock of tiny ones: the decode
    # kernels scale activations per token or per superblock, both must hold
    kt, ot = GGUF[dt]
    n, k, m = 96, 2048, 3
    raw = synthetic.gguf_weight(kt, n, k, seed=11)
    x = synthetic.activations(m, k, seed=12)
    x[0, 7] = 3.0e4
    x[1, 300:556] *= 1e-30
    x[2, 1000] = -5.0e3
    w = kq.Weight(path_ctx, kt, raw, n, k)
    y = np.empty((m, n), np.float32)
    w.linear(x, m, y)
    wf = oracle.gguf_dequant_rows(ot, raw, n, k).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    for t in range(m):
        assert rel_err(y[t], ref[t]) <= TOL


def test_nonfinite_activation_gives_nonfinite_rows(gpu_ctx):
    kt, ot = GGUF["Q4_K"]
    n, k = 64, 1024
    raw = synthetic.gguf_weight(kt, n, k, seed=13)
    x = synthetic.activations(2, k, seed=14)
    x[1, 5] = np.inf
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    y = np.empty((2, n), np.float32)
    w.linear(x, 2, y)
    ref = oracle.gguf_linear(ot, raw, n, k, x)
    assert np.isfinite(y[0]).all()
    assert rel_err(y[0], ref[0]) <= TOL
    assert not np.isfinite(ref[1]).any() and not np.isfinite(y[1]).any()


# ---- prefill: bf16 activations on tcgen05, <= 2e-2 against the f32 product ----

PREFILL_TOL = 2e-2
PREFILL_CASES = [
    ("Q4_K", 4096, 4096, 512),
    ("Q6_K", 1024, 4096, 300),   # m not a multiple of the 256-token tile
    ("Q4_K", 100, 1024, 37),     # partial row tile, few tokens
    ("Q6_K", 256, 4864, 257),
    ("Q6_K", 4864, 1024, 1000),  # 38 row tiles x 4 token tiles: 256-token tiles on 148 SMs
]


def to_bf16_bits(x):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16), t.float().numpy()


@pytest.mark.parametrize("dt,n,k,m", PREFILL_CASES)
def test_prefill_bf16_matches_f32_product(gpu_ctx, dt, n, k, m):
    kt, ot = GGUF[dt]
    raw = synthetic.gguf_weight(kt, n, k, seed=n + 3 * k)
    bits, xr = to_bf16_bits(synthetic.activations(m, k, seed=m + 1))
    bias = np.random.default_rng(4).standard_normal(n).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    y = np.empty((m, n), np.float32)
    w.linear_bf16(bits, m, y, bias)
    wf = oracle.gguf_dequant_rows(ot, raw, n, k).astype(np.float64)
    ref = xr.astype(np.float64) @ wf.T + bias
    assert rel_err(y, ref) <= PREFILL_TOL


@pytest.mark.parametrize("n", [4096, 14336])
def test_prefill_at_the_benchmark_shapes(gpu_ctx, n):
    """The prefill GEMM at every (N, K, M) the benchmark quotes: Q4_K weights
    of 4096x4096 and 14336x4096 against bf16 N(0, 1) activations at M = 512,
    2048 and 4096 tokens, each against the f64 product of the oracle's
    dequantized weight and the bf16-rounded activations (<= 2e-2 of max|y|)."""
    kt, ot = GGUF["Q4_K"]
    k = 4096
    raw = synthetic.gguf_weight(kt, n, k, seed=n + 7)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    wf = oracle.gguf_dequant_rows(ot, raw, n, k).astype(np.float64)
    for m in (512, 2048, 4096):
        bits, xr = to_bf16_bits(synthetic.activations(m, k, seed=m + n))
        y = np.empty((m, n), np.float32)
        w.linear_bf16(bits, m, y)
        ref = xr.astype(np.float64) @ wf.T
        err = rel_err(y, ref)
        assert err <= PREFILL_TOL, (n, m, err)
        assert np.isfinite(y).all()
    w.free()


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n,k,m", [(37, 300, 1), (37, 300, 5), (16, 16, 2), (5, 20, 1)])
def test_legacy_linear_matches_reference_forward(gpu_ctx, dt, n, k, m):
    kt, ot = LEGACY[dt]
    raw = synthetic.legacy_weight(kt, n, k, seed=7)
    x = synthetic.activations(m, k, seed=8)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    ql = kq.QuantizedLinear(raw, dt, k, n, bias, layout="pesti-legacy", ctx=gpu_ctx)
    y = ql.forward(x.reshape(-1), m)
    ref = oracle.legacy_forward(ot, raw, k, n, x, m, bias=bias)
    assert y.shape == (m * n,)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n,k", [(4096, 4096), (4096, 14336), (37, 256), (300, 2816), (64, 4000), (16, 32768)])
@pytest.mark.parametrize("m", [1, 3])
def test_legacy_small_batches_on_both_kernels(gpu_ctx, dt, n, k, m):
    """Up to 4 tokens over the reference's blocks: the single-token integer
    kernel (one pass per token) under AUTO where rows are whole 256-weight
    spans up to 30720 weights (the others fall through), the block kernel
    under another path; both against the reference's forward, every token,
    and against each other."""
    kt, ot = LEGACY[dt]
    raw = synthetic.legacy_weight(kt, n, k, seed=n + k)
    x = synthetic.activations(m, k, seed=k)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    ref = oracle.legacy_forward(ot, raw, k, n, x, m, bias=bias).reshape(m, n)
    y_auto = np.empty((m, n), np.float32)
    y_blk = np.empty((m, n), np.float32)
    try:
        w.linear(x, m, y_auto, bias)
        gpu_ctx.set_path(kq.KQ_PATH_MMA)
        w.linear(x, m, y_blk, bias)
    finally:
        gpu_ctx.set_path(kq.KQ_PATH_AUTO)
    for t in range(m):
        assert rel_err(y_auto[t], ref[t]) <= TOL
        assert rel_err(y_blk[t], ref[t]) <= TOL
        assert rel_err(y_auto[t], y_blk[t]) <= TOL
    w.free()


def test_device_pointer_path_on_a_torch_stream(gpu_ctx):
    import torch
    n, k, m = 4096, 4096, 4
    raw = synthetic.q4_k_weight(n, k, seed=21)
    x = synthetic.activations(m, k, seed=22)
    ql = kq.QuantizedLinear.from_quantized(raw, "Q4_K_M", k, n, ctx=gpu_ctx)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        xd = torch.from_numpy(x).cuda()
        before = gpu_ctx.launch_count
        yd = ql.forward_device(xd)
        assert gpu_ctx.launch_count > before
    s.synchronize()
    ref = oracle.gguf_linear(oracle.GGUF_Q4_K, raw, n, k, x)
    assert rel_err(yd.cpu().numpy(), ref) <= TOL


# ---- size-independent properties at full size ----------------------------

@pytest.mark.parametrize("dt,n,k", [("Q4_K", 4096, 4096), ("Q6_K", 4096, 14336)])
def test_linearity_and_zero_input(gpu_ctx, dt, n, k):
    kt, _ = GGUF[dt]
    raw = synthetic.gguf_weight(kt, n, k, seed=5)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    x1 = synthetic.activations(2, k, seed=1)
    x2 = synthetic.activations(2, k, seed=2)
    y1, y2, y3 = (np.empty((2, n), np.float32) for _ in range(3))
    w.linear(x1, 2, y1)
    w.linear(x2, 2, y2)
    w.linear(2.0 * x1 + x2, 2, y3)
    assert rel_err(y3, 2.0 * y1.astype(np.float64) + y2) <= TOL
    bias = np.arange(n, dtype=np.float32)
    y0 = np.empty((1, n), np.float32)
    w.linear(np.zeros((1, k), np.float32), 1, y0, bias)
    assert np.array_equal(y0.reshape(-1), bias)


def test_repeat_calls_are_deterministic(gpu_ctx):
    raw = synthetic.q6_k_weight(512, 4096, seed=9)
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q6_K, raw, 512, 4096)
    x = synthetic.activations(3, 4096, seed=10)
    a, b = np.empty((3, 512), np.float32), np.empty((3, 512), np.float32)
    w.linear(x, 3, a)
    w.linear(x, 3, b)
    assert np.array_equal(a, b)


# ---- drop-in behaviour and edge cases ------------------------------------

def test_quantized_linear_memory_accounting(gpu_ctx):
    raw = synthetic.q4_k_weight(8, 512, seed=1)
    ql = kq.QuantizedLinear.new(raw, kq.QuantDtype.Q4_K, 512, 8, np.zeros(8, np.float32), ctx=gpu_ctx)
    assert ql.memory_bytes() == raw.size + 32
    assert ql.f32_memory_bytes() == 8 * 512 * 4 + 32
    assert abs(ql.memory_savings() - (8 * 512 * 4 + 32) / (raw.size + 32)) < 1e-12


def test_short_weight_returns_zeros_like_the_reference(gpu_ctx, capsys):
    # quantized_linear.rs:108-114: decode error -> eprintln + zeros
    raw = synthetic.q4_k_weight(4, 256, seed=1).reshape(-1)[:-1]
    ql = kq.QuantizedLinear.from_quantized(raw, "Q4_K", 256, 4, ctx=gpu_ctx)
    y = ql.forward(np.ones(256, np.float32), 1)
    assert y.shape == (4,) and np.all(y == 0)
    assert "dequantize_full_row_range error" in capsys.readouterr().err


def test_empty_shapes(gpu_ctx):
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, np.zeros(0, np.uint8), 5, 0)
    bias = np.arange(5, dtype=np.float32)
    y = np.full((2, 5), -1.0, np.float32)
    w.linear(np.zeros((2, 0), np.float32), 2, y, bias)
    assert np.array_equal(y, np.stack([bias, bias]))
    w2 = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q6_K, synthetic.q6_k_weight(3, 256), 3, 256)
    w2.linear(np.zeros((0, 256), np.float32), 0, np.zeros((0, 3), np.float32))  # m = 0: no-op


def test_invalid_arguments_report_status(gpu_ctx):
    with pytest.raises(kq.KqError) as e:
        kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, np.zeros(144, np.uint8), 1, 300)
    assert e.value.status == kq.KQ_ERR_UNSUPPORTED
    with pytest.raises(kq.KqError) as e:
        kq.Weight(gpu_ctx, kq.KQ_GGUF_Q6_K, np.zeros(209, np.uint8), 1, 256)
    assert e.value.status == kq.KQ_ERR_SHORT_BUFFER
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q6_K, synthetic.q6_k_weight(3, 256), 3, 256)
    with pytest.raises(kq.KqError) as e:
        w.dequant(2, 5)
    assert e.value.status == kq.KQ_ERR_INVALID_ARG
    rc = gpu_ctx.lib.kq_linear_f32(gpu_ctx.handle, w.handle, None, 1, None, None, 0)
    assert rc == kq.KQ_ERR_INVALID_ARG
    rc = gpu_ctx.lib.kq_linear_f32(gpu_ctx.handle, w.handle, None, 1, None, None, 0x40)
    assert rc == kq.KQ_ERR_INVALID_ARG


def test_queued_host_pointer_calls_match_synchronous_ones(gpu_ctx):
    """KQ_ASYNC: host-pointer calls queued back to back through the same
    staging buffers, one synchronize at the end, give the synchronous results
    (stream order keeps each call's staging copies apart)."""
    import torch
    n, k, m = 1024, 4096, 3
    raws = [synthetic.gguf_weight(kt, n, k, seed=40 + i) for i, kt in enumerate((kq.KQ_GGUF_Q4_K, kq.KQ_GGUF_Q6_K,
                                                                                   kq.KQ_GGUF_Q4_K))]
    ws = [kq.Weight(gpu_ctx, kt, r, n, k) for kt, r in zip((kq.KQ_GGUF_Q4_K, kq.KQ_GGUF_Q6_K, kq.KQ_GGUF_Q4_K), raws)]
    xs = [torch.from_numpy(synthetic.activations(m, k, seed=50 + i)).pin_memory() for i in range(3)]
    ys = [torch.full((m, n), float("nan")).pin_memory() for _ in range(3)]
    for w, x, y in zip(ws, xs, ys):
        w.linear(x.numpy(), m, y.numpy(), queue=True)
    gpu_ctx.synchronize()
    for w, x, y in zip(ws, xs, ys):
        ref = np.empty((m, n), np.float32)
        w.linear(x.numpy(), m, ref)
        assert np.array_equal(y.numpy(), ref)
    rc = gpu_ctx.lib.kq_linear_f32(gpu_ctx.handle, ws[0].handle, None, 1, None, None,
                                   kq.KQ_DEVICE_PTRS | kq.KQ_ASYNC)
    assert rc == kq.KQ_ERR_INVALID_ARG
    for w in ws:
        w.free()
