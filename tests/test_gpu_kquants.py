"""GGUF Q2_K, Q3_K and Q5_K on the device (kq_kx.cu, the single-token dp4a
kernel of kq_dp4a.cu, batches on the integer-MMA kernel of kq_imma.cu) and the
reference's legacy Q5_K rows:
dequantization bit-exact with the oracle (on the gguf-py fixture superblocks
and on random weights), linears within 1e-3 of max|y| of the oracle's
sequential f32 product at 1 to 13 tokens, upload from a GGUF file, and the
drop-in constructors' dtype names."""
import os

import numpy as np
import pytest

import oracle
from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3
TYPES = [("Q2_K", kq.KQ_GGUF_Q2_K, oracle.GGUF_Q2_K, "q2k"), ("Q3_K", kq.KQ_GGUF_Q3_K, oracle.GGUF_Q3_K, "q3k"),
         ("Q5_K", kq.KQ_GGUF_Q5_K, oracle.GGUF_Q5_K, "q5k")]
GOLDEN_MORE = os.path.join(os.path.dirname(__file__), "golden", "gguf_kquant_more_golden.npz")


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
def test_dequant_of_the_fixture_superblocks_is_bit_exact(gpu_ctx, name, kt, ot, tag):
    g = np.load(GOLDEN_MORE)
    raw = g[f"{tag}_raw"]  # one superblock per row: edge cases (inf, nan, subnormal d) and random
    want = g[f"{tag}_bits"].view(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, raw.shape[0], 256)
    assert same_bits(w.dequant(), want)
    w.free()


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
@pytest.mark.parametrize("n,k", [(37, 1280), (300, 4096), (5, 256), (129, 2816)])
def test_dequant_of_random_weights_is_bit_exact(gpu_ctx, name, kt, ot, tag, n, k):
    raw = synthetic.gguf_weight(kt, n, k, seed=n + k)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    assert same_bits(w.dequant(), oracle.gguf_dequant_rows(ot, raw, n, k))
    assert same_bits(w.dequant(n // 2, 2), oracle.gguf_dequant_rows(ot, raw, n, k, n // 2, 2))
    w.free()


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
@pytest.mark.parametrize("n,k", [(4096, 4096), (37, 1280), (300, 2816), (1024, 14336)])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 13])
def test_linear_matches_the_oracle(gpu_ctx, name, kt, ot, tag, n, k, m):
    raw = synthetic.gguf_weight(kt, n, k, seed=3 * n + k)
    x = synthetic.activations(m, k, seed=m + 11)
    bias = np.linspace(-2, 2, n).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    y = np.empty((m, n), np.float32)
    w.linear(x, m, y, bias)
    ref = oracle.gguf_linear(ot, raw, n, k, x, bias)
    assert rel_err(y, ref) <= TOL
    for t in range(m):  # every token, not only the one with the largest output
        assert rel_err(y[t], ref[t]) <= TOL
    w.free()


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
@pytest.mark.parametrize("n,k", [(4096, 4096), (37, 1280), (1024, 14336), (16, 32768)])
def test_one_token_on_both_kernels(gpu_ctx, name, kt, ot, tag, n, k):
    """m = 1 runs the single-token dp4a kernel under AUTO (in_features up to
    30720; wider rows fall through to the f32 kernel) and the f32 kernel
    under another path; both against the oracle, and against each other."""
    raw = synthetic.gguf_weight(kt, n, k, seed=5 * n + k)
    x = synthetic.activations(1, k, seed=17)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    ref = oracle.gguf_linear(ot, raw, n, k, x, bias)
    y_auto = np.empty((1, n), np.float32)
    y_f32 = np.empty((1, n), np.float32)
    try:
        w.linear(x, 1, y_auto, bias)
        gpu_ctx.set_path(kq.KQ_PATH_MMA)
        w.linear(x, 1, y_f32, bias)
    finally:
        gpu_ctx.set_path(kq.KQ_PATH_AUTO)
    assert rel_err(y_auto, ref) <= TOL
    assert rel_err(y_f32, ref) <= TOL
    assert rel_err(y_auto, y_f32) <= TOL
    w.free()


@pytest.mark.parametrize("name,kt,ot", [("Q5_K", kq.KQ_GGUF_Q5_K, oracle.GGUF_Q5_K),
                                        ("Q3_K", kq.KQ_GGUF_Q3_K, oracle.GGUF_Q3_K),
                                        ("Q2_K", kq.KQ_GGUF_Q2_K, oracle.GGUF_Q2_K)], ids=["Q5_K", "Q3_K", "Q2_K"])
@pytest.mark.parametrize("n,k,m", [(4096, 4096, 8), (300, 2816, 5), (1024, 14336, 32), (130, 1280, 40)])
def test_batches_on_integer_mma_and_the_f32_kernel(gpu_ctx, name, kt, ot, n, k, m):
    """Q5_K, Q3_K and Q2_K at 2..64 tokens run the integer tensor-core kernel
    under AUTO (32-token chunks above 32) and the f32 kernel under another path."""
    raw = synthetic.gguf_weight(kt, n, k, seed=n + 7 * k + m)
    x = synthetic.activations(m, k, seed=m)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    ref = oracle.gguf_linear(ot, raw, n, k, x, bias)
    y_mma = np.empty((m, n), np.float32)
    y_f32 = np.empty((m, n), np.float32)
    try:
        w.linear(x, m, y_mma, bias)
        gpu_ctx.set_path(kq.KQ_PATH_MMA)
        w.linear(x, m, y_f32, bias)
    finally:
        gpu_ctx.set_path(kq.KQ_PATH_AUTO)
    for t in range(m):
        assert rel_err(y_mma[t], ref[t]) <= TOL
        assert rel_err(y_f32[t], ref[t]) <= TOL
    w.free()


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
def test_one_token_with_non_finite_and_zero_activations(gpu_ctx, name, kt, ot, tag):
    """The single-token kernel's per-superblock activation scale: an all-zero
    superblock of x gives exact zeros from it, and an inf in x makes NaN
    (or inf) the rows the f32 product makes non-finite, as the oracle does."""
    n, k = 64, 1024
    raw = synthetic.gguf_weight(kt, n, k, seed=9)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    x = synthetic.activations(1, k, seed=3)
    x[0, 256:512] = 0.0
    y = np.empty((1, n), np.float32)
    w.linear(x, 1, y)
    assert rel_err(y, oracle.gguf_linear(ot, raw, n, k, x)) <= TOL
    x[0, 700] = np.inf
    w.linear(x, 1, y)
    ref = oracle.gguf_linear(ot, raw, n, k, x)
    assert np.array_equal(np.isfinite(y), np.isfinite(ref))
    w.free()


@pytest.mark.parametrize("name,kt,ot,tag", TYPES, ids=[t[0] for t in TYPES])
def test_linear_on_a_device_stream_and_from_the_constructors(gpu_ctx, name, kt, ot, tag):
    import torch
    n, k, m = 512, 1536, 4
    raw = synthetic.gguf_weight(kt, n, k, seed=77)
    x = synthetic.activations(m, k, seed=78)
    ref = oracle.gguf_linear(ot, raw, n, k, x)
    ql = kq.QuantizedLinear.from_quantized(raw, name if name != "Q5_K" else "Q5_K_M", k, n, ctx=gpu_ctx)
    assert ql.kq_type == kt
    assert rel_err(ql.forward(x.reshape(-1), m), ref) <= TOL
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        yd = ql.forward_device(torch.from_numpy(x).cuda())
    s.synchronize()
    assert rel_err(yd.cpu().numpy(), ref) <= TOL
    with pytest.raises(kq.KqError) as e:  # no prefill (bf16) form for these types
        ql.weight.linear_bf16(np.zeros((m, k), np.uint16), m, np.empty((m, n), np.float32))
    assert e.value.status == kq.KQ_ERR_UNSUPPORTED


def test_upload_from_a_gguf_file(gpu_ctx, tmp_path):
    gguf = pytest.importorskip("gguf")
    tensors = {}
    path = tmp_path / "more.gguf"
    wr = gguf.GGUFWriter(str(path), "llama")
    for i, (name, kt, ot, tag) in enumerate(TYPES):
        n, k = 48 + i, 768
        raw = synthetic.gguf_weight(kt, n, k, seed=i)
        tensors[f"t{i}.weight"] = (raw, kt, ot, n, k)
        wr.add_tensor(f"t{i}.weight", raw, raw_dtype=getattr(gguf.GGMLQuantizationType, name))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    with kq.GgufFile(str(path)) as f:
        for tname, (raw, kt, ot, n, k) in tensors.items():
            wf = f.upload(gpu_ctx, tname)
            assert (wf.kq_type, wf.out_features, wf.in_features) == (kt, n, k)
            assert same_bits(wf.dequant(), oracle.gguf_dequant_rows(ot, raw, n, k))
            x = synthetic.activations(3, k, seed=5)
            y = np.empty((3, n), np.float32)
            wf.linear(x, 3, y)
            assert rel_err(y, oracle.gguf_linear(ot, raw, n, k, x)) <= TOL
            wf.free()
            layer = kq.QuantizedLinear.from_gguf(f, tname, ctx=gpu_ctx)
            assert layer.kq_type == kt


@pytest.mark.parametrize("n,k,m", [(37, 300, 1), (37, 300, 5), (16, 16, 2), (5, 20, 1)])
def test_legacy_q5k_matches_the_reference_forward(gpu_ctx, n, k, m):
    # QuantizedLinear::new(.., QuantDtype::Q5_K, ..): 36-byte-per-16 rows read as Q4_K tiles
    raw = synthetic.legacy_weight(kq.KQ_PESTI_Q5_K_LEGACY, n, k, seed=7)
    x = synthetic.activations(m, k, seed=8)
    bias = np.linspace(-1, 1, n).astype(np.float32)
    ql = kq.QuantizedLinear.new(raw, kq.QuantDtype.Q5_K, k, n, bias, layout="pesti-legacy", ctx=gpu_ctx)
    y = ql.forward(x.reshape(-1), m)
    ref = oracle.legacy_forward(oracle.PESTI_Q5_K_LEGACY, raw, k, n, x, m, bias=bias)
    assert rel_err(y, ref) <= TOL
    deq = ql.weight.dequant()
    assert same_bits(deq, oracle.legacy_dequant_rows(oracle.PESTI_Q5_K_LEGACY, raw, k, 0, n))
