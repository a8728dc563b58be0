"""CPU tests of the oracle itself: it must agree with every golden vector and
known-answer test before it is trusted as the checker for the CUDA library.

* GGUF (O1): bit-exact against the gguf-py 0.19.0 fixtures in tests/golden/
  (edge cases: zero / subnormal / max / inf / nan scales, saturated bits), and
  against gguf-py itself when it is importable.
* pesti-legacy (O2): the reference's own unit tests
  (pesti-runner/src/tile_dequant.rs:422-539, transformer/linear.rs:196-259,
  tests/dispatch_integration.rs:204-223) restated with its block layout.
"""
import os

import numpy as np
import pytest

import oracle
from pesti_b200 import synthetic

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gguf_kquant_golden.npz")
GOLDEN_MORE = os.path.join(os.path.dirname(__file__), "golden", "gguf_kquant_more_golden.npz")
MORE = [("q2k", oracle.GGUF_Q2_K), ("q3k", oracle.GGUF_Q3_K), ("q5k", oracle.GGUF_Q5_K)]


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    eq = a.view(np.uint32) == b.view(np.uint32)
    return bool(np.all(eq | (np.isnan(a) & np.isnan(b))))


def f16(v):
    return np.array([v], np.float16).view(np.uint8)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def golden_more():
    return np.load(GOLDEN_MORE)


# ---- O1: GGUF superblocks ------------------------------------------------

@pytest.mark.parametrize("tag,qtype", [("q4k", oracle.GGUF_Q4_K), ("q6k", oracle.GGUF_Q6_K)])
def test_gguf_dequant_matches_golden(golden, tag, qtype):
    raw = golden[f"{tag}_raw"]
    want = golden[f"{tag}_bits"].view(np.float32).reshape(-1)
    got = oracle.dequant_blocks(qtype, raw)
    assert same_bits(got, want)


def test_golden_covers_special_values(golden):
    for tag in ("q4k", "q6k"):
        vals = golden[f"{tag}_bits"].view(np.float32)
        assert np.isnan(vals).any() and np.isinf(vals).any()
        assert (vals == 0).any() and (np.abs(vals[np.isfinite(vals)]) > 1e3).any()


@pytest.mark.parametrize("qtype,bs", [(oracle.GGUF_Q4_K, 144), (oracle.GGUF_Q6_K, 210)])
def test_gguf_dequant_matches_gguf_py(qtype, bs):
    gguf = pytest.importorskip("gguf")
    qt = gguf.GGMLQuantizationType.Q4_K if qtype == oracle.GGUF_Q4_K else gguf.GGMLQuantizationType.Q6_K
    rng = np.random.default_rng(99)
    raw = rng.integers(0, 256, (20000, bs), dtype=np.uint8)
    with np.errstate(all="ignore"):
        want = gguf.quants.dequantize(raw, qt).reshape(-1).astype(np.float32)
    assert same_bits(oracle.dequant_blocks(qtype, raw), want)


@pytest.mark.parametrize("tag,qtype", [("q4k", oracle.GGUF_Q4_K), ("q6k", oracle.GGUF_Q6_K)])
def test_gguf_linear_matches_f64_fixture(golden, tag, qtype):
    w, x, y64 = golden[f"lin_{tag}_w"], golden[f"lin_{tag}_x"], golden[f"lin_{tag}_y64"]
    n, k = y64.shape[1], x.shape[1]
    y = oracle.gguf_linear(qtype, w, n, k, x)
    err = np.max(np.abs(y - y64)) / np.max(np.abs(y64))
    assert err < 1e-5


@pytest.mark.parametrize("tag,qtype", MORE)
def test_other_k_quants_match_golden(golden_more, tag, qtype):
    raw = golden_more[f"{tag}_raw"]
    want = golden_more[f"{tag}_bits"].view(np.float32).reshape(-1)
    assert same_bits(oracle.dequant_blocks(qtype, raw), want)
    vals = want
    assert np.isnan(vals).any() and np.isinf(vals).any() and (vals == 0).any()
    w, x, y64 = golden_more[f"lin_{tag}_w"], golden_more[f"lin_{tag}_x"], golden_more[f"lin_{tag}_y64"]
    y = oracle.gguf_linear(qtype, w, y64.shape[1], x.shape[1], x)
    assert np.max(np.abs(y - y64)) / np.max(np.abs(y64)) < 1e-5


@pytest.mark.parametrize("tag,qtype", MORE)
def test_other_k_quants_match_gguf_py(tag, qtype):
    gguf = pytest.importorskip("gguf")
    qt = {oracle.GGUF_Q2_K: gguf.GGMLQuantizationType.Q2_K, oracle.GGUF_Q3_K: gguf.GGMLQuantizationType.Q3_K,
          oracle.GGUF_Q5_K: gguf.GGMLQuantizationType.Q5_K}[qtype]
    rng = np.random.default_rng(98)
    raw = rng.integers(0, 256, (20000, oracle.GGUF_BLOCK_BYTES[qtype]), dtype=np.uint8)
    with np.errstate(all="ignore"):
        want = gguf.quants.dequantize(raw, qt).reshape(-1).astype(np.float32)
    assert same_bits(oracle.dequant_blocks(qtype, raw), want)


def test_legacy_q5k_rows_decode_as_q4k_tiles():
    # quantized_linear.rs:91,170-173: 36 bytes per 16 weights per row, read by the Q4_K tile routine
    n, k = 5, 300
    data = synthetic.legacy_weight(oracle.PESTI_Q5_K_LEGACY, n, k, seed=3)
    assert data.shape == (n, ((k + 15) // 16) * 36) == (n, oracle.legacy_row_bytes(oracle.PESTI_Q5_K_LEGACY, k))
    for r in range(n):
        want = oracle.legacy_dequant_tile(oracle.PESTI_Q4_K_LEGACY, data[r], k)
        got = oracle.legacy_dequant_rows(oracle.PESTI_Q5_K_LEGACY, data, k, r, 1)[0]
        assert same_bits(got, want)


def test_gguf_linear_threading_is_bitwise_stable():
    w = synthetic.q4_k_weight(37, 512, seed=3)
    x = synthetic.activations(2, 512, seed=4)
    b = np.linspace(-1, 1, 37).astype(np.float32)
    y1 = oracle.gguf_linear(oracle.GGUF_Q4_K, w, 37, 512, x, b, nthreads=1)
    y5 = oracle.gguf_linear(oracle.GGUF_Q4_K, w, 37, 512, x, b, nthreads=5)
    assert same_bits(y1, y5)


def test_gguf_row_bytes():
    assert oracle.gguf_row_bytes(oracle.GGUF_Q4_K, 4096) == 16 * 144
    assert oracle.gguf_row_bytes(oracle.GGUF_Q6_K, 14336) == 56 * 210
    assert oracle.gguf_row_bytes(oracle.GGUF_Q4_K, 300) == -1
    assert oracle.gguf_row_bytes(oracle.GGUF_Q2_K, 512) == 2 * 84
    assert oracle.gguf_row_bytes(oracle.GGUF_Q3_K, 512) == 2 * 110
    assert oracle.gguf_row_bytes(oracle.GGUF_Q5_K, 512) == 2 * 176


def test_f16_conversion_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    assert same_bits(got, want[::97])


# ---- O2: the reference's own tests, restated -----------------------------

def test_legacy_zero_block():  # tile_dequant.rs:422-432 / :450-458
    out = oracle.legacy_dequant_tile(oracle.PESTI_Q6_K_LEGACY, np.zeros(42, np.uint8), 16)
    assert np.all(out == 0.0)


def test_legacy_tile_sizes():  # tile_dequant.rs:434-448
    assert oracle.legacy_dequant_tile(oracle.PESTI_Q4_K_LEGACY, np.zeros(280, np.uint8), 50).size == 50
    assert oracle.legacy_dequant_tile(oracle.PESTI_Q6_K_LEGACY, np.zeros(420, np.uint8), 50).size == 50


def test_legacy_q6k_known_value():  # tile_dequant.rs:460-472
    data = np.zeros(42, np.uint8)
    data[0:2] = f16(1.0)
    data[2:4] = f16(1.0)
    out = oracle.legacy_dequant_tile(oracle.PESTI_Q6_K_LEGACY, data, 16)
    assert abs(out[0] - (-32.0)) < 0.01


def test_legacy_q4k_partial_block():  # tile_dequant.rs:475-508
    data = np.zeros(32, np.uint8)
    data[0:2] = f16(1.0)
    data[2:4] = f16(0.5)
    data[28:30] = f16(2.0)
    out = oracle.legacy_dequant_tile(oracle.PESTI_Q4_K_LEGACY, data, 20)
    assert out.size == 20
    assert np.all(np.abs(out[:16] - 1.0) < 0.01)
    assert np.all(np.abs(out[16:] - 2.0) < 0.01)


def test_legacy_q4k_300_elements():  # tile_dequant.rs:510-539
    nfull, rem = 300 // 16, 300 % 16
    data = np.zeros(nfull * 28 + (4 if rem else 0), np.uint8)
    for b in range(nfull):
        data[b * 28:b * 28 + 2] = f16(1.0)
    data[nfull * 28:nfull * 28 + 2] = f16(1.0)
    out = oracle.legacy_dequant_tile(oracle.PESTI_Q4_K_LEGACY, data, 300)
    assert out.size == 300 and np.all(np.abs(out - 1.0) < 0.01)


def test_legacy_short_tile_is_an_error():  # tile_dequant.rs:229-234
    with pytest.raises(oracle.OracleError):
        oracle.legacy_dequant_tile(oracle.PESTI_Q4_K_LEGACY, np.zeros(27, np.uint8), 16)
    with pytest.raises(oracle.OracleError):
        oracle.legacy_dequant_tile(oracle.PESTI_Q6_K_LEGACY, np.zeros(41, np.uint8), 1)


def _legacy_q4_block(values, delta=1.0, d=0.0):
    """A legacy Q4_K block whose 16 weights are ((delta*1)*(q-4)) + d."""
    b = np.zeros(28, np.uint8)
    b[0:2] = f16(d)
    b[2:4] = f16(delta)
    b[12:14] = f16(1.0)
    b[14:16] = f16(1.0)
    q = [int(v) + 4 for v in values] + [4] * (16 - len(values))
    lo = sum((q[i] & 0xF) << (4 * i) for i in range(8))
    hi = sum((q[8 + i] & 0xF) << (4 * i) for i in range(8))
    b[4:8] = np.array([lo], np.uint32).view(np.uint8)
    b[8:12] = np.array([hi], np.uint32).view(np.uint8)
    return b


def test_legacy_forward_linear_known_answer():
    # transformer/linear.rs:196-229: W = [[1,2,3],[4,5,6]], bias [0.1, 0.2],
    # x = [[1,2,3],[4,5,6]] -> [14.1, 32.2, 32.1, 77.2]; K padded to one block
    data = np.concatenate([_legacy_q4_block([1, 2, 3]), _legacy_q4_block([4, 5, 6])])
    x = np.zeros((2, 16), np.float32)
    x[0, :3] = [1, 2, 3]
    x[1, :3] = [4, 5, 6]
    y = oracle.legacy_forward(oracle.PESTI_Q4_K_LEGACY, data, 16, 2, x, 2,
                              bias=np.array([0.1, 0.2], np.float32))
    assert np.allclose(y.reshape(-1), [14.1, 32.2, 32.1, 77.2], atol=1e-5)


def test_legacy_forward_no_bias_known_answer():
    # transformer/linear.rs:231-259: W = [[1,2],[3,4],[5,6]], x = [1,2] -> [5, 11, 17]
    data = np.concatenate([_legacy_q4_block(r) for r in ([1, 2], [3, 4], [5, 6])])
    x = np.zeros(16, np.float32)
    x[:2] = [1, 2]
    y = oracle.legacy_forward(oracle.PESTI_Q4_K_LEGACY, data, 16, 3, x, 1)
    assert np.allclose(y.reshape(-1), [5, 11, 17], atol=1e-5)


def test_legacy_forward_dispatch_known_answer():
    # tests/dispatch_integration.rs:204-223: W = [[1,0.5],[0.5,1]], bias 0.1,
    # x = [1, 2] -> [2.1, 2.6].  0.5 * (q-4) with q in {5, 6} gives 0.5 / 1.0.
    data = np.concatenate([_legacy_q4_block([2, 1], delta=0.5), _legacy_q4_block([1, 2], delta=0.5)])
    x = np.zeros(16, np.float32)
    x[:2] = [1, 2]
    y = oracle.legacy_forward(oracle.PESTI_Q4_K_LEGACY, data, 16, 2, x, 1,
                              bias=np.array([0.1, 0.1], np.float32))
    assert np.allclose(y.reshape(-1), [2.1, 2.6], atol=1e-4)


@pytest.mark.parametrize("qtype", [oracle.PESTI_Q4_K_LEGACY, oracle.PESTI_Q6_K_LEGACY])
def test_legacy_forward_thread_split_is_bitwise_stable(qtype):
    n, k, m = 19, 300, 3
    data = synthetic.legacy_weight(qtype, n, k, seed=5)
    x = synthetic.activations(m, k, seed=6)
    a = oracle.legacy_forward(qtype, data, k, n, x, m, nthreads=1, threads_over_batch=True)
    b = oracle.legacy_forward(qtype, data, k, n, x, m, nthreads=4, threads_over_batch=False)
    assert same_bits(a, b)


def test_legacy_forward_matches_dequant_then_f64_dot():
    qtype, n, k, m = oracle.PESTI_Q6_K_LEGACY, 23, 200, 2
    data = synthetic.legacy_weight(qtype, n, k, seed=8)
    x = synthetic.activations(m, k, seed=9)
    w = oracle.legacy_dequant_rows(qtype, data, k, 0, n)
    y = oracle.legacy_forward(qtype, data, k, n, x, m)
    y64 = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(y - y64)) / np.max(np.abs(y64)) < 1e-5


def test_legacy_forward_short_data_is_an_error():
    qtype = oracle.PESTI_Q4_K_LEGACY
    data = np.zeros(28 * 2 - 1, np.uint8)
    with pytest.raises(oracle.OracleError):
        oracle.legacy_forward(qtype, data, 16, 2, np.zeros(16, np.float32), 1)
