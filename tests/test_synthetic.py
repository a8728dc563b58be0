"""The seeded generators reproduce the benchmark shapes and distributions."""
import numpy as np

from pesti_b200 import synthetic


def test_q4k_shape_and_distribution():
    w = synthetic.q4_k_weight(64, 1024, seed=0)
    assert w.shape == (64, 4 * 144) and w.dtype == np.uint8
    blk = w.reshape(-1, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float32)
    assert np.all(d >= 0) and np.all(dmin >= 0)
    assert 0.01 < float(np.mean(d)) < 0.025  # E|N(0, 0.02)| = 0.016
    assert np.array_equal(w, synthetic.q4_k_weight(64, 1024, seed=0))
    assert not np.array_equal(w, synthetic.q4_k_weight(64, 1024, seed=1))


def test_q6k_scales_and_d():
    w = synthetic.q6_k_weight(32, 512, seed=0)
    blk = w.reshape(-1, 210)
    sc = blk[:, 192:208].view(np.int8)
    assert sc.min() >= -32 and sc.max() <= 31
    d = blk[:, 208:210].copy().view(np.float16).astype(np.float32)
    assert np.all(d >= 0) and 0.002 < float(np.mean(d)) < 0.006


def test_legacy_row_stride():
    for qt, bs in ((synthetic.PESTI_Q4_K_LEGACY, 28), (synthetic.PESTI_Q6_K_LEGACY, 42)):
        w = synthetic.legacy_weight(qt, 5, 300, seed=2)
        assert w.shape == (5, 19 * bs)


def test_activations():
    x = synthetic.activations(3, 256, seed=1)
    assert x.shape == (3, 256) and x.dtype == np.float32
    assert abs(float(x.std()) - 1.0) < 0.1
