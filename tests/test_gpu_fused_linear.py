"""Single-token linears with the decoder's activation transform fused into
the GEMV's activation staging (kq_dec_norm_linear, kq_dec_swiglu_linear,
kq_dec_residual_linear) and the L2 prefetch hint (kq_ctx_prefetch_next),
against the oracle: RMSNorm / SwiGLU restated from pesti's transformer
(oracle/decoder_oracle.py) followed by the GGUF dequantization and an f64
product."""
import ctypes

import numpy as np
import pytest

import oracle
from oracle import decoder_oracle
from pesti_b200 import decoder as dec
from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max|y - yref| / max|yref|, as for the plain GEMV
GGUF = {"Q4_K": (kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K), "Q6_K": (kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K)}


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _lib(ctx):
    return dec._bind(ctx.lib)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _w64(ot, raw, n, k):
    return oracle.gguf_dequant_rows(ot, raw, n, k).astype(np.float64)


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n,k,dim", [(256, 1024, 896), (300, 4096, 4096), (64, 14336, 14336)])
def test_norm_linear_matches_rmsnorm_then_linear(gpu_ctx, dt, n, k, dim):
    kt, ot = GGUF[dt]
    rng = np.random.default_rng(n + k)
    raw = synthetic.gguf_weight(kt, n, k, seed=k)
    h = np.zeros((1, k), np.float32)
    h[0, :dim] = 3.0 * rng.standard_normal(dim)
    nw = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    hd, nwd, yd = _dev(h), _dev(nw), _dev(np.full((1, n), np.nan, np.float32))
    rc = _lib(gpu_ctx).kq_dec_norm_linear(gpu_ctx.handle, w.handle, _p(hd), _p(nwd), dim, 1e-5, -1, None, _p(yd),
                                          kq.KQ_SYNC)
    gpu_ctx.check(rc, "norm_linear")
    a = np.zeros((1, k), np.float32)
    a[0, :dim] = decoder_oracle.rmsnorm(h[:, :dim], nw, 1e-5)
    ref = a.astype(np.float64) @ _w64(ot, raw, n, k).T
    assert rel_err(yd.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("mode", [dec.SWIGLU_REFERENCE, dec.SWIGLU_SILU])
def test_norm_linear_with_swiglu_pairs(gpu_ctx, dt, mode):
    """Gate and up projections as interleaved row pairs of one weight, the
    SwiGLU applied in the GEMV's epilogue: y[j] = swiglu(gate_j . a, up_j . a)
    with a = rmsnorm(h)."""
    kt, ot = GGUF[dt]
    f, k, dim = 1000, 4096, 4000
    rng = np.random.default_rng(mode + 31)
    raw_g = synthetic.gguf_weight(kt, f, k, seed=41)
    raw_u = synthetic.gguf_weight(kt, f, k, seed=42)
    rb = raw_g.size // f
    pairs = np.stack([raw_g.reshape(f, rb), raw_u.reshape(f, rb)], axis=1).reshape(-1)
    h = np.zeros((1, k), np.float32)
    h[0, :dim] = 2.0 * rng.standard_normal(dim)
    nw = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, pairs, 2 * f, k)
    hd, nwd, yd = _dev(h), _dev(nw), _dev(np.full((1, f), np.nan, np.float32))
    rc = _lib(gpu_ctx).kq_dec_norm_linear(gpu_ctx.handle, w.handle, _p(hd), _p(nwd), dim, 1e-6, mode, None, _p(yd),
                                          kq.KQ_SYNC)
    gpu_ctx.check(rc, "norm_linear pairs")
    a = np.zeros((1, k), np.float32)
    a[0, :dim] = decoder_oracle.rmsnorm(h[:, :dim], nw, 1e-6)
    g = a.astype(np.float64) @ _w64(ot, raw_g, f, k).T
    u = a.astype(np.float64) @ _w64(ot, raw_u, f, k).T
    ref = decoder_oracle.swiglu(g.astype(np.float32), u.astype(np.float32), mode)
    assert rel_err(yd.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("mode", [dec.SWIGLU_REFERENCE, dec.SWIGLU_SILU])
def test_swiglu_linear_with_residual(gpu_ctx, dt, mode):
    kt, ot = GGUF[dt]
    n, k = 512, 4864
    rng = np.random.default_rng(mode + 7)
    raw = synthetic.gguf_weight(kt, n, k, seed=11)
    gu = (2.0 * rng.standard_normal((1, 2 * k))).astype(np.float32)
    h = rng.standard_normal((1, n)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    gud, hd = _dev(gu), _dev(h)
    rc = _lib(gpu_ctx).kq_dec_swiglu_linear(gpu_ctx.handle, w.handle, _p(gud), mode, _p(hd), _p(hd), kq.KQ_SYNC)
    gpu_ctx.check(rc, "swiglu_linear")
    s = decoder_oracle.swiglu(gu[:, :k], gu[:, k:], mode)
    ref = h.astype(np.float64) + s.astype(np.float64) @ _w64(ot, raw, n, k).T
    assert rel_err(hd.cpu().numpy() - h, ref - h) <= TOL


@pytest.mark.parametrize("dt", ["Q4_K", "Q6_K"])
def test_residual_linear_adds_in_place(gpu_ctx, dt):
    kt, ot = GGUF[dt]
    n, k = 1000, 2048
    raw = synthetic.gguf_weight(kt, n, k, seed=3)
    x = synthetic.activations(1, k, seed=4)
    h = np.random.default_rng(5).standard_normal((1, n)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    xd, hd = _dev(x), _dev(h)
    gpu_ctx.check(_lib(gpu_ctx).kq_dec_residual_linear(gpu_ctx.handle, w.handle, _p(xd), _p(hd), kq.KQ_SYNC),
                 "residual")
    prod = x.astype(np.float64) @ _w64(ot, raw, n, k).T
    assert rel_err(hd.cpu().numpy() - h, prod) <= TOL


def test_fused_linears_reject_what_they_cannot_run(gpu_ctx):
    lib = _lib(gpu_ctx)
    raw = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 8, 256, seed=1)
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, raw, 8, 256)
    x, y = _dev(np.zeros((1, 256), np.float32)), _dev(np.zeros((1, 8), np.float32))
    h = gpu_ctx.handle
    assert lib.kq_dec_norm_linear(h, w.handle, _p(x), _p(x), 6, 1e-5, -1, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dec_norm_linear(h, w.handle, _p(x), _p(x), 512, 1e-5, -1, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dec_norm_linear(h, w.handle, _p(x), _p(x), 256, 1e-5, 2, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    odd = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 7, 256, seed=1), 7, 256)
    assert lib.kq_dec_norm_linear(h, odd.handle, _p(x), _p(x), 256, 1e-5, 0, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dec_swiglu_linear(h, w.handle, _p(x), 2, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dec_residual_linear(h, w.handle, None, _p(y), 0) == kq.KQ_ERR_INVALID_ARG
    # a row too long for the single-token kernel (121 superblocks)
    kb = 121 * 256
    big = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 4, kb, seed=2), 4, kb)
    xb = _dev(np.zeros((1, kb), np.float32))
    assert lib.kq_dec_residual_linear(h, big.handle, _p(xb), _p(y), 0) == kq.KQ_ERR_UNSUPPORTED
    gpu_ctx.synchronize()


def test_prefetch_hint_leaves_results_unchanged(gpu_ctx):
    """A linear that prefetches the next weight into L2 computes the same bits,
    and the hint is consumed by exactly one call."""
    import torch
    ws, xs = [], []
    shapes = [(kq.KQ_GGUF_Q4_K, 700, 4096), (kq.KQ_GGUF_Q6_K, 900, 4096), (kq.KQ_GGUF_Q4_K, 64, 512)]
    for i, (kt, n, k) in enumerate(shapes):
        ws.append(kq.Weight(gpu_ctx, kt, synthetic.gguf_weight(kt, n, k, seed=20 + i), n, k))
        xs.append(_dev(synthetic.activations(1, k, seed=30 + i)))
    plain = []
    for w, x in zip(ws, xs):
        y = torch.empty((1, w.out_features), device="cuda")
        w.linear(x, 1, y, device_ptrs=True)
        plain.append(y)
    for j in range(3):
        for i, (w, x) in enumerate(zip(ws, xs)):
            gpu_ctx.prefetch_next(ws[(i + 1 + j) % len(ws)])
            y = torch.empty_like(plain[i])
            w.linear(x, 1, y, device_ptrs=True)
            gpu_ctx.synchronize()
            assert torch.equal(y, plain[i])
    gpu_ctx.prefetch_next(None)


BATCH_TYPES = {"Q4_K": (kq.KQ_GGUF_Q4_K, oracle.GGUF_Q4_K), "Q5_K": (kq.KQ_GGUF_Q5_K, oracle.GGUF_Q5_K),
               "Q6_K": (kq.KQ_GGUF_Q6_K, oracle.GGUF_Q6_K)}


@pytest.mark.parametrize("dt", ["Q4_K", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("n,k,dim,m", [(256, 1024, 896, 8), (300, 4096, 4096, 5), (1024, 14336, 14336, 3),
                                       (600, 4096, 4000, 40)])
def test_batched_norm_linear_matches_rmsnorm_then_linear(gpu_ctx, dt, n, k, dim, m):
    """kq_dec_norm_linear_batch: every token's RMSNorm inside the integer-MMA
    kernel's activation preparation; rows of x x_ld = k + 8 floats apart."""
    kt, ot = BATCH_TYPES[dt]
    if dt == "Q6_K" and m > 8:
        m = 8  # Q6_K runs integer MMA up to 8 tokens
    rng = np.random.default_rng(n + k + m)
    raw = synthetic.gguf_weight(kt, n, k, seed=k + 1)
    ld = k + 8
    h = np.zeros((m, ld), np.float32)
    h[:, :dim] = 3.0 * rng.standard_normal((m, dim))
    h[:, dim:] = 7.0  # past dim (and past k): must not enter
    nw = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    hd, nwd, yd = _dev(h), _dev(nw), _dev(np.full((m, n), np.nan, np.float32))
    rc = _lib(gpu_ctx).kq_dec_norm_linear_batch(gpu_ctx.handle, w.handle, _p(hd), ld, m, _p(nwd), dim, 1e-5, _p(yd),
                                                kq.KQ_SYNC)
    gpu_ctx.check(rc, "norm_linear_batch")
    a = np.zeros((m, k), np.float32)
    a[:, :dim] = decoder_oracle.rmsnorm(h[:, :dim], nw, 1e-5)
    ref = a.astype(np.float64) @ _w64(ot, raw, n, k).T
    y = yd.cpu().numpy()
    for t in range(m):
        assert rel_err(y[t], ref[t]) <= TOL
    w.free()


@pytest.mark.parametrize("dt", ["Q4_K", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("n,k,m", [(4096, 4096, 8), (4096, 14336, 4), (130, 1024, 33)])
def test_batched_residual_linear_adds_into_h(gpu_ctx, dt, n, k, m):
    """kq_dec_residual_linear_batch: h += x . W^T from the kernel's epilogue,
    with and without split-K (the 4096-row cases split K across CTAs)."""
    kt, ot = BATCH_TYPES[dt]
    if dt == "Q6_K" and m > 8:
        m = 8
    raw = synthetic.gguf_weight(kt, n, k, seed=n + 3)
    x = synthetic.activations(m, k, seed=m + 5)
    h0 = np.random.default_rng(9).standard_normal((m, n)).astype(np.float32)
    w = kq.Weight(gpu_ctx, kt, raw, n, k)
    xd, hd = _dev(x), _dev(h0)
    lib = _lib(gpu_ctx)
    for rep in range(2):  # twice: the second call adds onto the first's result
        gpu_ctx.check(lib.kq_dec_residual_linear_batch(gpu_ctx.handle, w.handle, _p(xd), m, _p(hd), kq.KQ_SYNC),
                      "residual_linear_batch")
        ref = h0.astype(np.float64) + (rep + 1) * (x.astype(np.float64) @ _w64(ot, raw, n, k).T)
        got = hd.cpu().numpy()
        for t in range(m):
            assert rel_err(got[t] - h0[t], ref[t] - h0[t]) <= TOL
    w.free()


def test_batched_forms_report_unsupported_cases(gpu_ctx):
    """Where AUTO picks another kernel family (one token; Q6_K above 8
    tokens; the reference's legacy blocks) the batched forms queue nothing
    and say so."""
    lib = _lib(gpu_ctx)
    x = _dev(np.zeros((16, 1024), np.float32))
    nwd = _dev(np.ones(1024, np.float32))
    y = _dev(np.zeros((16, 256), np.float32))
    for kt, m in [(kq.KQ_GGUF_Q4_K, 1), (kq.KQ_GGUF_Q6_K, 9), (kq.KQ_PESTI_Q4_K_LEGACY, 4)]:
        raw = (synthetic.legacy_weight(kt, 256, 1024, seed=1) if kt == kq.KQ_PESTI_Q4_K_LEGACY
               else synthetic.gguf_weight(kt, 256, 1024, seed=1))
        w = kq.Weight(gpu_ctx, kt, raw, 256, 1024)
        launches = gpu_ctx.launch_count
        assert lib.kq_dec_residual_linear_batch(gpu_ctx.handle, w.handle, _p(x), m, _p(y), 0) == kq.KQ_ERR_UNSUPPORTED
        assert lib.kq_dec_norm_linear_batch(gpu_ctx.handle, w.handle, _p(x), 1024, m, _p(nwd), 1024, 1e-5, _p(y),
                                            0) == kq.KQ_ERR_UNSUPPORTED
        assert gpu_ctx.launch_count == launches
        w.free()
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 256, 1024, seed=1), 256, 1024)
    # bad norm sizes and strides
    assert lib.kq_dec_norm_linear_batch(gpu_ctx.handle, w.handle, _p(x), 1024, 4, _p(nwd), 1026, 1e-5, _p(y),
                                        0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_dec_norm_linear_batch(gpu_ctx.handle, w.handle, _p(x), 1000, 4, _p(nwd), 1000, 1e-5, _p(y),
                                        0) == kq.KQ_ERR_INVALID_ARG
    w.free()
