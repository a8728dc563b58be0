"""The persistent decode-step kernel (kq_step_*) driven directly through the
C ABI: a hand-built program of linears against the oracle, and the builder's
argument checks.  The decoder tests (test_gpu_decoder.py) run it on whole
models."""
import ctypes

import numpy as np
import pytest

import oracle
from pesti_b200 import decoder as dec
from pesti_b200 import kq, synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-3
OT = {kq.KQ_GGUF_Q4_K: oracle.GGUF_Q4_K, kq.KQ_GGUF_Q6_K: oracle.GGUF_Q6_K}


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def rmsnorm(x, w, eps):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x) + eps) * w


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.fixture
def step_env(gpu_ctx):
    lib = dec._bind(gpu_ctx.lib)
    h = ctypes.c_void_p()
    assert lib.kq_step_create(gpu_ctx.handle, None, ctypes.byref(h)) == kq.KQ_OK
    yield lib, h
    lib.kq_step_destroy(h)


def test_a_program_of_linears_matches_the_oracle(gpu_ctx, step_env):
    """y1 = rmsnorm(x) . W1 (Q4_K), y2 = y1 . W2 (Q6_K, after a grid barrier),
    then W3 (Q4_K) as a partial residual update of h: h2 = h + y2 . W3, and
    y4 = rmsnorm(h2) . W4 (Q6_K) with h2 also written out."""
    import torch
    lib, h = step_env
    D, F, eps = 1024, 2816, 1e-5
    shapes = [(kq.KQ_GGUF_Q4_K, F, D), (kq.KQ_GGUF_Q6_K, 768, F), (kq.KQ_GGUF_Q4_K, D, 768),
              (kq.KQ_GGUF_Q6_K, 520, D)]
    raws = [synthetic.gguf_weight(t, n, k, seed=i + 3) for i, (t, n, k) in enumerate(shapes)]
    ws = [kq.Weight(gpu_ctx, t, r, n, k) for (t, n, k), r in zip(shapes, raws)]
    rng = np.random.default_rng(5)
    x = rng.standard_normal(D).astype(np.float32)
    nw1 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    nw4 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    hv = rng.standard_normal(D).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    xd, n1, n4, hd = dev(x), dev(nw1), dev(nw4), dev(hv)
    y1 = torch.zeros(F, device="cuda")
    y2 = torch.zeros(768, device="cuda")
    h2 = torch.zeros(D, device="cuda")
    y4 = torch.zeros(520, device="cuda")
    chk = lambda rc, what: gpu_ctx.check(rc, what)  # noqa: E731
    chk(lib.kq_step_linear(h, ws[0].handle, dec.STEP_IN_NORM, ptr(xd), ptr(n1), D, eps, None, dec.STEP_OUT_STORE,
                           ptr(y1), 0), "norm -> store")
    chk(lib.kq_step_linear(h, ws[1].handle, dec.STEP_IN_PLAIN, ptr(y1), None, 0, 0.0, None, dec.STEP_OUT_STORE,
                           ptr(y2), 0), "plain -> store")
    chk(lib.kq_step_linear(h, ws[2].handle, dec.STEP_IN_PLAIN, ptr(y2), None, 0, 0.0, ptr(hd), dec.STEP_OUT_PARTIAL,
                           None, 0), "plain -> partial update of h")
    chk(lib.kq_step_linear(h, ws[3].handle, dec.STEP_IN_RESIDUAL_NORM, None, ptr(n4), D, eps, ptr(h2),
                           dec.STEP_OUT_STORE, ptr(y4), 0), "residual + norm -> store")
    for _ in range(3):  # repeated runs: the sync words and the exchange epoch carry over
        y4.zero_()
        chk(lib.kq_step_run(h, 0, kq.KQ_SYNC), "kq_step_run")
        g1, g2, gh, g4 = (t.cpu().numpy() for t in (y1, y2, h2, y4))
        # every stage against the oracle on the input the device stage actually saw
        a1 = rmsnorm(x, nw1, eps).astype(np.float32)
        assert rel_err(g1, oracle.gguf_linear(OT[shapes[0][0]], raws[0], F, D, a1)) <= TOL
        assert rel_err(g2, oracle.gguf_linear(OT[shapes[1][0]], raws[1], 768, F, g1)) <= TOL
        upd = oracle.gguf_linear(OT[shapes[2][0]], raws[2], D, 768, g2).reshape(-1)
        assert rel_err(gh, hv.astype(np.float64) + upd) <= TOL
        a4 = rmsnorm(gh, nw4, eps).astype(np.float32)
        assert rel_err(g4, oracle.gguf_linear(OT[shapes[3][0]], raws[3], 520, D, a4)) <= TOL
    for w in ws:
        w.free()


def test_the_builder_rejects_bad_programs(gpu_ctx, step_env):
    import torch
    lib, h = step_env
    w = kq.Weight(gpu_ctx, kq.KQ_GGUF_Q4_K, synthetic.q4_k_weight(64, 512, seed=1), 64, 512)
    wl = kq.Weight(gpu_ctx, kq.KQ_PESTI_Q4_K_LEGACY, synthetic.legacy_weight(112, 8, 32, seed=1), 8, 32)
    x = torch.zeros(512, device="cuda")
    y = torch.zeros(64, device="cuda")
    h2 = torch.zeros(512, device="cuda")
    # nothing to run yet
    assert lib.kq_step_run(h, 0, 0) == kq.KQ_ERR_STATE
    # a residual input with no partial output before it
    assert lib.kq_step_linear(h, w.handle, dec.STEP_IN_RESIDUAL, None, None, 64, 0.0, ptr(h2),
                              dec.STEP_OUT_STORE, ptr(y), 0) == kq.KQ_ERR_STATE
    # weights outside the step kernel's types, bad modes, misaligned input
    assert lib.kq_step_linear(h, wl.handle, dec.STEP_IN_PLAIN, ptr(x), None, 0, 0.0, None, dec.STEP_OUT_STORE,
                              ptr(y), 0) == kq.KQ_ERR_UNSUPPORTED
    assert lib.kq_step_linear(h, w.handle, 9, ptr(x), None, 0, 0.0, None, dec.STEP_OUT_STORE, ptr(y),
                              0) == kq.KQ_ERR_INVALID_ARG
    assert lib.kq_step_linear(h, w.handle, dec.STEP_IN_PLAIN, ctypes.c_void_p(x.data_ptr() + 4), None, 0, 0.0, None,
                              dec.STEP_OUT_STORE, ptr(y), 0) == kq.KQ_ERR_INVALID_ARG
    # a partial output that nothing consumes cannot run on one GPU
    assert lib.kq_step_linear(h, w.handle, dec.STEP_IN_PLAIN, ptr(x), None, 0, 0.0, None, dec.STEP_OUT_PARTIAL,
                              None, 0) == kq.KQ_OK
    assert lib.kq_step_run(h, 0, 0) == kq.KQ_ERR_STATE
    # attention shapes the kernel does not serve
    kc = torch.zeros(2 * 16 * 96, dtype=torch.float16, device="cuda")
    assert lib.kq_step_attention(h, ptr(x), ptr(kc), ptr(kc), ptr(x), 4, 2, 96, 16, 1e4) == kq.KQ_ERR_UNSUPPORTED
    assert lib.kq_step_attention(h, ptr(x), ptr(kc), ptr(kc), ptr(x), 36, 2, 64, 16, 1e4) == kq.KQ_ERR_UNSUPPORTED
    w.free()
    wl.free()
