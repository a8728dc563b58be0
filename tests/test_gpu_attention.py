"""Decode attention on the GPU through the C ABI (kq_dec_attention,
kq_dec_rope_attention) against the oracle's restatement of pesti's
Attention::forward_with_cache (oracle/decoder_oracle.py): f16 caches, grouped
query heads, sequences of one to several 64-position tiles per split, and
the split counts the kernel picks for small and large batches."""
import ctypes

import numpy as np
import pytest

from oracle import decoder_oracle
from pesti_b200 import decoder as dec

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max|out - ref| / max|ref|: both products carry f32-level precision


def rel_err(y, ref):
    y = np.asarray(y, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _scratch(lib, ctx, batch, hq, hkv, hd, max_seq):
    import torch
    n = lib.kq_dec_attention_scratch(ctx.handle, batch, hq, hkv, hd, max_seq)
    return torch.zeros(max(n // 4, 1), dtype=torch.float32, device="cuda"), n


@pytest.mark.parametrize("hd,hq,hkv,batch,length", [
    (128, 32, 8, 1, 2049),   # Llama-shaped, many splits of one or two tiles
    (128, 32, 8, 32, 2049),  # batch 32: one split of 33 tiles per (token, kv head)
    (64, 14, 2, 1, 513),     # Qwen-shaped group of 7
    (64, 8, 8, 3, 1),        # one position
    (128, 16, 2, 2, 130),    # group of 8, a ragged last tile
    (64, 4, 4, 1, 64),       # exactly one tile
])
def test_attention_matches_the_oracle(gpu_ctx, hd, hq, hkv, batch, length):
    import torch
    lib = dec._bind(gpu_ctx.lib)
    rng = np.random.default_rng(hd + hq + batch + length)
    max_seq = length + 3
    q = rng.standard_normal((batch, hq * hd)).astype(np.float32) * 2.0
    kc = rng.standard_normal((batch, hkv, max_seq, hd)).astype(np.float16)
    vc = rng.standard_normal((batch, hkv, max_seq, hd)).astype(np.float16)
    qd = torch.from_numpy(q).cuda()
    kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    out = torch.full((batch, hq * hd), float("nan"), device="cuda")
    scratch, nbytes = _scratch(lib, gpu_ctx, batch, hq, hkv, hd, max_seq)
    ref = decoder_oracle.attention(q, kc.astype(np.float32), vc.astype(np.float32), length, hq, hkv, hd)
    for _ in range(2):  # the second call finds the arrival counters left at zero
        gpu_ctx.check(lib.kq_dec_attention(gpu_ctx.handle, _p(qd), hq * hd, _p(kd), _p(vd), _p(out), hq * hd,
                                           batch, hq, hkv, hd, length, max_seq, _p(scratch), nbytes),
                      "kq_dec_attention")
        gpu_ctx.synchronize()
        assert rel_err(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("hd,hq,hkv,batch,pos", [(128, 32, 8, 2, 700), (64, 14, 2, 1, 64), (128, 8, 2, 1, 0)])
def test_rope_attention_matches_rope_append_then_attention(gpu_ctx, hd, hq, hkv, batch, pos):
    """The fused kernel (rotate q, append the rotated k and v of position pos,
    attend over [0, pos]) against the separate append kernel followed by the
    plain attention: the same caches and outputs."""
    import torch
    lib = dec._bind(gpu_ctx.lib)
    rng = np.random.default_rng(pos + hd)
    max_seq = pos + 5
    ld = (hq + 2 * hkv) * hd
    qkv = torch.from_numpy(rng.standard_normal((batch, ld)).astype(np.float32)).cuda()
    k0 = torch.from_numpy(rng.standard_normal((batch, hkv, max_seq, hd)).astype(np.float16)).cuda()
    v0 = torch.from_numpy(rng.standard_normal((batch, hkv, max_seq, hd)).astype(np.float16)).cuda()
    theta = 5e5
    # fused
    k1, v1 = k0.clone(), v0.clone()
    out1 = torch.empty((batch, hq * hd), device="cuda")
    s1, n1 = _scratch(lib, gpu_ctx, batch, hq, hkv, hd, max_seq)
    gpu_ctx.check(lib.kq_dec_rope_attention(gpu_ctx.handle, _p(qkv), ld, _p(k1), _p(v1), _p(out1), hq * hd, batch,
                                            hq, hkv, hd, pos, max_seq, theta, _p(s1), n1), "kq_dec_rope_attention")
    # separate
    k2, v2, q2 = k0.clone(), v0.clone(), qkv.clone()
    out2 = torch.empty((batch, hq * hd), device="cuda")
    s2, n2 = _scratch(lib, gpu_ctx, batch, hq, hkv, hd, max_seq)
    gpu_ctx.check(lib.kq_dec_rope_append(gpu_ctx.handle, _p(q2), ld, _p(k2), _p(v2), batch, hq, hkv, hd, pos,
                                         max_seq, theta), "kq_dec_rope_append")
    gpu_ctx.check(lib.kq_dec_attention(gpu_ctx.handle, _p(q2), ld, _p(k2), _p(v2), _p(out2), hq * hd, batch, hq,
                                       hkv, hd, pos + 1, max_seq, _p(s2), n2), "kq_dec_attention")
    gpu_ctx.synchronize()
    # the appended rows: the same rotation in both kernels (up to one f16 rounding step)
    assert torch.allclose(k1.float(), k2.float(), rtol=1e-3, atol=1e-3)
    assert torch.equal(v1, v2)
    assert rel_err(out1.cpu().numpy(), out2.cpu().numpy()) <= TOL
