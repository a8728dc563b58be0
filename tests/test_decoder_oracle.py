"""Checks of the CPU decoder restatement (oracle/decoder_oracle.py) itself.
pesti's transformer module has no unit tests of its own for these functions,
so they are pinned here by their defining formulas and invariants."""
import numpy as np

from oracle import decoder_oracle as do


def test_rmsnorm_is_x_over_rms_times_weight():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 40)).astype(np.float32)
    w = rng.standard_normal(40).astype(np.float32)
    got = do.rmsnorm(x, w, 1e-5)
    rms = np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-5)
    assert np.allclose(got, x / rms * w, rtol=1e-6, atol=1e-6)


def test_rope_is_identity_at_position_zero_and_preserves_pair_norms():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 3 * 64)).astype(np.float32)
    assert np.array_equal(do.rope(x, 3, 64, 0, 1e4), x)
    y = do.rope(x, 3, 64, 37, 1e4).reshape(2, 3, 64)
    xr = x.reshape(2, 3, 64)
    n0 = xr[..., :32] ** 2 + xr[..., 32:] ** 2
    n1 = y[..., :32] ** 2 + y[..., 32:] ** 2
    assert np.allclose(n0, n1, rtol=1e-5, atol=1e-5)


def test_rope_angles_add():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 128)).astype(np.float32)
    a = do.rope(do.rope(x, 1, 128, 5, 5e5), 1, 128, 9, 5e5)
    b = do.rope(x, 1, 128, 14, 5e5)
    assert np.allclose(a, b, rtol=1e-4, atol=1e-5)


def test_swiglu_reference_branch_and_silu():
    g = np.array([-3.0, -0.5, 0.0, 0.7, 4.0], np.float32)
    u = np.array([2.0, -1.0, 3.0, 0.5, -2.0], np.float32)
    silu = g / (1 + np.exp(-g.astype(np.float64))) * u
    quirk = np.where(g >= 0, silu, g.astype(np.float64) ** 2 / (1 + np.exp(g.astype(np.float64))) * u)
    assert np.allclose(do.swiglu(g, u, 1), silu, rtol=1e-6)
    assert np.allclose(do.swiglu(g, u, 0), quirk, rtol=1e-6)


def _tiny(final_norm):
    from pesti_b200 import decoder as dec
    return dec.DecoderConfig("t", 1, 256, 2, 1, 128, 256, 10, 1e-5, 1e4, final_norm)


def _raw_zero(cfg):
    """A model whose every quantized weight is zero (all-zero superblocks)."""
    D, hd, F, V = cfg.dim, cfg.head_dim, cfg.ffn, cfg.vocab
    q4 = lambda n, k: np.zeros((n, k // 256 * 144), np.uint8)  # noqa: E731
    q6 = lambda n, k: np.zeros((n, k // 256 * 210), np.uint8)  # noqa: E731
    raw = {(0, "q"): q4(cfg.heads * hd, 256), (0, "k"): q4(cfg.kv_heads * hd, 256),
           (0, "v"): q4(cfg.kv_heads * hd, 256), (0, "o"): q4(D, 256), (0, "gate"): q4(F, 256),
           (0, "up"): q4(F, 256), (0, "down"): q6(D, F), (0, "attn_norm"): np.ones(D, np.float32),
           (0, "ffn_norm"): np.ones(D, np.float32), "head": q6(V, 256),
           "embed": np.arange(V * D, dtype=np.float32).reshape(V, D) / (V * D),
           "final_norm": np.ones(D, np.float32)}
    return raw


def test_zero_weights_give_zero_logits_and_append_the_cache():
    cfg = _tiny(True)
    raw = _raw_zero(cfg)
    kc = [np.ones((1, 1, 8, 128), np.float32)]
    vc = [np.ones((1, 1, 8, 128), np.float32)]
    logits = do.decode_step(cfg, raw, [3], 5, kc, vc)
    assert logits.shape == (1, 10) and not np.any(logits)
    assert not np.any(kc[0][0, 0, 5]) and not np.any(vc[0][0, 0, 5])  # k = v = 0 appended at pos 5
    assert np.all(kc[0][0, 0, :5] == 1)


def test_attention_over_equal_keys_averages_the_values():
    # with every cached key equal, softmax is uniform and the output is the
    # mean of the values (layer.rs:213-239), for every query head of a group
    rng = np.random.default_rng(4)
    kc = np.tile(rng.standard_normal(64).astype(np.float32), (2, 1, 6, 1))
    vc = rng.standard_normal((2, 1, 6, 64)).astype(np.float32)
    q = rng.standard_normal((2, 3 * 64)).astype(np.float32)
    out = do.attention(q, kc, vc, 5, 3, 1, 64).reshape(2, 3, 64)
    for h in range(3):
        assert np.allclose(out[:, h], vc[:, 0, :5].mean(axis=1), rtol=1e-5, atol=1e-6)


def test_attention_picks_the_matching_key():
    # one key aligned with a large query dominates the softmax
    hd = 64
    kc = np.zeros((1, 2, 4, hd), np.float32)
    vc = np.zeros((1, 2, 4, hd), np.float32)
    kc[0, 1, 2, 0] = 1.0
    vc[0, 1, 2] = 7.0
    q = np.zeros((1, 4 * hd), np.float32)
    q[0, 2 * hd] = 400.0  # head 2 -> kv group 1 (2 query heads per kv head)
    out = do.attention(q, kc, vc, 4, 4, 2, hd).reshape(4, hd)
    assert np.allclose(out[2], 7.0, rtol=1e-6)
