"""Verify-path attention kernel against a float64 restatement of src/model.rs:261-282 (GPU).

The reference attends in f32 over an f32 cache; the CUDA path stores K/V in f16. Both sides here
use the same f16-rounded keys and values, so the kernel must agree with the f64 restatement to
f32 accumulation accuracy. RoPE follows src/kernels.rs:242-252 (rotate-half, theta 1e6, inv_freq
computed in f64 then rounded to f32, angle = position as f32 times inv_freq).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rope_tab(hd, n, theta=1e6):
    half = hd // 2
    inv = (1.0 / np.power(theta, np.arange(half, dtype=np.float64) * 2 / hd)).astype(np.float32)
    ang = np.arange(n, dtype=np.float32)[:, None] * inv[None, :]
    return np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))


def rotate(x, c, s):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def reference(heads, kvh, hd, pos0, qkv, kc, vc):
    M = qkv.shape[0]
    H, KV = heads * hd, kvh * hd
    cos, sin = rope_tab(hd, pos0 + M)
    q = qkv[:, :H].astype(np.float64).reshape(M, heads, hd)
    k = qkv[:, H:H + KV].astype(np.float64).reshape(M, kvh, hd)
    v = qkv[:, H + KV:].astype(np.float64).reshape(M, kvh, hd)
    pos = pos0 + np.arange(M)
    q = rotate(q, cos[pos][:, None, :], sin[pos][:, None, :])
    k = rotate(k, cos[pos][:, None, :], sin[pos][:, None, :])
    k = k.astype(np.float32).astype(np.float16).astype(np.float64)  # the cache stores f16
    v = v.astype(np.float32).astype(np.float16).astype(np.float64)
    K = np.concatenate([kc.astype(np.float64), k.transpose(1, 0, 2)], axis=1) if pos0 else k.transpose(1, 0, 2)
    V = np.concatenate([vc.astype(np.float64), v.transpose(1, 0, 2)], axis=1) if pos0 else v.transpose(1, 0, 2)
    out = np.zeros((M, heads, hd))
    g = heads // kvh
    for t in range(M):
        ctx = pos0 + t + 1
        for h in range(heads):
            sc = K[h // g, :ctx] @ q[t, h] / np.sqrt(hd)
            p = np.exp(sc - sc.max())
            out[t, h] = (p / p.sum()) @ V[h // g, :ctx]
    return out.reshape(M, H)


@pytest.mark.parametrize("heads,kvh,hd,pos0,M", [(14, 2, 64, 0, 9), (14, 2, 64, 100, 1), (14, 2, 64, 700, 9),
                                                 (16, 2, 128, 300, 5), (4, 2, 16, 65, 33), (14, 2, 64, 4000, 16),
                                                 (14, 2, 64, 20000, 9), (16, 2, 128, 9000, 3)])
def test_attention_kernel_matches_float64_restatement(heads, kvh, hd, pos0, M):
    import layerstream_b200 as ls

    rng = np.random.default_rng(pos0 * 7 + M)
    qkv = rng.standard_normal((M, (heads + 2 * kvh) * hd)).astype(np.float32)
    kc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
    vc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
    got, _ = ls.attention(heads, kvh, hd, pos0, qkv, kc, vc)
    want = reference(heads, kvh, hd, pos0, qkv, kc, vc)
    assert np.max(np.abs(got - want)) < 2e-4 * (1 + np.max(np.abs(want)))


def test_timed_attention_over_cache_replicas_returns_the_same_output():
    """The timing loop runs the kernel over replicas of the cache: the output stays the untimed one."""
    import layerstream_b200 as ls

    heads, kvh, hd, pos0, M = 14, 2, 64, 3000, 9
    rng = np.random.default_rng(11)
    qkv = rng.standard_normal((M, (heads + 2 * kvh) * hd)).astype(np.float32)
    kc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
    vc = rng.standard_normal((kvh, pos0, hd)).astype(np.float16)
    once, _ = ls.attention(heads, kvh, hd, pos0, qkv, kc, vc)
    timed, ms = ls.attention(heads, kvh, hd, pos0, qkv, kc, vc, iters=4)
    assert ms > 0
    np.testing.assert_array_equal(once, timed)


def test_attention_rejects_bad_shapes():
    import layerstream_b200 as ls

    with pytest.raises(ls.LayerstreamError):
        ls.attention(14, 3, 64, 0, np.zeros((1, (14 + 6) * 64), np.float32))
    with pytest.raises(ls.LayerstreamError):
        ls.attention(14, 2, 48, 0, np.zeros((1, (14 + 4) * 48), np.float32))
