"""The oracle's restatement of decode attention and RoPE (oracle/kq_oracle.c,
ko_rope_* / ko_kv_append / ko_attention_decode), pinned on the CPU:

* against the reference's own test cases where they hold values:
  TestConcatenateSeqDim (internal/transformer/transformer_test.go:703-760)
  and the shape case of TestRoPE_ApplyRotation (:147-164); the reference's
  attention tests check shapes and cache lengths only (:285-378, :562-631),
  which the cache-growth case below mirrors;
* against independent numpy restatements: float32 RoPE bit for bit, and
  attention within 1e-6 of sum_j p_j |v_j| of a float64 computation;
* through properties the arithmetic fixes exactly: one key gives its value
  row, position 0 is the identity, grouped KV heads equal expanded ones.
"""
import numpy as np
import pytest

from oracle import kq_oracle as ko


def _rope_np(x, cos_t, sin_t, positions):
    c = cos_t[np.asarray(positions)]
    s = sin_t[np.asarray(positions)]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _attention_f64(q, kc, vc, length):
    B, H, D = q.shape
    g = H // kc.shape[1]
    out = np.empty((B, H, D))
    bound = np.empty((B, H, D))
    scale = np.float64(np.float32(1.0 / np.sqrt(D)))
    for b in range(B):
        for h in range(H):
            k = kc[b, h // g, :length].astype(np.float64)
            v = vc[b, h // g, :length].astype(np.float64)
            s = (k @ q[b, h].astype(np.float64)) * scale
            p = np.exp(s - s.max())
            p /= p.sum()
            out[b, h] = p @ v
            bound[b, h] = p @ np.abs(v)
    return out, bound


@pytest.mark.parametrize("head_dim,base,max_seq", [(64, 10000.0, 2048), (128, 1000000.0, 4096)])
def test_rope_tables_match_numpy(head_dim, base, max_seq):
    """NewRoPE's tables from the C restatement and from numpy: the same
    float64 formula, so the float32 entries agree except where the two
    libms round a double differently (at most one float32 step)."""
    from vibrant_b200 import vkq
    c1, s1 = ko.rope_tables(head_dim, base, max_seq)
    c2, s2 = vkq.rope_tables(head_dim, base, max_seq)
    for a, b in ((c1, c2), (s1, s2)):
        ulps = np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))
        assert int(ulps.max()) <= 1
        assert np.count_nonzero(ulps) <= a.size // 1000
    assert np.all(c1[0] == 1.0) and np.all(s1[0] == 0.0)


def test_rope_reference_shape_case():
    """TestRoPE_ApplyRotation: RoPE(64, 10000, 2048) on a zero [1, 4, 3, 64]
    tensor at positions 0, 1, 2 keeps the shape (and the zeros)."""
    cos_t, sin_t = ko.rope_tables(64, 10000.0, 2048)
    x = np.zeros((1, 4, 3, 64), np.float32)
    out = ko.rope_apply(x, cos_t, sin_t, [0, 1, 2])
    assert out.shape == x.shape
    assert not out.any()


@pytest.mark.parametrize("shape,positions", [((1, 4, 3, 64), [0, 1, 2]), ((2, 3, 5, 128), [7, 0, 2047, 100, 1]),
                                             ((1, 2, 1, 2), [5])])
def test_rope_apply_bit_exact_with_numpy(shape, positions):
    cos_t, sin_t = ko.rope_tables(shape[3], 10000.0, 2048)
    x = (np.random.default_rng(sum(shape)).standard_normal(shape) * 3).astype(np.float32)
    out = ko.rope_apply(x, cos_t, sin_t, positions)
    assert np.array_equal(out.view(np.uint32), _rope_np(x, cos_t, sin_t, positions).view(np.uint32))
    if positions[0] == 0:  # cos 1, sin 0: the identity, bit for bit
        assert np.array_equal(out[:, :, 0].view(np.uint32), x[:, :, 0].view(np.uint32))


def test_rope_position_outside_tables():
    cos_t, sin_t = ko.rope_tables(64, 10000.0, 16)
    with pytest.raises(ValueError):
        ko.rope_apply(np.ones((1, 1, 1, 64), np.float32), cos_t, sin_t, [16])


def test_kv_append_reference_values():
    """TestConcatenateSeqDim: cached [1, 2, 3, 4] holding s*10 + d, two new
    rows holding 100 + s*10 + d; the result holds the cached rows, then the
    new ones, in both heads."""
    cache = np.zeros((1, 2, 5, 4), np.float32)
    new = np.zeros((1, 2, 2, 4), np.float32)
    for h in range(2):
        for s in range(3):
            for d in range(4):
                cache[0, h, s, d] = s * 10 + d
        for s in range(2):
            for d in range(4):
                new[0, h, s, d] = 100 + s * 10 + d
    ko.kv_append(cache, new, 3)
    for h in range(2):
        for s in range(3):
            for d in range(4):
                assert cache[0, h, s, d] == s * 10 + d
        for s in range(2):
            for d in range(4):
                assert cache[0, h, 3 + s, d] == 100 + s * 10 + d
    with pytest.raises(ValueError):
        ko.kv_append(cache, new, 4)  # past the preallocated length


@pytest.mark.parametrize("B,H,KVH,D,length", [(1, 16, 2, 128, 300), (2, 8, 8, 64, 257), (1, 4, 1, 64, 5000),
                                              (1, 40, 8, 128, 64), (1, 2, 1, 128, 2)])
def test_attention_decode_vs_float64(B, H, KVH, D, length):
    rng = np.random.default_rng(length + H)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, length + 3, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, length + 3, D)).astype(np.float32)
    kc[:, :, length:] = np.nan  # rows past the valid length are never read
    vc[:, :, length:] = np.nan
    out = ko.attention_decode(q, kc, vc, length)
    ref, bound = _attention_f64(q, kc, vc, length)
    err = float(np.max(np.abs(out - ref) / np.maximum(bound, 1e-30)))
    assert err <= 1e-6, err


def test_attention_one_key_gives_its_value_row():
    """One cached key: softmax of one score is exactly 1, so the output is
    the value row bit for bit (the first decode step)."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 4, 64)).astype(np.float32)
    kc = rng.standard_normal((1, 2, 1, 64)).astype(np.float32)
    vc = rng.standard_normal((1, 2, 1, 64)).astype(np.float32)
    out = ko.attention_decode(q, kc, vc, 1)
    for h in range(4):
        assert np.array_equal(out[0, h], vc[0, h // 2, 0])


def test_attention_grouped_heads_equal_expanded():
    """expandKVHeads: 8 query heads over 2 KV heads give the same bits as the
    same caches copied out to 8 KV heads."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 8, 128)).astype(np.float32)
    kc = rng.standard_normal((1, 2, 40, 128)).astype(np.float32)
    vc = rng.standard_normal((1, 2, 40, 128)).astype(np.float32)
    grouped = ko.attention_decode(q, kc, vc, 40)
    expanded = ko.attention_decode(q, np.repeat(kc, 4, axis=1), np.repeat(vc, 4, axis=1), 40)
    assert np.array_equal(grouped.view(np.uint32), expanded.view(np.uint32))


def test_attention_cache_growth():
    """As TestAttention_CacheOperations: three cached tokens, then one decode
    step at a time; each step leaves the earlier rows as they were, adds one
    row, and attends over every row so far."""
    rng = np.random.default_rng(3)
    B, H, KVH, D, cap = 1, 4, 4, 32, 8
    cos_t, sin_t = ko.rope_tables(D, 10000.0, 64)
    kc = np.zeros((B, KVH, cap, D), np.float32)
    vc = np.zeros((B, KVH, cap, D), np.float32)
    k3 = rng.standard_normal((B, KVH, 3, D)).astype(np.float32)
    ko.kv_append(kc, ko.rope_apply(k3, cos_t, sin_t, [0, 1, 2]), 0)
    ko.kv_append(vc, rng.standard_normal((B, KVH, 3, D)).astype(np.float32), 0)
    for length in (4, 5):
        q = rng.standard_normal((B, H, D)).astype(np.float32)
        k_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
        v_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
        out, kc2, vc2 = ko.attention_rope_decode(q, k_new, v_new, kc, vc, length, cos_t, sin_t, [length - 1])
        assert np.array_equal(kc2[:, :, :length - 1], kc[:, :, :length - 1])
        assert np.array_equal(vc2[:, :, length - 1], v_new)
        want_k = _rope_np(k_new[:, :, None, :], cos_t, sin_t, [length - 1])[:, :, 0]
        assert np.array_equal(kc2[:, :, length - 1].view(np.uint32), want_k.view(np.uint32))
        qr = _rope_np(q[:, :, None, :], cos_t, sin_t, [length - 1])[:, :, 0]
        ref, bound = _attention_f64(qr, kc2, vc2, length)
        assert float(np.max(np.abs(out - ref) / bound)) <= 1e-6
        kc, vc = kc2, vc2
