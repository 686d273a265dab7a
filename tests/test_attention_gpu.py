"""vkq_attention_decode_f32: one query token per sequence against its KV
cache, against a float64 restatement of the reference's decode attention
(computeAttention, internal/transformer/attention.go:316-363, with the cache
of :147-162, grouped KV heads of expandKVHeads :280-314 and no mask for one
query row), and against the oracle's float32 restatement of the same
arithmetic (oracle/kq_oracle.c ko_attention_decode, with ko_rope_apply and
ko_kv_append for the fused step).  Parity bar: each output within 1e-5 of
sum_j p_j |v_j|; the cache rows the fused step writes bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref(q, kc, vc, length, heads, kv_heads):
    B, H, D = q.shape
    g = heads // kv_heads
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


def _oracle_err(o, q, kc, vc, length, bound):
    """Distance of the kernel's output from the oracle's float32 restatement
    of the reference's arithmetic (kq_oracle.attention_decode), in units of
    sum_j p_j |v_j|."""
    from oracle import kq_oracle
    ora = kq_oracle.attention_decode(q, kc, vc, length).astype(np.float64)
    return float(np.max(np.abs(o - ora) / np.maximum(bound, 1e-30)))


def _run(q, kc, vc, length, shift=0):
    """shift > 0 places q and the caches that many floats past an aligned
    start, so that no lane's values form a whole vector."""
    import torch
    from vibrant_b200 import vkq
    B, H, D = q.shape
    KVH, cap = kc.shape[1], kc.shape[2]

    def dev(a):
        t = torch.empty(a.size + shift, device="cuda")
        t[shift:] = torch.from_numpy(a.reshape(-1)).cuda()
        return t[shift:]

    qt, kt, vt = dev(q), dev(kc), dev(vc)
    o = torch.full((B, H, D), float("nan"), device="cuda")
    vkq.attention_decode_f32(qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), o.data_ptr(), B, H, KVH, length, cap, D,
                             device=0)
    torch.cuda.synchronize()
    assert vkq.device_status(0) == vkq.OK
    return o.cpu().numpy()


# The cluster size (CTAs splitting one head's keys) follows from len and
# heads x batch: 1 for the shortest, 4 with a ragged last chunk for 257 and
# 300 keys, 8 for 512 and 4096 keys, and 8 chunks of 51,200 for the longest.
@pytest.mark.parametrize("B,H,KVH,D,length,cap", [
    (1, 16, 2, 128, 1, 1),          # the first token: p = 1
    (1, 16, 2, 128, 7, 64),         # 3B-class heads (16 query, 2 KV), a preallocated cache
    (1, 16, 2, 128, 300, 300),
    (1, 16, 2, 128, 512, 512),      # 3B-class heads at a 512-token context
    (2, 8, 8, 64, 257, 512),        # no grouping, two sequences
    (1, 40, 8, 128, 4096, 5000),    # 14B-class heads, a long context
    (1, 4, 1, 64, 409600, 409600),  # the longest context served
], ids=lambda v: str(v))
def test_attention_decode_matches_reference(B, H, KVH, D, length, cap):
    rng = np.random.default_rng(length + H)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, cap, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, cap, D)).astype(np.float32)
    kc[:, :, length:] = np.nan  # rows past the valid length are never read
    vc[:, :, length:] = np.nan
    o = _run(q, kc, vc, length)
    ref, bound = _ref(q, kc, vc, length, H, KVH)
    err = float(np.max(np.abs(o - ref) / np.maximum(bound, 1e-30)))
    assert err <= 1e-5, err
    assert _oracle_err(o, q, kc, vc, length, bound) <= 1e-5


@pytest.mark.parametrize("D,length", [(128, 300), (64, 1000)])
def test_attention_decode_unaligned_buffers(D, length):
    """q and the caches one float past a 16-byte boundary: scalar lane loads."""
    B, H, KVH = 1, 8, 2
    rng = np.random.default_rng(D + length)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, length, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, length, D)).astype(np.float32)
    o = _run(q, kc, vc, length, shift=1)
    ref, bound = _ref(q, kc, vc, length, H, KVH)
    err = float(np.max(np.abs(o - ref) / np.maximum(bound, 1e-30)))
    assert err <= 1e-5, err
    assert _oracle_err(o, q, kc, vc, length, bound) <= 1e-5


def test_attention_decode_peaked_scores():
    """Scores far apart (one key dominates): the max subtraction keeps exp
    finite and the result follows that key's value row."""
    B, H, KVH, D, L = 1, 2, 1, 128, 33
    rng = np.random.default_rng(3)
    q = (rng.standard_normal((B, H, D)) * 8).astype(np.float32)
    kc = rng.standard_normal((B, KVH, L, D)).astype(np.float32)
    kc[0, 0, 17] = q[0, 0] * 4  # key 17 matches head 0's query strongly
    vc = rng.standard_normal((B, KVH, L, D)).astype(np.float32)
    o = _run(q, kc, vc, L)
    ref, bound = _ref(q, kc, vc, L, H, KVH)
    assert np.isfinite(o).all()
    assert float(np.max(np.abs(o - ref) / np.maximum(bound, 1e-30))) <= 1e-5
    assert np.allclose(o[0, 0], vc[0, 0, 17], atol=1e-4)


def test_attention_decode_error_paths():
    import torch
    from vibrant_b200 import vkq
    buf = torch.zeros(1 << 16, device="cuda")
    p = buf.data_ptr()

    def call(**kw):
        a = dict(batch=1, heads=16, kv_heads=2, length=4, cache_len=8, head_dim=128)
        a.update(kw)
        vkq.attention_decode_f32(p, p, p, p, a["batch"], a["heads"], a["kv_heads"], a["length"], a["cache_len"],
                                 a["head_dim"], device=0)

    for bad, status in [(dict(kv_heads=3), vkq.ERR_INVALID_ARGUMENT), (dict(length=9), vkq.ERR_INVALID_ARGUMENT),
                        (dict(length=0), vkq.ERR_INVALID_ARGUMENT), (dict(head_dim=96), vkq.ERR_UNSUPPORTED),
                        (dict(length=409601, cache_len=409601), vkq.ERR_INVALID_ARGUMENT)]:
        with pytest.raises(vkq.VkqError) as e:
            call(**bad)
        assert e.value.status == status, bad
    assert vkq.device_status(0) == vkq.OK


def _rope_rows(x, cos_t, sin_t, pos):
    """float32 RoPE of rows x [..., D] at one position, each product and sum
    rounded on its own (RoPE.ApplyRotation, rope.go:49-124)."""
    c, s = cos_t[pos], sin_t[pos]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _run_step(q, k_new, v_new, kc, vc, length, positions, max_seq, base=1000000.0):
    import torch
    from vibrant_b200 import vkq
    B, H, D = q.shape
    KVH, cap = kc.shape[1], kc.shape[2]
    cos_t, sin_t = vkq.rope_tables(D, base, max_seq)
    t = {k: torch.from_numpy(np.ascontiguousarray(a)).cuda()
         for k, a in dict(q=q, kn=k_new, vn=v_new, kc=kc, vc=vc, cos=cos_t, sin=sin_t,
                          pos=np.asarray(positions, dtype=np.int32)).items()}
    o = torch.full((B, H, D), float("nan"), device="cuda")
    vkq.attention_rope_decode_f32(t["q"].data_ptr(), t["kn"].data_ptr(), t["vn"].data_ptr(), t["cos"].data_ptr(),
                                  t["sin"].data_ptr(), t["pos"].data_ptr(), t["kc"].data_ptr(), t["vc"].data_ptr(),
                                  o.data_ptr(), B, H, KVH, length, cap, D, max_seq, device=0)
    torch.cuda.synchronize()
    return o.cpu().numpy(), t["kc"].cpu().numpy(), t["vc"].cpu().numpy(), vkq.device_status(0), cos_t, sin_t


@pytest.mark.parametrize("B,H,KVH,D,length,cap", [
    (1, 16, 2, 128, 1, 4),          # the first token: only the new key
    (1, 16, 2, 128, 1024, 1024),    # the 3B-class decode step's shape
    (2, 8, 8, 64, 257, 300),        # no grouping, two sequences, a ragged last chunk
    (1, 40, 8, 128, 4096, 5000),    # 14B-class heads
    (1, 4, 1, 64, 204801, 204801),  # 8 chunks of 25,601 keys, the last one ragged
], ids=lambda v: str(v))
def test_attention_rope_decode_matches_reference(B, H, KVH, D, length, cap):
    """The fused step against RoPE, append and attention restated: the new
    cache rows bit for bit, every other row untouched, the output within
    1e-5 of sum p|v|."""
    from vibrant_b200 import vkq
    rng = np.random.default_rng(length * 3 + H)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
    v_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, cap, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, cap, D)).astype(np.float32)
    kc[:, :, length - 1:] = np.nan  # row len-1 is written by the call, later rows never read
    vc[:, :, length - 1:] = np.nan
    positions = [length - 1 + 3 * b for b in range(B)]
    max_seq = length + 3 * B
    o, kc_out, vc_out, st, cos_t, sin_t = _run_step(q, k_new, v_new, kc, vc, length, positions, max_seq)
    assert st == vkq.OK
    kr = np.stack([_rope_rows(k_new[b], cos_t, sin_t, positions[b]) for b in range(B)])
    qr = np.stack([_rope_rows(q[b], cos_t, sin_t, positions[b]) for b in range(B)])
    want_k, want_v = kc.copy(), vc.copy()
    want_k[:, :, length - 1] = kr
    want_v[:, :, length - 1] = v_new
    assert np.array_equal(kc_out.view(np.uint32), want_k.view(np.uint32))
    assert np.array_equal(vc_out.view(np.uint32), want_v.view(np.uint32))
    ref, bound = _ref(qr, want_k, want_v, length, H, KVH)
    err = float(np.max(np.abs(o - ref) / np.maximum(bound, 1e-30)))
    assert err <= 1e-5, err
    # the oracle's whole decode branch: RoPE, append, attention
    from oracle import kq_oracle
    ora, ora_k, ora_v = kq_oracle.attention_rope_decode(q, k_new, v_new, kc, vc, length, cos_t, sin_t, positions)
    assert np.array_equal(kc_out.view(np.uint32), ora_k.view(np.uint32))
    assert np.array_equal(vc_out.view(np.uint32), ora_v.view(np.uint32))
    assert float(np.max(np.abs(o - ora.astype(np.float64)) / np.maximum(bound, 1e-30))) <= 1e-5


def test_attention_rope_decode_bad_position():
    """A position past the tables: that sequence's output and cache rows stay
    unwritten, the other sequence is served, and the device status says so."""
    from vibrant_b200 import vkq
    B, H, KVH, D, L = 2, 8, 2, 128, 40
    rng = np.random.default_rng(11)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    k_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
    v_new = rng.standard_normal((B, KVH, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, L, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, L, D)).astype(np.float32)
    o, kc_out, vc_out, st, cos_t, sin_t = _run_step(q, k_new, v_new, kc, vc, L, [L - 1, 64], 64)
    assert st == vkq.ERR_INVALID_ARGUMENT
    assert np.isnan(o[1]).all() and np.isfinite(o[0]).all()
    assert np.array_equal(kc_out[1], kc[1]) and np.array_equal(vc_out[1], vc[1])
    assert np.array_equal(kc_out[0, :, :L - 1], kc[0, :, :L - 1])
    assert vkq.device_status(0) == vkq.OK  # the status word was cleared by the read
