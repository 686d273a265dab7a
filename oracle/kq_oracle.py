"""ctypes wrapper of the CPU oracle (oracle/libkq_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg, always as the checker or the timed CPU reference,
never as part of the product path.  The oracle restates the reference Go code
of xupit3r/vibrant internal/tensor (see kq_oracle.h for the citations).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkq_oracle.so")

Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE, "libkq_oracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        i64 = ctypes.c_int64
        L.ko_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.ko_f16_to_f32.restype = ctypes.c_float
        L.ko_f32_to_f16.argtypes = [ctypes.c_float]
        L.ko_f32_to_f16.restype = ctypes.c_uint16
        L.ko_extract_scales_mins.argtypes = [u8p, u8p, u8p]
        L.ko_dequantize.argtypes = [ctypes.c_int, u8p, i64, f32p]
        L.ko_dequant_transpose.argtypes = [ctypes.c_int, u8p, i64, i64, f32p]
        L.ko_vector_dot.argtypes = [f32p, f32p, i64]
        L.ko_vector_dot.restype = ctypes.c_float
        L.ko_matmul_single_row_t.argtypes = [f32p, f32p, i64, i64, f32p, ctypes.c_int]
        L.ko_matmul_single_row_u.argtypes = [f32p, f32p, i64, i64, f32p]
        L.ko_matmul_quant.argtypes = [ctypes.c_int, f32p, i64, i64, u8p, i64, f32p, f32p, ctypes.c_int]
        L.ko_matmul_dequant_untransposed.argtypes = [ctypes.c_int, f32p, i64, i64, u8p, i64, f32p, f32p,
                                                     ctypes.c_int]
        L.ko_matmul_quant_sequential.argtypes = [ctypes.c_int, f32p, i64, i64, u8p, i64, f32p]
        L.ko_quantize_q4k.argtypes = [f32p, i64, u8p]
        L.ko_quantize_q6k.argtypes = [f32p, i64, u8p]
        i32p = ctypes.POINTER(ctypes.c_int32)
        L.ko_rope_tables.argtypes = [i64, ctypes.c_double, i64, f32p, f32p]
        L.ko_rope_tables.restype = None
        L.ko_rope_apply.argtypes = [f32p, f32p, f32p, f32p, i32p, i64, i64, i64, i64, i64]
        L.ko_kv_append.argtypes = [f32p, f32p, i64, i64, i64, i64, i64, i64]
        L.ko_attention_decode.argtypes = [f32p, f32p, f32p, f32p, i64, i64, i64, i64, i64, i64]
        _lib = L
    return _lib


def _f32p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _u8p(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def f16_to_f32(h: int) -> float:
    return lib().ko_f16_to_f32(h)


def f16_to_f32_bits(h: int) -> int:
    return int(np.array([lib().ko_f16_to_f32(h)], dtype=np.float32).view(np.uint32)[0])


def f32_to_f16(f: float) -> int:
    return int(lib().ko_f32_to_f16(f))


def extract_scales_mins(scales12: bytes):
    s = np.frombuffer(bytes(scales12), dtype=np.uint8).copy()
    sc = np.zeros(8, np.uint8)
    m = np.zeros(8, np.uint8)
    lib().ko_extract_scales_mins(_u8p(s), _u8p(sc), _u8p(m))
    return sc, m


def dequantize(qtype: int, data: np.ndarray, nblocks: int | None = None) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    bb = BLOCK_BYTES[qtype]
    if nblocks is None:
        nblocks = data.size // bb
    out = np.empty(nblocks * 256, np.float32)
    rc = lib().ko_dequantize(qtype, _u8p(data), nblocks, _f32p(out))
    assert rc == 0
    return out


def dequant_transpose(qtype: int, data: np.ndarray, M: int, N: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(M * N, np.float32)
    rc = lib().ko_dequant_transpose(qtype, _u8p(data), M, N, _f32p(out))
    assert rc == 0
    return out.reshape(N, M)


def matmul_quant(qtype: int, a: np.ndarray, bq: np.ndarray, K: int, N: int, nthreads: int = 1) -> np.ndarray:
    """tensor.MatMul(a, quantized b): GetOrDequantTranspose then the size dispatch."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1, K)
    M = a.shape[0]
    c = np.empty((M, N), np.float32)
    wt = np.empty(N * K, np.float32)
    rc = lib().ko_matmul_quant(qtype, _f32p(a), M, K, _u8p(np.ascontiguousarray(bq, np.uint8)), N,
                               _f32p(c), _f32p(wt), nthreads)
    assert rc == 0
    return c


def matmul_dequant_untransposed(qtype: int, a: np.ndarray, bq: np.ndarray, K: int, N: int,
                                nthreads: int = 1) -> np.ndarray:
    """The LM-head route: Dequantize (untransposed) then MatMul."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1, K)
    M = a.shape[0]
    c = np.empty((M, N), np.float32)
    nb = (K * N + 255) // 256
    w = np.empty(nb * 256, np.float32)
    rc = lib().ko_matmul_dequant_untransposed(qtype, _f32p(a), M, K,
                                              _u8p(np.ascontiguousarray(bq, np.uint8)), N,
                                              _f32p(c), _f32p(w), nthreads)
    assert rc == 0
    return c


def matmul_single_row_t(x: np.ndarray, wt: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """Warm-cache decode: dot products against a cached transposed float32 weight [N, K]."""
    N, K = wt.shape
    y = np.empty(N, np.float32)
    lib().ko_matmul_single_row_t(_f32p(np.ascontiguousarray(x, np.float32)), _f32p(wt), K, N, _f32p(y),
                                 nthreads)
    return y


def matmul_single_row_u(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Warm-cache LM head: outer product against an untransposed float32 weight [K, N]."""
    K, N = w.shape
    y = np.empty(N, np.float32)
    lib().ko_matmul_single_row_u(_f32p(np.ascontiguousarray(x, np.float32)), _f32p(w), K, N, _f32p(y))
    return y


def dot_abs_bound(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """sum_k |x[m,k] * W[k,n]| in float64 -- the denominator of the matmul error metric."""
    return np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64))


def quantize(qtype: int, values: np.ndarray) -> np.ndarray:
    """The reference's test quantizer for Q4_K or Q6_K (QuantizeQ4_K /
    QuantizeQ6_K), as raw super-block bytes."""
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    nb = (v.size + 255) // 256
    out = np.zeros(nb * BLOCK_BYTES[qtype], np.uint8)
    fn = {Q4_K: lib().ko_quantize_q4k, Q6_K: lib().ko_quantize_q6k}[qtype]
    assert fn(_f32p(v), v.size, _u8p(out)) == 0
    return out


def matmul_quant_sequential(qtype: int, a: np.ndarray, bq: np.ndarray, K: int, N: int) -> np.ndarray:
    """MatMulQ5K / MatMulQ6K (the reference's fused route): sequential-k
    float32 sums of a[i,k] * deq(k*N + j)."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1, K)
    c = np.empty((a.shape[0], N), np.float32)
    rc = lib().ko_matmul_quant_sequential(qtype, _f32p(a), a.shape[0], K,
                                          _u8p(np.ascontiguousarray(bq, np.uint8)), N, _f32p(c))
    assert rc == 0
    return c


# ---- decode attention and RoPE (internal/transformer) -----------------------

def rope_tables(head_dim: int, freq_base: float, max_seq: int):
    """NewRoPE's cos and sin tables [max_seq][head_dim/2] (rope.go:19-43)."""
    half = head_dim // 2
    c = np.empty((max_seq, half), np.float32)
    s = np.empty((max_seq, half), np.float32)
    lib().ko_rope_tables(head_dim, float(freq_base), max_seq, _f32p(c), _f32p(s))
    return c, s


def rope_apply(x: np.ndarray, cos_t: np.ndarray, sin_t: np.ndarray, positions) -> np.ndarray:
    """RoPE.ApplyRotation on x [batch][heads][seq][head_dim] (rope.go:49-124)."""
    x = np.ascontiguousarray(x, np.float32)
    B, H, S, D = x.shape
    pos = np.ascontiguousarray(np.asarray(positions, np.int32))
    assert pos.size == S
    out = np.empty_like(x)
    rc = lib().ko_rope_apply(_f32p(x), _f32p(out), _f32p(np.ascontiguousarray(cos_t, np.float32)),
                             _f32p(np.ascontiguousarray(sin_t, np.float32)),
                             pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), B, H, S, D, cos_t.shape[0])
    if rc != 0:
        raise ValueError("position outside the RoPE tables")
    return out


def kv_append(cache: np.ndarray, new_rows: np.ndarray, row0: int) -> None:
    """concatenateSeqDim (attention.go:529-569) in place: new_rows
    [batch][kv_heads][n][D] become rows row0 .. row0+n-1 of cache
    [batch][kv_heads][cache_len][D]."""
    assert cache.dtype == np.float32 and cache.flags.c_contiguous
    new_rows = np.ascontiguousarray(new_rows, np.float32)
    B, KVH, cap, D = cache.shape
    rc = lib().ko_kv_append(_f32p(cache), _f32p(new_rows), B, KVH, cap, row0, new_rows.shape[2], D)
    if rc != 0:
        raise ValueError("rows do not fit the cache")


def attention_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, length: int) -> np.ndarray:
    """computeAttention (attention.go:316-363) for one query row per (batch,
    head) against rows 0 .. length-1 of the caches, grouped KV heads expanded
    as expandKVHeads does.  q [batch][heads][D], caches
    [batch][kv_heads][cache_len][D]; returns [batch][heads][D]."""
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.float32)
    vc = np.ascontiguousarray(vc, np.float32)
    B, H, D = q.shape
    KVH, cap = kc.shape[1], kc.shape[2]
    out = np.empty((B, H, D), np.float32)
    rc = lib().ko_attention_decode(_f32p(q), _f32p(kc), _f32p(vc), _f32p(out), B, H, KVH, length, cap, D)
    assert rc == 0, rc
    return out


def attention_rope_decode(q, k_new, v_new, kc, vc, length: int, cos_t, sin_t, positions):
    """Attention.Forward's decode branch after the projections
    (attention.go:141-172) for one new token per sequence: RoPE on q and
    k_new at positions[b], the rotated k_new and v_new appended as row
    length-1 of copies of the caches, attention over rows 0 .. length-1.
    Returns (out, k_cache, v_cache)."""
    B, H, D = q.shape
    KVH = k_new.shape[1]
    qr = np.stack([rope_apply(q[b][None, :, None, :], cos_t, sin_t, [positions[b]])[0, :, 0] for b in range(B)])
    kr = np.stack([rope_apply(k_new[b][None, :, None, :], cos_t, sin_t, [positions[b]])[0, :, 0]
                   for b in range(B)])
    kc = np.array(kc, np.float32, copy=True, order="C")
    vc = np.array(vc, np.float32, copy=True, order="C")
    kv_append(kc, kr.reshape(B, KVH, 1, D), length - 1)
    kv_append(vc, np.asarray(v_new, np.float32).reshape(B, KVH, 1, D), length - 1)
    return attention_decode(qr, kc, vc, length), kc, vc
