"""Generate the golden fixtures under tests/golden/.

An independent numpy restatement of the reference arithmetic of
xupit3r/vibrant internal/tensor, written separately from the C oracle so the
two can pin each other:

* float16ToFloat32 (internal/tensor/tensor.go:629-676), including its two
  departures from IEEE (0x8000 -> +0, every NaN -> 0x7FC00000);
* the Q4_K / Q5_K / Q6_K block decoders (block_cache.go:82-248, byte offsets
  from parseQ*_KBlock quant_q4k.go:137-157, quant_q5k.go:229-252,
  quant_q6k.go:134-156), float32 mul/sub without FMA;
* vectorDotProduct (simd_ops.go:60-78) as used by matmulSIMDSingleRow /
  matmulSIMDParallel on the pre-transposed weight, and vectorScaleAdd
  (simd_ops.go:82-98) as used by the LM-head outer product.

Run:  python tests/golden/make_golden.py   (writes *.npz next to this file)
The fixtures are small and committed; the tests only read them.
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
NAMES = {Q4_K: "q4k", Q5_K: "q5k", Q6_K: "q6k"}


def f16_to_f32_go(h: np.ndarray) -> np.ndarray:
    """float16ToFloat32, tensor.go:629-676, vectorised."""
    h = h.astype(np.uint32)
    sign = (h >> 15) & 1
    exp = (h >> 10) & 0x1F
    mant = h & 0x3FF
    out = np.zeros(h.shape, np.uint32)
    normal = (exp != 0) & (exp != 31)
    out[normal] = (sign[normal] << 31) | ((exp[normal] - 15 + 127) << 23) | (mant[normal] << 13)
    sub = (exp == 0) & (mant != 0)
    if sub.any():
        m = mant[sub].copy()
        shift = np.zeros(m.shape, np.uint32)
        for _ in range(10):
            need = (m & 0x400) == 0
            m[need] <<= 1
            shift[need] += 1
        out[sub] = (sign[sub] << 31) | ((127 - 14 - shift) << 23) | ((m & 0x3FF) << 13)
    inf = (exp == 31) & (mant == 0)
    out[inf] = (sign[inf] << 31) | 0x7F800000
    nan = (exp == 31) & (mant != 0)
    out[nan] = 0x7FC00000
    # exp == 0 and mant == 0 stays 0 (+0 for both signs)
    return out.view(np.float32)


def scales_mins(s: np.ndarray):
    """extractScalesAndMins, quant_q5k.go:97-120, for s of shape [nb, 12]."""
    s = s.astype(np.uint32)
    sc = np.stack([
        s[:, 0] & 63, ((s[:, 0] >> 6) | (s[:, 1] << 2)) & 63, ((s[:, 1] >> 4) | (s[:, 2] << 4)) & 63,
        (s[:, 2] >> 2) & 63, s[:, 3] & 63, ((s[:, 3] >> 6) | (s[:, 4] << 2)) & 63,
        ((s[:, 4] >> 4) | (s[:, 5] << 4)) & 63, (s[:, 5] >> 2) & 63], axis=1)
    m = np.stack([
        s[:, 6] & 63, ((s[:, 6] >> 6) | (s[:, 7] << 2)) & 63, ((s[:, 7] >> 4) | (s[:, 8] << 4)) & 63,
        (s[:, 8] >> 2) & 63, s[:, 9] & 63, ((s[:, 9] >> 6) | (s[:, 10] << 2)) & 63,
        ((s[:, 10] >> 4) | (s[:, 11] << 4)) & 63, (s[:, 11] >> 2) & 63], axis=1)
    return sc.astype(np.uint8), m.astype(np.uint8)


def dequant(qtype: int, data: np.ndarray) -> np.ndarray:
    bb = BLOCK_BYTES[qtype]
    b = data.reshape(-1, bb)
    nb = b.shape[0]
    idx = np.arange(256)
    with np.errstate(all="ignore"):
        if qtype in (Q4_K, Q5_K):
            d = f16_to_f32_go(b[:, 0].astype(np.uint16) | (b[:, 1].astype(np.uint16) << 8))
            dmin = f16_to_f32_go(b[:, 2].astype(np.uint16) | (b[:, 3].astype(np.uint16) << 8))
            sc, m = scales_mins(b[:, 4:16])
            qs = b[:, 16:144] if qtype == Q4_K else b[:, 48:176]
            byte = qs[:, idx // 2]
            q = np.where(idx % 2 == 0, byte & 0x0F, byte >> 4).astype(np.uint8)
            if qtype == Q5_K:
                qh = b[:, 16:48]
                hi = (qh[:, idx // 8] >> (idx % 8).astype(np.uint8)) & 1
                q = q | (hi << 4).astype(np.uint8)
            scale = (d[:, None] * sc.astype(np.float32)).astype(np.float32)  # [nb, 8]
            mn = (dmin[:, None] * m.astype(np.float32)).astype(np.float32)
            prod = (scale[:, idx // 32] * q.astype(np.float32)).astype(np.float32)
            out = (prod - mn[:, idx // 32]).astype(np.float32)
        else:
            ql = b[:, 0:128]
            qh = b[:, 128:192]
            scales = b[:, 192:208].view(np.int8)
            d = f16_to_f32_go(b[:, 208].astype(np.uint16) | (b[:, 209].astype(np.uint16) << 8))
            byte = ql[:, idx // 2]
            lo = np.where(idx % 2 == 0, byte & 0x0F, byte >> 4).astype(np.int32)
            hi = ((qh[:, idx // 4] >> ((idx % 4) * 2).astype(np.uint8)) & 3).astype(np.int32)
            q = lo | (hi << 4)
            ds = (d[:, None] * scales[:, idx // 16].astype(np.float32)).astype(np.float32)
            out = (ds * (q - 32).astype(np.float32)).astype(np.float32)
    assert out.shape == (nb, 256)
    return out.reshape(-1)


def dot8_rows(x: np.ndarray, wt: np.ndarray) -> np.ndarray:
    """vectorDotProduct(x, wt[n, :]) for every n at once (simd_ops.go:60-78)."""
    N, K = wt.shape
    s = np.zeros((N, 8), np.float32)
    full = (K // 8) * 8
    with np.errstate(all="ignore"):
        for i in range(0, full, 8):
            s += (wt[:, i:i + 8] * x[i:i + 8]).astype(np.float32)
        for i in range(full, K):
            s[:, 0] += (wt[:, i] * x[i]).astype(np.float32)
        r = s[:, 0].copy()
        for j in range(1, 8):
            r = (r + s[:, j]).astype(np.float32)
    return r


def scale_add_rows(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """matmul_simd.go:189-199 outer product with vectorScaleAdd (simd_ops.go:82-98)."""
    K, N = w.shape
    y = np.zeros(N, np.float32)
    with np.errstate(all="ignore"):
        for k in range(K):
            if x[k] == 0:
                continue
            y += (w[k] * x[k]).astype(np.float32)
    return y


def synth_weights(qtype: int, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    """Blocks with the synthetic distributions of the benchmark workloads:
    Q4_K/Q5_K d = fp16(|N(0,1)|*0.01), dmin = fp16(|N(0,1)|*0.005), other bytes
    uniform; Q6_K d = fp16(|N(0,1)|*0.002), scales int8 U[-32,31], other bytes
    uniform."""
    bb = BLOCK_BYTES[qtype]
    b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    if qtype in (Q4_K, Q5_K):
        d = (np.abs(rng.standard_normal(nblocks)) * 0.01).astype(np.float16).view(np.uint16)
        dm = (np.abs(rng.standard_normal(nblocks)) * 0.005).astype(np.float16).view(np.uint16)
        b[:, 0] = d & 0xFF
        b[:, 1] = d >> 8
        b[:, 2] = dm & 0xFF
        b[:, 3] = dm >> 8
    else:
        b[:, 192:208] = rng.integers(-32, 32, size=(nblocks, 16), dtype=np.int8).view(np.uint8)
        d = (np.abs(rng.standard_normal(nblocks)) * 0.002).astype(np.float16).view(np.uint16)
        b[:, 208] = d & 0xFF
        b[:, 209] = d >> 8
    return b.reshape(-1)


SPECIAL_F16 = [0x0000, 0x8000, 0x0001, 0x8001, 0x00FD, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF,
               0x7C00, 0xFC00, 0x7E00, 0xFE01, 0x7C01, 0x3555]


def random_blocks(qtype: int, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    """Fully random bytes (d/dmin hit subnormal, zero, Inf and NaN codes), with
    the first blocks forced onto special half codes."""
    bb = BLOCK_BYTES[qtype]
    b = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    doff = 208 if qtype == Q6_K else 0
    for i, h in enumerate(SPECIAL_F16):
        if i >= nblocks:
            break
        b[i, doff] = h & 0xFF
        b[i, doff + 1] = h >> 8
        if qtype != Q6_K:
            h2 = SPECIAL_F16[(i + 5) % len(SPECIAL_F16)]
            b[i, 2] = h2 & 0xFF
            b[i, 3] = h2 >> 8
    return b.reshape(-1)


def main() -> None:
    rng = np.random.default_rng(20261201)
    # every half-precision code, for float16ToFloat32
    codes = np.arange(65536, dtype=np.uint32)
    np.savez_compressed(os.path.join(HERE, "f16_to_f32.npz"),
                        f32_bits=f16_to_f32_go(codes.astype(np.uint16)).view(np.uint32))
    for qt in (Q4_K, Q5_K, Q6_K):
        raw = random_blocks(qt, 96, rng)
        syn = synth_weights(qt, 64, rng)
        data = np.concatenate([raw, syn])
        out = dequant(qt, data)
        np.savez_compressed(os.path.join(HERE, f"dequant_{NAMES[qt]}.npz"), blocks=data,
                            f32_bits=out.view(np.uint32))
    # matmul fixtures: decode (M == 1) through the cached transposed weight
    # (the route MatMul takes for a quantized B) and through the untransposed
    # outer product (the LM-head route); N % 256 == 128 for the latter.
    cases = [(Q4_K, 512, 768, "dot"), (Q5_K, 256, 512, "dot"), (Q6_K, 512, 384, "dot"),
             (Q6_K, 256, 640, "outer"), (Q4_K, 128, 384, "outer")]
    for qt, K, N, route in cases:
        nb = (K * N + 255) // 256
        wq = synth_weights(qt, nb, rng)
        x = rng.standard_normal(K).astype(np.float32)
        w = dequant(qt, wq)[:K * N].reshape(K, N)
        if route == "dot":
            y = dot8_rows(x, np.ascontiguousarray(w.T))
        else:
            y = scale_add_rows(x, w)
        y64 = x.astype(np.float64) @ w.astype(np.float64)
        bound = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64))
        np.savez_compressed(os.path.join(HERE, f"matmul_{NAMES[qt]}_{K}x{N}_{route}.npz"),
                            wq=wq, x=x, y=y, y64=y64, bound=bound, K=K, N=N, qtype=qt)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
