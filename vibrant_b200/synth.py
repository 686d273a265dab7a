"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark workloads (there is no model file or dataset on this path):

* Q4_K / Q5_K super-blocks: d = fp16(|N(0,1)| * 0.01), dmin =
  fp16(|N(0,1)| * 0.005); the 12 packed scale/min bytes, the Q5_K high-bit
  bytes and the 4-bit quant bytes uniform in [0, 255].
* Q6_K super-blocks: ql and qh bytes uniform, the 16 int8 sub-block scales
  uniform in [-32, 31], d = fp16(|N(0,1)| * 0.002).
* activations x ~ N(0, 1), float32.

Block layouts: internal/tensor/quant_q4k.go:137-157, quant_q5k.go:229-252,
quant_q6k.go:134-156 of xupit3r/vibrant.
"""
from __future__ import annotations

import numpy as np

Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


def n_blocks(K: int, N: int) -> int:
    return (K * N + 255) // 256


def weights(qtype: int, K: int, N: int, seed: int) -> np.ndarray:
    """uint8 array of ceil(K*N/256) super-blocks."""
    nb = n_blocks(K, N)
    bb = BLOCK_BYTES[qtype]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    if qtype in (Q4_K, Q5_K):
        d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.01)).astype(np.float16)
        dm = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.005)).astype(np.float16)
        b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        b[:, 2:4] = dm.view(np.uint8).reshape(nb, 2)
    else:
        b[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
        d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.002)).astype(np.float16)
        b[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def random_bytes(qtype: int, K: int, N: int, seed: int) -> np.ndarray:
    """Fully random super-block bytes (scales reach subnormal, Inf and NaN codes)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=n_blocks(K, N) * BLOCK_BYTES[qtype], dtype=np.uint8)


def activations(M: int, K: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32)


# The benchmark workloads, by name.
WORKLOADS = {
    # decode GEMV of the 3B FFN gate/up projection, hidden 2048 -> FFN 11008
    "q4k_gemv_2048x11008": dict(qtype=Q4_K, K=2048, N=11008, M=1, seed=1),
    # vocabulary projection (LM head), hidden 2048 -> vocab 151936
    "q6k_vocab_gemv_2048x151936": dict(qtype=Q6_K, K=2048, N=151936, M=1, seed=2),
    # prefill GEMM of the FFN projection, 512 tokens
    "q5k_prefill_gemm_512x2048x11008": dict(qtype=Q5_K, K=2048, N=11008, M=512, seed=3),
}
