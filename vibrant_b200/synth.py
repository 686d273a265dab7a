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


def weights_device(qtype: int, K: int, N: int, seed: int, device):
    """Super-blocks with the same value distributions as `weights`, drawn on
    the GPU with torch's generator (for model-scale workloads whose GBs of
    weights would take minutes to draw on the host); returns a uint8 tensor."""
    import torch
    nb = n_blocks(K, N)
    bb = BLOCK_BYTES[qtype]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    b = torch.randint(0, 256, (nb, bb), dtype=torch.uint8, generator=g, device=device)
    if qtype in (Q4_K, Q5_K):
        d = (torch.randn(nb, generator=g, device=device).abs() * 0.01).half()
        dm = (torch.randn(nb, generator=g, device=device).abs() * 0.005).half()
        b[:, 0:2] = d.view(torch.uint8).view(nb, 2)
        b[:, 2:4] = dm.view(torch.uint8).view(nb, 2)
    else:
        b[:, 192:208] = torch.randint(-32, 32, (nb, 16), dtype=torch.int8, generator=g,
                                      device=device).view(torch.uint8)
        d = (torch.randn(nb, generator=g, device=device).abs() * 0.002).half()
        b[:, 208:210] = d.view(torch.uint8).view(nb, 2)
    return b.view(-1)


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

# Whole-model decode workloads: the linear layers of one decode step.
# 3B class: 36 layers, hidden 2048, 16 query / 2 KV heads of dim 128, FFN
# 11008, vocabulary 151936; q/k/v/o/gate/up Q4_K, down and the LM head Q6_K.
MODEL_3B = dict(layers=36, hidden=2048, q_out=16 * 128, kv_out=2 * 128, ffn=11008, vocab=151936,
                q4=Q4_K, down=Q6_K, head=Q6_K)
# 14B/32B class batched decode: hidden 5120, FFN 27648, 64 layers, 40 query /
# 8 KV heads of dim 128, every linear layer Q4_K.
MODEL_14B = dict(layers=64, hidden=5120, q_out=40 * 128, kv_out=8 * 128, ffn=27648)


def layer_shapes(model: dict) -> list[tuple[str, int, int, int]]:
    """(role, qtype, K, N) of the linear layers of one transformer layer, in
    the order the reference calls them (internal/transformer/attention.go:120,
    124, 128, 183; feedforward.go:87, 90, 98)."""
    h, f = model["hidden"], model["ffn"]
    q4 = model.get("q4", Q4_K)
    down = model.get("down", Q4_K)
    return [("q", q4, h, model["q_out"]), ("k", q4, h, model["kv_out"]), ("v", q4, h, model["kv_out"]),
            ("o", q4, model["q_out"], h), ("gate", q4, h, f), ("up", q4, h, f), ("down", down, f, h)]


def model_bytes(model: dict, with_head: bool = True) -> int:
    """Algorithmic weight bytes of one decode step (all layers, and the LM head)."""
    per = sum(n_blocks(K, N) * BLOCK_BYTES[qt] for _, qt, K, N in layer_shapes(model))
    total = per * model["layers"]
    if with_head and "vocab" in model:
        total += n_blocks(model["hidden"], model["vocab"]) * BLOCK_BYTES[model["head"]]
    return total
