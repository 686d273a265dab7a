"""Shared helpers for the parity tests (the oracle is the checker)."""
from __future__ import annotations

import numpy as np

Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
GEMV_TOL = 1e-5    # max |y - y_ref| / sum_k |x_k W_kn|, fp32-accumulate GEMV
GEMM_TOL = 2e-2    # same metric, bf16 tensor-core GEMM
# vkq_set_gemv_path values of the three GEMV kernels
GEMV_PATHS = {"simt": 1, "tc": 2, "strip": 3}


def matmul_error(y: np.ndarray, x: np.ndarray, w: np.ndarray, y_ref: np.ndarray | None = None,
                 col_chunk: int = 8192) -> float:
    """max over (m, n) of |y - y_exact| / sum_k |x[m,k] * W[k,n]|, with y_exact
    in float64 (or |y - y_ref| when y_ref is given).  w is float32 [K, N]."""
    x64 = x.astype(np.float64).reshape(-1, w.shape[0])
    worst = 0.0
    for c0 in range(0, w.shape[1], col_chunk):
        wc = w[:, c0:c0 + col_chunk].astype(np.float64)
        bound = np.abs(x64) @ np.abs(wc)
        ref = (x64 @ wc) if y_ref is None else y_ref.reshape(x64.shape[0], -1)[:, c0:c0 + col_chunk]
        err = np.abs(y.reshape(x64.shape[0], -1)[:, c0:c0 + col_chunk].astype(np.float64) - ref)
        ratio = np.where(bound > 0, err / np.where(bound > 0, bound, 1.0), np.where(err > 0, np.inf, 0.0))
        worst = max(worst, float(np.max(ratio)))
    return worst


def encode_q6k_exact(values: np.ndarray) -> np.ndarray:
    """Q6_K blocks holding small integers exactly: d = 1, every scale 1,
    q = v + 32 (v in [-32, 31])."""
    v = np.asarray(values, dtype=np.int64).reshape(-1)
    nb = (v.size + 255) // 256
    out = np.zeros((nb, 210), np.uint8)
    q = np.full(nb * 256, 32, np.int64)
    q[:v.size] = v + 32
    q = q.reshape(nb, 256)
    idx = np.arange(256)
    for i in range(256):
        lo, hi = q[:, i] & 0xF, q[:, i] >> 4
        out[:, i // 2] |= (lo << (4 * (i % 2))).astype(np.uint8)
        out[:, 128 + i // 4] |= (hi << (2 * (i % 4))).astype(np.uint8)
    del idx
    out[:, 192:208] = 1
    out[:, 208], out[:, 209] = 0x00, 0x3C
    return out.reshape(-1)


def encode_q45k_exact(values: np.ndarray, qtype: int) -> np.ndarray:
    """Q4_K / Q5_K blocks holding small non-negative integers exactly:
    d = 1, dmin = 0, every sub-block scale 1 (q = v, v < 16 or < 32)."""
    v = np.asarray(values, dtype=np.int64).reshape(-1)
    nb = (v.size + 255) // 256
    bb = BLOCK_BYTES[qtype]
    out = np.zeros((nb, bb), np.uint8)
    q = np.zeros(nb * 256, np.int64)
    q[:v.size] = v
    q = q.reshape(nb, 256)
    out[:, 0], out[:, 1] = 0x00, 0x3C          # d = 1.0
    # scales 0..7 = 1: 24-bit LE groups of four 6-bit fields -> 0x041041
    for g in range(2):
        out[:, 4 + 3 * g], out[:, 5 + 3 * g], out[:, 6 + 3 * g] = 0x41, 0x10, 0x04
    qs0 = 16 if qtype == Q4_K else 48
    for i in range(256):
        out[:, qs0 + i // 2] |= ((q[:, i] & 0xF) << (4 * (i % 2))).astype(np.uint8)
        if qtype == Q5_K:
            out[:, 16 + i // 8] |= (((q[:, i] >> 4) & 1) << (i % 8)).astype(np.uint8)
    return out.reshape(-1)


def quantize_q4k_subblocks(values: np.ndarray) -> np.ndarray:
    """Test data that looks like a real Q4_K weight: every 32-value sub-block
    gets its own 6-bit scale and min (the k-quant scheme: the sub-block's
    range min(0, lo)..hi in 15 steps, d and dmin the largest sub-block step
    and offset over 63), packed in the block layout of
    internal/tensor/quant_q4k.go:137-157 with the 24-bit scale groups read by
    extractScalesAndMins.  (The reference's own QuantizeQ4_K,
    quant_q4k.go:215-282, is a test helper that fills sub-block 0's scale and
    min only, so seven of its eight sub-blocks dequantize to zero.)  Written
    for these tests; not part of the reference."""
    v = np.asarray(values, dtype=np.float32).reshape(-1)
    nb = (v.size + 255) // 256
    x = np.zeros(nb * 256, np.float32)
    x[:v.size] = v
    x = x.reshape(nb, 8, 32).astype(np.float64)
    lo = np.minimum(x.min(axis=2), 0.0)
    hi = x.max(axis=2)
    step = np.maximum((hi - lo) / 15.0, 1e-12)
    d = np.maximum(step.max(axis=1) / 63.0, 1e-12)
    dmin = np.maximum((-lo).max(axis=1) / 63.0, 1e-12)
    d16, dmin16 = d.astype(np.float16), dmin.astype(np.float16)
    dq, dminq = np.maximum(d16.astype(np.float64), 6e-8), np.maximum(dmin16.astype(np.float64), 6e-8)
    sc = np.clip(np.rint(step / dq[:, None]), 1, 63).astype(np.int64)
    mn = np.clip(np.rint(-lo / dminq[:, None]), 0, 63).astype(np.int64)
    scale = dq[:, None] * sc
    offs = dminq[:, None] * mn
    q = np.clip(np.rint((x + offs[:, :, None]) / scale[:, :, None]), 0, 15).astype(np.int64).reshape(nb, 256)
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin16.view(np.uint8).reshape(nb, 2)
    for g, f in enumerate((sc[:, 0:4], sc[:, 4:8], mn[:, 0:4], mn[:, 4:8])):
        word = f[:, 0] | (f[:, 1] << 6) | (f[:, 2] << 12) | (f[:, 3] << 18)
        for k in range(3):
            out[:, 4 + 3 * g + k] = ((word >> (8 * k)) & 0xFF).astype(np.uint8)
    out[:, 16:] = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return out.reshape(-1)


def same_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Bitwise equality with NaN as one class."""
    ab, bb = a.view(np.uint32), b.view(np.uint32)
    return (ab == bb) | (np.isnan(a) & np.isnan(b))


def write_gguf(path: str, tensors: list[tuple[str, int, list[int], bytes]], version: int = 3,
               metadata: bool = True, alignment: int = 32) -> list[int]:
    """A GGUF file for the loader tests (the container of
    internal/gguf/parser.go:15-64): magic, version, counts, metadata of every
    value kind (skipped by the loader), tensor infos (name, dims in file
    order, GGML type, data offset relative to the data section) and the data
    section at the end of the infos rounded up to `alignment`.  Returns the
    relative offsets of the tensors."""
    import struct

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    kv = []
    if metadata:
        kv = [s("general.architecture") + struct.pack("<I", 8) + s("llama"),
              s("llama.block_count") + struct.pack("<II", 4, 36),
              s("general.flag") + struct.pack("<IB", 7, 1),
              s("llama.rope.freq_base") + struct.pack("<If", 6, 10000.0),
              s("general.big") + struct.pack("<IQ", 10, 1 << 40),
              s("general.ratio") + struct.pack("<Id", 12, 0.5),
              s("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, 3) + s("a") + s("bc") + s("<s>"),
              s("tokenizer.ggml.scores") + struct.pack("<IIQ", 9, 6, 3) + struct.pack("<3f", 0.1, 0.2, 0.3),
              s("nested") + struct.pack("<IIQ", 9, 9, 2) + struct.pack("<IQ", 4, 2) + struct.pack("<2I", 1, 2)
              + struct.pack("<IQ", 8, 1) + s("x")]
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv)) + b"".join(kv)
    offsets, rel = [], 0
    infos = b""
    for name, ggml_type, dims, data in tensors:
        offsets.append(rel)
        infos += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ggml_type, rel)
        rel += (len(data) + alignment - 1) // alignment * alignment
    body = head + infos
    body += b"\0" * ((-len(body)) % alignment)
    for (_, _, _, data), off in zip(tensors, offsets):
        body += data + b"\0" * ((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(body)
    return offsets
