"""torch-facing helpers over the C ABI: device buffers, workspaces and streams.

torch only supplies device memory and streams here; every computation is a
libvkq.so kernel reached through vibrant_b200.vkq (the C ABI).
"""
from __future__ import annotations

import numpy as np
import torch

from . import vkq


class QuantWeight:
    """A quantized [K, N] weight kept packed in device memory (the raw
    super-block stream, in vibrant's orientation: W[k][n] is value k*N + n)."""

    def __init__(self, qtype: int, K: int, N: int, data, device="cuda"):
        need = vkq.weight_bytes(qtype, K, N)
        if isinstance(data, np.ndarray):
            t = torch.from_numpy(np.ascontiguousarray(data, dtype=np.uint8))
        else:
            t = data
        if t.numel() < need:
            raise ValueError(f"weight data has {t.numel()} bytes, need {need}")
        self.qtype, self.K, self.N = qtype, K, N
        self.buf = t.to(device=device, dtype=torch.uint8).contiguous()
        if self.buf.data_ptr() % 16:
            raise ValueError("weight buffer is not 16-byte aligned")

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    @property
    def device_index(self) -> int:
        return self.buf.device.index if self.buf.device.index is not None else torch.cuda.current_device()


_WS: dict[tuple[int, int], torch.Tensor] = {}
_WS_NEED: dict[tuple, int] = {}


def workspace_bytes(qtype: int, M: int, K: int, N: int, device: int) -> int:
    """vkq_matmul_workspace_bytes, memoised per shape and device."""
    key = (qtype, M, K, N, device)
    v = _WS_NEED.get(key)
    if v is None:
        v = vkq.matmul_workspace_bytes(qtype, M, K, N, device=device)
        _WS_NEED[key] = v
    return v


def workspace(nbytes: int, device: int) -> torch.Tensor | None:
    """A zero-filled, cached workspace of at least nbytes on a device (one per
    device: calls on one stream may share it)."""
    if nbytes == 0:
        return None
    key = (device, 0)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=f"cuda:{device}")
        _WS[key] = ws
    return ws


def matmul(x: torch.Tensor, w: QuantWeight, out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
           stream: torch.cuda.Stream | None = None, path: str = "auto") -> torch.Tensor:
    """y = x @ W for float32 x [M, K] on the weight's device (vkq_matmul)."""
    if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != w.K:
        raise ValueError(f"x must be float32 [M, {w.K}], got {tuple(x.shape)} {x.dtype}")
    x = x.contiguous()
    M = x.shape[0]
    dev = w.device_index
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.float32, device=x.device)
    if ws is None:
        need = workspace_bytes(w.qtype, M, w.K, w.N, dev)
        if path == "gemm":
            need = max(need, workspace_bytes(w.qtype, max(M, 9), w.K, w.N, dev))
        ws = workspace(need, dev)
    ws_ptr = ws.data_ptr() if ws is not None else None
    ws_bytes = ws.numel() if ws is not None else 0
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    fn = {"gemv": vkq.gemv, "gemm": vkq.gemm}.get(path, vkq.matmul)
    fn(w.qtype, w.buf.data_ptr(), w.nbytes, w.K, w.N, x.data_ptr(), M, out.data_ptr(), ws_ptr, ws_bytes,
       device=dev, stream=st)
    return out


def dequantize(w: QuantWeight, stream=None) -> torch.Tensor:
    """All values of the weight's super-blocks as float32 (vkq_dequantize_f32)."""
    nb = w.nbytes // vkq.BLOCK_BYTES[w.qtype]
    out = torch.empty(nb * 256, dtype=torch.float32, device=w.buf.device)
    st = stream if stream is not None else torch.cuda.current_stream(w.buf.device)
    vkq.dequantize_f32(w.qtype, w.buf.data_ptr(), nb, out.data_ptr(), device=w.device_index, stream=st)
    return out


def dequant_transpose(w: QuantWeight, stream=None) -> torch.Tensor:
    """float32 [N, K] transposed copy (vkq_dequant_transpose_f32)."""
    out = torch.empty((w.N, w.K), dtype=torch.float32, device=w.buf.device)
    st = stream if stream is not None else torch.cuda.current_stream(w.buf.device)
    vkq.dequant_transpose_f32(w.qtype, w.buf.data_ptr(), w.K, w.N, out.data_ptr(), device=w.device_index,
                              stream=st)
    return out
