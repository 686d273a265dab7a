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


def linear_fused(x: torch.Tensor, weights: list[QuantWeight], norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                 silu_mul: bool = False, outs: list[torch.Tensor] | None = None,
                 stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
    """One launch of vkq_linear_fused: [x @ W_i] (or [SiLU(x @ W_0) * (x @ W_1)]),
    with x replaced by RMSNorm(x) * norm_w when norm_w is given."""
    if x.dtype != torch.float32 or x.dim() != 2 or any(w.K != x.shape[1] for w in weights):
        raise ValueError(f"x must be float32 [M, K] with K = every weight's K, got {tuple(x.shape)}")
    x = x.contiguous()
    M = x.shape[0]
    n_out = 1 if silu_mul else len(weights)
    if outs is None:
        outs = [torch.empty((M, weights[i].N), dtype=torch.float32, device=x.device) for i in range(n_out)]
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    vkq.linear_fused(weights[0].qtype, [w.buf.data_ptr() for w in weights], [w.nbytes for w in weights], x.shape[1],
                     [w.N for w in weights], x.data_ptr(), M, [o.data_ptr() for o in outs],
                     norm_w.data_ptr() if norm_w is not None else None, eps,
                     vkq.EPI_SILU_MUL if silu_mul else vkq.EPI_NONE, device=weights[0].device_index, stream=st)
    return outs


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


# ---- row-sharded matmul across the GPUs of one node ----

def shard_columns(N: int, world: int) -> tuple[int, list[tuple[int, int]]]:
    """Equal shard width (a multiple of 32, as the fast GEMV and the peer
    all-gather need) and each rank's [lo, hi) output columns; the last
    rank's range may be shorter than the width.  Same plan as
    vkq_shard_columns."""
    width = -(-N // world)
    width = -(-width // 32) * 32
    bounds = [(min(r * width, N), min((r + 1) * width, N)) for r in range(world)]
    return width, bounds


def shard_device(full: torch.Tensor, qtype: int, K: int, N: int, lo: int, hi: int) -> torch.Tensor:
    """Row-block shard of columns [lo, hi) built on the device from the full
    raw weight already there: the same bytes as vkq_shard_weight (for weights
    drawn on the GPU, whose GBs would be slow to bring back to the host)."""
    B = vkq.BLOCK_BYTES[qtype]
    rb, _ = vkq.shard_bytes(qtype, K, N, lo, hi)
    blocks = full.view(-1, B)
    dev = full.device
    k = torch.arange(K, device=dev, dtype=torch.int64)
    v0 = k * N + lo
    count = ((v0 & 255) + (hi - lo) - 1) // 256 + 1
    j = torch.arange(rb, device=dev, dtype=torch.int64)
    valid = j[None, :] < count[:, None]
    idx = torch.where(valid, (v0 >> 8)[:, None] + j[None, :], torch.zeros_like(j)[None, :])
    out = blocks[idx.reshape(-1)].view(K, rb, B)
    out[~valid] = 0
    return out.reshape(-1)


class ShardedWeight:
    """A rank's row-block shard of a quantized [K, N] weight, on its device:
    only the super-blocks under the rank's output columns (blocks straddling
    rows or shards duplicated).  Built from the full raw bytes on the host
    with vkq_shard_weight (numpy input), or on the device (torch input).
    `bounds` overrides the column range of vkq_shard_columns(N, world, rank)."""

    def __init__(self, qtype: int, K: int, N: int, world: int, rank: int, full_bytes, device="cuda",
                 bounds: tuple[int, int] | None = None):
        self.qtype, self.K, self.N, self.world, self.rank = qtype, K, N, world, rank
        self.lo, self.hi = bounds if bounds is not None else vkq.shard_columns(N, world, rank)
        if isinstance(full_bytes, torch.Tensor) and full_bytes.is_cuda:
            self.buf = shard_device(full_bytes, qtype, K, N, self.lo, self.hi).to(device)
        else:
            host = vkq.shard_weight(qtype, np.ascontiguousarray(full_bytes, dtype=np.uint8), K, N, self.lo, self.hi)
            self.buf = torch.from_numpy(host).to(device=device)
        if self.buf.data_ptr() % 16:
            raise ValueError("shard buffer is not 16-byte aligned")

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    @property
    def width(self) -> int:
        return self.hi - self.lo

    def as_weight(self) -> "QuantWeight":
        """The shard as a plain [K, hi - lo] weight: valid when the columns
        are whole super-block columns (N, lo and hi multiples of 256), where
        the shard is exactly that weight's stream."""
        if self.N % 256 or self.lo % 256 or self.hi % 256:
            raise ValueError("the shard is a plain weight only for whole super-block columns")
        return QuantWeight(self.qtype, self.K, self.width, self.buf, device=self.buf.device)


class _DeviceArray:
    """A raw device pointer seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "strides": None, "version": 3}


class PeerGather:
    """One all-gather channel for vkq_gemv_allgather, created collectively by
    every rank of a process group (one process per GPU).

    Rank r holds ShardedWeight(..., world, r) and computes output columns
    vkq_shard_columns(N, world, r); the kernel stores them into every rank's
    output [m_max, N] (the CUDA-core kernel), or sends them into every rank's
    channel buffer as flagged words that each rank copies into its own output
    (the Q4_K column-strip kernel).  Each rank allocates its output and its
    channel buffer (vkq_gather_channel_bytes(m_max, N)) with vkq_ipc_alloc,
    the 64-byte handles are exchanged over the group and every rank maps
    every other rank's buffers (vkq_ipc_open).  `gemv` then leaves the whole
    x @ W in `out` on every rank, with no collective library call on the data
    path.  Every rank must make the same sequence of calls."""

    def __init__(self, group, rank: int, world: int, device: int, N: int, m_max: int = 8):
        import torch.distributed as dist
        if N % 32:
            raise ValueError("N must be a multiple of 32")
        self.width, self.bounds = shard_columns(N, world)
        if any(hi <= lo for lo, hi in self.bounds):
            raise ValueError(f"N={N} leaves a rank of {world} without columns")
        self.group, self.rank, self.world, self.device, self.N, self.m_max = group, rank, world, device, N, m_max
        self.out_ptr, h_out = vkq.ipc_alloc(m_max * N * 4, device)
        self.chan_bytes = vkq.gather_channel_bytes(m_max, N)
        self.flags_ptr, h_flags = vkq.ipc_alloc(self.chan_bytes, device)
        self.sync_ptr, _ = vkq.ipc_alloc(256, device)
        handles: list = [None] * world
        dist.all_gather_object(handles, (h_out, h_flags), group=group)
        self._mapped: list[int] = []
        self.peer_out, self.peer_flags = [], []
        for r, (ho, hf) in enumerate(handles):
            if r == rank:
                self.peer_out.append(self.out_ptr)
                self.peer_flags.append(self.flags_ptr)
                continue
            po, pf = vkq.ipc_open(ho, device), vkq.ipc_open(hf, device)
            self._mapped += [po, pf]
            self.peer_out.append(po)
            self.peer_flags.append(pf)
        self.out = torch.as_tensor(_DeviceArray(self.out_ptr, (m_max, N)), device=f"cuda:{device}")
        self.flag_words = torch.as_tensor(_DeviceArray(self.flags_ptr, (self.chan_bytes // 4,), "<u4"),
                                          device=f"cuda:{device}")
        self.sync_words = torch.as_tensor(_DeviceArray(self.sync_ptr, (4,), "<u4"), device=f"cuda:{device}")

    def gemv(self, x: torch.Tensor, w: ShardedWeight, ws: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """x @ W across the group: returns out[:M] (vkq_gemv_allgather)."""
        if w.N != self.N or x.shape[1] != w.K or x.dtype != torch.float32:
            raise ValueError("the weight or x does not match the group")
        if (w.world, w.rank) != (self.world, self.rank):
            raise ValueError("the shard was built for another rank")
        M = x.shape[0]
        if M > self.m_max:
            raise ValueError(f"M={M} exceeds the group's m_max={self.m_max}")
        x = x.contiguous()
        if ws is None:
            ws = workspace(workspace_bytes(w.qtype, M, w.K, w.width, self.device), self.device)
        st = stream if stream is not None else torch.cuda.current_stream(x.device)
        vkq.gemv_allgather(w.qtype, w.buf.data_ptr(), w.nbytes, w.K, w.N, w.lo, w.hi, x.data_ptr(), M,
                           self.peer_out, self.peer_flags, self.sync_ptr, self.world, self.rank,
                           ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                           device=self.device, stream=st)
        return self.out[:M]

    def linear_fused(self, x: torch.Tensor, weights: list, norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                     silu_mul: bool = False, outs: list[torch.Tensor] | None = None,
                     stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """vkq_linear_fused_allgather: weights[0] (and weights[1] with
        silu_mul) is this rank's ShardedWeight of the group's N columns,
        gathered into `out`; further weights are whole QuantWeights computed
        here into outs[i - 1].  Returns out[:M] (SiLU(gate) * up with
        silu_mul)."""
        w0 = weights[0]
        if w0.N != self.N or (w0.world, w0.rank) != (self.world, self.rank):
            raise ValueError("weights[0] is not this rank's shard of the group's columns")
        M = x.shape[0]
        if M > self.m_max or x.dtype != torch.float32:
            raise ValueError("x does not match the group")
        x = x.contiguous()
        local = [] if silu_mul else weights[1:]
        if outs is None:
            outs = [torch.empty((M, w.N), dtype=torch.float32, device=x.device) for w in local]
        st = stream if stream is not None else torch.cuda.current_stream(x.device)
        vkq.linear_fused_allgather(
            w0.qtype, [w.buf.data_ptr() for w in weights], [w.nbytes for w in weights], w0.K, self.N, w0.lo, w0.hi,
            [0] + [w.N for w in local], x.data_ptr(), M, [0] + [o.data_ptr() for o in outs],
            self.peer_out, self.peer_flags, self.sync_ptr, self.world, self.rank,
            norm_w.data_ptr() if norm_w is not None else None, eps,
            vkq.EPI_SILU_MUL if silu_mul else vkq.EPI_NONE, device=self.device, stream=st)
        return self.out[:M]

    def reset(self) -> None:
        """Collective: zero every rank's channel (after a failed call)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.flag_words.zero_()
        self.sync_words.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._mapped:
            vkq.ipc_close(p, self.device)
        self._mapped = []
        dist.barrier(group=self.group)
        for p in (self.out_ptr, self.flags_ptr, self.sync_ptr):
            vkq.ipc_free(p, self.device)


class Comm:
    """In-process form (vkq_comm_init): one process drives every listed GPU.
    `gemv` runs one sharded call on every device and returns the per-device
    outputs [M, N], each holding the whole product once the streams finish."""

    def __init__(self, devices: list[int]):
        self.devices = list(devices)
        self.world = len(self.devices)
        self.handle = vkq.comm_init(self.devices)
        self.streams = [torch.cuda.Stream(device=d) for d in self.devices]

    def shards(self, qtype: int, K: int, N: int, full_bytes) -> list[ShardedWeight]:
        return [ShardedWeight(qtype, K, N, self.world, r, full_bytes, device=f"cuda:{d}")
                for r, d in enumerate(self.devices)]

    def gemv(self, xs: list[torch.Tensor], shards: list[ShardedWeight], ys: list[torch.Tensor]) -> list[torch.Tensor]:
        w0 = shards[0]
        M = xs[0].shape[0]
        wss = []
        for r, d in enumerate(self.devices):
            wss.append(workspace(workspace_bytes(w0.qtype, M, w0.K, shards[r].width, d), d))
        vkq.gemv_sharded(self.handle, w0.qtype, [s.buf.data_ptr() for s in shards], [s.nbytes for s in shards],
                         w0.K, w0.N, [x.data_ptr() for x in xs], M, [y.data_ptr() for y in ys],
                         [ws.data_ptr() if ws is not None else 0 for ws in wss],
                         [ws.numel() if ws is not None else 0 for ws in wss], self.streams)
        return ys

    def reset(self) -> None:
        vkq.comm_reset(self.handle)

    def close(self) -> None:
        if self.handle:
            vkq.comm_destroy(self.handle)
            self.handle = 0
