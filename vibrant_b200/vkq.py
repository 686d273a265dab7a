"""ctypes binding of libvkq.so (include/vkq.h).

This is how the tests and bench.py reach the kernels: through the same C ABI a
Go cgo shim would bind.  Loading fails loudly when the library is missing;
there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libvkq.so")

Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
QTYPE_NAMES = {Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_MISALIGNED, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE_TIMEOUT, \
    ERR_NCCL, ERR_PEER = range(9)

# every symbol declared in include/vkq.h, with (restype, argtypes)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
SIGNATURES = {
    "vkq_abi_version": (_int, []),
    "vkq_status_string": (ctypes.c_char_p, [_int]),
    "vkq_last_error": (ctypes.c_char_p, []),
    "vkq_block_bytes": (_i64, [_int]),
    "vkq_weight_bytes": (_int, [_int, _i64, _i64, ctypes.POINTER(_i64)]),
    "vkq_dequantize_f32": (_int, [_int, _int, _vp, _i64, _vp, _vp]),
    "vkq_dequant_transpose_f32": (_int, [_int, _int, _vp, _i64, _i64, _vp, _vp]),
    "vkq_matmul_workspace_bytes": (_int, [_int, _int, _i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "vkq_matmul": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _sz, _vp]),
    "vkq_gemv": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _sz, _vp]),
    "vkq_gemm": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _sz, _vp]),
    "vkq_matmul_host": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "vkq_matmul_upstream": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "vkq_gemv_noalloc": (_int, [_int, _int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "vkq_device_status": (_int, [_int, ctypes.POINTER(_int)]),
    "vkq_ipc_alloc": (_int, [_int, _sz, ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_ubyte * 64)]),
    "vkq_ipc_open": (_int, [_int, ctypes.POINTER(ctypes.c_ubyte * 64), ctypes.POINTER(_vp)]),
    "vkq_ipc_close": (_int, [_int, _vp]),
    "vkq_ipc_free": (_int, [_int, _vp]),
    "vkq_gemv_allgather": (_int, [_int, _int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _int,
                                  _int, _vp, _sz, _vp]),
    "vkq_set_gemv_path": (_int, [_int]),
    "vkq_gather_channel_bytes": (_sz, [_i64, _i64]),
    "vkq_linear_fused_allgather": (_int, [_int, _int, _int, ctypes.POINTER(_vp), ctypes.POINTER(_i64), _i64, _i64,
                                          _i64, _i64, ctypes.POINTER(_i64), _vp, _i64, _vp, ctypes.c_float, _int,
                                          ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp, _int,
                                          _int, _vp]),
    "vkq_silu_mul": (_int, [_int, _vp, _vp, _vp, _i64, _vp]),
    "vkq_rms_norm": (_int, [_int, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "vkq_rope_f32": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "vkq_attention_decode_f32": (_int, [_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "vkq_attention_rope_decode_f32": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                              _i64, _i64, _i64, _i64, _vp]),
    "vkq_linear_fused": (_int, [_int, _int, _int, ctypes.POINTER(_vp), ctypes.POINTER(_i64), _i64,
                                ctypes.POINTER(_i64), _vp, _i64, _vp, ctypes.c_float, _int, ctypes.POINTER(_vp), _vp]),
    "vkq_gguf_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "vkq_gguf_close": (_int, [_vp]),
    "vkq_gguf_tensor_count": (_i64, [_vp]),
    "vkq_gguf_find": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "vkq_gguf_tensor_info": (_int, [_vp, _i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_int),
                                    ctypes.POINTER(_int), ctypes.POINTER(_i64 * 4), ctypes.POINTER(_i64),
                                    ctypes.POINTER(_i64)]),
    "vkq_gguf_tensor_bytes": (_int, [_int, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "vkq_gguf_load_tensor": (_int, [_vp, _i64, _int, _vp, _i64, _vp]),
    "vkq_gguf_load_shard": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _i64, _vp]),
    "vkq_shard_columns": (_int, [_i64, _int, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "vkq_shard_bytes": (_int, [_int, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "vkq_shard_weight": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64]),
    "vkq_comm_init": (_int, [_int, ctypes.POINTER(_int), ctypes.POINTER(_vp)]),
    "vkq_comm_reset": (_int, [_vp]),
    "vkq_comm_destroy": (_int, [_vp]),
    "vkq_comm_size": (_int, [_vp]),
    "vkq_gemv_sharded": (_int, [_vp, _int, ctypes.POINTER(_vp), ctypes.POINTER(_i64), _i64, _i64, ctypes.POINTER(_vp),
                                _i64, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_sz),
                                ctypes.POINTER(_vp)]),
}


class VkqError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"vkq status {status}: {msg}")
        self.status = status


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libvkq.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `python -m vibrant_b200.build` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != OK:
        raise VkqError(status, load().vkq_last_error().decode(errors="replace"))


def last_error() -> str:
    return load().vkq_last_error().decode(errors="replace")


def weight_bytes(qtype: int, K: int, N: int) -> int:
    out = _i64()
    _check(load().vkq_weight_bytes(qtype, K, N, ctypes.byref(out)))
    return out.value


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream  # torch.cuda.Stream


def dequantize_f32(qtype: int, w_ptr: int, nblocks: int, out_ptr: int, device: int = -1, stream=None) -> None:
    _check(load().vkq_dequantize_f32(device, qtype, w_ptr, nblocks, out_ptr, _stream_ptr(stream)))


def dequant_transpose_f32(qtype: int, w_ptr: int, K: int, N: int, out_ptr: int, device: int = -1,
                          stream=None) -> None:
    _check(load().vkq_dequant_transpose_f32(device, qtype, w_ptr, K, N, out_ptr, _stream_ptr(stream)))


def matmul_workspace_bytes(qtype: int, M: int, K: int, N: int, device: int = -1) -> int:
    out = _sz()
    _check(load().vkq_matmul_workspace_bytes(device, qtype, M, K, N, ctypes.byref(out)))
    return out.value


def matmul(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_ptr: int, M: int, y_ptr: int,
           ws_ptr: int | None, ws_bytes: int, device: int = -1, stream=None) -> None:
    _check(load().vkq_matmul(device, qtype, w_ptr, w_bytes, K, N, x_ptr, M, y_ptr, ws_ptr, ws_bytes,
                             _stream_ptr(stream)))


def gemv(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_ptr: int, M: int, y_ptr: int,
         ws_ptr: int | None, ws_bytes: int, device: int = -1, stream=None) -> None:
    _check(load().vkq_gemv(device, qtype, w_ptr, w_bytes, K, N, x_ptr, M, y_ptr, ws_ptr, ws_bytes,
                           _stream_ptr(stream)))


def gemm(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_ptr: int, M: int, y_ptr: int,
         ws_ptr: int | None, ws_bytes: int, device: int = -1, stream=None) -> None:
    _check(load().vkq_gemm(device, qtype, w_ptr, w_bytes, K, N, x_ptr, M, y_ptr, ws_ptr, ws_bytes,
                           _stream_ptr(stream)))


def matmul_upstream(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_ptr: int, M: int, y_ptr: int,
                    device: int = -1, stream=None) -> None:
    """vkq_matmul_upstream: y[m][n] = sum_k x[m][k] * W[n][k] for a weight in
    the upstream GGUF orientation (row n = the blocks of output n along K)."""
    _check(load().vkq_matmul_upstream(device, qtype, w_ptr, w_bytes, K, N, x_ptr, M, y_ptr, _stream_ptr(stream)))


def matmul_host(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_host_ptr: int, M: int, y_host_ptr: int,
                x_dev_ptr: int, y_dev_ptr: int, ws_ptr: int | None, ws_bytes: int, device: int = -1,
                stream=None) -> None:
    """vkq_matmul_host: x from host memory, y back to host memory, around
    vkq_matmul, enqueued on the stream in one call."""
    _check(load().vkq_matmul_host(device, qtype, w_ptr, w_bytes, K, N, x_host_ptr, M, y_host_ptr, x_dev_ptr,
                                  y_dev_ptr, ws_ptr, ws_bytes, _stream_ptr(stream)))


def gemv_noalloc(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, x_ptr: int, M: int, y_ptr: int,
                 device: int = -1, stream=None) -> None:
    """vkq_gemv_noalloc: the GEMV with its scratch in the library's fixed device array."""
    _check(load().vkq_gemv_noalloc(device, qtype, w_ptr, w_bytes, K, N, x_ptr, M, y_ptr, _stream_ptr(stream)))


GEMV_AUTO, GEMV_SIMT, GEMV_TC, GEMV_STRIP = 0, 1, 2, 3


def set_gemv_path(path: int) -> int:
    """vkq_set_gemv_path: 0 automatic, 1 CUDA cores, 2 tensor cores, 3 column strips (process-wide);
    returns the previous choice."""
    old = load().vkq_set_gemv_path(path)
    if old < 0:
        raise VkqError(ERR_INVALID_ARGUMENT, last_error())
    return old


def silu_mul(gate_ptr: int, up_ptr: int, out_ptr: int, n: int, device: int = -1, stream=None) -> None:
    """vkq_silu_mul: out = SiLU(gate) * up."""
    _check(load().vkq_silu_mul(device, gate_ptr, up_ptr, out_ptr, n, _stream_ptr(stream)))


def rms_norm(x_ptr: int, w_ptr: int, out_ptr: int, rows: int, n: int, eps: float, device: int = -1,
             stream=None) -> None:
    """vkq_rms_norm: out[r] = x[r] / sqrt(mean(x[r]^2) + eps) * weight."""
    _check(load().vkq_rms_norm(device, x_ptr, w_ptr, out_ptr, rows, n, eps, _stream_ptr(stream)))


def rope_f32(x_ptr: int, out_ptr: int, cos_ptr: int, sin_ptr: int, pos_ptr: int, batch: int, heads: int, seq: int,
             head_dim: int, max_seq: int, device: int = -1, stream=None) -> None:
    """vkq_rope_f32: rotary position embedding over interleaved pairs of
    x [batch][heads][seq][head_dim] with cos/sin tables [max_seq][head_dim/2]."""
    _check(load().vkq_rope_f32(device, x_ptr, out_ptr, cos_ptr, sin_ptr, pos_ptr, batch, heads, seq, head_dim,
                               max_seq, _stream_ptr(stream)))


def attention_decode_f32(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, batch: int, heads: int, kv_heads: int,
                         length: int, cache_len: int, head_dim: int, device: int = -1, stream=None) -> None:
    """vkq_attention_decode_f32: one query token per sequence against its KV
    cache (rows 0 .. length-1 of [batch][kv_heads][cache_len][head_dim])."""
    _check(load().vkq_attention_decode_f32(device, q_ptr, k_ptr, v_ptr, out_ptr, batch, heads, kv_heads, length,
                                           cache_len, head_dim, _stream_ptr(stream)))


def attention_rope_decode_f32(q_ptr: int, k_new_ptr: int, v_new_ptr: int, cos_ptr: int, sin_ptr: int, pos_ptr: int,
                              k_cache_ptr: int, v_cache_ptr: int, out_ptr: int, batch: int, heads: int,
                              kv_heads: int, length: int, cache_len: int, head_dim: int, max_seq: int,
                              device: int = -1, stream=None) -> None:
    """vkq_attention_rope_decode_f32: RoPE on q and k_new at positions[b],
    the rotated k_new and v_new stored at row length-1 of the caches, and
    attention over rows 0 .. length-1, in one launch."""
    _check(load().vkq_attention_rope_decode_f32(device, q_ptr, k_new_ptr, v_new_ptr, cos_ptr, sin_ptr, pos_ptr,
                                                k_cache_ptr, v_cache_ptr, out_ptr, batch, heads, kv_heads, length,
                                                cache_len, head_dim, max_seq, _stream_ptr(stream)))


def rope_tables(head_dim: int, freq_base: float, max_seq: int):
    """cos and sin tables [max_seq][head_dim/2] as float32 numpy arrays, built
    as the reference's NewRoPE (internal/transformer/rope.go:19-43) builds
    them: angle = pos / freq_base^(2i/head_dim) in float64, then cos and sin
    rounded to float32 (this host's libm may differ from Go's math package in
    the last bit of an entry; the kernel takes the tables as given)."""
    import numpy as np
    half = head_dim // 2
    i = np.arange(half, dtype=np.float64)
    freq = 1.0 / np.power(freq_base, 2.0 * i / head_dim)
    angle = np.arange(max_seq, dtype=np.float64)[:, None] * freq[None, :]
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def device_status(device: int = -1) -> int:
    code = _int()
    _check(load().vkq_device_status(device, ctypes.byref(code)))
    return code.value


def ipc_alloc(nbytes: int, device: int = -1) -> tuple[int, bytes]:
    """vkq_ipc_alloc: zero-filled device memory another process can map;
    returns (device pointer, 64-byte handle)."""
    ptr, h = _vp(), (ctypes.c_ubyte * 64)()
    _check(load().vkq_ipc_alloc(device, nbytes, ctypes.byref(ptr), ctypes.byref(h)))
    return ptr.value, bytes(h)


def ipc_open(handle: bytes, device: int = -1) -> int:
    """vkq_ipc_open: this process's mapping of another process's buffer."""
    h = (ctypes.c_ubyte * 64).from_buffer_copy(handle)
    ptr = _vp()
    _check(load().vkq_ipc_open(device, ctypes.byref(h), ctypes.byref(ptr)))
    return ptr.value


def ipc_close(ptr: int, device: int = -1) -> None:
    _check(load().vkq_ipc_close(device, ptr))


def ipc_free(ptr: int, device: int = -1) -> None:
    _check(load().vkq_ipc_free(device, ptr))


def gemv_allgather(qtype: int, w_ptr: int, w_bytes: int, K: int, N: int, col_lo: int, col_hi: int, x_ptr: int,
                   M: int, peer_out: list[int], peer_flags: list[int], sync_ptr: int, world: int, rank: int,
                   ws_ptr: int | None, ws_bytes: int, device: int = -1, stream=None) -> None:
    """vkq_gemv_allgather: columns [col_lo, col_hi) of x @ W from this rank's
    row-block shard, stored into every rank's output [M, N] through peer
    memory; peer_out / peer_flags are host lists of device pointers."""
    po = (_vp * world)(*peer_out)
    pf = (_vp * world)(*peer_flags)
    _check(load().vkq_gemv_allgather(device, qtype, w_ptr, w_bytes, K, N, col_lo, col_hi, x_ptr, M, po, pf, sync_ptr,
                                     world, rank, ws_ptr, ws_bytes, _stream_ptr(stream)))


EPI_NONE, EPI_SILU_MUL = 0, 1


def linear_fused(qtype: int, w_ptrs: list[int], w_bytes: list[int], K: int, Ns: list[int], x_ptr: int, M: int,
                 y_ptrs: list[int], norm_w_ptr: int | None = None, eps: float = 1e-6, epilogue: int = EPI_NONE,
                 device: int = -1, stream=None) -> None:
    """vkq_linear_fused: several Q4_K weights over one input in one launch,
    with an optional RMSNorm prologue and the SiLU(gate) * up epilogue."""
    n = len(w_ptrs)
    ys = list(y_ptrs) + [0] * (n - len(y_ptrs))
    _check(load().vkq_linear_fused(device, qtype, n, (_vp * n)(*w_ptrs), (_i64 * n)(*w_bytes), K, (_i64 * n)(*Ns),
                                   x_ptr, M, norm_w_ptr, eps, epilogue, (_vp * n)(*ys), _stream_ptr(stream)))


def linear_fused_allgather(qtype: int, w_ptrs: list[int], w_bytes: list[int], K: int, N: int, col_lo: int,
                           col_hi: int, n_local: list[int], x_ptr: int, M: int, y_local: list[int],
                           peer_out: list[int], peer_flags: list[int], sync_ptr: int, world: int, rank: int,
                           norm_w_ptr: int | None = None, eps: float = 1e-6, epilogue: int = EPI_NONE,
                           device: int = -1, stream=None) -> None:
    """vkq_linear_fused_allgather: weight 0 (or the gate|up pair) is this
    rank's shard of columns [col_lo, col_hi), gathered into every rank's
    output; further weights are whole and local (n_local / y_local, entry 0
    unused)."""
    n = len(w_ptrs)
    nl = list(n_local) + [0] * (n - len(n_local))
    yl = list(y_local) + [0] * (n - len(y_local))
    _check(load().vkq_linear_fused_allgather(device, qtype, n, (_vp * n)(*w_ptrs), (_i64 * n)(*w_bytes), K, N,
                                             col_lo, col_hi, (_i64 * n)(*nl), x_ptr, M, norm_w_ptr, eps, epilogue,
                                             (_vp * n)(*yl), (_vp * world)(*peer_out), (_vp * world)(*peer_flags),
                                             sync_ptr, world, rank, _stream_ptr(stream)))


def gather_channel_bytes(m_max: int, N: int) -> int:
    """vkq_gather_channel_bytes: size of an all-gather channel buffer."""
    return int(load().vkq_gather_channel_bytes(m_max, N))


def shard_columns(N: int, world: int, rank: int) -> tuple[int, int]:
    """vkq_shard_columns: the [lo, hi) output columns of a rank."""
    lo, hi = _i64(), _i64()
    _check(load().vkq_shard_columns(N, world, rank, ctypes.byref(lo), ctypes.byref(hi)))
    return lo.value, hi.value


def shard_bytes(qtype: int, K: int, N: int, col_lo: int, col_hi: int) -> tuple[int, int]:
    """vkq_shard_bytes: (block slots per row, bytes) of a row-block shard."""
    rb, nb = _i64(), _i64()
    _check(load().vkq_shard_bytes(qtype, K, N, col_lo, col_hi, ctypes.byref(rb), ctypes.byref(nb)))
    return rb.value, nb.value


def shard_weight(qtype: int, w, K: int, N: int, col_lo: int, col_hi: int):
    """vkq_shard_weight on host bytes (numpy uint8): the row-block shard of
    columns [col_lo, col_hi) as a new numpy uint8 array."""
    import numpy as np
    w = np.ascontiguousarray(w, dtype=np.uint8)
    _, nb = shard_bytes(qtype, K, N, col_lo, col_hi)
    out = np.empty(nb, np.uint8)
    _check(load().vkq_shard_weight(qtype, w.ctypes.data, w.size, K, N, col_lo, col_hi, out.ctypes.data, nb))
    return out


def comm_init(devices: list[int]) -> int:
    """vkq_comm_init: an in-process communicator over `devices` (handle)."""
    arr = (_int * len(devices))(*devices)
    h = _vp()
    _check(load().vkq_comm_init(len(devices), arr, ctypes.byref(h)))
    return h.value


def comm_reset(comm: int) -> None:
    _check(load().vkq_comm_reset(comm))


def comm_destroy(comm: int) -> None:
    _check(load().vkq_comm_destroy(comm))


def gemv_sharded(comm: int, qtype: int, w_shards: list[int], w_bytes: list[int], K: int, N: int, x: list[int], M: int,
                 y: list[int], workspaces: list[int], ws_bytes: list[int], streams: list) -> None:
    """vkq_gemv_sharded: one call on every device of the communicator."""
    n = len(w_shards)
    _check(load().vkq_gemv_sharded(comm, qtype, (_vp * n)(*w_shards), (_i64 * n)(*w_bytes), K, N, (_vp * n)(*x), M,
                                   (_vp * n)(*y), (_vp * n)(*workspaces), (_sz * n)(*ws_bytes),
                                   (_vp * n)(*[_stream_ptr(s) for s in streams])))


class GGUF:
    """vkq_gguf_*: a memory-mapped GGUF file; tensors load to the device raw."""

    def __init__(self, path: str):
        h = _vp()
        _check(load().vkq_gguf_open(path.encode(), ctypes.byref(h)))
        self.handle = h.value

    def __len__(self) -> int:
        return load().vkq_gguf_tensor_count(self.handle)

    def find(self, name: str) -> int:
        i = _i64()
        _check(load().vkq_gguf_find(self.handle, name.encode(), ctypes.byref(i)))
        return i.value

    def info(self, index: int) -> dict:
        name, t, nd, dims, off, nb = ctypes.c_char_p(), _int(), _int(), (_i64 * 4)(), _i64(), _i64()
        _check(load().vkq_gguf_tensor_info(self.handle, index, ctypes.byref(name), ctypes.byref(t), ctypes.byref(nd),
                                           ctypes.byref(dims), ctypes.byref(off), ctypes.byref(nb)))
        return {"name": name.value.decode(), "type": t.value, "dims": list(dims)[:nd.value], "offset": off.value,
                "bytes": nb.value}

    def load(self, index: int, dst_ptr: int, dst_bytes: int, device: int = 0, stream=None) -> None:
        _check(load().vkq_gguf_load_tensor(self.handle, index, device, dst_ptr, dst_bytes, _stream_ptr(stream)))

    def load_shard(self, index: int, col_lo: int, col_hi: int, dst_ptr: int, dst_bytes: int, device: int = 0,
                   stream=None) -> None:
        _check(load().vkq_gguf_load_shard(self.handle, index, col_lo, col_hi, device, dst_ptr, dst_bytes,
                                          _stream_ptr(stream)))

    def close(self) -> None:
        if self.handle:
            _check(load().vkq_gguf_close(self.handle))
            self.handle = 0


def gguf_tensor_bytes(ggml_type: int, dims: list[int]) -> int:
    d = (_i64 * len(dims))(*dims)
    out = _i64()
    _check(load().vkq_gguf_tensor_bytes(ggml_type, len(dims), d, ctypes.byref(out)))
    return out.value
