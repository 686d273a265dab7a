"""Host side of the row-sharded matmul, on the CPU (world-size-2 `gloo`
process groups where ranks talk): the column plan tiles [0, N) in multiples
of 32 with no gap or overlap for every world size (Python and C plans agree);
the row-block shard of vkq_shard_weight holds, at the kernel's addressing
k * rs + ((k * N + lo) & 255) + n, exactly the values of the full weight's
columns [lo, hi) (bit-exact through the oracle's dequantization, including
blocks that straddle rows and shards); and assembling each rank's columns of
x @ W, computed from its own shard only, gives the full product.  No GPU."""
import os
import socket

import numpy as np
import pytest

from vibrant_b200.tensor import shard_columns

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("N", [96, 640, 4160, 11008, 151936])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_plan_tiles_the_columns(N, world):
    width, bounds = shard_columns(N, world)
    assert width % 32 == 0 and len(bounds) == world
    pos = 0
    for lo, hi in bounds:
        assert lo == pos and lo % 32 == 0 and hi % 32 == 0 and hi - lo <= width
        pos = hi
    assert pos == N


@pytest.mark.parametrize("N", [96, 640, 4160, 11008, 151936])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_c_and_python_plans_agree(N, world):
    from vibrant_b200 import vkq
    _, bounds = shard_columns(N, world)
    for r, (lo, hi) in enumerate(bounds):
        if hi > lo:
            assert vkq.shard_columns(N, world, r) == (lo, hi)
        else:  # a rank without columns is refused
            with pytest.raises(vkq.VkqError):
                vkq.shard_columns(N, world, r)


def _shard_values(qt, sh, K, N, lo, hi, rb):
    """Values n = 0 .. hi - lo of every row of a row-block shard, read at
    the position the kernel reads them."""
    from oracle import kq_oracle
    d = kq_oracle.dequantize(qt, sh)
    rows = []
    for k in range(K):
        off = (k * N + lo) & 255
        rows.append(d[k * rb * 256 + off:k * rb * 256 + off + hi - lo])
    return np.stack(rows)


@pytest.mark.parametrize("qt,K,N,world", [(14, 40, 151936, 8), (14, 33, 151936, 2), (12, 48, 11008, 4),
                                          (13, 32, 4160, 2), (14, 40, 640, 3), (12, 16, 2048, 8),
                                          (13, 9, 256, 8)])
def test_row_block_shards_hold_the_columns_bit_exactly(qt, K, N, world):
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    w = synth.random_bytes(qt, K, N, seed=K + N + world)
    full = kq_oracle.dequantize(qt, w)[:K * N].reshape(K, N)
    total = 0
    for r in range(world):
        lo, hi = vkq.shard_columns(N, world, r)
        rb, nb = vkq.shard_bytes(qt, K, N, lo, hi)
        sh = vkq.shard_weight(qt, w, K, N, lo, hi)
        assert sh.size == nb == K * rb * synth.BLOCK_BYTES[qt]
        vals = _shard_values(qt, sh, K, N, lo, hi, rb)
        ok = (vals.view(np.uint32) == full[:, lo:hi].view(np.uint32)) | (np.isnan(vals) & np.isnan(full[:, lo:hi]))
        assert ok.all(), (r, lo, hi)
        total += nb
    # sharding divides the weight: the shards together hold little more than the whole
    nfull = synth.n_blocks(K, N) * synth.BLOCK_BYTES[qt]
    assert total <= nfull + world * K * 2 * synth.BLOCK_BYTES[qt]
    if N % (256 * world) == 0:
        assert total == nfull


def test_shard_rejects_short_buffers_and_bad_columns():
    from vibrant_b200 import synth, vkq
    w = synth.weights(12, 8, 512, seed=1)
    with pytest.raises(vkq.VkqError):
        vkq.shard_columns(500, 2, 0)          # N not a multiple of 32
    with pytest.raises(vkq.VkqError):
        vkq.shard_columns(64, 4, 3)           # a rank without columns
    with pytest.raises(vkq.VkqError):
        vkq.shard_bytes(12, 8, 512, 256, 600)  # beyond N
    with pytest.raises(vkq.VkqError):
        vkq.shard_weight(12, w[:100], 8, 512, 0, 256)  # short source


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cols(x, w):
    """x @ w in float64, each column reduced on its own in a fixed order
    (independent of how many columns are computed together)."""
    return np.ascontiguousarray((x.astype(np.float64)[:, :, None] * w.astype(np.float64)[None]).sum(axis=1))


def _rank_shards(rank, world, port, qt, K, N, M):
    """Each rank computes its columns from its own row-block shard only."""
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    wq = synth.weights(qt, K, N, seed=5)
    x = synth.activations(M, K, seed=6)
    lo, hi = vkq.shard_columns(N, world, rank)
    rb, _ = vkq.shard_bytes(qt, K, N, lo, hi)
    mine = _cols(x, _shard_values(qt, vkq.shard_weight(qt, wq, K, N, lo, hi), K, N, lo, hi, rb))
    parts = [None] * world
    dist.all_gather_object(parts, (lo, hi, mine))
    y = np.zeros((M, N))
    for plo, phi, part in parts:
        y[:, plo:phi] = part
    full = _cols(x, kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N))
    assert np.array_equal(y, full)
    dist.destroy_process_group()


def test_two_rank_shards_assemble_the_full_product():
    import torch.multiprocessing as mp
    mp.spawn(_rank_shards, args=(2, _free_port(), 14, 24, 2336, 2), nprocs=2, join=True)


def _rank(rank, world, port, qt, K, N, M):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import kq_oracle
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=3)
    w = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    x = synth.activations(M, K, seed=4)
    _, bounds = shard_columns(N, world)
    lo, hi = bounds[rank]
    mine = torch.from_numpy(_cols(x, w[:, lo:hi]))
    parts = [None] * world
    dist.all_gather_object(parts, (lo, hi, mine.numpy()))
    y = np.zeros((M, N))
    for plo, phi, part in parts:
        y[:, plo:phi] = part
    full = _cols(x, w)
    assert np.array_equal(y, full)
    dist.destroy_process_group()


def test_two_rank_assembly_matches_the_full_product():
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, _free_port(), 14, 64, 640, 3), nprocs=2, join=True)
