"""Host side of the row-sharded matmul, on the CPU with world-size-2 `gloo`
process groups: the column plan of vibrant_b200.tensor.shard_columns tiles
[0, N) in multiples of 32 with no gap or overlap for every world size, and
assembling each rank's columns [lo, hi) of x @ W at columns lo.. of a
[M, N] output (the layout vkq_gemv_allgather writes into every rank's
buffer) gives exactly the full product.  The per-rank products come from the
oracle, so this needs no GPU."""
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


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cols(x, w):
    """x @ w in float64, each column reduced on its own in a fixed order
    (independent of how many columns are computed together)."""
    return np.ascontiguousarray((x.astype(np.float64)[:, :, None] * w.astype(np.float64)[None]).sum(axis=1))


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
