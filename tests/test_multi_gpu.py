"""Row-sharded GEMV with the all-gather fused into the kernel through peer
memory (vkq_gemv_allgather, vibrant_b200.tensor.PeerGather) on 2 GPUs.

Every rank keeps the full quantized weight, computes its columns and stores
them into every rank's output over NVLink.  After each call every rank's
output must equal the full product within the GEMV tolerance (1e-5 of
sum_k |x w|), for consecutive calls of different M and for a weight whose N
is not a multiple of 256 (super-blocks straddle the rows and the shards).
The ranks run as child processes; the test needs 2 GPUs and is skipped
otherwise."""
import os
import socket

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    for qt, K, N in cases:
        wq = synth.weights(qt, K, N, seed=K + N)
        w = vt.QuantWeight(qt, K, N, wq, device=f"cuda:{rank}")
        wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
        g = vt.PeerGather(dist.group.WORLD, rank, world, rank, N, m_max=4)
        for call, M in enumerate([1, 3, 1, 4, 2]):
            x = synth.activations(M, K, seed=100 * call + qt)
            y = g.gemv(torch.from_numpy(x).cuda(), w)
            torch.cuda.synchronize()
            err = helpers.matmul_error(y.cpu().numpy(), x, wd)
            assert err <= helpers.GEMV_TOL, (rank, qt, K, N, call, M, err)
        assert vkq.device_status(rank) == vkq.OK
        g.close()
    dist.destroy_process_group()


def test_allgather_through_peer_memory_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    cases = [
        (14, 2048, 151936 // 4),   # Q6_K, N % 256 == 0 only per 4 rows: shards straddle blocks
        (12, 2048, 11008),         # Q4_K FFN gate/up
        (13, 512, 4160),           # Q5_K, N % 256 == 64
    ]
    mp.spawn(_rank_main, args=(2, _free_port(), cases), nprocs=2, join=True)


@pytest.mark.parametrize("qt,K,N,world", [
    (14, 256, 151936, 2),  # wide shards: 64 values per lane
    (14, 2048, 37984, 2),  # shards straddle super-blocks
    (12, 2048, 11008, 4),
    (13, 512, 4160, 2),
])
def test_allgather_kernel_single_rank(qt, K, N, world):
    """The all-gather kernel run as rank 0 of 1 for each shard of a
    `world`-way split: the shard's columns land in the output at their
    global offset and match the oracle; the other columns stay untouched."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    wq = synth.weights(qt, K, N, seed=K + N + world)
    w = vt.QuantWeight(qt, K, N, wq)
    wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    _, bounds = vt.shard_columns(N, world)
    m_max = 4
    out, _ = vkq.ipc_alloc(m_max * N * 4)
    flags, _ = vkq.ipc_alloc(256)
    sync, _ = vkq.ipc_alloc(256)
    try:
        peer_out = torch.tensor([out], dtype=torch.int64, device="cuda")
        peer_flags = torch.tensor([flags], dtype=torch.int64, device="cuda")
        Y = torch.as_tensor(vt._DeviceArray(out, (m_max, N)), device="cuda")
        for M in (1, 3):
            for lo, hi in bounds:
                x = synth.activations(M, K, seed=M * 7 + lo)
                xt = torch.from_numpy(x).cuda()
                ws = vt.workspace(vt.workspace_bytes(qt, M, K, hi - lo, 0), 0)
                Y.fill_(123.0)
                vkq.gemv_allgather(qt, w.buf.data_ptr(), w.nbytes, K, N, lo, hi, xt.data_ptr(), M,
                                   peer_out.data_ptr(), peer_flags.data_ptr(), sync, 1, 0, ws.data_ptr(),
                                   ws.numel(), device=0)
                torch.cuda.synchronize()
                y = Y[:M].cpu().numpy()
                err = helpers.matmul_error(y[:, lo:hi], x, wd[:, lo:hi])
                assert err <= helpers.GEMV_TOL, (qt, K, N, M, lo, hi, err)
                assert (y[:, :lo] == 123.0).all() and (y[:, hi:] == 123.0).all()
        assert vkq.device_status(0) == vkq.OK
    finally:
        torch.cuda.synchronize()
        for p in (out, flags, sync):
            vkq.ipc_free(p)
