"""Row-sharded GEMV with the all-gather fused into the kernel through peer
memory (vkq_gemv_allgather / vkq_gemv_sharded / vkq_linear_fused_allgather).

Each rank holds only its row-block shard of the weight (vkq_shard_weight),
computes its columns and sends them to every other rank as flagged words
(value and call number in one 64-bit store) over NVLink; each rank copies
the other ranks' columns from its channel slots into its own output. After
each call every rank's output must equal the full product within the GEMV
tolerance (1e-5 of sum_k |x w|), for consecutive calls of different M and
for weights whose N is not a multiple of 256 (super-blocks straddle the rows
and the shards).

* one GPU: each kernel as rank 0 of 1 for every shard of a world-way split
  (the fused q|k|v and gate|up forms included); the channel with a second
  rank that never arrives (slots that nothing fills): the waits run out
  after VKQ_PEER_WAIT_MS, the status is VKQ_ERR_DEVICE_TIMEOUT, nothing is
  stored into the absent rank's output, the next call fails at once with
  VKQ_ERR_PEER, a slot of a later call is refused at once, and a reset
  channel works again;
* two GPUs: one process per GPU over CUDA IPC (plain and fused forms on the
  same channels), and one process driving both GPUs (vkq_comm_init);
  skipped on a box with fewer GPUs.
"""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("qt,K,N,world", [
    (14, 256, 151936, 2),  # wide shards: 64 values per lane; rows straddle blocks
    (14, 2048, 37984, 3),  # shards straddle super-blocks
    (12, 2048, 11008, 4),
    (12, 2048, 11008, 8),  # column-strip all-gather, shard offsets of 32 .. 224 values into a block
    (12, 5120, 1024, 2),
    (13, 512, 4160, 2),
    (14, 2048, 151936, 8),
])
@pytest.mark.parametrize("path", ["auto", "simt"])
def test_allgather_kernel_single_rank(qt, K, N, world, path):
    """The all-gather kernel run as rank 0 of 1 on each rank's shard of a
    `world`-way split: the shard's columns land in the output at their
    global offset and match the oracle; the other columns stay untouched.
    (Automatic choice: the column-strip all-gather for Q4_K shards of
    N % 256 == 0 weights, the CUDA-core one otherwise.)"""
    import torch
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    if path == "simt" and qt != 12:
        pytest.skip("the automatic choice is the CUDA-core kernel already")
    old_path = vkq.set_gemv_path(vkq.GEMV_SIMT if path == "simt" else vkq.GEMV_AUTO)
    wq = synth.weights(qt, K, N, seed=K + N + world)
    wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    m_max = 4
    out, _ = vkq.ipc_alloc(m_max * N * 4)
    flags, _ = vkq.ipc_alloc(256)
    sync, _ = vkq.ipc_alloc(256)
    try:
        Y = torch.as_tensor(vt._DeviceArray(out, (m_max, N)), device="cuda")
        for M in (1, 3):
            for r in range(world):
                sh = vt.ShardedWeight(qt, K, N, world, r, wq)
                lo, hi = sh.lo, sh.hi
                x = synth.activations(M, K, seed=M * 7 + lo)
                xt = torch.from_numpy(x).cuda()
                ws = vt.workspace(vt.workspace_bytes(qt, M, K, hi - lo, 0), 0)
                Y.fill_(123.0)
                vkq.gemv_allgather(qt, sh.buf.data_ptr(), sh.nbytes, K, N, lo, hi, xt.data_ptr(), M, [out], [flags],
                                   sync, 1, 0, ws.data_ptr() if ws is not None else None,
                                   ws.numel() if ws is not None else 0, device=0)
                torch.cuda.synchronize()
                y = Y[:M].cpu().numpy()
                err = helpers.matmul_error(y[:, lo:hi], x, wd[:, lo:hi])
                assert err <= helpers.GEMV_TOL, (qt, K, N, M, lo, hi, err)
                assert (y[:, :lo] == 123.0).all() and (y[:, hi:] == 123.0).all()
        assert vkq.device_status(0) == vkq.OK
    finally:
        torch.cuda.synchronize()
        vkq.set_gemv_path(old_path)
        for p in (out, flags, sync):
            vkq.ipc_free(p)


def _rms64(x, g, eps=1e-6):
    x64 = x.astype(np.float64)
    return x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + eps) * g.astype(np.float64)


def _silu32_ref(h, wg, wu):
    """SiLU(h W_g) * (h W_u) with SiLU in float32 as the reference computes it
    (x / (1 + expf(-x)), internal/gpu/cuda/kernels.cu:330-341), and the
    first-order error bound of the product."""
    gv, uv = h @ wg, h @ wu
    sig = 1.0 / (1.0 + np.exp(-gv))
    g32 = gv.astype(np.float32)
    with np.errstate(over="ignore"):
        silu32 = (g32 / (np.float32(1) + np.exp(-g32))).astype(np.float64)
    bound = (np.abs(sig * (1.0 + gv * (1.0 - sig))) * (np.abs(h) @ np.abs(wg)) * np.abs(uv)
             + np.abs(gv * sig) * (np.abs(h) @ np.abs(wu)))
    return silu32 * uv, bound


@pytest.mark.parametrize("world", [2, 4])
def test_fused_allgather_kernel_single_rank(world):
    """vkq_linear_fused_allgather run as rank 0 of 1 on each rank's shards of
    a `world`-way split: q's shard columns (beside whole k and v) and the
    SiLU(gate) * up shard land at their global offset, with the RMSNorm
    prologue, and match float64 products of the oracle's weights."""
    import torch
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    K, Nq, Nkv, Nf, M = 2048, 2048, 256, 11008, 1
    cols = {"q": Nq, "k": Nkv, "v": Nkv, "g": Nf, "u": Nf}
    w = {n: synth.weights(12, K, c, seed=c + i) for i, (n, c) in enumerate(cols.items())}
    wd = {n: kq_oracle.dequantize(12, w[n])[:K * c].reshape(K, c).astype(np.float64) for n, c in cols.items()}
    x = synth.activations(M, K, seed=7)
    g = (1.0 + 0.1 * np.random.default_rng(8).standard_normal(K)).astype(np.float32)
    h = _rms64(x, g)
    xt, gt = torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda()
    kw, vw = vt.QuantWeight(12, K, Nkv, w["k"]), vt.QuantWeight(12, K, Nkv, w["v"])
    for N, names in ((Nq, ("q",)), (Nf, ("g", "u"))):
        out, _ = vkq.ipc_alloc(M * N * 4)
        chan, _ = vkq.ipc_alloc(vkq.gather_channel_bytes(M, N))
        sync, _ = vkq.ipc_alloc(256)
        try:
            Y = torch.as_tensor(vt._DeviceArray(out, (M, N)), device="cuda")
            for r in range(world):
                sh = [vt.ShardedWeight(12, K, N, world, r, w[n]) for n in names]
                lo, hi = sh[0].lo, sh[0].hi
                Y.fill_(123.0)
                if names == ("q",):
                    ko, vo = torch.empty(M, Nkv, device="cuda"), torch.empty(M, Nkv, device="cuda")
                    vkq.linear_fused_allgather(12, [sh[0].buf.data_ptr(), kw.buf.data_ptr(), vw.buf.data_ptr()],
                                               [sh[0].nbytes, kw.nbytes, vw.nbytes], K, N, lo, hi, [0, Nkv, Nkv],
                                               xt.data_ptr(), M, [0, ko.data_ptr(), vo.data_ptr()], [out], [chan],
                                               sync, 1, 0, norm_w_ptr=gt.data_ptr(), device=0)
                    torch.cuda.synchronize()
                    for yy, name in ((ko, "k"), (vo, "v")):
                        assert helpers.matmul_error(yy.cpu().numpy(), h, wd[name]) <= helpers.GEMV_TOL
                    y = Y.cpu().numpy()
                    assert helpers.matmul_error(y[:, lo:hi], h, wd["q"][:, lo:hi]) <= helpers.GEMV_TOL
                else:
                    vkq.linear_fused_allgather(12, [sh[0].buf.data_ptr(), sh[1].buf.data_ptr()],
                                               [sh[0].nbytes, sh[1].nbytes], K, N, lo, hi, [], xt.data_ptr(), M, [],
                                               [out], [chan], sync, 1, 0, norm_w_ptr=gt.data_ptr(),
                                               epilogue=vkq.EPI_SILU_MUL, device=0)
                    torch.cuda.synchronize()
                    y = Y.cpu().numpy().astype(np.float64)
                    ref, bound = _silu32_ref(h, wd["g"][:, lo:hi], wd["u"][:, lo:hi])
                    assert np.max(np.abs(y[:, lo:hi] - ref) / np.maximum(bound, 1e-300)) <= helpers.GEMV_TOL
                assert (y[:, :lo] == 123.0).all() and (y[:, hi:] == 123.0).all()
            assert vkq.device_status(0) == vkq.OK
        finally:
            torch.cuda.synchronize()
            for ptr in (out, chan, sync):
                vkq.ipc_free(ptr)


_PROTOCOL_SCRIPT = textwrap.dedent("""
    import sys, time
    sys.path.insert(0, sys.argv[1])
    import numpy as np, torch
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    torch.cuda.set_device(0)
    path = int(sys.argv[2])
    vkq.set_gemv_path(path)  # 1: the CUDA-core all-gather; 0: automatic (Q4_K: column strips)
    qt, K, N, M = 12, 1024, 4096, 1
    wq = synth.weights(qt, K, N, seed=9)
    world = 2
    sh = vt.ShardedWeight(qt, K, N, world, 0, wq)
    x = torch.from_numpy(synth.activations(M, K, seed=1)).cuda()
    bufs = [vkq.ipc_alloc(M * N * 4)[0] for _ in range(world)]   # rank 1's buffer: nobody behind it
    chan = vkq.gather_channel_bytes(M, N)
    flags = [vkq.ipc_alloc(chan)[0] for _ in range(world)]
    sync = vkq.ipc_alloc(256)[0]
    Y = [torch.as_tensor(vt._DeviceArray(b, (M, N)), device="cuda") for b in bufs]
    F0 = torch.as_tensor(vt._DeviceArray(flags[0], (chan // 4,), "<u4"), device="cuda")
    S0 = torch.as_tensor(vt._DeviceArray(sync, (4,), "<u4"), device="cuda")
    ws = vt.workspace(max(vt.workspace_bytes(qt, M, K, sh.width, 0), vt.workspace_bytes(qt, M, K, N, 0)), 0)
    def call():
        vkq.gemv_allgather(qt, sh.buf.data_ptr(), sh.nbytes, K, N, sh.lo, sh.hi, x.data_ptr(), M, bufs, flags,
                           sync, world, 0, ws.data_ptr(), ws.numel(), device=0)
    Y[1].fill_(7.0)
    t0 = time.time(); call(); st = vkq.device_status(0); t1 = time.time()
    assert st == vkq.ERR_DEVICE_TIMEOUT, st
    assert 0.25 < t1 - t0 < 10.0, t1 - t0
    assert (Y[1] == 7.0).all().item(), "stored into the absent rank's buffer"
    assert torch.isfinite(Y[0][:, :sh.hi]).all().item()
    # the channel is marked failed: the next call fails at once, with no wait
    t0 = time.time(); call(); st = vkq.device_status(0); t1 = time.time()
    assert st == vkq.ERR_PEER, st
    assert t1 - t0 < 0.25, t1 - t0
    assert (Y[1] == 7.0).all().item()
    # reset; a slot of a later call (a rank ahead) is refused at once
    torch.cuda.synchronize(); F0.zero_(); S0.zero_(); torch.cuda.synchronize()
    F0[(256 + ((N - 1) * 2 + 1) * 8) // 4 + 1] = 3  # the slot of a rank-1 column carries call 3
    t0 = time.time(); call(); st = vkq.device_status(0); t1 = time.time()
    assert st == vkq.ERR_PEER, st
    assert t1 - t0 < 0.25, t1 - t0
    assert (Y[1] == 7.0).all().item()
    # reset; as rank 0 of 1 the same buffers work again
    torch.cuda.synchronize(); F0.zero_(); S0.zero_(); torch.cuda.synchronize()
    sh1 = vt.ShardedWeight(qt, K, N, 1, 0, wq)
    vkq.gemv_allgather(qt, sh1.buf.data_ptr(), sh1.nbytes, K, N, 0, N, x.data_ptr(), M, bufs[:1], flags[:1], sync,
                       1, 0, ws.data_ptr(), ws.numel(), device=0)
    assert vkq.device_status(0) == vkq.OK
    torch.cuda.synchronize()
    wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N).astype(np.float64)
    xv = x.cpu().numpy().astype(np.float64)
    err = np.max(np.abs(Y[0].cpu().numpy() - xv @ wd) / (np.abs(xv) @ np.abs(wd)))
    assert err <= 1e-5, ("reset channel", err)
    for p in bufs + flags + [sync]:
        vkq.ipc_free(p)
    print("protocol ok")
""")


@pytest.mark.parametrize("path", ["simt", "strip"])
def test_absent_peer_times_out_and_the_channel_fails_closed(path):
    """A second rank that never arrives (one GPU, a flag nothing sets), on
    the CUDA-core all-gather and on the column-strip one (the automatic
    choice for Q4_K shards with block-aligned rows)."""
    import torch
    assert torch.cuda.is_available()
    env = dict(os.environ, VKQ_PEER_WAIT_MS="300")
    r = subprocess.run([sys.executable, "-c", _PROTOCOL_SCRIPT, ROOT, "1" if path == "simt" else "0"], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "protocol ok" in r.stdout, r.stdout + r.stderr


def _rank_main(rank, world, port, cases):
    import datetime
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
        w = vt.ShardedWeight(qt, K, N, world, rank, wq, device=f"cuda:{rank}")
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
    # the fused linears of a sharded layer: q's shard gathered beside whole k
    # and v, and the gate|up shard pair with SiLU * up, alternating with
    # plain gathers on the same channels
    K, Nq, Nkv, Nf = 2048, 2048, 256, 11008
    cols = {"q": Nq, "k": Nkv, "v": Nkv, "g": Nf, "u": Nf}
    raw = {n: synth.weights(12, K, c, seed=3 * c + i) for i, (n, c) in enumerate(cols.items())}
    wd = {n: kq_oracle.dequantize(12, raw[n])[:K * c].reshape(K, c).astype(np.float64) for n, c in cols.items()}
    dev = f"cuda:{rank}"
    sq, sg, su = (vt.ShardedWeight(12, K, cols[n], world, rank, raw[n], device=dev) for n in ("q", "g", "u"))
    kw, vw = vt.QuantWeight(12, K, Nkv, raw["k"], device=dev), vt.QuantWeight(12, K, Nkv, raw["v"], device=dev)
    gq = vt.PeerGather(dist.group.WORLD, rank, world, rank, Nq, m_max=2)
    gf = vt.PeerGather(dist.group.WORLD, rank, world, rank, Nf, m_max=2)
    norm = torch.from_numpy((1.0 + 0.1 * np.random.default_rng(5).standard_normal(K)).astype(np.float32)).to(dev)
    for call, M in enumerate([1, 2, 1]):
        x = synth.activations(M, K, seed=50 + call)
        xt = torch.from_numpy(x).to(dev)
        h = _rms64(x, norm.cpu().numpy())
        q = gq.linear_fused(xt, [sq, kw, vw], norm_w=norm)
        torch.cuda.synchronize()
        assert helpers.matmul_error(q.cpu().numpy(), h, wd["q"]) <= helpers.GEMV_TOL, (rank, call, "q")
        act = gf.linear_fused(xt, [sg, su], norm_w=norm, silu_mul=True).cpu().numpy().astype(np.float64)
        ref, bound = _silu32_ref(h, wd["g"], wd["u"])
        assert np.max(np.abs(act - ref) / np.maximum(bound, 1e-300)) <= helpers.GEMV_TOL, (rank, call, "silu")
        y = gq.gemv(xt, sq)  # a plain gather on the same channel
        torch.cuda.synchronize()
        assert helpers.matmul_error(y.cpu().numpy(), x, wd["q"]) <= helpers.GEMV_TOL, (rank, call, "plain")
    assert vkq.device_status(rank) == vkq.OK
    gq.close()
    gf.close()
    dist.destroy_process_group()


def test_allgather_through_peer_memory_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    cases = [
        (14, 2048, 151936),        # Q6_K vocabulary projection: rows and shards straddle blocks
        (12, 2048, 11008),         # Q4_K FFN gate/up
        (13, 512, 4160),           # Q5_K, N % 256 == 64
    ]
    mp.spawn(_rank_main, args=(2, _free_port(), cases), nprocs=2, join=True)


def test_in_process_communicator_two_gpus():
    """One process drives both GPUs (vkq_comm_init / vkq_gemv_sharded)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    comm = vt.Comm([0, 1])
    try:
        for qt, K, N in [(14, 2048, 151936), (12, 2048, 11008), (13, 512, 4160)]:
            wq = synth.weights(qt, K, N, seed=K + N + 1)
            wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
            shards = comm.shards(qt, K, N, wq)
            for call, M in enumerate([1, 2, 1, 4]):
                x = synth.activations(M, K, seed=call + qt)
                xs = [torch.from_numpy(x).to(f"cuda:{d}") for d in comm.devices]
                ys = [torch.full((M, N), float("nan"), device=f"cuda:{d}") for d in comm.devices]
                for d in comm.devices:
                    torch.cuda.synchronize(d)
                comm.gemv(xs, shards, ys)
                for r, d in enumerate(comm.devices):
                    torch.cuda.synchronize(d)
                    err = helpers.matmul_error(ys[r].cpu().numpy(), x, wd)
                    assert err <= helpers.GEMV_TOL, (qt, K, N, call, M, r, err)
        for d in comm.devices:
            assert vkq.device_status(d) == vkq.OK
    finally:
        comm.close()
