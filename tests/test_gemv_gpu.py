"""Parity of the fp32-class GEMV (vkq_gemv / vkq_matmul with M <= 8) with the
oracle: max |y - y_ref| / sum_k |x_k W_kn| <= 1e-5, through the C ABI.  Every
test runs on both kernels (vkq_set_gemv_path): the CUDA-core kernel and the
tensor-core kernel (which serves M <= 4; larger M falls back to CUDA cores)."""
import glob
import os

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(params=["simt", "tc", "strip"], autouse=True)
def gemv_path(request):
    """Every test on each GEMV kernel (a kernel that does not serve a shape
    leaves it to the automatic choice)."""
    from vibrant_b200 import vkq
    old = vkq.set_gemv_path(helpers.GEMV_PATHS[request.param])
    yield request.param
    vkq.set_gemv_path(old)


@pytest.fixture(scope="module")
def tvk():
    import torch
    from vibrant_b200 import tensor as vt
    assert torch.cuda.is_available()
    return torch, vt


def run_gemv(tvk, qt, K, N, wq, x, path="auto"):
    torch, vt = tvk
    w = vt.QuantWeight(qt, K, N, wq)
    y = vt.matmul(torch.from_numpy(np.ascontiguousarray(x, np.float32).reshape(-1, K)).cuda(), w, path=path)
    torch.cuda.synchronize()
    return y.cpu().numpy()


# ---- known answers (tensor_cuda_test.go:218-318), each weight type ---------

@pytest.mark.parametrize("qt", [12, 13, 14])
def test_known_values_single_row(tvk, qt):
    # [1,2,3,4] @ [[1,2,3],[4,5,6],[7,8,9],[10,11,12]] = [70, 80, 90]
    vals = np.arange(1, 13)
    wq = helpers.encode_q6k_exact(vals) if qt == 14 else helpers.encode_q45k_exact(vals, qt)
    y = run_gemv(tvk, qt, 4, 3, wq, np.array([1, 2, 3, 4], np.float32))
    assert y.reshape(-1).tolist() == [70.0, 80.0, 90.0]


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_known_values_general(tvk, qt):
    # [[1,2,3],[4,5,6]] @ [[1,2],[3,4],[5,6]] = [[22,28],[49,64]]
    vals = np.arange(1, 7)
    wq = helpers.encode_q6k_exact(vals) if qt == 14 else helpers.encode_q45k_exact(vals, qt)
    y = run_gemv(tvk, qt, 3, 2, wq, np.array([[1, 2, 3], [4, 5, 6]], np.float32))
    assert y.reshape(-1).tolist() == [22.0, 28.0, 49.0, 64.0]


@pytest.mark.parametrize("qt", [12, 13, 14])
@pytest.mark.parametrize("K,N,M", [(64, 256, 1), (37, 1024, 1), (96, 640, 2), (200, 2304, 4), (16, 11008, 8)])
def test_exact_integer_products_fast_path(tvk, qt, K, N, M):
    # integer weights and activations: every partial sum is an exact float32
    # integer, so any summation order must give the same bits
    rng = np.random.default_rng(K * N + M + qt)
    hi = 31 if qt == 14 else (15 if qt == 12 else 31)
    lo = -32 if qt == 14 else 0
    vals = rng.integers(lo, hi + 1, K * N)
    wq = helpers.encode_q6k_exact(vals) if qt == 14 else helpers.encode_q45k_exact(vals, qt)
    x = rng.integers(-8, 9, (M, K)).astype(np.float32)
    y = run_gemv(tvk, qt, K, N, wq, x)
    ref = x.astype(np.int64) @ vals.reshape(K, N).astype(np.int64)
    assert np.array_equal(y, ref.astype(np.float32))


# ---- golden fixtures of the independent restatement ----------------------------

@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "matmul_*.npz"))), ids=os.path.basename)
def test_matches_golden_fixture(tvk, oracle, path):
    f = np.load(path)
    qt, K, N = int(f["qtype"]), int(f["K"]), int(f["N"])
    y = run_gemv(tvk, qt, K, N, f["wq"], f["x"]).reshape(-1)
    err = np.max(np.abs(y.astype(np.float64) - f["y64"]) / f["bound"])
    assert err <= helpers.GEMV_TOL
    # and against the reference-ordered float32 result of the fixture
    w = oracle.dequantize(qt, f["wq"])[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, f["x"], w, y_ref=f["y"].astype(np.float64)) <= 2 * helpers.GEMV_TOL


# ---- random shapes against the oracle's MatMul ---------------------------------

SHAPES = [
    (12, 2048, 11008, 1),   # 3B gate/up projection (full size)
    (12, 2048, 256, 1),     # k/v projection: one block column
    (14, 11008, 2048, 1),   # down projection
    (14, 512, 151936 // 8, 1),
    (14, 256, 1152, 1),     # N % 256 == 128: blocks straddle rows
    (13, 300, 1056, 1),     # N % 256 == 32
    (12, 5, 96, 1),         # N < 256
    (12, 1, 512, 1),        # K == 1
    (13, 2048, 11008, 2),
    (12, 1024, 2304, 3),
    (14, 768, 1280, 4),
    (13, 512, 4096, 5),
    (12, 2048, 2048, 8),
    (14, 33, 96, 7),
    (12, 5120, 1024, 2),    # 14B k/v projection, two rows
    (12, 333, 4096, 4),     # K split over a cluster with a ragged last range
    (12, 7, 256, 1),        # fewer rows than a cluster's CTAs would take
]


@pytest.mark.parametrize("qt,K,N,M", SHAPES, ids=lambda v: str(v))
def test_gemv_matches_oracle(tvk, oracle, qt, K, N, M):
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=K + N + M)
    x = synth.activations(M, K, seed=M * 7 + K)
    y = run_gemv(tvk, qt, K, N, wq, x)
    w = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, x, w) <= helpers.GEMV_TOL
    if (K * N) % 256 == 0:
        # the reference MatMul on a quantized B (GetOrDequantTranspose + dispatch)
        ref = oracle.matmul_quant(qt, x, wq, K, N, nthreads=8)
        assert helpers.matmul_error(y, x, w, y_ref=ref.astype(np.float64)) <= 2 * helpers.GEMV_TOL


@pytest.mark.parametrize("qt,K,N", [(12, 77, 832), (14, 9, 4000), (13, 5, 1000)])
def test_partial_tail_block(tvk, oracle, qt, K, N):
    # K*N % 256 != 0: the final super-block is partly used (Dequantize route,
    # internal/transformer/model.go:389-403)
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=5)
    x = synth.activations(1, K, seed=6)
    y = run_gemv(tvk, qt, K, N, wq, x)
    ref = oracle.matmul_dequant_untransposed(qt, x, wq, K, N)
    w = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, x, w) <= helpers.GEMV_TOL
    assert helpers.matmul_error(y, x, w, y_ref=ref.astype(np.float64)) <= 2 * helpers.GEMV_TOL


def test_lm_head_full_size(tvk, oracle):
    # Q6_K vocabulary projection 2048 -> 151936 against the LM-head route
    from vibrant_b200 import synth
    wl = synth.WORKLOADS["q6k_vocab_gemv_2048x151936"]
    qt, K, N = wl["qtype"], wl["K"], wl["N"]
    wq = synth.weights(qt, K, N, seed=wl["seed"])
    x = synth.activations(1, K, seed=99)
    y = run_gemv(tvk, qt, K, N, wq, x)
    w = oracle.dequantize(qt, wq).reshape(K, N)
    assert helpers.matmul_error(y, x, w) <= helpers.GEMV_TOL


@pytest.mark.parametrize("qt,K,N,M", [(12, 2048, 11008, 1), (14, 11008, 2048, 1), (12, 2048, 2048, 3),
                                      (14, 2048, 151936 // 2, 1)])
def test_deterministic_and_workspace_left_clean(tvk, qt, K, N, M):
    """Bitwise identical results on repeated calls (the split-K sums run in
    a fixed order, in one or two levels), and every split-K counter (the
    64 KiB head of the workspace) back at zero afterwards."""
    torch, vt = tvk
    from vibrant_b200 import synth, vkq
    w = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=1))
    x = torch.from_numpy(synth.activations(M, K, seed=2)).cuda()
    need = vkq.matmul_workspace_bytes(qt, M, K, N, device=0)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    y1 = vt.matmul(x, w, ws=ws).clone()
    y2 = vt.matmul(x, w, ws=ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))
    assert int(ws[: 64 * 1024].view(torch.int32).abs().sum()) == 0
    assert vkq.device_status(0) == vkq.OK


def test_side_stream_and_graph_capture(tvk):
    torch, vt = tvk
    from vibrant_b200 import synth
    qt, K, N = 14, 1024, 4096
    w = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=3))
    x = torch.from_numpy(synth.activations(1, K, seed=4)).cuda()
    ref = vt.matmul(x, w).clone()
    s = torch.cuda.Stream()
    out = torch.empty_like(ref)
    with torch.cuda.stream(s):
        vt.matmul(x, w, out=out)
    s.synchronize()
    assert torch.equal(out, ref)
    g = torch.cuda.CUDAGraph()
    out2 = torch.empty_like(ref)
    with torch.cuda.graph(g):
        vt.matmul(x, w, out=out2)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out2, ref)


def test_error_paths(tvk, gemv_path):
    torch, vt = tvk
    from vibrant_b200 import vkq
    K, N = 256, 256
    buf = torch.zeros(vkq.weight_bytes(12, K, N) + 32, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, K, device="cuda")
    y = torch.zeros(1, N, device="cuda")
    ws = torch.zeros(vkq.matmul_workspace_bytes(12, 1, K, N, device=0), dtype=torch.uint8, device="cuda")
    args = dict(device=0, stream=torch.cuda.current_stream())

    def call(**kw):
        a = dict(qtype=12, w=buf.data_ptr(), wb=buf.numel(), K=K, N=N, x=x.data_ptr(), M=1, y=y.data_ptr(),
                 ws=ws.data_ptr(), wsb=ws.numel())
        a.update(kw)
        vkq.matmul(a["qtype"], a["w"], a["wb"], a["K"], a["N"], a["x"], a["M"], a["y"], a["ws"], a["wsb"], **args)

    with pytest.raises(vkq.VkqError) as e:
        call(qtype=2)
    assert e.value.status == vkq.ERR_UNSUPPORTED
    with pytest.raises(vkq.VkqError) as e:
        call(K=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    with pytest.raises(vkq.VkqError) as e:
        call(wb=100)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    with pytest.raises(vkq.VkqError) as e:
        call(w=buf.data_ptr() + 8)
    assert e.value.status == vkq.ERR_MISALIGNED
    if gemv_path == "strip":
        call(ws=None, wsb=0)  # the column-strip kernel needs no workspace
    else:
        with pytest.raises(vkq.VkqError) as e:
            call(ws=None, wsb=0)
        assert e.value.status == vkq.ERR_WORKSPACE
        with pytest.raises(vkq.VkqError) as e:
            call(wsb=1024)  # below either kernel's need
        assert e.value.status == vkq.ERR_WORKSPACE
    with pytest.raises(vkq.VkqError) as e:
        call(x=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    call()  # and a valid call still works afterwards
    torch.cuda.synchronize()


def test_plans_of_different_tile_counts_share_one_workspace(tvk, oracle):
    # calls whose plans differ (M = 2: 512-wide tiles, M = 8: 256-wide tiles)
    # on one workspace: a call's split-K counters must start at zero whatever
    # the previous call left in the workspace (N = 37984 gives more than 128
    # of the 256-wide tiles)
    torch, vt = tvk
    from vibrant_b200 import synth, vkq
    qt, K, N = 14, 512, 37984
    wq = synth.weights(qt, K, N, seed=21)
    w = vt.QuantWeight(qt, K, N, wq)
    wd = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    Ms = [2, 8, 1, 4, 2, 8]
    ws = torch.zeros(max(vt.workspace_bytes(qt, M, K, N, 0) for M in Ms), dtype=torch.uint8, device="cuda")
    for i, M in enumerate(Ms):
        x = synth.activations(M, K, seed=30 + i)
        y = vt.matmul(torch.from_numpy(x).cuda(), w, ws=ws)
        torch.cuda.synchronize()
        assert helpers.matmul_error(y.cpu().numpy(), x, wd) <= helpers.GEMV_TOL, (i, M)
    assert vkq.device_status(0) == vkq.OK


@pytest.mark.parametrize("qt,K,N,M", [(13, 512, 1024, 1), (14, 512, 1280, 2), (12, 256, 2048, 3)])
def test_gemv_matches_sequential_fused_route(tvk, oracle, qt, K, N, M):
    """Against the reference's fused route MatMulQ5K / MatMulQ6K
    (internal/tensor/matmul_quant.go:30-191): a float32 sum over k in
    sequential order per output; the difference of summation orders stays
    within twice the GEMV bound."""
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=K * 3 + N)
    x = synth.activations(M, K, seed=M + 100)
    y = run_gemv(tvk, qt, K, N, wq, x)
    ref = oracle.matmul_quant_sequential(qt, x, wq, K, N)
    w = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, x, w, y_ref=ref.astype(np.float64)) <= 2 * helpers.GEMV_TOL


@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
@pytest.mark.parametrize("qt,K,N,M", [(12, 2048, 11008, 1), (14, 1024, 4096, 3), (13, 512, 768, 16),
                                      (12, 4, 256, 1), (14, 999, 1000, 2), (12, 600, 28672, 8)])
def test_matmul_host_matches_matmul(tvk, qt, K, N, M, pinned):
    """vkq_matmul_host (x from host memory, y back to it, one call) gives the
    bits vkq_matmul gives on device buffers: through the host mapping for
    pinned buffers (x read by a staging kernel, y stored by the GEMV; the
    28672-column case is above the 1 MiB limit for y at M = 8 and copies it),
    by cudaMemcpyAsync for pageable ones."""
    torch, vt = tvk
    from vibrant_b200 import synth, vkq
    w = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=K + N))
    x_host = torch.from_numpy(synth.activations(M, K, seed=M + 7))
    ref = vt.matmul(x_host.cuda(), w).cpu()
    y_host = torch.full((M, N), float("nan"))
    if pinned:
        x_host, y_host = x_host.pin_memory(), y_host.pin_memory()
    x_dev = torch.empty(M, K, device="cuda")
    y_dev = torch.empty(M, N, device="cuda")
    need = vkq.matmul_workspace_bytes(qt, M, K, N, device=0)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    vkq.matmul_host(qt, w.buf.data_ptr(), w.nbytes, K, N, x_host.data_ptr(), M, y_host.data_ptr(),
                    x_dev.data_ptr(), y_dev.data_ptr(), ws.data_ptr(), ws.numel(), device=0, stream=s)
    s.synchronize()
    assert torch.equal(y_host.view(torch.int32), ref.view(torch.int32))
    with pytest.raises(vkq.VkqError):
        vkq.matmul_host(qt, w.buf.data_ptr(), w.nbytes, K, N, 0, M, y_host.data_ptr(), x_dev.data_ptr(),
                        y_dev.data_ptr(), ws.data_ptr(), ws.numel(), device=0, stream=s)
    assert vkq.device_status(0) == vkq.OK
