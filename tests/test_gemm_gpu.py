"""Parity of the bf16 tensor-core GEMM (vkq_gemm, and vkq_matmul for M > 8)
with the oracle: max |y - y_ref| / sum_k |x_k W_kn| <= 2e-2, through the C ABI."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tvk():
    import torch
    from vibrant_b200 import tensor as vt
    assert torch.cuda.is_available()
    return torch, vt


def run(tvk, qt, K, N, wq, x, path):
    torch, vt = tvk
    w = vt.QuantWeight(qt, K, N, wq)
    y = vt.matmul(torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda(), w, path=path)
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_gemm_exact_small_integers(tvk, qt):
    # integers in bf16 range: products and sums exact in fp32 -> identical
    K, N, M = 128, 256, 16
    rng = np.random.default_rng(qt)
    lo, hi = (-32, 31) if qt == 14 else (0, 15 if qt == 12 else 31)
    vals = rng.integers(lo, hi + 1, K * N)
    wq = helpers.encode_q6k_exact(vals) if qt == 14 else helpers.encode_q45k_exact(vals, qt)
    x = rng.integers(-4, 5, (M, K)).astype(np.float32)
    y = run(tvk, qt, K, N, wq, x, "gemm")
    ref = x.astype(np.int64) @ vals.reshape(K, N).astype(np.int64)
    assert np.array_equal(y, ref.astype(np.float32))


SHAPES = [
    (13, 64, 512, 1024),     # one k-step group, one CTA row
    (12, 16, 256, 256),      # smallest tile
    (14, 300, 256, 640),     # N % 256 == 128 (blocks straddle rows), M between 256 and 512
    (13, 512, 2048, 1024),   # two accumulators
    (12, 1000, 512, 2048),   # two CTA rows along M
    (14, 9, 1024, 4096),     # M just above the GEMV range, via vkq_matmul
    (13, 130, 200, 96),      # K not a multiple of 64, N < 128
]


@pytest.mark.parametrize("qt,M,K,N", SHAPES, ids=lambda v: str(v))
def test_gemm_matches_oracle(tvk, oracle, qt, M, K, N):
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=M + K + N)
    x = synth.activations(M, K, seed=M)
    y = run(tvk, qt, K, N, wq, x, "auto")
    w = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, x, w) <= helpers.GEMM_TOL
    # and a 1e-5-class check against bf16-rounded operands: the only error is
    # the rounding of x and W to bf16
    err = helpers.matmul_error(y, x, w)
    assert err < 5e-3


def test_gemm_prefill_full_size_spot_rows(tvk, oracle):
    # Q5_K prefill GEMM 512 x 2048 x 11008; all outputs checked against the
    # bf16-operand float64 product, 24 rows against the exact float64 product
    from vibrant_b200 import synth
    wl = synth.WORKLOADS["q5k_prefill_gemm_512x2048x11008"]
    qt, K, N, M = wl["qtype"], wl["K"], wl["N"], wl["M"]
    wq = synth.weights(qt, K, N, seed=wl["seed"])
    x = synth.activations(M, K, seed=77)
    y = run(tvk, qt, K, N, wq, x, "auto")
    w = oracle.dequantize(qt, wq).reshape(K, N)
    rows = np.random.default_rng(5).choice(M, 24, replace=False)
    assert helpers.matmul_error(y[rows], x[rows], w) <= helpers.GEMM_TOL
    assert np.isfinite(y).all()


def test_matmul_dispatch_unaligned_shapes_fall_back_to_gemv(tvk, oracle):
    # N % 32 != 0: the tensor-core kernel does not serve it; vkq_matmul runs
    # the fp32 GEMV over 8-row chunks (so the 1e-5 bar applies)
    from vibrant_b200 import synth
    qt, M, K, N = 12, 20, 64, 100
    wq = synth.weights(qt, K, N, seed=3)
    x = synth.activations(M, K, seed=4)
    y = run(tvk, qt, K, N, wq, x, "auto")
    w = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    assert helpers.matmul_error(y, x, w) <= helpers.GEMV_TOL


def test_gemm_status_clean(tvk):
    from vibrant_b200 import vkq
    assert vkq.device_status(0) == vkq.OK


def test_gemm_then_gemv_share_one_workspace(tvk):
    # a GEMM call must leave a shared workspace ready for a GEMV call (whose
    # split-K tile counters live at its head and must be zero)
    torch, vt = tvk
    from vibrant_b200 import synth, vkq
    qt, K, N = 12, 512, 2048
    rng = np.random.default_rng(11)
    vals = rng.integers(0, 16, K * N)
    w = vt.QuantWeight(qt, K, N, helpers.encode_q45k_exact(vals, qt))
    need = max(vt.workspace_bytes(qt, 600, K, N, 0), vt.workspace_bytes(qt, 1, K, N, 0))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    xg = torch.from_numpy(synth.activations(600, K, seed=5)).cuda()
    x1 = rng.integers(-8, 9, (1, K)).astype(np.float32)
    ref = (x1.astype(np.int64) @ vals.reshape(K, N).astype(np.int64)).astype(np.float32)
    for _ in range(2):
        vt.matmul(xg, w, ws=ws, path="gemm")
        y1 = vt.matmul(torch.from_numpy(x1).cuda(), w, ws=ws)
        torch.cuda.synchronize()
        assert np.array_equal(y1.cpu().numpy(), ref)
    assert vkq.device_status(0) == vkq.OK
