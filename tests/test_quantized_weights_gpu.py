"""Parity on weights that look like real k-quant weights: Gaussian data
quantized by the reference's own test quantizers (QuantizeQ4_K,
internal/tensor/quant_q4k.go:215-282; QuantizeQ6_K, quant_q6k.go:214-294,
restated in the oracle), and for Q4_K also by the per-sub-block quantizer of
the test helpers (the reference's QuantizeQ4_K sets sub-block 0's scale and
min only).  Q6_K quants then cluster around the zero point q = 32 (the case
where a GEMV that accumulates a*q and subtracts 32*sum(a) loses the most),
and Q4_K sub-blocks carry negative mins, so d*sc*q and dmin*m cancel.

The three GEMV kernels (CUDA cores, tensor cores, Q4_K column strips) at
1e-5 of sum_k |x w| for M = 1..4, including row-straddling shapes
(N % 256 == 128), and the tensor-core GEMM at 2e-2 on every output of a
512-row prefill; plus activations of extreme magnitude."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _weights(oracle, qt, K, N, seed, sigma=0.02, quantizer="reference"):
    """Gaussian data quantized by the reference's test quantizer (restated in
    the oracle), or for Q4_K by the per-sub-block quantizer of the test
    helpers."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(K * N) * sigma).astype(np.float32)
    wq = helpers.quantize_q4k_subblocks(w) if quantizer == "subblock" else oracle.quantize(qt, w)
    wd = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    return wq, wd


@pytest.fixture(params=["simt", "tc", "strip"])
def path(request):
    from vibrant_b200 import vkq
    old = vkq.set_gemv_path(helpers.GEMV_PATHS[request.param])
    yield request.param
    vkq.set_gemv_path(old)


@pytest.mark.parametrize("qt,K,N,quantizer", [(14, 2048, 2048, "reference"), (12, 2048, 11008, "reference"),
                                              (12, 2048, 11008, "subblock"), (12, 5120, 1024, "subblock"),
                                              (14, 1024, 19072, "reference"), (14, 11008, 2048, "reference"),
                                              (12, 512, 4352, "reference"), (12, 256, 4352, "subblock")])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_gemv_on_quantized_gaussian_weights(oracle, path, qt, K, N, quantizer, M):
    import torch
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    wq, wd = _weights(oracle, qt, K, N, seed=K + N + qt, quantizer=quantizer)
    x = synth.activations(M, K, seed=M + K)
    w = vt.QuantWeight(qt, K, N, wq)
    y = vt.matmul(torch.from_numpy(x).cuda(), w).cpu().numpy()
    assert helpers.matmul_error(y, x, wd) <= helpers.GEMV_TOL
    from vibrant_b200 import vkq
    assert vkq.device_status(0) == vkq.OK


def test_q6k_quants_cluster_at_the_zero_point(oracle):
    """The premise of the test above: with Gaussian data the Q6_K quants
    cluster around 32 (d = max|x| / 32, so |q - 32| ~ 11 |x| / sigma)."""
    wq, _ = _weights(oracle, 14, 64, 1024, seed=1)
    b = wq.reshape(-1, 210)
    lo = np.stack([b[:, i // 2] >> (4 * (i % 2)) & 15 for i in range(256)], 1).astype(int)
    hi = np.stack([b[:, 128 + i // 4] >> (2 * (i % 4)) & 3 for i in range(256)], 1).astype(int)
    q = lo | (hi << 4)
    assert np.mean(np.abs(q - 32) <= 16) > 0.8 and np.mean(np.abs(q - 32) <= 4) > 0.25


@pytest.mark.parametrize("qt", [12, 14])
def test_gemm_full_size_prefill_every_output(oracle, qt):
    """The tcgen05 GEMM on quantized Gaussian weights, 512 x 2048 x 11008 (Q4_K)
    or 512 x 2048 x 2048 (Q6_K): every one of the M x N outputs within 2e-2."""
    import torch
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    K, N, M = 2048, (11008 if qt == 12 else 2048), 512
    wq, wd = _weights(oracle, qt, K, N, seed=77 + qt)
    x = synth.activations(M, K, seed=5)
    w = vt.QuantWeight(qt, K, N, wq)
    y = vt.matmul(torch.from_numpy(x).cuda(), w, path="gemm").cpu().numpy()
    assert np.isfinite(y).all()
    assert helpers.matmul_error(y, x, wd) <= helpers.GEMM_TOL


@pytest.mark.parametrize("kernel", ["simt", "tc", "strip", "gemm"])
def test_extreme_activation_magnitudes(oracle, kernel):
    """Activations from 1e-30 to 1e20 (the GEMM scales x by 2^49 before its
    bf16 conversion, which stays finite below 2^79 ~ 6e23)."""
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    qt, K, N = 12, 512, 2048
    wq = synth.weights(qt, K, N, seed=3)
    wd = oracle.dequantize(qt, wq)[:K * N].reshape(K, N)
    M = 16 if kernel == "gemm" else 2
    x = synth.activations(M, K, seed=4)
    x[:, ::7] *= np.float32(1e20)
    x[:, 3::7] *= np.float32(1e-30)
    w = vt.QuantWeight(qt, K, N, wq)
    old = vkq.set_gemv_path(helpers.GEMV_PATHS.get(kernel, vkq.GEMV_SIMT))
    try:
        y = vt.matmul(torch.from_numpy(x).cuda(), w, path="gemm" if kernel == "gemm" else "auto").cpu().numpy()
    finally:
        vkq.set_gemv_path(old)
    assert np.isfinite(y).all()
    tol = helpers.GEMM_TOL if kernel == "gemm" else helpers.GEMV_TOL
    assert helpers.matmul_error(y, x, wd) <= tol
