"""vkq_matmul_upstream: the decode GEMV for weights in the upstream GGUF
orientation ([out][in]: row n of the weight is the K/256 super-blocks of
output n, W[n][k] = value n*K + k of the stream), against float64 products of
the oracle's dequantized weights read in that orientation.  Parity bar: each
output within 1e-5 of sum_k |x_k W_nk|, as for the other fp32 GEMVs."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _upstream(qt, K, N, wq, x):
    import torch
    from vibrant_b200 import vkq
    w = torch.from_numpy(np.ascontiguousarray(wq, dtype=np.uint8)).cuda()
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    M = x.shape[0]
    y = torch.full((M, N), float("nan"), device="cuda")
    vkq.matmul_upstream(qt, w.data_ptr(), w.numel(), K, N, xt.data_ptr(), M, y.data_ptr(), device=0)
    torch.cuda.synchronize()
    assert vkq.device_status(0) == vkq.OK
    return y.cpu().numpy()


def _check(oracle, qt, K, N, wq, x, y):
    w = oracle.dequantize(qt, wq)[:K * N].reshape(N, K).astype(np.float64)  # [out][in]
    x64 = x.astype(np.float64)
    ref = x64 @ w.T
    bound = np.abs(x64) @ np.abs(w).T
    err = float(np.max(np.abs(y.astype(np.float64) - ref) / np.maximum(bound, 1e-300)))
    assert err <= helpers.GEMV_TOL, err


@pytest.mark.parametrize("qt,K,N,M", [
    (12, 2048, 11008, 1),    # the 3B gate/up projection as GGUF stores it
    (13, 2048, 1024, 2),
    (14, 11008, 2048, 1),    # Q6_K down projection: 9,030-byte rows, only 2-byte aligned
    (14, 2048, 4096, 3),
    (12, 256, 512, 5),       # one block per row; five rows of x = two launches
    (12, 5120, 1024, 4),
    (13, 768, 300, 8),
    (14, 512, 33, 1),
], ids=lambda v: str(v))
def test_upstream_matches_oracle(oracle, qt, K, N, M):
    from vibrant_b200 import synth
    wq = synth.weights(qt, K, N, seed=K + 3 * N + M)
    x = synth.activations(M, K, seed=M + 5)
    y = _upstream(qt, K, N, wq, x)
    assert np.isfinite(y).all()
    _check(oracle, qt, K, N, wq, x, y)


def test_upstream_realistic_weights(oracle):
    """Gaussian weights quantized with per-sub-block scales and (negative)
    mins, as real Q4_K files hold them."""
    K, N = 2048, 2048
    rng = np.random.default_rng(21)
    wq = helpers.quantize_q4k_subblocks((rng.standard_normal(K * N) * 0.02).astype(np.float32))
    x = (rng.standard_normal((2, K)) * 3).astype(np.float32)
    y = _upstream(12, K, N, wq, x)
    _check(oracle, 12, K, N, wq, x, y)


def test_upstream_is_the_transposed_vibrant_product():
    """The same bytes read as [N][K] give W^T x: vkq_matmul_upstream with
    (K, N) equals the float64 product of vibrant's orientation with the
    dimensions swapped, computed from vkq_dequantize_f32."""
    import torch
    from vibrant_b200 import synth, vkq
    qt, K, N = 12, 1024, 768
    wq = synth.weights(qt, K, N, seed=2)
    w = torch.from_numpy(wq).cuda()
    deq = torch.empty(vkq.weight_bytes(qt, K, N) // 144 * 256, device="cuda")
    vkq.dequantize_f32(qt, w.data_ptr(), deq.numel() // 256, deq.data_ptr(), device=0)
    x = torch.from_numpy(synth.activations(1, K, seed=3)).cuda()
    y = torch.empty(1, N, device="cuda")
    vkq.matmul_upstream(qt, w.data_ptr(), w.numel(), K, N, x.data_ptr(), 1, y.data_ptr(), device=0)
    torch.cuda.synchronize()
    wt = deq[:K * N].view(N, K).double()
    ref = (wt @ x.double().view(K)).view(1, N)
    bound = (wt.abs() @ x.double().abs().view(K)).view(1, N)
    assert float(((y.double() - ref).abs() / bound).max()) <= helpers.GEMV_TOL


def test_upstream_error_paths():
    import torch
    from vibrant_b200 import vkq
    K, N = 512, 256
    w = torch.zeros(vkq.weight_bytes(12, K, N), dtype=torch.uint8, device="cuda")
    x = torch.zeros(2, K, device="cuda")
    y = torch.zeros(2, N, device="cuda")
    with pytest.raises(vkq.VkqError) as e:  # K not a whole number of blocks per row
        vkq.matmul_upstream(12, w.data_ptr(), w.numel(), 300, N, x.data_ptr(), 1, y.data_ptr(), device=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    with pytest.raises(vkq.VkqError) as e:  # x not 16-byte aligned
        vkq.matmul_upstream(12, w.data_ptr(), w.numel(), K, N, x.data_ptr() + 4, 1, y.data_ptr(), device=0)
    assert e.value.status == vkq.ERR_MISALIGNED
    with pytest.raises(vkq.VkqError) as e:  # weight buffer too small
        vkq.matmul_upstream(12, w.data_ptr(), w.numel() - 144, K, N, x.data_ptr(), 1, y.data_ptr(), device=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    with pytest.raises(vkq.VkqError) as e:
        vkq.matmul_upstream(11, w.data_ptr(), w.numel(), K, N, x.data_ptr(), 1, y.data_ptr(), device=0)
    assert e.value.status == vkq.ERR_UNSUPPORTED
    assert vkq.device_status(0) == vkq.OK
