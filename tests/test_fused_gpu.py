"""vkq_linear_fused: the fused linears of a decode step (several Q4_K
weights over one input, the RMSNorm prologue, the SiLU(gate) * up
epilogue) against float64 products of the oracle's dequantized weights.

Parity bar: each output within 1e-5 of sum_k |h_k W_kn| (the GEMV metric on
the normalised input h); the SiLU product within 1e-5 of the first-order
error bound |SiLU'(g)| sum|h W_g| |u| + |SiLU(g)| sum|h W_u|."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


def _weight(oracle, qt, K, N, seed, gaussian):
    from vibrant_b200 import synth
    if gaussian:  # every sub-block with its own scale and (negative) min
        rng = np.random.default_rng(seed)
        wq = helpers.quantize_q4k_subblocks((rng.standard_normal(K * N) * 0.02).astype(np.float32))
    else:
        wq = synth.weights(qt, K, N, seed=seed)
    return wq, oracle.dequantize(qt, wq)[:K * N].reshape(K, N).astype(np.float64)


def _rms(x, g, eps):
    x64 = x.astype(np.float64)
    return x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + eps) * g.astype(np.float64)


def _run(oracle, shapes, M, norm, silu, seed=0, gaussian=False, eps=1e-6):
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    K = shapes[0][0]
    ws, wds = [], []
    for i, (_, N) in enumerate(shapes):
        wq, wd = _weight(oracle, 12, K, N, seed + 17 * i, gaussian)
        ws.append(vt.QuantWeight(12, K, N, wq))
        wds.append(wd)
    x = synth.activations(M, K, seed=seed + 5)
    g = (1.0 + 0.1 * np.random.default_rng(seed + 9).standard_normal(K)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    gt = torch.from_numpy(g).cuda() if norm else None
    outs = vt.linear_fused(xt, ws, norm_w=gt, eps=eps, silu_mul=silu)
    torch.cuda.synchronize()
    assert vkq.device_status(0) == vkq.OK
    h = _rms(x, g, eps) if norm else x.astype(np.float64)
    return [o.cpu().numpy().astype(np.float64) for o in outs], h, wds


def _check_linear(y, h, wd):
    ref = h @ wd
    bound = np.abs(h) @ np.abs(wd)
    err = np.max(np.abs(y - ref) / np.maximum(bound, 1e-300))
    assert err <= helpers.GEMV_TOL, err


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("M,gaussian", [(1, False), (1, True), (2, False), (3, True)])
def test_qkv_in_one_launch(oracle, M, norm, gaussian):
    """q, k and v of the 3B attention (2048 -> 2048, 256, 256) from one launch."""
    ys, h, wds = _run(oracle, [(2048, 2048), (2048, 256), (2048, 256)], M, norm, False, seed=M, gaussian=gaussian)
    for y, wd in zip(ys, wds):
        _check_linear(y, h, wd)


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("M,gaussian", [(1, False), (1, True), (2, True), (3, False)])
def test_gate_up_silu(oracle, M, norm, gaussian):
    """SiLU(h W_gate) * (h W_up) for the 3B FFN (2048 -> 11008), one launch."""
    K, N = 2048, 11008
    ys, h, (wg, wu) = _run(oracle, [(K, N), (K, N)], M, norm, True, seed=11 + M, gaussian=gaussian)
    gv, uv = h @ wg, h @ wu
    bg, bu = np.abs(h) @ np.abs(wg), np.abs(h) @ np.abs(wu)
    sig = 1.0 / (1.0 + np.exp(-gv))
    silu = gv * sig
    dsilu = sig * (1.0 + gv * (1.0 - sig))
    # SiLU as the reference computes it, in float32: x / (1 + expf(-x))
    # (internal/gpu/cuda/kernels.cu:330-341), which is -0 for x < -88.72
    # where expf overflows although the true value is still a float
    g32 = gv.astype(np.float32)
    with np.errstate(over="ignore"):
        silu32 = (g32 / (np.float32(1) + np.exp(-g32))).astype(np.float64)
    ref = silu32 * uv
    bound = np.abs(dsilu) * bg * np.abs(uv) + np.abs(silu) * bu
    err = np.max(np.abs(ys[0] - ref) / np.maximum(bound, 1e-300))
    assert err <= helpers.GEMV_TOL, err


@pytest.mark.parametrize("shapes", [[(4096, 256), (4096, 256), (4096, 512)], [(333, 768)], [(11008, 2048)]],
                         ids=["kv-like-4096", "ragged-K", "wide-K"])
def test_k_split_over_a_cluster_with_the_norm(oracle, shapes):
    """Narrow weights: the plan splits K over a cluster, whose CTAs add their
    sums (and their shares of sum x^2) through DSMEM."""
    ys, h, wds = _run(oracle, shapes, 1, True, False, seed=3)
    for y, wd in zip(ys, wds):
        _check_linear(y, h, wd)


def test_fused_is_deterministic():
    """Repeated fused calls give bitwise identical outputs (fixed-order sums)."""
    import torch
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    K = 2048
    ws = [vt.QuantWeight(12, K, n, synth.weights(12, K, n, seed=40 + n)) for n in (2048, 256, 256)]
    x = torch.from_numpy(synth.activations(1, K, seed=8)).cuda()
    a = [o.clone() for o in vt.linear_fused(x, ws)]
    b = vt.linear_fused(x, ws)
    torch.cuda.synchronize()
    for u, v in zip(a, b):
        assert torch.equal(u.view(torch.int32), v.view(torch.int32))


def test_error_paths():
    import torch
    from vibrant_b200 import vkq
    K, N = 256, 256
    buf = torch.zeros(vkq.weight_bytes(12, K, N), dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, K, device="cuda")
    y = torch.zeros(1, N, device="cuda")

    def call(**kw):
        a = dict(qtype=12, w=[buf.data_ptr()], wb=[buf.numel()], N=[N], y=[y.data_ptr()], M=1, epi=vkq.EPI_NONE)
        a.update(kw)
        vkq.linear_fused(a["qtype"], a["w"], a["wb"], K, a["N"], x.data_ptr(), a["M"], a["y"], epilogue=a["epi"],
                         device=0)

    for kw, status in [(dict(qtype=14), vkq.ERR_UNSUPPORTED), (dict(N=[128]), vkq.ERR_INVALID_ARGUMENT),
                       (dict(epi=vkq.EPI_SILU_MUL), vkq.ERR_INVALID_ARGUMENT),
                       (dict(M=5), vkq.ERR_INVALID_ARGUMENT), (dict(wb=[100]), vkq.ERR_INVALID_ARGUMENT),
                       (dict(w=[buf.data_ptr() + 8]), vkq.ERR_MISALIGNED)]:
        with pytest.raises(vkq.VkqError) as e:
            call(**kw)
        assert e.value.status == status, kw
    call()  # a valid call still works afterwards
    torch.cuda.synchronize()
    assert vkq.device_status(0) == vkq.OK
