"""The steps between the linear layers of a decode step (vkq_silu_mul,
vkq_rms_norm) against a float64 restatement of the reference kernels
(internal/gpu/cuda/kernels.cu:209-288, 306-341), through the C ABI; and the
device-side row-block shard builder against vkq_shard_weight."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [11008, 27648, 4, 1000])
def test_silu_mul_matches_reference_formula(n):
    import torch
    from vibrant_b200 import vkq
    g = torch.randn(n, device="cuda") * 4
    u = torch.randn(n, device="cuda")
    out = torch.empty(n, device="cuda")
    vkq.silu_mul(g.data_ptr(), u.data_ptr(), out.data_ptr(), n, device=0)
    torch.cuda.synchronize()
    g64, u64 = g.double().cpu(), u.double().cpu()
    ref = g64 / (1.0 + torch.exp(-g64)) * u64
    err = ((out.double().cpu() - ref).abs() / (ref.abs() + 1e-30)).max().item()
    assert err < 2e-6, err
    assert vkq.device_status(0) == vkq.OK


@pytest.mark.parametrize("rows,n", [(1, 2048), (3, 5120), (2, 1000)])
def test_rms_norm_matches_reference_formula(rows, n):
    import torch
    from vibrant_b200 import vkq
    x = torch.randn(rows, n, device="cuda") * 3
    w = torch.rand(n, device="cuda") + 0.5
    out = torch.empty(rows, n, device="cuda")
    vkq.rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, n, 1e-6, device=0)
    torch.cuda.synchronize()
    x64 = x.double().cpu()
    ref = x64 / torch.sqrt((x64 * x64).mean(dim=1, keepdim=True) + 1e-6) * w.double().cpu()
    err = ((out.double().cpu() - ref).abs() / (ref.abs() + 1e-30)).max().item()
    assert err < 2e-6, err
    assert vkq.device_status(0) == vkq.OK


def test_silu_mul_rejects_misaligned_buffers():
    import torch
    from vibrant_b200 import vkq
    a = torch.zeros(64, device="cuda")
    with pytest.raises(vkq.VkqError) as e:
        vkq.silu_mul(a.data_ptr() + 4, a.data_ptr(), a.data_ptr(), 8, device=0)
    assert e.value.status == vkq.ERR_MISALIGNED


@pytest.mark.parametrize("qt,K,N,world", [(14, 64, 151936, 8), (12, 96, 11008, 3), (12, 40, 27648, 8)])
def test_device_shards_equal_host_shards(qt, K, N, world):
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    full = synth.weights_device(qt, K, N, seed=5, device="cuda")
    host = full.cpu().numpy()
    for r in range(world):
        lo, hi = vkq.shard_columns(N, world, r)
        dev = vt.shard_device(full, qt, K, N, lo, hi).cpu().numpy()
        assert np.array_equal(dev, vkq.shard_weight(qt, host, K, N, lo, hi))
