"""vkq_gemv_noalloc: the GEMV for callers that cannot allocate device memory
(their allocator owns the whole device, or their memory plan is fixed before
they run).  Its split-K scratch is a fixed array inside the library, so the
call takes no workspace.  Checked through the C ABI against vkq_gemv on two
calls in a row (the second call sees whatever the first one left in the
shared array).  Kept in its own file so that pytest collects it last."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt,K,N,M", [(14, 2048, 151936 // 8, 1), (12, 2048, 11008, 1), (13, 512, 4096, 2),
                                      (12, 1024, 2304, 4), (14, 300, 96, 1)])
def test_noalloc_matches_gemv_twice(qt, K, N, M):
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt

    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    wq = synth.weights(qt, K, N, seed=K + N)
    w = vt.QuantWeight(qt, K, N, wq)
    st = torch.cuda.current_stream()
    ws = torch.zeros(max(1, vkq.matmul_workspace_bytes(qt, M, K, N, device=0)), dtype=torch.uint8, device="cuda")
    for call in range(2):
        x = torch.from_numpy(synth.activations(M, K, seed=call + 10)).cuda()
        y_ref = torch.empty(M, N, device="cuda")
        y_new = torch.full((M, N), float("nan"), device="cuda")
        vkq.gemv(qt, w.buf.data_ptr(), w.nbytes, K, N, x.data_ptr(), M, y_ref.data_ptr(), ws.data_ptr(),
                 ws.numel(), device=0, stream=st)
        vkq.gemv_noalloc(qt, w.buf.data_ptr(), w.nbytes, K, N, x.data_ptr(), M, y_new.data_ptr(), device=0,
                         stream=st)
        torch.cuda.synchronize()
        a, b = y_new.cpu().numpy(), y_ref.cpu().numpy()
        wf = np.frombuffer(wq, np.uint8)
        from oracle import kq_oracle
        wd = kq_oracle.dequantize(qt, wf)[:K * N].reshape(K, N)
        assert helpers.matmul_error(a, x.cpu().numpy(), wd, y_ref=b.astype(np.float64)) <= helpers.GEMV_TOL
        assert helpers.matmul_error(a, x.cpu().numpy(), wd) <= helpers.GEMV_TOL
    assert vkq.device_status(0) == vkq.OK


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_noalloc_scratch_covers_every_plan(qt):
    """The fixed 8 MiB scratch holds every GEMV plan on this device: the
    split-K partials are bounded by the grid (two CTAs per SM x 2 x M x the
    tile width, plus the 64 KiB counter head), whatever K and N are, so on a
    148-SM B200 the largest need (M = 8) is about 5.2 MB and the rejection
    path (VKQ_ERR_WORKSPACE, nothing launched) cannot be reached here.  The
    extreme shapes below check the bound and run through vkq_gemv_noalloc."""
    import torch
    from vibrant_b200 import synth, vkq
    limit = 8 << 20
    worst = 0
    for M in (1, 2, 4, 5, 8):
        for K, N in ((1, 1 << 20), (64, 262144), (65536, 256), (2048, 151936), (11008, 2048)):
            worst = max(worst, vkq.matmul_workspace_bytes(qt, M, K, N, device=0))
    assert 0 < worst <= limit, worst
    K, N, M = 64, 262144, 8
    w = torch.from_numpy(synth.weights(qt, K, N, seed=2)).cuda()
    x = torch.from_numpy(synth.activations(M, K, seed=3)).cuda()
    y = torch.full((M, N), float("nan"), device="cuda")
    vkq.gemv_noalloc(qt, w.data_ptr(), w.numel(), K, N, x.data_ptr(), M, y.data_ptr(), device=0)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all().item()
    assert vkq.device_status(0) == vkq.OK
