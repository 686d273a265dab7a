"""Bit-exact parity of the dequantization kernels with the oracle (and the
golden fixtures): every non-NaN value identical, NaN where the reference
gives NaN."""
import os

import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def tvk():
    import torch
    from vibrant_b200 import tensor as vt
    assert torch.cuda.is_available()
    return torch, vt


def _gpu_dequant(tvk, qt, data, offset=0):
    torch, vt = tvk
    from vibrant_b200 import vkq
    nb = data.size // helpers.BLOCK_BYTES[qt]
    buf = torch.zeros(data.size + 64, dtype=torch.uint8, device="cuda")
    buf[offset:offset + data.size] = torch.from_numpy(data).cuda()
    out = torch.empty(nb * 256, dtype=torch.float32, device="cuda")
    vkq.dequantize_f32(qt, buf.data_ptr() + offset, nb, out.data_ptr(), device=0,
                       stream=torch.cuda.current_stream())
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("name,qt", [("q4k", 12), ("q5k", 13), ("q6k", 14)])
def test_dequant_matches_golden(tvk, name, qt):
    f = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    got = _gpu_dequant(tvk, qt, f["blocks"])
    assert np.all(helpers.same_f32(got, f["f32_bits"].view(np.float32)))


@pytest.mark.parametrize("qt", [12, 13, 14])
@pytest.mark.parametrize("offset", [0, 1, 2, 6])
def test_dequant_random_bytes_any_alignment(tvk, oracle, qt, offset):
    rng = np.random.default_rng(100 + qt + offset)
    data = rng.integers(0, 256, 3001 * helpers.BLOCK_BYTES[qt], dtype=np.uint8)
    got = _gpu_dequant(tvk, qt, data, offset)
    ref = oracle.dequantize(qt, data)
    assert np.all(helpers.same_f32(got, ref))


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_dequant_synthetic_weights(tvk, oracle, qt):
    from vibrant_b200 import synth
    data = synth.weights(qt, 512, 2048, seed=7)
    got = _gpu_dequant(tvk, qt, data)
    assert np.array_equal(got.view(np.uint32), oracle.dequantize(qt, data).view(np.uint32))


@pytest.mark.parametrize("qt,K,N", [(12, 256, 256), (13, 256, 256), (14, 256, 256), (14, 96, 640),
                                    (12, 130, 96), (13, 7, 300), (14, 4, 96)])
def test_dequant_transpose_matches_oracle(tvk, oracle, qt, K, N):
    # dequant_transpose.go:15-157, including the unexpanded trailing partial block
    torch, vt = tvk
    from vibrant_b200 import synth
    data = synth.random_bytes(qt, K, N, seed=K * N + qt)
    # keep d/dmin finite so that equality is informative everywhere
    bb = helpers.BLOCK_BYTES[qt]
    blocks = data.reshape(-1, bb)
    dpos = [208] if qt == 14 else [0, 2]
    for p in dpos:
        blocks[:, p + 1] &= 0x3B
    w = vt.QuantWeight(qt, K, N, data)
    got = vt.dequant_transpose(w)
    torch.cuda.synchronize()
    ref = oracle.dequant_transpose(qt, data, K, N)
    assert got.shape == (N, K)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))
