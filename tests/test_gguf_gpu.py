"""The on-device GGUF loader: raw k-quant bytes (never expanded to float32)
and row-block shards uploaded through pinned staging, checked byte for byte
against the file and vkq_shard_weight, then used by the GEMV (end to end from
a file to a result checked against the oracle)."""
import numpy as np
import pytest

import helpers

pytestmark = pytest.mark.gpu

Q4_K, Q5_K, Q6_K, F32 = 12, 13, 14, 0


def _file(tmp_path):
    from vibrant_b200 import synth
    rng = np.random.default_rng(7)
    ts = [("blk.0.ffn_gate.weight", Q4_K, [2048, 1280], synth.weights(Q4_K, 2048, 1280, seed=11).tobytes()),
          ("output.weight", Q6_K, [512, 3968], synth.weights(Q6_K, 512, 3968, seed=12).tobytes()),
          ("blk.0.attn_v.weight", Q5_K, [256, 768], synth.weights(Q5_K, 256, 768, seed=13).tobytes()),
          ("output_norm.weight", F32, [2048], rng.standard_normal(2048).astype(np.float32).tobytes())]
    path = str(tmp_path / "m.gguf")
    helpers.write_gguf(path, ts)
    return path, ts


def test_load_tensors_raw(tmp_path):
    import torch
    from vibrant_b200 import vkq
    path, ts = _file(tmp_path)
    g = vkq.GGUF(path)
    try:
        for name, _, _, data in ts:
            i = g.find(name)
            buf = torch.full((len(data) + 64,), 0xAB, dtype=torch.uint8, device="cuda")
            g.load(i, buf.data_ptr(), buf.numel(), device=0)
            got = buf.cpu().numpy()
            assert got[:len(data)].tobytes() == data, name
            assert (got[len(data):] == 0xAB).all(), name
            with pytest.raises(vkq.VkqError):
                g.load(i, buf.data_ptr(), len(data) - 1, device=0)
    finally:
        g.close()


@pytest.mark.parametrize("name,world", [("blk.0.ffn_gate.weight", 2), ("blk.0.ffn_gate.weight", 3),
                                        ("output.weight", 2), ("output.weight", 4), ("blk.0.attn_v.weight", 3)])
def test_load_shards_match_the_host_shard(tmp_path, name, world):
    import torch
    from vibrant_b200 import vkq
    path, ts = _file(tmp_path)
    t, dims, data = next((t, d, b) for n, t, d, b in ts if n == name)
    K, N = dims
    g = vkq.GGUF(path)
    try:
        i = g.find(name)
        for r in range(world):
            lo, hi = vkq.shard_columns(N, world, r)
            ref = vkq.shard_weight(t, np.frombuffer(data, np.uint8), K, N, lo, hi)
            buf = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
            g.load_shard(i, lo, hi, buf.data_ptr(), buf.numel(), device=0)
            assert np.array_equal(buf.cpu().numpy(), ref), (name, world, r)
    finally:
        g.close()


def test_gemv_from_the_file(tmp_path):
    """A Q4_K weight loaded from the file straight into the GEMV (and its
    row-block shards into the all-gather kernel as rank 0 of 1)."""
    import torch
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    path, ts = _file(tmp_path)
    name, t, (K, N), data = ts[0]
    g = vkq.GGUF(path)
    try:
        i = g.find(name)
        buf = torch.empty(len(data), dtype=torch.uint8, device="cuda")
        g.load(i, buf.data_ptr(), buf.numel(), device=0)
        w = vt.QuantWeight(t, K, N, buf)
        x = synth.activations(1, K, seed=3)
        y = vt.matmul(torch.from_numpy(x).cuda(), w).cpu().numpy()
        wd = kq_oracle.dequantize(t, np.frombuffer(data, np.uint8))[:K * N].reshape(K, N)
        assert helpers.matmul_error(y, x, wd) <= helpers.GEMV_TOL
        assert vkq.device_status(0) == vkq.OK
    finally:
        g.close()
