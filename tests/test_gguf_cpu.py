"""The GGUF parser of the on-device loader (vkq_gguf_*, gguf.cu) on files
written by the test: tensor infos, data offsets, calculateTensorSize
(internal/gguf/metadata.go:170-204, Q4_K included, which LoadTensor's
expectedSize, internal/gguf/loader.go:35-48, misses) and malformed files.
Host only: nothing here touches a GPU."""
import os

import numpy as np
import pytest

import helpers

F32, F16, Q4_K, Q5_K, Q6_K = 0, 1, 12, 13, 14


def _tensors():
    from vibrant_b200 import synth
    rng = np.random.default_rng(3)
    return [("blk.0.ffn_up.weight", Q4_K, [512, 768], synth.weights(Q4_K, 512, 768, seed=1).tobytes()),
            ("output.weight", Q6_K, [256, 640], synth.weights(Q6_K, 256, 640, seed=2).tobytes()),
            ("output_norm.weight", F32, [512], rng.standard_normal(512).astype(np.float32).tobytes()),
            ("blk.0.attn_k.weight", Q5_K, [256, 256], synth.weights(Q5_K, 256, 256, seed=4).tobytes())]


@pytest.fixture
def gguf_file(tmp_path):
    ts = _tensors()
    path = str(tmp_path / "model.gguf")
    offs = helpers.write_gguf(path, ts)
    return path, ts, offs


def test_parse_tensor_infos(gguf_file):
    from vibrant_b200 import vkq
    path, ts, offs = gguf_file
    g = vkq.GGUF(path)
    try:
        assert len(g) == len(ts)
        raw = open(path, "rb").read()
        for (name, t, dims, data), off in zip(ts, offs):
            i = g.find(name)
            info = g.info(i)
            assert info["name"] == name and info["type"] == t and info["dims"] == dims
            assert info["bytes"] == len(data)
            assert raw[info["offset"]:info["offset"] + len(data)] == data
            assert info["offset"] % 32 == 0 and info["offset"] - off == g.info(0)["offset"] - offs[0]
        with pytest.raises(vkq.VkqError):
            g.find("no.such.tensor")
    finally:
        g.close()


@pytest.mark.parametrize("t,dims,expect", [(Q4_K, [2048, 11008], 2048 * 11008 // 256 * 144),
                                           (Q5_K, [2048, 11008], 2048 * 11008 // 256 * 176),
                                           (Q6_K, [2048, 151936], 2048 * 151936 // 256 * 210),
                                           (Q4_K, [300], 288),  # a partial block rounds up
                                           (F32, [7, 3], 84), (F16, [5], 10)])
def test_calculate_tensor_size(t, dims, expect):
    from vibrant_b200 import vkq
    assert vkq.gguf_tensor_bytes(t, dims) == expect


def test_version_2_and_no_metadata(tmp_path):
    from vibrant_b200 import vkq
    ts = _tensors()[:2]
    path = str(tmp_path / "v2.gguf")
    helpers.write_gguf(path, ts, version=2, metadata=False)
    g = vkq.GGUF(path)
    try:
        assert len(g) == 2 and g.info(g.find("output.weight"))["dims"] == [256, 640]
    finally:
        g.close()


def test_malformed_files_are_refused(tmp_path):
    from vibrant_b200 import vkq
    ts = _tensors()[:1]
    good = str(tmp_path / "good.gguf")
    helpers.write_gguf(good, ts)
    raw = open(good, "rb").read()
    cases = {
        "magic": b"GGUX" + raw[4:],
        "version": raw[:4] + (1).to_bytes(4, "little") + raw[8:],
        "truncated-header": raw[:40],
        "truncated-data": raw[:-100],
        "huge-count": raw[:8] + (1 << 40).to_bytes(8, "little") + raw[16:],
    }
    for what, data in cases.items():
        p = str(tmp_path / f"{what}.gguf")
        open(p, "wb").write(data)
        with pytest.raises(vkq.VkqError) as e:
            vkq.GGUF(p)
        assert e.value.status in (vkq.ERR_INVALID_ARGUMENT, vkq.ERR_UNSUPPORTED), what
    with pytest.raises(vkq.VkqError):
        vkq.GGUF(os.path.join(str(tmp_path), "missing.gguf"))
