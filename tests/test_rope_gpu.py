"""vkq_rope_f32: rotary position embedding over interleaved pairs, bit for
bit against a numpy float32 restatement of the reference's CPU path
(RoPE.ApplyRotation, internal/transformer/rope.go:49-124: each product and
each sum rounded to float32 on its own), on tables built as NewRoPE builds
them (rope.go:19-43)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rope_ref(x, cos_t, sin_t, positions):
    c = cos_t[positions]  # [seq, half]
    s = sin_t[positions]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _run(x, cos_t, sin_t, positions, inplace=False):
    import torch
    from vibrant_b200 import vkq
    B, H, S, D = x.shape
    xt = torch.from_numpy(x).cuda()
    out = xt if inplace else torch.full_like(xt, float("nan"))
    ct, st = torch.from_numpy(cos_t).cuda(), torch.from_numpy(sin_t).cuda()
    pt = torch.from_numpy(np.asarray(positions, dtype=np.int32)).cuda()
    vkq.rope_f32(xt.data_ptr(), out.data_ptr(), ct.data_ptr(), st.data_ptr(), pt.data_ptr(), B, H, S, D,
                 cos_t.shape[0], device=0)
    torch.cuda.synchronize()
    return out.cpu().numpy(), vkq.device_status(0)


@pytest.mark.parametrize("shape,positions,base", [
    ((1, 4, 3, 64), [0, 1, 2], 10000.0),               # the shape of the reference's TestRoPE_ApplyRotation
    ((1, 16, 1, 128), [37], 1000000.0),                 # one decode token, 3B-class heads
    ((2, 2, 5, 128), [5, 100, 2047, 0, 1], 10000.0),
    ((1, 3, 7, 2), [0, 1, 2, 3, 4, 5, 6], 10000.0),     # one pair per head
])
def test_rope_bit_exact(shape, positions, base):
    from vibrant_b200 import vkq
    cos_t, sin_t = vkq.rope_tables(shape[3], base, 2048)
    x = (np.random.default_rng(len(positions)).standard_normal(shape) * 4).astype(np.float32)
    out, st = _run(x, cos_t, sin_t, positions)
    assert st == vkq.OK
    ref = _rope_ref(x, cos_t, sin_t, np.asarray(positions))
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_rope_in_place():
    from vibrant_b200 import vkq
    cos_t, sin_t = vkq.rope_tables(64, 10000.0, 512)
    x = np.random.default_rng(7).standard_normal((1, 8, 4, 64)).astype(np.float32)
    out, st = _run(x.copy(), cos_t, sin_t, [3, 2, 1, 0], inplace=True)
    assert st == vkq.OK
    assert np.array_equal(out, _rope_ref(x, cos_t, sin_t, np.array([3, 2, 1, 0])))


def test_rope_position_out_of_range_is_reported():
    """A token whose position has no table row is left unwritten and the
    status word says so; the other tokens are rotated."""
    from vibrant_b200 import vkq
    cos_t, sin_t = vkq.rope_tables(16, 10000.0, 8)
    x = np.random.default_rng(8).standard_normal((1, 2, 3, 16)).astype(np.float32)
    out, st = _run(x, cos_t, sin_t, [1, 8, 2])
    assert st == vkq.ERR_INVALID_ARGUMENT
    assert np.isnan(out[:, :, 1]).all()
    ref = _rope_ref(x, cos_t, sin_t, np.array([1, 0, 2]))
    assert np.array_equal(out[:, :, [0, 2]], ref[:, :, [0, 2]])
    assert vkq.device_status(0) == vkq.OK  # the status word was cleared by the read


def test_rope_error_paths():
    import torch
    from vibrant_b200 import vkq
    x = torch.zeros(64, device="cuda")
    t = torch.zeros(64, device="cuda")
    p = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(vkq.VkqError) as e:  # odd head_dim
        vkq.rope_f32(x.data_ptr(), x.data_ptr(), t.data_ptr(), t.data_ptr(), p.data_ptr(), 1, 1, 4, 15, 8, device=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    with pytest.raises(vkq.VkqError) as e:  # x not 8-byte aligned
        vkq.rope_f32(x.data_ptr() + 4, x.data_ptr(), t.data_ptr(), t.data_ptr(), p.data_ptr(), 1, 1, 4, 8, 8,
                     device=0)
    assert e.value.status == vkq.ERR_MISALIGNED
    with pytest.raises(vkq.VkqError) as e:  # no positions
        vkq.rope_f32(x.data_ptr(), x.data_ptr(), t.data_ptr(), t.data_ptr(), 0, 1, 1, 4, 8, 8, device=0)
    assert e.value.status == vkq.ERR_INVALID_ARGUMENT
    assert vkq.device_status(0) == vkq.OK
