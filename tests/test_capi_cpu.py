"""CPU-side checks of the C ABI: libvkq.so loads, exports every symbol that
include/vkq.h declares, and its host-only paths (sizes, argument checks,
status strings) behave; no kernel is launched here."""
import ctypes
import os
import re

import numpy as np
import pytest

import helpers

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"^VKQ_API\s+[\w\s\*]*?\b(vkq_\w+)\s*\(", text, flags=re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from vibrant_b200 import build, vkq
    if not os.path.exists(vkq.LIB_PATH):
        build.build()
    return vkq.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("vkq_matmul", "vkq_gemv", "vkq_dequantize_f32", "vkq_dequant_transpose_f32",
              "vkq_matmul_workspace_bytes", "vkq_weight_bytes", "vkq_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from vibrant_b200 import vkq
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in vkq.SIGNATURES, f"{name} has no ctypes signature in vibrant_b200/vkq.py"


def test_only_declared_symbols_are_exported(lib):
    from vibrant_b200 import vkq
    out = os.popen(f"nm -D --defined-only {vkq.LIB_PATH}").read()
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    vkq_syms = {s for s in exported if s.startswith("vkq_")}
    assert vkq_syms == declared_symbols()


def test_abi_version_and_block_bytes(lib):
    assert lib.vkq_abi_version() == 5
    assert [lib.vkq_block_bytes(t) for t in (12, 13, 14)] == [144, 176, 210]
    assert lib.vkq_block_bytes(2) == 0


@pytest.mark.parametrize("qt,K,N", [(12, 2048, 11008), (14, 2048, 151936), (13, 8, 4), (14, 3, 5)])
def test_weight_bytes_matches_calculate_tensor_size(lib, qt, K, N):
    # calculateTensorSize, internal/gguf/metadata.go:170-204
    from vibrant_b200 import vkq
    assert vkq.weight_bytes(qt, K, N) == ((K * N + 255) // 256) * helpers.BLOCK_BYTES[qt]


def test_weight_bytes_rejects_bad_input(lib):
    out = ctypes.c_int64()
    assert lib.vkq_weight_bytes(99, 4, 4, ctypes.byref(out)) == 2
    assert b"unsupported" in lib.vkq_last_error()
    assert lib.vkq_weight_bytes(12, 0, 4, ctypes.byref(out)) == 1


def test_status_strings(lib):
    assert lib.vkq_status_string(0) == b"ok"
    assert lib.vkq_status_string(4) == b"workspace missing or too small"
    assert lib.vkq_status_string(123) == b"unknown status"


def test_calls_without_gpu_fail_loudly(lib):
    # no silent fallback: without a usable device every compute entry point
    # returns an error status and a message
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st = lib.vkq_gemv(0, 12, None, 0, 1, 1, None, 1, None, None, 0, None)
    assert st != 0 and lib.vkq_last_error() != b""


def test_exact_encoders_round_trip(oracle):
    v6 = np.arange(-32, 32).repeat(5)[:300]
    assert np.array_equal(oracle.dequantize(14, helpers.encode_q6k_exact(v6))[:300], v6.astype(np.float32))
    v4 = np.arange(16).repeat(20)[:300]
    assert np.array_equal(oracle.dequantize(12, helpers.encode_q45k_exact(v4, 12))[:300], v4.astype(np.float32))
    v5 = np.arange(32).repeat(10)[:300]
    assert np.array_equal(oracle.dequantize(13, helpers.encode_q45k_exact(v5, 13))[:300], v5.astype(np.float32))


def test_build_never_flushes_subnormals():
    """The decode feeds raw quants to fma as subnormal operands (q * 2^-149)
    and the dequantization keeps subnormal results: a flush-to-zero build
    would turn every weight into zero (or -dmin*m).  nvcc exposes no macro for
    it, so the build flags pin it."""
    from vibrant_b200 import build
    flags = build.NVCC_FLAGS
    assert "-ftz=false" in flags
    assert not any(f in flags for f in ("--use_fast_math", "-use_fast_math", "-ftz=true", "--ftz=true"))


def test_rope_tables_follow_the_reference_formula():
    """rope_tables restates NewRoPE (internal/transformer/rope.go:19-43)."""
    import math
    from vibrant_b200 import vkq
    c, s = vkq.rope_tables(64, 10000.0, 16)
    assert c.shape == (16, 32) and c.dtype == np.float32
    for pos, i in [(0, 0), (1, 0), (5, 7), (15, 31)]:
        angle = pos * (1.0 / math.pow(10000.0, 2 * i / 64))
        assert abs(float(c[pos, i]) - math.cos(angle)) <= 1e-7
        assert abs(float(s[pos, i]) - math.sin(angle)) <= 1e-7
