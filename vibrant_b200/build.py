"""Build libvkq.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m vibrant_b200.build        # or vibrant_b200.build.build()

Objects go to vibrant_b200/_build/, the library to vibrant_b200/_lib/libvkq.so.
nvcc cross-compiles for sm_100a without a GPU.  Sources are recompiled only
when they (or a header) are newer than their object.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libvkq.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -ftz=false -prec-div=true -prec-sqrt=true: the decode uses raw quants as
# subnormal fma operands and the bit-exact dequantization keeps subnormal
# results, so no flush-to-zero (and no --use_fast_math) may ever reach these
# kernels; nvcc exposes no macro a source file could check, so the flags are
# pinned here and tests/test_capi_cpu.py checks them.
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
              "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; libvkq.so cannot be built")
    return cand


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(ROOT, "include", "vkq.h")]


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep and not extra:
        return obj
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
