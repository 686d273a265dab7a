"""vibrant_b200 -- B200 (sm_100a) kernels for xupit3r/vibrant's k-quant
(Q4_K / Q5_K / Q6_K) dequantize-and-matmul path, behind the C ABI in
include/vkq.h (built into vibrant_b200/_lib/libvkq.so).

Modules:
  vkq      ctypes binding of the C ABI (what a cgo shim binds)
  tensor   torch-facing helpers over that binding (device buffers, streams)
  synth    seeded synthetic workloads
  build    nvcc build of libvkq.so
"""
__all__ = ["vkq", "synth", "build"]
