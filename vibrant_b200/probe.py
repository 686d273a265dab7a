"""Run one k-quant matmul workload through the C ABI and print its CUDA-event
time per launch (CUDA-graph replay of ITERS launches).  Used for profiling:

    python -m vibrant_b200.probe QTYPE K N M ITERS [COPIES]

QTYPE is the GGML code (12 Q4_K, 13 Q5_K, 14 Q6_K); COPIES rotated weight
copies keep a small weight from being served out of the L2.
"""
import sys

import torch

from vibrant_b200 import synth, vkq
from vibrant_b200 import tensor as vt


def main(argv):
    qt, K, N, M, iters = [int(a) for a in argv[:5]]
    copies = int(argv[5]) if len(argv) > 5 else 1
    w = [vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=1))]
    for _ in range(copies - 1):
        w.append(vt.QuantWeight(qt, K, N, w[0].buf.clone()))
    x = torch.from_numpy(synth.activations(M, K, seed=2)).cuda()
    y = torch.empty(M, N, device="cuda")
    for i in range(3):
        vt.matmul(x, w[i % copies], out=y)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            vt.matmul(x, w[i % copies], out=y, stream=st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        g.replay()
        st.synchronize()
        e0.record(st)
        g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / iters
    b = synth.n_blocks(K, N) * synth.BLOCK_BYTES[qt] + 4 * M * (K + N)
    print(f"qt={qt} K={K} N={N} M={M}: {dt * 1e6:.2f} us/launch  {b / dt / 1e9:.1f} GB/s  "
          f"{2 * M * K * N / dt / 1e12:.1f} TFLOP/s  status={vkq.device_status(0)}")


if __name__ == "__main__":
    main(sys.argv[1:])
