#!/usr/bin/env python
"""Benchmark of the k-quant dequantize-and-matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the hot path over one batch of synthetic input: the
Q6_K vocabulary projection (LM head) GEMV, x fp32 [1, 2048] . W [2048 x 151936]
Q6_K -> logits fp32 [1, 151936] (255,868,416 algorithmic bytes: weight +
x + y).  With N > 1 GPUs (one process per GPU under torchrun) the weight is
row-sharded by output columns and each rank runs one kernel that computes
its shard and stores it into every rank's logits buffer through peer memory
over NVLink (`--gather nccl` uses an NCCL all-gather instead; strong scaling).

Rank 0 prints one JSON line.  `value` is GB/s of algorithmic bytes for the
whole job with the weight resident in HBM; `e2e` is the same metric through
the C ABI with x copied from pinned host memory and the logits copied back
every step.  `--impl reference` times the reference's CPU implementation of
the path (the oracle's restatement of vibrant's Go code) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV GB/s (% HBM peak); prefill GEMM TFLOP/s; at 1/2/4/8 B200"
WORKLOAD = "q6k_vocab_gemv_2048x151936"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the extra workloads at N == 1")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: all-gather fused into the GEMV through peer memory, or an NCCL all-gather")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


def committed_traffic(workload: str):
    """(dram bytes per launch, kernel name) of the dominant kernel from the
    committed ncu summary."""
    p = os.path.join(ROOT, "profiles", f"{workload}.traffic.json")
    if os.path.exists(p):
        try:
            d = json.load(open(p))
            return d.get("dram_bytes_per_launch"), d.get("kernel")
        except Exception:
            return None, None
    return None, None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [num(r[3]) for r in self.rows if num(r[3]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "power_w_max": max(pw) if pw else None}


# --------------------------------------------------------------------------------------------
def cpu_reference_run(steps: int, warmup: int, budget_s: float):
    """The reference's CPU implementation of this step (oracle restatement of
    internal/transformer/model.go:389-403 + matmul_simd.go:189-199): the Q6_K
    weight is dequantized once (cached, as outputWeightCache does) and each
    step is the single-threaded outer product over the float32 [K, N] weight.
    Returns (seconds per step, rows per step sampled, K)."""
    import numpy as np
    from oracle import kq_oracle
    from vibrant_b200 import synth
    wl = synth.WORKLOADS[WORKLOAD]
    K, N, qt = wl["K"], wl["N"], wl["qtype"]
    wq = synth.weights(qt, K, N, seed=wl["seed"])
    x = synth.activations(1, K, seed=11).reshape(-1)
    w = kq_oracle.dequantize(qt, wq).reshape(K, N)   # the cached float32 weight
    # size the per-step sample so the whole run stays within the budget
    t0 = time.perf_counter()
    kq_oracle.matmul_single_row_u(x[:64], w[:64])
    per_row = (time.perf_counter() - t0) / 64
    total_steps = max(1, steps + warmup)
    rows = int(min(K, max(16, budget_s / max(per_row, 1e-9) / total_steps)))
    for _ in range(warmup):
        kq_oracle.matmul_single_row_u(x[:rows], w[:rows])
    t0 = time.perf_counter()
    for _ in range(steps):
        kq_oracle.matmul_single_row_u(x[:rows], w[:rows])
    dt = (time.perf_counter() - t0) / steps
    return dt, rows, K


def algorithmic_bytes(qtype: int, K: int, N: int, M: int) -> int:
    from vibrant_b200 import synth
    return synth.n_blocks(K, N) * synth.BLOCK_BYTES[qtype] + 4 * M * K + 4 * M * N


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from vibrant_b200 import synth
    wl = synth.WORKLOADS[WORKLOAD]
    dt, rows, K = cpu_reference_run(max(1, args.steps), max(0, args.warmup), budget_s=60.0)
    full_bytes = algorithmic_bytes(wl["qtype"], wl["K"], wl["N"], 1)
    gbs = full_bytes * (rows / K) / dt / 1e9
    sample = (f"{rows} of {K} rows of the outer product per step (x[:rows] . W[:rows, :]), "
              f"float32 weight cached as the reference's outputWeightCache; bytes scaled by rows/K")
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded; d, dmin, scale and quant distributions of the workload description)",
            "config": {"workload": WORKLOAD, "qtype": "Q6_K", "K": wl["K"], "N": wl["N"], "M": 1,
                       "parallelism": "single host thread (matmul_simd.go:189-199 has no fan-out)"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port", "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def time_gemv_graph(torch, vt, weights, x, outs, steps, warmup, stream):
    """CUDA-event time of `steps` launches (rotating weight copies) replayed
    from one CUDA graph; returns (seconds per launch, graph)."""
    for i in range(warmup):
        vt.matmul(x, weights[i % len(weights)], out=outs[i % len(outs)], stream=stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            vt.matmul(x, weights[i % len(weights)], out=outs[i % len(outs)], stream=stream)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):   # CUDAGraph.replay launches on the current stream
        g.replay()  # untimed replay
        stream.synchronize()
        ev0.record(stream)
        g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / 1e3 / steps, g


def secondary_q4k(torch, vt, hbm_peak):
    """Q4_K decode GEMV 2048 -> 11008 (the 3B FFN gate/up projection), 40
    rotated weight copies (507 MB > 126 MB L2), CUDA-event timed."""
    from vibrant_b200 import synth
    wl = synth.WORKLOADS["q4k_gemv_2048x11008"]
    qt, K, N = wl["qtype"], wl["K"], wl["N"]
    base = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=wl["seed"]))
    copies = [base] + [vt.QuantWeight(qt, K, N, base.buf.clone()) for _ in range(39)]
    x = torch.from_numpy(synth.activations(1, K, seed=5)).cuda()
    outs = [torch.empty(1, N, device="cuda") for _ in range(4)]
    stream = torch.cuda.Stream()
    dt, g = time_gemv_graph(torch, vt, copies, x, outs, 2000, 10, stream)
    del g
    b = algorithmic_bytes(qt, K, N, 1)
    gbs = b / dt / 1e9
    return {"workload": "q4k_gemv_2048x11008", "value": round(gbs, 2), "unit": "GB/s",
            "us_per_launch": round(dt * 1e6, 3), "hbm_frac": round(gbs / hbm_peak, 4),
            "algorithmic_bytes": b, "l2": "40 rotated weight copies (507 MB)"}


def secondary_gemm(torch, vt, bf16_peak, peak_kind):
    """Q5_K prefill GEMM 512 x 2048 x 11008 (the 3B FFN gate/up projection for
    a 512-token prompt) on the tcgen05 tensor-core path, 4 rotated weight
    copies, CUDA-event timed over a graph of launches."""
    from vibrant_b200 import synth
    wl = synth.WORKLOADS["q5k_prefill_gemm_512x2048x11008"]
    qt, K, N, M = wl["qtype"], wl["K"], wl["N"], wl["M"]
    base = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=wl["seed"]))
    copies = [base] + [vt.QuantWeight(qt, K, N, base.buf.clone()) for _ in range(3)]
    x = torch.from_numpy(synth.activations(M, K, seed=6)).cuda()
    outs = [torch.empty(M, N, device="cuda") for _ in range(2)]
    stream = torch.cuda.Stream()
    dt, g = time_gemv_graph(torch, vt, copies, x, outs, 200, 5, stream)
    del g
    flops = 2 * M * K * N
    tf = flops / dt / 1e12
    return {"workload": "q5k_prefill_gemm_512x2048x11008", "value": round(tf, 2), "unit": "TFLOP/s",
            "us_per_launch": round(dt * 1e6, 3), "dtype": "bf16 operands, fp32 accumulate",
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": round(tf / bf16_peak, 4), "peak_kind": peak_kind + " bf16 burst",
                         "algorithmic_flops_per_launch": flops},
            "launches_per_step": 2, "kernels": "x_to_bf16_kernel + vkq::gemm_kernel<Q5_K>"}


def run_ours(args):
    import numpy as np
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    hbm_peak, bf16_peak, peak_kind = peaks()
    wl = synth.WORKLOADS[WORKLOAD]
    qt, K, N = wl["qtype"], wl["K"], wl["N"]
    width, bounds = vt.shard_columns(N, world)
    lo, hi = bounds[rank]
    peer = world > 1 and args.gather == "peer"
    if world == 1 or peer:
        # the whole [K, N] weight (every rank keeps it; a rank reads only its columns)
        n_local = N if world == 1 else hi - lo
        wq = synth.weights(qt, K, N, seed=wl["seed"])
        w0 = vt.QuantWeight(qt, K, N, wq, device=dev)
    else:
        # NCCL baseline: a canonical [K, width] shard per rank (the last rank's tail is padding)
        n_local = width
        wq = synth.weights(qt, K, n_local, seed=wl["seed"] * 1000 + rank)
        w0 = vt.QuantWeight(qt, K, n_local, wq, device=dev)
    w1 = vt.QuantWeight(w0.qtype, w0.K, w0.N, w0.buf.clone(), device=dev)
    weights = [w0, w1]     # two copies: 2 x 255 MB per GPU, larger than the 126 MB L2
    x_host = torch.from_numpy(synth.activations(1, K, seed=11)).pin_memory()
    x = x_host.to(dev)
    y_local = torch.empty(1, n_local if not (world == 1) else N, device=dev)
    y_full = torch.empty(world * n_local, device=dev)
    stream = torch.cuda.Stream(device=dev)
    gather = None
    if peer:
        gather = vt.PeerGather(pg.group.WORLD, rank, world, local, N, m_max=1)
        y_full = gather.out[0]

    def step(wt):
        if gather is not None:   # one kernel: shard GEMV + stores into every rank's logits
            gather.gemv(x, wt, stream=stream)
            return
        vt.matmul(x, wt, out=y_local, stream=stream)
        if pg is not None:
            with torch.cuda.stream(stream):
                pg.all_gather_into_tensor(y_full, y_local.view(-1))

    # warm-up (>= 3 untimed steps), then capture exactly `steps` steps in a graph
    warm = max(3, args.warmup)
    for i in range(warm):
        step(weights[i % 2])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(args.steps):
            step(weights[i % 2])
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):   # CUDAGraph.replay launches on the current stream
        t_soak = time.time()
        while time.time() - t_soak < 1.0:   # bring clocks to their loaded state
            g.replay()
            stream.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    sampler.stop()
    dt_local = ev0.elapsed_time(ev1) / 1e3
    dt = dt_local
    if pg is not None:
        t = torch.tensor([dt_local], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        dt = float(t.item())
    del g

    # kernel-only timing of the dominant kernel (for its roofline): the GEMV,
    # or at N > 1 with the peer all-gather the fused kernel
    if gather is not None:
        for i in range(3):
            gather.gemv(x, weights[i % 2], stream=stream)
        torch.cuda.synchronize()
        kg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kg, stream=stream):
            for i in range(args.steps):
                gather.gemv(x, weights[i % 2], stream=stream)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            kg.replay()
            stream.synchronize()
            pg.barrier()
            k0.record(stream)
            kg.replay()
            k1.record(stream)
        torch.cuda.synchronize()
        k_dt = k0.elapsed_time(k1) / 1e3 / args.steps
    else:
        k_dt, kg = time_gemv_graph(torch, vt, weights, x, [y_local], args.steps, 3, stream)
    del kg

    # end to end through the C ABI: x from pinned host memory, logits back to pinned host memory
    y_host = torch.empty(y_full.numel() if pg is not None else n_local, dtype=torch.float32).pin_memory()
    y_src = y_full if pg is not None else y_local.view(-1)
    e_steps = max(10, min(args.steps, 500))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            x.copy_(x_host, non_blocking=True)
            step(weights[i % 2])
            y_host.copy_(y_src, non_blocking=True)
        stream.synchronize()
        if pg is not None:
            pg.barrier()
        e0.record(stream)
        for i in range(e_steps):
            x.copy_(x_host, non_blocking=True)
            step(weights[i % 2])
            y_host.copy_(y_src, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    e_dt = e0.elapsed_time(e1) / 1e3 / e_steps
    if pg is not None:
        t = torch.tensor([e_dt], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e_dt = float(t.item())

    total_bytes = algorithmic_bytes(qt, K, N, 1)     # the whole matrix: all ranks together
    step_s = dt / args.steps
    value = total_bytes / step_s / 1e9
    shard_bytes = algorithmic_bytes(qt, K, n_local, 1)
    achieved = shard_bytes / k_dt / 1e9
    traffic, kernel_name = committed_traffic(WORKLOAD) if world == 1 else (None, None)
    launches_per_step = 1    # the GEMV (with the all-gather fused in when N > 1)
    line = None
    if rank == 0:
        secondary = {}
        cpu = None
        if world == 1:
            if not args.no_secondary:
                try:
                    secondary["q4k_gemv_2048x11008"] = secondary_q4k(torch, vt, hbm_peak)
                except Exception as e:  # reported, not hidden
                    secondary["q4k_gemv_2048x11008"] = {"error": str(e)}
                try:
                    secondary["q5k_prefill_gemm_512x2048x11008"] = secondary_gemm(torch, vt, bf16_peak, peak_kind)
                except Exception as e:  # reported, not hidden
                    secondary["q5k_prefill_gemm_512x2048x11008"] = {"error": str(e)}
            cdt, rows, Kc = cpu_reference_run(3, 1, budget_s=args.cpu_seconds)
            cgbs = total_bytes * (rows / Kc) / cdt / 1e9
            cpu = {"value": round(cgbs, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                   "sample": f"{rows} of {Kc} rows of the LM-head outer product (matmul_simd.go:189-199, "
                             f"single goroutine) on the cached float32 weight, 3 timed passes; "
                             f"bytes scaled by rows/K"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": round(step_s * 1e3, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded; d, dmin, scale and quant distributions of the workload description)",
            "config": {"workload": WORKLOAD, "qtype": "Q6_K", "K": K, "N": N, "M": 1,
                       "columns_per_rank": n_local,
                       "parallelism": "single GPU" if world == 1 else
                       f"row-sharded output columns over {world} GPUs, " + (
                           "all-gather fused into the GEMV (stores into every rank's logits over NVLink)"
                           if gather is not None else "NCCL all-gather"),
                       "l2": "inputs larger than L2: two rotated copies of the weight "
                             f"({2 * w0.nbytes / 1e6:.0f} MB per GPU)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                         "peak_kind": peak_kind, "kernel": kernel_name or "vkq::gemv_kernel<Q6_K,1,64>",
                         "algorithmic_bytes_per_launch": shard_bytes,
                         "us_per_launch": round(k_dt * 1e6, 3)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total_bytes / e_dt / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 4 * K, "d2h_bytes_per_step": 4 * y_host.numel(),
                    "ms_per_step": round(e_dt * 1e3, 5), "path": "vkq_matmul via ctypes, eager launches"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
            "secondary": secondary,
        }
    if gather is not None:
        gather.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
