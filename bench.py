#!/usr/bin/env python
"""Benchmark of the k-quant dequantize-and-matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --probe QTYPE,K,N,M[,COPIES] [--steps K]    (one workload, for profiling)

One step = one pass of the hot path over one batch of synthetic input: the
Q4_K decode GEMV x fp32 [1, 2048] . W Q4_K [2048 x 11008] -> y fp32 [1, 11008]
(the 3B model's FFN gate/up projection; 12,733,440 algorithmic bytes: weight +
x + y).  With N > 1 GPUs (one process per GPU under torchrun) each rank holds
its row-block shard of the weight (its output columns only) and runs one
kernel that computes its columns and stores them into every rank's output
through peer memory over NVLink (strong scaling: the whole matrix per step).

Rank 0 prints one JSON line.  `value` is GB/s of algorithmic bytes for the
whole job with the weights resident in HBM (rotated copies, larger than L2 in
all, and L2 flushed before the timed region); `e2e` is the same metric through
the public API with x copied from pinned host memory and y copied back every
step.  `secondary` holds the other workloads: the Q6_K vocabulary projection,
the Q5_K prefill GEMM, the full 3B decode step (every N) and the 14B/32B
batched-decode sweep (every N).  `--impl reference` times the reference's CPU
implementation of the headline (the oracle's restatement of vibrant's Go
code: the transposed single-row dot over every host core) on the host.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV GB/s (% HBM peak); prefill GEMM TFLOP/s; at 1/2/4/8 B200"
HEADLINE = "q4k_gemv_2048x11008"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
ROTATION_BYTES = 512 << 20      # rotated weight copies per GPU: 4x the 126 MB L2
FLUSH_BYTES = 256 << 20         # L2 flush before every timed region
CTX_3B = 1024                   # tokens in every layer's KV cache in the 3B decode step


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="headline only")
    ap.add_argument("--only", default=None, help="comma list of secondary workloads to run (default: all)")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU baseline sample budget")
    ap.add_argument("--probe", default=None, help="QTYPE,K,N,M[,COPIES]: time one workload (profiling)")
    ap.add_argument("--probe-fused", default=None, choices=["qkv", "gate_up"],
                    help="time one fused launch of the 3B layer (RMSNorm + q|k|v, or RMSNorm + gate|up + SiLU*up)")
    ap.add_argument("--gemv", default="auto", choices=["auto", "simt", "tc", "strip"],
                    help="GEMV kernel for M <= 8 (vkq_set_gemv_path): automatic, CUDA cores, tensor cores or "
                         "Q4_K column strips")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained",
                                                                            d["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def committed_traffic(workload: str):
    """(dram bytes per launch, kernel name) of the dominant kernel from the
    committed ncu summary of the current build, or (None, None)."""
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
        self.gpu, self.rows, self.proc, self.t = gpu_index, [], None, None

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


def algorithmic_bytes(qtype: int, K: int, N: int, M: int) -> int:
    from vibrant_b200 import synth
    return synth.n_blocks(K, N) * synth.BLOCK_BYTES[qtype] + 4 * M * K + 4 * M * N


# ---------------------------------------------------------------- CPU reference
def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference(steps: int, warmup: int, budget_s: float):
    """The reference's CPU implementation of the headline step (the oracle's
    restatement of vibrant's Go code): the Q4_K weight is expanded once into
    the cached float32 transposed copy (GetOrDequantTranspose,
    internal/tensor/tensor.go:535-588), then every step is the transposed
    single-row dot with runtime.NumCPU() workers (matmulSIMDSingleRow,
    internal/tensor/matmul_simd.go:164-188).  Cold: the expansion
    (DequantTransposeQ4K, dequant_transpose.go:15-157) inside every step.
    Returns a dict of per-step seconds and the sample description."""
    from oracle import kq_oracle
    from vibrant_b200 import synth
    wl = synth.WORKLOADS[HEADLINE]
    qt, K, N = wl["qtype"], wl["K"], wl["N"]
    wq = synth.weights(qt, K, N, seed=wl["seed"])
    x = synth.activations(1, K, seed=11).reshape(-1)
    cores = host_cores()
    wt = kq_oracle.dequant_transpose(qt, wq, K, N)            # the cached float32 [N, K] weight
    t0 = time.perf_counter()
    kq_oracle.matmul_single_row_t(x, wt, nthreads=cores)
    one = time.perf_counter() - t0
    n = max(3, min(steps, int(budget_s * 0.7 / max(one, 1e-6))))
    for _ in range(min(warmup, 3)):
        kq_oracle.matmul_single_row_t(x, wt, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(n):
        kq_oracle.matmul_single_row_t(x, wt, nthreads=cores)
    warm = (time.perf_counter() - t0) / n
    nc = 2   # cold: the expansion and the dot in every step
    t0 = time.perf_counter()
    for _ in range(nc):
        w2 = kq_oracle.dequant_transpose(qt, wq, K, N)
        kq_oracle.matmul_single_row_t(x, w2, nthreads=cores)
    cold = (time.perf_counter() - t0) / nc
    return {"warm_s": warm, "cold_s": cold, "steps": n, "cold_steps": nc, "cores": cores, "cpu": cpu_model()}


def cpu_line(c, total_bytes):
    gbs = total_bytes / c["warm_s"] / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": c["cores"], "kind": "port",
            "cold_value": round(total_bytes / c["cold_s"] / 1e9, 4),
            "sample": (f"whole headline step (x [1,2048] . Q4_K [2048 x 11008]) {c['steps']} times: the oracle's C "
                       f"restatement of matmulSIMDSingleRow (transposed dot, {c['cores']} worker threads = every "
                       f"host core, {c['cpu']}) on the cached float32 transposed weight (warm, as after "
                       f"WarmWeightCache); cold_value adds DequantTransposeQ4K to every step "
                       f"({c['cold_steps']} steps); bytes are the Q4_K algorithmic bytes")}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from vibrant_b200 import synth
    wl = synth.WORKLOADS[HEADLINE]
    total = algorithmic_bytes(wl["qtype"], wl["K"], wl["N"], 1)
    c = cpu_reference(max(1, args.steps), max(0, args.warmup), budget_s=min(60.0, max(10.0, args.cpu_seconds)))
    cb = cpu_line(c, total)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": world,
            "steps": c["steps"], "warmup": args.warmup, "ms_per_step": round(c["warm_s"] * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded; d, dmin, scale and quant distributions of the workload description)",
            "config": {"workload": HEADLINE, "qtype": "Q4_K", "K": wl["K"], "N": wl["N"], "M": 1,
                       "parallelism": f"{c['cores']} host threads (runtime.NumCPU() goroutines)"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU helpers
class Ctx:
    """Per-process state: device, process group, stream, peaks."""

    def __init__(self, torch, rank, world, local, pg):
        self.torch, self.rank, self.world, self.local, self.pg = torch, rank, world, local, pg
        self.dev = torch.device("cuda", local)
        self.stream = torch.cuda.Stream(device=self.dev)
        self.hbm, self.bf16, self.bf16_sus, self.peak_kind = peaks()
        self.flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=self.dev)

    def allmax(self, v: float) -> float:
        if self.pg is None:
            return v
        t = self.torch.tensor([float(v)], device=self.dev, dtype=self.torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()
        self.torch.cuda.synchronize(self.dev)

    def status(self, where: str):
        """Device status of every rank after a phase; exits on a failure."""
        from vibrant_b200 import vkq
        st = vkq.device_status(self.local)
        worst = int(self.allmax(st))
        if worst != vkq.OK:
            if self.rank == 0:
                print(json.dumps({"error": f"device status {worst} ({vkq.load().vkq_status_string(worst).decode()})"
                                           f" after {where}", "n_gpus": self.world}), flush=True)
            sys.exit(3)

    def flush_l2(self):
        with self.torch.cuda.stream(self.stream):
            self.flush_buf.zero_()


def timed_graph(ctx, step, steps: int, warmup: int, align=None, sampler=None, soak_s: float = 0.0):
    """Capture `steps` calls of step(i) in one CUDA graph and time one replay
    with CUDA events on the launching stream (max over ranks).  Warm-up calls
    first; an optional soak of replays (the same count on every rank) brings
    the clocks to their loaded state; the L2 is flushed before the timed
    replay; `align` (one untimed collective call) makes every rank's timed
    region start together.  Returns seconds per step."""
    torch = ctx.torch
    with torch.cuda.stream(ctx.stream):
        for i in range(max(3, warmup)):
            step(i)
    torch.cuda.synchronize(ctx.dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ctx.stream):
        for i in range(steps):
            step(i)
    torch.cuda.synchronize(ctx.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(ctx.stream):
        e0.record(ctx.stream)
        g.replay()
        e1.record(ctx.stream)
    torch.cuda.synchronize(ctx.dev)
    one = ctx.allmax(e0.elapsed_time(e1) / 1e3)
    n_soak = max(0, min(500, int(math.ceil(soak_s / max(one, 1e-6))))) if soak_s > 0 else 0
    n_soak = int(ctx.allmax(n_soak))          # the same count on every rank
    if sampler is not None:
        sampler.start()
    with torch.cuda.stream(ctx.stream):
        for _ in range(n_soak):
            g.replay()
    torch.cuda.synchronize(ctx.dev)
    ctx.flush_l2()
    ctx.barrier()
    with torch.cuda.stream(ctx.stream):
        if align is not None:
            align()
        e0.record(ctx.stream)
        g.replay()
        e1.record(ctx.stream)
    torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    if sampler is not None:
        sampler.stop()
    dt = ctx.allmax(e0.elapsed_time(e1) / 1e3)
    del g
    return dt / steps


def n_copies(nbytes: int) -> int:
    return max(2, int(math.ceil(ROTATION_BYTES / max(1, nbytes))))


def _clone(w):
    c = w.__class__.__new__(w.__class__)
    c.__dict__.update(w.__dict__)
    c.buf = w.buf.clone()
    return c


# ---------------------------------------------------------------- headline
def headline(ctx, args):
    """Q4_K decode GEMV 2048 -> 11008 (config 0), row-sharded at N > 1."""
    import numpy as np
    torch = ctx.torch
    from oracle import kq_oracle
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    wl = synth.WORKLOADS[HEADLINE]
    qt, K, N = wl["qtype"], wl["K"], wl["N"]
    wq = synth.weights(qt, K, N, seed=wl["seed"])
    gather = None
    if ctx.world == 1:
        base = vt.QuantWeight(qt, K, N, wq, device=ctx.dev)
        lo, hi = 0, N
    else:
        base = vt.ShardedWeight(qt, K, N, ctx.world, ctx.rank, wq, device=ctx.dev)
        lo, hi = base.lo, base.hi
        gather = vt.PeerGather(ctx.pg.group.WORLD, ctx.rank, ctx.world, ctx.local, N, m_max=1)
    nc = n_copies(base.nbytes)
    copies = [base] + [_clone(base) for _ in range(nc - 1)]
    x_host = torch.from_numpy(synth.activations(1, K, seed=11)).pin_memory()
    x = x_host.to(ctx.dev)
    y = torch.empty(1, N, device=ctx.dev)
    ws = vt.workspace(vt.workspace_bytes(qt, 1, K, hi - lo, ctx.local), ctx.local)

    def step(i):
        if gather is not None:
            gather.gemv(x, copies[i % nc], ws=ws, stream=ctx.stream)
        else:
            vt.matmul(x, copies[i % nc], out=y, ws=ws, stream=ctx.stream)

    y_out = gather.out[:1] if gather is not None else y
    sampler = ClockSampler(ctx.local)
    align = (lambda: step(nc - 1)) if gather is not None else None
    dt = timed_graph(ctx, step, args.steps, args.warmup, align=align, sampler=sampler, soak_s=1.0)
    ctx.status("the headline timed region")

    # end to end through the public API: x from pinned host memory, y back to pinned host memory
    y_host = torch.empty(N, dtype=torch.float32).pin_memory()
    e_steps = max(10, min(args.steps, 500))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(ctx.stream):
        for i in range(3):
            x.copy_(x_host, non_blocking=True)
            step(i)
            y_host.copy_(y_out.view(-1), non_blocking=True)
    ctx.flush_l2()
    ctx.barrier()
    from vibrant_b200 import vkq
    ws_ptr, ws_n = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    # raw pointers, as a host program holds them
    w_ptrs, w_bytes = [c.buf.data_ptr() for c in copies], base.nbytes
    xh_ptr, yh_ptr, xd_ptr, yd_ptr = x_host.data_ptr(), y_host.data_ptr(), x.data_ptr(), y.data_ptr()
    s_ptr = ctx.stream.cuda_stream
    with torch.cuda.stream(ctx.stream):
        if align is not None:
            align()
        e0.record(ctx.stream)
        if gather is None:  # one call per step: x up, the product, y down (vkq_matmul_host)
            for i in range(e_steps):
                vkq.matmul_host(qt, w_ptrs[i % nc], w_bytes, K, N, xh_ptr, 1, yh_ptr, xd_ptr, yd_ptr, ws_ptr, ws_n,
                                device=ctx.local, stream=s_ptr)
        else:
            for i in range(e_steps):
                x.copy_(x_host, non_blocking=True)
                step(i)
                y_host.copy_(y_out.view(-1), non_blocking=True)
        e1.record(ctx.stream)
    torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    e_dt = ctx.allmax(e0.elapsed_time(e1) / 1e3 / e_steps)
    ctx.status("the end-to-end loop")

    # parity of the gathered result on every rank, against the oracle (1e-5 of sum |x w|)
    xp = synth.activations(1, K, seed=12)
    x.copy_(torch.from_numpy(xp))
    with torch.cuda.stream(ctx.stream):
        step(0)
    torch.cuda.synchronize(ctx.dev)
    yv = y_out.view(-1).cpu().numpy().copy()
    wd = kq_oracle.dequantize(qt, wq)[:K * N].reshape(K, N).astype(np.float64)
    x64 = xp.astype(np.float64).reshape(-1)
    err = float(np.max(np.abs(yv.astype(np.float64) - x64 @ wd) / (np.abs(x64) @ np.abs(wd))))
    err = ctx.allmax(err)
    ctx.status("the parity call")
    if err > 1e-5:
        if ctx.rank == 0:
            print(json.dumps({"error": f"parity: max relative error {err:.3e} above 1e-5", "n_gpus": ctx.world}),
                  flush=True)
        sys.exit(4)
    if gather is not None:
        gather.close()
    total = algorithmic_bytes(qt, K, N, 1)
    shard_alg = synth.n_blocks(K, hi - lo) * synth.BLOCK_BYTES[qt] + 4 * K + 4 * (hi - lo)
    traffic, kname = committed_traffic(HEADLINE) if ctx.world == 1 else (None, None)
    return {
        "dt": dt, "e_dt": e_dt, "total": total, "shard_alg": shard_alg, "lo": lo, "hi": hi, "copies": nc,
        "copy_bytes": base.nbytes, "err": err, "clocks": sampler.summary(), "traffic": traffic,
        "kernel": kname or ("vkq::gemv_strip_kernel<1> (all-gather)" if gather is not None else
                            "vkq::gemv_strip_kernel<1>"),
        "h2d": 4 * K, "d2h": 4 * N,
    }


# ---------------------------------------------------------------- secondary workloads (N == 1)
def gemv_workload(ctx, name, steps):
    """A single-GPU GEMV / GEMM workload of synth.WORKLOADS with rotated copies."""
    torch = ctx.torch
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    wl = synth.WORKLOADS[name]
    qt, K, N, M = wl["qtype"], wl["K"], wl["N"], wl["M"]
    base = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=wl["seed"]), device=ctx.dev)
    nc = n_copies(base.nbytes)
    copies = [base] + [_clone(base) for _ in range(nc - 1)]
    x = torch.from_numpy(synth.activations(M, K, seed=6)).to(ctx.dev)
    y = torch.empty(M, N, device=ctx.dev)
    ws = vt.workspace(max(vt.workspace_bytes(qt, M, K, N, ctx.local), 1), ctx.local)

    def step(i):
        vt.matmul(x, copies[i % nc], out=y, ws=ws, stream=ctx.stream)

    dt = timed_graph(ctx, step, steps, 5)
    ctx.status(name)
    return dt, qt, K, N, M, nc, base.nbytes


def secondary_q6k(ctx, args):
    name = "q6k_vocab_gemv_2048x151936"
    dt, qt, K, N, M, nc, nb = gemv_workload(ctx, name, max(20, min(args.steps, 200)))
    b = algorithmic_bytes(qt, K, N, M)
    gbs = b / dt / 1e9
    traffic, kname = committed_traffic(name)
    return {"workload": name, "value": round(gbs, 2), "unit": "GB/s", "us_per_launch": round(dt * 1e6, 3),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": ctx.hbm, "unit": "GB/s",
                         "frac": round(gbs / ctx.hbm, 4), "traffic": traffic, "peak_kind": ctx.peak_kind,
                         "kernel": kname or "vkq::gemv_kernel<Q6_K,1,64>", "algorithmic_bytes_per_launch": b},
            "l2": f"{nc} rotated weight copies ({nc * nb / 1e6:.0f} MB), L2 flushed before the timed region"}


def secondary_upstream(ctx, args):
    """The headline's weight (11008 outputs x 2048 inputs, Q4_K) in the
    upstream GGUF orientation, through vkq_matmul_upstream."""
    torch = ctx.torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    qt, K, N = synth.Q4_K, 2048, 11008
    base = vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=5), device=ctx.dev)
    nc = n_copies(base.nbytes)
    copies = [base] + [_clone(base) for _ in range(nc - 1)]
    x = torch.from_numpy(synth.activations(1, K, seed=6)).to(ctx.dev)
    y = torch.empty(1, N, device=ctx.dev)

    def step(i):
        c = copies[i % nc]
        vkq.matmul_upstream(qt, c.buf.data_ptr(), c.nbytes, K, N, x.data_ptr(), 1, y.data_ptr(), device=ctx.local,
                            stream=ctx.stream)

    dt = timed_graph(ctx, step, max(20, min(args.steps, 200)), 5)
    ctx.status("the upstream-orientation GEMV")
    b = algorithmic_bytes(qt, K, N, 1)
    gbs = b / dt / 1e9
    return {"workload": "q4k_upstream_gemv_11008x2048", "value": round(gbs, 2), "unit": "GB/s",
            "us_per_launch": round(dt * 1e6, 3),
            "orientation": "upstream GGUF [out][in]: row n = the 8 super-blocks of output n along K",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": ctx.hbm, "unit": "GB/s",
                         "frac": round(gbs / ctx.hbm, 4), "traffic": None, "peak_kind": ctx.peak_kind,
                         "kernel": "vkq::gemv_rows_kernel<Q4_K,1>", "algorithmic_bytes_per_launch": b},
            "l2": f"{nc} rotated weight copies ({nc * base.nbytes / 1e6:.0f} MB), L2 flushed before the timed region"}


def secondary_gemm(ctx, args):
    name = "q5k_prefill_gemm_512x2048x11008"
    dt, qt, K, N, M, nc, nb = gemv_workload(ctx, name, max(20, min(args.steps, 200)))
    flops = 2 * M * K * N
    tf = flops / dt / 1e12
    traffic, kname = committed_traffic(name)
    return {"workload": name, "value": round(tf, 2), "unit": "TFLOP/s", "us_per_launch": round(dt * 1e6, 3),
            "dtype": "bf16 operands, fp32 accumulate",
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": ctx.bf16, "unit": "TFLOP/s",
                         "frac": round(tf / ctx.bf16, 4), "peak_kind": ctx.peak_kind + " bf16 burst",
                         "traffic": traffic, "kernel": kname or "vkq::gemm_kernel<Q5_K>",
                         "algorithmic_flops_per_launch": flops},
            "launches_per_step": 2, "kernels": "x_to_bf16_kernel + vkq::gemm_kernel<Q5_K>",
            "l2": f"{nc} rotated weight copies ({nc * nb / 1e6:.0f} MB), L2 flushed before the timed region"}


# ---------------------------------------------------------------- whole-model decode
class Linear:
    """One linear layer of a model step on this rank: the full weight
    (1 GPU, or replicated narrow layers), or this rank's shard with a channel
    that all-gathers the output into every rank's buffer ("gemm": a whole
    super-block column shard run through the GEMM, gathered by NCCL)."""

    def __init__(self, ctx, qtype, K, N, seed, M, channel=None, replicate=False, bounds=None):
        torch = ctx.torch
        from vibrant_b200 import synth
        from vibrant_b200 import tensor as vt
        self.ctx, self.qtype, self.K, self.N, self.M = ctx, qtype, K, N, M
        full = synth.weights_device(qtype, K, N, seed, ctx.dev)
        self.channel = None if (ctx.world == 1 or replicate) else channel
        if self.channel is None:
            self.w = vt.QuantWeight(qtype, K, N, full, device=ctx.dev)
            self.out = torch.empty(M, N, device=ctx.dev)
            self.width = N
        else:
            self.w = vt.ShardedWeight(qtype, K, N, ctx.world, ctx.rank, full, device=ctx.dev, bounds=bounds)
            self.width = self.w.width
            self.out = None
            if self.channel == "gemm":
                self.plain = self.w.as_weight()
                self.out = torch.empty(M, self.width, device=ctx.dev)
        del full
        self.ws = vt.workspace(max(1, vt.workspace_bytes(qtype, max(M, 9) if M > 8 else M, K, self.width,
                                                         ctx.local)), ctx.local)

    def __call__(self, x):
        from vibrant_b200 import tensor as vt
        if self.channel is None:
            vt.matmul(x, self.w, out=self.out, ws=self.ws, stream=self.ctx.stream)
            return self.out
        if self.channel == "gemm":
            vt.matmul(x, self.plain, out=self.out, ws=self.ws, stream=self.ctx.stream)
            return self.out
        return self.channel.gemv(x, self.w, ws=self.ws, stream=self.ctx.stream)


def decode_3b(ctx, args):
    """The full 3B-class decode step (config 3): 36 layers of {RMSNorm, q, k,
    v, RoPE on q and k, the new token's K and V appended to the layer's KV
    cache, attention over the cache, o, RMSNorm, gate, up, SiLU*up, down} and
    the final RMSNorm + Q6_K LM head, batch 1, at a context of CTX_3B tokens
    (the caches hold random keys and values for the earlier tokens).  At N > 1
    every linear layer is row-sharded with the all-gather fused into its
    GEMV, except k and v (256 outputs: replicated, their whole weight is one
    super-block column); RoPE and attention then run whole on every rank."""
    torch = ctx.torch
    import numpy as np
    from oracle import kq_oracle
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    m = synth.MODEL_3B
    chans = {}
    if ctx.world > 1:
        for role, n in (("q", m["q_out"]), ("o", m["hidden"]), ("gate", m["ffn"]), ("up", m["ffn"]),
                        ("down", m["hidden"]), ("lm", m["vocab"])):
            chans[role] = vt.PeerGather(ctx.pg.group.WORLD, ctx.rank, ctx.world, ctx.local, n, m_max=1)
    layers = []
    for li in range(m["layers"]):
        lay = {}
        for j, (role, qt, K, N) in enumerate(synth.layer_shapes(m)):
            lay[role] = Linear(ctx, qt, K, N, seed=1000 * li + j, M=1, channel=chans.get(role),
                               replicate=role in ("k", "v"))
        layers.append(lay)
    head = Linear(ctx, m["head"], m["hidden"], m["vocab"], seed=999_999, M=1, channel=chans.get("lm"))
    norm_w = torch.ones(max(m["hidden"], m["q_out"]), device=ctx.dev)
    x0 = torch.from_numpy(synth.activations(1, m["hidden"], seed=21)).to(ctx.dev)
    h = torch.empty(1, m["hidden"], device=ctx.dev)
    h2 = torch.empty(1, m["hidden"], device=ctx.dev)
    act = torch.empty(1, m["ffn"], device=ctx.dev)
    st = ctx.stream
    taps = {}

    # attention: 16 query / 2 KV heads of 128, this token at position
    # CTX_3B - 1 of every layer's cache [kv_heads][CTX_3B][128]
    hd = 128
    heads, kvh = m["q_out"] // hd, m["kv_out"] // hd
    cos_t, sin_t = (torch.from_numpy(t).to(ctx.dev) for t in vkq.rope_tables(hd, 1000000.0, CTX_3B))
    pos = torch.full((1,), CTX_3B - 1, dtype=torch.int32, device=ctx.dev)
    gen = torch.Generator(device=ctx.dev)
    gen.manual_seed(31)
    kcache = [torch.randn(kvh, CTX_3B, hd, device=ctx.dev, generator=gen) for _ in range(m["layers"])]
    vcache = [torch.randn(kvh, CTX_3B, hd, device=ctx.dev, generator=gen) for _ in range(m["layers"])]
    attn = torch.empty(1, m["q_out"], device=ctx.dev)

    def attend(li, q, k, v):
        """RoPE on q and k, the new K and V appended at row CTX_3B - 1 of the
        layer's caches and attention over the whole cache, in one launch."""
        vkq.attention_rope_decode_f32(q.data_ptr(), k.data_ptr(), v.data_ptr(), cos_t.data_ptr(), sin_t.data_ptr(),
                                      pos.data_ptr(), kcache[li].data_ptr(), vcache[li].data_ptr(), attn.data_ptr(),
                                      1, heads, kvh, CTX_3B, CTX_3B, hd, CTX_3B, ctx.local, st)
        return attn

    # q|k|v and gate|up(+SiLU) in one launch each, RMSNorm folded in; on
    # several GPUs q and gate|up are this rank's shards, gathered in the
    # launch, and k, v whole on every rank
    fused = True
    qkv_out = [torch.empty(1, n, device=ctx.dev) for n in (m["q_out"], m["kv_out"], m["kv_out"])]
    g_hidden = norm_w[:m["hidden"]]

    def qkv(x, lay):
        if chans:
            return chans["q"].linear_fused(x, [lay["q"].w, lay["k"].w, lay["v"].w], norm_w=g_hidden, eps=1e-6,
                                           outs=qkv_out[1:], stream=st)
        return vt.linear_fused(x, [lay["q"].w, lay["k"].w, lay["v"].w], norm_w=g_hidden, eps=1e-6,
                               outs=qkv_out, stream=st)[0]

    def gate_up(o, lay):
        if chans:
            return chans["gate"].linear_fused(o, [lay["gate"].w, lay["up"].w], norm_w=g_hidden, eps=1e-6,
                                              silu_mul=True, stream=st)
        vt.linear_fused(o, [lay["gate"].w, lay["up"].w], norm_w=g_hidden, eps=1e-6, silu_mul=True, outs=[act],
                        stream=st)
        return act

    def token_fused(_i):
        x = x0
        for li, lay in enumerate(layers):
            q = qkv(x, lay)
            o = lay["o"](attend(li, q, qkv_out[1], qkv_out[2]))
            a = gate_up(o, lay)
            x = lay["down"](a)
        vkq.rms_norm(x.data_ptr(), norm_w.data_ptr(), h.data_ptr(), 1, m["hidden"], 1e-6, ctx.local, st)
        return head(h)

    def token(_i):
        x = x0
        for li, lay in enumerate(layers):
            vkq.rms_norm(x.data_ptr(), norm_w.data_ptr(), h.data_ptr(), 1, m["hidden"], 1e-6, ctx.local, st)
            q = lay["q"](h)
            k = lay["k"](h)
            v = lay["v"](h)
            o = lay["o"](attend(li, q, k, v))
            vkq.rms_norm(o.data_ptr(), norm_w.data_ptr(), h2.data_ptr(), 1, m["hidden"], 1e-6, ctx.local, st)
            g = lay["gate"](h2)
            u = lay["up"](h2)
            vkq.silu_mul(g.data_ptr(), u.data_ptr(), act.data_ptr(), m["ffn"], ctx.local, st)
            x = lay["down"](act)
            if li == 0:
                taps["h"], taps["q"] = h, q
        vkq.rms_norm(x.data_ptr(), norm_w.data_ptr(), h.data_ptr(), 1, m["hidden"], 1e-6, ctx.local, st)
        return head(h)

    align = (lambda: chans["q"].gemv(h, layers[0]["q"].w, ws=layers[0]["q"].ws, stream=st)) if chans else None
    steps = max(3, min(args.steps, 20))
    dt = timed_graph(ctx, token_fused if fused else token, steps, 2, align=align)
    ctx.status("the 3B decode step")
    # parity of layer 0's q projection on every rank: the (h, q) pair of one token
    with torch.cuda.stream(st):
        vkq.rms_norm(x0.data_ptr(), norm_w.data_ptr(), h.data_ptr(), 1, m["hidden"], 1e-6, ctx.local, st)
        if fused:
            q = qkv(x0, layers[0])
        else:
            q = layers[0]["q"](h)
    torch.cuda.synchronize(ctx.dev)
    hv = h.cpu().numpy().copy()
    qv = q.cpu().numpy().copy()
    wq0 = synth.weights_device(m["q4"], m["hidden"], m["q_out"], 0, ctx.dev).cpu().numpy()
    wd = kq_oracle.dequantize(m["q4"], wq0)[:m["hidden"] * m["q_out"]].reshape(m["hidden"], m["q_out"])
    wd = wd.astype(np.float64)
    x64 = hv.astype(np.float64).reshape(-1)
    err = float(np.max(np.abs(qv.reshape(-1).astype(np.float64) - x64 @ wd) / (np.abs(x64) @ np.abs(wd))))
    err = ctx.allmax(err)
    ctx.status("the 3B parity call")
    for c in chans.values():
        c.close()
    nbytes = synth.model_bytes(m)
    kv_bytes = m["layers"] * 2 * kvh * CTX_3B * hd * 4  # the caches attention reads, K and V
    launches = m["layers"] * ((4 if fused else 10) + 1) + 2  # + the fused RoPE/append/attention launch
    return {"workload": "decode_3b_q4k_q6k_36x2048", "value": round(1.0 / dt, 2), "unit": "tokens/s",
            "ms_per_token": round(dt * 1e3, 4), "weight_bytes_per_token": nbytes,
            "context_tokens": CTX_3B, "kv_cache_bytes_per_token": kv_bytes,
            "gbs": round((nbytes + kv_bytes) / dt / 1e9, 1),
            "hbm_frac_per_gpu": round((nbytes / ctx.world + kv_bytes) / dt / 1e9 / ctx.hbm, 4),
            "launches_per_token": launches, "parity_layer0_q_max_rel_err": err,
            "fused": ("rms_norm+q|k|v and rms_norm+gate|up+SiLU*up in one launch each "
                      + ("(vkq_linear_fused_allgather: q and gate|up sharded and gathered in the launch)"
                         if chans else "(vkq_linear_fused)"))
            if fused else "none: every linear and elementwise step is its own launch",
            "parallelism": "single GPU" if ctx.world == 1 else
            f"q, o, gate|up, down and the LM head row-sharded over {ctx.world} GPUs with the all-gather fused "
            "into their launches (k, v replicated)",
            "steps": steps}


def sweep_14b(ctx, args):
    """14B/32B-class batched decode (config 4): 64 layers x {q, k, v, o, gate,
    up, down}, all Q4_K, for M in {1, 4, 16, 64}.  Every linear takes a fixed
    activation of its input width.  M <= 8 runs the fp32 GEMV (at N > 1
    row-sharded with the fused all-gather); M > 8 the tcgen05 GEMM (at N > 1
    on whole super-block column shards, outputs all-gathered with NCCL).
    k and v (1024 outputs, four super-block columns) are replicated at N > 1."""
    torch = ctx.torch
    from vibrant_b200 import synth
    from vibrant_b200 import tensor as vt
    m = synth.MODEL_14B
    out = {"workload": "decode_sweep_14b_q4k_64x5120", "per_m": {}}
    nbytes = synth.model_bytes(m, with_head=False)
    params = sum(K * N for _, _, K, N in synth.layer_shapes(m)) * m["layers"]

    def block_bounds(N):
        nb = N // 256
        per, extra = divmod(nb, ctx.world)
        lo = (ctx.rank * per + min(ctx.rank, extra)) * 256
        return lo, lo + (per + (1 if ctx.rank < extra else 0)) * 256

    for M in (1, 4, 16, 64):
        chans = {}
        if ctx.world > 1 and M <= 8:
            for n in (m["hidden"], m["ffn"]):
                chans[n] = vt.PeerGather(ctx.pg.group.WORLD, ctx.rank, ctx.world, ctx.local, n, m_max=M)
        layers = []
        for li in range(m["layers"]):
            lay = []
            for j, (role, qt, K, N) in enumerate(synth.layer_shapes(m)):
                rep = role in ("k", "v") and ctx.world > 1
                if ctx.world > 1 and M > 8 and not rep:
                    lin = Linear(ctx, qt, K, N, seed=7000 * li + j, M=M, channel="gemm", bounds=block_bounds(N))
                else:
                    lin = Linear(ctx, qt, K, N, seed=7000 * li + j, M=M, channel=chans.get(N), replicate=rep)
                lay.append((K, lin, role))
            layers.append(lay)
        xs = {K: torch.from_numpy(synth.activations(M, K, seed=K + M)).to(ctx.dev)
              for K in (m["hidden"], m["q_out"], m["ffn"])}
        gathered = {}
        # M == 1: the decode step's fused launches (q|k|v in one, gate|up with
        # SiLU * up in one; sharded and gathered in the launch at N > 1)
        fused = M == 1
        kv_outs = [torch.empty(M, m["kv_out"], device=ctx.dev) for _ in range(2)]
        act = torch.empty(M, m["ffn"], device=ctx.dev)

        def fused_layer(lay):
            r = {role: lin for _, lin, role in lay}
            h, f = m["hidden"], m["ffn"]
            if chans:
                chans[m["q_out"]].linear_fused(xs[h], [r["q"].w, r["k"].w, r["v"].w], outs=kv_outs, stream=ctx.stream)
                r["o"](xs[m["q_out"]])
                chans[f].linear_fused(xs[h], [r["gate"].w, r["up"].w], silu_mul=True, stream=ctx.stream)
            else:
                vt.linear_fused(xs[h], [r["q"].w, r["k"].w, r["v"].w], outs=[r["q"].out] + kv_outs,
                                stream=ctx.stream)
                r["o"](xs[m["q_out"]])
                vt.linear_fused(xs[h], [r["gate"].w, r["up"].w], silu_mul=True, outs=[act], stream=ctx.stream)
            r["down"](xs[f])

        def step(_i):
            for lay in layers:
                if fused:
                    fused_layer(lay)
                    continue
                for K, lin, _ in lay:
                    y = lin(xs[K])
                    if lin.channel == "gemm":
                        maxw = -(-lin.N // 256 // ctx.world) * 256
                        key = (lin.N, maxw)
                        if key not in gathered:
                            gathered[key] = (torch.empty(M * maxw, device=ctx.dev),
                                             torch.empty(ctx.world * M * maxw, device=ctx.dev))
                        send, recv = gathered[key]
                        send[:M * lin.width].copy_(y.view(-1))
                        ctx.pg.all_gather_into_tensor(recv, send)

        steps = max(3, min(args.steps, 8))
        if not (ctx.world > 1 and M > 8):
            dt = timed_graph(ctx, step, steps, 2)
        else:   # NCCL calls inside: eager, timed with events (the same count on every rank)
            with torch.cuda.stream(ctx.stream):
                for i in range(2):
                    step(i)
            ctx.flush_l2()
            ctx.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(ctx.stream):
                e0.record(ctx.stream)
                for i in range(steps):
                    step(i)
                e1.record(ctx.stream)
            torch.cuda.synchronize(ctx.dev)
            ctx.barrier()
            dt = ctx.allmax(e0.elapsed_time(e1) / 1e3 / steps)
        ctx.status(f"the 14B sweep at M={M}")
        tf = 2 * M * params / dt / 1e12
        gbs = nbytes / dt / 1e9
        out["per_m"][str(M)] = {
            "ms_per_step": round(dt * 1e3, 4), "tokens_per_s": round(M / dt, 1), "gbs": round(gbs, 1),
            "tflops": round(tf, 2), "hbm_frac_per_gpu": round(gbs / ctx.world / ctx.hbm, 4),
            "tensor_frac_per_gpu": round(tf / ctx.world / ctx.bf16, 4),
            "path": ("fp32 GEMV" + (" + fused peer all-gather" if ctx.world > 1 else "")
                     + (", q|k|v and gate|up+SiLU*up fused (4 launches per layer)" if fused else "")) if M <= 8 else
            ("tcgen05 GEMM" + (" + NCCL all-gather" if ctx.world > 1 else ""))}
        for c in chans.values():
            c.close()
        del layers
        torch.cuda.empty_cache()
    out["weight_bytes_per_step"] = nbytes
    out["parallelism"] = "single GPU" if ctx.world == 1 else f"row-sharded over {ctx.world} GPUs"
    return out


# ---------------------------------------------------------------- driver
SECONDARY = (("q6k_vocab_gemv_2048x151936", secondary_q6k, True),
             ("q5k_prefill_gemm_512x2048x11008", secondary_gemm, True),
             ("q4k_upstream_gemv_11008x2048", secondary_upstream, True),
             ("decode_3b", decode_3b, False),
             ("decode_sweep_14b", sweep_14b, False))


def run_ours(args):
    import torch
    from vibrant_b200 import vkq
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1 and (local >= torch.cuda.device_count() or world > torch.cuda.device_count()):
        # ranks whose kernels wait on one another must never share a GPU
        raise SystemExit(f"{world} ranks need {world} GPUs (one process per GPU); {torch.cuda.device_count()} visible")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", local))
        pg = dist
    vkq.load()
    ctx = Ctx(torch, rank, world, local, pg)
    hl = headline(ctx, args)
    secondary, cpu = {}, None
    only = set(args.only.split(",")) if args.only else None
    if not args.no_secondary:
        for name, fn, single in SECONDARY:
            if (single and world > 1) or (only is not None and name not in only):
                continue
            t0 = time.time()
            secondary[name] = fn(ctx, args)
            secondary[name]["wall_s"] = round(time.time() - t0, 1)
    if rank == 0 and world == 1:
        cpu = cpu_line(cpu_reference(3, 1, budget_s=args.cpu_seconds), hl["total"])
    step_s = hl["dt"]
    value = hl["total"] / step_s / 1e9
    achieved = hl["shard_alg"] / step_s / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(step_s * 1e3, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; d, dmin, scale and quant distributions of the workload description)",
        "config": {"workload": HEADLINE, "qtype": "Q4_K", "K": 2048, "N": 11008, "M": 1,
                   "columns_per_rank": hl["hi"] - hl["lo"],
                   "parallelism": "single GPU" if world == 1 else
                   f"row-sharded output columns over {world} GPUs (each holds its row-block shard only), "
                   "all-gather fused into the GEMV (flagged-word stores into every other rank's channel over NVLink)",
                   "l2": f"{hl['copies']} rotated weight copies ({hl['copies'] * hl['copy_bytes'] / 1e6:.0f} MB per "
                         "GPU) and the L2 flushed before the timed region"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": ctx.hbm, "unit": "GB/s",
                     "frac": round(achieved / ctx.hbm, 4), "traffic": hl["traffic"], "peak_kind": ctx.peak_kind,
                     "kernel": hl["kernel"], "algorithmic_bytes_per_launch": hl["shard_alg"],
                     "us_per_launch": round(step_s * 1e6, 3)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(hl["total"] / hl["e_dt"] / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": hl["h2d"], "d2h_bytes_per_step": hl["d2h"],
                "ms_per_step": round(hl["e_dt"] * 1e3, 5),
                "path": "vkq_matmul_host (N=1: one call per step; pinned buffers reached through the host mapping: a staging kernel reads x, the GEMV stores y into host memory) / copies around vkq_gemv_allgather (N>1); ctypes, eager launches"},
        "parity": {"max_rel_err": hl["err"], "tolerance": 1e-5, "checked": "all columns on every rank vs the oracle"},
        "gpu_launches": args.steps,
        "clocks": hl["clocks"],
        "secondary": secondary,
    }
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_probe(args):
    """One workload through the C ABI, CUDA-event time per launch (graph
    replay of --steps launches over COPIES rotated weight copies)."""
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    parts = [int(v) for v in args.probe.split(",")]
    qt, K, N, M = parts[:4]
    copies = parts[4] if len(parts) > 4 else 1
    torch.cuda.set_device(0)
    w = [vt.QuantWeight(qt, K, N, synth.weights(qt, K, N, seed=1))]
    for _ in range(copies - 1):
        w.append(vt.QuantWeight(qt, K, N, w[0].buf.clone()))
    x = torch.from_numpy(synth.activations(M, K, seed=2)).cuda()
    y = torch.empty(M, N, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(3):
            vt.matmul(x, w[i % copies], out=y, stream=st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(args.steps):
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
    dt = e0.elapsed_time(e1) / 1e3 / args.steps
    b = synth.n_blocks(K, N) * synth.BLOCK_BYTES[qt] + 4 * M * (K + N)
    print(f"qt={qt} K={K} N={N} M={M}: {dt * 1e6:.2f} us/launch  {b / dt / 1e9:.1f} GB/s  "
          f"{2 * M * K * N / dt / 1e12:.1f} TFLOP/s  status={vkq.device_status(0)}", flush=True)


def run_probe_fused(args):
    """One fused launch of the 3B layer (vkq_linear_fused, RMSNorm prologue)
    over rotated weight copies, CUDA-event time per launch of a graph
    replay of --steps launches."""
    import torch
    from vibrant_b200 import synth, vkq
    from vibrant_b200 import tensor as vt
    m = synth.MODEL_3B
    K = m["hidden"]
    widths = (m["q_out"], m["kv_out"], m["kv_out"]) if args.probe_fused == "qkv" else (m["ffn"], m["ffn"])
    silu = args.probe_fused == "gate_up"
    torch.cuda.set_device(0)
    one = sum(synth.n_blocks(K, n) * synth.BLOCK_BYTES[vkq.Q4_K] for n in widths)
    copies = max(2, -(-(512 << 20) // one))
    sets = [[vt.QuantWeight(vkq.Q4_K, K, n, synth.weights_device(vkq.Q4_K, K, n, 100 * c + i, 0))
             for i, n in enumerate(widths)] for c in range(copies)]
    x = torch.from_numpy(synth.activations(1, K, seed=2)).cuda()
    g = torch.ones(K, device="cuda")
    outs = [torch.empty(1, widths[0], device="cuda")] if silu else [torch.empty(1, n, device="cuda") for n in widths]
    st = torch.cuda.Stream()

    def launch(i):
        vt.linear_fused(x, sets[i % copies], norm_w=g, eps=1e-6, silu_mul=silu, outs=outs, stream=st)

    with torch.cuda.stream(st):
        for i in range(3):
            launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(args.steps):
            launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        graph.replay()
        st.synchronize()
        e0.record(st)
        graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / args.steps
    b = one + 4 * K + 4 * (widths[0] if silu else sum(widths)) + 4 * K
    print(f"fused {args.probe_fused} 2048 -> {'+'.join(map(str, widths))}: {dt * 1e6:.2f} us/launch  "
          f"{b / dt / 1e9:.1f} GB/s ({copies} weight sets)  status={vkq.device_status(0)}", flush=True)


def main():
    args = parse()
    if args.gemv != "auto" and args.impl == "ours":
        from vibrant_b200 import vkq
        vkq.set_gemv_path({"simt": vkq.GEMV_SIMT, "tc": vkq.GEMV_TC, "strip": vkq.GEMV_STRIP}[args.gemv])
    if args.probe:
        run_probe(args)
    elif args.probe_fused:
        run_probe_fused(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
