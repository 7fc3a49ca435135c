#!/usr/bin/env python
"""Benchmark of the Q8_0 W8A8 hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload gemv|gemm]

Workloads (seeded synthetic data, weights quantized with the reference's Q8_0 rule):
  gemv   config 0: one step = the fused activation quantize + the decode GEMV y = W x, W 8192 x 2048 (gs 64).
         Inputs rotate through enough weight copies to exceed L2 (126 MB) three times over, so every step streams W
         from HBM.
  gemm   config 1: one step = quantize X [T x 4096] + the prefill GEMM against W1 [14336 x 4096], T = 2048.

--impl reference times the reference's own CPU implementation (oracle/_ref, compiled from its sources) of the same
step on all host cores, through its own API (k_quantize + k_matmul_q8 / k_gemm_q8 on a worker team of every core).
Multi-GPU (torchrun): every rank runs an independent replica of the step (the kernel-level workloads do not shard);
value is the sum over ranks, timed as the max over ranks.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
METRIC = "Q8_0 8B decode tok/s & prefill tok/s at 1/2/4/8 B200; GEMV HBM GB/s %"
L2_BYTES = 126 * 1024 * 1024


def load_package():
    import importlib.util
    if "llama3x_b200" in sys.modules:
        return sys.modules["llama3x_b200"]
    pkg = ROOT / "llama3.x.c_b200"
    spec = importlib.util.spec_from_file_location("llama3x_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llama3x_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        if not self.proc or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- workloads --------------------------------------------------------------------------------------------------

def gemv_workload(kc, torch, d=8192, n=2048, gs=64):
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    w = torch.randn((d, n), generator=g, device="cuda") * 0.02
    wq, ws = kc.quantize(w, gs)
    del w
    wbytes = wq.numel() + ws.numel() * 4
    copies = max(2, -(-3 * L2_BYTES // wbytes))
    W = [(wq.clone(), ws.clone()) for _ in range(copies)]
    g.manual_seed(1)
    x = torch.randn(n, generator=g, device="cuda")
    xq = torch.empty(n, dtype=torch.int8, device="cuda")
    xs = torch.empty(n // gs, device="cuda")
    y = torch.empty(d, device="cuda")
    alg_bytes = d * n + d * (n // gs) * 4 + n + (n // gs) * 4 + d * 4

    def step(i, ev=None):
        kc.k_quantize(xq, xs, x, n, gs)
        a, b = W[i % copies]
        if ev:
            ev[0].record()
        kc.k_matmul_q8(y, xq, xs, a, b, n, d, gs)
        if ev:
            ev[1].record()

    # end-to-end: pinned host x in, pinned host y out, through the public API
    xh = torch.randn(n, generator=torch.Generator().manual_seed(1)).pin_memory()
    yh = torch.empty(d).pin_memory()

    def step_e2e(i):
        x.copy_(xh, non_blocking=True)
        step(i)
        yh.copy_(y, non_blocking=True)

    return dict(step=step, step_e2e=step_e2e, launches=2, alg_bytes=alg_bytes, unit="GB/s",
                per_step_units=alg_bytes / 1e9, workload=f"config0 GEMV {d}x{n} gs{gs} (+ fused-quantize launch)",
                kernel="gemv_q8_kernel", h2d=n * 4, d2h=d * 4, copies=copies, dtype="int8 x int8 -> int32 -> f32",
                shape=dict(d=d, n=n, gs=gs))


def cpu_reference_gemv(seconds=5.0, d=8192, n=2048, gs=64):
    """The reference's k_matmul_q8 (LLAMA_KERNELS=auto: AVX-512 VNNI where the CPU has it) on a team of every core."""
    from oracle import oracle as O
    L = O.ref()
    L.kernels_backend_init()
    isa = O.KERNELS_AVX512 if O.ref_select(O.KERNELS_AVX512) else O.KERNELS_SCALAR
    O.ref_select(isa)
    wq, ws = O.seeded_q8_matrix(d, n, gs, 0)
    copies = max(2, -(-512 * 2**20 // (wq.nbytes + ws.nbytes)))  # rotate past the host caches (gemm_bench --cold-mib)
    W = [(wq.copy(), ws.copy()) for _ in range(copies)]
    xq, xs = O.quantize(np.random.default_rng(1).standard_normal(n).astype(np.float32), gs)
    out = np.empty(d, np.float32)
    inp = O.K8Input(O._p(xq, O._i8p), O._p(xs, O._f32p), None)
    ws_ = [O.K8Weight(O._p(a, O._i8p), O._p(b, O._f32p)) for a, b in W]
    for i in range(3):
        L.k_matmul_q8(O._p(out, O._f32p), ctypes.byref(inp), ws_[i % copies], n, d, gs)
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        L.k_matmul_q8(O._p(out, O._f32p), ctypes.byref(inp), ws_[calls % copies], n, d, gs)
        calls += 1
    dt = time.perf_counter() - t0
    gb = calls * (d * n + d * (n // gs) * 4 + n + (n // gs) * 4 + d * 4) / 1e9
    return {"value": gb / dt, "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
            "sample": f"{calls} calls of k_matmul_q8 {d}x{n} ({'avx512' if isa else 'scalar'}) over {dt:.1f} s, "
                      f"{copies} rotating weight copies"}


def run_ours(args):
    import torch
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    kc = load_package()
    kc.init()
    wl = gemv_workload(kc, torch)
    hbm, bf16, peak_kind = peaks()
    stream = torch.cuda.current_stream()
    K = args.steps
    for i in range(args.warmup):
        wl["step"](i)
    kc.status()
    # The K steps are captured once into a CUDA graph and replayed: the timed region is then GPU-bound (the kernels'
    # own time), not bound by Python's per-call launch overhead. External event nodes bracket every hot-path kernel.
    K = args.steps
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(K)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(K):
            wl["step"](i, evs[i])
    graph.replay()
    torch.cuda.synchronize()
    kc.status()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        start.record(stream)
        graph.replay()
        stop.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    kc.status()
    ms = max_over_ranks(world, start.elapsed_time(stop))
    kernel_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    value = world * K * wl["per_step_units"] / (ms / 1e3)
    del graph
    # end-to-end through the public API with host buffers (plain calls, host launch overhead included)
    for i in range(args.warmup):
        wl["step_e2e"](i)
    torch.cuda.synchronize()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        wl["step_e2e"](i)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    kc.status()
    e2e_ms = max_over_ranks(world, t0.elapsed_time(t1))
    e2e = world * K * wl["per_step_units"] / (e2e_ms / 1e3)
    achieved = wl["alg_bytes"] / (kernel_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": wl["unit"], "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms / K, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": wl["workload"], "l2": f"inputs rotate over {wl['copies']} weight copies (> 3x L2)",
                   "parallelism": f"replicas x{world}", **wl["shape"]},
        "e2e": {"value": round(e2e, 2), "unit": wl["unit"], "h2d_bytes_per_step": wl["h2d"],
                "d2h_bytes_per_step": wl["d2h"]},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None, "kernel": wl["kernel"],
                     "kernel_us": round(kernel_ms * 1e3, 3), "peak_source": f"{peak_kind} hbm_gbs"},
        "gpu_launches": wl["launches"] * K,
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_gemv(seconds=args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libllama_ref.so was not built "
                                                              "(make -C oracle where the reference sources exist)"}))
        return
    res = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference_gemv(seconds=max(0.5, args.cpu_seconds / max(1, args.steps)))
        if i >= args.warmup:
            res.append(r)
    v = float(np.mean([r["value"] for r in res]))
    line = {"metric": METRIC, "impl": "reference", "value": round(v, 3), "unit": "GB/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "int8",
            "data": "synthetic", "config": {"workload": "config0 GEMV 8192x2048 gs64"},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": res[-1]["cores"], "kind": "reference",
                             "sample": res[-1]["sample"]},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=5.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
