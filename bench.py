#!/usr/bin/env python
"""Benchmark of the Q8_0 W8A8 path on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 8b|1b|gemv|ffn|gemm|sweep] [--profile-request] [--no-cpu-baseline]
                    [--sweep-t 1,2,...] [--sweep-s 1,2,4,8] [--sweep-rows-max 16]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N   (N = 2, 4, 8)

Workloads (seeded synthetic data, random-init weights of the named architecture, Q8_0 gs 64):
  8b    config 3 (default): Llama-3.1-8B architecture (dim 4096, hidden 14336, 32 layers, 32/8 heads, vocab 128256,
        context 8192, untied classifier). One step = one request through engine_generate: a 2048-token uniform-random
        prompt batch-prefilled, then 256 tokens greedy-decoded. Tensor parallel over the N GPUs (one request, one
        token stream: strong scaling). value = decode tok/s; prefill tok/s rides along.
  1b    config 2: Llama-3.2-1B architecture (tied classifier), 128-token prompt, 256 tokens.
  gemv  config 0 kernel alone: the GEMV 8192 x 2048 on activations quantized beforehand (not the headline).
  ffn   the dominant decode kernel alone: the 8B SwiGLU GEMV (W1 and W3, 14336 x 4096 each) on rotating weights.
  gemm  config 1: the prefill GEMM alone (8B up and down projections, T = 128 / 512 / 2048).
  sweep config 4: every 8B projection's rank-0 shard at S = 1/2/4/8 times T activation rows, the tensor-core GEMM
        against one decode GEMV per row, and the crossover T per shard.

--profile-request (8b / 1b) runs one short request (the prefill and 4 greedy tokens) and nothing else, for an ncu launch
list of every kernel the request launches.

The weights (8.5 GB at 8B) exceed L2 many times over, so every decode step streams them from HBM.

--impl reference times the reference's own CPU engine (oracle/_ref/libllama_ref_engine.so, built from its sources:
engine_forward_batch + engine_forward) on all host cores on the GPU arm's workload: the same checkpoint bytes (the
engine library's engine_write_random, seed 1), the same prompt, the prompt prefilled once, then each step a bounded
sample of the greedy decode (8 tokens) at the same positions. Under torchrun only rank 0 runs it.

The 8b / 1b lines carry a `parity` block: the timed request's first 64 greedy tokens and the prompt's last logits
against the reference's own run of the same workload (tests/golden/bench_golden.npz), and whether every rank holds the
same logits. For the
gemv, ffn and gemm workloads it runs the reference's own microbenchmark instead (oracle/_ref/gemm-bench, built from
tests/gemm_bench.c) on the same shapes; those workloads' own lines carry the same figures as cpu_baseline.
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

ARCH = {
    "8b": dict(dim=4096, hidden_dim=14336, n_layers=32, n_heads=32, n_kv_heads=8, vocab_size=128256, seq_len=8192,
               shared=False),
    "1b": dict(dim=2048, hidden_dim=8192, n_layers=16, n_heads=32, n_kv_heads=8, vocab_size=128256, seq_len=2048,
               shared=True),
}
REQUEST = {"8b": (2048, 256), "1b": (128, 256)}  # prompt tokens, generated tokens
REF_DECODE = 8  # greedy tokens per timed step of the reference's engine (a bounded sample of the 256)


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


def load_engine():
    import importlib
    load_package()
    return importlib.import_module("llama3x_b200.engine")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path("/tmp") / f"llama3x_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
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
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
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
    # NCCL reduces device tensors; a gloo group (the CPU tests of this helper) reduces host tensors.
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompt_tokens(n, vocab, seed=3):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


# ---- the benchmark model: one seeded checkpoint for the GPU engine and the reference's engine --------------------

CKPT_SEED = 1
GOLDEN = ROOT / "tests" / "golden" / "bench_golden.npz"  # the reference's own tokens and logits on these workloads


def checkpoint_bytes(a, gs=64):
    d, h, L, V = a["dim"], a["hidden_dim"], a["n_layers"], a["vocab_size"]
    kv = d // a["n_heads"] * a["n_kv_heads"]

    def q8(n):
        return n + n // gs * 4

    return 256 + (2 * L + 1) * d * 4 + q8(V * d) * (1 if a["shared"] else 2) + \
        L * (2 * q8(d * d) + 2 * q8(d * kv) + 3 * q8(d * h))


def checkpoint_dir():
    shm = Path("/dev/shm")
    if shm.exists() and os.statvfs(shm).f_bavail * os.statvfs(shm).f_frsize > 24 * 2**30:
        return shm
    return Path("/tmp")


def bench_checkpoint(arch, rank=0, world=1):
    """engine_write_random's seeded checkpoint of the architecture (seed 1): written once by rank 0 (kept when a file of
    the right size is already there: the reference's arm writes the same bytes), then read by every rank."""
    a = ARCH[arch]
    path = checkpoint_dir() / f"llama3x_bench_{arch}.bin"
    if rank == 0 and not (path.exists() and path.stat().st_size == checkpoint_bytes(a)):
        load_engine().write_random(path, **a, seed=CKPT_SEED)
    barrier(world)
    return path


# ---- the dominant kernel: the decode GEMV, timed alone ------------------------------------------------------------

def gemv_roofline(kc, torch, rows, cols, gs=64, launches=60, swiglu=True):
    """The SwiGLU decode GEMV (W1 and W3, `rows` x `cols` each, the largest per-layer weight stream) on enough rotating
    weight copies to exceed L2 three times, each launch bracketed by CUDA events inside one captured graph.
    Returns (algorithmic bytes per launch, mean launch microseconds)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    mats = []
    for _ in range(2 if swiglu else 1):
        w = torch.randn((rows, cols), generator=g, device="cuda") * 0.02
        mats.append(kc.quantize(w, gs))
        del w
    wbytes = sum(q.numel() + s.numel() * 4 for q, s in mats)
    copies = max(2, -(-3 * L2_BYTES // wbytes))
    W = [[(q.clone(), s.clone()) for q, s in mats] for _ in range(copies)]
    x = torch.randn(cols, generator=g, device="cuda")
    xq, xs = kc.quantize(x, gs)
    y = torch.empty(rows, device="cuda")
    alg = wbytes + cols + (cols // gs) * 4 + rows * 4

    def launch(i):
        m = W[i % copies]
        if swiglu:
            kc.gemv(xq, xs, m[0][0], m[0][1], gs, kind=kc.K_SWIGLU, out=y, w3=m[1])
        else:
            kc.gemv(xq, xs, m[0][0], m[0][1], gs, out=y)

    for i in range(5):
        launch(i)
    kc.status()
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(launches)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(launches):
            evs[i][0].record()
            launch(i)
            evs[i][1].record()
    graph.replay()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    kc.status()
    us = float(np.mean([a.elapsed_time(b) for a, b in evs])) * 1e3
    del graph
    return alg, us


# ---- the reference's CPU path: its engine, and its kernels alone ---------------------------------------------------

def reference_engine_sample(arch, steps, warmup, decode_per_step=REF_DECODE):
    """The reference's Q8 engine (oracle/_ref/libllama_ref_engine.so: engine_forward_batch over the prompt in its own
    microbatches, then engine_forward per greedy token) on all host cores, on the GPU arm's workload: the same
    checkpoint bytes (engine_write_random, seed 1), the same prompt, decoding at the same positions. The prompt is
    prefilled once (timed: prefill tok/s); each step then decodes `decode_per_step` tokens continuing the greedy stream
    from position len(prompt) on; the first `warmup` steps are not timed. Returns the dict of a cpu_baseline entry plus
    prefill tok/s."""
    from oracle import oracle as O
    lib_path = O.HERE / "_ref" / "libllama_ref_engine.so"
    if not lib_path.exists():
        return {"unavailable": "oracle/_ref/libllama_ref_engine.so was not built (make -C oracle where the reference "
                               "sources exist)"}
    cores = os.cpu_count() or 1
    os.environ.setdefault("LLAMA_THREADS", str(cores))
    a = ARCH[arch]
    t0 = time.perf_counter()
    path = bench_checkpoint(arch)
    gen_s = time.perf_counter() - t0
    eng = load_engine()  # the layout-compatible Model struct (include/runtime.h) and the checkpoint writer
    L = ctypes.CDLL(str(lib_path))
    MP = ctypes.POINTER(eng.Model)
    L.engine_load_context.argtypes = [MP, ctypes.c_char_p, ctypes.c_int]
    L.engine_forward.argtypes = [MP, ctypes.c_int, ctypes.c_int]
    L.engine_forward.restype = ctypes.POINTER(ctypes.c_float)
    L.engine_forward_batch.argtypes = [MP, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.engine_forward_batch.restype = ctypes.POINTER(ctypes.c_float)
    L.engine_max_batch.argtypes = [MP]
    L.engine_free.argtypes = [MP]
    P, D = REQUEST[arch]
    total = (warmup + steps) * decode_per_step
    model = eng.Model()
    t0 = time.perf_counter()
    L.engine_load_context(ctypes.byref(model), os.fsencode(str(path)), P + total)
    load_s = time.perf_counter() - t0
    V = a["vocab_size"]
    prompt = prompt_tokens(P, V)
    mb = L.engine_max_batch(ctypes.byref(model))
    t0 = time.perf_counter()
    i = 0
    while i < P:
        n = min(mb, P - i)
        logits = L.engine_forward_batch(ctypes.byref(model), (ctypes.c_int * n)(*prompt[i:i + n].tolist()), n, i,
                                        eng.LOGITS_LAST if i + n == P else eng.LOGITS_NONE)
        i += n
    prefill_s = time.perf_counter() - t0
    tok = int(np.argmax(np.ctypeslib.as_array(logits, (V,))))
    pos, dec = P, []
    for s in range(warmup + steps):
        t0 = time.perf_counter()
        for _ in range(decode_per_step):
            logits = L.engine_forward(ctypes.byref(model), tok, pos)
            tok = int(np.argmax(np.ctypeslib.as_array(logits, (V,))))
            pos += 1
        if s >= warmup:
            dec.append(time.perf_counter() - t0)
    L.engine_free(ctypes.byref(model))
    decode = decode_per_step * len(dec) / sum(dec)
    return {"value": round(decode, 3), "unit": "tok/s", "cores": int(os.environ["LLAMA_THREADS"]), "kind": "reference",
            "prefill_tok_s": round(P / prefill_s, 2),
            "sample": f"reference engine (engine_forward_batch in microbatches of {mb}, then engine_forward; "
                      f"LLAMA_KERNELS=auto) on the {arch} architecture, the GPU arm's checkpoint and prompt: the "
                      f"{P}-token prefill once, then {steps} timed steps of {decode_per_step} greedy tokens at "
                      f"positions {P + warmup * decode_per_step}..{P + total - 1} after {warmup} untimed; checkpoint "
                      f"ready in {gen_s:.0f} s, loaded in {load_s:.0f} s"}


def reference_kernel_bench(bench_args, reps, kernels="auto"):
    """The reference's own GEMV/GEMM microbenchmark (tests/gemm_bench.c, compiled from its sources into
    oracle/_ref/gemm-bench by oracle/Makefile) with `--kernel q8 <bench_args> --reps <reps>` on all host cores and
    LLAMA_KERNELS=<kernels>. Returns {"cores", "lines", "command"} with its JSON lines, or {"unavailable": why}."""
    exe = ROOT / "oracle" / "_ref" / "gemm-bench"
    if not exe.exists():
        return {"unavailable": "oracle/_ref/gemm-bench was not built (make -C oracle where the reference sources exist)"}
    env = dict(os.environ, LLAMA_KERNELS=kernels)
    env.setdefault("LLAMA_THREADS", str(os.cpu_count() or 1))
    cmd = [str(exe), "--kernel", "q8", *bench_args, "--reps", str(reps)]
    try:
        out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference gemm-bench did not finish within 600 s"}
    if out.returncode:
        return {"unavailable": f"reference gemm-bench exited {out.returncode}: {out.stderr.strip()[-200:]}"}
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    return {"cores": int(env["LLAMA_THREADS"]), "lines": lines,
            "command": f"LLAMA_KERNELS={kernels} " + " ".join(["gemm-bench", *cmd[1:]])}


def reference_gemv_baseline(rows, cols):
    """cpu_baseline of the decode GEMV: the reference's k_matmul_q8 (gemm-bench --gemv, one activation row, its decode
    selection LLAMA_KERNELS=auto) on one rows x cols matrix, weights cycled through 512 MiB of copies. GB/s counts the
    weight values and scales."""
    r = reference_kernel_bench(["--shapes", f"{rows}x{cols}", "--m", "1", "--gemv", "--cold-mib", "512"], reps=20)
    if "unavailable" in r:
        return r
    line = next((l for l in r["lines"] if l.get("kernel") == "gemv_rows_q8"), None)
    if line is None:
        return {"unavailable": "reference gemm-bench printed no gemv_rows_q8 line"}
    return {"value": line["weight_gbs_median"], "unit": "GB/s", "cores": r["cores"], "kind": "reference",
            "sample": f"{r['command']} ({line['isa']}): median of {line['reps']} k_matmul_q8 "
                      f"calls on {rows} x {cols}, {line['median_s'] * 1e6:.1f} us each; weight bytes / time"}


def reference_gemm_points(shapes, ts):
    """The reference's k_gemm_q8 (gemm-bench, STORE) per (N, K, T): {(N, K, T): (median us, int8 TOPS, isa)}, plus the
    run's core count and command; or {"unavailable": why}. Its fastest W8A8 prefill backend is AMX-INT8, which
    LLAMA_KERNELS=auto does not select in this tool; hosts without AMX take auto (AVX-512)."""
    args = ["--shapes", ",".join(f"{n}x{k}" for n, k in shapes), "--m", ",".join(str(t) for t in ts), "--cold-mib",
            "512"]
    r = reference_kernel_bench(args, reps=3, kernels="amx")
    if "unavailable" in r:
        r = reference_kernel_bench(args, reps=3, kernels="auto")
    if "unavailable" in r:
        return r
    pts = {(l["n"], l["k"], l["m"]): (l["median_s"] * 1e6, l["gflops_median"] / 1e3, l["isa"])
           for l in r["lines"] if l.get("kernel") == "gemm_q8"}
    return {"points": pts, "cores": r["cores"], "command": r["command"]}


# ---- our engine ---------------------------------------------------------------------------------------------------

def run_profile_request(args):
    """One request (prefill + 4 greedy tokens) on the workload's model, nothing timed: an ncu launch list target."""
    eng = load_engine()
    a = ARCH[args.workload]
    P, _ = REQUEST[args.workload]
    with eng.Engine.random(**a, seed=1, context=a["seq_len"]) as m:
        tokens = m.generate(prompt_tokens(P, a["vocab_size"]), 4)
    print(json.dumps({"profile_request": args.workload, "prompt": P, "tokens": tokens}), flush=True)


def parity_block(eng, m, arch, world, rank, prompt, tokens):
    """The GPU engine against the reference's own run of this workload (tests/golden/bench_golden.npz, made by the
    reference's engine on the same checkpoint bytes and prompt: tests/golden/make_bench_golden.py): the first 64 greedy
    tokens of the timed request, the first step's logits (the prompt's last row) bit for bit, and whether every rank
    holds the same logits. On 2 GPUs the reference's two-socket run (its own tensor-parallel split) is the comparison;
    it splits over at most two sockets, so 4 and 8 GPUs compare with its one-socket run."""
    import hashlib
    logits = m.forward_batch(prompt, 0, eng.LOGITS_LAST)
    digest = hashlib.sha256(np.ascontiguousarray(logits, np.float32).tobytes()).hexdigest()
    same = True
    if world > 1:
        import torch.distributed as dist
        digests = [None] * world
        dist.all_gather_object(digests, digest)
        same = all(d == digests[0] for d in digests)
    key = f"{arch}_s2" if world == 2 else f"{arch}_s1"
    block = {"reduction": m.reduction(), "ranks_logits_identical": same}
    if not GOLDEN.exists():
        block["unavailable"] = "tests/golden/bench_golden.npz is missing"
        return block
    g = np.load(GOLDEN)
    if key + "_tokens" not in g.files:
        block["unavailable"] = f"no reference run {key} in tests/golden/bench_golden.npz"
        return block
    ref, margins, maxes, first = (g[key + t] for t in ("_tokens", "_margins", "_maxes", "_first"))
    n = len(ref)
    ours = [int(t) for t in tokens[:n]]
    div = next((i for i, (x, y) in enumerate(zip(ours, ref.tolist())) if x != y), None)
    if div is None and len(ours) < n:
        div = len(ours)
    block.update({
        "reference": f"{key}: the reference's engine, {g[key + '_env']}" +
                     ("" if world in (1, 2) else " (its one-socket run: it splits over at most two sockets)"),
        "tokens_compared": n, "tokens_equal": div is None, "first_divergence_step": div,
        "ref_margin_at_divergence": None if div is None or div >= n else round(float(margins[div] / maxes[div]), 6),
        "first_logits_bitwise": bool((np.asarray(logits, np.float32).view(np.int32) == first.view(np.int32)).all()),
        "first_logits_max_rel_diff": float(np.abs(logits - first).max() / np.abs(first).max()),
    })
    if world > 2:
        drift = reference_split_drift(g, arch)
        if drift is not None:
            block["reference_two_socket_vs_one"] = drift
    return block


def reference_split_drift(g, arch):
    """How far the reference's own two-socket split moves it from its one-socket run on the benchmark request (both in
    tests/golden/bench_golden.npz): the scale against which a split this engine runs, and the reference cannot, is to
    be read. None when the golden file lacks either run."""
    s1, s2 = f"{arch}_s1", f"{arch}_s2"
    if s1 + "_tokens" not in g.files or s2 + "_tokens" not in g.files:
        return None
    first, margins, maxes = g[s1 + "_first"], g[s1 + "_margins"], g[s1 + "_maxes"]
    r1, r2 = g[s1 + "_tokens"].tolist(), g[s2 + "_tokens"].tolist()
    rdiv = next((i for i, (x, y) in enumerate(zip(r1, r2)) if x != y), None)
    return {"first_logits_max_rel_diff": float(np.abs(g[s2 + "_first"] - first).max() / np.abs(first).max()),
            "first_divergence_step": rdiv,
            "ref_margin_at_divergence": None if rdiv is None else round(float(margins[rdiv] / maxes[rdiv]), 6)}


def run_engine(args):
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    kc = load_package()
    eng = load_engine()
    a = ARCH[args.workload]
    P, D = REQUEST[args.workload]
    nccl_id = eng.share_comm_id(rank, world) if world > 1 else None
    t0 = time.perf_counter()
    path = bench_checkpoint(args.workload, rank, world)
    ckpt_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    m = eng.Engine.load(str(path), context=a["seq_len"], tp=(rank, world, local, nccl_id) if world > 1 else None)
    init_s = time.perf_counter() - t0
    prompt = prompt_tokens(P, a["vocab_size"])
    for _ in range(args.warmup):
        m.generate(prompt, D)
    barrier(world)
    torch.cuda.synchronize()
    m.stats_reset()
    with Clocks(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tokens = m.generate(prompt, D)
        wall = time.perf_counter() - t0
    st = m.stats()
    barrier(world)
    prefill_ms = max_over_ranks(world, st["prefill_ms"])
    decode_ms = max_over_ranks(world, st["decode_ms"])
    wall = max_over_ranks(world, wall)
    decode = st["decode_tokens"] / (decode_ms / 1e3)
    prefill = st["prefill_tokens"] / (prefill_ms / 1e3)

    parity = parity_block(eng, m, args.workload, world, rank, prompt, tokens)

    # End to end through the reference-facing API with host buffers: engine_forward per token (the token and position
    # go host -> device, the vocabulary's logits come back to the host), host argmax over the returned buffer, as
    # probe-int8 generate does with the pointer engine_forward returns.
    E = 32
    logits = m.forward_batch(prompt, 0, eng.LOGITS_LAST)
    tok = int(np.argmax(logits))
    for j in range(3):
        m.forward(tok, P + j)
    barrier(world)
    t0 = time.perf_counter()
    for j in range(E):
        tok = int(np.argmax(m.forward_view(tok, P + j)))
    e2e_s = max_over_ranks(world, time.perf_counter() - t0)
    m.close()

    # The dominant kernel alone: the SwiGLU decode GEMV of this rank's W1/W3 shard.
    hbm, peak_kind = peaks()
    rows = a["hidden_dim"] // world
    alg, us = gemv_roofline(kc, torch, rows, a["dim"])
    achieved = alg / (us / 1e6) / 1e9
    traffic = None  # DRAM bytes per launch from the ncu capture of this kernel at this shape, when one is committed
    tf = ROOT / "profiles" / f"gemv_swiglu_{rows}x{a['dim']}_full.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = int(line.split(":")[1].split()[0])
    weights = sum(v for v in weight_bytes(a, world).values())
    kernels = kernel_figures(kc, torch, args) if world == 1 and args.workload == "8b" else None
    line = {
        "metric": METRIC, "value": round(decode, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round((prefill_ms + decode_ms) / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 (W8A8, fp32 accumulate)",
        "data": "synthetic: seeded random-init Q8_0 checkpoint (engine_write_random, N(0,0.02)), uniform-random "
                "prompt ids; the same bytes the reference's arm loads",
        "config": engine_config(args.workload, P, D, world),
        "prefill_tok_s": round(prefill, 1), "decode_tok_s": round(decode, 2),
        "decode_ms_per_token": round(decode_ms / max(1, st["decode_tokens"]), 4),
        "decode_weight_gbs": round(weights / (decode_ms / max(1, st["decode_tokens"]) / 1e3) / 1e9, 1),
        "wall_s": round(wall, 3), "init_s": round(init_s, 2), "checkpoint_s": round(ckpt_s, 2),
        "tokens_last_step": len(tokens),
        "parity": parity,
        "e2e": {"value": round(E / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4 * a["vocab_size"],
                "path": "engine_forward per token (host token in, host logits out, host argmax)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "kernel": f"gemv_q8 SwiGLU {rows}x{a['dim']} x2 (decode W1/W3)", "kernel_us": round(us, 3),
                     "alg_bytes_per_launch": alg, "peak_source": f"{peak_kind} hbm_gbs"},
        "gpu_launches": int(st["kernel_launches"]),
        "clocks": clocks.summary(),
    }
    if kernels:
        line["kernels"] = kernels
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = reference_engine_sample(args.workload, steps=2, warmup=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def kernel_figures(kc, torch, args):
    """The two kernel metrics BASELINE names beside the engine, measured in the same run on one GPU: the config 0 GEMV
    (8192 x 2048, activations already quantized) as HBM GB/s and its fraction of the measured copy peak, and the
    config 1 GEMM (k_gemm_q8 STORE, up and down projections at T = 2048) as int8 TOPS and the fraction of the int8
    roof. Same timing method as --workload gemv / gemm."""
    hbm, peak_kind = peaks()
    int8_tops, int8_source = int8_peak()
    alg, us = gemv_roofline(kc, torch, *GEMV_SHAPES["gemv"], launches=40, swiglu=False)
    gbs = alg / (us / 1e6) / 1e9
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    gemm = []
    for name, (N, K) in GEMM_SHAPES.items():
        gemm += gemm_points(kc, torch, g, name, N, K, (GEMM_T[-1],), 3, 8, int8_tops, hbm)
    for p in gemm:
        del p["key"]
    torch.cuda.empty_cache()
    return {"config0_gemv": {"shape": "8192x2048", "kernel_us": round(us, 3), "achieved_gbs": round(gbs, 1),
                             "frac": round(gbs / hbm, 4), "peak": hbm, "peak_source": f"{peak_kind} hbm_gbs"},
            "config1_gemm": {"shapes": gemm, "int8_peak_tops": int8_tops, "peak_source": int8_source}}


def engine_config(arch, P, D, world):
    """The workload's `config` entry, shared by both arms."""
    a = ARCH[arch]
    return {"workload": f"config {3 if arch == '8b' else 2}: {arch.upper()} architecture, {P}-token prefill + {D} "
                        "greedy tokens per request",
            "model": f"llama-{arch}-arch", **{k: a[k] for k in ("dim", "hidden_dim", "n_layers", "n_heads",
                                                                 "n_kv_heads", "vocab_size")},
            "context": a["seq_len"], "global_batch": 1, "seq_len": P + D,
            "parallelism": f"tp{world}" if world else "cpu", "l2": "weights >> L2: every decode step streams them"}


def weight_bytes(a, world, gs=64):
    d, h, L, V = a["dim"], a["hidden_dim"], a["n_layers"], a["vocab_size"]
    kv = d // a["n_heads"] * a["n_kv_heads"]

    def q8(n):
        return n + n // gs * 4

    layer = (2 * q8(d * d) + 2 * q8(d * kv) + 3 * q8(d * h)) // world
    return {"layers": L * layer, "classifier": q8(V * d) // world}


# ---- the reference arm --------------------------------------------------------------------------------------------

def run_reference_kernels(args):
    """--impl reference for the kernel workloads (gemv, ffn, gemm): the reference's own gemm-bench on the shapes of
    this arm's line, on every host core. Each figure is the median of a bounded number of calls (20 GEMVs, 3 GEMMs
    per shape)."""
    if args.workload == "gemm":
        metric, unit = GEMM_METRIC, "TOPS"
        ref = reference_gemm_points(list(GEMM_SHAPES.values()), GEMM_T)
        if "unavailable" not in ref:
            _, tops, isa = ref["points"].get((*GEMM_SHAPES["up"], GEMM_T[-1]), (None, None, None))
            shapes = [{"shape": f"{name} T={t} N={n} K={k}", "cpu_us": round(ref["points"][(n, k, t)][0], 2),
                       "cpu_tops": round(ref["points"][(n, k, t)][1], 2)}
                      for name, (n, k) in GEMM_SHAPES.items() for t in GEMM_T if (n, k, t) in ref["points"]]
            ref = {"value": None if tops is None else round(tops, 2), "unit": unit, "cores": ref["cores"],
                   "kind": "reference", "shapes": shapes,
                   "sample": f"{ref['command']} ({isa}): median of 3 k_gemm_q8 calls per shape"}
    else:
        metric, unit = GEMV_METRIC[args.workload], "GB/s"
        ref = reference_gemv_baseline(*GEMV_SHAPES[args.workload])
    if "unavailable" in ref:
        print(json.dumps({"impl": "reference", "unavailable": ref["unavailable"]}), flush=True)
        return
    line = {"metric": metric, "impl": "reference", "value": ref["value"], "unit": unit, "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 (W8A8, fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"{args.workload}: the reference's kernel on the host cores", "parallelism": "cpu"},
            "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": ref["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if "shapes" in ref:
        line["shapes"] = ref["shapes"]
    print(json.dumps(line), flush=True)


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.workload in GEMV_SHAPES or args.workload == "gemm":
        run_reference_kernels(args)
        return
    wl = args.workload if args.workload in ARCH else "8b"
    r = reference_engine_sample(wl, steps=args.steps, warmup=args.warmup)
    if "unavailable" in r:
        print(json.dumps({"impl": "reference", "unavailable": r["unavailable"]}), flush=True)
        return
    P, D = REQUEST[wl]
    line = {"metric": METRIC, "impl": "reference", "value": r["value"], "unit": "tok/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 (W8A8, fp32 accumulate)",
            "data": "synthetic: the GPU arm's seeded checkpoint (engine_write_random) and prompt",
            "config": engine_config(wl, P, D, 0),
            "prefill_tok_s": r["prefill_tok_s"], "decode_tok_s": r["value"],
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- config 0 kernel alone (profiling) ----------------------------------------------------------------------------

GEMV_SHAPES = {"gemv": (8192, 2048), "ffn": (14336, 4096)}  # (weight rows, K) of one matrix
GEMV_METRIC = {"gemv": "config 0 GEMV HBM GB/s", "ffn": "8B SwiGLU decode GEMV (W1, W3 14336 x 4096) HBM GB/s"}
GEMM_METRIC = "config 1 prefill GEMM int8 TOPS (8B up projection, T=2048)"

def run_gemv(args):
    import torch
    kc = load_package()
    kc.init()
    hbm, peak_kind = peaks()
    rows, cols = GEMV_SHAPES[args.workload]
    alg, us = gemv_roofline(kc, torch, rows, cols, launches=args.steps, swiglu=args.workload == "ffn")
    name = GEMV_METRIC[args.workload]
    gbs = alg / (us / 1e6) / 1e9
    line = {"metric": name, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "kernel_us": round(us, 3),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_source": f"{peak_kind} hbm_gbs"}}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = reference_gemv_baseline(*GEMV_SHAPES[args.workload])
    print(json.dumps(line), flush=True)


# ---- timing of a kernel alone ----------------------------------------------------------------------------------

def timed_graph(torch, launch, warmup, launches):
    """Mean microseconds of `launch(i)`: warm-up calls, then `launches` calls captured in one graph with a pair of CUDA
    events around each, replayed once."""
    for i in range(warmup):
        launch(i)
    evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
           for _ in range(launches)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(launches):
            evs[i][0].record()
            launch(warmup + i)
            evs[i][1].record()
    graph.replay()
    torch.cuda.synchronize()
    del graph
    return float(np.mean([a.elapsed_time(b) for a, b in evs])) * 1e3


# ---- config 1: the prefill GEMM alone ---------------------------------------------------------------------------

GEMM_SHAPES = {"up": (14336, 4096), "down": (4096, 14336)}  # (N weight rows, K)
GEMM_T = (128, 512, 2048)


def gemm_points(kc, torch, g, name, N, K, ts, warmup, launches, int8_tops, hbm, gs=64):
    """k_gemm_q8 (STORE) of an N x K weight at each T in ts, timed with timed_graph over enough weight copies to exceed
    L2 three times. Per T: microseconds, int8 TOPS and the fraction of the binding roof (the int8 tensor peak or HBM
    for the call's bytes, whichever takes longer)."""
    w = torch.randn((N, K), generator=g, device="cuda") * 0.02
    wq, ws = kc.quantize(w, gs)
    del w
    wbytes = wq.numel() + ws.numel() * 4
    copies = max(2, -(-3 * L2_BYTES // wbytes))
    W = [(wq.clone(), ws.clone()) for _ in range(copies)]
    out = []
    for T in ts:
        x = torch.randn((T, K), generator=g, device="cuda")
        xq, xs = kc.quantize(x, gs)
        c = torch.empty((T, N), device="cuda")

        def launch(i):
            kc.k_gemm_q8(xq, xs, T, K, gs, [kc.segment(c, W[i % copies])])

        us = timed_graph(torch, launch, warmup, launches)
        kc.status()
        ops = 2.0 * T * N * K
        nbytes = wbytes + T * K * (1 + 4 / gs) + 4 * T * N
        t_tensor, t_hbm = ops / (int8_tops * 1e12), nbytes / (hbm * 1e9)
        out.append({"shape": f"{name} T={T} N={N} K={K}", "key": (N, K, T), "us": round(us, 2),
                    "int8_tops": round(ops / (us * 1e-6) / 1e12, 1), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                    "bound": "tensor" if t_tensor >= t_hbm else "hbm",
                    "frac": round(max(t_tensor, t_hbm) / (us * 1e-6), 4)})
        del x, xq, xs, c
    del W, wq, ws
    return out


def int8_peak():
    """The int8 tensor roof in TOPS: twice the measured dense bf16 GEMM peak (the dense int8/bf16 ratio), and its
    source."""
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        return 2 * float(json.loads(pk.read_text())["bf16_tflops"]), "2 x measured bf16_tflops"
    return 2 * 1590.0, "2 x fallback bf16_tflops"


def run_gemm(args):
    """Config 1: k_gemm_q8 (STORE) on the 8B up (14336 x 4096) and down (4096 x 14336) projections at T = 128, 512 and
    2048 activation rows, each launch timed with CUDA events inside a captured graph, the weights rotating over enough
    copies to exceed L2 three times. Per shape: int8 TOPS against the binding roof, the int8 tensor peak (taken as
    twice the measured bf16 GEMM peak, the dense int8/bf16 ratio) or HBM for its bytes, whichever takes longer."""
    import torch
    kc = load_package()
    kc.init()
    hbm, peak_kind = peaks()
    int8_tops, int8_source = int8_peak()
    shapes = []
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    for name, (N, K) in GEMM_SHAPES.items():
        shapes += gemm_points(kc, torch, g, name, N, K, GEMM_T, args.warmup, max(4, args.steps), int8_tops, hbm)
    head = next(s for s in shapes if s["key"] == (*GEMM_SHAPES["up"], GEMM_T[-1]))
    line = {"metric": GEMM_METRIC, "value": head["int8_tops"],
            "unit": "TOPS", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "dtype": "int8",
            "peaks": {"int8_tops": int8_tops, "hbm_gbs": hbm,
                      "source": f"{int8_source}; {peak_kind} hbm_gbs"},
            "shapes": shapes}
    if not args.no_cpu_baseline:
        ref = reference_gemm_points(list(GEMM_SHAPES.values()), GEMM_T)
        if "unavailable" in ref:
            line["cpu_baseline"] = ref
        else:
            for sh in shapes:
                n, k, t = sh["key"]
                if (n, k, t) in ref["points"]:
                    sh["cpu_us"], sh["cpu_tops"] = (round(v, 2) for v in ref["points"][(n, k, t)][:2])
            _, tops_, isa = ref["points"].get(head["key"], (None, None, None))
            line["cpu_baseline"] = {"value": None if tops_ is None else round(tops_, 2), "unit": "TOPS",
                                    "cores": ref["cores"], "kind": "reference",
                                    "sample": f"{ref['command']} ({isa}): median of 3 k_gemm_q8 "
                                              "calls per shape; value is up T=2048, per-shape figures in shapes"}
    for sh in shapes:
        del sh["key"]
    print(json.dumps(line), flush=True)


# ---- config 4: the GEMV -> tensor-core GEMM crossover sweep -------------------------------------------------------

# Every 8B projection as (weight rows N, K, split): "rows" shards split the output rows over S ranks (wq, wk/wv, w1/w3,
# the classifier), "cols" shards the input columns (wo, w2), as the reference's shard plan does (src/shards.c:223-248).
SWEEP_PROJECTIONS = {"wq": (4096, 4096, "rows"), "wk/wv": (1024, 4096, "rows"), "wo": (4096, 4096, "cols"),
                     "w1/w3": (14336, 4096, "rows"), "w2": (4096, 14336, "cols"), "cls": (128256, 4096, "rows")}
SWEEP_T = (1, 2, 4, 8, 16, 64, 256, 1024, 4096)


def run_sweep(args):
    """Config 4 on one GPU: each 8B projection's rank-0 shard at S = 1/2/4/8 (rows N/S for row-split weights, columns
    K/S for wo and w2; the all-reduce that joins column shards is not part of this figure) times T activation rows.
    At every T the tensor-core GEMM (k_gemm_q8's Q8_GEMM_GPU_TCGEN05 rung) runs; up to T = --sweep-rows-max the
    one-GEMV-per-row rung (Q8_GEMM_GPU_DP4A, what k_gemm_q8 takes below its row threshold) runs beside it. Weights
    rotate over enough copies to exceed L2 three times and the copy index runs on across launches, so every launch
    reads weights no recent launch touched. The crossover of a shard is the smallest swept T from which the GEMM is
    faster at every larger T where both ran."""
    import torch
    kc = load_package()
    kc.init()
    hbm, peak_kind = peaks()
    int8_tops, int8_source = int8_peak()
    ts = [int(t) for t in args.sweep_t.split(",")] if args.sweep_t else list(SWEEP_T)
    splits = [int(s) for s in args.sweep_s.split(",")]
    gs, points, crossover = 64, [], {}
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    for S in splits:
        for name, (N, K, split) in SWEEP_PROJECTIONS.items():
            n, k = (N // S, K) if split == "rows" else (N, K // S)
            w = torch.randn((n, k), generator=g, device="cuda") * 0.02
            wq, ws = kc.quantize(w, gs)
            del w
            wbytes = wq.numel() + ws.numel() * 4
            copies = max(2, -(-3 * L2_BYTES // wbytes))
            W = [(wq.clone(), ws.clone()) for _ in range(copies)]
            del wq, ws
            ctr = [0]
            wins = {}
            for T in ts:
                x = torch.randn((T, k), generator=g, device="cuda")
                xq, xs = kc.quantize(x, gs)
                del x
                c = torch.empty((T, n), device="cuda")

                def launch(backend):
                    def f(_i):
                        wq_, ws_ = W[ctr[0] % copies]
                        ctr[0] += 1
                        if not kc.k_gemm_q8_backend_test(backend, xq, xs, T, k, gs, [kc.segment(c, (wq_, ws_))]):
                            raise kc.KernelError(f"backend {backend} is not compiled in")
                    return f

                tc_us = timed_graph(torch, launch(kc.Q8_GEMM_GPU_TCGEN05), args.warmup, args.steps)
                kc.status()
                rows_us = None
                if T <= args.sweep_rows_max:
                    rows_us = timed_graph(torch, launch(kc.Q8_GEMM_GPU_DP4A), args.warmup, args.steps)
                    kc.status()
                    wins[T] = tc_us <= rows_us
                ops = 2.0 * T * n * k
                nbytes = wbytes + T * k * (1 + 4 / gs) + 4 * T * n
                t_tensor, t_hbm = ops / (int8_tops * 1e12), nbytes / (hbm * 1e9)
                points.append({"proj": name, "S": S, "N": n, "K": k, "T": T, "tc_us": round(tc_us, 2),
                               "rows_us": None if rows_us is None else round(rows_us, 2),
                               "tc_tops": round(ops / (tc_us * 1e-6) / 1e12, 1),
                               "tc_gbs": round(nbytes / (tc_us * 1e-6) / 1e9, 1),
                               "bound": "tensor" if t_tensor >= t_hbm else "hbm",
                               "frac": round(max(t_tensor, t_hbm) / (tc_us * 1e-6), 4)})
                del xq, xs, c
            cross = None
            for T in sorted(wins, reverse=True):
                if not wins[T]:
                    break
                cross = T
            crossover[f"{name} S={S}"] = cross
            del W
            torch.cuda.empty_cache()
    known = [v for v in crossover.values() if v is not None]
    print(json.dumps({"metric": "config 4 GEMV -> tensor-core GEMM crossover (activation rows), per-rank shards",
                      "value": max(known) if known else None, "unit": "rows", "higher_is_better": False,
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "dtype": "int8",
                      "data": "synthetic: seeded N(0,0.02) weights, N(0,1) activations, Q8_0 gs 64",
                      "config": {"workload": "config 4: 8B projections x T x S (rank-0 shard shapes on one GPU)",
                                 "T": ts, "S": splits, "rows_rung_max_T": args.sweep_rows_max,
                                 "l2": "weights rotate over > 3x L2"},
                      "peaks": {"int8_tops": int8_tops, "hbm_gbs": hbm,
                                "source": f"{int8_source}; {peak_kind} hbm_gbs"},
                      "crossover": crossover, "points": points}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["8b", "1b", "gemv", "ffn", "gemm", "sweep"], default="8b")
    ap.add_argument("--sweep-t", default="", help="sweep: comma-separated activation row counts (default: config 4's)")
    ap.add_argument("--sweep-s", default="1,2,4,8", help="sweep: comma-separated tensor-parallel splits")
    ap.add_argument("--sweep-rows-max", type=int, default=16, help="sweep: largest T timed on the per-row GEMV rung")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-request", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("gemv", "ffn"):
        run_gemv(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.profile_request:
        run_profile_request(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
