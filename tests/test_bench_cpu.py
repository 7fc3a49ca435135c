"""Host logic of bench.py, on the CPU with a fake kernel library and a fake timer.
- The configuration-4 sweep: the rank-0 shard shapes of every 8B projection at each split (row-split weights keep K
  and divide N, wo and w2 keep N and divide K, as the reference's shard plan does, src/shards.c:223-248), the
  activation rows of each launch, which rung runs at which T, and the crossover rule (the smallest swept T from which
  the GEMM wins at every larger swept T).
- The CPU baselines of the kernel workloads: the reference's own gemm-bench (tests/gemm_bench.c) lines, parsed and
  merged into the configuration-0/1 lines and the reference arm's line."""
import argparse
import importlib.util
import json
import types
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture
def bench(monkeypatch):
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    class Generator:
        def __init__(self, device=None):
            pass

        def manual_seed(self, _):
            return self

    empty, zeros = torch.empty, torch.zeros
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(torch, "Generator", Generator)
    monkeypatch.setattr(torch, "randn", lambda shape, generator=None, device=None: zeros(shape))
    monkeypatch.setattr(torch, "empty", lambda shape, device=None, dtype=None: empty(shape, dtype=dtype or torch.float32))
    mod.L2_BYTES = 1 << 16  # a few weight copies on the CPU
    mod.SWEEP_PROJECTIONS = {k: (n // 64, kk // 64, split) for k, (n, kk, split) in mod.SWEEP_PROJECTIONS.items()}
    return mod


def fake_library(calls):
    """Stand-in for the kernel library that checks and records every launch: (rung, rows, weight rows, K)."""
    kc = types.SimpleNamespace(Q8_GEMM_GPU_DP4A=16, Q8_GEMM_GPU_TCGEN05=17, KernelError=RuntimeError)
    kc.init = kc.status = lambda: None
    kc.quantize = lambda x, gs: (torch.zeros(x.shape, dtype=torch.int8), torch.zeros(x.shape[:-1] + (x.shape[-1] // gs,)))
    kc.segment = lambda c, w: (c, w)

    def backend_test(backend, xq, xs, m, k, gs, segs):
        c, (wq, ws) = segs[0]
        assert xq.shape == (m, k) and xs.shape == (m, k // gs) and c.shape == (m, wq.shape[0])
        assert wq.shape[1] == k and ws.shape == (wq.shape[0], k // gs)
        calls.append((backend, m, wq.shape[0], k))
        return 1

    kc.k_gemm_q8_backend_test = backend_test
    kc.k_gemm_q8 = lambda xq, xs, m, k, gs, segs: backend_test(0, xq, xs, m, k, gs, segs)
    return kc


def run(bench, monkeypatch, capsys, gemm_us, row_us, **kw):
    calls = []
    kc = fake_library(calls)
    monkeypatch.setattr(bench, "load_package", lambda: kc)
    # The timing helper runs the launches and reports gemm_us(T) for the tensor-core rung, T * row_us per-row.
    def timed(torch_, launch, warmup, launches):
        n0 = len(calls)
        for i in range(warmup + launches):
            launch(i)
        assert len(calls) == n0 + warmup + launches
        backend, m = calls[-1][0], calls[-1][1]
        return gemm_us(m) if backend == kc.Q8_GEMM_GPU_TCGEN05 else m * row_us

    monkeypatch.setattr(bench, "timed_graph", timed)
    args = argparse.Namespace(steps=2, warmup=3, sweep_t=kw.get("t", ""), sweep_s=kw.get("s", "1,2,4,8"),
                              sweep_rows_max=kw.get("rows_max", 16))
    bench.run_sweep(args)
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1]), calls


def test_sweep_shard_shapes_and_rungs(bench, monkeypatch, capsys):
    line, calls = run(bench, monkeypatch, capsys, gemm_us=lambda t: 40.0, row_us=10.0)
    assert line["config"]["T"] == [1, 2, 4, 8, 16, 64, 256, 1024, 4096]
    points = line["points"]
    assert len(points) == 4 * 6 * 9
    for p in points:
        n, k, split = bench.SWEEP_PROJECTIONS[p["proj"]]
        assert (p["N"], p["K"]) == ((n // p["S"], k) if split == "rows" else (n, k // p["S"]))
        assert (p["rows_us"] is None) == (p["T"] > 16)
    # Each shard and T: warm-up + timed launches of the GEMM, and of the row rung up to T = 16.
    gemm = [c for c in calls if c[0] == 17]
    rows = [c for c in calls if c[0] == 16]
    assert len(gemm) == 4 * 6 * 9 * 5 and len(rows) == 4 * 6 * 5 * 5


def test_sweep_crossover_rule(bench, monkeypatch, capsys):
    # The GEMM costs 40 us at every T, a row 10 us: rows win below T = 4; the tie at T = 4 goes to the GEMM.
    line, _ = run(bench, monkeypatch, capsys, gemm_us=lambda t: 40.0, row_us=10.0, s="1")
    assert set(line["crossover"].values()) == {4}
    assert line["value"] == 4
    # The GEMM never wins within the swept row range: no crossover is reported.
    line, _ = run(bench, monkeypatch, capsys, gemm_us=lambda t: 1e6, row_us=10.0, s="2")
    assert set(line["crossover"].values()) == {None}
    assert line["value"] is None


def gemm_bench_lines(shapes, ts, isa="amx"):
    """gemm-bench's JSON lines for k_gemm_q8 (the fields bench.py reads), with made-up but distinct timings."""
    return [{"kernel": "gemm_q8", "isa": isa, "n": n, "k": k, "m": t, "reps": 3, "median_s": 1e-3 * (i + 1),
             "gflops_median": 100.0 * (i + 1)} for i, ((n, k), t) in enumerate((s, t) for s in shapes for t in ts)]


def test_gemm_line_carries_the_reference_per_shape(bench, monkeypatch, capsys):
    calls = []
    kc = fake_library(calls)
    monkeypatch.setattr(bench, "load_package", lambda: kc)
    monkeypatch.setattr(bench, "timed_graph", lambda torch_, launch, warmup, launches: (
        [launch(i) for i in range(warmup + launches)], 50.0)[1])
    monkeypatch.setattr(bench, "GEMM_SHAPES", {"up": (256, 512), "down": (128, 768)})
    monkeypatch.setattr(bench, "GEMM_T", (8, 32))
    asked = []

    def fake_bench(args, reps, kernels="auto"):
        asked.append(kernels)
        if kernels == "amx":  # a host without AMX: the reference arm falls back to its auto selection
            return {"unavailable": "no AMX"}
        return {"cores": 4, "command": "gemm-bench ...", "lines": gemm_bench_lines([(256, 512), (128, 768)], (8, 32),
                                                                                    isa="avx512")}

    monkeypatch.setattr(bench, "reference_kernel_bench", fake_bench)
    bench.run_gemm(argparse.Namespace(steps=2, warmup=3, no_cpu_baseline=False))
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert asked == ["amx", "auto"]
    assert [s["shape"] for s in line["shapes"]] == ["up T=8 N=256 K=512", "up T=32 N=256 K=512",
                                                   "down T=8 N=128 K=768", "down T=32 N=128 K=768"]
    assert [s["cpu_us"] for s in line["shapes"]] == [1000.0, 2000.0, 3000.0, 4000.0]
    assert all("key" not in s for s in line["shapes"])
    assert line["cpu_baseline"]["value"] == 0.2 and line["cpu_baseline"]["kind"] == "reference"
    assert line["cpu_baseline"]["cores"] == 4 and "avx512" in line["cpu_baseline"]["sample"]
    # Every shape and T: 3 warm-up launches and at least 4 timed ones.
    assert {c[1] for c in calls} == {8, 32} and len(calls) == 2 * 2 * (3 + 4)


def test_reference_arm_for_the_kernel_workloads(bench, monkeypatch, capsys):
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setattr(bench, "reference_kernel_bench", lambda args, reps, kernels="auto": {
        "cores": 16, "command": f"LLAMA_KERNELS={kernels} gemm-bench",
        "lines": gemm_bench_lines(list(bench.GEMM_SHAPES.values()), bench.GEMM_T) + [
            {"kernel": "gemv_rows_q8", "isa": "avx512", "reps": 20, "median_s": 2.5e-4, "weight_gbs_median": 70.5}]})
    bench.run_reference(argparse.Namespace(workload="gemv", steps=5, warmup=3))
    line = json.loads(capsys.readouterr().out)
    assert line["impl"] == "reference" and line["metric"] == bench.GEMV_METRIC["gemv"]
    assert line["value"] == 70.5 and line["unit"] == "GB/s" and line["cpu_baseline"]["cores"] == 16
    assert line["e2e"] == {"value": 70.5, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    bench.run_reference(argparse.Namespace(workload="gemm", steps=5, warmup=3))
    line = json.loads(capsys.readouterr().out)
    assert line["metric"] == bench.GEMM_METRIC and line["unit"] == "TOPS"
    assert line["value"] == 0.3  # up (the first shape) at the last T: the third line of the fake output
    assert "LLAMA_KERNELS=amx" in line["cpu_baseline"]["sample"] and len(line["shapes"]) == 6


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "gemm-bench").exists(), reason="the reference was not compiled here")
def test_reference_gemm_bench_output_parses(bench):
    # The real tool on small shapes: the fields bench.py reads are there and the figures are positive.
    g = bench.reference_gemv_baseline(256, 512)
    assert g["kind"] == "reference" and g["value"] > 0 and g["cores"] >= 1
    pts = bench.reference_gemm_points([(256, 512)], (8, 32))
    assert set(pts["points"]) == {(256, 512, 8), (256, 512, 32)}
    assert all(us > 0 and tops > 0 for us, tops, _ in pts["points"].values())


def test_reference_split_drift_from_the_golden_runs(bench):
    """The reference's own two-socket run against its one-socket run on the benchmark request (the committed golden
    file): its first logits move by 6.3% of the largest and its tokens part at step 5, at a 1.8e-3 margin. The bench
    reports this beside its 4- and 8-GPU parity, which can only be compared with the one-socket run."""
    import numpy as np
    g = np.load(Path(__file__).parent / "golden" / "bench_golden.npz")
    d = bench.reference_split_drift(g, "8b")
    assert d["first_divergence_step"] == 5
    assert 0.06 < d["first_logits_max_rel_diff"] < 0.07
    assert d["ref_margin_at_divergence"] < 2e-3
    assert bench.reference_split_drift(g, "1b") is None  # no two-socket run of the 1B request
