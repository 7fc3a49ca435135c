"""Host side of tensor parallelism on CPU, as two gloo ranks: they agree on the NCCL id that joins the engine's ranks
(share_comm_id, the rendezvous bench.py uses under torchrun), and bench.py's timing takes the maximum over ranks behind
a barrier. No GPU and no collective of the engine is involved."""
import multiprocessing as mp
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from conftest import load_engine
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out.put((rank, load_engine().share_comm_id(rank, world)))
    finally:
        dist.destroy_process_group()


def test_ranks_share_one_nccl_id():
    pytest.importorskip("torch")
    ctx = mp.get_context("spawn")
    out, port = ctx.Queue(), _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(out.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert len(got[0]) == 128 and got[0] == got[1]


def _bench_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import importlib.util
    from pathlib import Path
    import torch.distributed as dist
    spec = importlib.util.spec_from_file_location("bench_rank", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.barrier(world)
        # Each rank's own time; every rank must report the slowest (a step is as slow as its slowest rank).
        out.put((rank, bench.max_over_ranks(world, 10.0 + 5.0 * rank), bench.max_over_ranks(world, -1.0 - rank)))
        bench.barrier(world)
    finally:
        dist.destroy_process_group()


def test_bench_takes_the_max_over_ranks():
    pytest.importorskip("torch")
    ctx = mp.get_context("spawn")
    out, port = ctx.Queue(), _free_port()
    procs = [ctx.Process(target=_bench_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = {r: (a, b) for r, a, b in (out.get(timeout=120) for _ in procs)}
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == {0: (15.0, -1.0), 1: (15.0, -1.0)}


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    # Under torchrun the reference's CPU engine runs once, on rank 0; the other ranks exit without work or output.
    import argparse
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench_ref_arm", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    ran = []
    monkeypatch.setattr(bench, "reference_engine_sample", lambda *a, **k: ran.append(1) or {"unavailable": "test"})
    args = argparse.Namespace(workload="8b", steps=1, warmup=3)
    monkeypatch.setenv("RANK", "1")
    bench.run_reference(args)
    assert not ran and capsys.readouterr().out == ""
    monkeypatch.setenv("RANK", "0")
    bench.run_reference(args)
    assert ran and '"unavailable": "test"' in capsys.readouterr().out
