"""Host side of tensor parallelism on CPU: two gloo ranks agree on the NCCL id that joins the engine's ranks
(share_comm_id, the rendezvous bench.py uses under torchrun). No GPU and no collective of the engine is involved."""
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
