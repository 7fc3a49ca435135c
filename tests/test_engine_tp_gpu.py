"""Tensor-parallel engine on 2, 4 and 8 GPUs (one spawned process per GPU, NCCL), against the reference's tokens and
the one-GPU engine. Skipped when the box has fewer GPUs than the case needs.

Bars: the greedy tokens equal the reference's (tests/golden/engine_golden.npz) over the reference's self-consistency
horizon, or part from them first at a near-tie (same_tokens in test_engine_gpu.py); the last-position logits agree with
the one-GPU engine's within 2e-3 of the largest |logit| (the residual sums p0 + p1 + ... of the column shards round
differently from the one-GPU row sums), with the same argmax.
"""
import multiprocessing as mp
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import models  # noqa: E402
from test_engine_gpu import same_tokens  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "engine_golden.npz")


def _rank(rank, world, nccl_id, path, prompt, out, peer=True):
    try:
        import os
        os.environ["LLAMA_PEER_ALLREDUCE"] = "1" if peer else "0"
        os.environ["LLAMA_PEER_GEMV"] = "0" if peer == "kernel" else "1"
        from conftest import load_engine
        eng = load_engine()
        with eng.Engine.load(path, tp=(rank, world, rank, nccl_id)) as m:
            tokens = m.generate(prompt, 64)
            logits = m.forward_batch(prompt, 0, eng.LOGITS_LAST)
        out.put((rank, tokens, logits, None))
    except Exception as e:  # reported to the parent, which fails the test
        out.put((rank, None, None, repr(e)))


def run_ranks(world, path, prompt, peer=True):
    from conftest import load_engine
    nccl_id = load_engine().comm_unique_id()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, nccl_id, str(path), prompt, out, peer)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, tokens, logits, err = out.get(timeout=600)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = (tokens, logits)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return results


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    return models.write_model(tmp_path_factory.mktemp("tp") / "small.bin", "small")


@pytest.mark.parametrize("world,peer", [(2, True), (4, True), (8, True), (2, "kernel"), (2, False)])
def test_tensor_parallel_matches_reference_and_one_gpu(small, world, peer):
    """peer: the decode residual reduced through peer memory (True, the default: inside the Wo / W2 GEMV where the
    shard shapes allow it, which the small model's do at 2 ranks, else kd_peer_allreduce_add), through
    kd_peer_allreduce_add after a PARTIAL GEMV ("kernel", LLAMA_PEER_GEMV=0), or through NCCL (False)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    prompt = GOLDEN["small_prompt"]
    results = run_ranks(world, small, prompt, peer)
    from conftest import load_engine
    eng = load_engine()
    with eng.Engine.load(small) as m:
        one = m.forward_batch(prompt, 0, eng.LOGITS_LAST)
    for rank in range(world):
        tokens, logits = results[rank]
        assert same_tokens("small", tokens), f"rank {rank}"
        assert np.abs(logits - one).max() <= 2e-3 * np.abs(one).max() and logits.argmax() == one.argmax()
        assert (logits.view(np.int32) == results[0][1].view(np.int32)).all(), "ranks disagree"
