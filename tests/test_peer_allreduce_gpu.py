"""The peer-memory all-reduce of the decode residual (kd_peer_allreduce_add) on 2, 4 and 8 GPUs, one spawned process
per GPU, against numpy: x + (((p_0 + p_1) + p_2) + ...) in float32, bitwise, on every rank, for several calls in a
row (both buffer parities, vectors shorter than the buffers). Skipped when the box has fewer GPUs than the case needs.
"""
import multiprocessing as mp

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DIM, CALLS = 4096, 5


def inputs(world, call, n):
    rng = np.random.default_rng(1000 * call + n)
    x = rng.standard_normal(n).astype(np.float32)
    parts = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    return x, parts


def expected(world, call, n):
    x, parts = inputs(world, call, n)
    s = parts[0].copy()
    for r in range(1, world):
        s = (s + parts[r]).astype(np.float32)
    return (x + s).astype(np.float32)


def _rank(rank, world, nccl_id, out):
    try:
        import ctypes
        from conftest import load_engine
        eng = load_engine()
        lib = eng.load_library()
        torch.cuda.set_device(rank)
        lib.kd_set_device(rank)
        kc = eng._kc()
        kc._lib.kc_set_fail_mode(1)  # errors come back to this process instead of exiting it
        kc._lib.kernels_init()
        comm = lib.kd_comm_init(rank, world, nccl_id)
        assert comm, "kd_comm_init failed"
        peer = lib.kd_peer_init(comm, rank, world, DIM)
        assert peer, "kd_peer_init failed"
        results = []
        for call in range(CALLS):
            n = DIM if call % 2 == 0 else DIM - 64 * call
            x, parts = inputs(world, call, n)
            xd = torch.from_numpy(x).cuda()
            pd = torch.from_numpy(parts[rank]).cuda()
            torch.cuda.synchronize()
            assert lib.kd_peer_allreduce_add(peer, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(pd.data_ptr()),
                                             n) == 0
            lib.kd_sync()
            results.append(xd.cpu().numpy())
        eng._check()
        lib.kd_peer_free(peer)
        lib.kd_comm_free(comm)
        out.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        out.put((rank, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_add_bitwise(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from conftest import load_engine
    nccl_id = load_engine().comm_unique_id()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, nccl_id, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, res, err = out.get(timeout=300)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for call in range(CALLS):
        n = DIM if call % 2 == 0 else DIM - 64 * call
        want = expected(world, call, n)
        for rank in range(world):
            assert (results[rank][call].view(np.int32) == want.view(np.int32)).all(), (rank, call)
