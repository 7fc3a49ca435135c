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


# kd_peer_matmul_q8_add cases, one call each, in this order: (rows d, inputs n). They cover a partial last 1024-column
# chunk (3584), fewer rows than CTAs (100: idle CTAs still count the call) and a peer all-reduce between two reducing
# calls (call 2), so consecutive calls use different row partitions and both slot regions.
GEMV_CASES = [(4096, 1024), (4096, 3584), (1000, 512), (100, 256), (4096, 2048)]


def gemv_inputs(oracle, call, rank, d, n, gs=64):
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, 100 * call + rank)
    xq, xs = oracle.quantize(np.random.default_rng(10 * call + rank).standard_normal(n).astype(np.float32), gs)
    x0 = np.random.default_rng(call).standard_normal(d).astype(np.float32)
    return x0, xq, xs, wq, ws


def gemv_expected(oracle, world, call, d, n):
    """x0 + (((p_0 + p_1) + ...) in float32, p_r = rank r's product in the reference's GEMV order; call 2 adds the standalone
    all-reduce of the result (every rank contributes its x, which all ranks hold equal)."""
    x0 = gemv_inputs(oracle, call, 0, d, n)[0]
    s = None
    for r in range(world):
        _, xq, xs, wq, ws = gemv_inputs(oracle, call, r, d, n)
        part = oracle.gemv(xq, xs, wq, ws, 64)
        s = part if s is None else (s + part).astype(np.float32)
    want = (x0 + s).astype(np.float32)
    if call == 2:
        acc = want.copy()
        for _ in range(1, world):
            acc = (acc + want).astype(np.float32)
        want = (want + acc).astype(np.float32)
    return want


def _gemv_rank(rank, world, nccl_id, out):
    try:
        import ctypes
        from conftest import load_engine
        from oracle import oracle as O
        eng = load_engine()
        lib = eng.load_library()
        torch.cuda.set_device(rank)
        lib.kd_set_device(rank)
        kc = eng._kc()
        kc._lib.kc_set_fail_mode(1)
        kc._lib.kernels_init()
        comm = lib.kd_comm_init(rank, world, nccl_id)
        assert comm, "kd_comm_init failed"
        peer = lib.kd_peer_init(comm, rank, world, DIM)
        assert peer, "kd_peer_init failed"
        results = []
        for call, (d, n) in enumerate(GEMV_CASES):
            dev = [torch.from_numpy(v).cuda() for v in gemv_inputs(O, call, rank, d, n)]
            torch.cuda.synchronize()
            p = [ctypes.c_void_p(t.data_ptr()) for t in dev]
            assert lib.kd_peer_matmul_q8_add(peer, p[0], p[1], p[2], p[3], p[4], n, n, d, 64) == 0
            if call == 2:  # the residual reduced once more by the standalone kernel: x += sum of x over ranks
                part = dev[0].clone()
                assert lib.kd_peer_allreduce_add(peer, p[0], ctypes.c_void_p(part.data_ptr()), d) == 0
            lib.kd_sync()
            results.append(dev[0].cpu().numpy())
        eng._check()
        lib.kd_peer_free(peer)
        lib.kd_comm_free(comm)
        out.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        out.put((rank, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_reducing_gemv_bitwise(world, oracle):
    """Rank r holds column slice r of the weights and of the activations; after each call every rank's x equals
    x0 + (((p_0 + p_1) + p_2) + ...) with p_r rank r's product in the reference's GEMV order (the oracle), bit for bit."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from conftest import load_engine
    nccl_id = load_engine().comm_unique_id()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_gemv_rank, args=(r, world, nccl_id, out)) for r in range(world)]
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
    for call, (d, n) in enumerate(GEMV_CASES):
        want = gemv_expected(oracle, world, call, d, n)
        for rank in range(world):
            assert (results[rank][call].view(np.int32) == want.view(np.int32)).all(), (rank, call)


def test_peer_single_rank_reducing_gemv(kc, oracle):
    """One rank (no communicator, no IPC): the same call sequence on one GPU, where every slot is this GPU's own, so
    x + (0 + p) must equal the oracle's x + p bitwise. Covers the slot indexing, both parities, the call counters
    with row partitions that change between calls and idle CTAs, without a second GPU."""
    import ctypes
    from conftest import load_engine
    eng = load_engine()
    lib = eng.load_library()
    peer = lib.kd_peer_init(None, 0, 1, DIM)
    assert peer, "kd_peer_init failed"
    try:
        for call, (d, n) in enumerate(GEMV_CASES):
            dev = [torch.from_numpy(v).cuda() for v in gemv_inputs(oracle, call, 0, d, n)]
            torch.cuda.synchronize()
            p = [ctypes.c_void_p(t.data_ptr()) for t in dev]
            assert lib.kd_peer_matmul_q8_add(peer, p[0], p[1], p[2], p[3], p[4], n, n, d, 64) == 0
            if call == 2:
                part = dev[0].clone()
                assert lib.kd_peer_allreduce_add(peer, p[0], ctypes.c_void_p(part.data_ptr()), d) == 0
            got = dev[0].cpu().numpy()
            kc.status()
            want = gemv_expected(oracle, 1, call, d, n)
            assert (got.view(np.int32) == want.view(np.int32)).all(), call
    finally:
        lib.kd_peer_free(peer)


def test_peer_absent_rank_times_out(kc, oracle):
    """A rank that never arrives (kd_peer_test_absent: rank 0 of 2, the other rank's slots never written), the GPU form
    of the reference's exchange-fail tests: the reducing GEMV and the standalone all-reduce each give up after the
    2 s device wait limit, kc_status reports the timeout, x keeps its value, and the context stays usable."""
    import ctypes
    import time
    from conftest import load_engine
    lib = load_engine().load_library()
    kc.status()
    d, n = 256, 256
    dev = [torch.from_numpy(v).cuda() for v in gemv_inputs(oracle, 0, 0, d, n)]
    x0 = dev[0].cpu().numpy()
    part = torch.ones(d, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    p = [ctypes.c_void_p(t.data_ptr()) for t in dev]
    peer = lib.kd_peer_test_absent(2, DIM)
    assert peer, "kd_peer_test_absent failed"
    try:
        start = time.monotonic()
        assert lib.kd_peer_matmul_q8_add(peer, p[0], p[1], p[2], p[3], p[4], n, n, d, 64) == 0
        with pytest.raises(kc.KernelError, match="timed out"):
            kc.status()
        assert lib.kd_peer_allreduce_add(peer, p[0], ctypes.c_void_p(part.data_ptr()), d) == 0
        with pytest.raises(kc.KernelError, match="timed out"):
            kc.status()
        assert time.monotonic() - start < 30
        assert (dev[0].cpu().numpy().view(np.int32) == x0.view(np.int32)).all()
    finally:
        lib.kd_peer_free(peer)
    # The same context runs the next reduction normally.
    one = lib.kd_peer_init(None, 0, 1, DIM)
    assert one, "kd_peer_init failed"
    try:
        assert lib.kd_peer_matmul_q8_add(one, p[0], p[1], p[2], p[3], p[4], n, n, d, 64) == 0
        got = dev[0].cpu().numpy()
        kc.status()
    finally:
        lib.kd_peer_free(one)
    want = gemv_expected(oracle, 1, 0, d, n)
    assert (got.view(np.int32) == want.view(np.int32)).all()
