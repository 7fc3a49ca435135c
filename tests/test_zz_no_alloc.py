"""k_gemm_q8_noalloc (the GEMM entry point that allocates no device memory) through the C-ABI.

Bars (no tolerance anywhere):
  - bitwise k_gemm_q8 on the same operands (the same kernels run), and bitwise the oracle: the AMX-INT8 order
    (oracle.gemm, src/gemm.c:554-610) on the tensor-core rung, the AVX-512 GEMV order per row (oracle.gemv,
    src/gemv.c:109-139) on the row rung;
  - two calls in a row with different shapes: nothing left in the fixed scale array leaks into the next call;
  - no allocation: the device's free memory (cudaMemGetInfo) is unchanged across a call whose scale array fills the
    whole fixed array, a size no earlier k_gemm_q8 call of the suite grew its scratch to;
  - the size limit is enforced with the documented message.
This file is named to be collected last so that it also runs after every other GPU test in one process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def operands(oracle, m, n, k, gs, seed):
    rng = np.random.default_rng(seed)
    wq, ws = oracle.seeded_q8_matrix(n, k, gs, seed)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), gs)
    base = rng.standard_normal((m, n)).astype(np.float32)
    return xq, xs, wq, ws, base


def run_both(kc, oracle, m, n, k, seed, kind=None, gs=64):
    xq, xs, wq, ws, base = operands(oracle, m, n, k, gs, seed)
    xq_d, xs_d, wq_d, ws_d = dev(xq), dev(xs), dev(wq), dev(ws)
    kind = kc.GEMM_STORE if kind is None else kind
    c_ref, c_new = dev(base), dev(base)
    kc.k_gemm_q8(xq_d, xs_d, m, k, gs, [kc.segment(c_ref, (wq_d, ws_d), kind)])
    kc.k_gemm_q8_noalloc(xq_d, xs_d, m, k, gs, [kc.segment(c_new, (wq_d, ws_d), kind)])
    kc.status()
    okind = oracle.ADD if kind == kc.GEMM_ADD else oracle.STORE
    return c_ref.cpu().numpy(), c_new.cpu().numpy(), (xq, xs, wq, ws, base, okind)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.int32)


def test_noalloc_matches_k_gemm_q8_and_the_oracle_two_calls_in_a_row(kc, oracle):
    a_ref, a_new, (xq, xs, wq, ws, base, kind) = run_both(kc, oracle, 200, 300, 1024, 1)
    assert (bits(a_ref) == bits(a_new)).all()
    assert (bits(a_new) == bits(oracle.gemm(xq, xs, wq, ws, 64, kind=kind, c=base))).all()
    b_ref, b_new, (xq, xs, wq, ws, base, kind) = run_both(kc, oracle, 33, 128, 4096, 2, kind=kc.GEMM_ADD)
    assert (bits(b_ref) == bits(b_new)).all()
    assert (bits(b_new) == bits(oracle.gemm(xq, xs, wq, ws, 64, kind=kind, c=base))).all()


def test_noalloc_row_rung_matches_the_oracle(kc, oracle):
    # K = 320 is not a multiple of 256, so both entry points take the per-row GEMV rung (no scratch at all).
    m, n, k = 3, 96, 320
    ref, new, (xq, xs, wq, ws, base, kind) = run_both(kc, oracle, m, n, k, 3)
    assert (bits(ref) == bits(new)).all()
    want = np.stack([oracle.gemv(xq[r], xs[r], wq, ws, 64) for r in range(m)])
    assert (bits(new) == bits(want)).all()


def test_noalloc_allocates_nothing(kc, oracle):
    # (16384 / 64) * 4096 = 2^20 scale floats: the whole fixed array, and a 4 MiB scratch k_gemm_q8 would have to grow.
    m, n, k, gs = 4096, 128, 16384, 64
    xq, xs, wq, ws, base = operands(oracle, m, n, k, gs, 4)
    xq_d, xs_d, wq_d, ws_d = dev(xq), dev(xs), dev(wq), dev(ws)
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    # A first small call loads the kernels (lazy module loading may take device memory once).
    small = torch.zeros((8, n), dtype=torch.float32, device="cuda")
    kc.k_gemm_q8_noalloc(xq_d[:8], xs_d[:8], 8, k, gs, [kc.segment(small, (wq_d, ws_d))])
    kc.status()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    kc.k_gemm_q8_noalloc(xq_d, xs_d, m, k, gs, [kc.segment(c, (wq_d, ws_d))])
    kc.status()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    rows = np.random.default_rng(5).choice(m, 24, replace=False)
    rows.sort()
    got = c.cpu().numpy()[rows]
    assert (bits(got) == bits(oracle.gemm(xq[rows], xs[rows], wq, ws, gs))).all()


def test_noalloc_rejects_shapes_beyond_the_fixed_array(kc, oracle):
    # (16384 / 64) * 4100 scale floats is above the 2^20 the array holds; real buffers of that size are passed so
    # the call could not read out of bounds even if the check were missing.
    m, n, k, gs = 4100, 128, 16384, 64
    xq = torch.zeros((m, k), dtype=torch.int8, device="cuda")
    xs = torch.ones((m, k // gs), dtype=torch.float32, device="cuda")
    wq = torch.zeros((n, k), dtype=torch.int8, device="cuda")
    ws = torch.ones((n, k // gs), dtype=torch.float32, device="cuda")
    c = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    with pytest.raises(kc.KernelError, match="above the fixed"):
        kc.k_gemm_q8_noalloc(xq, xs, m, k, gs, [kc.segment(c, (wq, ws))])
    kc.status()
