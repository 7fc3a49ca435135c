"""k_gemm_q8_noalloc (the GEMM entry point that allocates no device memory) against k_gemm_q8, through the C-ABI.

Tolerance: none — both entry points run the same kernels on the same operands, so the outputs must agree bit for
bit. Two calls in a row with different shapes check that nothing left in the fixed scale array leaks into the next
call. This file is named to be collected last so that it also runs after every other GPU test in one process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_both(kc, oracle, m, n, k, seed, kind=None):
    gs = 64
    rng = np.random.default_rng(seed)
    wq, ws = oracle.seeded_q8_matrix(n, k, gs, seed)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), gs)
    xq_d, xs_d, wq_d, ws_d = dev(xq), dev(xs), dev(wq), dev(ws)
    base = rng.standard_normal((m, n)).astype(np.float32)
    kind = kc.GEMM_STORE if kind is None else kind
    c_ref, c_new = dev(base), dev(base)
    kc.k_gemm_q8(xq_d, xs_d, m, k, gs, [kc.segment(c_ref, (wq_d, ws_d), kind)])
    kc.k_gemm_q8_noalloc(xq_d, xs_d, m, k, gs, [kc.segment(c_new, (wq_d, ws_d), kind)])
    kc.status()
    return c_ref.cpu().numpy(), c_new.cpu().numpy()


def test_noalloc_matches_k_gemm_q8_two_calls_in_a_row(kc, oracle):
    a_ref, a_new = run_both(kc, oracle, 200, 300, 1024, 1)
    b_ref, b_new = run_both(kc, oracle, 33, 128, 4096, 2, kind=kc.GEMM_ADD)
    assert (a_ref.view(np.int32) == a_new.view(np.int32)).all()
    assert (b_ref.view(np.int32) == b_new.view(np.int32)).all()


def test_noalloc_small_batch_takes_the_row_path(kc, oracle):
    ref, new = run_both(kc, oracle, 3, 96, 512, 3)
    assert (ref.view(np.int32) == new.view(np.int32)).all()


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
