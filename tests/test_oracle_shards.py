"""CPU tests: the properties of the Q8 arithmetic that tensor parallelism relies on, on the oracle at 2/4/8-way splits
of the 8B shapes. The reference's tests check them for its two sockets:
- a rank quantizes only its own column slice of an activation, and because the group size divides the slice, that
  equals the slice of the full quantization, bit for bit (tests/kernels.c:517-527);
- the ranks' PARTIAL products of their column slices sum to the full product within the reference's GEMV budget,
  2e-5 * sum|w * x| + 1e-6 per output (tests/kernels.c:528-551);
- a row shard's outputs are the same rows of the full product, bit for bit, because every output is its own chain
  of groups in ascending order (amx_q8_chunk, src/gemm.c:554-610);
- quantizing a batch of rows equals quantizing each row alone (tests/q8.c:185-195)."""
import numpy as np
import pytest

SPLITS = [2, 4, 8]


def bits(a):
    return np.ascontiguousarray(a).view(np.int32)


@pytest.mark.parametrize("S", SPLITS)
@pytest.mark.parametrize("n,gs", [(4096, 64), (14336, 64), (14336, 128), (4096, 16)])
def test_slice_quantization_equals_full(oracle, S, n, gs):
    x = np.random.default_rng(n + S + gs).standard_normal(n).astype(np.float32)
    x[::97] *= 40  # groups with very different maxima
    q, s = oracle.quantize(x, gs)
    w = n // S
    for r in range(S):
        qr, sr = oracle.quantize(x[r * w:(r + 1) * w], gs)
        assert (qr == q[r * w:(r + 1) * w]).all()
        assert (bits(sr) == bits(s[r * w // gs:(r + 1) * w // gs])).all()


@pytest.mark.parametrize("S", SPLITS)
def test_partial_column_slices_sum_to_full_product(oracle, S):
    # Wo at the 8B shape, dim 4096 -> 4096 (sampled rows): each rank's [d][4096/S] slice times its own quantized slice
    # of the activation, summed in rank order as the engine's residual update does.
    d, n, gs = 48, 4096, 64
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, seed=S)
    x = np.random.default_rng(S).standard_normal(n).astype(np.float32)
    xq, xs = oracle.quantize(x, gs)
    groups = n // gs
    dots = xq.reshape(groups, gs).astype(np.int64)[None] * wq.reshape(d, groups, gs).astype(np.int64)
    ref = (dots.sum(-1) * ws.astype(np.float64) * xs.astype(np.float64)[None]).sum(-1)
    mag = (np.abs(dots).sum(-1) * ws.astype(np.float64) * xs.astype(np.float64)[None]).sum(-1)
    w = n // S
    total = np.zeros(d, np.float32)
    for r in range(S):
        qr, sr = oracle.quantize(x[r * w:(r + 1) * w], gs)
        part = oracle.gemm(qr, sr, wq[:, r * w:(r + 1) * w], ws[:, r * w // gs:(r + 1) * w // gs], gs)[0]
        total = (total + part).astype(np.float32)
    assert (np.abs(total.astype(np.float64) - ref) <= 2e-5 * mag + 1e-6).all()
    full = oracle.gemm(xq, xs, wq, ws, gs)[0]
    assert (np.abs(full.astype(np.float64) - ref) <= 2e-5 * mag + 1e-6).all()


@pytest.mark.parametrize("S", SPLITS)
def test_row_shards_are_rows_of_the_full_product(oracle, S):
    # W1 at the 8B shape, 4096 inputs (sampled to 256 rows), three tokens: rank r's rows of the output.
    d, n, gs = 256, 4096, 64
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, seed=10 + S)
    xq, xs = oracle.quantize(np.random.default_rng(S).standard_normal((3, n)).astype(np.float32), gs)
    full = oracle.gemm(xq, xs, wq, ws, gs)
    h = d // S
    for r in range(S):
        part = oracle.gemm(xq, xs, wq[r * h:(r + 1) * h], ws[r * h:(r + 1) * h], gs)
        assert (bits(part) == bits(full[:, r * h:(r + 1) * h])).all()


def test_batched_quantize_equals_per_token(oracle):
    x = np.random.default_rng(7).standard_normal((9, 4096)).astype(np.float32)
    x[4] *= 1e-30  # tiny but nonzero scales
    x[6] = 0  # an all-zero row: scale 0, values 0
    q, s = oracle.quantize(x, 64)
    for t in range(x.shape[0]):
        qt, st = oracle.quantize(x[t], 64)
        assert (qt == q[t]).all() and (bits(st) == bits(s[t])).all()
    assert not q[6].any() and not s[6].any()
