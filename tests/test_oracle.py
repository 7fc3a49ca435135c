"""CPU tests: the oracle (the C restatement under oracle/) against the reference's golden vectors and, where the
reference was compiled here (oracle/_ref), against the reference itself on fresh seeded inputs."""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = np.load(Path(__file__).parent / "golden" / "q8_golden.npz")


def bits(a):
    return np.ascontiguousarray(a).view(np.int32 if a.dtype == np.float32 else a.dtype)


def test_quantize_known_answer_ties(oracle):
    # tests/kernels.c:111-116: scale exactly 1, roundf's half-away-from-zero ties, an all-zero group.
    x, gs = GOLDEN["quant_ties_x"], int(GOLDEN["quant_ties_gs"])
    q, s = oracle.quantize(x, gs)
    assert (q == GOLDEN["quant_ties_q"]).all()
    assert (bits(s) == bits(GOLDEN["quant_ties_s"])).all()
    assert s[0] == 1.0 and list(q[:8]) == [127, 3, -4, 1, -1, 2, -127, 0]
    assert s[1] == 0.0 and not q[16:32].any()


@pytest.mark.parametrize("n,gs", [(256, 64), (4096, 64), (512, 128), (192, 32), (1792, 64)])
def test_quantize_golden(oracle, n, gs):
    q, s = oracle.quantize(GOLDEN[f"quant_{n}_{gs}_x"], gs)
    assert (q == GOLDEN[f"quant_{n}_{gs}_q"]).all()
    assert (bits(s) == bits(GOLDEN[f"quant_{n}_{gs}_s"])).all()


def test_quantize_rejects_nonfinite(oracle):
    x = np.ones(64, np.float32)
    x[5] = np.inf
    with pytest.raises(ValueError):
        oracle.quantize(x, 64)


@pytest.mark.parametrize("d,n", [(37, 1024), (16, 4096)])
def test_gemv_scalar_golden(oracle, d, n):
    k = f"gemv_{d}_{n}"
    y = oracle.gemv_scalar(GOLDEN[k + "_xq"], GOLDEN[k + "_xs"], GOLDEN[k + "_wq"], GOLDEN[k + "_ws"], 64)
    assert (bits(y) == bits(GOLDEN[k + "_y"])).all()


GEMV512_CASES = [(37, 1024, 64), (16, 4096, 64), (9, 512, 128), (5, 768, 256), (8, 14336, 64)]


@pytest.mark.parametrize("d,n,gs", GEMV512_CASES)
def test_gemv_reference_order_golden(oracle, d, n, gs):
    """The decode GEMV the GPU reproduces: the reference's k_matmul_q8 on its AVX-512 ISA (dots_q8_body's 16 lanes and
    _mm512_reduce_add_ps), bitwise; ADD adds that product to the output in one rounding."""
    k = f"gemv512_{d}_{n}_{gs}"
    xq, xs, wq, ws = (GOLDEN[k + t] for t in ("_xq", "_xs", "_wq", "_ws"))
    y = oracle.gemv(xq, xs, wq, ws, gs)
    assert (bits(y) == bits(GOLDEN[k + "_y"])).all()
    base = np.linspace(-1, 1, d).astype(np.float32)
    assert (bits(oracle.gemv(xq, xs, wq, ws, gs, kind=oracle.ADD, out=base)) == bits(base + GOLDEN[k + "_y"])).all()


AMX_CASES = [(1, 40, 512), (7, 48, 1024), (33, 32, 256)]


W8A32_CASES = [(37, 1024, 64), (16, 512, 32), (20, 256, 16), (9, 384, 128), (8, 96, 48), (6, 40, 2)]


@pytest.mark.parametrize("d,n,gs", W8A32_CASES)
def test_gemv_f32_golden(oracle, d, n, gs):
    """W8A32: the reference's k_matmul_q8 on fp32 activations (its AVX-512 lane order for gs % 16 == 0, its portable
    loop for gs 2), bitwise."""
    k = f"gemvf_{d}_{n}_{gs}"
    y = oracle.gemv_f32(GOLDEN[k + "_x"], GOLDEN[k + "_wq"], GOLDEN[k + "_ws"], gs)
    assert (bits(y) == bits(GOLDEN[k + "_y"])).all()


@pytest.mark.parametrize("m,d,k", AMX_CASES)
def test_gemm_amx_order_golden(oracle, m, d, k):
    key = f"amx_{m}_{d}_{k}"
    if key + "_c" not in GOLDEN:
        pytest.skip("golden file was made on a CPU without AMX")
    c = oracle.gemm(GOLDEN[key + "_xq"], GOLDEN[key + "_xs"], GOLDEN[key + "_wq"], GOLDEN[key + "_ws"], 64)
    assert (bits(c) == bits(GOLDEN[key + "_c"])).all()
    dots = oracle.group_dots(GOLDEN[key + "_xq"], GOLDEN[key + "_wq"], 64)
    assert (dots == GOLDEN[key + "_dots"]).all()


@pytest.mark.parametrize("n", [17, 64, 2048, 4099])
def test_rmsnorm_golden(oracle, n):
    x, w = GOLDEN[f"rms_{n}_x"], GOLDEN[f"rms_{n}_w"]
    assert (bits(oracle.rmsnorm(x, w, 1e-5)) == bits(GOLDEN[f"rms_{n}_avx512"])).all()
    assert (bits(oracle.rmsnorm(x, w, 1e-5, order="scalar")) == bits(GOLDEN[f"rms_{n}_scalar"])).all()


def test_gemv_orders_agree_within_reference_budget(oracle):
    # tests/kernels.c:138-170: |y - exact| <= 2e-5 * sum|w.x| + 1e-6 for every Q8 kernel; the scalar order, the AMX
    # order (the GPU's GEMM) and the AVX-512 order (the GPU's GEMV) are three such kernels.
    rng = np.random.default_rng(5)
    wq, ws = oracle.seeded_q8_matrix(64, 4096, 64, seed=3)
    xq, xs = oracle.quantize(rng.standard_normal(4096).astype(np.float32), 64)
    a = oracle.gemv_scalar(xq, xs, wq, ws, 64)
    b = oracle.gemm(xq, xs, wq, ws, 64)[0]
    dots = oracle.group_dots(xq, wq, 64)[:, 0, :].astype(np.float64)
    sa = np.abs(oracle.group_dots(np.abs(xq).astype(np.int8), np.abs(wq).astype(np.int8), 64)[:, 0, :])
    exact = (dots * ws.T.astype(np.float64) * xs[:, None]).sum(0)
    mag = (sa * ws.T.astype(np.float64) * xs[:, None]).sum(0)
    assert np.all(np.abs(a - exact) <= 2e-5 * mag + 1e-6)
    assert np.all(np.abs(b - exact) <= 2e-5 * mag + 1e-6)
    assert np.all(np.abs(oracle.gemv(xq, xs, wq, ws, 64) - exact) <= 2e-5 * mag + 1e-6)


needs_ref = pytest.mark.skipif(not Path(__file__).resolve().parents[1].joinpath("oracle/_ref/libllama_ref.so").exists(),
                               reason="the reference was not compiled here")


@needs_ref
@pytest.mark.parametrize("seed", [1, 2])
def test_oracle_matches_compiled_reference(oracle, seed):
    rng = np.random.default_rng(seed)
    for n, gs in [(4096, 64), (14336, 64), (64, 16)]:
        x = rng.standard_normal(n).astype(np.float32)
        q0, s0 = oracle.quantize(x, gs)
        q1, s1 = oracle.ref_quantize(x, gs, oracle.KERNELS_SCALAR)
        assert (q0 == q1).all() and (bits(s0) == bits(s1)).all()
    wq, ws = oracle.seeded_q8_matrix(24, 2048, 64, seed=seed)
    xq, xs = oracle.quantize(rng.standard_normal(2048).astype(np.float32), 64)
    assert (bits(oracle.gemv_scalar(xq, xs, wq, ws, 64)) == bits(oracle.ref_gemv(xq, xs, wq, ws, 64))).all()
    for gs in (64, 128, 32):  # the AVX-512 body for gs % 64 == 0, the portable loop below
        wq3, ws3 = oracle.seeded_q8_matrix(19, 1024, gs, seed=seed + gs)
        xq3, xs3 = oracle.quantize(rng.standard_normal(1024).astype(np.float32), gs)
        ref = oracle.ref_gemv(xq3, xs3, wq3, ws3, gs, oracle.KERNELS_AVX512)
        oracle.ref_select(oracle.KERNELS_SCALAR)
        assert (bits(oracle.gemv(xq3, xs3, wq3, ws3, gs)) == bits(ref)).all()
    if oracle.ref_amx_unavailable() is None:
        xq2, xs2 = oracle.quantize(rng.standard_normal((5, 2048)).astype(np.float32), 64)
        assert (bits(oracle.gemm(xq2, xs2, wq, ws, 64)) == bits(oracle.ref_gemm_amx(xq2, xs2, wq, ws, 64))).all()
