"""GPU parity tests of the sm_100a kernels through the C-ABI, against the oracle (and the reference's golden vectors).

Bar (written per test): bit-exact for int8 values, scales, int32 group dots and the fp32 GEMV/GEMM outputs. The decode
GEMV follows the reference's k_matmul_q8 on an AVX-512 host (dots_q8_body's 16-lane order for gs % 64 == 0, the
portable loop otherwise); the tensor-core GEMM follows its AMX-INT8 rescale order. Both stay within the reference's own
budget (2e-5 * sum|w.x| + 1e-6, tests/kernels.c:138-170) of the exact product; SwiGLU within 2 ulp (expf) of the
oracle.
"""
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "q8_golden.npz")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.int32) if a.dtype == np.float32 else a


def ulp_diff(a, b):
    a, b = bits(np.asarray(a, np.float32)).astype(np.int64), bits(np.asarray(b, np.float32)).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


# ---- quantizer ------------------------------------------------------------------------------------------------------

def test_quantize_ties_known_answer(kc):
    x, gs = GOLDEN["quant_ties_x"], int(GOLDEN["quant_ties_gs"])
    q, s = kc.quantize(dev(x), gs)
    kc.status()
    assert (host(q) == GOLDEN["quant_ties_q"]).all()
    assert (bits(host(s)) == bits(GOLDEN["quant_ties_s"])).all()


@pytest.mark.parametrize("n,gs", [(256, 64), (4096, 64), (512, 128), (192, 32), (1792, 64)])
def test_quantize_golden(kc, n, gs):
    q, s = kc.quantize(dev(GOLDEN[f"quant_{n}_{gs}_x"]), gs)
    kc.status()
    assert (host(q) == GOLDEN[f"quant_{n}_{gs}_q"]).all()
    assert (bits(host(s)) == bits(GOLDEN[f"quant_{n}_{gs}_s"])).all()


@pytest.mark.parametrize("m,n,gs,ldx", [(1, 64, 64, 64), (7, 4096, 64, 4100), (128, 14336, 64, 14336),
                                        (3, 96, 16, 96), (2, 2048, 256, 2048)])
def test_quantize_rows_matches_oracle(kc, oracle, m, n, gs, ldx):
    rng = np.random.default_rng(m * n)
    x = (rng.standard_normal((m, ldx)) * rng.uniform(1e-3, 1e3, (m, 1))).astype(np.float32)
    x[:, :gs] = 0.0  # an all-zero group per row: scale 0, values 0
    xt = dev(x)
    q = torch.empty((m, n), dtype=torch.int8, device="cuda")
    s = torch.empty((m, n // gs), dtype=torch.float32, device="cuda")
    kc.k_quantize_rows(q, s, xt, ldx, m, n, gs)
    kc.status()
    oq, os_ = oracle.quantize(x[:, :n], gs)
    assert (host(q) == oq).all()
    assert (bits(host(s)) == bits(os_)).all()


def test_quantize_nonfinite_fails_like_the_reference(kc):
    x = torch.ones(128, device="cuda")
    x[70] = float("nan")
    kc.quantize(x, 64)
    with pytest.raises(kc.KernelError, match="nonfinite activation"):
        kc.status()
    assert kc.status() == 0  # the error word was cleared


def test_invalid_arguments_fail_like_the_reference(kc):
    x = torch.ones(128, device="cuda")
    q = torch.empty(128, dtype=torch.int8, device="cuda")
    s = torch.empty(2, device="cuda")
    w = torch.empty((4, 128), dtype=torch.int8, device="cuda")
    with pytest.raises(kc.KernelError, match="row stride"):
        kc.k_matmul_q8_ld(torch.empty(4, device="cuda"), q, s, w, s, 100, 128, 4, 64, kc.K_STORE)
    with pytest.raises(kc.KernelError, match="invalid epilogue kind"):
        kc.k_matmul_q8_ld(torch.empty(4, device="cuda"), q, s, w, s, 128, 128, 4, 64, kc.K_SWIGLU)
    with pytest.raises(kc.KernelError, match="segments"):
        kc.k_gemm_q8(q, s, 1, 128, 64, [])


# ---- decode GEMV ----------------------------------------------------------------------------------------------------

def make_case(oracle, d, n, gs, seed, ld=None):
    rng = np.random.default_rng(seed)
    ld = ld or n
    wq, ws = oracle.seeded_q8_matrix(d, ld, gs, seed)
    xq, xs = oracle.quantize(rng.standard_normal(n).astype(np.float32), gs)
    return wq, ws, xq, xs


# The reference suite's own shapes (tests/kernels.c:101: n/d/gs 64/5/16, 192/7/32, 256/4/64, 4096/9/64, 512/3/128,
# 64/2/4) -- the odd ones run on the general rung -- plus the configs' shapes and ragged row counts.
GEMV_SHAPES = [(5, 64, 16), (7, 192, 32), (4, 256, 64), (9, 4096, 64), (3, 512, 128), (2, 64, 4),
               (37, 1024, 64), (8192, 2048, 64), (4096, 14336, 64), (1, 64, 64), (300, 512, 16), (65, 1024, 128),
               (6144, 4096, 64), (77, 1792, 64), (1000, 2048, 256)]


@pytest.mark.parametrize("d,n,gs", GEMV_SHAPES)
def test_gemv_store_bitwise(kc, oracle, d, n, gs):
    wq, ws, xq, xs = make_case(oracle, d, n, gs, d + n)
    y = kc.gemv(dev(xq), dev(xs), dev(wq), dev(ws), gs)
    kc.status()
    ref = oracle.gemv(xq, xs, wq, ws, gs)
    assert (bits(host(y)) == bits(ref)).all()


def test_gemv_golden_reference(kc, oracle):
    """The reference's own decode GEMV outputs (k_matmul_q8 on its AVX-512 ISA, golden gemv512_*), bitwise; and its
    scalar-ISA outputs (golden gemv_*) within its Q8 budget."""
    keys = sorted({k[:-2] for k in GOLDEN.files if k.startswith("gemv512_") and k.endswith("_y")})
    assert keys
    for k in keys:
        gs = int(k.split("_")[-1])
        y = kc.gemv(dev(GOLDEN[k + "_xq"]), dev(GOLDEN[k + "_xs"]), dev(GOLDEN[k + "_wq"]), dev(GOLDEN[k + "_ws"]), gs)
        kc.status()
        assert (bits(host(y)) == bits(GOLDEN[k + "_y"])).all(), k
    for d, n in [(37, 1024), (16, 4096)]:
        k = f"gemv_{d}_{n}"
        wq, ws, xq, xs = (GOLDEN[k + s] for s in ("_wq", "_ws", "_xq", "_xs"))
        y = host(kc.gemv(dev(xq), dev(xs), dev(wq), dev(ws), 64))
        kc.status()
        dots = oracle.group_dots(xq, wq, 64)[:, 0, :].astype(np.float64)
        mag = oracle.group_dots(np.abs(xq).astype(np.int8), np.abs(wq).astype(np.int8), 64)[:, 0, :]
        exact = (dots * ws.T * xs[:, None]).sum(0)
        budget = 2e-5 * (mag * ws.T * xs[:, None]).sum(0) + 1e-6
        assert np.all(np.abs(y - GOLDEN[k + "_y"]) <= 2 * budget)
        assert np.all(np.abs(y - exact) <= budget)


@pytest.mark.parametrize("d,n,gs", [(37, 1024, 64), (4096, 4096, 64)])
def test_gemv_add_and_partial(kc, oracle, d, n, gs):
    wq, ws, xq, xs = make_case(oracle, d, n, gs, 7)
    base = np.random.default_rng(1).standard_normal(d).astype(np.float32)
    out = dev(base)
    kc.gemv(dev(xq), dev(xs), dev(wq), dev(ws), gs, kind=kc.K_ADD, out=out)
    part = kc.gemv(dev(xq), dev(xs), dev(wq), dev(ws), gs, kind=kc.K_PARTIAL)
    kc.status()
    ref = oracle.gemv(xq, xs, wq, ws, gs, kind=oracle.ADD, out=base)
    assert (bits(host(out)) == bits(ref)).all()
    assert (bits(host(part)) == bits(oracle.gemv(xq, xs, wq, ws, gs))).all()


def test_gemv_column_slice_with_row_stride(kc, oracle):
    # A column shard (Wo / W2 under tensor parallelism): rows of stride ld, the owned n columns, the owned activations.
    d, ld, n, gs = 96, 2048, 512, 64
    wq, ws, xq, xs = make_case(oracle, d, ld, gs, 11)
    col0 = 1024
    wslice, sslice = np.ascontiguousarray(wq[:, col0:col0 + n]), np.ascontiguousarray(ws[:, col0 // gs:(col0 + n) // gs])
    rng = np.random.default_rng(2)
    xq2, xs2 = oracle.quantize(rng.standard_normal(n).astype(np.float32), gs)
    wt, st = dev(wq), dev(ws)
    out = torch.zeros(d, device="cuda")
    kc.k_matmul_q8_ld(out, dev(xq2), dev(xs2), wt[:, col0:], st[:, col0 // gs:], ld, n, d, gs, kc.K_PARTIAL)
    kc.status()
    assert (bits(host(out)) == bits(oracle.gemv(xq2, xs2, wslice, sslice, gs))).all()


@pytest.mark.parametrize("n,dq,dkv", [(2048, 2048, 512), (1024, 100, 37), (4096, 4096, 1024)])
def test_gemv_qkv_three_segments(kc, oracle, n, dq, dkv):
    gs = 64
    mats = [make_case(oracle, r, n, gs, 20 + i)[:2] for i, r in enumerate((dq, dkv, dkv))]
    _, _, xq, xs = make_case(oracle, 1, n, gs, 23)
    outs = [torch.zeros(r, device="cuda") for r in (dq, dkv, dkv)]
    kc.k_matmul_q8_qkv(*outs, dev(xq), dev(xs), *[(dev(a), dev(b)) for a, b in mats], n, dq, dkv, gs)
    kc.status()
    for o, (wq, ws) in zip(outs, mats):
        assert (bits(host(o)) == bits(oracle.gemv(xq, xs, wq, ws, gs))).all()


@pytest.mark.parametrize("d,n", [(40, 1024), (8192, 2048), (14336, 4096)])
def test_gemv_swiglu(kc, oracle, d, n):
    gs = 64
    w1q, w1s, xq, xs = make_case(oracle, d, n, gs, 31)
    w3q, w3s = oracle.seeded_q8_matrix(d, n, gs, 32)
    out = kc.gemv(dev(xq), dev(xs), dev(w1q), dev(w1s), gs, kind=kc.K_SWIGLU, w3=(dev(w3q), dev(w3s)))
    kc.status()
    ref = oracle.gemv(xq, xs, w1q, w1s, gs, kind=oracle.SWIGLU, w3q=w3q, w3s=w3s)
    assert ulp_diff(host(out), ref).max() <= 2


@pytest.mark.parametrize("workers", [1, 3, 7])
def test_ld_worker_shares_make_the_full_product(kc, oracle, workers):
    """k_matmul_q8_ld_worker: every member's static share (src/gemv.c:488-495) together equals k_matmul_q8_ld bitwise,
    and done(r0, r1) reports each share once its rows are written, covering [0, d) without overlap."""
    d, ld, n, gs = 100, 512, 512, 64
    wq, ws, xq, xs = make_case(oracle, d, ld, gs, 61)
    full = torch.zeros(d, device="cuda")
    kc.k_matmul_q8_ld(full, dev(xq), dev(xs), dev(wq), dev(ws), ld, n, d, gs, kc.K_STORE)
    out = torch.zeros(d, device="cuda")
    ranges = []
    for w in range(workers):
        kc.k_matmul_q8_ld_worker(out, dev(xq), dev(xs), dev(wq), dev(ws), ld, n, d, gs, kc.K_STORE, w, workers,
                                 done=lambda r0, r1: ranges.append((r0, r1, host(out)[r0:r1].copy())))
    kc.status()
    assert (bits(host(out)) == bits(host(full))).all()
    assert [r[:2] for r in ranges] == [(d * w // workers, d * (w + 1) // workers) for w in range(workers)]
    for r0, r1, rows in ranges:  # the rows were already written when done() ran
        assert (bits(rows) == bits(host(full)[r0:r1])).all()


# ---- W8A32 (K8Input.q NULL, fp32 activations): the reference's AVX-512 order (gs % 16 == 0) and portable loop ----
W8A32_SHAPES = [(37, 1024, 64), (16, 512, 32), (20, 256, 16), (9, 384, 128), (8, 96, 48), (6, 40, 2),
                (4096, 4096, 64), (33, 14336, 64), (1000, 2048, 256), (3, 64, 8)]


@pytest.mark.parametrize("d,n,gs", W8A32_SHAPES)
def test_w8a32_gemv_bitwise(kc, oracle, d, n, gs):
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, d + 3 * n)
    x = (np.random.default_rng(d).standard_normal(n) * 2).astype(np.float32)
    y = kc.gemv(dev(x), None, dev(wq), dev(ws), gs)
    kc.status()
    assert (bits(host(y)) == bits(oracle.gemv_f32(x, wq, ws, gs))).all()


def test_w8a32_golden(kc):
    """The reference's own W8A32 outputs (tests/golden/q8_golden.npz, gemvf_*), bitwise."""
    keys = sorted({k[:-2] for k in GOLDEN.files if k.startswith("gemvf_") and k.endswith("_y")})
    assert keys
    for k in keys:
        gs = int(k.split("_")[-1])
        y = kc.gemv(dev(GOLDEN[k + "_x"]), None, dev(GOLDEN[k + "_wq"]), dev(GOLDEN[k + "_ws"]), gs)
        kc.status()
        assert (bits(host(y)) == bits(GOLDEN[k + "_y"])).all(), k


@pytest.mark.parametrize("gs", [64, 8])
def test_w8a32_epilogues(kc, oracle, gs):
    """ADD, PARTIAL on a column slice with a row stride, three QKV segments and SwiGLU, on fp32 activations."""
    rng = np.random.default_rng(gs)
    d, n = 96, 512
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, 41)
    x = rng.standard_normal(n).astype(np.float32)
    base = rng.standard_normal(d).astype(np.float32)
    out = dev(base)
    kc.gemv(dev(x), None, dev(wq), dev(ws), gs, kind=kc.K_ADD, out=out)
    kc.status()
    assert (bits(host(out)) == bits(base + oracle.gemv_f32(x, wq, ws, gs))).all()
    # Column slice [col0, col0 + m) of rows with stride ld.
    col0, m = 128, 256
    part = torch.zeros(d, device="cuda")
    wt, st = dev(wq), dev(ws)
    kc.k_matmul_q8_ld(part, dev(x[col0:col0 + m]), None, wt[:, col0:], st[:, col0 // gs:], n, m, d, gs, kc.K_PARTIAL)
    kc.status()
    ref = oracle.gemv_f32(x[col0:col0 + m], np.ascontiguousarray(wq[:, col0:col0 + m]),
                          np.ascontiguousarray(ws[:, col0 // gs:(col0 + m) // gs]), gs)
    assert (bits(host(part)) == bits(ref)).all()
    mats = [oracle.seeded_q8_matrix(r, n, gs, 50 + i) for i, r in enumerate((64, 32, 32))]
    outs = [torch.zeros(r, device="cuda") for r in (64, 32, 32)]
    kc.k_matmul_q8_qkv(*outs, dev(x), None, *[(dev(a), dev(b)) for a, b in mats], n, 64, 32, gs)
    kc.status()
    for o, (a, b) in zip(outs, mats):
        assert (bits(host(o)) == bits(oracle.gemv_f32(x, a, b, gs))).all()
    w3q, w3s = oracle.seeded_q8_matrix(d, n, gs, 42)
    sw = kc.gemv(dev(x), None, dev(wq), dev(ws), gs, kind=kc.K_SWIGLU, w3=(dev(w3q), dev(w3s)))
    kc.status()
    a1, a3 = oracle.gemv_f32(x, wq, ws, gs), oracle.gemv_f32(x, w3q, w3s, gs)
    ref = np.array([oracle.lib().orc_silu_gate(float(p), float(q)) for p, q in zip(a1, a3)], np.float32)
    assert ulp_diff(host(sw), ref).max() <= 2


def test_gemv_config0_full_size_properties(kc, oracle):
    # Config 0 (8192 x 2048, N(0, 0.02) weights, N(0, 1) activations): bitwise against the oracle, and linear in the
    # activation scales (doubling every xs doubles y exactly: the rescale multiplies by a power of two).
    wq, ws, xq, xs = make_case(oracle, 8192, 2048, 64, 0)
    y = host(kc.gemv(dev(xq), dev(xs), dev(wq), dev(ws), 64))
    y2 = host(kc.gemv(dev(xq), dev(xs * 2), dev(wq), dev(ws), 64))
    kc.status()
    assert (bits(y) == bits(oracle.gemv(xq, xs, wq, ws, 64))).all()
    assert (bits(y2) == bits(y * 2)).all()


# ---- GEMM (k_gemm_q8) -----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,d,k", [(1, 40, 512), (7, 48, 1024), (33, 32, 256)])
def test_gemm_golden_amx(kc, m, d, k):
    key = f"amx_{m}_{d}_{k}"
    if key + "_c" not in GOLDEN:
        pytest.skip("golden file was made on a CPU without AMX")
    c = kc.gemm(dev(GOLDEN[key + "_xq"]), dev(GOLDEN[key + "_xs"]), dev(GOLDEN[key + "_wq"]), dev(GOLDEN[key + "_ws"]),
                64)
    kc.status()
    assert (bits(host(c)) == bits(GOLDEN[key + "_c"])).all()


@pytest.mark.parametrize("m", [5, 1])
def test_gemm_segments_and_kinds(kc, oracle, m):
    """An ADD segment beside a SwiGLU pair: the tensor-core kernel takes a SwiGLU pair only as its sole segment, so
    k_gemm_q8_pick reports the row rung and k_gemm_q8 runs it, every row in the reference's GEMV order. The ADD segment
    alone goes to the tensor cores at any row count, in the AMX order."""
    k, gs = 1024, 64
    rng = np.random.default_rng(3)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), gs)
    wa = oracle.seeded_q8_matrix(64, k, gs, 40)
    wb = oracle.seeded_q8_matrix(48, k, gs, 41)
    w3 = oracle.seeded_q8_matrix(48, k, gs, 42)
    base = rng.standard_normal((m, 64)).astype(np.float32)
    ca, cb = dev(base), torch.zeros((m, 48), device="cuda")
    segs = [kc.segment(ca, (dev(wa[0]), dev(wa[1])), kc.GEMM_ADD),
            kc.segment(cb, (dev(wb[0]), dev(wb[1])), kc.GEMM_SWIGLU, w3=(dev(w3[0]), dev(w3[1])))]
    assert kc.k_gemm_q8_pick(gs, segs) == kc.Q8_GEMM_GPU_DP4A
    kc.k_gemm_q8(dev(xq), dev(xs), m, k, gs, segs)
    kc.status()
    for r in range(m):
        assert (bits(host(ca)[r]) == bits(oracle.gemv(xq[r], xs[r], *wa, gs, kind=oracle.ADD, out=base[r]))).all()
        ref = oracle.gemv(xq[r], xs[r], *wb, gs, kind=oracle.SWIGLU, w3q=w3[0], w3s=w3[1])
        assert ulp_diff(host(cb)[r], ref).max() <= 2
    ca = dev(base)
    alone = [kc.segment(ca, (dev(wa[0]), dev(wa[1])), kc.GEMM_ADD)]
    assert kc.k_gemm_q8_pick(gs, alone) == kc.Q8_GEMM_GPU_TCGEN05
    kc.k_gemm_q8(dev(xq), dev(xs), m, k, gs, alone)
    kc.status()
    assert (bits(host(ca)) == bits(oracle.gemm(xq, xs, *wa, gs, kind=oracle.ADD, c=base))).all()


# ---- RMSNorm, fused quantize, RoPE ----------------------------------------------------------------------------------

@pytest.mark.parametrize("n", [17, 64, 2048, 4099])
def test_rmsnorm_bitwise_avx512_order(kc, n):
    x, w = GOLDEN[f"rms_{n}_x"], GOLDEN[f"rms_{n}_w"]
    out = torch.empty(n, device="cuda")
    kc.k_rmsnorm(out, dev(x), dev(w), n, 1e-5)
    kc.status()
    assert (bits(host(out)) == bits(GOLDEN[f"rms_{n}_avx512"])).all()
    assert np.allclose(host(out), GOLDEN[f"rms_{n}_scalar"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("rows,size,gs", [(1, 4096, 64), (37, 2048, 64), (3, 512, 128)])
def test_rmsnorm_quantize_fused(kc, oracle, rows, size, gs):
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, size)).astype(np.float32) * 3
    w = rng.uniform(0.5, 1.5, size).astype(np.float32)
    q = torch.empty((rows, size), dtype=torch.int8, device="cuda")
    s = torch.empty((rows, size // gs), device="cuda")
    o = torch.empty((rows, size), device="cuda")
    kc.k_rmsnorm_q8_rows(q, s, o, dev(x), size, dev(w), rows, size, 1e-5, gs)
    kc.status()
    ro = oracle.rmsnorm(x, w, 1e-5)
    rq, rs = oracle.quantize(ro, gs)
    assert (bits(host(o)) == bits(ro)).all()
    assert (host(q) == rq).all() and (bits(host(s)) == bits(rs)).all()


def test_rope_rows_bitwise(kc, oracle):
    rows, nh, nkv, hd = 5, 8, 2, 64
    rng = np.random.default_rng(9)
    q = rng.standard_normal((rows, nh * hd)).astype(np.float32)
    k = rng.standard_normal((rows, nkv * hd)).astype(np.float32)
    tables = np.stack([oracle.rope_table(100 + i, hd) for i in range(rows)])
    qt, kt = dev(q), dev(k)
    kc.k_rope_apply_rows(qt, nh * hd, kt, nkv * hd, dev(tables), 2 * hd, rows, nh, nkv, hd)
    kc.status()
    for i in range(rows):
        rq, rk = oracle.rope_apply(q[i], k[i], tables[i], nh, nkv, hd)
        assert (bits(host(qt)[i]) == bits(rq)).all() and (bits(host(kt)[i]) == bits(rk)).all()


# ---- tensor-core GEMM (tcgen05) -------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,n,k", [(128, 128, 256), (5, 40, 512), (200, 300, 1024), (1, 7, 256)])
def test_gemm_tc_group_dots_exact(kc, oracle, m, n, k):
    # The int32 group dots straight out of TMEM (k_gemm_q8_dots_test), against the exact integer oracle.
    rng = np.random.default_rng(m + n + k)
    wq = rng.integers(-127, 128, (n, k), dtype=np.int8)
    xq = rng.integers(-127, 128, (m, k), dtype=np.int8)
    dots = torch.zeros((k // 64, m, n), dtype=torch.int32, device="cuda")
    assert kc.k_gemm_q8_dots_test(dots, dev(xq), m, k, 64, dev(wq), n) == 1
    kc.status()
    assert (host(dots) == oracle.group_dots(xq, wq, 64)).all()


def test_gemm_tc_group_dots_exact_at_the_extremes(kc, oracle):
    """The group dots at the largest magnitudes int8 allows (64 x 127 x 127 = 1032256 per group, positive and
    negative, and sign patterns between), exact like the integer oracle."""
    m, n, k = 130, 136, 512
    rng = np.random.default_rng(5)
    xq = np.full((m, k), 127, np.int8)
    xq[1::2] = -127
    xq[2::5] = rng.choice(np.array([-127, 127], np.int8), (len(xq[2::5]), k))
    wq = np.full((n, k), 127, np.int8)
    wq[3::3] = -127
    wq[5::7] = rng.integers(-127, 128, (len(wq[5::7]), k), dtype=np.int8)
    dots = torch.zeros((k // 64, m, n), dtype=torch.int32, device="cuda")
    assert kc.k_gemm_q8_dots_test(dots, dev(xq), m, k, 64, dev(wq), n) == 1
    kc.status()
    ref = oracle.group_dots(xq, wq, 64)
    assert np.abs(ref).max() == 64 * 127 * 127
    assert (host(dots) == ref).all()


# Partial token tiles skip the promotion of 16-column chunks past the last token (each epilogue warp holds 32 of a
# tile's 128 token columns): M = 64 fills exactly two quarters, M = 65, 33 and 97 put one token in the next quarter,
# M = 17 one token in a quarter's second chunk, M = 7 fills part of one chunk.
TC_SHAPES = [(128, 128, 256), (33, 48, 1024), (257, 300, 2048), (7, 4096, 4096), (130, 129, 14336), (64, 200, 512),
             (65, 96, 768), (17, 64, 256), (97, 130, 512)]


@pytest.mark.parametrize("m,n,k", TC_SHAPES)
def test_gemm_tc_store_bitwise(kc, oracle, m, n, k):
    rng = np.random.default_rng(m * 7 + n)
    wq, ws = oracle.seeded_q8_matrix(n, k, 64, n)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), 64)
    c = kc.gemm(dev(xq), dev(xs), dev(wq), dev(ws), 64, backend=kc.Q8_GEMM_GPU_TCGEN05)
    kc.status()
    assert (bits(host(c)) == bits(oracle.gemm(xq, xs, wq, ws, 64))).all()


@pytest.mark.parametrize("m,d,k", [(7, 48, 1024), (33, 32, 256)])
def test_gemm_tc_golden_amx(kc, m, d, k):
    # Bitwise the reference's own AMX-INT8 backend (golden vectors made by the compiled reference).
    key = f"amx_{m}_{d}_{k}"
    if key + "_c" not in GOLDEN:
        pytest.skip("golden file was made on a CPU without AMX")
    c = kc.gemm(dev(GOLDEN[key + "_xq"]), dev(GOLDEN[key + "_xs"]), dev(GOLDEN[key + "_wq"]), dev(GOLDEN[key + "_ws"]),
                64, backend=kc.Q8_GEMM_GPU_TCGEN05)
    kc.status()
    assert (bits(host(c)) == bits(GOLDEN[key + "_c"])).all()


def test_gemm_tc_add_swiglu_and_segments(kc, oracle):
    m, k, gs = 150, 1024, 64
    rng = np.random.default_rng(11)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), gs)
    wa, wb, wc = (oracle.seeded_q8_matrix(r, k, gs, 50 + r) for r in (100, 37, 37))
    base = rng.standard_normal((m, 100)).astype(np.float32)
    ca, cb, cc = dev(base), torch.zeros((m, 37), device="cuda"), torch.zeros((m, 37), device="cuda")
    segs = [kc.segment(ca, (dev(wa[0]), dev(wa[1])), kc.GEMM_ADD), kc.segment(cb, (dev(wb[0]), dev(wb[1]))),
            kc.segment(cc, (dev(wc[0]), dev(wc[1])), kc.GEMM_PARTIAL)]
    assert kc.k_gemm_q8_backend_test(kc.Q8_GEMM_GPU_TCGEN05, dev(xq), dev(xs), m, k, gs, segs) == 1
    kc.status()
    assert (bits(host(ca)) == bits(oracle.gemm(xq, xs, *wa, gs, kind=oracle.ADD, c=base))).all()
    assert (bits(host(cb)) == bits(oracle.gemm(xq, xs, *wb, gs))).all()
    assert (bits(host(cc)) == bits(oracle.gemm(xq, xs, *wc, gs))).all()
    w1, w3 = oracle.seeded_q8_matrix(200, k, gs, 61), oracle.seeded_q8_matrix(200, k, gs, 62)
    out = kc.gemm(dev(xq), dev(xs), dev(w1[0]), dev(w1[1]), gs, kind=kc.GEMM_SWIGLU, w3=(dev(w3[0]), dev(w3[1])),
                  backend=kc.Q8_GEMM_GPU_TCGEN05)
    kc.status()
    ref = oracle.gemm(xq, xs, *w1, gs, kind=oracle.SWIGLU, w3q=w3[0], w3s=w3[1])
    assert ulp_diff(host(out), ref).max() <= 2


def test_gemm_tc_config1_full_size(kc, oracle):
    # Config 1 up-projection at T=128 (14336 x 4096): bitwise the oracle on a sample of 96 weight rows; the decode GEMV
    # of 3 token rows (the reference's AVX-512 order) against the oracle on the same rows, and within the reference's
    # Q8 budget of the GEMM's AMX-order rows.
    T, N, K, gs = 128, 14336, 4096, 64
    g = torch.Generator(device="cuda").manual_seed(0)
    wq, ws = kc.quantize(torch.randn((N, K), generator=g, device="cuda") * 0.02, gs)
    xq, xs = kc.quantize(torch.randn((T, K), generator=g, device="cuda"), gs)
    c = kc.gemm(xq, xs, wq, ws, gs, backend=kc.Q8_GEMM_GPU_TCGEN05)
    kc.status()
    rows = np.random.default_rng(1).choice(N, 96, replace=False)
    hw = host(wq)[rows]
    ref = oracle.gemm(host(xq), host(xs), hw, host(ws)[rows], gs)
    assert (bits(host(c)[:, rows]) == bits(ref)).all()
    for t in (0, 77, 127):
        y = host(kc.gemv(xq[t], xs[t], wq, ws, gs))
        kc.status()
        assert (bits(y[rows]) == bits(oracle.gemv(host(xq)[t], host(xs)[t], hw, host(ws)[rows], gs))).all()
        mag = oracle.group_dots(np.abs(host(xq)[t]).astype(np.int8), np.abs(hw).astype(np.int8), gs)[:, 0, :]
        budget = 2e-5 * (mag * host(ws)[rows].T * host(xs)[t][:, None]).sum(0) + 1e-6
        assert np.all(np.abs(y[rows] - host(c)[t, rows]) <= 2 * budget)


@pytest.mark.parametrize("N,K", [(14336, 4096), (4096, 14336)], ids=["up", "down"])
def test_gemm_tc_config1_t2048(kc, oracle, N, K):
    # Config 1 at its largest batch, T = 2048, on both FFN projections: bitwise the oracle on 48 sampled weight rows
    # (every one of the 2048 token rows, so every token tile and every column quarter of the epilogue is covered).
    T, gs = 2048, 64
    g = torch.Generator(device="cuda").manual_seed(N + K)
    wq, ws = kc.quantize(torch.randn((N, K), generator=g, device="cuda") * 0.02, gs)
    xq, xs = kc.quantize(torch.randn((T, K), generator=g, device="cuda"), gs)
    c = kc.gemm(xq, xs, wq, ws, gs, backend=kc.Q8_GEMM_GPU_TCGEN05)
    kc.status()
    rows = np.sort(np.random.default_rng(N).choice(N, 48, replace=False))
    ref = oracle.gemm(host(xq), host(xs), host(wq)[rows], host(ws)[rows], gs)
    assert (bits(host(c)[:, rows]) == bits(ref)).all()


def test_k_gemm_q8_picks_tensor_cores_for_batches(kc, oracle):
    m, k, gs = 64, 1024, 64
    rng = np.random.default_rng(4)
    wq, ws = oracle.seeded_q8_matrix(96, k, gs, 9)
    xq, xs = oracle.quantize(rng.standard_normal((m, k)).astype(np.float32), gs)
    c = kc.gemm(dev(xq), dev(xs), dev(wq), dev(ws), gs)
    kc.status()
    assert (bits(host(c)) == bits(oracle.gemm(xq, xs, wq, ws, gs))).all()


# ---- the fused-input GEMV (k_matmul_q8_fused): RMSNorm / quantize inside the kernel ----------------------------------

@pytest.mark.parametrize("n", [512, 2048, 4096])
def test_fused_norm_qkv_bitwise(kc, oracle, n):
    """RMSNorm + quantize + 3-segment GEMV in one launch equals k_rmsnorm_q8_rows + k_matmul_q8_qkv and the oracle."""
    gs, dq, dkv = 64, n, n // 4
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    mats = [oracle.seeded_q8_matrix(r, n, gs, 100 + i) for i, r in enumerate((dq, dkv, dkv))]
    dm = [(dev(a), dev(b)) for a, b in mats]
    fused = [torch.zeros(r, device="cuda") for r in (dq, dkv, dkv)]
    segs = [kc.segment(o, m) for o, m in zip(fused, dm)]
    kc.k_matmul_q8_fused(dev(x), dev(w), 1e-5, n, n, gs, segs)
    q = torch.empty(n, dtype=torch.int8, device="cuda")
    s = torch.empty(n // gs, device="cuda")
    kc.k_rmsnorm_q8_rows(q, s, None, dev(x), n, dev(w), 1, n, 1e-5, gs)
    apart = [torch.zeros(r, device="cuda") for r in (dq, dkv, dkv)]
    kc.k_matmul_q8_qkv(*apart, q, s, *dm, n, dq, dkv, gs)
    kc.status()
    rq, rs = oracle.quantize(oracle.rmsnorm(x, w, 1e-5), gs)
    for f, a, (wq, ws) in zip(fused, apart, mats):
        assert (bits(host(f)) == bits(host(a))).all()
        assert (bits(host(f)) == bits(oracle.gemv(rq, rs, wq, ws, gs))).all()


def test_fused_norm_swiglu_and_quantize_add_bitwise(kc, oracle):
    gs, n, hidden = 64, 4096, 14336
    rng = np.random.default_rng(7)
    x = rng.standard_normal(n).astype(np.float32)
    w = np.ones(n, np.float32)
    w1, w3 = oracle.seeded_q8_matrix(hidden, n, gs, 1), oracle.seeded_q8_matrix(hidden, n, gs, 3)
    hb = torch.zeros(hidden, device="cuda")
    kc.k_matmul_q8_fused(dev(x), dev(w), 1e-5, n, n, gs,
                         [kc.segment(hb, (dev(w1[0]), dev(w1[1])), kc.GEMM_SWIGLU, w3=(dev(w3[0]), dev(w3[1])))])
    q = torch.empty(n, dtype=torch.int8, device="cuda")
    s = torch.empty(n // gs, device="cuda")
    kc.k_rmsnorm_q8_rows(q, s, None, dev(x), n, dev(w), 1, n, 1e-5, gs)
    ref = kc.gemv(q, s, dev(w1[0]), dev(w1[1]), gs, kind=kc.K_SWIGLU, w3=(dev(w3[0]), dev(w3[1])))
    kc.status()
    assert (bits(host(hb)) == bits(host(ref))).all()
    # The down projection on fp32 input (quantize only), accumulated into a residual.
    w2 = oracle.seeded_q8_matrix(n, hidden, gs, 5)
    base = rng.standard_normal(n).astype(np.float32)
    res_f, res_a = dev(base), dev(base)
    kc.k_matmul_q8_fused(hb, None, 0.0, hidden, hidden, gs, [kc.segment(res_f, (dev(w2[0]), dev(w2[1])), kc.GEMM_ADD)])
    hq, hs = kc.quantize(hb, gs)
    kc.gemv(hq, hs, dev(w2[0]), dev(w2[1]), gs, kind=kc.K_ADD, out=res_a)
    kc.status()
    assert (bits(host(res_f)) == bits(host(res_a))).all()
    rq, rs = oracle.quantize(host(hb), gs)
    assert (bits(host(res_f)) == bits(oracle.gemv(rq, rs, *w2, gs, kind=oracle.ADD, out=base))).all()


def test_fused_partial_on_a_column_slice(kc, oracle):
    """A tensor-parallel W2 shard: PARTIAL over a column slice (row stride ld > n) on fp32 input."""
    gs, rows, full, n, c0 = 64, 256, 1024, 256, 512
    wq, ws = oracle.seeded_q8_matrix(rows, full, gs, 9)
    x = np.random.default_rng(3).standard_normal(n).astype(np.float32)
    out = torch.zeros(rows, device="cuda")
    wd = (dev(wq)[:, c0:], dev(ws)[:, c0 // gs:])
    seg = kc.GemmQ8Segment()
    seg.c, seg.ldc, seg.n, seg.kind = kc._ptr(out), rows, rows, kc.GEMM_PARTIAL
    seg.w = kc.K8Weight(kc._ptr(wd[0]), kc._ptr(wd[1]))
    seg._tensors = (out,) + wd
    kc.k_matmul_q8_fused(dev(x), None, 0.0, full, n, gs, [seg])
    kc.status()
    rq, rs = oracle.quantize(x, gs)
    ref = oracle.gemv(rq, rs, np.ascontiguousarray(wq[:, c0:c0 + n]), np.ascontiguousarray(ws[:, c0 // gs:(c0 + n) // gs]),
                      gs)
    assert (bits(host(out)) == bits(ref)).all()


def test_fused_rejects_mixed_kinds(kc, oracle):
    wq, ws = oracle.seeded_q8_matrix(64, 256, 64, 1)
    a, b = torch.zeros(64, device="cuda"), torch.zeros(64, device="cuda")
    x = torch.zeros(256, device="cuda")
    with pytest.raises(kc.KernelError, match="one kind"):
        kc.k_matmul_q8_fused(x, None, 0.0, 256, 256, 64, [kc.segment(a, (dev(wq), dev(ws))),
                                                           kc.segment(b, (dev(wq), dev(ws)), kc.GEMM_ADD)])


# ---- the tail GEMV (k_matmul_q8_tail): the next step's small work done once by the last CTA -------------------------

def _tail(kc, kind, **kw):
    t = kc.KernelTail()
    t.kind = kind
    for k, v in kw.items():
        setattr(t, k, kc._ptr(v) if hasattr(v, "data_ptr") else v)
    return t


def test_tail_norm_quantize_after_add_bitwise(kc, oracle):
    """Wo-like: x += W a, then the next GEMV's input rmsnorm+quantize(x) by the last CTA; three calls in a row."""
    gs, n, d = 64, 4096, 4096
    rng = np.random.default_rng(21)
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, 21)
    nw = dev((1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    x = dev(rng.standard_normal(d).astype(np.float32))
    x_ref = x.clone()
    for step in range(3):
        a = rng.standard_normal(n).astype(np.float32)
        aq, as_ = kc.quantize(dev(a), gs)
        q = torch.empty(d, dtype=torch.int8, device="cuda")
        s = torch.empty(d // gs, device="cuda")
        tail = _tail(kc, kc.K_TAIL_NORM_QUANTIZE, x=x, weight=nw, epsilon=1e-5, q=q, s=s, n=d)
        kc.k_matmul_q8_tail(aq, as_, n, n, gs, [kc.segment(x, (dev(wq), dev(ws)), kc.GEMM_ADD)], tail)
        kc.gemv(aq, as_, dev(wq), dev(ws), gs, kind=kc.K_ADD, out=x_ref)
        rq = torch.empty(d, dtype=torch.int8, device="cuda")
        rs = torch.empty(d // gs, device="cuda")
        kc.k_rmsnorm_q8_rows(rq, rs, None, x_ref, d, nw, 1, d, 1e-5, gs)
        kc.status()
        assert (bits(host(x)) == bits(host(x_ref))).all(), step
        assert (host(q) == host(rq)).all() and (bits(host(s)) == bits(host(rs))).all(), step


def test_tail_quantize_after_swiglu_bitwise(kc, oracle):
    gs, n, hidden = 64, 4096, 14336
    rng = np.random.default_rng(22)
    w1, w3 = oracle.seeded_q8_matrix(hidden, n, gs, 1), oracle.seeded_q8_matrix(hidden, n, gs, 2)
    xq, xs = kc.quantize(dev(rng.standard_normal(n).astype(np.float32)), gs)
    hb = torch.zeros(hidden, device="cuda")
    hq = torch.empty(hidden, dtype=torch.int8, device="cuda")
    hs = torch.empty(hidden // gs, device="cuda")
    tail = _tail(kc, kc.K_TAIL_QUANTIZE, x=hb, q=hq, s=hs, n=hidden)
    seg = kc.segment(hb, (dev(w1[0]), dev(w1[1])), kc.GEMM_SWIGLU, w3=(dev(w3[0]), dev(w3[1])))
    kc.k_matmul_q8_tail(xq, xs, n, n, gs, [seg], tail)
    ref = kc.gemv(xq, xs, dev(w1[0]), dev(w1[1]), gs, kind=kc.K_SWIGLU, w3=(dev(w3[0]), dev(w3[1])))
    rq, rs = kc.quantize(ref, gs)
    kc.status()
    assert (bits(host(hb)) == bits(host(ref))).all()
    assert (host(hq) == host(rq)).all() and (bits(host(hs)) == bits(host(rs))).all()


@pytest.mark.parametrize("hidden", [14336, 1792, 192])
def test_output_quantizer_after_fused_swiglu_bitwise(kc, oracle, hidden):
    """The decode FFN's first GEMV as the engine runs it: RMSNorm + quantize of x inside the kernel, SwiGLU, and its
    output quantized for W2 group by group by the CTAs that complete each group (K_TAIL_QUANTIZE_OUTPUT). Equal to
    k_rmsnorm_q8_rows + the SwiGLU GEMV + k_quantize bitwise; three calls in a row (the counters reset), shapes with
    many rows per CTA, a TP shard, and fewer rows than CTAs."""
    gs, n = 64, 4096
    rng = np.random.default_rng(hidden)
    w1, w3 = oracle.seeded_q8_matrix(hidden, n, gs, 3), oracle.seeded_q8_matrix(hidden, n, gs, 4)
    nw = dev((1 + 0.1 * rng.standard_normal(n)).astype(np.float32))
    seg_w = ((dev(w1[0]), dev(w1[1])), (dev(w3[0]), dev(w3[1])))
    for step in range(3):
        x = dev(rng.standard_normal(n).astype(np.float32))
        hb = torch.zeros(hidden, device="cuda")
        hq = torch.empty(hidden, dtype=torch.int8, device="cuda")
        hs = torch.empty(hidden // gs, device="cuda")
        tail = _tail(kc, kc.K_TAIL_QUANTIZE_OUTPUT, q=hq, s=hs)
        kc.k_matmul_q8_fused(x, nw, 1e-5, n, n, gs, [kc.segment(hb, seg_w[0], kc.GEMM_SWIGLU, w3=seg_w[1])], tail)
        xq = torch.empty(n, dtype=torch.int8, device="cuda")
        xs = torch.empty(n // gs, device="cuda")
        kc.k_rmsnorm_q8_rows(xq, xs, None, x, n, nw, 1, n, 1e-5, gs)
        ref = kc.gemv(xq, xs, *seg_w[0], gs, kind=kc.K_SWIGLU, w3=seg_w[1])
        rq, rs = kc.quantize(ref, gs)
        kc.status()
        assert (bits(host(hb)) == bits(host(ref))).all(), step
        assert (host(hq) == host(rq)).all() and (bits(host(hs)) == bits(host(rs))).all(), step


def test_output_quantizer_store_segment_bitwise(kc, oracle):
    """K_TAIL_QUANTIZE_OUTPUT on a STORE GEMV with int8 input, group size 128, rows that do not split evenly; a group
    size the lane-order kernel does not take (32: the reference's portable order) is refused, not run elsewhere."""
    gs, n, d = 128, 2048, 4096 + 5 * 128
    with pytest.raises(kc.KernelError, match="shape not supported"):
        z = torch.zeros(64, device="cuda")
        kc.k_matmul_q8_tail(torch.zeros(256, dtype=torch.int8, device="cuda"), torch.zeros(8, device="cuda"), 256, 256,
                            32, [kc.segment(z, (torch.zeros((64, 256), dtype=torch.int8, device="cuda"),
                                                torch.zeros((64, 8), device="cuda")))],
                            _tail(kc, kc.K_TAIL_QUANTIZE_OUTPUT, q=torch.empty(64, dtype=torch.int8, device="cuda"),
                                  s=torch.empty(2, device="cuda")))
    rng = np.random.default_rng(23)
    wq, ws = oracle.seeded_q8_matrix(d, n, gs, 23)
    xq, xs = kc.quantize(dev(rng.standard_normal(n).astype(np.float32)), gs)
    out = torch.zeros(d, device="cuda")
    q = torch.empty(d, dtype=torch.int8, device="cuda")
    s = torch.empty(d // gs, device="cuda")
    kc.k_matmul_q8_tail(xq, xs, n, n, gs, [kc.segment(out, (dev(wq), dev(ws)))], _tail(kc, kc.K_TAIL_QUANTIZE_OUTPUT,
                                                                                       q=q, s=s))
    ref = kc.gemv(xq, xs, dev(wq), dev(ws), gs)
    rq, rs = kc.quantize(ref, gs)
    kc.status()
    assert (bits(host(out)) == bits(host(ref))).all()
    assert (host(q) == host(rq)).all() and (bits(host(s)) == bits(host(rs))).all()


@pytest.mark.parametrize("nh,nkv,hd", [(32, 8, 128), (8, 4, 32)])
def test_tail_rope_kv_store_bitwise(kc, oracle, nh, nkv, hd):
    gs, n, seq, pos = 64, nh * hd, 64, 37
    rng = np.random.default_rng(nh)
    mats = [oracle.seeded_q8_matrix(r, n, gs, 30 + i) for i, r in enumerate((nh * hd, nkv * hd, nkv * hd))]
    dm = [(dev(a), dev(b)) for a, b in mats]
    xq, xs = kc.quantize(dev(rng.standard_normal(n).astype(np.float32)), gs)
    table = dev(np.stack([oracle.rope_table(p, hd, 500000.0) for p in range(seq)]))
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    outs = [torch.zeros(r, device="cuda") for r in (nh * hd, nkv * hd, nkv * hd)]
    kcache, vcache = torch.zeros((nkv, seq, hd), device="cuda"), torch.zeros((nkv, seq, hd), device="cuda")
    tail = _tail(kc, kc.K_TAIL_ROPE_KV_STORE, rope_table=table, position=p, key_cache=kcache, value_cache=vcache,
                 n_heads=nh, n_kv_heads=nkv, head_dim=hd, seq_len=seq)
    kc.k_matmul_q8_tail(xq, xs, n, n, gs, [kc.segment(o, m) for o, m in zip(outs, dm)], tail)
    ref = [torch.zeros(r, device="cuda") for r in (nh * hd, nkv * hd, nkv * hd)]
    kc.k_matmul_q8_qkv(*ref, xq, xs, *dm, n, nh * hd, nkv * hd, gs)
    rk, rv = torch.zeros_like(kcache), torch.zeros_like(vcache)
    kc.k_rope_kv_store_rows(ref[0], nh * hd, ref[1], ref[2], nkv * hd, rk, rv, table, p, 0, 1, nh, nkv, hd, seq)
    kc.status()
    assert (bits(host(outs[0])) == bits(host(ref[0]))).all()
    assert torch.equal(kcache, rk) and torch.equal(vcache, rv)
