"""CPU tests of the C-ABI's argument checks (include/kernels_cuda.h): invalid arguments fail on the host with a message
and queue no work, so no kernel ever receives them. Under KC_FAIL_RETURN the message is kept and the call returns; by
default the library exits with it, as the reference's fail() does (include/runtime.h:29).

The buffers are made-up aligned addresses: every call here is rejected before anything could read them, and the
process has no CUDA context at all."""
import ctypes

import pytest

from conftest import load_package

A = 0x10000  # a 16-byte aligned address that is never read


@pytest.fixture(scope="module")
def lib():
    kc = load_package()
    L = kc.load()
    L.kc_set_fail_mode(kc.KC_FAIL_RETURN)
    return kc, L


def rejected(L):
    msg = L.kc_last_error()
    L.kc_clear_error()
    assert msg, "the call was accepted"
    return msg.decode()


def w8a8(kc):
    return ctypes.byref(kc.K8Input(A, A, None))


def test_quantize_and_gemv_shapes(lib):
    kc, L = lib
    # n need not be a whole number of groups: the reference quantizes the whole groups and leaves the tail.
    L.k_quantize_rows(A, A, A, 128, 1, 128, 0)
    assert rejected(L) == "k_quantize_rows: invalid shape m=1 n=128 ldx=128 gs=0"
    L.k_quantize_rows(A, A, A, 64, 2, 128, 64)
    assert rejected(L) == "k_quantize_rows: invalid shape m=2 n=128 ldx=64 gs=64"
    L.k_matmul_q8(A, w8a8(kc), kc.K8Weight(A, A), 100, 4, 64)
    assert rejected(L) == "k_matmul_q8: 100 inputs are not a whole number of 64-groups"
    L.k_matmul_q8(A, w8a8(kc), kc.K8Weight(A, A), 128, 4, 0)
    assert rejected(L) == "k_matmul_q8: invalid group size 0"
    L.k_matmul_q8_ld(A, w8a8(kc), ctypes.byref(kc.K8Weight(A, A)), 100, 128, 4, 64, kc.K_STORE)
    assert "row stride 100 must be at least 128 and a multiple of the group size 64" in rejected(L)
    L.k_matmul_q8_ld(A, w8a8(kc), ctypes.byref(kc.K8Weight(A, A)), 128, 128, 4, 64, kc.K_SWIGLU)
    assert rejected(L) == "k_matmul_q8_ld: invalid epilogue kind 3"
    L.k_matmul_q8_ld_worker(A, w8a8(kc), ctypes.byref(kc.K8Weight(A, A)), 128, 128, 4, 64, kc.K_STORE, 3, 2, None,
                            None, None)
    assert "invalid member 3 of 2" in rejected(L)


def test_gemv_missing_pointers(lib):
    kc, L = lib
    L.k_matmul_q8(A, ctypes.byref(kc.K8Input(None, None, None)), kc.K8Weight(A, A), 128, 4, 64)
    assert "the input needs int8 values and scales, or (W8A32) fp32 activations" in rejected(L)
    L.k_matmul_q8(A, ctypes.byref(kc.K8Input(A, None, None)), kc.K8Weight(A, A), 128, 4, 64)
    assert "the input needs int8 values and scales" in rejected(L)
    L.k_matmul_q8(A, w8a8(kc), kc.K8Weight(None, A), 128, 4, 64)
    assert rejected(L) == "k_matmul_q8: missing weight values or scales"
    L.k_matmul_q8(None, w8a8(kc), kc.K8Weight(A, A), 128, 4, 64)
    assert rejected(L) == "k_matmul_q8: missing output"


def segs(kc, *items):
    return (kc.GemmQ8Segment * len(items))(*items)


def seg(kc, n=4, kind=None, c=A, w=(A, A), w3=(None, None), ldc=None):
    return kc.GemmQ8Segment(c, n if ldc is None else ldc, kc.K8Weight(*w), kc.K8Weight(*w3), None, None, n,
                            kc.GEMM_STORE if kind is None else kind)


def test_gemm_arguments(lib):
    kc, L = lib
    L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, seg(kc)), 0)
    assert rejected(L) == "GEMM needs 1..3 segments, got 0"
    # More segments than the kernel takes: rejected before anything copies them into its fixed-size table.
    L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, *[seg(kc)] * 5), 5)
    assert rejected(L) == "GEMM needs 1..3 segments, got 5"
    L.k_gemm_q8(A, A, 16, 128, 64, None, 1)
    assert rejected(L) == "GEMM needs 1..3 segments, got 0"
    L.k_gemm_q8(A, A, 16, 100, 64, segs(kc, seg(kc)), 1)
    assert rejected(L) == "Q8 GEMM: K=100 is not a multiple of the group size 64"
    L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, seg(kc, kind=kc.GEMM_SWIGLU)), 1)
    assert rejected(L) == "GEMM_SWIGLU needs a second weight matrix"
    L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, seg(kc, ldc=3)), 1)
    assert rejected(L) == "k_gemm_q8: ldc 3 is shorter than the 4 outputs"
    L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, seg(kc, kind=7)), 1)
    assert rejected(L) == "k_gemm_q8: invalid GEMM kind 7"
    L.k_gemm_q8(A, A, -1, 128, 64, segs(kc, seg(kc)), 1)
    assert rejected(L) == "k_gemm_q8: negative shape"


def test_gemm_missing_pointers(lib):
    kc, L = lib
    L.k_gemm_q8(A, None, 16, 128, 64, segs(kc, seg(kc)), 1)
    assert rejected(L) == "k_gemm_q8: missing activations"
    for bad in (seg(kc, c=None), seg(kc, w=(A, None)), seg(kc, w=(None, A)),
                seg(kc, kind=kc.GEMM_SWIGLU, w3=(A, None))):
        L.k_gemm_q8(A, A, 16, 128, 64, segs(kc, seg(kc), bad), 2)
        assert rejected(L) == "k_gemm_q8: segment 1 is missing its output, weight values or scales"


def test_noalloc_rejects_sizes_beyond_its_array(lib):
    # m = 8192 tokens at k = 14336 need 224 * 8192 transposed scales, above the fixed 2^20.
    kc, L = lib
    assert L.k_gemm_q8_noalloc(A, A, 8192, 14336, 64, segs(kc, seg(kc, n=4096)), 1) == -1
    assert rejected(L) == "k_gemm_q8_noalloc: m=8192 k=14336 needs 1835008 scale floats, above the fixed 1048576"
    assert L.k_gemm_q8_noalloc(A, A, 16, 100, 64, segs(kc, seg(kc)), 1) == -1
    assert rejected(L) == "Q8 GEMM: K=100 is not a multiple of the group size 64"


def test_support_kernel_shapes(lib):
    kc, L = lib
    L.k_rmsnorm_rows(A, A, A, -1, 64, 1e-5)
    assert rejected(L) == "k_rmsnorm_rows: invalid shape rows=-1 size=64"
    L.k_rmsnorm_rows(A, A, A, 1, 0, 1e-5)
    assert rejected(L) == "k_rmsnorm_rows: invalid shape rows=1 size=0"


def test_fused_and_tail_gemv_arguments(lib):
    kc, L = lib
    L.k_matmul_q8_fused(A, A, 1e-5, 128, 128, 64, segs(kc, seg(kc), seg(kc, c=None)), 2, None)
    assert rejected(L) == "k_matmul_q8_fused: segment 1 is missing its output"
    L.k_matmul_q8_fused(A, A, 1e-5, 128, 128, 64, None, 1, None)
    assert rejected(L) == "k_matmul_q8_fused: needs 1..3 segments, got 0"
    L.k_matmul_q8_fused(A, A, 1e-5, 128, 128, 64, segs(kc, seg(kc), seg(kc, kind=kc.GEMM_ADD)), 2, None)
    assert "segments need one kind" in rejected(L)
    L.k_matmul_q8_fused(None, A, 1e-5, 128, 128, 64, segs(kc, seg(kc)), 1, None)
    assert rejected(L) == "k_matmul_q8_fused: missing activations"
    L.k_matmul_q8_tail(w8a8(kc), 128, 128, 64, segs(kc, seg(kc)), 1, None)
    assert rejected(L) == "k_matmul_q8_tail: missing tail"
    tail = kc.KernelTail(kind=kc.K_TAIL_QUANTIZE_OUTPUT)  # without q and s
    L.k_matmul_q8_tail(w8a8(kc), 128, 128, 64, segs(kc, seg(kc, n=128)), 1, ctypes.byref(tail))
    assert "the output quantizer needs one STORE or SWIGLU segment" in rejected(L)
    tail = kc.KernelTail(kind=9)
    L.k_matmul_q8_tail(w8a8(kc), 128, 128, 64, segs(kc, seg(kc)), 1, ctypes.byref(tail))
    assert rejected(L) == "k_matmul_q8_tail: invalid tail kind 9"
