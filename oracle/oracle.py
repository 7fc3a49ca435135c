"""TEST INFRASTRUCTURE ONLY: numpy bindings of the CPU checker (liboracle.so) and of the reference compiled from its
own sources (_ref/libllama_ref.so, present only where oracle/Makefile could build it).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only as the checker or
the timed CPU baseline -- never as the implementation under test. Every restated function cites the reference file and
line it follows (q8_oracle.h).
"""
import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libllama_ref.so"
PROBE_INT8 = HERE / "_ref" / "probe-int8"

STORE, ADD, PARTIAL, SWIGLU = 0, 1, 2, 3

_i8p = ctypes.POINTER(ctypes.c_int8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


def _p(a, t):
    return a.ctypes.data_as(t)


def reference_checkout():
    """The reference's sources: $LLAMA3X_REFERENCE, else a checkout named `reference` beside this repository; None
    when neither holds src/gemv.c."""
    import os
    for cand in (os.environ.get("LLAMA3X_REFERENCE"), HERE.parent.parent / "reference"):
        if cand and (Path(cand) / "src" / "gemv.c").exists():
            return Path(cand)
    return None


def build():
    """Compile liboracle.so (and the reference under _ref/ when its sources are found) with oracle/Makefile."""
    import subprocess
    ref = reference_checkout()
    subprocess.run(["make", "-s", "-C", str(HERE)] + ([f"REF={ref}"] if ref else []), check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.orc_quantize.argtypes = [_i8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_quantize.restype = ctypes.c_int
        L.orc_quantize_rows.argtypes = [_i8p, _f32p, _f32p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_quantize_rows.restype = ctypes.c_int
        L.orc_group_dots.argtypes = [_i32p, _i8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i8p, ctypes.c_size_t,
                                     ctypes.c_int]
        for name in ("orc_gemv_f32_avx512_order", "orc_gemv_f32_scalar"):
            getattr(L, name).argtypes = [_f32p, _f32p, _i8p, _f32p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int]
        L.orc_gemv_scalar.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int]
        L.orc_gemm_amx_order.argtypes = [_f32p, ctypes.c_int, _i8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         _i8p, _f32p, _i8p, _f32p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
        L.orc_silu_gate.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_exp512.argtypes = [ctypes.c_float]
        L.orc_exp512.restype = ctypes.c_float
        L.orc_attention_chunks.argtypes = [ctypes.c_int] * 4
        L.orc_attention_chunks.restype = ctypes.c_int
        L.orc_attention_decode.argtypes = [_f32p] * 4 + [ctypes.c_int] * 7
        L.orc_attention_decode.restype = ctypes.c_int
        L.orc_attention_tiled.argtypes = [_f32p] * 4 + [ctypes.c_int] * 8
        L.orc_attention_tiled.restype = ctypes.c_int
        L.orc_gemv_ref_order.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, _i8p, _f32p, ctypes.c_size_t, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_silu_gate.restype = ctypes.c_float
        L.orc_rmsnorm_scalar.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.orc_rmsnorm_avx512_order.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.orc_rope_table.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.orc_rope_apply.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _lib = L
    return _lib


def quantize(x, gs):
    """k_quantize over the last axis of x (rows quantized independently, src/gemm.c:818-830)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    q = np.empty(rows.shape, np.int8)
    s = np.empty((rows.shape[0], n // gs), np.float32)
    rc = lib().orc_quantize_rows(_p(q, _i8p), _p(s, _f32p), _p(rows, _f32p), n, rows.shape[0], n, gs)
    if rc:
        raise ValueError("nonfinite activation during INT8 quantization")
    return q.reshape(x.shape), s.reshape(x.shape[:-1] + (n // gs,))


def group_dots(xq, wq, gs):
    """int32 dots[g][m][n] of activation rows xq[m][k] and weight rows wq[n][k]."""
    xq = np.ascontiguousarray(np.atleast_2d(xq), dtype=np.int8)
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    m, k = xq.shape
    n = wq.shape[0]
    out = np.empty((k // gs, m, n), np.int32)
    lib().orc_group_dots(_p(out, _i32p), _p(xq, _i8p), m, k, gs, _p(wq, _i8p), wq.shape[1], n)
    return out


def gemv_scalar(xq, xs, wq, ws, gs):
    """q8_dots in the scalar order (src/gemv.c:417-438) for one activation row."""
    xq = np.ascontiguousarray(xq, np.int8)
    xs = np.ascontiguousarray(xs, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, ld = wq.shape
    out = np.empty(d, np.float32)
    lib().orc_gemv_scalar(_p(out, _f32p), _p(xq, _i8p), _p(xs, _f32p), _p(wq, _i8p), _p(ws, _f32p), ld, xq.shape[-1],
                          d, gs)
    return out


def gemv_f32(x, wq, ws, gs):
    """W8A32 (fp32 activations): the reference's AVX-512 order (dots_q8f_body, src/gemv.c:141-180) when gs % 16 == 0,
    else its portable loop (src/gemv.c:427-436); one activation row, d rows of weights."""
    x = np.ascontiguousarray(x, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, ld = wq.shape
    out = np.empty(d, np.float32)
    f = lib().orc_gemv_f32_avx512_order if gs % 16 == 0 else lib().orc_gemv_f32_scalar
    f(_p(out, _f32p), _p(x, _f32p), _p(wq, _i8p), _p(ws, _f32p), ld, x.shape[-1], d, gs)
    return out


def gemv(xq, xs, wq, ws, gs, kind=STORE, out=None, w3q=None, w3s=None, n=None):
    """The reference's decode GEMV (k_matmul_q8 on an AVX-512 host, src/gemv.c:401-528) for one activation row and d
    weight rows (row stride wq.shape[1]; n inputs, default all): dots_q8_body's 16-lane order for gs % 64 == 0, the
    portable loop otherwise, with the STORE / ADD / PARTIAL / SWIGLU epilogues."""
    xq = np.ascontiguousarray(np.ravel(xq), np.int8)
    xs = np.ascontiguousarray(np.ravel(xs), np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, ld = wq.shape
    n = xq.shape[0] if n is None else n
    y = np.zeros(d, np.float32) if out is None else np.array(out, np.float32, copy=True).reshape(d)
    a3 = b3 = None
    if kind == SWIGLU:
        w3q = np.ascontiguousarray(w3q, np.int8)
        w3s = np.ascontiguousarray(w3s, np.float32)
        a3, b3 = _p(w3q, _i8p), _p(w3s, _f32p)
    lib().orc_gemv_ref_order(_p(y, _f32p), _p(xq, _i8p), _p(xs, _f32p), _p(wq, _i8p), _p(ws, _f32p), a3, b3, ld, n, d,
                             gs, kind)
    return y


def gemm(xq, xs, wq, ws, gs, kind=STORE, c=None, w3q=None, w3s=None):
    """C[m][n] in the AMX-INT8 order (src/gemm.c:554-610) with the epilogues of src/gemm.c:963-989."""
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    m, k = xq.shape
    n, ldw = wq.shape
    out = np.zeros((m, n), np.float32) if c is None else np.array(c, np.float32, copy=True).reshape(m, n)
    if kind == SWIGLU:
        w3q = np.ascontiguousarray(w3q, np.int8)
        w3s = np.ascontiguousarray(w3s, np.float32)
        a3, b3 = _p(w3q, _i8p), _p(w3s, _f32p)
    else:
        a3, b3 = None, None
    lib().orc_gemm_amx_order(_p(out, _f32p), n, _p(xq, _i8p), _p(xs, _f32p), m, k, gs, _p(wq, _i8p), _p(ws, _f32p),
                             a3, b3, ldw, n, kind)
    return out


def silu_gate(v, g):
    f = lib().orc_silu_gate
    return np.array([f(float(a), float(b)) for a, b in zip(np.ravel(v), np.ravel(g))], np.float32).reshape(np.shape(v))


def rmsnorm(x, w, eps, order="avx512"):
    """k_rmsnorm over the last axis, in the AVX-512 order (src/kernels_simd.c:136-161) or the scalar one."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    out = np.empty_like(rows)
    f = lib().orc_rmsnorm_avx512_order if order == "avx512" else lib().orc_rmsnorm_scalar
    for r in range(rows.shape[0]):
        f(_p(out[r], _f32p), _p(rows[r], _f32p), _p(w, _f32p), n, eps)
    return out.reshape(x.shape)


def rope_table(position, head_dim, theta=500000.0, rope_type=0, factor=1.0, low=1.0, high=4.0, original=8192):
    t = np.empty(2 * head_dim, np.float32)
    lib().orc_rope_table(_p(t, _f32p), position, head_dim, theta, rope_type, factor, low, high, original)
    return t


def rope_apply(q, k, table, n_heads, n_kv_heads, head_dim):
    q = np.array(q, np.float32, copy=True)
    k = np.array(k, np.float32, copy=True)
    lib().orc_rope_apply(_p(q, _f32p), _p(k, _f32p), _p(np.ascontiguousarray(table, np.float32), _f32p), n_heads,
                         n_kv_heads, head_dim)
    return q, k


# ---- the reference itself (compiled from its sources by oracle/Makefile) -------------------------------------------

class K8Weight(ctypes.Structure):
    _fields_ = [("q", _i8p), ("s", _f32p)]


class K8Input(ctypes.Structure):
    _fields_ = [("q", _i8p), ("s", _f32p), ("f", _f32p)]


class GemmQ8Segment(ctypes.Structure):
    _fields_ = [("c", _f32p), ("ldc", ctypes.c_int), ("w", K8Weight), ("w3", K8Weight), ("pw", _i8p), ("pw3", _i8p),
                ("n", ctypes.c_int), ("kind", ctypes.c_int)]


KERNELS_SCALAR, KERNELS_AVX512, KERNELS_AMX = 0, 1, 2
Q8_GEMM_PORTABLE, Q8_GEMM_AVX512, Q8_GEMM_AMX = 0, 1, 2

_ref = None


def ref_available():
    return REF_SO.exists()


def ref():
    """The reference library (fail() inside it exits the process: call it with valid arguments only)."""
    global _ref
    if _ref is None:
        L = ctypes.CDLL(str(REF_SO))
        L.kernels_select.argtypes = [ctypes.c_int]
        L.kernels_select.restype = ctypes.c_int
        L.k_quantize.argtypes = [_i8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.k_matmul_q8.argtypes = [_f32p, ctypes.POINTER(K8Input), K8Weight, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.k_gemm_q8_backend_test.argtypes = [ctypes.c_int, _i8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.POINTER(GemmQ8Segment), ctypes.c_int]
        L.k_gemm_q8_backend_test.restype = ctypes.c_int
        L.k_gemm_q8_amx_dots_test.argtypes = [_i32p, _i8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i8p, ctypes.c_int]
        L.k_gemm_q8_amx_dots_test.restype = ctypes.c_int
        L.s8_vnni_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.s8_vnni_bytes.restype = ctypes.c_size_t
        L.pack_s8_vnni.argtypes = [_i8p, _i8p, ctypes.c_int, ctypes.c_int, ctypes.c_size_t]
        L.gemm_amx_unavailable.restype = ctypes.c_char_p
        L.k_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
        L.kernels_init()
        _ref = L
    return _ref


def ref_select(isa):
    return bool(ref().kernels_select(isa))


def ref_amx_unavailable():
    """None when the reference's AMX-INT8 backend can run on this CPU, else the reason."""
    r = ref().gemm_amx_unavailable()
    return None if r is None else r.decode()


def ref_quantize(x, gs, isa=KERNELS_SCALAR):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.int8)
    s = np.empty(x.shape[0] // gs, np.float32)
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    ref().k_quantize(_p(q, _i8p), _p(s, _f32p), _p(x, _f32p), x.shape[0], gs)
    return q, s


def ref_gemv(xq, xs, wq, ws, gs, isa=KERNELS_SCALAR):
    xq = np.ascontiguousarray(xq, np.int8)
    xs = np.ascontiguousarray(xs, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, n = wq.shape
    out = np.empty(d, np.float32)
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    inp = K8Input(_p(xq, _i8p), _p(xs, _f32p), None)
    ref().k_matmul_q8(_p(out, _f32p), ctypes.byref(inp), K8Weight(_p(wq, _i8p), _p(ws, _f32p)), n, d, gs)
    return out


def ref_gemv_f32(x, wq, ws, gs, isa=KERNELS_AVX512):
    """The reference's k_matmul_q8 on fp32 activations (W8A32: K8Input.q NULL, f = x)."""
    x = np.ascontiguousarray(x, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, n = wq.shape
    out = np.empty(d, np.float32)
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    inp = K8Input(None, None, _p(x, _f32p))
    ref().k_matmul_q8(_p(out, _f32p), ctypes.byref(inp), K8Weight(_p(wq, _i8p), _p(ws, _f32p)), n, d, gs)
    ref_select(KERNELS_SCALAR)
    return out


def ref_gemm_amx(xq, xs, wq, ws, gs):
    """k_gemm_q8 on the AMX-INT8 backend (exact int32 group dots, src/gemm.c:554-610), STORE epilogue."""
    L = ref()
    if not ref_select(KERNELS_AMX):
        raise RuntimeError("AMX unavailable: %s" % ref_amx_unavailable())
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    m, k = xq.shape
    pad = np.zeros(((m + 31) // 32 * 32, k), np.int8)  # AMX reads activation rows up to a multiple of 32
    pad[:m] = xq
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    n = wq.shape[0]
    packed = np.zeros(L.s8_vnni_bytes(n, k), np.int8)
    L.pack_s8_vnni(_p(packed, _i8p), _p(wq, _i8p), n, k, k)
    c = np.zeros((m, n), np.float32)
    seg = GemmQ8Segment(_p(c, _f32p), n, K8Weight(_p(wq, _i8p), _p(ws, _f32p)), K8Weight(None, None),
                        _p(packed, _i8p), None, n, STORE)
    ok = L.k_gemm_q8_backend_test(Q8_GEMM_AMX, _p(pad, _i8p), _p(xs, _f32p), m, k, gs, ctypes.byref(seg), 1)
    if not ok:
        raise RuntimeError("AMX backend not compiled in")
    ref_select(KERNELS_SCALAR)
    return c


def ref_rmsnorm(x, w, eps, isa=KERNELS_AVX512):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    ref().k_rmsnorm(_p(out, _f32p), _p(x, _f32p), _p(w, _f32p), x.shape[0], eps)
    return out


def seeded_q8_matrix(rows, cols, gs, seed, std=0.02):
    """A W[rows][cols] ~ N(0, std) fp32 matrix (numpy PCG64 `seed`) quantized per row in gs-groups with k_quantize's
    rule (round half away from zero), the generator the benchmark configurations describe."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)).astype(np.float32)
    return quantize(w, gs)


def env_threads():
    return int(os.environ.get("LLAMA_THREADS", os.cpu_count() or 1))


class RefAttentionWork(ctypes.Structure):
    """The reference's AttentionWork (include/kernels.h:127-132)."""
    _fields_ = [("partial", ctypes.c_void_p), ("max_chunks", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("workers", ctypes.c_int), ("external", ctypes.c_int),
                ("capacity", ctypes.c_size_t)]


def ref_attention(q, key_cache, value_cache, n_heads, n_kv_heads, head_dim, seq_len, position, isa=KERNELS_AVX512):
    """The reference's decode attention on the head-major cache [n_kv][seq][hd] (k_attention_layout with
    pos_stride = head_dim, head_base = seq_len * head_dim, what k_attention_kv runs by default, src/attention.c:1434-1442),
    serial (no team)."""
    L = ref()
    L.k_attention_init.argtypes = [ctypes.POINTER(RefAttentionWork), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
    L.k_attention_free.argtypes = [ctypes.POINTER(RefAttentionWork)]
    L.k_attention_layout.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.POINTER(RefAttentionWork)] + \
        [ctypes.c_int] * 5 + [ctypes.c_size_t, ctypes.c_size_t]
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(key_cache, np.float32)
    vc = np.ascontiguousarray(value_cache, np.float32)
    out = np.zeros(n_heads * head_dim, np.float32)
    att = np.zeros(n_heads * seq_len, np.float32)
    work = RefAttentionWork()
    L.k_attention_init(ctypes.byref(work), n_heads, n_kv_heads, head_dim, seq_len)
    L.k_attention_layout(_p(out, _f32p), _p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), _p(att, _f32p),
                         ctypes.byref(work), n_heads, n_kv_heads, head_dim, seq_len, position, head_dim,
                         seq_len * head_dim)
    L.k_attention_free(ctypes.byref(work))
    ref_select(KERNELS_SCALAR)
    return out


def attention_limit(n_kv_heads, seq_len, workers=1):
    """attention_max_chunks (src/attention.c:527-530): the work's chunk limit for a team of `workers`."""
    return max((workers + n_kv_heads - 1) // n_kv_heads, (seq_len + 255) // 256)


def attention_decode(q, key_cache, value_cache, n_heads, n_kv_heads, head_dim, seq_len, position, workers=1):
    """The reference's split decode attention (orc_attention_decode) on the head-major cache [n_kv][seq][hd]."""
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(key_cache, np.float32)
    vc = np.ascontiguousarray(value_cache, np.float32)
    out = np.zeros(n_heads * head_dim, np.float32)
    rc = lib().orc_attention_decode(_p(out, _f32p), _p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), n_heads, n_kv_heads,
                                    head_dim, seq_len, position, workers,
                                    attention_limit(n_kv_heads, seq_len, workers))
    assert rc == 0
    return out


def attention_tiled(q, key_cache, value_cache, n_heads, n_kv_heads, head_dim, seq_len, pos0, m, workers=1):
    """The reference's default batched attention (orc_attention_tiled) for m > 1 rows at positions pos0.."""
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(key_cache, np.float32)
    vc = np.ascontiguousarray(value_cache, np.float32)
    out = np.zeros((m, n_heads * head_dim), np.float32)
    rc = lib().orc_attention_tiled(_p(out, _f32p), _p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), n_heads, n_kv_heads,
                                   head_dim, seq_len, pos0, m, workers, attention_limit(n_kv_heads, seq_len, workers))
    assert rc == 0
    return out


def ref_attention_batch(q, key_cache, value_cache, n_heads, n_kv_heads, head_dim, seq_len, pos0, m,
                        isa=KERNELS_AVX512):
    """The reference's batched attention (k_attention_batch_kv on its default head-major layout, src/attention.c:
    1444-1453), serial (no team), its default variant (tiled)."""
    L = ref()
    L.k_attention_init_rows.argtypes = [ctypes.POINTER(RefAttentionWork)] + [ctypes.c_int] * 5 + [_f32p]
    L.k_attention_free.argtypes = [ctypes.POINTER(RefAttentionWork)]
    L.k_attention_batch_kv.argtypes = [_f32p] * 5 + [ctypes.POINTER(RefAttentionWork)] + [ctypes.c_int] * 6
    if not ref_select(isa):
        raise RuntimeError("instruction set unavailable")
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(key_cache, np.float32)
    vc = np.ascontiguousarray(value_cache, np.float32)
    out = np.zeros((m, n_heads * head_dim), np.float32)
    att = np.zeros(n_heads * seq_len, np.float32)
    work = RefAttentionWork()
    L.k_attention_init_rows(ctypes.byref(work), n_heads, n_kv_heads, head_dim, seq_len, m, None)
    L.k_attention_batch_kv(_p(out, _f32p), _p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), _p(att, _f32p),
                           ctypes.byref(work), n_heads, n_kv_heads, head_dim, seq_len, pos0, m)
    L.k_attention_free(ctypes.byref(work))
    ref_select(KERNELS_SCALAR)
    return out
