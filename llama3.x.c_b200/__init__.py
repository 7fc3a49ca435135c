"""Host-side mirror of llama3.x.c's Q8_0 W8A8 kernel API on the sm_100a library (libllama3x_cuda.so).

The functions keep the reference's names, argument meaning and error behaviour (include/kernels.h, include/gemm.h of
LucianCrainic/llama3.x.c); tensors are CUDA tensors whose device pointers go straight through the C-ABI declared in
include/kernels_cuda.h. PyTorch only supplies device memory and the current stream. There is no CPU fallback: without
the built library every call raises.

The directory name has dots, so load it as a module by path::

    from importlib.util import spec_from_file_location, module_from_spec
    spec = spec_from_file_location("llama3x_b200", "llama3.x.c_b200/__init__.py",
                                   submodule_search_locations=["llama3.x.c_b200"])
"""
import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libllama3x_cuda.so"

K_STORE, K_ADD, K_PARTIAL, K_SWIGLU = 0, 1, 2, 3            # include/kernels.h:84
GEMM_STORE, GEMM_ADD, GEMM_SWIGLU, GEMM_PARTIAL = 0, 1, 2, 3  # include/gemm.h:15-20
Q8_GEMM_PORTABLE, Q8_GEMM_AVX512, Q8_GEMM_AMX = 0, 1, 2
Q8_GEMM_GPU_DP4A, Q8_GEMM_GPU_TCGEN05 = 16, 17
KC_FAIL_EXIT, KC_FAIL_RETURN = 0, 1

_i8p = ctypes.c_void_p
_f32p = ctypes.c_void_p


class K8Weight(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("s", ctypes.c_void_p)]


class K8Input(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("f", ctypes.c_void_p)]


class GemmQ8Segment(ctypes.Structure):
    _fields_ = [("c", ctypes.c_void_p), ("ldc", ctypes.c_int), ("w", K8Weight), ("w3", K8Weight),
                ("pw", ctypes.c_void_p), ("pw3", ctypes.c_void_p), ("n", ctypes.c_int), ("kind", ctypes.c_int)]


class KernelTail(ctypes.Structure):
    """include/kernels_cuda.h: work the decode GEMV's last CTA does once."""
    _fields_ = [("kind", ctypes.c_int), ("x", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("epsilon", ctypes.c_float),
                ("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("n", ctypes.c_int), ("rope_table", ctypes.c_void_p),
                ("position", ctypes.c_void_p), ("key_cache", ctypes.c_void_p), ("value_cache", ctypes.c_void_p),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("seq_len", ctypes.c_int)]


K_TAIL_NONE, K_TAIL_QUANTIZE, K_TAIL_NORM_QUANTIZE, K_TAIL_ROPE_KV_STORE, K_TAIL_QUANTIZE_OUTPUT = 0, 1, 2, 3, 4


class AttentionWork(ctypes.Structure):
    """include/kernels_cuda.h: split-K partials in device memory, in the reference's layout
    (include/kernels.h:127-132)."""
    _fields_ = [("partial", ctypes.c_void_p), ("max_chunks", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("workers", ctypes.c_int), ("external", ctypes.c_int),
                ("capacity", ctypes.c_size_t)]


# Every symbol include/kernels_cuda.h declares, with its ctypes signature (restype, argtypes).
_c = ctypes
_SIGNATURES = {
    "kernels_init": (None, []),
    "kernels_name": (_c.c_char_p, []),
    "kernels_set_stream": (None, [_c.c_void_p]),
    "kernels_set_pdl": (None, [_c.c_int]),
    "kc_set_fail_mode": (None, [_c.c_int]),
    "kc_last_error": (_c.c_char_p, []),
    "kc_clear_error": (None, []),
    "kc_status": (_c.c_int, []),
    "k_quantize": (None, [_i8p, _f32p, _f32p, _c.c_int, _c.c_int]),
    "k_quantize_rows": (None, [_i8p, _f32p, _f32p, _c.c_size_t, _c.c_int, _c.c_int, _c.c_int]),
    "k_matmul_q8": (None, [_f32p, _c.POINTER(K8Input), K8Weight, _c.c_int, _c.c_int, _c.c_int]),
    "k_matmul_q8_add": (None, [_f32p, _c.POINTER(K8Input), K8Weight, _c.c_int, _c.c_int, _c.c_int]),
    "k_matmul_q8_qkv": (None, [_f32p, _f32p, _f32p, _c.POINTER(K8Input), K8Weight, K8Weight, K8Weight, _c.c_int,
                               _c.c_int, _c.c_int, _c.c_int]),
    "k_matmul_q8_swiglu": (None, [_f32p, _c.POINTER(K8Input), K8Weight, K8Weight, _c.c_int, _c.c_int, _c.c_int]),
    "k_matmul_q8_ld": (None, [_f32p, _c.POINTER(K8Input), _c.POINTER(K8Weight), _c.c_size_t, _c.c_int, _c.c_int,
                              _c.c_int, _c.c_int]),
    "k_matmul_q8_swiglu_ld": (None, [_f32p, _c.POINTER(K8Input), _c.POINTER(K8Weight), _c.POINTER(K8Weight),
                                     _c.c_size_t, _c.c_int, _c.c_int, _c.c_int]),
    "k_gemm_q8": (None, [_i8p, _f32p, _c.c_int, _c.c_int, _c.c_int, _c.POINTER(GemmQ8Segment), _c.c_int]),
    "k_matmul_q8_ld_worker": (None, [_f32p, _c.POINTER(K8Input), _c.POINTER(K8Weight), _c.c_size_t, _c.c_int,
                                     _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p,
                                     _c.c_void_p]),
    "kernels_backend_init": (None, []),
    "kernels_backend_free": (None, []),
    "s8_vnni_bytes": (_c.c_size_t, [_c.c_int, _c.c_int]),
    "pack_s8_vnni": (None, [_i8p, _i8p, _c.c_int, _c.c_int, _c.c_size_t]),
    "pack_s8_vnni_tiles": (None, [_i8p, _i8p, _c.c_int, _c.c_int, _c.c_size_t, _c.c_int, _c.c_int]),
    "pack_s8_vnni_many": (None, [_c.c_void_p, _c.c_int]),
    "k_matmul_q8_fused": (None, [_f32p, _f32p, _c.c_float, _c.c_size_t, _c.c_int, _c.c_int,
                                 _c.POINTER(GemmQ8Segment), _c.c_int, _c.c_void_p]),
    "k_matmul_q8_tail": (None, [_c.POINTER(K8Input), _c.c_size_t, _c.c_int, _c.c_int, _c.POINTER(GemmQ8Segment),
                                _c.c_int, _c.POINTER(KernelTail)]),
    "k_gemm_q8_pick": (_c.c_int, [_c.c_int, _c.POINTER(GemmQ8Segment), _c.c_int]),
    "k_gemm_q8_backend_test": (_c.c_int, [_c.c_int, _i8p, _f32p, _c.c_int, _c.c_int, _c.c_int,
                                          _c.POINTER(GemmQ8Segment), _c.c_int]),
    "k_gemm_q8_dots_test": (_c.c_int, [_c.c_void_p, _i8p, _c.c_int, _c.c_int, _c.c_int, _i8p, _c.c_int]),
    "k_gemm_q8_noalloc": (_c.c_int, [_i8p, _f32p, _c.c_int, _c.c_int, _c.c_int, _c.POINTER(GemmQ8Segment),
                                     _c.c_int]),
    "k_rmsnorm": (None, [_f32p, _f32p, _f32p, _c.c_int, _c.c_float]),
    "k_rmsnorm_rows": (None, [_f32p, _f32p, _f32p, _c.c_int, _c.c_int, _c.c_float]),
    "k_rmsnorm_q8_rows": (None, [_i8p, _f32p, _f32p, _f32p, _c.c_size_t, _f32p, _c.c_int, _c.c_int, _c.c_float,
                                 _c.c_int]),
    "k_rope_apply": (None, [_f32p, _f32p, _f32p, _c.c_int, _c.c_int, _c.c_int]),
    "k_rope_apply_rows": (None, [_f32p, _c.c_size_t, _f32p, _c.c_size_t, _f32p, _c.c_size_t, _c.c_int, _c.c_int,
                                 _c.c_int, _c.c_int]),
    "kc_fail_message": (None, [_c.c_char_p]),
    "kc_launch_count": (_c.c_ulonglong, []),
    "k_kv_strides": (None, [_c.c_int, _c.c_int, _c.c_int, _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t)]),
    "k_kv_store": (None, [_f32p, _f32p, _c.c_size_t, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_attention_bytes_rows": (_c.c_size_t, [_c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_attention_init_rows": (None, [_c.POINTER(AttentionWork), _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int,
                                     _c.c_void_p]),
    "k_attention_free": (None, [_c.POINTER(AttentionWork)]),
    "k_attention_kv": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _c.POINTER(AttentionWork), _c.c_int, _c.c_int,
                              _c.c_int, _c.c_int, _c.c_int]),
    "k_attention_batch_kv": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _c.POINTER(AttentionWork), _c.c_int,
                                    _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_rope_kv_store_rows": (None, [_f32p, _c.c_size_t, _f32p, _f32p, _c.c_size_t, _f32p, _f32p, _f32p, _c.c_void_p,
                                    _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_attention_q8_rows": (None, [_f32p, _i8p, _f32p, _f32p, _f32p, _f32p, _c.POINTER(AttentionWork), _c.c_int,
                                   _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_int, _c.c_int, _c.c_int]),
    "k_rope_attention_q8_step_ok": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_rope_attention_q8_step": (None, [_f32p, _i8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                        _c.POINTER(AttentionWork), _c.c_int, _c.c_int, _c.c_int, _c.c_int,
                                        _c.c_void_p, _c.c_int]),
    "k_embed_q8_rows": (None, [_f32p, _c.c_void_p, K8Weight, _c.c_int, _c.c_int, _c.c_int, _c.c_int]),
    "k_add": (None, [_f32p, _f32p, _c.c_size_t]),
    "k_argmax_key": (None, [_c.c_void_p, _f32p, _c.c_int, _c.c_int]),
    "k_greedy_advance": (None, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "k_random_q8": (None, [_i8p, _f32p, _c.c_int, _c.c_int, _c.c_size_t, _c.c_size_t, _c.c_size_t, _c.c_ulonglong,
                           _c.c_ulonglong, _c.c_float, _c.c_int]),
    "k_fill": (None, [_f32p, _c.c_size_t, _c.c_float]),
}


class KernelError(RuntimeError):
    """What the reference reports through fail(): raised here instead of exiting (KC_FAIL_RETURN mode)."""


_lib = None


def load(path=LIB_PATH):
    """Loads the library and binds every declared symbol; raises if it is missing (there is no fallback)."""
    global _lib
    if _lib is None:
        if not Path(path).exists():
            raise RuntimeError(f"{path} is not built: run llama3.x.c_b200/build.py (no CPU fallback exists)")
        L = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGNATURES)


_ready = False


def init():
    """kernels_init on the current device, with errors raised as KernelError rather than exiting."""
    global _ready
    L = load()
    if not _ready:
        L.kc_set_fail_mode(KC_FAIL_RETURN)
        L.kernels_init()
        _check_host()
        _ready = True
    return L


def _check_host():
    msg = _lib.kc_last_error()
    if msg:
        _lib.kc_clear_error()
        raise KernelError(msg.decode())


def _stream():
    import torch
    load().kernels_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _call(name, *args):
    L = init()
    _stream()
    r = getattr(L, name)(*args)
    _check_host()
    return r


def status():
    """kc_status: waits for the stream, raises KernelError if a kernel flagged an error."""
    L = init()
    _stream()
    bits = L.kc_status()
    _check_host()
    return bits


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _weight(q, s):
    return K8Weight(_ptr(q), _ptr(s))


# ---- the reference-named entry points (device tensors) --------------------------------------------------------------

def k_quantize(q, s, x, n, gs):
    _call("k_quantize", _ptr(q), _ptr(s), _ptr(x), n, gs)


def k_quantize_rows(q, s, x, ldx, m, n, gs):
    _call("k_quantize_rows", _ptr(q), _ptr(s), _ptr(x), ldx, m, n, gs)


def _input(xq, xs):
    """K8Input: int8 values xq and scales xs (W8A8), or fp32 activations in xq with xs None (W8A32: q NULL, f set)."""
    if xs is None and xq is not None and str(getattr(xq, "dtype", "")) in ("torch.float32", "float32"):
        return K8Input(None, None, _ptr(xq))
    return K8Input(_ptr(xq), _ptr(xs), None)


def k_matmul_q8(out, xq, xs, wq, ws, n, d, gs):
    inp = _input(xq, xs)
    _call("k_matmul_q8", _ptr(out), ctypes.byref(inp), _weight(wq, ws), n, d, gs)


def k_matmul_q8_add(out, xq, xs, wq, ws, n, d, gs):
    inp = _input(xq, xs)
    _call("k_matmul_q8_add", _ptr(out), ctypes.byref(inp), _weight(wq, ws), n, d, gs)


def k_matmul_q8_qkv(q, k, v, xq, xs, wq, wk, wv, n, dq, dkv, gs):
    inp = _input(xq, xs)
    _call("k_matmul_q8_qkv", _ptr(q), _ptr(k), _ptr(v), ctypes.byref(inp), _weight(*wq), _weight(*wk),
          _weight(*wv), n, dq, dkv, gs)


def k_matmul_q8_swiglu(out, xq, xs, w1, w3, n, d, gs):
    inp = _input(xq, xs)
    _call("k_matmul_q8_swiglu", _ptr(out), ctypes.byref(inp), _weight(*w1), _weight(*w3), n, d, gs)


def k_matmul_q8_ld(out, xq, xs, wq, ws, ld, n, d, gs, kind):
    inp = _input(xq, xs)
    w = _weight(wq, ws)
    _call("k_matmul_q8_ld", _ptr(out), ctypes.byref(inp), ctypes.byref(w), ld, n, d, gs, kind)


def k_matmul_q8_swiglu_ld(out, xq, xs, w1, w3, ld, n, d, gs):
    inp = _input(xq, xs)
    a, b = _weight(*w1), _weight(*w3)
    _call("k_matmul_q8_swiglu_ld", _ptr(out), ctypes.byref(inp), ctypes.byref(a), ctypes.byref(b), ld, n, d, gs)


def segment(c, w, kind=GEMM_STORE, w3=None, ldc=None):
    """A GemmQ8Segment for k_gemm_q8: c [m][n] float32 (row stride ldc), w = (wq [n][k], ws [n][k/gs])."""
    n = w[0].shape[0]
    seg = GemmQ8Segment(_ptr(c), ldc if ldc is not None else c.stride(0), _weight(*w),
                        _weight(*w3) if w3 is not None else K8Weight(None, None), None, None, n, kind)
    seg._tensors = (c, w, w3)  # the struct holds raw pointers: keep the device memory alive with it
    return seg


def _segments(segs):
    arr = (GemmQ8Segment * len(segs))(*segs)
    return arr, len(segs)


def k_gemm_q8(xq, xs, m, k, gs, segs):
    arr, count = _segments(segs)
    _call("k_gemm_q8", _ptr(xq), _ptr(xs), m, k, gs, arr, count)


def k_matmul_q8_fused(x, weight, eps, ld, n, gs, segs, tail=None):
    """The decode GEMV on fp32 activations: RMSNorm (weight not None) + quantize inside the kernel; `tail` an optional
    KernelTail."""
    arr, count = _segments(segs)
    _call("k_matmul_q8_fused", _ptr(x), _ptr(weight), eps, ld, n, gs, arr, count,
          ctypes.addressof(tail) if tail is not None else None)


def k_matmul_q8_tail(xq, xs, ld, n, gs, segs, tail):
    """The decode GEMV on int8 input, then `tail` (a KernelTail) done once by its last CTA."""
    arr, count = _segments(segs)
    inp = _input(xq, xs)
    _call("k_matmul_q8_tail", ctypes.byref(inp), ld, n, gs, arr, count, ctypes.byref(tail))


ROWS_DONE = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.c_int)


def k_matmul_q8_ld_worker(out, xq, xs, wq, ws, ld, n, d, gs, kind, worker, workers, done=None):
    """Member `worker` of `workers`' share of k_matmul_q8_ld; done(r0, r1) once its rows are in memory."""
    inp = _input(xq, xs)
    w = _weight(wq, ws)
    cb = ROWS_DONE(lambda ctx, r0, r1: done(r0, r1)) if done else None
    _call("k_matmul_q8_ld_worker", _ptr(out), ctypes.byref(inp), ctypes.byref(w), ld, n, d, gs, kind, worker, workers,
          None, ctypes.cast(cb, ctypes.c_void_p) if cb else None, None)


def pack_s8_vnni(w, rows, cols, ld):
    """The reference's AMX tile layout of an int8 matrix (host numpy array in, host numpy array out)."""
    import numpy as np
    L = load()  # host code: no device needed
    out = np.zeros(L.s8_vnni_bytes(rows, cols), np.int8)
    w = np.ascontiguousarray(w, np.int8)
    L.pack_s8_vnni(out.ctypes.data_as(ctypes.c_void_p), w.ctypes.data_as(ctypes.c_void_p), rows, cols, ld)
    return out


def k_gemm_q8_pick(gs, segs):
    arr, count = _segments(segs)
    return _call("k_gemm_q8_pick", gs, arr, count)


def k_gemm_q8_backend_test(backend, xq, xs, m, k, gs, segs):
    arr, count = _segments(segs)
    return _call("k_gemm_q8_backend_test", backend, _ptr(xq), _ptr(xs), m, k, gs, arr, count)


def k_gemm_q8_dots_test(dots, xq, m, k, gs, wq, n):
    return _call("k_gemm_q8_dots_test", _ptr(dots), _ptr(xq), m, k, gs, _ptr(wq), n)


def k_gemm_q8_noalloc(xq, xs, m, k, gs, segs):
    """k_gemm_q8 with its scale scratch in the library's fixed device array; raises KernelError when rejected."""
    arr, count = _segments(segs)
    if _call("k_gemm_q8_noalloc", _ptr(xq), _ptr(xs), m, k, gs, arr, count) != 0:
        raise KernelError("k_gemm_q8_noalloc rejected its arguments")


def k_rmsnorm(out, x, weight, size, eps):
    _call("k_rmsnorm", _ptr(out), _ptr(x), _ptr(weight), size, eps)


def k_rmsnorm_rows(out, x, weight, rows, size, eps):
    _call("k_rmsnorm_rows", _ptr(out), _ptr(x), _ptr(weight), rows, size, eps)


def k_rmsnorm_q8_rows(q, s, out, x, ldx, weight, rows, size, eps, gs):
    _call("k_rmsnorm_q8_rows", _ptr(q), _ptr(s), _ptr(out), _ptr(x), ldx, _ptr(weight), rows, size, eps, gs)


def k_rope_apply_rows(q, q_stride, k, k_stride, table, table_stride, rows, n_heads, n_kv_heads, head_dim):
    _call("k_rope_apply_rows", _ptr(q), q_stride, _ptr(k), k_stride, _ptr(table), table_stride, rows, n_heads,
          n_kv_heads, head_dim)


# ---- conveniences over the entry points (allocate outputs with torch) -----------------------------------------------

def quantize(x, gs):
    """k_quantize_rows over the last axis of a CUDA float32 tensor -> (int8 values, float32 scales)."""
    import torch
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    q = torch.empty(rows.shape, dtype=torch.int8, device=x.device)
    s = torch.empty((rows.shape[0], n // gs), dtype=torch.float32, device=x.device)
    k_quantize_rows(q, s, rows, rows.stride(0), rows.shape[0], n, gs)
    return q.reshape(x.shape), s.reshape(x.shape[:-1] + (n // gs,))


def gemv(xq, xs, wq, ws, gs, kind=K_STORE, out=None, w3=None):
    """One activation row against W [d][n]: the k_matmul_q8 family."""
    import torch
    d, n = wq.shape
    if out is None:
        out = torch.zeros(d, dtype=torch.float32, device=wq.device)
    if kind == K_SWIGLU:
        k_matmul_q8_swiglu(out, xq, xs, (wq, ws), w3, n, d, gs)
    elif kind == K_ADD:
        k_matmul_q8_add(out, xq, xs, wq, ws, n, d, gs)
    else:
        k_matmul_q8_ld(out, xq, xs, wq, ws, n, n, d, gs, kind)
    return out


def gemm(xq, xs, wq, ws, gs, kind=GEMM_STORE, c=None, w3=None, backend=None):
    """C[m][n] (op)= Xq . Wq^T through k_gemm_q8 (or one named backend)."""
    import torch
    m, k = xq.shape
    n = wq.shape[0]
    if c is None:
        c = torch.zeros((m, n), dtype=torch.float32, device=wq.device)
    seg = segment(c, (wq, ws), kind, w3)
    if backend is None:
        k_gemm_q8(xq, xs, m, k, gs, [seg])
    elif not k_gemm_q8_backend_test(backend, xq, xs, m, k, gs, [seg]):
        raise KernelError(f"backend {backend} is not compiled in")
    return c


# ---- engine kernels (device tensors in, nothing allocated here) ------------------------------------------------------

def attention_work(n_heads, n_kv_heads, head_dim, seq_len, rows=1):
    """k_attention_init_rows with library-allocated device memory; release with k_attention_free."""
    w = AttentionWork()
    _call("k_attention_init_rows", ctypes.byref(w), n_heads, n_kv_heads, head_dim, seq_len, rows, None)
    return w


def k_attention_free(work):
    _call("k_attention_free", ctypes.byref(work))


def k_attention_kv(out, q, kc, vc, work, n_heads, n_kv_heads, head_dim, seq_len, position):
    _call("k_attention_kv", _ptr(out), _ptr(q), _ptr(kc), _ptr(vc), None, ctypes.byref(work), n_heads, n_kv_heads,
          head_dim, seq_len, position)


def k_attention_batch_kv(out, q, kc, vc, work, n_heads, n_kv_heads, head_dim, seq_len, pos0, m):
    _call("k_attention_batch_kv", _ptr(out), _ptr(q), _ptr(kc), _ptr(vc), None, ctypes.byref(work), n_heads,
          n_kv_heads, head_dim, seq_len, pos0, m)


def k_attention_q8_rows(out, oq, os_, q, kc, vc, work, n_heads, n_kv_heads, head_dim, seq_len, position, pos0, rows,
                        gs):
    _call("k_attention_q8_rows", _ptr(out), _ptr(oq), _ptr(os_), _ptr(q), _ptr(kc), _ptr(vc), ctypes.byref(work),
          n_heads, n_kv_heads, head_dim, seq_len, _ptr(position) if position is not None else None, pos0, rows, gs)


def k_rope_attention_q8_step_ok(n_heads, n_kv_heads, head_dim, gs):
    return int(load().k_rope_attention_q8_step_ok(n_heads, n_kv_heads, head_dim, gs))


def k_rope_attention_q8_step(out, oq, os_, q, k, v, kc, vc, table, work, n_heads, n_kv_heads, head_dim, seq_len,
                             position, gs):
    _call("k_rope_attention_q8_step", _ptr(out), _ptr(oq), _ptr(os_), _ptr(q), _ptr(k), _ptr(v), _ptr(kc), _ptr(vc),
          _ptr(table), ctypes.byref(work), n_heads, n_kv_heads, head_dim, seq_len, _ptr(position), gs)


def k_kv_store(cache, src, src_ld, pos0, count, n_kv_heads, head_dim, seq_len):
    _call("k_kv_store", _ptr(cache), _ptr(src), src_ld, pos0, count, n_kv_heads, head_dim, seq_len)


def k_rope_kv_store_rows(q, q_ld, k, v, kv_ld, kc, vc, table, position, pos0, rows, n_heads, n_kv_heads, head_dim,
                         seq_len):
    _call("k_rope_kv_store_rows", _ptr(q), q_ld, _ptr(k), _ptr(v), kv_ld, _ptr(kc), _ptr(vc), _ptr(table),
          _ptr(position) if position is not None else None, pos0, rows, n_heads, n_kv_heads, head_dim, seq_len)


def k_embed_q8_rows(x, tokens, embed, rows, dim, gs, vocab):
    _call("k_embed_q8_rows", _ptr(x), _ptr(tokens), K8Weight(_ptr(embed[0]), _ptr(embed[1])), rows, dim, gs, vocab)


def k_argmax_key(key, logits, n, offset):
    _call("k_argmax_key", _ptr(key), _ptr(logits), n, offset)


def k_greedy_advance(out, step, token, position, key):
    _call("k_greedy_advance", _ptr(out), _ptr(step), _ptr(token), _ptr(position), _ptr(key))


def k_random_q8(q, s, rows, cols, row0, col0, full_cols, seed, tensor, std, gs):
    _call("k_random_q8", _ptr(q), _ptr(s), rows, cols, row0, col0, full_cols, seed, tensor, std, gs)
