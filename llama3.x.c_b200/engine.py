"""ctypes mirror of include/engine_cuda.h (the reference's engine API, include/runtime.h:98-116, on the GPU) and of the
device runtime shim include/device_cuda.h.

    from llama3x_b200 import engine
    m = engine.Engine.load("model.bin")            # engine_load_context
    logits = m.forward(token, pos)                  # engine_forward -> numpy copy of the model-owned logits
    tokens = m.generate(prompt, steps=64)           # engine_generate (greedy on the device)

Errors raise KernelError with the engine's message (the library runs in KC_FAIL_RETURN mode under Python).
"""
import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ENGINE_LIB_PATH = HERE / "libllama3x_engine.so"


class Config(ctypes.Structure):
    """include/runtime.h:9-17"""
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
                                             "seq_len", "format", "max_seq_len", "shared", "head_dim")] + \
               [(n, ctypes.c_float) for n in ("norm_eps", "rope_theta", "rope_factor", "rope_low", "rope_high")] + \
               [(n, ctypes.c_int) for n in ("rope_type", "rope_original", "bos_id", "eos_id", "eot_id", "eom_id")] + \
               [("name", ctypes.c_char * 128)]


class Model(ctypes.Structure):
    """include/runtime.h:86-97"""
    _fields_ = [("config", Config), ("implementation", ctypes.c_void_p), ("file_bytes", ctypes.c_size_t),
                ("mapped_bytes", ctypes.c_size_t), ("max_batch", ctypes.c_int), ("prefill_logits", ctypes.c_int),
                ("prefill_gemm", ctypes.c_int), ("prefill_kernel", ctypes.c_char_p), ("prefill_bf16", ctypes.c_int)]


class EngineStats(ctypes.Structure):
    """include/engine_cuda.h"""
    _fields_ = [("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double), ("prefill_tokens", ctypes.c_longlong),
                ("decode_tokens", ctypes.c_longlong), ("kernel_launches", ctypes.c_longlong)]


class KvStats(ctypes.Structure):
    """include/engine_cuda.h (the reference's KvStats, include/runtime.h:76-85)"""
    _fields_ = [("reserved_bytes", ctypes.c_size_t), ("active_bytes", ctypes.c_size_t),
                ("resident_bytes", ctypes.c_size_t), ("node", ctypes.c_int), ("verified", ctypes.c_int),
                ("full", ctypes.c_int), ("pages_queried", ctypes.c_size_t), ("pages_wrong_node", ctypes.c_size_t),
                ("pages_missing", ctypes.c_size_t)]


LOGITS_NONE, LOGITS_LAST, LOGITS_ALL = 0, 1, 2
COMM_ID_BYTES = 128

_c = ctypes
_MP = _c.POINTER(Model)
_IP = _c.POINTER(_c.c_int)
# Every symbol include/engine_cuda.h and include/device_cuda.h declare, with its ctypes signature.
ENGINE_SIGNATURES = {
    "engine_load": (None, [_MP, _c.c_char_p]),
    "engine_load_context": (None, [_MP, _c.c_char_p, _c.c_int]),
    "engine_forward": (_c.POINTER(_c.c_float), [_MP, _c.c_int, _c.c_int]),
    "engine_forward_batch": (_c.POINTER(_c.c_float), [_MP, _IP, _c.c_int, _c.c_int, _c.c_int]),
    "engine_max_batch": (_c.c_int, [_MP]),
    "engine_kv_stats": (None, [_MP, _c.c_int, _c.c_int, _c.POINTER(KvStats)]),
    "k_rope_table": (None, [_c.POINTER(Config), _c.c_int, _c.POINTER(_c.c_float)]),
    "engine_free": (None, [_MP]),
    "engine_precision": (_c.c_char_p, []),
    "engine_group_size": (_c.c_int, []),
    "engine_set_tp": (_c.c_int, [_c.c_int, _c.c_int, _c.c_int, _c.c_char_p]),
    "engine_init_random": (None, [_MP, _c.POINTER(Config), _c.c_int, _c.c_ulonglong, _c.c_int]),
    "engine_generate": (_c.c_int, [_MP, _IP, _c.c_int, _c.c_int, _IP]),
    "engine_save": (_c.c_int, [_MP, _c.c_char_p]),
    "engine_write_random": (_c.c_int, [_c.c_char_p, _c.POINTER(Config), _c.c_int, _c.c_ulonglong]),
    "engine_stream": (_c.c_void_p, [_MP]),
    "engine_reduction": (_c.c_char_p, [_MP]),
    "engine_stats": (None, [_MP, _c.POINTER(EngineStats)]),
    "engine_stats_reset": (None, [_MP]),
}
ENGINE_DATA = ["engine_q8"]
DEVICE_SIGNATURES = {
    "kd_device_count": (_c.c_int, []),
    "kd_set_device": (_c.c_int, [_c.c_int]),
    "kd_get_device": (_c.c_int, []),
    "kd_malloc": (_c.c_void_p, [_c.c_size_t]),
    "kd_free": (None, [_c.c_void_p]),
    "kd_host_alloc": (_c.c_void_p, [_c.c_size_t]),
    "kd_host_free": (None, [_c.c_void_p]),
    "kd_memset": (_c.c_int, [_c.c_void_p, _c.c_int, _c.c_size_t]),
    "kd_copy": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "kd_copy_2d": (_c.c_int, [_c.c_void_p, _c.c_size_t, _c.c_void_p, _c.c_size_t, _c.c_size_t, _c.c_size_t]),
    "kd_stream_create": (_c.c_void_p, []),
    "kd_stream_free": (None, [_c.c_void_p]),
    "kd_sync": (_c.c_int, []),
    "kd_capture_begin": (_c.c_int, []),
    "kd_capture_end": (_c.c_void_p, []),
    "kd_graph_launch": (_c.c_int, [_c.c_void_p]),
    "kd_graph_free": (None, [_c.c_void_p]),
    "kd_event_create": (_c.c_void_p, []),
    "kd_event_record": (_c.c_int, [_c.c_void_p]),
    "kd_event_ms": (_c.c_float, [_c.c_void_p, _c.c_void_p]),
    "kd_event_free": (None, [_c.c_void_p]),
    "kd_comm_unique_id": (_c.c_int, [_c.c_char_p]),
    "kd_comm_init": (_c.c_void_p, [_c.c_int, _c.c_int, _c.c_char_p]),
    "kd_allreduce_sum_f32": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "kd_allreduce_max_u64": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "kd_allgather_f32": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "kd_comm_free": (None, [_c.c_void_p]),
    "kd_peer_init": (_c.c_void_p, [_c.c_void_p, _c.c_int, _c.c_int, _c.c_size_t]),
    "kd_peer_allreduce_add": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "kd_peer_free": (None, [_c.c_void_p]),
    "kd_peer_matmul_q8_add": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                         _c.c_size_t, _c.c_int, _c.c_int, _c.c_int]),
    "kd_peer_test_absent": (_c.c_void_p, [_c.c_int, _c.c_size_t]),
}

_engine = None


def _kc():
    import importlib
    import sys
    mod = sys.modules.get("llama3x_b200")
    if mod is None:
        import importlib.util
        spec = importlib.util.spec_from_file_location("llama3x_b200", HERE / "__init__.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules["llama3x_b200"] = mod
        spec.loader.exec_module(mod)
    return mod


def load_library(path=ENGINE_LIB_PATH):
    """Loads libllama3x_engine.so (and through it libllama3x_cuda.so) and binds every declared symbol."""
    global _engine
    if _engine is None:
        kc = _kc()
        kc.load().kc_set_fail_mode(kc.KC_FAIL_RETURN)
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in {**ENGINE_SIGNATURES, **DEVICE_SIGNATURES}.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _engine = lib
    return _engine


def _check():
    kc = _kc()
    msg = kc._lib.kc_last_error()
    if msg:
        kc._lib.kc_clear_error()
        raise kc.KernelError(msg.decode())


def _ints(values):
    a = (ctypes.c_int * len(values))(*[int(v) for v in values])
    return a


def comm_unique_id():
    """kd_comm_unique_id: the 128-byte NCCL id rank 0 hands to every rank."""
    lib = load_library()
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    if lib.kd_comm_unique_id(buf) != 0:
        _check()
    return buf.raw


class Engine:
    """One loaded (or random-initialized) model on this process's GPU; engine_free on close()."""

    def __init__(self):
        self.lib = load_library()
        self.model = Model()
        self._m = ctypes.byref(self.model)

    @staticmethod
    def _prepare(tp):
        """Selects the rank's device before anything touches CUDA, then kernels_init and engine_set_tp."""
        lib = load_library()
        if tp is not None:
            if lib.kd_set_device(int(tp[2])) != 0:
                _check()
        _kc().init()
        if tp is not None:
            rank, world, device, nccl_id = tp
            if lib.engine_set_tp(rank, world, device, nccl_id) != 0:
                _check()

    @classmethod
    def load(cls, path, context=0, tp=None):
        """engine_load_context; tp = (rank, world, device, nccl_id) for tensor parallelism."""
        cls._prepare(tp)
        self = cls()
        self.lib.engine_load_context(self._m, os.fsencode(str(path)), context)
        _check()
        if not self.model.implementation:
            raise _kc().KernelError("engine_load_context failed")
        return self

    @classmethod
    def random(cls, dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, group_size=64, seed=0,
               shared=False, context=0, tp=None):
        """engine_init_random: the seeded random-init model of that architecture, device-resident."""
        cls._prepare(tp)
        self = cls()
        cfg = Config()
        for k, v in dict(dim=dim, hidden_dim=hidden_dim, n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv_heads,
                         vocab_size=vocab_size, seq_len=seq_len, shared=int(bool(shared))).items():
            setattr(cfg, k, v)
        self.lib.engine_init_random(self._m, ctypes.byref(cfg), group_size, seed, context)
        _check()
        if not self.model.implementation:
            raise _kc().KernelError("engine_init_random failed")
        return self

    @property
    def config(self):
        return self.model.config

    @property
    def max_batch(self):
        return self.lib.engine_max_batch(self._m)

    @property
    def stream(self):
        return self.lib.engine_stream(self._m)

    def forward(self, token, position):
        p = self.lib.engine_forward(self._m, int(token), int(position))
        _check()
        if not p:
            raise _kc().KernelError("engine_forward failed")
        return np.ctypeslib.as_array(p, (self.config.vocab_size,)).copy()

    def forward_view(self, token, position):
        """engine_forward with the reference's contract kept: a view of the engine's own host logits, valid until the
        next call on this model (forward() returns a copy instead)."""
        p = self.lib.engine_forward(self._m, int(token), int(position))
        _check()
        if not p:
            raise _kc().KernelError("engine_forward failed")
        return np.ctypeslib.as_array(p, (self.config.vocab_size,))

    def forward_batch(self, tokens, pos0, want=LOGITS_LAST):
        arr = _ints(tokens)
        p = self.lib.engine_forward_batch(self._m, arr, len(tokens), int(pos0), want)
        _check()
        V = self.config.vocab_size
        if want == LOGITS_NONE:
            return None
        if not p:
            raise _kc().KernelError("engine_forward_batch failed")
        rows = len(tokens) if want == LOGITS_ALL else 1
        out = np.ctypeslib.as_array(p, (rows * V,)).copy().reshape(rows, V)
        return out if want == LOGITS_ALL else out[0]

    def generate(self, prompt, steps):
        out = (ctypes.c_int * steps)()
        n = self.lib.engine_generate(self._m, _ints(prompt), len(prompt), steps, out)
        _check()
        if n < 0:
            raise _kc().KernelError("engine_generate failed")
        return list(out[:n])

    def stats(self):
        st = EngineStats()
        self.lib.engine_stats(self._m, ctypes.byref(st))
        return {f: getattr(st, f) for f, _ in EngineStats._fields_}

    def stats_reset(self):
        self.lib.engine_stats_reset(self._m)

    def reduction(self):
        """engine_reduction: how the decode step joins the Wo/W2 shards (none, peer_gemv, peer_kernel or nccl)."""
        return self.lib.engine_reduction(self._m).decode()

    def kv_stats(self, position, verify=0):
        """engine_kv_stats: the K/V cache accounting of the reference's report (include/runtime.h:111-113)."""
        st = KvStats()
        self.lib.engine_kv_stats(self._m, position, verify, ctypes.byref(st))
        _check()
        return {f: getattr(st, f) for f, _ in KvStats._fields_}

    def save(self, path):
        if self.lib.engine_save(self._m, os.fsencode(str(path))) != 0:
            _check()

    def close(self):
        if self.model.implementation:
            self.lib.engine_free(self._m)
            _check()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def write_random(path, dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, shared=False,
                 group_size=64, seed=1):
    """engine_write_random: the seeded random-init checkpoint of this architecture at `path` (returns the path)."""
    c = Config(dim=dim, hidden_dim=hidden_dim, n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv_heads,
               vocab_size=vocab_size, seq_len=seq_len, shared=int(shared))
    if load_library().engine_write_random(os.fsencode(str(path)), ctypes.byref(c), group_size, seed) != 0:
        _check()
        raise _kc().KernelError("engine_write_random failed")
    return path


def rope_table(config, position):
    """k_rope_table (include/kernels.h:67) for `config` (a Config) at `position`: 2 * head_dim floats."""
    import numpy as np
    out = np.zeros(2 * config.head_dim, np.float32)
    load_library().k_rope_table(ctypes.byref(config), position, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def share_comm_id(rank, world):
    """Rank 0 makes the NCCL id and broadcasts it over torch.distributed's default group (any backend); every rank
    returns the same 128 bytes for Engine.load / Engine.random(tp=(rank, world, device, id))."""
    import torch.distributed as dist
    obj = [comm_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(obj, src=0)
    return obj[0]
