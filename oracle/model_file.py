"""TEST / BASELINE INFRASTRUCTURE: writes seeded benchmark-size Q8_0 checkpoints (the reference's version 2 format,
src/runtime.c:179-310, tensor order src/shards.c:80-97) for the reference's CPU engine, with the oracle's C generator
(orc_random_q8: N(0, std) weights quantized by k_quantize's rule) on every host core. RMSNorm weights are 1.

Only bench.py's CPU-baseline leg and its --impl reference arm use this, to give the reference's engine the model
architecture the GPU engine runs.
"""
import ctypes
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from . import oracle as O


def _lib():
    L = O.lib()
    L.orc_random_q8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
    L.orc_random_q8.restype = None
    return L


def random_q8(rows, cols, gs, seed, tensor, std=0.02, threads=None):
    L = _lib()
    q = np.empty((rows, cols), np.int8)
    s = np.empty((rows, cols // gs), np.float32)
    threads = threads or os.cpu_count() or 1
    step = max(1, -(-rows // (threads * 4)))

    def block(r0):
        n = min(step, rows - r0)
        L.orc_random_q8(q[r0:].ctypes.data, s[r0:].ctypes.data, r0, n, cols, gs, seed, tensor, std)

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(block, range(0, rows, step)))
    return q, s


def write_random_checkpoint(path, dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, shared=False,
                            gs=64, seed=1):
    """Writes the checkpoint unless `path` already holds one of exactly the expected size; returns the path."""
    path = Path(path)
    d, h, L, V = dim, hidden_dim, n_layers, vocab_size
    kv = d // n_heads * n_kv_heads

    def q8_bytes(n):
        return n + n // gs * 4

    size = 256 + (2 * L + 1) * d * 4 + q8_bytes(V * d) * (1 if shared else 2) + \
        L * (2 * q8_bytes(d * d) + 2 * q8_bytes(d * kv) + 3 * q8_bytes(d * h))
    if path.exists() and path.stat().st_size == size:
        return path
    tmp = path.with_suffix(".tmp")
    with open(tmp, "wb") as f:
        header = struct.pack("<Ii7iBi", 0x616B3432, 2, d, h, L, n_heads, n_kv_heads, V, seq_len, int(shared), gs)
        f.write(header + bytes(256 - len(header)))
        f.write(np.ones((2 * L + 1) * d, np.float32).tobytes())

        def put(rows, cols, tensor):
            q, s = random_q8(rows, cols, gs, seed, tensor)
            f.write(q.tobytes())
            f.write(s.tobytes())

        put(V, d, 0)
        shapes = [(d, d), (kv, d), (kv, d), (d, d), (h, d), (d, h), (h, d)]
        for role, (rows, cols) in enumerate(shapes):
            for layer in range(L):
                put(rows, cols, 2 + 7 * layer + role)
        if not shared:
            put(V, d, 1)
    os.replace(tmp, path)
    return path
