"""Seeded Q8_0 checkpoints for the engine tests (test infrastructure).

write_model(path, name) writes a version 2 Q8_0 checkpoint (the reference's format, src/runtime.c:179-310, tensor
order src/shards.c:80-97) whose weights are numpy PCG64 N(0, 0.02) draws quantized with k_quantize's rule by the
oracle, RMSNorm weights 1 + N(0, 0.05) so the norm multiply is exercised. The embedding rows are N(0, 1): with the
benchmark's N(0, 0.02) embeddings the residual stream is so small that one int8 rounding step of an activation moves
the logits by ~1%, and the reference's own kernel selections (scalar, AVX-512, AMX) then disagree on greedy tokens
after a few dozen steps; a residual dominated by the embedding keeps the models far less chaotic. The same bytes come out on any machine, so
the GPU tests regenerate the files the golden outputs were computed from.

The three shapes cover: tiny -- tied classifier, small head dim; small -- untied classifier, 8 KV heads (tensor
parallel up to 8 GPUs); wide -- head_dim 128 with 4 query heads per KV head (the 8B geometry) and a context long enough
for several attention splits.
"""
import struct
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

GS = 64
MODELS = {
    "tiny": dict(dim=256, hidden_dim=512, n_layers=2, n_heads=8, n_kv_heads=4, vocab_size=512, seq_len=256, shared=1,
                 seed=11, embed_std=1.0),
    "small": dict(dim=512, hidden_dim=1536, n_layers=3, n_heads=16, n_kv_heads=8, vocab_size=2048, seq_len=512,
                  shared=0, seed=12, embed_std=1.0),
    "wide": dict(dim=1024, hidden_dim=2048, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=1024, seq_len=1024,
                 shared=0, seed=13, embed_std=1.0),
}


def _q8(f, rows, cols, seed, std=0.02):
    q, s = O.seeded_q8_matrix(rows, cols, GS, seed, std)
    f.write(np.ascontiguousarray(q).tobytes())
    f.write(np.ascontiguousarray(s, dtype=np.float32).tobytes())


def write_model(path, name):
    c = MODELS[name]
    d, h, L, H, KV, V = c["dim"], c["hidden_dim"], c["n_layers"], c["n_heads"], c["n_kv_heads"], c["vocab_size"]
    kv = d // H * KV
    base = c["seed"] * 1000
    rng = np.random.default_rng(base)
    with open(path, "wb") as f:
        header = struct.pack("<Ii7iBi", 0x616B3432, 2, d, h, L, H, KV, V, c["seq_len"], c["shared"], GS)
        f.write(header + bytes(256 - len(header)))
        norms = (1 + 0.05 * rng.standard_normal((2 * L + 1) * d)).astype(np.float32)
        f.write(norms.tobytes())  # rms_att[L], rms_ffn[L], rms_final
        _q8(f, V, d, base + 1, c.get("embed_std", 0.02))  # embedding
        shapes = [(d, d), (kv, d), (kv, d), (d, d), (h, d), (d, h), (h, d)]  # wq wk wv wo w1 w2 w3
        for role, (rows, cols) in enumerate(shapes):
            for layer in range(L):
                _q8(f, rows, cols, base + 10 + 100 * role + layer)
        if not c["shared"]:
            _q8(f, V, d, base + 2)
    return path


def prompt(name, count, seed=3):
    """Uniform-random token ids (the benchmark's prompt distribution)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, MODELS[name]["vocab_size"], count).astype(np.int32)
