"""Generates tests/golden/bench_golden.npz: the REFERENCE's own engine (oracle/_ref/libllama_ref_engine.so, built from
its sources by oracle/Makefile: src/engine.c + src/runq.c + its kernels) on the benchmark workloads, for the parity
checks of bench.py and tests/test_bench_parity_gpu.py.

    make -C oracle REF=REFERENCE_CHECKOUT && python tests/golden/make_bench_golden.py

Workloads (BASELINE configs 3 and 2): the seeded random-init Q8_0 checkpoints (seed 1) of the 8B and 1B
architectures written by oracle/model_file.py (the GPU side writes the same bytes with engine_write_random), the
uniform-random prompt of bench.py (seed 3; 2048 tokens for 8B, 128 for 1B), prefilled with engine_forward_batch in the
reference's default microbatches, then 64 tokens chosen greedily (sample_argmax) with engine_forward, as its probe's
`generate` does (tests/probe.c:110-141). Runs:
  8b_s1   one socket, LLAMA_THREADS=8
  8b_s2   two sockets (its tensor-parallel split, src/tp.c), LLAMA_SOCKETS=2 LLAMA_TOPOLOGY=virtual:2x4
  1b_s1   one socket, LLAMA_THREADS=8
Teams of at most one thread per (local) KV head give the attention the chunk plan of a team of one, the plan the GPU
engine uses (larger teams split prompts shorter than 256 positions per thread group differently).
Stored per run: the 64 tokens, the top-1 minus top-2 logit margin and the largest |logit| at each step, and the
first step's logits (the prompt's last row) in full.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
STEPS = 64
RUNS = {"8b_s1": ("8b", {"LLAMA_THREADS": "8"}),
        "8b_s2": ("8b", {"LLAMA_SOCKETS": "2", "LLAMA_TOPOLOGY": "virtual:2x4"}),
        "1b_s1": ("1b", {"LLAMA_THREADS": "8"})}

CHILD = r'''
import ctypes, json, os, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import bench
from oracle import model_file
arch, out = sys.argv[2], sys.argv[3]
a = bench.ARCH[arch]
P = bench.REQUEST[arch][0]
path = model_file.write_random_checkpoint(os.path.join("/dev/shm", "llama3x_golden_%s.bin" % arch), **a, seed=1)
eng = bench.load_engine()
L = ctypes.CDLL(os.path.join(sys.argv[1], "oracle", "_ref", "libllama_ref_engine.so"))
MP = ctypes.POINTER(eng.Model)
L.engine_load_context.argtypes = [MP, ctypes.c_char_p, ctypes.c_int]
L.engine_forward.argtypes = [MP, ctypes.c_int, ctypes.c_int]
L.engine_forward.restype = ctypes.POINTER(ctypes.c_float)
L.engine_forward_batch.argtypes = [MP, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int, ctypes.c_int]
L.engine_forward_batch.restype = ctypes.POINTER(ctypes.c_float)
L.engine_max_batch.argtypes = [MP]
model = eng.Model()
L.engine_load_context(ctypes.byref(model), os.fsencode(path), P + __STEPS__)
V = a["vocab_size"]
prompt = bench.prompt_tokens(P, V)
mb = L.engine_max_batch(ctypes.byref(model))
i = 0
while i < P:
    n = min(mb, P - i)
    lg = L.engine_forward_batch(ctypes.byref(model), (ctypes.c_int * n)(*prompt[i:i + n].tolist()), n, i,
                                1 if i + n == P else 0)
    i += n
toks, margins, maxes, first = [], [], [], None
for s in range(__STEPS__):
    x = np.ctypeslib.as_array(lg, (V,)).copy()
    if first is None:
        first = x
    o = np.argsort(x)[::-1][:2]
    toks.append(int(o[0])); margins.append(float(x[o[0]] - x[o[1]])); maxes.append(float(np.abs(x).max()))
    if s + 1 < __STEPS__:
        lg = L.engine_forward(ctypes.byref(model), int(o[0]), P + s)
np.savez(out, tokens=np.array(toks, np.int32), margins=np.array(margins, np.float32),
         maxes=np.array(maxes, np.float32), first=first, max_batch=np.int32(mb))
'''.replace("__STEPS__", str(STEPS))


def main():
    if not (ROOT / "oracle" / "_ref" / "libllama_ref_engine.so").exists():
        raise SystemExit("oracle/_ref/libllama_ref_engine.so is missing: run `make -C oracle REF=<reference checkout>`")
    out = {}
    for name, (arch, env) in RUNS.items():
        tmp = Path("/tmp") / f"llama3x_golden_{name}.npz"
        subprocess.run([sys.executable, "-c", CHILD, str(ROOT), arch, str(tmp)], check=True,
                       env={**{k: v for k, v in os.environ.items() if not k.startswith("LLAMA_")}, **env})
        z = np.load(tmp)
        for k in ("tokens", "margins", "maxes", "first", "max_batch"):
            out[f"{name}_{k}"] = z[k]
        out[f"{name}_env"] = np.array(json.dumps(env))
        print(name, z["tokens"][:8].tolist(), flush=True)
    np.savez_compressed(HERE / "bench_golden.npz", **out)
    print("wrote", HERE / "bench_golden.npz")


if __name__ == "__main__":
    main()
