"""Generates tests/golden/engine_golden.npz: the REFERENCE's own end-to-end outputs (oracle/_ref/probe-int8, its
tests/probe.c driver built from its sources by oracle/Makefile) on the seeded checkpoints of models.py.

    make -C oracle REF=REFERENCE_CHECKOUT && python tests/golden/make_engine_golden.py

Per model (prompt = models.prompt(name, P)):
  <name>_prompt     the prompt token ids
  <name>_generate   `probe-int8 generate MODEL 64 prompt...` with the default kernels (tests/probe.c:110-141)
  <name>_horizon    how many leading tokens the reference's three kernel selections (LLAMA_KERNELS=auto, avx512,
                    scalar) agree on: the reference's own self-consistency
  <name>_margin     per generated token, (top1 - top2) / max|logit| of the logits it was chosen from
                    (`probe-int8 tail MODEL 64 prompt+tokens...`): a divergence from the reference is only acceptable
                    at a near-tie
  <name>_logits     per-position logits (probe-int8 MODEL tokens..., tests/probe.c:174-183) of the first <name>_stable
                    prompt positions, the leading positions where the scalar and default kernels agree within 1e-6 of
                    the largest |logit| (at most 8)
  <name>_batch      `probe-int8 batch MODEL prompt[:stable]...`: the LAST logits of the batched prefill
  <name>_w8a32_*    for tiny and small, the same with LLAMA_Q8_ACTIVATIONS=fp32 (W8A32); its horizon compares the
                    default and scalar kernels, its stable positions agree within 1e-5
The reference runs with LLAMA_THREADS=8.
"""
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import models  # noqa: E402

PROMPTS = {"tiny": 20, "small": 40, "wide": 300}
STEPS = 64


def probe(args, kernels="auto", activations="int8"):
    env = dict(os.environ, LLAMA_THREADS="8", LLAMA_KERNELS=kernels, LLAMA_Q8_ACTIVATIONS=activations)
    r = subprocess.run([str(models.O.PROBE_INT8), *map(str, args)], capture_output=True, env=env, check=True)
    return r.stdout


W8A32_MODELS = ("tiny", "small")


def w8a32(out, name, path, p, V):
    """The same outputs with LLAMA_Q8_ACTIVATIONS=fp32 (fp32 activations against the int8 weights), under
    <name>_w8a32_*: generate, horizon (auto against scalar kernels), margin, stable, logits."""
    f32 = "fp32"
    a = [int(t) for t in probe(["generate", path, STEPS, *p], "auto", f32).split()]
    c = [int(t) for t in probe(["generate", path, STEPS, *p], "scalar", f32).split()]
    horizon = next((i for i in range(min(len(a), len(c))) if a[i] != c[i]), min(len(a), len(c)))
    head = p[:8]
    la = np.frombuffer(probe([path, *head], "auto", f32), np.float32).reshape(-1, V)
    ls = np.frombuffer(probe([path, *head], "scalar", f32), np.float32).reshape(-1, V)
    rel = np.abs(la - ls).max(1) / np.abs(ls).max(1)
    stable = int(next((i for i, r in enumerate(rel) if r > 1e-5), len(rel)))
    steps = len(a)
    tail = np.frombuffer(probe(["tail", path, steps, *p, *a[:steps - 1]], "auto", f32), np.float32).reshape(steps, V)
    assert (tail.argmax(1) == np.array(a)).all()
    top2 = np.sort(tail, axis=1)[:, -2:]
    out[f"{name}_w8a32_generate"] = np.array(a, np.int32)
    out[f"{name}_w8a32_horizon"] = np.int32(horizon)
    out[f"{name}_w8a32_stable"] = np.int32(stable)
    out[f"{name}_w8a32_logits"] = la[:stable]
    out[f"{name}_w8a32_margin"] = ((top2[:, 1] - top2[:, 0]) / np.abs(tail).max(1)).astype(np.float32)
    print(f"{name} W8A32: horizon {horizon}, stable positions {stable}, tokens {a[:12]}...")


def main():
    if not models.O.PROBE_INT8.exists():
        raise SystemExit("oracle/_ref/probe-int8 is missing: run `make -C oracle REF=<reference checkout>`")
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, n in PROMPTS.items():
            path = models.write_model(Path(tmp) / f"{name}.bin", name)
            p = models.prompt(name, n)
            V = models.MODELS[name]["vocab_size"]
            streams = {k: [int(t) for t in probe(["generate", path, STEPS, *p], k).split()]
                       for k in ("auto", "avx512", "scalar")}
            a, b, c = streams["auto"], streams["avx512"], streams["scalar"]
            horizon = next((i for i in range(min(map(len, (a, b, c)))) if not a[i] == b[i] == c[i]),
                           min(map(len, (a, b, c))))
            head = p[:8]
            la = np.frombuffer(probe([path, *head]), np.float32).reshape(-1, V)
            ls = np.frombuffer(probe([path, *head], "scalar"), np.float32).reshape(-1, V)
            rel = np.abs(la - ls).max(1) / np.abs(ls).max(1)
            stable = int(next((i for i, r in enumerate(rel) if r > 1e-6), len(rel)))
            out[f"{name}_prompt"] = p
            out[f"{name}_generate"] = np.array(a, np.int32)
            out[f"{name}_horizon"] = np.int32(horizon)
            out[f"{name}_stable"] = np.int32(stable)
            out[f"{name}_logits"] = la[:stable]
            out[f"{name}_batch"] = np.frombuffer(probe(["batch", path, *p[:stable]]), np.float32).reshape(-1, V)[-1]
            steps = len(a)
            tail = np.frombuffer(probe(["tail", path, steps, *p, *a[:steps - 1]]), np.float32).reshape(steps, V)
            assert (tail.argmax(1) == np.array(a)).all()
            top2 = np.sort(tail, axis=1)[:, -2:]
            out[f"{name}_margin"] = ((top2[:, 1] - top2[:, 0]) / np.abs(tail).max(1)).astype(np.float32)
            print(f"{name}: horizon {horizon}, stable positions {stable}, tokens {a[:12]}...")
            if name in W8A32_MODELS:
                w8a32(out, name, path, p, V)
    np.savez_compressed(HERE / "engine_golden.npz", **out)


if __name__ == "__main__":
    main()
