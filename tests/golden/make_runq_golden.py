"""Generates tests/golden/runq_golden.npz from the REFERENCE's own CLI (oracle/_ref/runq, src/app.c + src/runq.c
compiled from its sources by oracle/Makefile) on the reference's own test fixture (tests/fixtures.py `create`, the
`shared` fixture: Q8_0 group size 2, vocabulary 128010, and its byte-level tokenizer), greedy:

    runq int8.bin -z tokenizer.bin -i A --seed 123 -t 0 -n 24      (the flags of its tests/test_runtime.py:38-40)

with LLAMA_TOKENS_OUT recording the prompt ids and the generated ids. Stored: the tokenizer bytes, the command's flags
and the two id lists; the checkpoint is the one tests/golden/ref_fixture.npz already holds (checked here). tests/test_engine_gpu.py runs the same command with oracle/_ref/runq-gpu (the
same CLI linked against the GPU engine) and compares.

    make -C oracle REF=REFERENCE_CHECKOUT && python tests/golden/make_runq_golden.py REFERENCE_CHECKOUT
"""
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
FLAGS = ["-i", "A", "--seed", "123", "-t", "0", "-n", "24"]


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_runq_golden.py REFERENCE_CHECKOUT")
    ref = Path(sys.argv[1])
    spec = importlib.util.spec_from_file_location("reference_fixtures", ref / "tests" / "fixtures.py")
    fixtures = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fixtures)
    runq = ROOT / "oracle" / "_ref" / "runq"
    if not runq.exists():
        raise SystemExit("oracle/_ref/runq is missing: run `make -C oracle REF=<reference checkout>`")
    with tempfile.TemporaryDirectory() as tmp:
        root = fixtures.create(Path(tmp) / "shared")
        out = Path(tmp) / "tokens.json"
        subprocess.run([str(runq), str(root / "int8.bin"), "-z", str(root / "tokenizer.bin"), *FLAGS], check=True,
                       capture_output=True, env={**os.environ, "LLAMA_TOKENS_OUT": str(out), "LLAMA_THREADS": "1"})
        ids = json.loads(out.read_text())
        held = np.load(HERE / "ref_fixture.npz")["int8_bin"].tobytes()
        assert held == (root / "int8.bin").read_bytes(), "ref_fixture.npz holds another checkpoint"
        np.savez_compressed(HERE / "runq_golden.npz",
                            tokenizer_bin=np.frombuffer((root / "tokenizer.bin").read_bytes(), np.uint8),
                            flags=np.array(FLAGS), prompt=np.array(ids["prompt"], np.int32),
                            generated=np.array(ids["generated"], np.int32))
    print(f"wrote {HERE / 'runq_golden.npz'}: prompt {ids['prompt']}, generated {ids['generated']}")


if __name__ == "__main__":
    main()
