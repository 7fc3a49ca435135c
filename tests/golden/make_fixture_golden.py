"""Generates tests/golden/ref_fixture.npz from the REFERENCE's own test fixture and its committed golden values:

  int8_bin  the Q8_0 checkpoint that the reference's tests/fixtures.py `create` writes for its `shared` fixture
            (dim 4, hidden 8, 2 layers, 2 heads, 1 KV head, vocabulary 128010, context 32, group size 2), byte for byte
  runq      tests/baseline_logits.json["runq"]: the 48 values its test-int8 prints (tests/unit.c:55-62: logits[0..11]
            of engine_forward(65 + p, p) for p = 0..3), which its tests/test_runtime.py:55-70 checks at
            rel_tol 2e-5, abs_tol 2e-6

The reference is imported from its checkout at generation time (it is not vendored). Where oracle/_ref/probe-int8
exists, the reference compiled here is run on the fixture first and must reproduce those 48 values.

    python tests/golden/make_fixture_golden.py REFERENCE_CHECKOUT
"""
import importlib.util
import json
import math
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_fixture_golden.py REFERENCE_CHECKOUT")
    ref = Path(sys.argv[1])
    spec = importlib.util.spec_from_file_location("reference_fixtures", ref / "tests" / "fixtures.py")
    fixtures = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fixtures)
    runq = json.loads((ref / "tests" / "baseline_logits.json").read_text())["runq"]
    assert len(runq) == 48
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp) / "shared"
        fixtures.create(root)
        blob = (root / "int8.bin").read_bytes()
        probe = ROOT / "oracle" / "_ref" / "probe-int8"
        if probe.exists():
            out = subprocess.run([str(probe), str(root / "int8.bin"), "65", "66", "67", "68"], capture_output=True,
                                 check=True, env={"LLAMA_THREADS": "1"}).stdout
            logits = np.frombuffer(out, np.float32).reshape(4, -1)[:, :12].reshape(-1)
            assert all(math.isclose(a, b, rel_tol=2e-5, abs_tol=2e-6) for a, b in zip(logits, runq)), "probe"
    np.savez_compressed(HERE / "ref_fixture.npz", int8_bin=np.frombuffer(blob, np.uint8),
                        runq=np.array(runq, np.float64))
    print(f"wrote {HERE / 'ref_fixture.npz'} ({len(blob)} checkpoint bytes)")


if __name__ == "__main__":
    main()
