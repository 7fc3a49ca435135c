"""CPU tests of the engine's checkpoint loader (engine_load_context): every header and file that the reference's
checkpoint_map and validate_config reject (src/runtime.c:148-168, 179-290) is rejected with the reference's message,
before the engine touches a GPU. The library runs under KC_FAIL_RETURN, so the message is kept and the process lives.
No test here reaches a valid load: that would allocate device memory."""
import ctypes
import os
import struct
from pathlib import Path

import pytest

from conftest import load_engine

MAGIC = 0x616B3432
SMALL = dict(dim=64, hidden=128, layers=1, heads=2, kv=1, vocab=32, seq=16)


def v2_header(dim, hidden, layers, heads, kv, vocab, seq, shared=0, gs=64):
    h = struct.pack("<Ii7iBi", MAGIC, 2, dim, hidden, layers, heads, kv, vocab, seq, shared, gs)
    return h + bytes(256 - len(h))


def v3_header(dim, hidden, layers, heads, kv, vocab, seq, shared=0, gs=64, precision=1, eos=1, name=b"tiny",
              reserved=0):
    h = bytearray(256)
    struct.pack_into("<Ii7iiii", h, 0, MAGIC, 3, dim, hidden, layers, heads, kv, vocab, seq, precision, shared, gs)
    struct.pack_into("<ffifffiiiiiii", h, 48, 1e-5, 500000.0, 0, 1.0, 1.0, 4.0, 8192, seq, dim // heads, 0, eos,
                     -1, -1)
    h[100:100 + len(name)] = name
    h[255] = reserved
    return bytes(h)


def q8_bytes(n, gs=64):
    return n + n // gs * 4


def file_bytes(dim, hidden, layers, heads, kv, vocab, seq, shared=0, gs=64):
    kvd = dim // heads * kv
    n = 256 + (2 * layers + 1) * dim * 4 + q8_bytes(vocab * dim, gs)
    n += layers * (2 * q8_bytes(dim * dim, gs) + 2 * q8_bytes(dim * kvd, gs) + 3 * q8_bytes(dim * hidden, gs))
    return n + (0 if shared else q8_bytes(vocab * dim, gs))


@pytest.fixture(scope="module")
def load():
    eng = load_engine()
    lib = eng.load_library()  # binds the engine and selects KC_FAIL_RETURN

    def run(path, context=0):
        model = eng.Model()
        lib.engine_load_context(ctypes.byref(model), os.fsencode(str(path)), context)
        with pytest.raises(eng._kc().KernelError) as err:
            eng._check()
        assert not model.implementation
        return str(err.value)

    return run


def write(tmp_path, data, name="model.bin"):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def test_missing_and_short_files(load, tmp_path):
    assert load(tmp_path / "absent.bin").startswith(f"cannot open checkpoint '{tmp_path / 'absent.bin'}': ")
    assert "invalid/truncated checkpoint" in load(write(tmp_path, bytes(100)))
    assert "expected a regular file" in load(tmp_path)  # a directory


@pytest.mark.parametrize("header,message", [
    (bytes(256), "unsupported INT8 checkpoint: expected ak42 version 2 or 3"),
    (struct.pack("<Ii", MAGIC, 4) + bytes(248), "unsupported checkpoint version 4 for this executable"),
    (v3_header(**SMALL, precision=0), "checkpoint precision requires run executable"),
    (v3_header(**SMALL, precision=7), "unsupported checkpoint precision 7"),
    (v2_header(**SMALL, shared=2), "invalid classifier flag in '"),
    (v2_header(**{**SMALL, "dim": 0}), "invalid checkpoint dimensions: all seven dimensions must be positive"),
    (v2_header(**{**SMALL, "heads": 3}), "unsupported attention dimensions"),
    (v2_header(**{**SMALL, "heads": 4, "kv": 3}), "unsupported attention dimensions"),
    (v2_header(**SMALL, gs=48), "unsupported INT8 group size 48"),
    (v3_header(**SMALL, eos=SMALL["vocab"]), "invalid special token metadata"),
    (v3_header(**SMALL, name=b"x" * 128), "unterminated model name"),
    (v3_header(**SMALL, reserved=1), "unsupported nonzero reserved checkpoint metadata"),
    # tensor_bytes (src/runtime.c:170-177): gs 2 divides dim 6 and hidden 4, but the 3 x 6 embedding has 18 elements,
    # not a multiple of 4, so its scales would start unaligned.
    (v2_header(dim=6, hidden=4, layers=1, heads=1, kv=1, vocab=3, seq=4, gs=2),
     "unsupported INT8 tensor alignment/group size: 18 elements"),
])
def test_headers_the_reference_rejects(load, tmp_path, header, message):
    assert message in load(write(tmp_path, header + bytes(4096)))


def test_sizes_that_overflow_are_rejected_not_wrapped(load, tmp_path):
    # Valid divisibility, but the layer tensors' byte count exceeds 2^64: the reference's checked_mul fails.
    huge = dict(dim=1 << 30, hidden=1 << 30, layers=1 << 30, heads=1 << 20, kv=1 << 20, vocab=1 << 30, seq=1)
    assert "size multiplication overflow" in load(write(tmp_path, v2_header(**huge)))


def test_truncated_and_trailing_bytes(load, tmp_path):
    need = file_bytes(**SMALL)
    msg = load(write(tmp_path, v2_header(**SMALL) + bytes(need - 256 - 1)))
    assert f"need {need} bytes, found {need - 1}" in msg and msg.startswith("truncated checkpoint '")
    assert load(write(tmp_path, v3_header(**SMALL) + bytes(need - 256 + 4))) == \
        "version 3 checkpoint has unexpected trailing bytes"


def test_context_beyond_the_checkpoint(load, tmp_path):
    path = write(tmp_path, v2_header(**SMALL) + bytes(file_bytes(**SMALL) - 256))
    assert load(path, context=SMALL["seq"] + 1) == "requested context exceeds checkpoint context"


def test_random_models_are_validated_like_checkpoints(load):
    # engine_init_random applies the same configuration rules before it allocates anything.
    eng = load_engine()
    lib = eng.load_library()

    def init(gs=64, context=0, **kw):
        cfg = eng.Config()
        for k, v in {**dict(dim=64, hidden_dim=128, n_layers=1, n_heads=2, n_kv_heads=1, vocab_size=32, seq_len=16),
                     **kw}.items():
            setattr(cfg, k, v)
        model = eng.Model()
        lib.engine_init_random(ctypes.byref(model), ctypes.byref(cfg), gs, 1, context)
        with pytest.raises(eng._kc().KernelError) as err:
            eng._check()
        assert not model.implementation
        return str(err.value)

    assert "unsupported INT8 group size 48" in init(gs=48)
    assert "unsupported attention dimensions" in init(n_heads=3)
    assert init(context=17) == "requested context exceeds the model's context"


@pytest.mark.parametrize("name,value,message", [
    ("LLAMA_PRECISION", "fp16", "LLAMA_PRECISION must be fp32 or bf16"),
    ("LLAMA_PRECISION", "bf16", "LLAMA_PRECISION=bf16 applies to FP32 checkpoints (run)"),
    ("LLAMA_Q8_ACTIVATIONS", "int4", "LLAMA_Q8_ACTIVATIONS must be int8 or fp32"),
    ("LLAMA_PREFILL_GEMM", "maybe", "LLAMA_PREFILL_GEMM must be auto, on or off"),
    ("LLAMA_PREFILL_BATCH", "0", "LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX"),
    ("LLAMA_PREFILL_BATCH", "-4", "LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX"),
    ("LLAMA_PREFILL_BATCH", " 8", "LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX"),
    ("LLAMA_PREFILL_BATCH", "2147483648", "LLAMA_PREFILL_BATCH must be a positive integer <= INT_MAX"),
    ("LLAMA_PREFILL_LOGITS", "first", "LLAMA_PREFILL_LOGITS must be last or all"),
])
def test_environment_the_reference_rejects(load, tmp_path, monkeypatch, name, value, message):
    # prefill_precision / prefill_configure (src/prefill.c:9-50) and src/engine.c:131-135: checked before the file.
    monkeypatch.setenv(name, value)
    assert message in load(tmp_path / "absent.bin")


@pytest.mark.parametrize("name,value", [
    ("LLAMA_PRECISION", "fp32"), ("LLAMA_Q8_ACTIVATIONS", "fp32"), ("LLAMA_Q8_ACTIVATIONS", "int8"),
    ("LLAMA_PREFILL_GEMM", "off"), ("LLAMA_PREFILL_GEMM", "auto"), ("LLAMA_PREFILL_BATCH", "2147483647"),
    ("LLAMA_PREFILL_LOGITS", "all"), ("LLAMA_PREFILL_LOGITS", ""),
])
def test_environment_the_reference_accepts(load, tmp_path, monkeypatch, name, value):
    # Accepted settings get as far as opening the checkpoint.
    monkeypatch.setenv(name, value)
    assert load(tmp_path / "absent.bin").startswith("cannot open checkpoint")


@pytest.mark.parametrize("shared", [False, True])
def test_write_random_equals_the_oracle_checkpoint(tmp_path, shared):
    """engine_write_random (the product's benchmark checkpoint writer) writes byte for byte the checkpoint of the
    oracle's generator (oracle/model_file.py), so the GPU engine and the reference load the same model."""
    from conftest import load_engine
    from oracle import model_file
    eng = load_engine()
    cfg = dict(dim=256, hidden_dim=384, n_layers=2, n_heads=8, n_kv_heads=2, vocab_size=300, seq_len=64, shared=shared)
    a = eng.write_random(tmp_path / "gpu.bin", **cfg, seed=1)
    b = model_file.write_random_checkpoint(tmp_path / "oracle.bin", **cfg, seed=1)
    assert Path(a).read_bytes() == Path(b).read_bytes()
