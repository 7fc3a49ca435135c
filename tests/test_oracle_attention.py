"""CPU tests: the oracle's restatement of the reference's attention (orc_attention_decode: the split decode,
src/attention.c:40-105 + 664-682 + 760-810; orc_attention_tiled: the default batched variant, src/attention.c:245-334 +
1078-1229; orc_exp512, src/kernels_internal.h:62-76) against the reference's own outputs (tests/golden/
attention_golden.npz, made by the compiled reference) bitwise, and against the reference live where oracle/_ref exists.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_attention_golden as G  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "attention_golden.npz")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.int32)


@pytest.mark.parametrize("case", range(len(G.CASES)))
def test_decode_matches_reference_golden(oracle, case):
    n_heads, n_kv, hd, seq, positions = G.CASES[case]
    q, kc, vc = G.inputs(case)
    for pos in positions:
        got = oracle.attention_decode(q, kc, vc, n_heads, n_kv, hd, seq, pos)
        assert (bits(got) == bits(GOLDEN[f"case{case}_pos{pos}_avx512"])).all(), pos


@pytest.mark.parametrize("case", range(len(G.BATCH_CASES)))
def test_tiled_batch_matches_reference_golden(oracle, case):
    n_heads, n_kv, hd, seq, pos0, m = G.BATCH_CASES[case]
    q, kc, vc = G.batch_inputs(case)
    got = oracle.attention_tiled(q, kc, vc, n_heads, n_kv, hd, seq, pos0, m)
    assert (bits(got) == bits(GOLDEN[f"batch{case}"])).all()


def test_chunk_plan():
    """attention_chunks (src/attention.c:516-526): one chunk per 256 positions for a team no larger than the KV heads;
    a larger team splits short contexts further, at least 32 positions a chunk."""
    from oracle import oracle as O
    f = O.lib().orc_attention_chunks
    assert [f(p, 8, 36, 1) for p in (1, 256, 257, 2049, 8192)] == [1, 1, 2, 9, 32]
    assert [f(p, 8, 36, 16) for p in (1, 33, 300, 600)] == [1, 2, 2, 3]
    assert f(9000, 8, 32, 1) == 32


def test_exp512_close_to_exp(oracle):
    """exp512 is a Cephes-style approximation (about 2 ulp): close to the correctly rounded exponential on the softmax
    range, exactly 1 at 0, and clamped below."""
    f = oracle.lib().orc_exp512
    xs = np.linspace(-80, 0, 20001, dtype=np.float32)
    got = np.array([f(float(x)) for x in xs], np.float32)
    want = np.exp(xs.astype(np.float64)).astype(np.float32)
    assert np.abs(got.astype(np.float64) / want - 1).max() < 1e-6
    assert f(0.0) == 1.0 and f(-1e30) == f(-87.33654)


needs_ref = pytest.mark.skipif(not HERE.parent.joinpath("oracle/_ref/libllama_ref.so").exists(),
                               reason="the reference was not compiled here")


@needs_ref
@pytest.mark.parametrize("seed", [1, 2])
def test_attention_matches_compiled_reference(oracle, seed):
    rng = np.random.default_rng(seed)
    for nh, nkv, hd, seq, pos0, m in [(32, 8, 128, 1024, 250, 40), (8, 2, 64, 700, 0, 300), (4, 4, 2, 64, 5, 30)]:
        q = (rng.standard_normal((m, nh * hd)) * 2).astype(np.float32)
        kc = rng.standard_normal((nkv, seq, hd)).astype(np.float32)
        vc = rng.standard_normal((nkv, seq, hd)).astype(np.float32)
        assert (bits(oracle.attention_tiled(q, kc, vc, nh, nkv, hd, seq, pos0, m)) ==
                bits(oracle.ref_attention_batch(q, kc, vc, nh, nkv, hd, seq, pos0, m))).all()
        for r in (0, m // 2, m - 1):
            assert (bits(oracle.attention_decode(q[r], kc, vc, nh, nkv, hd, seq, pos0 + r)) ==
                    bits(oracle.ref_attention(q[r], kc, vc, nh, nkv, hd, seq, pos0 + r))).all()
