"""GPU parity of the engine's per-token kernels through the C-ABI.

Bars:
  - attention bitwise the reference's own: one row (k_attention_kv, the split variant) against its AVX-512 decode
    attention (tests/golden/attention_golden.npz, case*_avx512), a batch (k_attention_batch_kv, the tiled variant)
    against its batched attention (batch*), at positions across 256-position chunks and 32-position tiles, and both
    against the oracle's restatements on fresh inputs; within 1e-5 of its scalar attention;
  - bitwise: the fused output quantization equals k_quantize of the fp32 output; RoPE + K/V store equals the oracle's
    k_rope_apply and the head-major copy; embedding rows equal q * s;
  - greedy keys: the first maximum wins, as sample_argmax (src/sampler.c:9-23);
  - seeded weights: a shard equals the same slice of the whole tensor, bitwise.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_attention_golden as AG  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "attention_golden.npz")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.int32)


@pytest.mark.parametrize("case", range(len(AG.CASES)))
def test_attention_matches_reference(kc, case):
    n_heads, n_kv, hd, seq, positions = AG.CASES[case]
    q, kcache, vcache = (dev(a) for a in AG.inputs(case))
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        for pos in positions:
            out = torch.zeros(n_heads * hd, device="cuda")
            kc.k_attention_kv(out, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos)
            kc.status()
            got = out.cpu().numpy()
            assert (bits(got) == bits(GOLDEN[f"case{case}_pos{pos}_avx512"])).all(), pos
            want = GOLDEN[f"case{case}_pos{pos}_scalar"]
            assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max(), pos
    finally:
        kc.k_attention_free(work)


@pytest.mark.parametrize("case", range(len(AG.BATCH_CASES)))
def test_batch_matches_reference(kc, case):
    """The reference's batched attention (its default tiled variant) on its golden inputs, bitwise."""
    n_heads, n_kv, hd, seq, pos0, m = AG.BATCH_CASES[case]
    q, kcache, vcache = (dev(a) for a in AG.batch_inputs(case))
    work = kc.attention_work(n_heads, n_kv, hd, seq, rows=m)
    try:
        out = torch.zeros((m, n_heads * hd), device="cuda")
        kc.k_attention_batch_kv(out, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos0, m)
        kc.status()
    finally:
        kc.k_attention_free(work)
    assert (bits(host(out)) == bits(GOLDEN[f"batch{case}"])).all()


@pytest.mark.parametrize("n_heads,n_kv,hd,seq,pos0,m,rows", [(32, 8, 128, 1024, 200, 150, 150),
                                                              (8, 2, 64, 600, 0, 300, 20),
                                                              (4, 4, 2, 64, 3, 40, 40),
                                                              (16, 8, 32, 512, 7, 100, 100)])
def test_batch_and_single_rows_match_the_oracle(kc, oracle, n_heads, n_kv, hd, seq, pos0, m, rows):
    """A batch (the tiled variant; `rows` of work: waves when fewer than m) and the same rows one at a time (the split
    variant) each bitwise their oracle restatement; the fused output quantization bitwise k_quantize of the fp32
    output; the two variants within fp32 rounding of each other. head_dim 2 runs the slow kernels."""
    rng = np.random.default_rng(hd + m)
    qh = rng.standard_normal((m, n_heads * hd), dtype=np.float32)
    kh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    vh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    q, kcache, vcache = dev(qh), dev(kh), dev(vh)
    gs = 64 if (n_heads // n_kv * hd) % 64 == 0 else 2
    work = kc.attention_work(n_heads, n_kv, hd, seq, rows=rows)
    try:
        batch = torch.zeros((m, n_heads * hd), device="cuda")
        kc.k_attention_batch_kv(batch, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos0, m)
        fused, oq = torch.zeros_like(batch), torch.zeros((m, n_heads * hd), dtype=torch.int8, device="cuda")
        os_ = torch.zeros((m, n_heads * hd // gs), device="cuda")
        kc.k_attention_q8_rows(fused, oq, os_, q, kcache, vcache, work, n_heads, n_kv, hd, seq, None, pos0, m, gs)
        single = torch.zeros_like(batch)
        for r in range(m):
            kc.k_attention_kv(single[r], q[r], kcache, vcache, work, n_heads, n_kv, hd, seq, pos0 + r)
        kc.status()
    finally:
        kc.k_attention_free(work)
    b, s, f = (host(t) for t in (batch, single, fused))
    assert (bits(b) == bits(oracle.attention_tiled(qh, kh, vh, n_heads, n_kv, hd, seq, pos0, m))).all()
    for r in (0, m // 3, m - 1):
        assert (bits(s[r]) == bits(oracle.attention_decode(qh[r], kh, vh, n_heads, n_kv, hd, seq, pos0 + r))).all()
    assert (bits(f) == bits(b)).all()
    assert np.abs(b - s).max() <= 1e-5 * np.abs(s).max()
    wq, ws = oracle.quantize(b, gs)
    assert (host(oq) == wq).all() and (bits(host(os_)) == bits(ws)).all()


@pytest.mark.parametrize("n_heads,n_kv,seq", [(8, 2, 1024), (4, 1, 8192), (8, 2, 8192)])
def test_device_position_matches_host_position(kc, n_heads, n_kv, seq):
    """Also at the per-rank shapes of the 8B model under tensor parallelism (8 ranks: 4 heads on 1 KV head; 4 ranks:
    8 on 2) and its full context."""
    hd = 128
    rng = np.random.default_rng(6)
    q = dev(rng.standard_normal(n_heads * hd, dtype=np.float32))
    kcache = dev(rng.standard_normal((n_kv, seq, hd), dtype=np.float32))
    vcache = dev(rng.standard_normal((n_kv, seq, hd), dtype=np.float32))
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        for pos in (0, 130, seq - 1):
            a, b = torch.zeros(n_heads * hd, device="cuda"), torch.zeros(n_heads * hd, device="cuda")
            kc.k_attention_kv(a, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos)
            p = torch.tensor([pos], dtype=torch.int32, device="cuda")
            kc.k_attention_q8_rows(b, None, None, q, kcache, vcache, work, n_heads, n_kv, hd, seq, p, 0, 1, 64)
            kc.status()
            assert (a.cpu().numpy().view(np.int32) == b.cpu().numpy().view(np.int32)).all()
    finally:
        kc.k_attention_free(work)


@pytest.mark.parametrize("n_heads,n_kv,hd,gs", [(32, 8, 128, 64), (8, 2, 64, 32), (16, 2, 128, 128)])
def test_decode_step_quantized_output(kc, oracle, n_heads, n_kv, hd, gs):
    """One row at a device position with the output quantized for Wo (the decode step's call): the fp32 output
    bitwise the host-position call and the oracle, the int8 values and group scales bitwise k_quantize of it, across
    chunk counts 1 to 9 (the merge that the last CTA of each KV head runs, its quantization in the warp)."""
    seq = 4096
    rng = np.random.default_rng(hd + gs)
    qh = rng.standard_normal(n_heads * hd, dtype=np.float32)
    kh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    vh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    q, kcache, vcache = dev(qh), dev(kh), dev(vh)
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        for pos in (5, 255, 256, 2303):
            a, b = torch.zeros(n_heads * hd, device="cuda"), torch.zeros(n_heads * hd, device="cuda")
            oq = torch.zeros(n_heads * hd, dtype=torch.int8, device="cuda")
            os_ = torch.zeros(n_heads * hd // gs, device="cuda")
            kc.k_attention_kv(a, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos)
            p = torch.tensor([pos], dtype=torch.int32, device="cuda")
            kc.k_attention_q8_rows(b, oq, os_, q, kcache, vcache, work, n_heads, n_kv, hd, seq, p, 0, 1, gs)
            kc.status()
            got = host(b)
            assert (bits(got) == bits(host(a))).all(), pos
            assert (bits(got) == bits(oracle.attention_decode(qh, kh, vh, n_heads, n_kv, hd, seq, pos))).all(), pos
            wq, ws = oracle.quantize(got, gs)
            assert (host(oq) == wq).all() and (bits(host(os_)) == bits(ws)).all(), pos
    finally:
        kc.k_attention_free(work)


@pytest.mark.parametrize("n_heads,n_kv,hd", [(32, 8, 128), (4, 1, 128), (8, 2, 64)])
def test_rope_attention_step_equals_the_two_calls(kc, oracle, n_heads, n_kv, hd):
    """k_rope_attention_q8_step (the decode step's RoPE, K/V store and attention in one launch) bitwise
    k_rope_kv_store_rows followed by k_attention_q8_rows: outputs, quantized outputs and scales, and the cache row it
    writes; positions in the first and later chunks, and the context's last. The 8B shapes at 1 and 8 ranks."""
    seq, gs = 4096, 64
    assert kc.k_rope_attention_q8_step_ok(n_heads, n_kv, hd, gs) == 1
    rng = np.random.default_rng(n_heads + hd)
    kh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    vh = rng.standard_normal((n_kv, seq, hd), dtype=np.float32)
    table = dev(np.stack([oracle.rope_table(p, hd) for p in range(seq)]))
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        for pos in (0, 255, 256, 2303, seq - 1):
            qh = rng.standard_normal(n_heads * hd, dtype=np.float32)
            k_, v_ = rng.standard_normal(n_kv * hd, dtype=np.float32), rng.standard_normal(n_kv * hd, dtype=np.float32)
            p = torch.tensor([pos], dtype=torch.int32, device="cuda")
            outs = []
            for fused in (False, True):
                q, kd, vd, kcache, vcache = dev(qh), dev(k_), dev(v_), dev(kh), dev(vh)
                out = torch.zeros(n_heads * hd, device="cuda")
                oq = torch.zeros(n_heads * hd, dtype=torch.int8, device="cuda")
                os_ = torch.zeros(n_heads * hd // gs, device="cuda")
                if fused:
                    kc.k_rope_attention_q8_step(out, oq, os_, q, kd, vd, kcache, vcache, table, work, n_heads, n_kv,
                                                hd, seq, p, gs)
                else:
                    kc.k_rope_kv_store_rows(q, n_heads * hd, kd, vd, n_kv * hd, kcache, vcache, table, p, 0, 1,
                                            n_heads, n_kv, hd, seq)
                    kc.k_attention_q8_rows(out, oq, os_, q, kcache, vcache, work, n_heads, n_kv, hd, seq, p, 0, 1, gs)
                kc.status()
                outs.append([host(t) for t in (out, oq, os_, kcache[:, pos], vcache[:, pos])])
            for a, b in zip(*outs):
                assert (a.view(np.uint8) == b.view(np.uint8)).all(), pos
    finally:
        kc.k_attention_free(work)


def test_rope_kv_store_bitwise(kc, oracle):
    n_heads, n_kv, hd, seq, rows, pos0 = 8, 2, 64, 64, 5, 30
    rng = np.random.default_rng(7)
    q = rng.standard_normal((rows, n_heads * hd), dtype=np.float32)
    k = rng.standard_normal((rows, n_kv * hd), dtype=np.float32)
    v = rng.standard_normal((rows, n_kv * hd), dtype=np.float32)
    table = np.stack([oracle.rope_table(p, hd, 500000.0) for p in range(seq)])
    qd, kd, vd = dev(q), dev(k), dev(v)
    kcache, vcache = torch.zeros((n_kv, seq, hd), device="cuda"), torch.zeros((n_kv, seq, hd), device="cuda")
    kc.k_rope_kv_store_rows(qd, n_heads * hd, kd, vd, n_kv * hd, kcache, vcache, dev(table), None, pos0, rows, n_heads,
                            n_kv, hd, seq)
    kc.status()
    for r in range(rows):
        qr, kr = oracle.rope_apply(q[r], k[r], table[pos0 + r], n_heads, n_kv, hd)
        assert (qd[r].cpu().numpy().view(np.int32) == qr.view(np.int32)).all()
        assert (kcache[:, pos0 + r].cpu().numpy().reshape(-1).view(np.int32) == kr.view(np.int32)).all()
        assert (vcache[:, pos0 + r].cpu().numpy().reshape(-1) == v[r]).all()
    plain = torch.zeros((n_kv, seq, hd), device="cuda")
    kc.k_kv_store(plain, vd, n_kv * hd, pos0, rows, n_kv, hd, seq)
    kc.status()
    assert torch.equal(plain, vcache)


def test_embedding_rows(kc, oracle):
    V, dim, gs = 300, 256, 64
    wq, ws = oracle.seeded_q8_matrix(V, dim, gs, 9)
    tokens = np.array([0, 299, 17, 17], np.int32)
    x = torch.zeros((4, dim), device="cuda")
    kc.k_embed_q8_rows(x, dev(tokens), (dev(wq), dev(ws)), 4, dim, gs, V)
    kc.status()
    want = wq[tokens].astype(np.float32) * np.repeat(ws[tokens], gs, axis=1)
    assert (x.cpu().numpy().view(np.int32) == want.view(np.int32)).all()


def test_argmax_first_maximum_and_greedy_advance(kc):
    logits = np.full(5000, -3.0, np.float32)
    logits[[10, 4000, 4999]] = 2.5  # ties: the first index wins
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    kc.k_argmax_key(key, dev(logits), 5000, 1000)
    out = torch.zeros(4, dtype=torch.int32, device="cuda")
    step, token, pos = (torch.tensor([v], dtype=torch.int32, device="cuda") for v in (2, 0, 41))
    kc.k_greedy_advance(out, step, token, pos, key)
    kc.status()
    assert out.tolist() == [0, 0, 1010, 0] and step.item() == 3 and token.item() == 1010 and pos.item() == 42
    neg = np.full(100, -7.0, np.float32)
    neg[50] = -1e-30
    kc.k_argmax_key(key, dev(neg), 100, 0)
    kc.k_greedy_advance(out, step, token, pos, key)
    kc.status()
    assert token.item() == 50


def test_random_weights_shard_equals_slice(kc):
    rows, cols, gs = 96, 512, 64
    q, s = torch.zeros((rows, cols), dtype=torch.int8, device="cuda"), torch.zeros((rows, cols // gs), device="cuda")
    kc.k_random_q8(q, s, rows, cols, 0, 0, cols, 123, 4, 0.02, gs)
    qs, ss = torch.zeros((32, 128), dtype=torch.int8, device="cuda"), torch.zeros((32, 2), device="cuda")
    kc.k_random_q8(qs, ss, 32, 128, 40, 256, cols, 123, 4, 0.02, gs)
    kc.status()
    assert torch.equal(qs, q[40:72, 256:384]) and torch.equal(ss, s[40:72, 4:6])
    w = (q.float() * s.repeat_interleave(gs, dim=1)).cpu().numpy()
    assert abs(w.std() - 0.02) < 0.002 and abs(w.mean()) < 0.002
    assert q.abs().max().item() == 127
