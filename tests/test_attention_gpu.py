"""GPU parity of the engine's per-token kernels through the C-ABI.

Bars:
  - k_attention_kv within 1e-5 of the largest |output| of the reference's own decode attention (its AVX-512 split-K
    and scalar kernels, tests/golden/attention_golden.npz; the two agree to ~1e-6), at positions on both sides of the
    GPU kernel's 128-position splits;
  - the flash-style prefill kernel (a batch of rows) within the same 1e-5 of the reference at those positions, and of
    the decode kernel on the same rows (the two sum in different orders);
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
            for tag in ("avx512", "scalar"):
                want = GOLDEN[f"case{case}_pos{pos}_{tag}"]
                assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max(), (pos, tag)
    finally:
        kc.k_attention_free(work)


@pytest.mark.parametrize("case", range(len(AG.CASES)))
def test_prefill_rows_match_reference(kc, case):
    """A batch of rows ending at each golden position, the last row carrying the golden query: the flash kernel's last
    row against the reference's attention at that position."""
    n_heads, n_kv, hd, seq, positions = AG.CASES[case]
    qv, kcache, vcache = (dev(a) for a in AG.inputs(case))
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        for pos in positions:
            m = min(pos + 1, 37)
            q = torch.randn((m, n_heads * hd), device="cuda")
            q[-1] = qv
            out = torch.zeros((m, n_heads * hd), device="cuda")
            kc.k_attention_batch_kv(out, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos - m + 1, m)
            kc.status()
            got = host(out)[-1]
            for tag in ("avx512", "scalar"):
                want = GOLDEN[f"case{case}_pos{pos}_{tag}"]
                assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max(), (pos, tag)
    finally:
        kc.k_attention_free(work)


def test_batch_rows_match_single_rows_and_fused_quantize(kc, oracle):
    n_heads, n_kv, hd, seq = 32, 8, 128, 1024
    rng = np.random.default_rng(5)
    m, pos0 = 150, 200
    q = dev(rng.standard_normal((m, n_heads * hd), dtype=np.float32))
    kcache = dev(rng.standard_normal((n_kv, seq, hd), dtype=np.float32))
    vcache = dev(rng.standard_normal((n_kv, seq, hd), dtype=np.float32))
    work = kc.attention_work(n_heads, n_kv, hd, seq)
    try:
        batch = torch.zeros((m, n_heads * hd), device="cuda")
        kc.k_attention_batch_kv(batch, q, kcache, vcache, work, n_heads, n_kv, hd, seq, pos0, m)
        fused, oq = torch.zeros_like(batch), torch.zeros((m, n_heads * hd), dtype=torch.int8, device="cuda")
        os_ = torch.zeros((m, n_heads * hd // 64), device="cuda")
        kc.k_attention_q8_rows(fused, oq, os_, q, kcache, vcache, work, n_heads, n_kv, hd, seq, None, pos0, m, 64)
        single, sq = torch.zeros_like(batch), torch.zeros((m, n_heads * hd), dtype=torch.int8, device="cuda")
        ss = torch.zeros((m, n_heads * hd // 64), device="cuda")
        for r in range(m):
            kc.k_attention_q8_rows(single[r], sq[r], ss[r], q[r], kcache, vcache, work, n_heads, n_kv, hd, seq, None,
                                   pos0 + r, 1, 64)
        kc.status()
    finally:
        kc.k_attention_free(work)
    b, s, f = (host(t) for t in (batch, single, fused))
    assert (f.view(np.int32) == b.view(np.int32)).all()
    assert np.abs(b - s).max() <= 1e-5 * np.abs(s).max()
    for out, q8, sc in ((b, oq, os_), (s, sq, ss)):  # the quantized output is k_quantize of the fp32 one, bit for bit
        wq, ws = oracle.quantize(out, 64)
        assert (host(q8) == wq).all() and (host(sc).view(np.int32) == ws.view(np.int32)).all()


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
