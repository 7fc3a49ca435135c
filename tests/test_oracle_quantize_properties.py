"""CPU property tests: the C oracle's quantizer, bit for bit, against an independent numpy restatement of the
reference's rule (k_quantize, src/gemv.c:589-624) on generated inputs. Per gs-group: wmax = max |x| in float32,
scale = wmax / 127.0f, q = roundf(clamp(x / scale, -127, 127)) with ties away from zero, and q = 0 when scale == 0.
The generated values include exact ties, subnormals, zeros, signed zeros and values near float32's range."""
import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.extra import numpy as hnp  # noqa: E402


def quantize_rule(x, gs):
    g = x.reshape(-1, gs)
    wmax = np.abs(g).max(axis=1)
    scale = (wmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where(scale[:, None] == 0, np.float32(0), g / scale[:, None]).astype(np.float32)
    v = np.minimum(np.float32(127), np.maximum(np.float32(-127), v))
    v64 = v.astype(np.float64)  # |v| + 0.5 is exact in float64: roundf's half-away-from-zero
    q = (np.sign(v64) * np.floor(np.abs(v64) + 0.5)).astype(np.int8)
    return q.reshape(x.shape), scale


SPECIAL = [0.0, -0.0, 0.5, -0.5, 1.5, -2.5, 126.5, -126.5, 1e-45, -1e-45, 1e-38, 3e38, -3e38, 1.0, -1.0]
values = st.one_of(st.sampled_from(SPECIAL),
                   st.floats(min_value=-float(np.float32(3e38)), max_value=float(np.float32(3e38)), allow_nan=False,
                             allow_infinity=False, width=32))


@settings(max_examples=300, deadline=None, derandomize=True)
@given(gs=st.sampled_from([2, 4, 16, 32, 64, 128]), groups=st.integers(1, 6), data=st.data())
def test_quantizer_follows_the_published_rule(oracle, gs, groups, data):
    x = data.draw(hnp.arrays(np.float32, groups * gs, elements=values))
    q, s = oracle.quantize(x, gs)
    want_q, want_s = quantize_rule(x, gs)
    assert (s.view(np.int32) == want_s.view(np.int32)).all()
    assert (q == want_q).all()
    assert np.abs(q.astype(np.int32)).max() <= 127


@settings(max_examples=100, deadline=None, derandomize=True)
@given(scale=st.sampled_from([1.0, 0.5, 2.0, 1e-3, 7.0]), data=st.data())
def test_exact_ties_round_away_from_zero(oracle, scale, data):
    # With a group maximum of 127 * scale, x = (k + 1/2) * scale divides back to an exact tie for these scales.
    ks = data.draw(hnp.arrays(np.int32, 63, elements=st.integers(-126, 125)))
    x = np.concatenate([[127 * scale], (ks + 0.5) * scale]).astype(np.float32)
    q, s = oracle.quantize(x, 64)
    want_q, want_s = quantize_rule(x, 64)
    assert (q == want_q).all() and (s.view(np.int32) == want_s.view(np.int32)).all()
