"""The integer-only C restatement of the reference's CPU path (oracle/exact_oracle_int.c) against the reference's
golden vectors and against the numpy oracle. The two restatements share no arithmetic: the numpy oracle's dot
products are float64 BLAS products, the C oracle's are int32/int64 integer sums. Agreement on every golden case,
and on full-range digits at the largest K the kernels accept (65536), pins the numpy oracle's exactness argument."""
import numpy as np
import pytest
import torch

import recipes as R
from oracle import c_oracle as C
from oracle import exact_oracle as O


def _np(t):
    return t.detach().cpu().float().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _built():
    try:
        C.lib()
    except RuntimeError as e:
        pytest.skip(str(e))


def test_config1_golden(golden):
    g = golden["config1"]
    x, w = R.config1()
    xd, wd = C.digitize(_np(x), 14), C.digitize(_np(w), 14)
    assert [R.sha(t) for t in xd] == g["xd_sha"]
    assert [R.sha(t) for t in wd] == g["wd_sha"]
    _, y = C.exact_linear(xd, wd, 14, True)
    assert R.sha(y) == g["y_f32_sha"]
    assert R.sha(O.f32_to_bf16_bits(y)) == g["y_bf16_sha"]


@pytest.mark.parametrize("idx", range(8))
def test_extreme_digit_cases_golden(golden, idx):
    """The reference GPU test's shapes and extreme-digit fixture (x[:, 7] *= 300, w[:, 3] *= 300) in both modes."""
    c = golden["extreme_digit_cases"][idx]
    x, w = R.extreme_digits(c["M"], c["N"], c["K"])
    xd, wd = C.digitize(_np(x), c["F"]), C.digitize(_np(w), c["F"])
    assert [R.sha(t) for t in xd] == c["xd_sha"]
    assert [R.sha(t) for t in wd] == c["wd_sha"]
    tot, y = C.exact_linear(xd, wd, c["F"], c["trunc"])
    assert R.sha(y) == c["y_f32_sha"]
    assert np.array_equal(tot, O.exact_linear_i64(xd, wd, c["F"], c["trunc"]))


def test_ref_cpu_fixture_and_digitize_golden(golden):
    x, w = R.ref_cpu_xw()
    for c in golden["ref_cpu_xw"]:
        F, tr = c["F"], c["trunc"]
        _, y = C.exact_linear(C.digitize(_np(x), F), C.digitize(_np(w), F), F, tr)
        assert R.sha(y) == c["y_f32_sha"], (F, tr)
    xb, xe = R.digitize_bf16_input(), R.digitize_edge_rows()
    for F in (14, 15):
        assert [R.sha(t) for t in C.digitize(_np(xb), F)] == golden["digitize_bf16"]["out"][str(F)]
        assert [R.sha(t) for t in C.digitize(_np(xe), F)] == golden["digitize_edge"]["out"][str(F)]


@pytest.mark.parametrize("F,trunc", [(14, True), (14, False), (15, True), (15, False)])
def test_full_range_digits_at_max_k(F, trunc):
    """Arbitrary int8 digits (every value in [-128, 127], far beyond what the digitizer emits) at K = 65536: integer
    totals and float32 outputs of both oracles agree bit for bit."""
    rng = np.random.default_rng(F * 2 + trunc)
    M, N, K = 3, 5, 65536
    xd = [rng.integers(-128, 128, (M, K), dtype=np.int8) for _ in range(2)]
    wd = [rng.integers(-128, 128, (N, K), dtype=np.int8) for _ in range(2)]
    xd[0][0], wd[0][0] = -128, -128  # one row pair with every product at its maximum, 2^14 per term
    xd += [rng.integers(-2**20, 2**20, M, dtype=np.int32), rng.integers(6, 13, M, dtype=np.int32)]
    wd += [rng.integers(-2**20, 2**20, N, dtype=np.int32), rng.integers(16, 19, N, dtype=np.int32)]
    tot, y = C.exact_linear(xd, wd, F, trunc)
    assert np.array_equal(tot, O.exact_linear_i64(xd, wd, F, trunc))
    assert np.array_equal(y.view(np.uint32), O.exact_linear(xd, wd, F, trunc).view(np.uint32))


def test_given_row_maxima_match_whole_rows():
    """Digitizing K slices with the whole rows' maxima (the tensor-parallel rule) gives the slices of the whole-row
    digits, in both oracles."""
    x, _ = R.ref_cpu_xw()
    x = _np(x)
    amax = np.abs(x).max(axis=1)
    for F in (14, 15):
        whole = C.digitize(x, F)
        for a, b in ((0, 300), (300, 777), (777, x.shape[1])):
            part_c = C.digitize(x[:, a:b], F, amax)
            part_o = O.digitize(x[:, a:b], F, amax)
            for t in (0, 1, 3):
                assert np.array_equal(part_c[t], part_o[t])
            assert np.array_equal(part_c[0], whole[0][:, a:b]) and np.array_equal(part_c[1], whole[1][:, a:b])


def test_digitize_agrees_on_random_magnitudes():
    """Rows drawn across the whole finite float32 range (normal and subnormal maxima, mixed signs, zeros): the two
    digitizers agree on every digit, row sum and shift (frexp of subnormals, scale bits wrapping for large shifts,
    truncation toward zero). NaN and Inf are outside the contract, as for the reference."""
    hyp = pytest.importorskip("hypothesis")
    st = pytest.importorskip("hypothesis.strategies")
    hnp = pytest.importorskip("hypothesis.extra.numpy")

    @hyp.settings(max_examples=300, deadline=None, derandomize=True)
    @hyp.given(hnp.arrays(np.float32, hnp.array_shapes(min_dims=2, max_dims=2, min_side=1, max_side=40),
                          elements=st.floats(allow_nan=False, allow_infinity=False, width=32)),
               st.sampled_from([14, 15]))
    def check(x, F):
        for a, b in zip(C.digitize(x, F), O.digitize(x, F)):
            assert np.array_equal(a, b)

    check()
