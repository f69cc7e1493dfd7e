"""Pin the CPU oracle to the reference: every output of oracle/exact_oracle.py must hash to the value that the
reference's own CPU path produced on the same seeded inputs (tests/golden/make_golden.py). Also restates the
reference's CPU self-checks (tests/test_reference_cpu.py:16-60) against the oracle."""
import numpy as np
import pytest
import torch

import recipes as R
from oracle import exact_oracle as O


def _np(t):
    return t.detach().cpu().float().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


def test_config1_bitexact(golden):
    g = golden["config1"]
    x, w = R.config1()
    assert R.sha(x) == g["x_sha"] and R.sha(w) == g["w_sha"], "torch generator changed: inputs differ"
    xd, wd = O.digitize(_np(x), 14), O.digitize(_np(w), 14)
    assert [R.sha(t) for t in xd] == g["xd_sha"]
    assert [R.sha(t) for t in wd] == g["wd_sha"]
    y32 = O.exact_linear(xd, wd, 14, True)
    assert R.sha(y32) == g["y_f32_sha"]
    yb = O.f32_to_bf16_bits(y32)
    assert R.sha(yb) == g["y_bf16_sha"] == "5e328d30f41524bb3806f02788b2372938a9d3579577fd71aa83e1a18faf4e39"
    assert list(O.bf16_bits_to_f32(yb[0, :6])) == g["y0_6"]


@pytest.mark.parametrize("idx", range(8))
def test_extreme_digit_cases(golden, idx):
    c = golden["extreme_digit_cases"][idx]
    x, w = R.extreme_digits(c["M"], c["N"], c["K"])
    assert R.sha(x) == c["x_sha"] and R.sha(w) == c["w_sha"]
    xd, wd = O.digitize(_np(x), c["F"]), O.digitize(_np(w), c["F"])
    assert [R.sha(t) for t in xd] == c["xd_sha"]
    assert [R.sha(t) for t in wd] == c["wd_sha"]
    y = O.exact_linear(xd, wd, c["F"], c["trunc"])
    assert R.sha(y) == c["y_f32_sha"]
    assert R.sha(O.f32_to_bf16_bits(y)) == c["y_bf16_sha"]


def test_ref_cpu_fixture_all_modes(golden):
    x, w = R.ref_cpu_xw()
    for c in golden["ref_cpu_xw"]:
        F, tr = c["F"], c["trunc"]
        y = O.exact_linear(O.digitize(_np(x), F), O.digitize(_np(w), F), F, tr)
        assert R.sha(y) == c["y_f32_sha"], (F, tr)


def test_digitize_golden(golden):
    xb = R.digitize_bf16_input()
    assert R.sha(xb) == golden["digitize_bf16"]["x_sha"]
    xe = R.digitize_edge_rows()
    assert R.sha(xe) == golden["digitize_edge"]["x_sha"]
    for F in (14, 15):
        assert [R.sha(t) for t in O.digitize(_np(xb), F)] == golden["digitize_bf16"]["out"][str(F)]
        out = O.digitize(_np(xe), F)
        assert [int(v) for v in out[3]] == golden["digitize_edge"]["sh"][str(F)]
        assert [R.sha(t) for t in out] == golden["digitize_edge"]["out"][str(F)]


def test_attention_oracle_matches_reference(golden):
    ref = np.load(R.__file__.replace("recipes.py", "attn_small.npz"))
    for i, c in enumerate(golden["attention"]):
        q, kv, bt, sl = R.paged_case(c["B"], c["L"], c["BS"], c["H"], c["KV"], c["D"], ctx_jitter=c["jitter"])
        assert R.sha(kv) == c["kv_sha"] and R.sha(bt) == c["bt_sha"] and R.sha(sl) == c["sl_sha"]
        kc, vc = R.kv_views(kv, c["D"])
        out = O.paged_decode(_np(q), _np(kc), _np(vc), bt.numpy(), sl.numpy(), c["scale"], c["B"])
        assert np.abs(out - ref[f"case{i}"]).max() < 1e-5


# ---- the reference's CPU self-checks (tests/test_reference_cpu.py), restated against the oracle ----
def test_digitize_reconstructs():
    x, _ = R.ref_cpu_xw()
    x = x.numpy()
    for F in (14, 15):
        h, l, cs, sh = O.digitize(x, F)
        q = 256 * h.astype(np.int64) + l + (128 if F == 15 else 0)
        err = np.abs(q * np.ldexp(1.0, -sh.astype(np.int64))[:, None] - x).max(1) / np.abs(x).max(1)
        assert err.max() < 2.0 ** -(F - 1)
        if F == 15:
            assert np.array_equal(cs, (256 * h.astype(np.int64) + l).sum(1).astype(np.int32))


def test_exact_linear_close_to_float():
    x, w = R.ref_cpu_xw(outlier=False)
    x, w = x.numpy(), w.numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    for F, tr in ((15, False), (14, True)):
        y = O.exact_linear(O.digitize(x, F), O.digitize(w, F), F, tr).astype(np.float64)
        assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-3


def test_rows_independent():
    x, w = R.ref_cpu_xw(M=9)
    x, w = x.numpy(), w.numpy()
    for F, tr in ((15, False), (14, True)):
        wd = O.digitize(w, F)
        full = O.exact_linear(O.digitize(x, F), wd, F, tr)
        for i in (0, 4, 8):
            one = O.exact_linear(O.digitize(x[i:i + 1], F), wd, F, tr)
            assert np.array_equal(one[0], full[i])


def test_k_split_is_exact():
    x, w = R.ref_cpu_xw(K=1024)
    xd, wd = O.digitize(x.numpy(), 14), O.digitize(w.numpy(), 14)
    whole = O.exact_linear_i64(xd, wd, 14, True)
    parts = 0
    for s in (slice(0, 300), slice(300, 777), slice(777, 1024)):
        parts = parts + O.exact_linear_i64([xd[0][:, s], xd[1][:, s], xd[2], xd[3]],
                                           [wd[0][:, s], wd[1][:, s], wd[2], wd[3]], 14, True)
    assert np.array_equal(whole, parts)


def _reference_nd(qsl: torch.Tensor) -> int:
    """The reference's own expression for the decode count of a mixed step (paged_attn.py:155-157)."""
    ql = qsl[1:] - qsl[:-1]
    return int(torch.cumprod((ql == 1).to(torch.int32), 0).sum().item())


def test_leading_decodes_rule():
    """oracle.leading_decodes equals the reference's expression, and the per-request rule the attention kernels apply
    on the device (request b decoded iff every query length up to b is 1) selects exactly requests [0, nd)."""
    rng = np.random.default_rng(0)
    cases = [[1] * 8, [1, 1, 1, 4, 1, 2], [3, 1, 1], [1, 1, 0, 0], [], [1], [2], [1, 1, 1, 1, 2]]
    cases += [list(rng.choice([0, 1, 1, 1, 2, 5], size=int(rng.integers(0, 13)))) for _ in range(300)]
    for ql in cases:
        qsl = torch.tensor([0] + list(np.cumsum(ql, dtype=np.int64)), dtype=torch.int32)
        nd = O.leading_decodes(qsl.numpy())
        assert nd == _reference_nd(qsl), ql
        q = qsl.numpy()
        device_rule = [all(q[i + 1] - q[i] == 1 for i in range(b + 1)) for b in range(len(ql))]
        assert device_rule == [b < nd for b in range(len(ql))], ql


def test_mixed_step_request_bound():
    """Host side of the patched mixed step: the request count handed to the kernel comes from tensor shapes only."""
    from vllm_exact import paged_attn as P
    qsl = torch.zeros(7, dtype=torch.int32)
    assert P.mixed_step_requests(qsl, torch.zeros(6, 4), torch.zeros(6), torch.zeros(10, 2, 2)) == 6
    assert P.mixed_step_requests(qsl, torch.zeros(4, 4), torch.zeros(6), torch.zeros(10, 2, 2)) == 4
    assert P.mixed_step_requests(qsl, torch.zeros(6, 4), torch.zeros(6), torch.zeros(3, 2, 2)) == 3
    assert P.mixed_step_requests(torch.zeros(1, dtype=torch.int32), torch.zeros(6, 4), torch.zeros(6),
                                 torch.zeros(3, 2, 2)) == 0
