"""Bit parity of the exact GEMM at the headline workload's own shapes: every (K, N) of the
sweep x M in {1, 16, 64, 256, 4096}, F = 14 truncated, bf16 output, with the bench's seeds and value distributions.

The reference's GPU test (tests/test_gpu.py:13-32) pins small shapes only; these shapes exercise the grid sizes the
benchmark times (lm_head's 1,187 n-tiles, M = 4096 plans with several chunks of sibling m-tiles, split tiles at every
M). Each output row depends only on its own activation row (reference tests/test_reference_cpu.py:37-46), so a row
sample checked against the CPU oracle over all N columns is a faithful check: every row at M <= 64, and eight rows
spread over the m-tiles and sibling chunks at M = 256 and 4096. Also the reference's extreme-digit fixture
(x[:, 7] *= 300, w[:, 3] *= 300, tests/test_gpu.py:21-23) at K = 12288, N = 151936."""
import numpy as np
import pytest
import torch

import bench
from oracle import exact_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
MS = [1, 16, 64, 256, 4096]


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from vllm_exact import kernels
    return kernels


def _rows(M):
    if M <= 64:
        return list(range(M))
    # first/last rows, a 128-token tile boundary, and rows inside the later sibling chunks of m-tiles
    return sorted({0, 1, 127, 128, M // 2 + 5, M - 129, M - 2, M - 1})


def _check(xd_rows, wdig, y_rows, chunk=16384):
    """Oracle over all N columns in chunks of weight rows; returns the number of mismatching bf16 outputs."""
    N = wdig[0].shape[0]
    bad = 0
    for c0 in range(0, N, chunk):
        c1 = min(N, c0 + chunk)
        wd = [t[c0:c1].cpu().numpy() for t in wdig]
        ref = O.f32_to_bf16_bits(O.exact_linear(xd_rows, wd, 14, True))
        bad += int((ref != y_rows[:, c0:c1]).sum())
    return bad


@pytest.mark.parametrize("shape", bench.SHAPES, ids=[s[0] for s in bench.SHAPES])
def test_headline_shapes_bitwise(K, shape):
    """Every M of the sweep for this (K, N): the GPU's bf16 output rows equal the oracle's, and the GPU digitizer's
    digits of those rows equal the oracle's digitizer."""
    name, Kd, N = shape
    i = [s[0] for s in bench.SHAPES].index(name)
    W = bench.make_weight_digits(Kd, N, 1000 + i, torch.device(DEV))
    xs, ys = [], []
    for M in MS:
        x = bench.make_activation(M, Kd, 17 * M + i, torch.device(DEV))
        xd = K.digitize(x, 14)
        y = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        K.exact_linear(xd, W, 14, True, out=y)
        rows = _rows(M)
        ref_xd = O.digitize(x[rows].float().cpu().numpy(), 14)
        for a, b in zip(ref_xd, xd):
            assert np.array_equal(a, b[rows].cpu().numpy()), (name, M, "digits")
        xs.append(ref_xd)
        ys.append(y[rows].cpu().view(torch.int16).numpy().view(np.uint16))
        del x, xd, y
    # rows are independent: one oracle pass over the weights for the rows of every M
    xd_all = [np.concatenate([d[j] for d in xs]) for j in range(4)]
    assert _check(xd_all, W, np.concatenate(ys)) == 0, name
    from vllm_exact import _lib
    assert _lib.device_error() == 0


def test_extreme_digits_lm_head_k12288(K):
    """The reference's extreme-digit fixture at the widest shape: K = 12288, N = 151936 (weight values generated on
    the GPU, activation rows with the fixture's outlier column), M = 16: every row, every column."""
    M, Kd, N = 16, 12288, 151936
    g = torch.Generator(device=DEV).manual_seed(11)
    W = K._alloc_digits(N, Kd, torch.device(DEV))
    wsample = []
    for r0 in range(0, N, 8192):
        r1 = min(N, r0 + 8192)
        w = torch.randn(r1 - r0, Kd, generator=g, device=DEV) * 0.02
        w[:, 3] *= 300
        K.digitize(w, 14, out=tuple(t[r0:r1] for t in W))
        if r0 == 0:
            wsample = w[:4].cpu().numpy()
    # the weight digitizer on a few rows of the fixture
    for a, b in zip(O.digitize(wsample, 14), W):
        assert np.array_equal(a, b[:4].cpu().numpy())
    x = torch.randn(M, Kd, generator=g, device=DEV)
    x[:, 7] *= 300
    xd = K.digitize(x, 14)
    y = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.exact_linear(xd, W, 14, True, out=y)
    ref_xd = O.digitize(x.cpu().numpy(), 14)
    yr = y.cpu().view(torch.int16).numpy().view(np.uint16)
    assert _check(ref_xd, W, yr) == 0
    # extreme digits really occur
    assert int(W[0].abs().max()) >= 32 and int(xd[0].abs().max()) >= 32
