"""ex_linear_noalloc: the exact linear layer for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc (or let a library do it): a serving engine that has reserved
almost all device memory for its KV cache, a host that owns every device allocation, or code in a region where
allocation calls are not allowed. ex_linear_noalloc takes no workspace; its split-K scratch is a static device
array inside the library. This test calls it through the C ABI and checks that it returns exactly the same bits as
ex_linear with a caller-provided workspace, on two calls in a row (the second call reuses scratch that the first one
must have left zeroed), and that a shape needing more scratch than the static array holds is refused cleanly.

The file is named so that pytest collects it last.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from vllm_exact import _lib, kernels as K
    return _lib, K


def _inputs(K, M, N, Kd, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, Kd, generator=g)
    x[torch.rand(M, Kd, generator=g) < 0.001] *= 50
    w = torch.randn(N, Kd, generator=g) * 0.02
    return K.digitize(x.bfloat16().to(DEV), 14), K.digitize(w.bfloat16().to(DEV), 14)


def _noalloc(L, xd, wd, out, algo=0, split_k=0):
    (xh, xl, cx, sx), (wh, wl, cw, sw) = xd, wd
    M, Kd = xh.shape
    N = wh.shape[0]
    return L.ex_linear_noalloc(xh.data_ptr(), xl.data_ptr(), xh.stride(0), cx.data_ptr(), sx.data_ptr(),
                               wh.data_ptr(), wl.data_ptr(), wh.stride(0), cw.data_ptr(), sw.data_ptr(), M, N, Kd,
                               14, 1, out.data_ptr(), 1, out.stride(0), split_k, algo,
                               torch.cuda.current_stream().cuda_stream)


def _with_workspace(L, xd, wd, out, algo=0, split_k=0):
    (xh, xl, cx, sx), (wh, wl, cw, sw) = xd, wd
    M, Kd = xh.shape
    N = wh.shape[0]
    need = L.ex_linear_workspace_bytes(M, N, Kd, split_k, algo)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=DEV)
    return L.ex_linear(xh.data_ptr(), xl.data_ptr(), xh.stride(0), cx.data_ptr(), sx.data_ptr(), wh.data_ptr(),
                       wl.data_ptr(), wh.stride(0), cw.data_ptr(), sw.data_ptr(), M, N, Kd, 14, 1, out.data_ptr(), 1,
                       out.stride(0), ws.data_ptr(), need, split_k, algo, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,Kd,algo,split_k", [(64, 4096, 4096, 0, 0),    # tensor cores, cluster-reduced split
                                                 (16, 6144, 4096, 0, 0),
                                                 (64, 24576, 4096, 0, 0),   # tensor cores, split tiles in scratch
                                                 (5, 1000, 12288, 2, 4),    # tensor cores, explicit split
                                                 (7, 300, 2048, 1, 4)])     # SIMT, explicit split
def test_noalloc_matches_workspace_entry_point(env, M, N, Kd, algo, split_k):
    lib, K = env
    L = lib.lib()
    xd, wd = _inputs(K, M, N, Kd, seed=M + N)
    ref = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    assert _with_workspace(L, xd, wd, ref, algo, split_k) == lib.EX_OK
    for _ in range(2):  # the second call runs on the scratch the first call returned to zero
        out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16)
        assert _noalloc(L, xd, wd, out, algo, split_k) == lib.EX_OK
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert lib.device_error() == 0


def test_noalloc_recovers_from_dirty_scratch(env):
    """A call stopped by a timed-out wait can leave split-K partials and tickets in the shared scratch, which would
    make every later call wrong. Stand in for that by filling the scratch with non-zero bytes (no GPU fault is
    involved: the kernels never wait on a ticket, so dirty tickets only leave split tiles unfinished), check that a
    call then goes wrong, and that ex_linear_noalloc_reset brings back the exact bits on two calls in a row."""
    lib, K = env
    L = lib.lib()
    M, N, Kd = 64, 24576, 4096  # the automatic tensor-core plan splits tiles across CTAs through the scratch
    assert L.ex_linear_workspace_bytes(M, N, Kd, 0, lib.EX_ALGO_TC_I8) > 0
    xd, wd = _inputs(K, M, N, Kd, seed=7)
    ref = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    assert _with_workspace(L, xd, wd, ref) == lib.EX_OK
    st = torch.cuda.current_stream().cuda_stream
    assert L.ex_linear_noalloc_fill_scratch(0x5A, st) == lib.EX_OK
    out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16)
    assert _noalloc(L, xd, wd, out) == lib.EX_OK
    torch.cuda.synchronize()
    assert not torch.equal(out, ref)  # dirty tickets: split tiles are never finished
    assert L.ex_linear_noalloc_reset(st) == lib.EX_OK
    for _ in range(2):
        out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16)
        assert _noalloc(L, xd, wd, out) == lib.EX_OK
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert L.ex_linear_noalloc_fill_scratch(256, st) == lib.EX_ERR_ARG
    assert lib.device_error() == 0


def test_noalloc_refuses_oversized_plan(env):
    """A SIMT split-K plan for M=1024, N=4096 needs 32 MiB of int64 partials, more than the static scratch."""
    lib, K = env
    L = lib.lib()
    M, N, Kd = 1024, 4096, 4096
    xd, wd = _inputs(K, M, N, Kd, seed=1)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    assert L.ex_linear_workspace_bytes(M, N, Kd, 16, lib.EX_ALGO_SIMT) > (24 << 20)
    rc = _noalloc(L, xd, wd, out, lib.EX_ALGO_SIMT, 16)
    assert rc == lib.EX_ERR_WORKSPACE
    assert b"EX_NOALLOC_SCRATCH_BYTES" in L.ex_last_error_string()
