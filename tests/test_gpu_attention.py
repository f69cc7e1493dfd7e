"""GPU tests of the batch-invariant paged decode attention (reference tests/test_gpu.py:46-78 and BASELINE config 4).

Attention is floating point, so parity with the oracle is a tolerance (max abs error < 1e-3 against the float32
reference, as the reference's own test), while invariance is bitwise: a request's output must not change when it runs
alone, in a prefix of the batch, in a different batch, or with its pages moved elsewhere in the cache."""
import numpy as np
import pytest
import torch

import recipes as R
from oracle import exact_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3  # reference tests/test_gpu.py:68


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from vllm_exact import paged_attn
    old = paged_attn.MAX_LEN
    paged_attn.MAX_LEN = 20480
    yield paged_attn
    paged_attn.MAX_LEN = old


def _oracle(q, kc, vc, bt, sl, scale, n):
    f = lambda t: t.detach().cpu().float().numpy()
    return O.paged_decode(f(q), f(kc), f(vc), bt.cpu().numpy(), sl.cpu().numpy(), scale, n)


def _case(B, L, BS, H, KV, D, jitter=False, seed=0):
    q, kv, bt, sl = R.paged_case(B, L, BS, H, KV, D, seed=seed, ctx_jitter=jitter)
    return q.to(DEV), kv.to(DEV), bt.to(DEV), sl.to(DEV)


@pytest.mark.parametrize("B,L,BS", [(8, 300, 16), (8, 5000, 528), (4, 9000, 528), (64, 8192, 528)])
def test_reference_cases(P, B, L, BS):
    """Reference tests/test_gpu.py:57-78 (H=16, KV=4, D=256): tolerance against the oracle on the first 4 requests;
    computing only the first n requests gives bitwise equal rows; permuting physical pages (block table remapped)
    gives bitwise equal output."""
    H, KV, D = 16, 4, 256
    q, kv, bt, sl = _case(B, L, BS, H, KV, D)
    kc, vc = R.kv_views(kv, D)
    o = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, 1 / 16, o, B, int(sl.max()))
    n = min(B, 4)
    ref = _oracle(q, kc, vc, bt, sl, 1 / 16, n)
    assert np.abs(o[:n].float().cpu().numpy() - ref).max() < TOL
    o2 = torch.empty_like(o)
    P.paged_decode(q, kc, vc, bt, sl, 1 / 16, o2, n, int(sl.max()))
    assert torch.equal(o[:n], o2[:n])
    newpos = torch.randperm(kv.shape[0], generator=torch.Generator().manual_seed(5)).to(DEV)
    kv2 = torch.empty_like(kv)
    kv2[newpos] = kv
    kc2, vc2 = R.kv_views(kv2, D)
    o3 = torch.empty_like(o)
    P.paged_decode(q, kc2, vc2, newpos[bt.long()].to(torch.int32), sl, 1 / 16, o3, B, int(sl.max()))
    assert torch.equal(o, o3)


def test_golden_reference_outputs(P, golden):
    """Outputs of the reference's own CPU oracle (tests/golden/attn_small.npz) within tolerance."""
    ref = np.load(R.__file__.replace("recipes.py", "attn_small.npz"))
    for i, c in enumerate(golden["attention"]):
        q, kv, bt, sl = _case(c["B"], c["L"], c["BS"], c["H"], c["KV"], c["D"], c["jitter"])
        kc, vc = R.kv_views(kv, c["D"])
        o = torch.empty(c["B"], c["H"], c["D"], device=DEV, dtype=torch.float32)
        P.paged_decode(q, kc, vc, bt, sl, c["scale"], o, c["B"])
        assert np.abs(o.cpu().numpy() - ref[f"case{i}"]).max() < TOL, i


@pytest.mark.parametrize("n,ctx", [(256, 1024), (64, 8192), (16, 16384)])
def test_baseline_invariance(P, n, ctx):
    """BASELINE config 4 geometry (H=32, KV=8, D=128, page 16, lengths +-25%): 16 target requests give bitwise
    identical output alone (n=1), in a small batch and inside the full batch; tolerance against the oracle."""
    H, KV, D, BS = 32, 8, 128, 16
    q, kv, bt, sl = _case(n, ctx, BS, H, KV, D, jitter=True)
    kc, vc = R.kv_views(kv, D)
    scale = 1 / D ** 0.5
    full = torch.empty(n, H, D, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, scale, full, n)
    tg = torch.randperm(n, generator=torch.Generator().manual_seed(11))[:16].to(DEV)
    for i in range(4):  # alone
        b = int(tg[i])
        o1 = torch.empty(1, H, D, device=DEV, dtype=torch.bfloat16)
        P.paged_decode(q[b:b + 1], kc, vc, bt[b:b + 1], sl[b:b + 1], scale, o1, 1)
        assert torch.equal(o1[0], full[b])
    small = torch.empty(16, H, D, device=DEV, dtype=torch.bfloat16)  # the 16 targets as their own batch
    P.paged_decode(q[tg], kc, vc, bt[tg], sl[tg], scale, small, 16)
    assert torch.equal(small, full[tg])
    m = 2
    ref = _oracle(q[tg[:m]], kc, vc, bt[tg[:m]], sl[tg[:m]], scale, m)
    assert np.abs(small[:m].float().cpu().numpy() - ref).max() < TOL


def test_vllm022_layout_views(P):
    """The (2, num_blocks, block_size, KV, D) KV layout of vLLM 0.22 gives the same bits as the reference layout."""
    H, KV, D, BS, B = 32, 8, 128, 16, 8
    q, kv, bt, sl = _case(B, 700, BS, H, KV, D)
    kc, vc = R.kv_views(kv, D)
    kv22 = torch.stack([kc.contiguous(), vc.contiguous()])
    k2, v2 = P.kv_views(kv22, D)
    a = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    b = torch.empty_like(a)
    P.paged_decode(q, kc, vc, bt, sl, 0.1, a, B)
    P.paged_decode(q, k2, v2, bt, sl, 0.1, b, B)
    assert torch.equal(a, b)


def test_zero_and_short_lengths(P):
    """Requests of length 1 and exactly one page, and a segment boundary: finite outputs within tolerance."""
    H, KV, D, BS = 32, 8, 128, 16
    q, kv, bt, sl = _case(4, 4200, BS, H, KV, D)
    sl = torch.tensor([1, 16, 4096, 4097], dtype=torch.int32, device=DEV)
    kc, vc = R.kv_views(kv, D)
    o = torch.empty(4, H, D, device=DEV, dtype=torch.float32)
    P.paged_decode(q, kc, vc, bt, sl, 0.088, o, 4)
    ref = _oracle(q, kc, vc, bt, sl, 0.088, 4)
    assert np.abs(o.cpu().numpy() - ref).max() < TOL


MIXED_QL = [[1] * 8, [1, 1, 1, 4, 1, 2, 1, 1], [3, 1, 1, 1, 1, 1, 1, 1], [1, 1, 0, 0, 0, 0, 0, 0],
            [1, 1, 1, 1, 1, 1, 1, 2], [2] * 8]


def _qsl(ql):
    return torch.tensor(np.concatenate([[0], np.cumsum(ql)]), dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("H,KV,D", [(32, 8, 128), (16, 4, 256)])  # TMA page-gather kernel, cp.async kernel
@pytest.mark.parametrize("ql", MIXED_QL)
def test_mixed_step_leading_decodes(P, H, KV, D, ql):
    """Mixed prefill + decode step (reference paged_attn.py:153-159) without a host sync: given query_start_loc, the
    kernel computes exactly the leading requests of query length 1 (count from the oracle's restatement of the
    reference rule), bitwise equal to a plain decode of them, and leaves every other output row untouched."""
    B, BS = len(ql), 16
    q, kv, bt, sl = _case(B, 700, BS, H, KV, D, jitter=True)
    kc, vc = R.kv_views(kv, D)
    qsl = _qsl(ql)
    nd = O.leading_decodes(qsl.cpu().numpy())
    full = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, 0.1, full, B)
    o = torch.full((B, H, D), 7.0, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, 0.1, o, B, query_start_loc=qsl)
    assert torch.equal(o[:nd], full[:nd])
    assert bool((o[nd:] == 7.0).all())


def test_mixed_step_graph_replay_follows_query_start_loc(P):
    """The mixed-step call captured once in a CUDA graph: replays with different query_start_loc contents decode
    exactly the leading one-token requests of each (the count is made on the device at every replay)."""
    H, KV, D, BS, B = 32, 8, 128, 16, 8
    q, kv, bt, sl = _case(B, 700, BS, H, KV, D, jitter=True)
    kc, vc = R.kv_views(kv, D)
    full = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, 0.1, full, B)
    qsl = _qsl(MIXED_QL[0])
    o = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    ws = torch.empty(P.workspace_bytes(B, H, D), dtype=torch.uint8, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        P.paged_decode(q, kc, vc, bt, sl, 0.1, o, B, workspace=ws, query_start_loc=qsl)  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        P.paged_decode(q, kc, vc, bt, sl, 0.1, o, B, workspace=ws, query_start_loc=qsl)
    for ql in MIXED_QL[1:] + MIXED_QL[:1]:
        qsl.copy_(_qsl(ql))
        o.fill_(7.0)
        g.replay()
        torch.cuda.synchronize()
        nd = O.leading_decodes(qsl.cpu().numpy())
        assert torch.equal(o[:nd], full[:nd]), ql
        assert bool((o[nd:] == 7.0).all()), ql
    del g


@pytest.mark.parametrize("H,KV,D", [(32, 8, 128), (16, 4, 256)])  # TMA page-gather kernel, cp.async kernel
def test_kv_head_sharding_bitwise(P, H, KV, D):
    """Tensor parallelism shards attention by KV head with no communication: each half of the KV heads, with its query
    heads, computed on its own (strided views of the same cache, as a rank sees its shard) gives bitwise the rows of
    the full computation."""
    B, BS = 8, 16
    q, kv, bt, sl = _case(B, 900, BS, H, KV, D, jitter=True)
    kc, vc = R.kv_views(kv, D)
    full = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    P.paged_decode(q, kc, vc, bt, sl, 0.1, full, B)
    for r in range(2):
        k0, k1, h0, h1 = r * KV // 2, (r + 1) * KV // 2, r * H // 2, (r + 1) * H // 2
        o = torch.empty(B, H // 2, D, device=DEV, dtype=torch.bfloat16)
        P.paged_decode(q[:, h0:h1], kc[:, :, k0:k1], vc[:, :, k0:k1], bt, sl, 0.1, o, B)
        assert torch.equal(o, full[:, h0:h1]), r
