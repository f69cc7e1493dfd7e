"""Seeded input recipes shared by the golden-vector generator (make_golden.py) and the tests.

All inputs come from torch's CPU generator so that the same bytes are produced here and on the GPU box; every recipe's
output bytes are pinned by a sha256 in golden.json, so a change in the generator would fail loudly instead of silently
testing different data.
"""
import hashlib

import numpy as np
import torch


def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        t = a.detach().cpu().contiguous()
        a = t.view(torch.int16).numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config1():
    """M=8, K=N=1024; activations bf16 ~N(0,1) with 0.1% of entries x50; weights bf16 ~N(0,0.02)."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(8, 1024, generator=g)
    m = torch.rand(8, 1024, generator=g) < 0.001
    x[m] *= 50
    x = x.bfloat16()
    w = (torch.randn(1024, 1024, generator=g) * 0.02).bfloat16()
    return x, w


# shapes of the reference's bitwise GPU test (tests/test_gpu.py:14) with its extreme-digit fixture (:21-23)
REF_GPU_SHAPES = [(24, 384, 4096), (5, 200, 12288), (1, 64, 4096), (300, 256, 12288)]
REF_GPU_MODES = [(14, True), (15, False)]


def extreme_digits(M, N, K, seed=0):
    """x[:, 7] *= 300 and w[:, 3] *= 300 push digits to |d| close to 128 (reference tests/test_gpu.py:18-23)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    x[:, 7] *= 300
    w = torch.randn(N, K, generator=g) * 0.02
    w[:, 3] *= 300
    return x, w


def ref_cpu_xw(M=7, N=33, K=512, seed=0, outlier=True):
    """Fixture of the reference's CPU self-checks (tests/test_reference_cpu.py:7-13)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if outlier:
        x[:, 3] *= 500
    w = torch.randn(N, K, generator=g) * 0.02
    return x, w


def digitize_bf16_input():
    """Reference tests/test_gpu.py:35-43 input: (300, 4096) bf16, 3 * N(0,1), seed 1."""
    g = torch.Generator().manual_seed(1)
    return (torch.randn(300, 4096, generator=g) * 3).to(torch.bfloat16)


def digitize_edge_rows():
    """Rows that exercise the corner cases of the digitizer: zero row, subnormal maximum, exact power of two,
    all-negative, a single huge outlier, the largest finite bf16 value, mixed tiny/large values."""
    K = 256
    g = torch.Generator().manual_seed(7)
    rows = [torch.zeros(K),
            torch.randn(K, generator=g) * 1e-39,          # subnormal row maximum (fp32 subnormals)
            torch.full((K,), 0.5),                        # max exactly a power of two
            -torch.rand(K, generator=g) - 0.25,           # all negative
            torch.cat([torch.tensor([3.0e4]), torch.randn(K - 1, generator=g)]),
            torch.cat([torch.tensor([3.3895e38]), torch.randn(K - 1, generator=g)]),
            torch.randn(K, generator=g) * 1e-30,
            torch.randn(K, generator=g) * 1e20,
            torch.cat([torch.tensor([1.0e-40]), torch.zeros(K - 1)]),  # a single subnormal
            torch.randn(K, generator=g)]
    return torch.stack(rows).bfloat16().float()


def paged_case(B, L, BS, H, KV, D, seed=0, ctx_jitter=False):
    """Paged KV cache in the reference test layout (tests/test_gpu.py:46-54): kv (nblocks, KV, BS, 2D) bf16, a random
    permutation of physical pages as block table, lengths in [L/2, L] (or [0.75 L, 1.25 L] with ctx_jitter).
    Returns q (B,H,D), kv, block_table (B, pages), seq_lens (B,), all CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    Lmax = (L * 5 + 3) // 4 if ctx_jitter else L
    nbp = (Lmax + BS - 1) // BS
    nblocks = B * nbp + 7
    kv = (torch.randn(nblocks, KV, BS, 2 * D, generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.randperm(nblocks, generator=g)[:B * nbp].view(B, nbp).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    lo, hi = ((3 * L) // 4, Lmax) if ctx_jitter else (L // 2, L)
    sl = torch.randint(lo, hi + 1, (B,), generator=g).to(torch.int32)
    return q, kv, bt, sl


def kv_views(kv, D):
    """key_cache, value_cache (num_blocks, BS, KV, D) strided views of kv (nblocks, KV, BS, 2D) (paged_attn.py:145)."""
    return kv.transpose(1, 2).split(D, dim=-1)
