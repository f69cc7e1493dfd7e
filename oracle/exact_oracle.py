"""CPU oracle for the two hot paths of vllm-exact -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and only as the checker
or as the timed CPU baseline. The product (vllm_exact package and its CUDA library) never calls it: there is no CPU
fallback.

This is a numpy restatement of the reference's CPU integer path:

* ``digitize``        follows ``digitize_torch``      (reference: src/vllm_exact/kernels.py:22-39)
* ``exact_linear_i64``/``epilogue``/``exact_linear``
                      follow ``exact_linear_torch``   (reference: src/vllm_exact/kernels.py:89-100)
* ``paged_decode``    follows ``paged_decode_torch``  (reference: src/vllm_exact/paged_attn.py:117-132)

Parity pin: tests/test_oracle_golden.py checks this module against golden vectors produced by the reference itself
(tests/golden/make_golden.py imports the reference and records its outputs), including the sha256 of the
configuration-1 bf16 output.

A second restatement in plain C with integer-only dot products (exact_oracle_int.c, wrapped by c_oracle.py) is
checked against the same golden vectors and against this module on full-range digits at K = 65536
(tests/test_oracle_c.py).

Integer dot products are computed with float64 BLAS matrix products. This is exact: every digit is an integer with
|d| <= 128, so every product is an integer with |p| <= 2^14 and every partial sum of K terms is an integer with
|s| <= K * 2^14, far below 2^53 for any K this code is used with (checked below). Integers below 2^53 are represented
exactly in float64, so no rounding happens in any summation order, and the int64 result equals the reference's int64
torch matmul bit for bit.
"""
from __future__ import annotations

import numpy as np

_MAX_EXACT_K = 1 << 38  # K * 2^14 < 2^53 keeps every float64 partial sum an exact integer


# ----------------------------------------------------------------------------------------------------------------
# fixed-point digitization (reference kernels.py:22-39)
# ----------------------------------------------------------------------------------------------------------------
def _frexp_exponent(a: np.ndarray) -> np.ndarray:
    """Exponent e of a = m * 2^e with m in [0.5, 1), like torch.frexp / C frexp; 0 where a == 0 (kernels.py:26-27)."""
    _, e = np.frexp(a.astype(np.float32))
    e = e.astype(np.int32)
    return np.where(a > 0, e, 0).astype(np.int32)


def digitize(x: np.ndarray, F: int, amax: np.ndarray | None = None):
    """(R, K) float -> (h int8, l int8, cs int32, sh int32), bit for bit like digitize_torch (kernels.py:22-39).

    Per row: a = max|x|, e = frexp exponent of a (0 for an all-zero row), sh = F - e, scale = 2^sh built from float32
    bits with int32 wrap-around exactly as the reference does ((sh + 127) << 23, kernels.py:29), q = trunc(x * scale)
    toward zero (kernels.py:30). F = 14: balanced digits l = ((q + 128) & 255) - 128, h = (q - l) >> 8, cs = 0
    (kernels.py:36-38). F = 15: offset digits l = (q & 255) - 128, h = (q - l - 128) >> 8 and the row sum
    cs = sum(256 h + l) (kernels.py:32-34). With `amax` given, a is taken from it instead of from the row itself (the
    digits of a K slice are then the matching slice of the whole row's digits).
    """
    if F not in (14, 15):
        raise ValueError("F must be 14 or 15")
    x = np.ascontiguousarray(x, dtype=np.float32)
    if amax is not None:  # row maximum supplied (tensor parallelism: the maximum over every K shard of the row)
        a = np.asarray(amax, dtype=np.float32)
    else:
        a = np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32)
    e = _frexp_exponent(a)
    sh = (F - e).astype(np.int32)
    bits = ((sh.astype(np.int64) + 127) << 23).astype(np.uint64) & np.uint64(0xFFFFFFFF)  # int32 wrap-around
    scale = bits.astype(np.uint32).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        prod = (x * scale[:, None]).astype(np.float32)
    q = np.trunc(prod).astype(np.int64).astype(np.int32)
    if F == 15:
        l = (q & 255) - 128
        h = (q - l - 128) >> 8
        cs = (256 * h.astype(np.int64) + l).sum(axis=1)
        cs = ((cs + (1 << 31)) % (1 << 32) - (1 << 31)).astype(np.int32)  # int32 accumulation like the reference
    else:
        l = ((q + 128) & 255) - 128
        h = (q - l) >> 8
        cs = np.zeros_like(sh)
    return h.astype(np.int8), l.astype(np.int8), cs.astype(np.int32), sh.astype(np.int32)


# ----------------------------------------------------------------------------------------------------------------
# exact linear layer (reference kernels.py:89-100)
# ----------------------------------------------------------------------------------------------------------------
def _idot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact integer a @ b.T for integer-valued digit matrices (see the module docstring)."""
    if a.shape[1] >= _MAX_EXACT_K:
        raise ValueError("K too large for exact float64 accumulation")
    return np.rint(a.astype(np.float64) @ b.astype(np.float64).T).astype(np.int64)


def exact_linear_i64(xd, wd, F: int, trunc: bool) -> np.ndarray:
    """Integer total of the two-digit product, before scaling (kernels.py:93-97):
    tot = 2^16 xh.wh + 2^8 (xh.wl + xl.wh) [+ xl.wl if not trunc] [+ 128 (cx + cw) + 2^14 K if F == 15]."""
    xh, xl, cx, _ = xd
    wh, wl, cw, _ = wd
    K = xh.shape[1]
    tot = _idot(xh, wh) * 65536 + (_idot(xh, wl) + _idot(xl, wh)) * 256
    if not trunc:
        tot = tot + _idot(xl, wl)
    if F == 15:
        tot = tot + 128 * (cx.astype(np.int64)[:, None] + cw.astype(np.int64)[None, :]) + 128 * 128 * K
    return tot


def scale_bits(sx: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """float64 2^-(sx + sw) built from bits with int64 arithmetic, as kernels.py:98-99."""
    e = -(sx.astype(np.int64)[:, None] + sw.astype(np.int64)[None, :])
    return (((e + 1023) << 52).astype(np.uint64)).view(np.float64)


def epilogue(tot: np.ndarray, sx: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """int64 -> float64 (exact) times 2^-(sx + sw) -> float32 with one rounding (kernels.py:98-100)."""
    with np.errstate(over="ignore", under="ignore"):
        return (tot.astype(np.float64) * scale_bits(sx, sw)).astype(np.float32)


def exact_linear(xd, wd, F: int, trunc: bool = False) -> np.ndarray:
    """float32 (M, N) output of the exact linear layer, bit for bit like exact_linear_torch (kernels.py:89-100)."""
    return epilogue(exact_linear_i64(xd, wd, F, trunc), xd[3], wd[3])


# ----------------------------------------------------------------------------------------------------------------
# dtype helpers (round to nearest even, like torch's .to(bfloat16) / .to(float16))
# ----------------------------------------------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


# ----------------------------------------------------------------------------------------------------------------
# paged decode attention (reference paged_attn.py:117-132)
# ----------------------------------------------------------------------------------------------------------------
def paged_decode(q: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, block_table: np.ndarray,
                 seq_lens: np.ndarray, scale: float, n: int) -> np.ndarray:
    """float32 decode attention over a paged KV cache, one (request, head) at a time (paged_attn.py:117-132).

    q: (>=n, H, D); key_cache / value_cache: (num_blocks, BS, KV, D); block_table: (>=n, pages) int; seq_lens: (>=n,).
    Token t of request b lives in page block_table[b, t // BS] at offset t % BS; query head h reads KV head h // G.
    """
    BS = key_cache.shape[1]
    H = q.shape[1]
    KV = key_cache.shape[2]
    G = H // KV
    out = np.empty((n, H, q.shape[2]), dtype=np.float32)
    for b in range(n):
        L = int(seq_lens[b])
        pos = np.arange(L)
        pages = block_table[b, pos // BS].astype(np.int64)
        k = key_cache[pages, pos % BS].astype(np.float32)  # (L, KV, D)
        v = value_cache[pages, pos % BS].astype(np.float32)
        for h in range(H):
            sc = (k[:, h // G] @ q[b, h].astype(np.float32)) * np.float32(scale)
            sc = sc - sc.max() if L else sc
            p = np.exp(sc.astype(np.float64)).astype(np.float32)
            out[b, h] = (p / p.sum()) @ v[:, h // G] if L else np.nan
    return out


def leading_decodes(query_start_loc: np.ndarray) -> int:
    """Number of leading requests of a mixed prefill + decode step whose query length is 1, i.e. the requests the
    patched attention decodes (reference paged_attn.py:153-159: ql = qsl[1:] - qsl[:-1]; nd = cumprod(ql == 1).sum())."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    ql = qsl[1:] - qsl[:-1]
    return int(np.cumprod((ql == 1).astype(np.int64)).sum())
