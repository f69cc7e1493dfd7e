"""Exact INT8 two-digit linear layer on B200: digitization + exact GEMM through the sm_100a C ABI.

Mirrors the GPU entry points of the reference's src/vllm_exact/kernels.py (same names, argument meaning and results):

* ``digitize(x, F, out=None)``                          reference kernels.py:74-85
* ``digitize_weight(w, F)``                             reference kernels.py:42-43
* ``exact_linear(xd, wd, F, trunc=False, out=None, cfg=None)``   reference kernels.py:257-289

Numerical spec (identical to the reference, kernels.py:3-9): activations and weights are converted per row to F-bit
fixed point with one power-of-two scale per row and split into two INT8 digits q = 256 h + l (F = 15 offset digits
with a row-sum correction, F = 14 balanced digits; trunc drops the l*l term). Digit products are exact and summed in
integers, so results do not depend on tiling, split-K, batch size or the other rows of the batch; then
int64 -> fp64 (exact) -> fp32 (one rounding) -> output dtype.

There is no CPU path: tensors must be on a CUDA device and the library must be built. The CPU integer restatement
used to check this module lives in the repository's oracle/ directory (test infrastructure only).
"""
from __future__ import annotations

import threading
import weakref

import torch

from . import _lib
from ._lib import EX_ALGO_AUTO, EX_ALGO_SIMT, EX_ALGO_TC_I8, check, lib

__all__ = ["digitize", "digitize_weight", "exact_linear", "exact_linear_partial_i64", "exact_epilogue",
           "autotune_exact", "EXACT_CFGS", "reserve_workspace", "reset_workspaces", "mark_static", "is_static",
           "EX_ALGO_AUTO", "EX_ALGO_SIMT", "EX_ALGO_TC_I8"]

_DT = {torch.float32: _lib.EX_DTYPE_F32, torch.bfloat16: _lib.EX_DTYPE_BF16, torch.float16: _lib.EX_DTYPE_F16}
_LD_ALIGN = 16  # digit rows are padded to 16 bytes so the tensor-core kernels can TMA them


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("vllm_exact B200 kernels need CUDA tensors (there is no CPU fallback)")


# ------------------------------------------------------------------------------------------------------------------
# split-K workspace: zero-filled once, every call returns it to zero
# ------------------------------------------------------------------------------------------------------------------
_WS = {}
_WS_RETIRED = []  # outgrown workspaces, kept alive: CUDA graphs captured earlier may still use them
_WS_LOCK = threading.Lock()


def _workspace(dev: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor | None:
    """The split-K workspace of (device, stream), grown geometrically. A workspace is never freed once it has been
    handed out: a CUDA graph captured with it keeps its address, so a later, larger call (for instance vLLM capturing
    a bigger batch after a smaller one) gets a new workspace and the old one stays valid for the old graph. A
    workspace first allocated during a capture is zero-filled by that graph's replays (the fill is captured too), and
    every call leaves it zero again."""
    if nbytes <= 0:
        return None
    key = (dev.index, _stream(dev) if stream is None else stream)
    with _WS_LOCK:
        ws = _WS.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 2 * (ws.numel() if ws is not None else 0), 1 << 20)
            if ws is not None:
                _WS_RETIRED.append(ws)
            ws = torch.zeros(size, dtype=torch.uint8, device=dev)
            _WS[key] = ws
    return ws


def reset_workspaces() -> None:
    """Re-zero every split-K workspace (current and retired). Needed only after a device error: a call stopped by a
    timed-out wait can leave partial sums behind (_lib.device_error() runs this when it reports an error)."""
    with _WS_LOCK:
        for ws in list(_WS.values()) + _WS_RETIRED:
            ws.zero_()


_lib.ON_DEVICE_ERROR.append(reset_workspaces)


def reserve_workspace(nbytes: int, device=None, stream=None) -> None:
    """Pre-allocate the split-K workspace of `stream` (default: the current stream), e.g. for the stream a CUDA graph
    will be captured on: a workspace first allocated during capture is zero-filled on every replay."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    _workspace(dev, nbytes, None if stream is None else stream.cuda_stream)


# ------------------------------------------------------------------------------------------------------------------
# static weight digits: may be read before the kernels ahead of a GEMM on the stream have finished
# ------------------------------------------------------------------------------------------------------------------
_STATIC = {}  # data_ptr -> number of live marked tensors starting there
_STATIC_LOCK = threading.Lock()


def _unmark(ptr: int) -> None:
    with _STATIC_LOCK:
        n = _STATIC.get(ptr, 0) - 1
        if n > 0:
            _STATIC[ptr] = n
        else:
            _STATIC.pop(ptr, None)


def mark_static(*tensors: torch.Tensor) -> None:
    """Declare weight digit tensors static. Synchronizes their devices first, so every kernel that wrote them has
    finished; from then on exact_linear lets the tensor-core GEMM start loading them before the kernels ahead of it on
    the stream have finished (EX_LINEAR_STATIC_WEIGHTS), which takes the weight stream's start off the critical path
    of back-to-back layers. A tensor stays marked while it is alive, and must not be written afterwards (writing
    through digitize(out=...) removes the mark). digitize_weight marks its results."""
    for dev in {t.device for t in tensors if t.is_cuda}:
        torch.cuda.synchronize(dev)
    for t in tensors:
        ptr = t.data_ptr()
        with _STATIC_LOCK:
            _STATIC[ptr] = _STATIC.get(ptr, 0) + 1
        weakref.finalize(t, _unmark, ptr)


def is_static(*tensors: torch.Tensor) -> bool:
    """True when every tensor starts where a live tensor marked by mark_static starts."""
    with _STATIC_LOCK:
        return all(t.data_ptr() in _STATIC for t in tensors)


def _clear_marks(*tensors: torch.Tensor) -> None:
    with _STATIC_LOCK:
        for t in tensors:
            _STATIC.pop(t.data_ptr(), None)


# ------------------------------------------------------------------------------------------------------------------
# digitization
# ------------------------------------------------------------------------------------------------------------------
def _alloc_digits(R: int, K: int, dev):
    ld = max(_LD_ALIGN, (K + _LD_ALIGN - 1) // _LD_ALIGN * _LD_ALIGN)
    h = torch.empty((R, ld), dtype=torch.int8, device=dev)[:, :K]
    l = torch.empty((R, ld), dtype=torch.int8, device=dev)[:, :K]
    cs = torch.empty(R, dtype=torch.int32, device=dev)
    sh = torch.empty(R, dtype=torch.int32, device=dev)
    return h, l, cs, sh


def digitize(x: torch.Tensor, F: int, out=None):
    """x (R, K) fp32/bf16/fp16 CUDA tensor -> (h int8, l int8, cs int32, sh int32), bitwise like the reference's
    digitize_torch (kernels.py:22-39). Digit rows are allocated with a 16-byte-aligned leading dimension."""
    _need_cuda(x)
    if x.dim() != 2:
        raise ValueError("digitize expects a 2-D tensor")
    if x.dtype not in _DT:
        raise TypeError(f"unsupported dtype {x.dtype}")
    if x.stride(1) != 1:
        x = x.contiguous()
    R, K = x.shape
    if out is None:
        out = _alloc_digits(R, K, x.device)
    elif _STATIC:
        _clear_marks(*out)
    h, l, cs, sh = out
    if h.stride(1) != 1 or l.stride(1) != 1 or h.stride(0) != l.stride(0):
        raise ValueError("digit buffers must be row-major with equal leading dimensions")
    with torch.cuda.device(x.device):
        check("ex_digitize", lib().ex_digitize(x.data_ptr(), _DT[x.dtype], x.stride(0), R, K, F, h.data_ptr(),
                                               l.data_ptr(), h.stride(0), cs.data_ptr(), sh.data_ptr(),
                                               _stream(x.device)))
    return out


def digitize_weight(w: torch.Tensor, F: int, rows_per_block: int = 32768):
    """Digitize a weight matrix once at load time (reference plugin.py:72-79), in row blocks. The digits are marked
    static (mark_static, which synchronizes the device)."""
    _need_cuda(w)
    N, K = w.shape
    out = _alloc_digits(N, K, w.device)
    for i in range(0, N, rows_per_block):
        j = min(N, i + rows_per_block)
        digitize(w[i:j], F, out=tuple(t[i:j] for t in out))
    mark_static(*out)
    return out


# ------------------------------------------------------------------------------------------------------------------
# exact linear
# ------------------------------------------------------------------------------------------------------------------
def _parse_cfg(cfg):
    """cfg: None (automatic), {"algo": ..., "split_k": ...}, or a reference-style tuple
    (BM, BN, BK, warps, stages, GM[, split_k[, mma]]) where only split_k carries meaning here. The reference's mma
    flag (0 = INT8, 1 = bf16 tensor cores, same bits either way) selects the INT8 tensor-core kernel for both values:
    B200 runs INT8 MMAs at twice the bf16 rate, so a bf16-digit kernel could only be slower. The Triton tile sizes
    have no counterpart."""
    if cfg is None:
        return EX_ALGO_AUTO, 0
    if isinstance(cfg, dict):
        return int(cfg.get("algo", EX_ALGO_AUTO)), int(cfg.get("split_k", 0))
    sk = int(cfg[6]) if len(cfg) > 6 else 0
    algo = EX_ALGO_TC_I8 if len(cfg) > 7 else EX_ALGO_AUTO
    return algo, sk


def _operands(xd, wd):
    xh, xl, cx, sx = xd
    wh, wl, cw, sw = wd
    _need_cuda(xh, xl, cx, sx, wh, wl, cw, sw)
    for t in (xh, xl, wh, wl):
        if t.dtype != torch.int8 or t.dim() != 2 or (t.numel() and t.stride(1) != 1):
            raise ValueError("digits must be row-major int8 matrices")
    if xh.shape != xl.shape or wh.shape != wl.shape or xh.shape[1] != wh.shape[1]:
        raise ValueError("digit shape mismatch")
    if xh.stride(0) != xl.stride(0) or wh.stride(0) != wl.stride(0):
        raise ValueError("h and l digits must share a leading dimension")
    for t in (cx, sx, cw, sw):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError("row scales / sums must be contiguous int32")
    return xh, xl, cx, sx, wh, wl, cw, sw


# Candidate configurations of autotune_exact. The reference lists Triton tile configurations here
# (kernels.py:250-253); the B200 kernels choose their tiles from the shape, so a configuration selects what is left
# free: the algorithm and the split-K factor (0 = the automatic plan of that algorithm). Every one gives the same bits.
EXACT_CFGS = ([{"algo": EX_ALGO_TC_I8, "split_k": s} for s in (0, 1, 2, 4, 8)] +
              [{"algo": EX_ALGO_SIMT, "split_k": 0}])
_CFG_CACHE = {}  # (M, N, K, F, trunc) -> configuration chosen by autotune_exact


def autotune_exact(xd, wd, F: int, trunc: bool):
    """Time every configuration of EXACT_CFGS on these operands (one warm-up call, then 10 calls between CUDA events
    on the current stream), remember the fastest for (M, N, K, F, trunc) and return it (reference kernels.py:292-316).
    Configurations the operands do not support (e.g. tensor-core algorithms on unaligned digits) are skipped.
    exact_linear(cfg=None) uses the remembered configuration; without a tuning call it takes the automatic plan, so
    nothing is ever timed inside a CUDA-graph capture. The choice changes speed only, never result bits."""
    xh, wh = xd[0], wd[0]
    M, K = xh.shape
    N = wh.shape[0]
    best = None
    for c in EXACT_CFGS:
        try:
            exact_linear(xd, wd, F, trunc, cfg=c)
            torch.cuda.synchronize(xh.device)
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            for _ in range(10):
                exact_linear(xd, wd, F, trunc, cfg=c)
            en.record()
            torch.cuda.synchronize(xh.device)
            t = st.elapsed_time(en)
        except _lib.ExactError:
            continue
        if best is None or t < best[0]:
            best = (t, c)
    if best is None:
        raise RuntimeError("autotune_exact: no configuration runs on these operands")
    _CFG_CACHE[(M, N, K, F, bool(trunc))] = best[1]
    return best[1]


def exact_linear(xd, wd, F: int, trunc: bool = False, out: torch.Tensor | None = None, cfg=None) -> torch.Tensor:
    """Exact linear layer y = x . w^T from digits (reference kernels.py:257-289). Returns fp32 (M, N) unless `out`
    (fp32, bf16 or fp16; row-major) is given. Bitwise identical to the reference's exact_linear_torch for every
    cfg (algorithm / split-K). cfg=None: the configuration autotune_exact chose for this shape, else the automatic
    plan."""
    xh, xl, cx, sx, wh, wl, cw, sw = _operands(xd, wd)
    M, K = xh.shape
    N = wh.shape[0]
    if out is None:
        out = torch.empty((M, N), device=xh.device, dtype=torch.float32)
    if out.dtype not in _DT or out.shape != (M, N) or (out.numel() and out.stride(1) != 1):
        raise ValueError("out must be a row-major (M, N) fp32/bf16/fp16 tensor")
    if cfg is None and _CFG_CACHE:
        cfg = _CFG_CACHE.get((M, N, K, F, bool(trunc)))
    algo, sk = _parse_cfg(cfg)
    L = lib()
    with torch.cuda.device(xh.device):
        nbytes = L.ex_linear_workspace_bytes(M, N, K, sk, algo)
        ws = _workspace(xh.device, nbytes)
        if _STATIC and is_static(wh, wl):
            algo |= _lib.EX_LINEAR_STATIC_WEIGHTS
        check("ex_linear", L.ex_linear(xh.data_ptr(), xl.data_ptr(), xh.stride(0), cx.data_ptr(), sx.data_ptr(),
                                       wh.data_ptr(), wl.data_ptr(), wh.stride(0), cw.data_ptr(), sw.data_ptr(), M, N,
                                       K, F, int(bool(trunc)), out.data_ptr(), _DT[out.dtype], out.stride(0),
                                       ws.data_ptr() if ws is not None else None, nbytes, sk, algo,
                                       _stream(xh.device)))
    return out


def exact_linear_partial_i64(xd, wd, F: int, trunc: bool = False, out: torch.Tensor | None = None,
                             cfg=None) -> torch.Tensor:
    """Exact int64 total of this K slice, before scaling (row-parallel building block). Totals of disjoint K slices
    add up exactly to the total of the whole K range."""
    xh, xl, cx, sx, wh, wl, cw, sw = _operands(xd, wd)
    M, K = xh.shape
    N = wh.shape[0]
    if out is None:
        out = torch.empty((M, N), device=xh.device, dtype=torch.int64)
    if out.dtype != torch.int64 or out.shape != (M, N) or (out.numel() and out.stride(1) != 1):
        raise ValueError("out must be a row-major (M, N) int64 tensor")
    algo, sk = _parse_cfg(cfg)
    L = lib()
    with torch.cuda.device(xh.device):
        nbytes = L.ex_linear_workspace_bytes(M, N, K, sk, algo)
        ws = _workspace(xh.device, nbytes)
        if _STATIC and is_static(wh, wl):
            algo |= _lib.EX_LINEAR_STATIC_WEIGHTS
        check("ex_linear_partial_i64",
              L.ex_linear_partial_i64(xh.data_ptr(), xl.data_ptr(), xh.stride(0), cx.data_ptr(), wh.data_ptr(),
                                      wl.data_ptr(), wh.stride(0), cw.data_ptr(), M, N, K, F, int(bool(trunc)),
                                      out.data_ptr(), out.stride(0), ws.data_ptr() if ws is not None else None,
                                      nbytes, sk, algo, _stream(xh.device)))
    return out


def exact_epilogue(tot: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = fp32(fp64(tot) * 2^-(sx + sw)) rounded to out's dtype (reference kernels.py:172-177)."""
    _need_cuda(tot, sx, sw, out)
    M, N = tot.shape
    if tot.dtype != torch.int64 or out.shape != (M, N) or out.dtype not in _DT:
        raise ValueError("bad epilogue operands")
    with torch.cuda.device(tot.device):
        check("ex_epilogue_i64", lib().ex_epilogue_i64(tot.data_ptr(), tot.stride(0), sx.data_ptr(), sw.data_ptr(), M,
                                                       N, out.data_ptr(), _DT[out.dtype], out.stride(0),
                                                       _stream(tot.device)))
    return out
