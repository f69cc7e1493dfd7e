"""Tensor parallelism for the exact linear layer: exact, bitwise identical to one GPU for any number of ranks.

The reference runs on one GPU only (README.md:95). Sharding the exact layer across GPUs needs care in two places:

* Column-parallel layers (output-sharded: QKV, gate_up, GDN in_proj, vocab-parallel lm_head): every rank holds full-K
  weight rows and the full activation rows, so the per-row scales are the same as on one GPU. Nothing to do.
* Row-parallel layers (K-sharded: o_proj, down, GDN out_proj): the fixed-point scale of a row must be taken over
  the WHOLE row (digitize_torch takes max|x| over the row, reference kernels.py:25-29), so:
    1. each rank computes the row maxima of its K slice and the ranks all-reduce them with MAX (exact, order-free);
    2. each rank digitizes its slice with the global maxima -> its digits are exactly the slice of the 1-GPU digits;
    3. each rank computes the exact int64 total of its slice (F = 15 offset terms of the slice included);
    4. the ranks all-reduce the int64 totals with SUM: integer addition is exact in any order, so the sum is the
       1-GPU total bit for bit under any ring / tree order;
    5. every rank applies the scaling epilogue.
  Steps 1-2 also run once for the weights at load time (the rows of a weight matrix are K-sharded too).

The collectives are torch.distributed calls on the tensor-parallel group (NCCL over NVLink on GPUs). The compute
steps go through an `ops` object; the product uses the sm_100a library (CudaOps). Tests can pass another `ops` to
exercise the collective logic on CPU ranks (gloo), the way a fake device layer is used in host tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels as K
from ._lib import check, lib


class CudaOps:
    """Compute steps of the row-parallel layer on the sm_100a library."""

    @staticmethod
    def row_absmax(x: torch.Tensor) -> torch.Tensor:
        R, Kd = x.shape
        out = torch.empty(R, dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            check("ex_row_absmax", lib().ex_row_absmax(x.data_ptr(), K._DT[x.dtype], x.stride(0), R, Kd,
                                                       out.data_ptr(), K._stream(x.device)))
        return out

    @staticmethod
    def digitize_given(x: torch.Tensor, F: int, amax: torch.Tensor):
        R, Kd = x.shape
        h, l, cs, sh = K._alloc_digits(R, Kd, x.device)
        amax = amax.contiguous()
        with torch.cuda.device(x.device):
            check("ex_digitize_given_absmax",
                  lib().ex_digitize_given_absmax(x.data_ptr(), K._DT[x.dtype], x.stride(0), R, Kd, F, amax.data_ptr(),
                                                 h.data_ptr(), l.data_ptr(), h.stride(0), cs.data_ptr(),
                                                 sh.data_ptr(), K._stream(x.device)))
        return h, l, cs, sh

    @staticmethod
    def partial(xd, wd, F: int, trunc: bool) -> torch.Tensor:
        return K.exact_linear_partial_i64(xd, wd, F, trunc)

    @staticmethod
    def epilogue(tot: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, dtype) -> torch.Tensor:
        out = torch.empty(tot.shape, dtype=dtype, device=tot.device)
        return K.exact_epilogue(tot, sx, sw, out)


def _default_group():
    try:
        from vllm.distributed import get_tp_group
        return get_tp_group().device_group
    except Exception:
        return dist.group.WORLD


def global_row_absmax(x: torch.Tensor, group=None, ops=CudaOps) -> torch.Tensor:
    """Row maxima of the whole (K-sharded) rows: local maxima, then an exact MAX all-reduce over the group."""
    amax = ops.row_absmax(x)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group if group is not None else _default_group())
    return amax


def digitize_weight_row_sharded(w: torch.Tensor, F: int, group=None, ops=CudaOps, rows_per_block: int = 32768):
    """Digitize this rank's K slice of a weight matrix with whole-row scales (load time)."""
    parts = []
    for i in range(0, w.shape[0], rows_per_block):
        wb = w[i:i + rows_per_block]
        parts.append(ops.digitize_given(wb, F, global_row_absmax(wb, group, ops)))
    if len(parts) == 1:
        return parts[0]
    # concatenate, keeping the 16-byte-aligned leading dimension of the digit rows
    N, Kd = w.shape
    h, l, cs, sh = K._alloc_digits(N, Kd, w.device) if w.is_cuda else [None] * 4
    if h is None:
        return tuple(torch.cat([p[j] for p in parts]) for j in range(4))
    r = 0
    for p in parts:
        n = p[0].shape[0]
        for dst, src in zip((h, l, cs, sh), p):
            dst[r:r + n].copy_(src)
        r += n
    return h, l, cs, sh


def row_parallel_linear(x: torch.Tensor, wh, wl, cw, sw, F: int, trunc: bool, group=None, ops=CudaOps,
                        out_dtype=None) -> torch.Tensor:
    """y = x . w^T for a K-sharded layer: x is this rank's (..., K_local) slice, (wh, wl, cw, sw) its weight digits
    made by digitize_weight_row_sharded. Every rank returns the full (..., N) output, bitwise identical to the 1-GPU
    exact layer."""
    g = group if group is not None else _default_group()
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    amax = global_row_absmax(x2, g, ops)
    xd = ops.digitize_given(x2, F, amax)
    tot = ops.partial(xd, (wh, wl, cw, sw), F, trunc)
    dist.all_reduce(tot, op=dist.ReduceOp.SUM, group=g)
    y = ops.epilogue(tot, xd[3], sw, out_dtype or x.dtype)
    return y.reshape(*shp[:-1], wh.shape[0])
