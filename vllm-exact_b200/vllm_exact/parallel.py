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

The collectives of row_parallel_linear are torch.distributed calls on the tensor-parallel group (NCCL over NVLink on
GPUs). PeerRowParallel runs the same steps with both exchanges as peer-memory kernels over NVLink (CUDA IPC mappings):
steps 1-2 in one kernel (row maxima exchanged, slice digitized), steps 4-5 in another (reduce-scatter, epilogue of
this rank's columns, all-gather of the finished values), without NCCL on the data path. The compute
steps go through an `ops` object; the product uses the sm_100a library (CudaOps). Tests can pass another `ops` to
exercise the collective logic on CPU ranks (gloo), the way a fake device layer is used in host tests.
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib
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
    def epilogue(tot: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, dtype, out=None) -> torch.Tensor:
        if out is None:
            out = torch.empty(tot.shape, dtype=dtype, device=tot.device)
        return K.exact_epilogue(tot, sx, sw, out)


def _default_group():
    try:
        from vllm.distributed import get_tp_group
        return get_tp_group().device_group
    except Exception:
        return dist.group.WORLD


# Row-parallel calls of at most PEER_ROWS rows and PEER_COLS (even) output columns go through a PeerRowParallel object
# of their (device, group) where one exists; larger calls, and groups where peer memory is unavailable, take the NCCL
# path (bitwise the same results). VLLM_EXACT_B200_PEER_ROWS=0 turns the peer path off.
PEER_ROWS = int(os.environ.get("VLLM_EXACT_B200_PEER_ROWS", "256"))
PEER_COLS = 16384
_PEERS = {}  # (device index, group) -> PeerRowParallel, or None where it could not be made


def peer_for(device, group=None, create: bool = False):
    """The PeerRowParallel object of (device, group), or None. With create=True it is made on first request: that is
    a collective step, so every rank of the group must ask at the same point of its program, outside CUDA graph
    capture (the plugin asks while loading the weights of its first row-parallel layer). If the peer mappings fail on
    any rank, every rank records None and keeps the NCCL path."""
    g = group if group is not None else _default_group()
    dev = torch.device(device)
    key = (dev.index, g)
    if key in _PEERS or not create:
        return _PEERS.get(key)
    if PEER_ROWS <= 0 or not 2 <= dist.get_world_size(g) <= _lib.EX_TP_MAX_WORLD:
        _PEERS[key] = None  # off, a single rank, or more ranks than the peer kernels take: NCCL path
        return None
    try:
        _PEERS[key] = PeerRowParallel(PEER_ROWS, PEER_COLS, group=g, device=dev)
    except RuntimeError:
        _PEERS[key] = None
    return _PEERS[key]


def row_parallel_linear_auto(x2: torch.Tensor, wh, wl, cw, sw, F: int, trunc: bool, out: torch.Tensor,
                             group=None) -> torch.Tensor:
    """One row-parallel call (x2: M x K_local rows with unit column stride, out: M x N): over peer memory when the
    (device, group) has a PeerRowParallel object and the call fits it, else row_parallel_linear. The choice depends
    only on shapes and on objects made at the same point on every rank, so every rank takes the same path."""
    peer = peer_for(x2.device, group)
    M, N = x2.shape[0], wh.shape[0]
    if peer is not None and M <= peer.max_rows and N <= peer.max_cols and N % 2 == 0 and out.stride(0) % 2 == 0:
        return peer.linear(x2, wh, wl, cw, sw, F, trunc, out=out)
    return row_parallel_linear(x2, wh, wl, cw, sw, F, trunc, group=group, out=out)


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
        out = parts[0]
    else:
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
        out = (h, l, cs, sh)
    if w.is_cuda:
        K.mark_static(*out)  # load time: later GEMMs may start streaming these digits early
    return out


def row_parallel_linear(x: torch.Tensor, wh, wl, cw, sw, F: int, trunc: bool, group=None, ops=CudaOps,
                        out_dtype=None, out=None) -> torch.Tensor:
    """y = x . w^T for a K-sharded layer: x is this rank's (..., K_local) slice, (wh, wl, cw, sw) its weight digits
    made by digitize_weight_row_sharded. Every rank returns the full (..., N) output, bitwise identical to the 1-GPU
    exact layer; `out` (M x N, row-major, M = rows of x) receives it when given."""
    g = group if group is not None else _default_group()
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    amax = global_row_absmax(x2, g, ops)
    xd = ops.digitize_given(x2, F, amax)
    tot = ops.partial(xd, (wh, wl, cw, sw), F, trunc)
    dist.all_reduce(tot, op=dist.ReduceOp.SUM, group=g)
    if out is not None:
        return ops.epilogue(tot, xd[3], sw, out.dtype, out=out)
    y = ops.epilogue(tot, xd[3], sw, out_dtype or x.dtype)
    return y.reshape(*shp[:-1], wh.shape[0])


class PeerRowParallel:
    """Row-parallel exact layers with both exchange steps over peer memory instead of NCCL: ex_tp_digitize (row
    maxima of the K slice sent to every rank as (epoch, value) words, whole-row maxima, digits of the slice) and
    ex_allreduce_epilogue_i64 (reduce-scatter of the int64 partial totals, exact epilogue of this rank's 1/p of the
    columns, all-gather of the finished values as (epoch, value) words), plain loads and stores over NVLink into
    buffers shared through CUDA IPC handles exchanged once with all_gather_object (plain peer mappings, no multicast
    objects). Between the two runs the partial GEMM, written straight into this rank's shared partial buffer.

    One object per process group and largest call (max_rows x max_cols outputs). Same arguments and bitwise the same
    result as row_parallel_linear. Calls must be issued in the same order on every rank of the group, and on one rank
    they must not overlap on the GPU: each kernel reads its call epoch from the device, so two overlapping calls would
    take the same epoch and leave this rank out of step with the others. A call issued on another stream than the
    previous one is made to wait for that stream; inside graph capture the capturing stream must order them. The
    epochs live on the device, so calls can be captured in CUDA graphs."""

    def __init__(self, max_rows: int, max_cols: int, group=None, device=None):
        g = group if group is not None else _default_group()
        self.group = g
        self.rank, self.world = dist.get_rank(g), dist.get_world_size(g)
        if self.world > _lib.EX_TP_MAX_WORLD:
            raise ValueError(f"PeerRowParallel supports up to {_lib.EX_TP_MAX_WORLD} ranks")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.max_rows, self.max_cols = max_rows, max_cols
        self._opened = []
        self._bases = {}  # exported allocation handle -> mapped base (tensors may share one allocation)
        self._last_stream = None
        # Every rank takes the same two collective steps whatever fails locally, so a failure on one rank raises on
        # all of them (no rank left waiting in a collective, none left with a half-made object).
        try:
            self.xch = torch.zeros(2 * self.world * max_rows, dtype=torch.int64, device=dev)  # (epoch, max) words
            self.part = torch.zeros(max_rows * max_cols, dtype=torch.int64, device=dev)
            self.outx = torch.zeros(max_rows * max_cols, dtype=torch.int64, device=dev)  # epoch words (fp32: one each)
            self.flags = torch.zeros(_lib.tp_flag_words(self.world), dtype=torch.int32, device=dev)
            self.ctl = torch.zeros(4, dtype=torch.int32, device=dev)  # [0:2] ex_tp_digitize, [2:4] the all-reduce
            torch.cuda.synchronize(dev)
            mine = [self._handle(t) for t in (self.xch, self.part, self.outx, self.flags)]
        except RuntimeError:  # out of memory, or no IPC handle for the allocation
            mine = None
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=g)
        ok = all(hs is not None for hs in every)
        if ok:
            try:
                ptrs = []  # ptrs[p] = device addresses of rank p's buffers, as seen from this GPU
                for p, hs in enumerate(every):
                    if p == self.rank:
                        ptrs.append([t.data_ptr() for t in (self.xch, self.part, self.outx, self.flags)])
                    else:
                        ptrs.append([self._open(h) + off for h, off in hs])
                self.xch_ptrs, self.part_ptrs, self.outx_ptrs, self.flag_ptrs = (
                    torch.tensor([ptrs[p][k] for p in range(self.world)], dtype=torch.int64, device=dev)
                    for k in range(4))
                torch.cuda.synchronize(dev)
            except RuntimeError:
                ok = False
        oks = [None] * self.world
        dist.all_gather_object(oks, ok, group=g)  # also: every rank has mapped every buffer before the first call
        if not all(oks):
            self.close()
            raise RuntimeError("peer memory between the ranks of the group is not available on every rank")

    def _ordered(self, dev) -> None:
        """Order this call after the previous one when it is issued on another stream (outside graph capture, where
        the capturing stream orders the calls): two calls overlapping on the GPU would take the same epoch."""
        s = torch.cuda.current_stream(dev)
        if self._last_stream is not None and s != self._last_stream and not torch.cuda.is_current_stream_capturing():
            s.wait_stream(self._last_stream)
        self._last_stream = s

    def _handle(self, t: torch.Tensor):
        """(handle of the allocation holding t, byte offset of t inside it)."""
        buf = (ctypes.c_ubyte * _lib.EX_IPC_HANDLE_BYTES)()
        off = ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            check("ex_ipc_get_handle", lib().ex_ipc_get_handle(t.data_ptr(), buf, ctypes.byref(off)))
        return bytes(buf), off.value

    def _open(self, h: bytes) -> int:
        """Base address of another rank's exported allocation, mapped once per allocation."""
        if h not in self._bases:
            buf = (ctypes.c_ubyte * _lib.EX_IPC_HANDLE_BYTES).from_buffer_copy(h)
            ptr = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                check("ex_ipc_open_handle", lib().ex_ipc_open_handle(buf, ctypes.byref(ptr)))
            self._opened.append(ptr.value)
            self._bases[h] = ptr.value
        return self._bases[h]

    def close(self) -> None:
        """Unmap the peers' buffers (after the last call has completed on every rank)."""
        if not self._opened:
            self._bases = {}
            return
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib().ex_ipc_close_handle(p)
        self._opened = []
        self._bases = {}

    def digitize(self, x2: torch.Tensor, F: int, out=None):
        """Step 1 (ex_tp_digitize): this rank's K slice x2 (M x K_local, row-major) digitized with the whole-row
        maxima of all ranks. Every rank must call it with the same M."""
        M, Kd = x2.shape
        if M > self.max_rows:
            raise ValueError(f"PeerRowParallel holds {self.max_rows} rows, the call has {M}")
        dev = x2.device
        h, l, cs, sh = out if out is not None else K._alloc_digits(M, Kd, dev)
        self._ordered(dev)
        with torch.cuda.device(dev):
            check("ex_tp_digitize",
                  lib().ex_tp_digitize(x2.data_ptr(), K._DT[x2.dtype], x2.stride(0), M, Kd, F,
                                       self.xch_ptrs.data_ptr(), self.max_rows, self.ctl.data_ptr(), self.rank,
                                       self.world, h.data_ptr(), l.data_ptr(), h.stride(0), cs.data_ptr(),
                                       sh.data_ptr(), K._stream(dev)))
        return h, l, cs, sh

    def partial(self, M: int, N: int) -> torch.Tensor:
        """This rank's shared int64 partial buffer, as an (M, N) view: the partial GEMM writes here."""
        if M > self.max_rows or N > self.max_cols:
            raise ValueError(f"PeerRowParallel holds {self.max_rows} x {self.max_cols} outputs, the call needs "
                             f"{M} x {N}")
        return self.part[: M * N].view(M, N)

    def reduce(self, M: int, N: int, sx: torch.Tensor, sw: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Step 3 (ex_allreduce_epilogue_i64): the partials every rank wrote into its partial(M, N) summed, scaled
        and written to `out` (M x N, row-major, bf16/fp16/fp32)."""
        dev = out.device
        self._ordered(dev)
        with torch.cuda.device(dev):
            check("ex_allreduce_epilogue_i64",
                  lib().ex_allreduce_epilogue_i64(self.part_ptrs.data_ptr(), N, self.outx_ptrs.data_ptr(),
                                                  self.flag_ptrs.data_ptr(), self.ctl.data_ptr() + 8, self.rank,
                                                  self.world, sx.data_ptr(), sw.data_ptr(), M, N, out.data_ptr(),
                                                  K._DT[out.dtype], out.stride(0), K._stream(dev)))
        return out

    def linear(self, x: torch.Tensor, wh, wl, cw, sw, F: int, trunc: bool, out_dtype=None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """row_parallel_linear with both exchanges over peer memory: same arguments and bitwise the same result."""
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        M = x2.shape[0]
        N = wh.shape[0]
        part = self.partial(M, N)
        xd = self.digitize(x2, F)
        K.exact_linear_partial_i64(xd, (wh, wl, cw, sw), F, trunc, out=part)
        y = out if out is not None else torch.empty(M, N, dtype=out_dtype or x.dtype, device=x2.device)
        self.reduce(M, N, xd[3], sw, y)
        return y if out is not None else y.reshape(*shp[:-1], N)
