"""The torch custom ops of the exact linear layer, without any vLLM import.

``exactmm::linear`` (reference src/vllm_exact/plugin.py:51-69): same name, signature and semantics as the reference:
x (*, K) bf16/fp16 activations and the digitized weight buffers (wh, wl, cw, sw) -> (*, N) in x's dtype. Rows are
processed in blocks of RB (rows are independent, so the block size never changes results). The body calls the sm_100a
library: digitize, then the exact GEMM with fused epilogue.

``exactmm::linear_row_parallel`` (no reference counterpart: the reference runs on one GPU): the same for a K-sharded
(row-parallel) layer of a tensor-parallel group, x being this rank's K slice; the exchange steps (over peer memory
for calls of up to parallel.PEER_ROWS rows, else NCCL; bitwise the same) run inside the op, so torch.compile sees one
opaque call, as for the 1-GPU op.

F and TRUNC are set by vllm_exact.enable().
"""
import torch

from . import kernels as K

F = 14
TRUNC = True
RB = 16384


@torch.library.custom_op("exactmm::linear", mutates_args=())
def exact_linear_op(x: torch.Tensor, wh: torch.Tensor, wl: torch.Tensor, cw: torch.Tensor,
                    sw: torch.Tensor) -> torch.Tensor:
    shp = x.shape
    N = wh.shape[0]
    x2 = x.reshape(-1, shp[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    out = x.new_empty(M, N)
    for i in range(0, M, RB):
        xb = x2[i:i + RB]
        xd = K.digitize(xb, F)  # reads bf16 directly (bf16 -> fp32 is exact, same digits)
        K.exact_linear(xd, (wh, wl, cw, sw), F, TRUNC, out=out[i:i + RB])  # writes bf16 directly
    return out.reshape(*shp[:-1], N)


@exact_linear_op.register_fake
def _(x, wh, wl, cw, sw):
    return x.new_empty(*x.shape[:-1], wh.shape[0])


@torch.library.custom_op("exactmm::linear_row_parallel", mutates_args=())
def exact_linear_row_parallel_op(x: torch.Tensor, wh: torch.Tensor, wl: torch.Tensor, cw: torch.Tensor,
                                 sw: torch.Tensor) -> torch.Tensor:
    from . import parallel
    shp = x.shape
    N = wh.shape[0]
    x2 = x.reshape(-1, shp[-1])
    M = x2.shape[0]
    out = x.new_empty(M, N)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    for i in range(0, M, RB):  # every rank holds the same rows, so every rank makes the same collective calls
        parallel.row_parallel_linear_auto(x2[i:i + RB], wh, wl, cw, sw, F, TRUNC, out=out[i:i + RB])
    return out.reshape(*shp[:-1], N)


@exact_linear_row_parallel_op.register_fake
def _(x, wh, wl, cw, sw):
    return x.new_empty(*x.shape[:-1], wh.shape[0])
