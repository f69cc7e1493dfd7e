"""vLLM quantization plugin quantization="exact_int8" on B200 (reference src/vllm_exact/plugin.py:1-133).

Every linear layer (and lm_head unless disabled) runs the exact INT8 two-digit linear layer of kernels.py through the
torch custom op ``exactmm::linear`` of ops.py (same name and signature as the reference, plugin.py:51-69), whose body
calls the sm_100a C ABI. No changes to vLLM source: register_quantization_config + the custom op. Imported and configured by
vllm_exact.enable().

Tensor parallelism: column-parallel layers (output-sharded: QKV, gate_up, GDN in_proj, vocab-parallel lm_head) hold
full-K weight rows, so they need nothing special. Row-parallel layers (K-sharded: o_proj, down, GDN out_proj) go
through parallel.py: global row scales (a MAX all-reduce of row maxima), an exact int64 partial GEMM on the local K
slice, an int64 SUM all-reduce (exact under any reduction order) and the scaling epilogue; decode-sized calls run
both exchanges as peer-memory kernels (parallel.PeerRowParallel), larger ones through NCCL. vLLM's own bf16
all-reduce of that layer is switched off, because a sum of rounded partials is neither exact nor order-invariant.
"""
import json
import os
from pathlib import Path

import torch

from . import kernels as K
from . import ops
from vllm.model_executor.layers.linear import LinearBase, RowParallelLinear, UnquantizedLinearMethod
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead, UnquantizedEmbeddingMethod

# set by enable() (which also sets ops.F / ops.TRUNC, read by the custom op)
F = 14
TRUNC = True
LMHEAD = True
_TABLE = None
RB = ops.RB  # rows per block: rows are independent, results unchanged, temporary memory bounded (plugin.py:24)
# The reference keeps the bf16 weight beside its digits (plugin.py:72-79). VLLM_EXACT_DROP_BF16_WEIGHT=1 releases it
# after digitization: weight memory goes from 4 to 2 bytes per element, at the price of no later weight reload. A
# tied lm_head shares its tensor with the embedding, which keeps it (only this layer's reference is dropped).
DROP_BF16_WEIGHT = os.environ.get("VLLM_EXACT_DROP_BF16_WEIGHT", "0") == "1"


def load_table(path):
    """Accepted for compatibility with the reference's tuning tables (plugin.py:27-34). The B200 kernels choose their
    tiles from the shape; a table never changes results, so its contents are only recorded."""
    global _TABLE
    if path is None:
        _TABLE = None
        return
    _TABLE = json.loads(Path(path).read_text())


def _is_row_sharded(layer) -> bool:
    return isinstance(layer, RowParallelLinear) and getattr(layer, "tp_size", 1) > 1


def _digitize_layer(layer):
    """Digitize the weight once after loading into non-persistent buffers ex_wh / ex_wl (int8, rows padded to 16
    bytes for TMA) and ex_cw / ex_sw (int32) (reference plugin.py:72-79)."""
    w = layer.weight.data
    if _is_row_sharded(layer):
        from . import parallel
        h, l, cs, sh = parallel.digitize_weight_row_sharded(w, F)
        # the peer-memory exchange buffers of the group, made by the first row-parallel layer on every rank (a
        # collective step at the same point of every rank's loading, outside graph capture)
        parallel.peer_for(w.device, create=True)
    else:
        h, l, cs, sh = K.digitize_weight(w, F)
    layer.register_buffer("ex_wh", h, persistent=False)
    layer.register_buffer("ex_wl", l, persistent=False)
    layer.register_buffer("ex_cw", cs.contiguous(), persistent=False)
    layer.register_buffer("ex_sw", sh.contiguous(), persistent=False)
    if _is_row_sharded(layer):
        layer.reduce_results = False  # the exact int64 all-reduce inside apply replaces vLLM's bf16 all-reduce
    if DROP_BF16_WEIGHT:
        drop_bf16_weight(layer)


def drop_bf16_weight(layer):
    """Replace layer.weight by an empty tensor of the same dtype and device (shape (0, K)); the digit buffers are the
    only weights apply() reads. The parameter's attributes (weight_loader, ...) go with it."""
    w = layer.weight
    layer.weight = torch.nn.Parameter(torch.empty((0,) + tuple(w.shape[1:]), dtype=w.dtype, device=w.device),
                                      requires_grad=False)


def _apply(layer, x, bias):
    # one opaque custom op per call in both cases, so torch.compile never traces into the library's ctypes calls
    op = torch.ops.exactmm.linear_row_parallel if _is_row_sharded(layer) else torch.ops.exactmm.linear
    y = op(x, layer.ex_wh, layer.ex_wl, layer.ex_cw, layer.ex_sw)
    return y if bias is None else y + bias


class ExactLinearMethod(UnquantizedLinearMethod):
    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        _digitize_layer(layer)

    def apply(self, layer, x, bias=None):
        return _apply(layer, x, bias)


class ExactLMHeadMethod(UnquantizedEmbeddingMethod):
    """lm_head through the exact linear layer. lm_head does no embedding lookup; the parent embedding() is kept."""

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        _digitize_layer(layer)

    def apply(self, layer, x, bias=None):
        return _apply(layer, x, bias)


@register_quantization_config("exact_int8")
class ExactInt8Config(QuantizationConfig):
    def __init__(self):
        super().__init__()

    def get_name(self):
        return "exact_int8"

    def get_supported_act_dtypes(self):
        return [torch.bfloat16, torch.float16]

    @classmethod
    def get_min_capability(cls):
        return 100  # the kernels are built for sm_100a only

    @staticmethod
    def get_config_filenames():
        return []

    @classmethod
    def from_config(cls, config):
        return cls()

    def get_quant_method(self, layer, prefix):
        if isinstance(layer, LinearBase):
            return ExactLinearMethod()
        if LMHEAD and isinstance(layer, ParallelLMHead):
            return ExactLMHeadMethod()
        return None
