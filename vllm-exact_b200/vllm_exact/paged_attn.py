"""Batch-invariant paged decode attention on B200 and the patch of vLLM's FlashAttention backend.

Mirrors the reference's src/vllm_exact/paged_attn.py:

* ``paged_decode(query, key_cache, value_cache, block_table, seq_lens, scale, out, n, max_seq_len, ...)``
  (reference paged_attn.py:97-114): same arguments, same in-place write of rows [0, n) of `out`.
* ``install()`` (reference paged_attn.py:135-163): patches ``FlashAttentionImpl.forward`` so decode tokens always go
  through ``paged_decode`` and prefill tokens through vLLM's own implementation.

Kernel parameters are module constants that never depend on the batch (reference paged_attn.py:21-28): SPLIT keys
per segment and the number of segments ceil(MAX_LEN / SPLIT) fix the floating-point reduction order of every
request, so a request's output bits are the same alone, in any batch, and under any placement of its pages.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib

SPLIT = 4096       # keys per segment (fixed per deployment: it sets the reduction order)
MAX_LEN = 16384    # number of segments = ceil(MAX_LEN / SPLIT); enable() sets it to max_model_len
BLK = 64           # kept for signature compatibility; the B200 kernel's key block is fixed by the head size
WARPS = 4
STAGES = 3

_DT = {torch.float32: _lib.EX_DTYPE_F32, torch.bfloat16: _lib.EX_DTYPE_BF16, torch.float16: _lib.EX_DTYPE_F16}


def workspace_bytes(n: int, H: int, D: int, max_len: int | None = None, split: int | None = None) -> int:
    return lib().ex_paged_decode_workspace_bytes(n, H, D, MAX_LEN if max_len is None else max_len,
                                                  SPLIT if split is None else split)


def paged_decode(query, key_cache, value_cache, block_table, seq_lens, scale, out, n, max_seq_len=None, blk=None,
                 warps=None, stages=None, split=None, workspace=None, query_start_loc=None):
    """query (>=n, H, D) bf16; key_cache / value_cache (num_blocks, block_size, KV, D) bf16 views (any strides with a
    contiguous last dimension); block_table (>=n, pages) int32; seq_lens (>=n,) int32; out (>=n, H, D).
    Computes the first n requests only. `max_seq_len`, `blk`, `warps` and `stages` are accepted for signature
    compatibility with the reference; the segment count comes from MAX_LEN as in the reference.

    query_start_loc (int32, >= n + 1 entries; mixed prefill + decode steps): of the first n requests, compute only
    the leading run whose query length is 1 (the requests [0, nd) of reference paged_attn.py:153-159) and leave the
    other rows of `out` untouched. The run is found on the device, so there is no host sync."""
    if n <= 0:
        return out
    tensors = (query, key_cache, value_cache, block_table, seq_lens, out)
    if query_start_loc is not None:
        if query_start_loc.dtype != torch.int32 or query_start_loc.dim() != 1:
            raise TypeError("query_start_loc must be a 1-D int32 tensor")
        if query_start_loc.numel() < n + 1:
            raise ValueError("query_start_loc needs at least n + 1 entries")
        query_start_loc = query_start_loc.contiguous()
        tensors = tensors + (query_start_loc,)
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("paged_decode needs CUDA tensors (there is no CPU fallback)")
    if query.dtype != torch.bfloat16 or key_cache.dtype != torch.bfloat16 or value_cache.dtype != torch.bfloat16:
        raise TypeError("paged_decode expects bf16 query and KV cache")
    if key_cache.stride() != value_cache.stride():
        raise ValueError("key and value caches must share strides")
    if query.stride(2) != 1 or key_cache.stride(3) != 1 or out.stride(2) != 1 or block_table.stride(1) != 1:
        raise ValueError("the head dimension (and block table rows) must be contiguous")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_table and seq_lens must be int32")
    seq_lens = seq_lens.contiguous()
    H, D = query.shape[1], query.shape[2]
    BS, KV = key_cache.shape[1], key_cache.shape[2]
    split = split or SPLIT
    nbytes = workspace_bytes(n, H, D, MAX_LEN, split)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=query.device)
    with torch.cuda.device(query.device):
        check("ex_paged_decode", lib().ex_paged_decode_leading(
            query.data_ptr(), query.stride(0), query.stride(1), key_cache.data_ptr(), value_cache.data_ptr(),
            key_cache.stride(0), key_cache.stride(1), key_cache.stride(2), key_cache.shape[0], block_table.data_ptr(),
            block_table.stride(0), seq_lens.data_ptr(),
            None if query_start_loc is None else query_start_loc.data_ptr(), n, H, KV, D, BS, float(scale),
            MAX_LEN, split, out.data_ptr(), out.stride(0), out.stride(1), _DT[out.dtype], workspace.data_ptr(),
            nbytes, torch.cuda.current_stream(query.device).cuda_stream))
    return out


def kv_views(kv_cache: torch.Tensor, head_size: int):
    """(key_cache, value_cache) as (num_blocks, block_size, KV, D) views of a vLLM FlashAttention KV cache.

    vLLM 0.32 layout [num_blocks, KV, block_size, 2 * D] (reference paged_attn.py:8-9, :145) and vLLM 0.22 layout
    (2, num_blocks, block_size, KV, D) (vllm/v1/attention/backends/flash_attn.py get_kv_cache_shape) are both
    accepted; the kernel reads them through strides."""
    if kv_cache.dim() == 5 and kv_cache.shape[0] == 2:
        return kv_cache[0], kv_cache[1]
    if kv_cache.dim() == 4 and kv_cache.shape[-1] == 2 * head_size:
        return kv_cache.transpose(1, 2).split(head_size, dim=-1)
    raise ValueError(f"unrecognised KV cache layout {tuple(kv_cache.shape)}")


def mixed_step_requests(query_start_loc, block_table, seq_lens, out) -> int:
    """Number of requests handed to the kernel in a mixed step: every request query_start_loc describes, bounded by
    the rows of the block table, seq_lens and the output (shapes only: no device value is read). The kernel then
    computes the leading one-token requests among them."""
    return max(0, min(query_start_loc.shape[0] - 1, block_table.shape[0], seq_lens.shape[0], out.shape[0]))


def install():
    """Patch vLLM's FlashAttentionImpl.forward (call before creating the LLM, with VLLM_ENABLE_V1_MULTIPROCESSING=0).

    Pure decode steps (max_query_len == 1) go entirely through paged_decode (CUDA-graph safe, no host sync). Mixed
    steps run vLLM's implementation first, then overwrite the leading decode tokens (vLLM orders decodes first) with
    paged_decode, so every decode token is always computed by this kernel (reference paged_attn.py:141-160). The
    reference counts those leading decodes on the host (an .item() sync); here the kernel reads query_start_loc and
    finds them itself, so mixed steps are also free of host syncs."""
    from vllm.v1.attention.backends import flash_attn as fa
    if hasattr(fa.FlashAttentionImpl.forward, "_vllm_exact_b200_orig"):
        return fa.FlashAttentionImpl.forward._vllm_exact_b200_orig  # already installed (install is idempotent)
    orig = fa.FlashAttentionImpl.forward
    DEC = fa.AttentionType.DECODER

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if attn_metadata is None or self.attn_type != DEC:
            return orig(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                        output_block_scale)
        D = self.head_size
        key_cache, value_cache = kv_views(kv_cache, D)
        out3 = output.view(output.shape[0], self.num_heads, D)
        if attn_metadata.max_query_len == 1:
            n = attn_metadata.num_actual_tokens
            if n > 0:  # the KV cache write happens outside forward (unified_kv_cache_update) in these vLLM versions
                paged_decode(query, key_cache, value_cache, attn_metadata.block_table, attn_metadata.seq_lens,
                             self.scale, out3, n, attn_metadata.max_seq_len)
            return output
        res = orig(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale, output_block_scale)
        qsl = attn_metadata.query_start_loc
        nreq = mixed_step_requests(qsl, attn_metadata.block_table, attn_metadata.seq_lens, out3)
        if nreq > 0:
            paged_decode(query, key_cache, value_cache, attn_metadata.block_table, attn_metadata.seq_lens,
                         self.scale, out3, nreq, attn_metadata.max_seq_len, query_start_loc=qsl)
        return res

    forward._vllm_exact_b200_orig = orig
    fa.FlashAttentionImpl.forward = forward
    return orig

