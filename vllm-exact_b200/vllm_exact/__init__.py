"""vllm-exact on B200: batch-invariant vLLM inference for the Qwen3.5 hybrid architecture, with the two hot paths
(exact INT8 two-digit linear layers and batch-invariant paged decode attention) as hand-written sm_100a kernels.

Drop-in for the reference package (src/vllm_exact/__init__.py:1-68): same import name, same ``enable()`` signature and
returned LLM keyword arguments, same ``quantization="exact_int8"`` plugin and FlashAttention patch.

    import vllm_exact
    kw = vllm_exact.enable(max_model_len=16784)   # must run before importing vllm
    from vllm import LLM
    llm = LLM(model=..., dtype="bfloat16", max_model_len=16784, **kw)

What enable() does (reference __init__.py:32-68):
1. turns on vLLM's batch-invariant mode (VLLM_BATCH_INVARIANT=1) and keeps the engine core in this process
   (VLLM_ENABLE_V1_MULTIPROCESSING=0) so the plugin and the patch apply to it;
2. bypasses vLLM's GDN backend check for batch invariance;
3. registers quantization="exact_int8" (every linear layer, lm_head by default);
4. returns the LLM arguments: prompts never chunked, Triton GDN prefill, FLASH_ATTN backend, no prefix caching;
5. patches FlashAttentionImpl.forward so decode attention uses this package's batch-invariant kernel.
"""
import os
import sys

__version__ = "0.1.0"
_ENABLED = False
TABLES = {"h200": None, "b300": None, "b200": None}  # the B200 kernels pick tiles by shape; no tuning table


def enable(max_model_len, f=14, lm_head=True, attention=True, cfg_table="b200", max_num_batched_tokens=131072):
    """Returns keyword arguments to pass to vllm.LLM(...) (reference __init__.py:32-68).

    max_model_len: same value as passed to LLM (the attention kernel fixes its number of segments from it).
    f: 14 (truncated, 3 digit products; default and fastest) or 15 (4 products).
    cfg_table: accepted for compatibility; the reference's Triton tuning tables have no meaning for the B200 kernels,
      whose tile choice depends only on the shape and never changes results.
    max_num_batched_tokens: must exceed the length of every prompt (chunk boundaries change GDN numerics).
    """
    global _ENABLED
    if _ENABLED:
        raise RuntimeError("vllm_exact.enable() can only be called once")
    if "vllm" in sys.modules:
        raise RuntimeError("vllm_exact.enable() must be called before importing vllm")
    if f not in (14, 15):
        raise ValueError("f must be 14 or 15")
    os.environ["VLLM_BATCH_INVARIANT"] = "1"
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"

    from . import ops, plugin  # registers exact_int8 (first import of vllm happens here)
    plugin.F = ops.F = f
    plugin.TRUNC = ops.TRUNC = f == 14
    plugin.LMHEAD = lm_head
    plugin.load_table(TABLES.get(cfg_table, cfg_table) if cfg_table else None)

    from vllm.v1.attention.backends.gdn_attn import GDNAttentionBackend
    GDNAttentionBackend.supports_batch_invariance = classmethod(lambda cls: True)

    kw = dict(quantization="exact_int8", max_num_batched_tokens=max_num_batched_tokens, enable_prefix_caching=False,
              additional_config={"gdn_prefill_backend": "triton"})
    if attention:
        from . import paged_attn
        paged_attn.MAX_LEN = max_model_len
        paged_attn.install()
        kw["attention_config"] = {"backend": "FLASH_ATTN"}
    _ENABLED = True
    return kw
