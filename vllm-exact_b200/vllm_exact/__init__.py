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
import json
import os
import sys

__version__ = "0.1.0"
_ENABLED = False
TABLES = {"h200": None, "b300": None, "b200": None}  # the B200 kernels pick tiles by shape; no tuning table
# enable()'s settings, recorded for vLLM's other processes (tensor-parallel workers), which never run enable()
SETTINGS_ENV = "VLLM_EXACT_B200_SETTINGS"
_APPLIED = None


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
    settings = {"f": f, "lm_head": lm_head, "attention": attention, "max_model_len": max_model_len,
                "cfg_table": TABLES.get(cfg_table, cfg_table) if cfg_table else None}
    os.environ[SETTINGS_ENV] = json.dumps(settings)
    _apply(settings)

    kw = dict(quantization="exact_int8", max_num_batched_tokens=max_num_batched_tokens, enable_prefix_caching=False,
              additional_config={"gdn_prefill_backend": "triton"})
    if attention:
        kw["attention_config"] = {"backend": "FLASH_ATTN"}
    _ENABLED = True
    return kw


def _apply(settings: dict) -> None:
    """Register exact_int8 with these settings, bypass the GDN batch-invariance check and install the attention patch
    (steps 2, 3 and 5 of enable()). Idempotent within a process."""
    global _APPLIED
    if _APPLIED is not None:
        if _APPLIED != settings:
            raise RuntimeError(f"vllm_exact already applied with {_APPLIED}, not {settings}")
        return
    from . import ops, plugin  # registers exact_int8 (first import of vllm happens here)
    f = settings["f"]
    plugin.F = ops.F = f
    plugin.TRUNC = ops.TRUNC = f == 14
    plugin.LMHEAD = settings["lm_head"]
    plugin.load_table(settings.get("cfg_table"))

    from vllm.v1.attention.backends.gdn_attn import GDNAttentionBackend
    GDNAttentionBackend.supports_batch_invariance = classmethod(lambda cls: True)
    if settings["attention"]:
        from . import paged_attn
        paged_attn.MAX_LEN = settings["max_model_len"]
        paged_attn.install()
    _APPLIED = dict(settings)


# "module:function" hooks (comma-separated) that vllm_plugin also runs in every vLLM process, for registrations a
# worker process needs as well (e.g. ModelRegistry.register_model of an out-of-tree model class)
EXTRA_PLUGINS_ENV = "VLLM_EXACT_B200_EXTRA_PLUGINS"


def vllm_plugin() -> None:
    """vLLM general-plugin entry point (group ``vllm.general_plugins``, declared in this package's dist-info next to
    it). vLLM runs it in every one of its processes, including the tensor-parallel worker processes, which import
    vLLM afresh and never run enable(): there it applies the settings enable() recorded in the environment, so every
    worker has exact_int8 and the attention patch, and then runs the hooks named in VLLM_EXACT_B200_EXTRA_PLUGINS.
    Without enable() (no recorded settings) it does nothing."""
    s = os.environ.get(SETTINGS_ENV)
    if not s:
        return
    _apply(json.loads(s))
    import importlib
    for hook in filter(None, os.environ.get(EXTRA_PLUGINS_ENV, "").split(",")):
        mod, fn = hook.strip().split(":")
        getattr(importlib.import_module(mod), fn)()
