"""Driver for the drop-in-surface tests. Runs in a fresh interpreter because vllm_exact.enable() must be called before
vLLM is imported (reference __init__.py:44-47). Prints one JSON object with the checks it made.

    python tests/surface_driver.py enable      # CPU: enable() kwargs, registration, patch, guards
    python tests/surface_driver.py plugin      # GPU: exact_int8 linear / lm_head methods and the FA decode patch
    python tests/surface_driver.py worker      # CPU: the vLLM general-plugin entry point in a process without enable()
"""
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "vllm-exact_b200", ROOT / "tests" / "golden"):
    sys.path.insert(0, str(p))


def check_enable():
    import vllm_exact
    out = {}
    kw = vllm_exact.enable(max_model_len=20480)
    out["kwargs"] = kw
    out["env"] = [os.environ.get("VLLM_BATCH_INVARIANT"), os.environ.get("VLLM_ENABLE_V1_MULTIPROCESSING")]
    from vllm.model_executor.layers.quantization import get_quantization_config
    out["quant_config"] = get_quantization_config("exact_int8").__module__
    from vllm.v1.attention.backends import flash_attn as fa
    out["fa_forward_file"] = Path(fa.FlashAttentionImpl.forward.__code__.co_filename).name
    from vllm.v1.attention.backends.gdn_attn import GDNAttentionBackend
    out["gdn_invariant"] = bool(GDNAttentionBackend.supports_batch_invariance())
    from vllm_exact import paged_attn, plugin
    out["max_len"] = paged_attn.MAX_LEN
    out["plugin"] = [plugin.F, plugin.TRUNC, plugin.LMHEAD]
    try:
        vllm_exact.enable(max_model_len=1)
        out["second_call"] = "accepted"
    except RuntimeError as e:
        out["second_call"] = str(e)
    import torch
    out["custom_op"] = str(torch.ops.exactmm.linear)
    # the vLLM general-plugin entry point is discoverable, and running it again in this process changes nothing
    from importlib.metadata import entry_points
    out["entry_points"] = [e.value for e in entry_points(group="vllm.general_plugins") if "vllm_exact" in e.value]
    before = fa.FlashAttentionImpl.forward
    vllm_exact.vllm_plugin()
    out["plugin_idempotent"] = fa.FlashAttentionImpl.forward is before
    out["settings_env"] = json.loads(os.environ[vllm_exact.SETTINGS_ENV])
    return out


def check_worker():
    """A process that never ran enable(), as a vLLM tensor-parallel worker: vLLM calls the general-plugin entry point,
    which applies the settings enable() recorded in the environment."""
    import vllm  # noqa: F401  (a worker has vLLM imported before plugins load)
    import vllm_exact
    vllm_exact.vllm_plugin()
    out = {}
    from vllm.model_executor.layers.quantization import get_quantization_config
    out["quant_config"] = get_quantization_config("exact_int8").__module__
    from vllm.v1.attention.backends import flash_attn as fa
    out["fa_forward_file"] = Path(fa.FlashAttentionImpl.forward.__code__.co_filename).name
    from vllm.v1.attention.backends.gdn_attn import GDNAttentionBackend
    out["gdn_invariant"] = bool(GDNAttentionBackend.supports_batch_invariance())
    from vllm_exact import ops, paged_attn, plugin
    out["max_len"] = paged_attn.MAX_LEN
    out["plugin"] = [plugin.F, plugin.TRUNC, plugin.LMHEAD, ops.F]
    return out


def check_plugin():
    import numpy as np
    import torch
    import vllm_exact
    vllm_exact.enable(max_model_len=20480)
    from types import SimpleNamespace

    import recipes as R
    from oracle import exact_oracle as O
    from vllm_exact import paged_attn as P, plugin
    dev = torch.device("cuda", 0)
    out = {}
    cfg = plugin.ExactInt8Config()
    # linear layer: weights loaded as bf16, digitized after loading, apply() = exact linear (+ bias)
    x, w = R.config1()
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(w.to(dev), requires_grad=False)
    from vllm.model_executor.layers.linear import ReplicatedLinear
    m = cfg.get_quant_method(ReplicatedLinear.__new__(ReplicatedLinear), "layer.0")
    out["linear_method"] = type(m).__name__
    m.process_weights_after_loading(layer)
    out["buffers"] = sorted(n for n, _ in layer.named_buffers())
    y = m.apply(layer, x.to(dev).view(2, 4, 1024))  # (*, K) input keeps its leading shape
    out["shape"] = list(y.shape)
    out["config1_sha_ok"] = R.sha(y.reshape(8, 1024)) == "5e328d30f41524bb3806f02788b2372938a9d3579577fd71aa83e1a18faf4e39"
    bias = torch.randn(1024, device=dev).bfloat16()
    yb = m.apply(layer, x.to(dev), bias)
    out["bias_ok"] = bool(torch.equal(yb, y.reshape(8, 1024) + bias))
    # optional release of the bf16 weight after digitization: apply() gives the same bits without it
    plugin.DROP_BF16_WEIGHT = True
    layer2 = torch.nn.Module()
    layer2.weight = torch.nn.Parameter(w.to(dev), requires_grad=False)
    m.process_weights_after_loading(layer2)
    plugin.DROP_BF16_WEIGHT = False
    out["dropped_weight_shape"] = list(layer2.weight.shape)
    out["dropped_same_bits"] = bool(torch.equal(m.apply(layer2, x.to(dev).view(2, 4, 1024)), y))
    from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead
    lm = cfg.get_quant_method(ParallelLMHead.__new__(ParallelLMHead), "lm_head")
    out["lm_head_method"] = type(lm).__name__
    # the patched FlashAttentionImpl.forward, pure decode step, vLLM 0.22 cache layout (2, nb, BS, KV, D)
    from vllm.v1.attention.backends import flash_attn as fa
    n, H, KV, D, BS = 6, 32, 8, 128, 16
    q, kv, bt, sl = R.paged_case(n, 900, BS, H, KV, D, ctx_jitter=True)
    kc, vc = R.kv_views(kv, D)
    cache = torch.stack([kc.contiguous(), vc.contiguous()]).to(dev)
    impl = SimpleNamespace(attn_type=fa.AttentionType.DECODER, head_size=D, num_heads=H, scale=D ** -0.5)
    meta = SimpleNamespace(max_query_len=1, num_actual_tokens=n, block_table=bt.to(dev), seq_lens=sl.to(dev),
                           max_seq_len=int(sl.max()), query_start_loc=torch.arange(n + 1, device=dev))
    output = torch.full((n + 2, H * D), 7.0, device=dev, dtype=torch.bfloat16)  # 2 padding rows stay untouched
    qd = q.to(dev)
    fa.FlashAttentionImpl.forward(impl, None, qd, None, None, cache, meta, output)
    ref = torch.empty(n, H, D, device=dev, dtype=torch.bfloat16)
    P.paged_decode(qd, cache[0], cache[1], bt.to(dev), sl.to(dev), D ** -0.5, ref, n)
    out["patch_matches_kernel"] = bool(torch.equal(output[:n].view(n, H, D), ref))
    out["padding_untouched"] = bool((output[n:] == 7.0).all())
    f = lambda t: t.detach().cpu().float().numpy()
    o_ref = O.paged_decode(f(q), f(kc), f(vc), bt.numpy(), sl.numpy(), D ** -0.5, n)
    out["patch_max_err"] = float(np.abs(f(output[:n].view(n, H, D)) - o_ref).max())
    # mixed prefill + decode step: vLLM's own forward (stubbed here: it fills the output with 3.0) runs first, then
    # the leading one-token requests (3 of ql = 1,1,1,4,1,2) are overwritten by the kernel without a host sync
    fa.FlashAttentionImpl.forward = lambda self, layer, query, key, value, kv_cache, md, output, *a: output.fill_(3.0)
    P.install()
    ql = [1, 1, 1, 4, 1, 2]
    qsl = torch.tensor([0] + list(np.cumsum(ql)), dtype=torch.int32, device=dev)
    meta.max_query_len, meta.num_actual_tokens, meta.query_start_loc = 4, int(qsl[-1]), qsl
    T = int(qsl[-1])
    qm = torch.randn(T, H, D, generator=torch.Generator().manual_seed(3)).bfloat16().to(dev)
    qm[:n] = qd
    outm = torch.full((T, H * D), 7.0, device=dev, dtype=torch.bfloat16)
    fa.FlashAttentionImpl.forward(impl, None, qm, None, None, cache, meta, outm)
    nd = O.leading_decodes(qsl.cpu().numpy())
    out["mixed_nd"] = nd
    out["mixed_decodes_match"] = bool(torch.equal(outm[:nd].view(nd, H, D), ref[:nd]))
    out["mixed_rest_from_vllm"] = bool((outm[nd:] == 3.0).all())
    return out


if __name__ == "__main__":
    mode = sys.argv[1]
    res = {"enable": check_enable, "plugin": check_plugin, "worker": check_worker}[mode]()
    print("SURFACE_JSON " + json.dumps(res), flush=True)
