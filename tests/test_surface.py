"""The drop-in surface (reference __init__.py:32-68, plugin.py:105-133, paged_attn.py:135-163), each check in a fresh
interpreter (tests/surface_driver.py) because enable() must run before vLLM is imported."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _run(mode, timeout=600, env=None):
    p = subprocess.run([sys.executable, str(ROOT / "tests" / "surface_driver.py"), mode], capture_output=True,
                       text=True, timeout=timeout, cwd=str(ROOT), env=env)
    lines = [l for l in p.stdout.splitlines() if l.startswith("SURFACE_JSON ")]
    assert p.returncode == 0 and lines, p.stdout[-2000:] + p.stderr[-4000:]
    return json.loads(lines[-1][len("SURFACE_JSON "):])


def test_enable_returns_reference_kwargs_and_installs_everything():
    r = _run("enable")
    assert r["kwargs"] == {"quantization": "exact_int8", "max_num_batched_tokens": 131072,
                           "enable_prefix_caching": False, "additional_config": {"gdn_prefill_backend": "triton"},
                           "attention_config": {"backend": "FLASH_ATTN"}}
    assert r["env"] == ["1", "0"]
    assert r["quant_config"] == "vllm_exact.plugin"
    assert r["fa_forward_file"] == "paged_attn.py"
    assert r["gdn_invariant"] is True
    assert r["max_len"] == 20480
    assert r["plugin"] == [14, True, True]
    assert "only be called once" in r["second_call"]
    assert r["custom_op"] == "exactmm.linear"
    assert r["entry_points"] == ["vllm_exact:vllm_plugin"]
    assert r["plugin_idempotent"] is True
    assert r["settings_env"] == {"f": 14, "lm_head": True, "attention": True, "max_model_len": 20480,
                                 "cfg_table": None}


def test_general_plugin_applies_settings_in_worker_processes():
    """vLLM's tensor-parallel workers import vLLM afresh and never run enable(); the package's general-plugin entry
    point (run by vLLM in every process) applies the settings enable() recorded in the environment."""
    import os
    env = dict(os.environ)
    env["VLLM_EXACT_B200_SETTINGS"] = json.dumps({"f": 15, "lm_head": False, "attention": True,
                                                  "max_model_len": 4096, "cfg_table": None})
    env["VLLM_BATCH_INVARIANT"] = "1"
    r = _run("worker", env=env)
    assert r["quant_config"] == "vllm_exact.plugin"
    assert r["fa_forward_file"] == "paged_attn.py"
    assert r["gdn_invariant"] is True
    assert r["max_len"] == 4096
    assert r["plugin"] == [15, False, False, 15]


def test_enable_after_vllm_import_is_refused():
    code = ("import sys; sys.path.insert(0, 'vllm-exact_b200'); import vllm, vllm_exact\n"
            "try:\n    vllm_exact.enable(max_model_len=16)\nexcept RuntimeError as e:\n    print('REFUSED', e)\n")
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert "REFUSED" in p.stdout and "before importing vllm" in p.stdout


@pytest.mark.gpu
def test_plugin_methods_and_attention_patch_on_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    r = _run("plugin")
    assert r["linear_method"] == "ExactLinearMethod"
    assert r["lm_head_method"] == "ExactLMHeadMethod"
    assert r["buffers"] == ["ex_cw", "ex_sw", "ex_wh", "ex_wl"]
    assert r["shape"] == [2, 4, 1024]
    assert r["config1_sha_ok"] is True
    assert r["bias_ok"] is True
    assert r["dropped_weight_shape"] == [0, 1024] and r["dropped_same_bits"] is True  # DROP_BF16_WEIGHT
    assert r["patch_matches_kernel"] is True and r["padding_untouched"] is True
    assert r["patch_max_err"] < 1e-3
    assert r["mixed_nd"] == 3  # mixed step: leading decodes found on the device, the rest left to vLLM's forward
    assert r["mixed_decodes_match"] is True and r["mixed_rest_from_vllm"] is True


def test_custom_op_fake_impl_for_tracing():
    """exactmm::linear carries a fake implementation (reference plugin.py:67-69), so torch.compile / graph tracing sees
    (*, K) -> (*, N) in x's dtype without running the kernel; checked under FakeTensorMode, no GPU or library needed."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    import vllm_exact.ops  # noqa: F401  (registers the op; importing it loads no library)
    with FakeTensorMode():
        for shape, dt in (((2, 5, 4096), torch.bfloat16), ((7, 4096), torch.float16), ((0, 4096), torch.bfloat16)):
            x = torch.empty(*shape, dtype=dt)
            w = [torch.empty(6144, 4096, dtype=torch.int8) for _ in range(2)]
            s = [torch.empty(6144, dtype=torch.int32) for _ in range(2)]
            y = torch.ops.exactmm.linear(x, w[0], w[1], s[0], s[1])
            assert tuple(y.shape) == shape[:-1] + (6144,) and y.dtype == dt
