"""Config 5 through the real vLLM engine with tensor parallelism (TP = 2): 16 target sequences
(1,024-token random prompts, 256 generated tokens, greedy and temperature 1.0 with per-request seeds) give bitwise the
same tokens and logprobs alone and interleaved into a batch of 64, on 2 GPUs. exact_int8 and the attention patch reach
vLLM's tensor-parallel worker processes through the package's general-plugin entry point; row-parallel layers take
the exact int64 path. A 4-layer model of the configs[4] widths (3 Gated-DeltaNet layers + 1 full-attention layer,
dummy weights) keeps the run short. Skipped with fewer than 2 GPUs. The method is bench.py --case engine (the
reference's scripts/check_invariance.py)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_engine_tp2_targets_bitwise_alone_and_batched():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--case", "engine:exact:tp=2:layers=4:inv"],
                       capture_output=True, text=True, timeout=1800, cwd=str(ROOT), env=env)
    lines = [l for l in p.stdout.splitlines() if l.startswith("ENGINE_JSON ")]
    assert p.returncode == 0 and lines, p.stdout[-3000:] + p.stderr[-6000:]
    res = json.loads(lines[-1][len("ENGINE_JSON "):])
    assert res["tp"] == 2
    inv = res["invariance"]
    assert set(inv) == {"T1.0", "T0.0"}
    for t, r in inv.items():
        assert r["A_vs_B_tokens_logprobs"] == "16/16, 16/16", (t, r)
        assert r["A_vs_C_tokens_logprobs"] == "16/16, 16/16", (t, r)
