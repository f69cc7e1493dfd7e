"""CPU check of the tensor-core GEMM's work plan: tests/planner_check.cpp is compiled with g++ against the planner
header the kernel itself uses (vllm-exact_b200/csrc/ex_tc_plan.h) and enumerates 85,050 plans (token tiles, group
partitions, explicit split-K, SM counts from 1 to 148, three cluster-capacity models): every tile's K range covered
exactly once, one distinct in-bounds workspace slot per split tile, and in cluster plans every K part of a tile held
by one cluster. These properties are why every partition gives identical bits."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_tc_plan_covers_every_tile_exactly_once(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "planner_check"
    subprocess.run([gxx, "-O2", "-std=c++17", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-I",
                    str(ROOT / "vllm-exact_b200" / "csrc"), str(ROOT / "tests" / "planner_check.cpp"), "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=300)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    word, plans, segments, cluster_plans = r.stdout.split()
    assert word == "OK" and int(plans) == 85050 and int(segments) > 15_000_000 and int(cluster_plans) > 1000


# The automatic plans of the configs[1] shapes on a 148-SM B200 (clusters in groups of 18 SMs), as measured and
# chosen: M <= 64 qkv / o_proj / down reduce K parts inside clusters of 3-4 CTAs (no workspace), gate_up and lm_head
# take the balanced partition over all 148 SMs with a workspace; at M = 256 o_proj takes 64-token tiles (no split),
# gate_up whole-tile groups of 3 tiles, down 2 K parts in clusters; at M = 4096 groups of 8 sibling m-tiles.
# Columns: M N K BT m_tiles n_tiles KI gs groups chunks G cs ks ws_bytes.
HEADLINE_PLANS = """
1 6144 4096 8 1 48 32 1 144 1 144 3 3 0
1 4096 4096 8 1 32 32 1 128 1 128 4 4 0
1 24576 4096 8 1 192 32 1 148 1 148 1 0 1204992
1 4096 12288 8 1 32 96 1 128 1 128 4 4 0
1 151936 4096 8 1 1187 32 1 148 1 148 1 0 1204992
16 6144 4096 16 1 48 32 1 144 1 144 3 3 0
16 4096 4096 16 1 32 32 1 128 1 128 4 4 0
16 24576 4096 16 1 192 32 1 148 1 148 1 0 2409216
16 4096 12288 16 1 32 96 1 128 1 128 4 4 0
16 151936 4096 16 1 1187 32 1 148 1 148 1 0 2409216
64 6144 4096 64 1 48 32 1 144 1 144 3 3 0
64 4096 4096 64 1 32 32 1 128 1 128 4 4 0
64 24576 4096 64 1 192 32 1 148 1 148 1 0 9634560
64 4096 12288 64 1 32 96 1 128 1 128 4 4 0
64 151936 4096 64 1 1187 32 1 148 1 148 1 0 9634560
256 6144 4096 128 2 48 32 2 48 1 96 1 0 0
256 4096 4096 64 4 32 32 4 32 1 128 1 0 0
256 24576 4096 128 2 192 32 2 64 1 128 1 0 0
256 4096 12288 128 2 32 96 2 64 1 128 4 2 0
256 151936 4096 128 2 1187 32 2 74 1 148 1 0 19137280
4096 6144 4096 128 32 48 32 8 16 4 128 1 0 0
4096 4096 4096 128 32 32 32 8 16 4 128 1 0 0
4096 24576 4096 128 32 192 32 8 18 4 144 1 0 71305472
4096 4096 12288 128 32 32 96 8 16 4 128 1 0 0
4096 151936 4096 128 32 1187 32 8 18 4 144 1 0 71305472
"""


def test_headline_plans_are_the_measured_ones(tmp_path):
    """A change of the planner that changes a headline shape's plan fails here: the plans above are the ones the
    bench measured (bits never depend on the plan, only speed does, so a new plan needs a new measurement)."""
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "planner_check"
    subprocess.run([gxx, "-O2", "-std=c++17", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-I",
                    str(ROOT / "vllm-exact_b200" / "csrc"), str(ROOT / "tests" / "planner_check.cpp"), "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=300)
    r = subprocess.run([str(exe), "dump"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == HEADLINE_PLANS.split()
