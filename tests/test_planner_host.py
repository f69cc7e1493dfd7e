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
