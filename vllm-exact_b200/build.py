"""Build the sm_100a library of vllm-exact B200 in-tree.

    python vllm-exact_b200/build.py            # -> vllm-exact_b200/vllm_exact/libvllm_exact_b200.so

One translation unit (csrc/ex_capi.cu includes every kernel header), compiled by nvcc for sm_100a only, with the
CUDA runtime linked statically so the library has no dependency beyond the driver. The result is written next to
the Python package that loads it, so it travels with the source tree.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "vllm_exact" / "libvllm_exact_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return (sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) +
            [ROOT / "include" / "vllm_exact_b200.h"])


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O3",
           "-cudart", "static", "-I", str(ROOT / "include"), "-I", str(CSRC), *extra,
           str(CSRC / "ex_capi.cu"), "-o", str(OUT) + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    xs = [a for a in sys.argv[1:] if a not in ("-f", "-v")]
    print(build(force="-f" in sys.argv, verbose=True, extra=xs))
