"""ctypes wrapper of oracle/exact_oracle_int.c -- TEST INFRASTRUCTURE ONLY.

A second CPU restatement of the reference's integer path (digitize_torch, kernels.py:22-39; exact_linear_torch,
kernels.py:89-100) with integer-only dot products, used by tests to cross-check exact_oracle.py. build() compiles it
with gcc next to this file (ISO C, so no floating-point contraction); __graft_entry__.build() calls it.
"""
from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "exact_oracle_int.c"
LIB = HERE / "libexact_oracle_int.so"
_L = None


def build(out: Path = LIB) -> Path:
    """Compile the C restatement unless the shared library is newer than its source."""
    if out.exists() and out.stat().st_mtime >= SRC.stat().st_mtime:
        return out
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler found for the integer oracle")
    tmp = out.with_name(out.name + ".tmp")
    subprocess.run([cc, "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-Werror", str(SRC), "-o", str(tmp), "-lm"],
                   check=True, capture_output=True, text=True)
    tmp.replace(out)
    return out


def lib():
    global _L
    if _L is None:
        L = ctypes.CDLL(str(build()))
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.eo_digitize.argtypes = [vp, i64, i64, i32, vp, vp, vp, vp, vp]
        L.eo_exact_linear.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, i32, vp, vp]
        _L = L
    return _L


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def digitize(x: np.ndarray, F: int, amax: np.ndarray | None = None):
    """(R, K) float32 -> (h int8, l int8, cs int32, sh int32), as oracle.exact_oracle.digitize."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, K = x.shape
    h = np.empty((R, K), np.int8)
    l = np.empty((R, K), np.int8)
    cs = np.empty(R, np.int32)
    sh = np.empty(R, np.int32)
    am = None if amax is None else np.ascontiguousarray(amax, dtype=np.float32)
    rc = lib().eo_digitize(_p(x), R, K, F, None if am is None else _p(am), _p(h), _p(l), _p(cs), _p(sh))
    if rc != 0:
        raise ValueError("eo_digitize rejected its arguments")
    return h, l, cs, sh


def exact_linear(xd, wd, F: int, trunc: bool = False):
    """(int64 totals, float32 outputs) of the exact linear layer, as exact_oracle.exact_linear_i64 / exact_linear."""
    # every array is bound to a name for the duration of the call (a bare pointer does not keep its array alive)
    xh, xl = (np.ascontiguousarray(t, dtype=np.int8) for t in xd[:2])
    wh, wl = (np.ascontiguousarray(t, dtype=np.int8) for t in wd[:2])
    cx, sx = (np.ascontiguousarray(t, dtype=np.int32) for t in xd[2:])
    cw, sw = (np.ascontiguousarray(t, dtype=np.int32) for t in wd[2:])
    M, K = xh.shape
    N = wh.shape[0]
    if wh.shape[1] != K or xl.shape != xh.shape or wl.shape != wh.shape:
        raise ValueError("digit shapes differ")
    tot = np.empty((M, N), np.int64)
    y = np.empty((M, N), np.float32)
    rc = lib().eo_exact_linear(_p(xh), _p(xl), _p(cx), _p(sx), _p(wh), _p(wl), _p(cw), _p(sw), M, N, K, F,
                               int(bool(trunc)), _p(tot), _p(y))
    if rc != 0:
        raise ValueError("eo_exact_linear rejected its arguments")
    return tot, y
