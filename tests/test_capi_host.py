"""CPU tests of the C-ABI library: it loads without a GPU, exports every symbol the header declares, and rejects bad
arguments with the documented status codes before touching the device (no compute call runs here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "vllm_exact_b200.h"


@pytest.fixture(scope="module")
def L():
    from vllm_exact import _lib
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    return _lib.lib()


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\*?(ex_[a-z_0-9]+)\(", text, re.M)))


def test_header_symbols_exported(L):
    from vllm_exact import _lib
    names = _declared()
    assert len(names) >= 11
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover exactly the header's entry points"


def test_version_and_status_strings(L):
    assert b"sm_100a" in L.ex_version()
    assert L.ex_status_string(0) == b"ok"
    assert L.ex_status_string(3).startswith(b"workspace")


def test_argument_validation_without_gpu(L):
    from vllm_exact import _lib as X
    p = ctypes.c_void_p(16)  # never dereferenced: every call below must fail validation first
    # digitize: bad F, bad dtype, negative rows
    assert L.ex_digitize(p, 1, 64, 4, 64, 13, p, p, 64, p, p, None) == X.EX_ERR_ARG
    assert L.ex_digitize(p, 9, 64, 4, 64, 14, p, p, 64, p, p, None) == X.EX_ERR_DTYPE
    assert L.ex_digitize(p, 1, 64, -1, 64, 14, p, p, 64, p, p, None) == X.EX_ERR_ARG
    assert L.ex_digitize(p, 1, 32, 4, 64, 14, p, p, 64, p, p, None) == X.EX_ERR_ARG  # ldx < K
    assert L.ex_digitize(None, 1, 64, 0, 64, 14, None, None, 64, None, None, None) == X.EX_OK  # empty
    # linear: K beyond the int32-exact range, bad F, bad out dtype, ldo < N
    args = lambda M, N, K, F, od, ldo: (p, p, K, p, p, p, p, K, p, p, M, N, K, F, 1, p, od, ldo, None, 0, 0, 0, None)
    assert L.ex_linear(*args(4, 8, 1 << 17, 14, 1, 8)) == X.EX_ERR_UNSUPPORTED
    assert L.ex_linear(*args(4, 8, 64, 16, 1, 8)) == X.EX_ERR_ARG
    assert L.ex_linear(*args(4, 8, 64, 14, 7, 8)) == X.EX_ERR_DTYPE
    assert L.ex_linear(*args(4, 8, 64, 14, 1, 4)) == X.EX_ERR_ARG
    assert L.ex_linear(*args(0, 8, 64, 14, 1, 8)) == X.EX_OK  # empty batch is a no-op
    # split-K needs a workspace: SIMT with 4 splits, none given
    a = list(args(4, 8, 4096, 14, 1, 8))
    a[20], a[21] = 4, X.EX_ALGO_SIMT
    assert L.ex_linear(*a) == X.EX_ERR_WORKSPACE
    assert L.ex_linear_workspace_bytes(4, 8, 4096, 4, X.EX_ALGO_SIMT) >= 4 * 8 * 8
    assert L.ex_linear_workspace_bytes(4, 8, 4096, 1, X.EX_ALGO_SIMT) == 0
    # epilogue / paged decode
    assert L.ex_epilogue_i64(p, 4, p, p, 4, 8, p, 1, 8, None) == X.EX_ERR_ARG
    pd = lambda H, KV, D, ws, wsb: (p, 64, 32, ctypes.c_void_p(256), ctypes.c_void_p(256), 64, 64, 64, 100, p, 4, p,
                                   2, H, KV, D, 16, 0.1, 4096, 4096, p, 64, 32, 1, ws, wsb, None)
    assert L.ex_paged_decode(*pd(32, 6, 128, None, 0)) == X.EX_ERR_ARG      # H % KV != 0
    assert L.ex_paged_decode(*pd(32, 8, 96, None, 0)) == X.EX_ERR_UNSUPPORTED  # head size
    assert L.ex_paged_decode(*pd(64, 2, 128, None, 0)) == X.EX_ERR_UNSUPPORTED  # 32 query heads per KV head
    assert L.ex_paged_decode(*pd(32, 8, 128, None, 0)) == X.EX_ERR_WORKSPACE
    assert L.ex_paged_decode_workspace_bytes(2, 32, 128, 4096, 4096) >= 2 * 32 * (128 + 2) * 4
    # mixed-step variant: query_start_loc inserted after seq_lens; int32 loads need a 4-byte aligned array
    lead = lambda qsl: pd(32, 8, 128, None, 0)[:12] + (qsl,) + pd(32, 8, 128, None, 0)[12:]
    assert L.ex_paged_decode_leading(*lead(ctypes.c_void_p(18))) == X.EX_ERR_ALIGN
    assert L.ex_paged_decode_leading(*lead(ctypes.c_void_p(16))) == X.EX_ERR_WORKSPACE
    assert L.ex_paged_decode_leading(*lead(None)) == X.EX_ERR_WORKSPACE  # NULL: plain decode of all n requests
    # peer-memory all-reduce + epilogue: rank outside [0, world), world < 1 or > 16, bad dtype, leading dimensions
    # < N, NULL buffers, odd N / leading dimensions (column pairs)
    ar = lambda rank, world, od, ldt, ldo, M=4, N=8, parts=p, outs=p: (parts, ldt, outs, p, p, rank, world, p, p, M,
                                                                      N, p, od, ldo, None)
    assert L.ex_allreduce_epilogue_i64(*ar(2, 2, 1, 8, 8)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 0, 1, 8, 8)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 17, 1, 8, 8)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(-1, 2, 1, 8, 8)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 9, 8, 8)) == X.EX_ERR_DTYPE
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 4, 8)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 8, 4)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 8, 8, M=-1)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 8, 8, parts=None)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 8, 8, outs=None)) == X.EX_ERR_ARG
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 9, 9, N=7)) == X.EX_ERR_ALIGN
    assert L.ex_allreduce_epilogue_i64(*ar(0, 2, 1, 9, 8)) == X.EX_ERR_ALIGN
    # peer-memory row-maxima exchange + digitize: bad F, dtype, rank / world, rows beyond the exchange slots, NULLs
    td = lambda F=14, dt=1, rank=0, world=2, rows=4, max_rows=8, xch=p: (p, dt, 64, rows, 64, F, xch, max_rows, p,
                                                                         rank, world, p, p, 64, p, p, None)
    assert L.ex_tp_digitize(*td(F=13)) == X.EX_ERR_ARG
    assert L.ex_tp_digitize(*td(dt=9)) == X.EX_ERR_DTYPE
    assert L.ex_tp_digitize(*td(rank=2)) == X.EX_ERR_ARG
    assert L.ex_tp_digitize(*td(world=17)) == X.EX_ERR_ARG
    assert L.ex_tp_digitize(*td(rows=9)) == X.EX_ERR_ARG
    assert L.ex_tp_digitize(*td(xch=None)) == X.EX_ERR_ARG
    assert L.ex_tp_digitize(*td(rows=0)) == X.EX_OK  # empty: every rank skips it alike
    # IPC helpers: NULL arguments are rejected before any driver call
    off = ctypes.c_uint64(0)
    assert L.ex_ipc_get_handle(None, ctypes.create_string_buffer(X.EX_IPC_HANDLE_BYTES), ctypes.byref(off)) == X.EX_ERR_ARG
    assert L.ex_ipc_get_handle(p, None, ctypes.byref(off)) == X.EX_ERR_ARG
    assert L.ex_ipc_open_handle(None, ctypes.byref(ctypes.c_void_p())) == X.EX_ERR_ARG
    assert L.ex_ipc_close_handle(None) == X.EX_ERR_ARG


def test_exact_cfgs_parse():
    """Every autotuning candidate is a configuration exact_linear accepts (algorithm, split-K), and reference-style
    tuples keep their meaning (split-K at index 6; either MMA kind at index 7 selects the INT8 tensor cores)."""
    from vllm_exact import kernels as K
    seen = {K._parse_cfg(c) for c in K.EXACT_CFGS}
    assert len(seen) == len(K.EXACT_CFGS)
    assert all(a in (K.EX_ALGO_TC_I8, K.EX_ALGO_SIMT) and sk >= 0 for a, sk in seen)
    assert K._parse_cfg(None) == (K.EX_ALGO_AUTO, 0)
    assert K._parse_cfg((64, 128, 128, 4, 4, 8, 4, 0)) == (K.EX_ALGO_TC_I8, 4)
    assert K._parse_cfg((64, 128, 128, 4, 4, 8, 2, 1)) == (K.EX_ALGO_TC_I8, 2)  # bf16-MMA request: same bits


def test_header_is_plain_c_and_links(tmp_path):
    """tests/c_abi_check.c includes the header as strict C99 (-pedantic-errors), links the library and calls the entry
    points that answer before touching a device: the boundary is a C ABI any FFI can bind, not a C++ one."""
    import shutil
    import subprocess
    from vllm_exact import _lib
    gcc = shutil.which("gcc")
    if gcc is None or not _lib.LIB_PATH.exists():
        pytest.skip("gcc or the built library is missing")
    exe = tmp_path / "c_abi_check"
    libdir = str(_lib.LIB_PATH.parent)
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic-errors", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi_check.c"), "-L", libdir, "-l" + _lib.LIB_PATH.stem[3:],
                    "-Wl,-rpath," + libdir, "-o", str(exe)], check=True, capture_output=True, text=True, timeout=120)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "OK", (r.returncode, r.stdout, r.stderr)
