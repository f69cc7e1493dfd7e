"""ctypes binding of the sm_100a C ABI (include/vllm_exact_b200.h).

The library is built in-tree (vllm-exact_b200/build.py) next to this file. There is no fallback: if the library is
missing or cannot be loaded, every entry point raises.
"""
import ctypes
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("VLLM_EXACT_B200_LIB", Path(__file__).with_name("libvllm_exact_b200.so")))

EX_OK, EX_ERR_ARG, EX_ERR_ALIGN, EX_ERR_WORKSPACE, EX_ERR_DTYPE, EX_ERR_UNSUPPORTED, EX_ERR_CUDA, EX_ERR_DEVICE = range(8)
EX_DTYPE_F32, EX_DTYPE_BF16, EX_DTYPE_F16 = 0, 1, 2
EX_IPC_HANDLE_BYTES = 64
EX_TP_MAX_WORLD, EX_TP_MAX_BLOCKS = 16, 256


def tp_flag_words(world: int) -> int:
    """int32 flag words per rank of ex_allreduce_epilogue_i64 (EX_TP_FLAG_WORDS)."""
    return world
EX_ALGO_AUTO, EX_ALGO_SIMT, EX_ALGO_TC_I8 = 0, 1, 2
EX_LINEAR_STATIC_WEIGHTS = 0x100  # flag OR-ed into algo (vllm_exact_b200.h)

c_i64, c_i32, c_vp, c_sz, c_f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "ex_version": (ctypes.c_char_p, []),
    "ex_status_string": (ctypes.c_char_p, [c_i32]),
    "ex_last_error_string": (ctypes.c_char_p, []),
    "ex_device_error": (c_i32, [ctypes.POINTER(c_i32)]),
    "ex_digitize": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "ex_row_absmax": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "ex_digitize_given_absmax": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
                                         c_vp]),
    "ex_linear_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64, c_i32, c_i32]),
    "ex_linear": (c_i32, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32,
                          c_i32, c_vp, c_i32, c_i64, c_vp, c_sz, c_i32, c_i32, c_vp]),
    "ex_linear_noalloc": (c_i32, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                  c_i32, c_i32, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp]),
    "ex_linear_noalloc_reset": (c_i32, [c_vp]),
    "ex_linear_noalloc_fill_scratch": (c_i32, [c_i32, c_vp]),
    "ex_linear_partial_i64": (c_i32, [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i32,
                                      c_i32, c_vp, c_i64, c_vp, c_sz, c_i32, c_i32, c_vp]),
    "ex_epilogue_i64": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_vp, c_i32, c_i64, c_vp]),
    "ex_ipc_get_handle": (c_i32, [c_vp, c_vp, ctypes.POINTER(ctypes.c_uint64)]),
    "ex_ipc_open_handle": (c_i32, [c_vp, ctypes.POINTER(c_vp)]),
    "ex_ipc_close_handle": (c_i32, [c_vp]),
    "ex_tp_digitize": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_i32, c_vp, c_i64, c_vp, c_i32, c_i32, c_vp, c_vp,
                               c_i64, c_vp, c_vp, c_vp]),
    "ex_allreduce_epilogue_i64": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_i64, c_i64, c_vp,
                                          c_i32, c_i64, c_vp]),
    "ex_paged_decode_workspace_bytes": (c_sz, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "ex_paged_decode": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i32,
                                c_i32, c_i32, c_i32, c_i32, c_f32, c_i32, c_i32, c_vp, c_i64, c_i64, c_i32, c_vp, c_sz,
                                c_vp]),
    "ex_paged_decode_leading": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp,
                                        c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_f32, c_i32, c_i32, c_vp, c_i64, c_i64,
                                        c_i32, c_vp, c_sz, c_vp]),
}

_LIB = None
ON_DEVICE_ERROR = []  # callables run when device_error() reports an error (e.g. re-zeroing split-K workspaces)


class ExactError(RuntimeError):
    """A C-ABI call returned a status other than EX_OK."""

    def __init__(self, fn, status, detail=""):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {detail}")


def lib():
    """Load (once) and return the library; raises if it is missing."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"vllm-exact B200 library not found at {LIB_PATH}; build it with "
                               "`python vllm-exact_b200/build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def check(fn_name, status):
    if status != EX_OK:
        L = lib()
        detail = L.ex_status_string(status).decode()
        if status == EX_ERR_CUDA:
            detail += ": " + L.ex_last_error_string().decode()
        raise ExactError(fn_name, status, detail)


def device_error() -> int:
    """Synchronize, return and clear the device error word (0 = no bounded wait timed out). On an error, the
    library re-zeroes the static scratch of ex_linear_noalloc and the hooks in ON_DEVICE_ERROR re-zero the split-K
    workspaces this package owns, since a call stopped by a timed-out wait may have left partial sums in them."""
    code = c_i32(0)
    check("ex_device_error", lib().ex_device_error(ctypes.byref(code)))
    if code.value != 0:
        for fn in ON_DEVICE_ERROR:
            fn()
    return code.value
