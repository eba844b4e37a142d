"""ctypes binding of libhoa.so (the C ABI declared in include/hoa.h).

The library is the only compute path: if it cannot be loaded, every op raises.
There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libhoa.so")

HOA_F32, HOA_BF16 = 0, 1
HOA_GEN_BANKED = 0x100        # generator layout flag OR'ed into a_dtype
# status codes (include/hoa.h)
(HOA_OK, HOA_ERR_INVALID_ARG, HOA_ERR_UNSUPPORTED, HOA_ERR_LAUNCH, HOA_ERR_WORKSPACE, HOA_ERR_TIMEOUT,
 HOA_ERR_BOUNDS) = range(7)

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/hoa.h
SIGNATURES = {
    "hoa_abi_version": (c_int, []),
    "hoa_max_head_dim": (c_int, []),
    "hoa_status_string": (ctypes.c_char_p, [c_int]),
    "hoa_plan_chunk": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "hoa_gen_stride": (c_int, [c_int, c_int]),
    "hoa_gen_banked_map": (c_int, [c_int, c_void_p]),
    "hoa_core_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "hoa_core_forward": (c_int, [c_void_p, c_int, c_void_p, c_float, c_void_p, c_int, c_void_p, c_int, c_int,
                                 c_float, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                 c_void_p, c_size_t, c_void_p]),
    "hoa_link_local": (c_int, [c_void_p, c_int, c_void_p, c_float, c_void_p, c_int, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "hoa_carry_scan": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                               c_void_p]),
    "hoa_carry_apply": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                c_int, c_int, c_int, c_int, c_void_p]),
    "hoa_vt_stride": (c_int, [c_int]),
    "hoa_attn_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_int, c_int,
                             c_int, c_int, c_int, c_void_p]),
    "hoa_attn_tc_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int,
                                c_int, c_int, c_int, c_int, c_void_p]),
    "hoa_attn_general_fwd": (c_int, [c_void_p] * 7 + [c_float, c_int, c_int, c_int, c_void_p]),
    "hoa_chain_matvec": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "hoa_apply_paths": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                c_void_p]),
    "hoa_edge_gelu_split": (c_int, [c_void_p, c_void_p, ctypes.c_longlong, c_int, c_int, c_void_p]),
    "hoa_compose_paths": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "hoa_out_transport": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int,
                                  c_int, c_int, c_int, c_void_p]),
    "hoa_core_forward_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_float, c_void_p, c_int, c_void_p, c_int,
                                         c_int, c_float, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_int, c_int, c_void_p]),
    "hoa_noalloc_status_word": (c_int, [ctypes.POINTER(c_void_p)]),
    "hoa_set_wait_bound": (c_int, [ctypes.c_longlong]),
    "hoa_debug_bounds": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "hoa_selftest_wait": (c_int, [c_void_p, ctypes.c_longlong, c_void_p]),
    "hoa_edge_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                              c_size_t, c_void_p]),
    "hoa_edge_gelu_split8": (c_int, [c_void_p, c_void_p, c_void_p, ctypes.c_longlong, c_int, c_float,
                                     c_void_p]),
    "hoa_edge_gemm_fp8_acc": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_void_p,
                                      c_size_t, c_void_p]),
}

_lock = threading.Lock()
_lib = None


class HoaError(RuntimeError):
    """A libhoa entry point returned a non-zero hoa_status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


DEBUG_LIB_PATH = os.path.join(_PKG, "libhoa_debug.so")


def _declare(lib):
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load(path: str = LIB_PATH):
    """Load libhoa.so (once) and declare every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m holonomyawareattention_b200._build` "
                "(the CUDA library is the only implementation; there is no fallback)")
        _lib = _declare(ctypes.CDLL(path))
        return _lib


def load_debug():
    """A handle on libhoa_debug.so (the same C ABI, with the device-side index checks
    of hoa_debug_bounds compiled in); separate from the product library."""
    if not os.path.exists(DEBUG_LIB_PATH):
        raise RuntimeError(f"{DEBUG_LIB_PATH} is missing: build it with "
                           "`python -m holonomyawareattention_b200._build --debug-bounds`")
    return _declare(ctypes.CDLL(DEBUG_LIB_PATH))


def check(fn: str, status: int) -> None:
    if status != 0:
        lib = load()
        raise HoaError(fn, status, lib.hoa_status_string(status).decode())


def call(fn: str, *args) -> None:
    lib = load()
    check(fn, getattr(lib, fn)(*args))
