"""ctypes binding of the fe_kv C ABI (include/fe_kv.h).

The library is ``flashengine.cpp_b200/lib/libfe_kv_b200.so``, built in-tree by
``flashengine.cpp_b200/build.py``. There is no fallback: if the library is
missing, :func:`load` raises.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libfe_kv_b200.so")
SHIM_PATH = os.path.join(PKG_DIR, "lib", "libfe_native_cuda_b200.so")

FE_OK = 0
FE_ERR_INVALID_ARGUMENT = 1
FE_ERR_CAPACITY = 2
FE_ERR_CONTEXT = 3
FE_ERR_CUDA = 4
FE_ERR_UNSUPPORTED = 5
FE_ERR_DEVICE = 6
FE_ERR_NO_DEVICE = 7

FE_DTYPE_F16 = 0
FE_DTYPE_BF16 = 1

FE_DEVERR_SLOT_RANGE = 0x1
FE_DEVERR_PAGE_RANGE = 0x2
FE_DEVERR_NTOK_RANGE = 0x4
FE_DEVERR_TIMEOUT = 0x8
FE_DEVERR_SMEM_ALIGN = 0x10
FE_DEVERR_POS_RANGE = 0x20
FE_DEVERR_PLAN = 0x40

FE_MAX_LAYERS = 128

FE_ATTN_LISTS_DECODE = 1
FE_ATTN_LISTS_ROWS = 2
FE_ATTN_LISTS_ALL = 3

# Every function the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
SIGNATURES = {
    "fe_status_string": (ctypes.c_char_p, [_I]),
    "fe_last_error": (ctypes.c_char_p, []),
    "fe_abi_version": (_I, []),
    "fe_device_errors": (_I, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "fe_kv_append": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "fe_kv_copy_blocks": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "fe_kv_clear_pages": (_I, [_P, _I, _P, _I, _I, _I, _I, _I, _P]),
    "fe_kv_gather": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "fe_kv_fork_copies": (_I, [_I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I, ctypes.POINTER(_I)]),
    "fe_attn_plan_create": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "fe_attn_plan_destroy": (_I, [_P]),
    "fe_attn_plan_prepare": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "fe_attn_run": (_I, [_P, _P, _P, _P, _P, _I, _P]),
    "fe_attn_run_lists": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "fe_attn_plan_get_info": (_I, [_P, _P]),
    "fe_attn_plan_create_host": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "fe_attn_plan_debug_meta": (_I, [_P, _P, _I64, ctypes.POINTER(_I64)]),
    "fe_attn_plan_prepare_device": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "fe_step_prepare_device": (_I, [_P, _P, _I, _P, _I, _I, _P, _P, _P]),
    "fe_attn_plan_debug_device_meta": (_I, [_P, _P, _I64, _P]),
    "fe_paged_decode_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fe_rope": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "fe_rope_append": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I64,
                            _P]),
    "fe_accept": (_I, [_P, _P, _P, _I, _I, _P]),
}


class FeError(RuntimeError):
    """A non-zero fe_status from the library."""

    def __init__(self, status: int, what: str, detail: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status}): {detail}")


class PlanInfo(ctypes.Structure):
    _fields_ = [("batch", _I), ("rows", _I), ("decode_items", _I), ("prefill_items", _I),
                ("split_sequences", _I), ("chunk_tiles", _I), ("grid_ctas", _I),
                ("kv_tokens", _I64)]


_lib = None


def load():
    """Load libfe_kv_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `python flashengine.cpp_b200/build.py`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().fe_status_string(int(status)).decode()


def last_error() -> str:
    return load().fe_last_error().decode("utf-8", "replace")


def check(status: int, what: str):
    if status != FE_OK:
        raise FeError(status, what, last_error())
