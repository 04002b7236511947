"""ctypes binding of the C ABI in include/fa_sm100.h (libfa_sm100.so, built in-tree).

This is the exact binding a Python caller of the reference's launch API would
write; it carries no compute of its own. If the library is missing the import
of the product path fails loudly: there is no fallback implementation.
"""
import ctypes
import os
import threading

from .build import LIB_PATH

STATUS_OK = 0
STATUS_INVALID_ARGUMENT = 1001
STATUS_UNSUPPORTED = 1002
STATUS_MISALIGNED = 1003
STATUS_NO_SM100 = 1004
STATUS_DRIVER_ENTRY = 1005
STATUS_TENSOR_MAP = 1006
STATUS_DEVICE_TIMEOUT = 1007
STATUS_HOST_ALLOC = 1008
STATUS_BUILD_MISMATCH = 1009
STATUS_STATIC_TOO_LARGE = 1010

#: Every symbol include/fa_sm100.h declares, with (restype, argtypes).
_VP = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
SIGNATURES = {
    "fa_sm100_fwd": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP]),
    "fa_sm100_fwd_slabs": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _LL, _LL, _VP]),
    "fa_sm100_supported": (_I, [_I]),
    "fa_sm100_query": (_I, [_I, _VP]),
    "fa_sm100_hbm_bytes": (ctypes.c_double, [_I, _I, _I, _I, _I]),
    "fa_sm100_min_bytes": (ctypes.c_double, [_I, _I, _I, _I]),
    "fa_attention_flops": (ctypes.c_double, [_I, _I, _I, _I, _I]),
    "fa_default_scale": (ctypes.c_float, [_I]),
    "fa_sm100_device_status": (_I, [ctypes.POINTER(ctypes.c_uint)]),
    "fa_sm100_status_string": (ctypes.c_char_p, [_I]),
    "fa_sm100_debug_read": (_I, [_VP, ctypes.c_size_t]),
    "fa_sm100_fwd_inject_stall": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, ctypes.c_ulonglong, _VP]),
    "fa_sm100_test_arm_stall": (_I, [ctypes.c_ulonglong]),
    "fa_sm100_test_force_kernel": (_I, [_I]),
    "fa_sm100_test_force_split": (_I, [_I]),
    "fa_sm100_fwd_host": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I]),
    "fa_sm100_release_staging": (_I, []),
    "fa_sm100_fwd_host_static": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP]),
    "fa_sm100_static_staging_bytes": (ctypes.c_size_t, []),
}


class FaTilingInfo(ctypes.Structure):
    """Layout of FaTilingInfo (include/fa_sm100.h), the reference's FusedTilingInfo."""
    _fields_ = [(name, ctypes.c_int) for name in (
        "supported", "block_size", "tile_kv", "rows_per_block", "shared_bytes_per_block",
        "registers_per_thread", "local_bytes_per_thread", "max_blocks_per_sm",
        "device_shared_bytes_per_sm", "shared_limited_blocks_per_sm")]


_lock = threading.Lock()
_lib = None


def library_path():
    return os.environ.get("FA_SM100_LIBRARY", LIB_PATH)


def load():
    """Load libfa_sm100.so once and attach the signatures. Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"the sm_100a extension {path} is not built; run "
                    "`python -m cuda_fused_attention_b200.build` (or __graft_entry__.build())")
            lib = ctypes.CDLL(path)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
        return _lib
