"""ctypes binding of the C ABI in ``include/tattn.h`` (``libtattn_b200.so``, built in-tree).

The library is loaded lazily on first use. There is no fallback: if it is missing or cannot be
loaded the call raises, so a CPU or library substitute can never run silently in its place.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libtattn_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

TATTN_F16, TATTN_F32 = 0, 1
OK, ERR_INVALID_ARGUMENT, ERR_LAYOUT, ERR_CUDA, ERR_NO_DEVICE, ERR_DEVICE_STATUS, ERR_UNSUPPORTED = range(7)
ERR_TOO_LARGE = 7
BWD_NOALLOC_MAX_ROWS = 4194304  # TATTN_BWD_NOALLOC_MAX_ROWS
DEV_WAIT_TIMEOUT, DEV_ABORTED = 1, 2  # device status word bits (TATTN_DEV_*)

# Every symbol include/tattn.h declares, with its ctypes signature.
_P, _I, _F, _I64P = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_int64)
_U64 = ctypes.c_uint64
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tattn_fwd": (_I, [_P, _P, _P, _P, _P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "tattn_bwd_preprocess": (_I, [_P, _P, _P, _I64P, _I, _I, _I, _I, _I, _P]),
    "tattn_bwd_dkdv": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "tattn_bwd_dq": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _P]),
    "tattn_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64P, _I, _I, _I, _I, _I, _I, _F, _P]),
    "tattn_bwd_fused": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64P, _I, _I, _I, _I, _I, _I, _F, _P]),
    "tattn_bwd_fused_workspace_bytes": (ctypes.c_int64, [_I, _I, _I, _I]),
    "tattn_layout_ok": (_I, [_P, _I64P, _I, _I, _I, _I]),
    "tattn_selftest_exp2": (_I, [_P, _P, _P, _P, _I, _P]),
    "tattn_selftest_exp2_poly4": (_I, [_P, _P, _I, _P]),
    "tattn_selftest_wait": (_I, [_P]),
    "tattn_set_wait_limit_ns": (_I, [_U64]),
    "tattn_get_wait_limit_ns": (_U64, []),
    "tattn_tile_configs": (_I, [_I]),
    "tattn_tile_config_info": (_I, [_I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "tattn_tile_default": (_I, [_I, _I, _I, _I]),
    "tattn_tile_supported": (_I, [_I, _I, _I]),
    "tattn_device_status": (_I, [_P, ctypes.POINTER(ctypes.c_int), _I]),
    "tattn_status_string": (ctypes.c_char_p, [_I]),
    "tattn_abi_version": (_I, []),
}
ABI_VERSION = 3

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class TattnError(RuntimeError):
    """A nonzero status from the CUDA library."""

    def __init__(self, fn: str, code: int, msg: str) -> None:
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the shared library. Raises RuntimeError if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"tattn_b200 CUDA library not found at {path}; build it with "
                "`python triton-attn_b200/build.py` (needs nvcc). There is no CPU fallback."
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.tattn_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{path}: ABI version {lib.tattn_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().tattn_status_string(code).decode()


def check(fn: str, code: int) -> None:
    if code != OK:
        raise TattnError(fn, code, status_string(code))


def strides_array(*stride_tuples: tuple[int, ...]) -> ctypes.Array:
    flat = [int(s) for st in stride_tuples for s in st]
    return (ctypes.c_int64 * len(flat))(*flat)


def device_status(stream: int = 0, clear: bool = True) -> int:
    """Synchronise ``stream`` and return (and by default clear) the device status word bits."""
    out = ctypes.c_int(0)
    check("tattn_device_status", load().tattn_device_status(stream, ctypes.byref(out), int(clear)))
    return out.value
