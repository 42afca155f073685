"""Loader for the in-tree C-ABI library ``libnvfp4_b200.so`` (include/nvfp4_b200.h).

The library is the only compute path: if it is missing or fails to load,
every entry point raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import threading

_LIB_NAME = "libnvfp4_b200.so"
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)

NVFP4_OK = 0
ERRORS = {
    1: "invalid argument",
    2: "alignment",
    3: "unsupported",
    4: "CUDA error",
    5: "driver error",
    6: "workspace",
}
STATUS = {
    0: "ok",
    1: "producer wait timed out",
    2: "MMA wait timed out",
    3: "epilogue wait timed out",
    4: "teardown drain timed out",
    5: "bad group entry",
}

# Every symbol include/nvfp4_b200.h declares (the ABI test checks this list
# against the header and the shared object).
EXPORTED = (
    "nvfp4_last_error",
    "nvfp4_abi_version",
    "nvfp4_set_timeout_ns",
    "nvfp4_status_get",
    "nvfp4_status_reset",
    "nvfp4_gemm",
    "nvfp4_gemm_ex",
    "nvfp4_grouped_gemm_workspace_size",
    "nvfp4_grouped_gemm",
    "nvfp4_grouped_gemm_ex",
    "nvfp4_grouped_gemm_noalloc",
    "nvfp4_quantize",
    "nvfp4_gemm_multi",
    "nvfp4_ipc_handle_size",
    "nvfp4_ipc_get_handle",
    "nvfp4_ipc_open_handle",
    "nvfp4_ipc_close",
)


class Nvfp4Options(ctypes.Structure):
    _fields_ = [
        ("operand_order", ctypes.c_int),
        ("tile_n", ctypes.c_int),
        ("max_ctas", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("debug", ctypes.c_int),
        ("dev_status", ctypes.c_void_p),
        ("stage_k", ctypes.c_int),
        ("cta_pair", ctypes.c_int),
        ("stream_k", ctypes.c_int),
        ("bias", ctypes.c_void_p),
        ("activation", ctypes.c_int),
        ("out_dtype", ctypes.c_int),
    ]


class Nvfp4Error(RuntimeError):
    pass


_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises ImportError when it is absent."""
    if _lib is not None:
        return _lib
    return _load_slow()


def _load_slow() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            raise ImportError(
                f"{_LIB_NAME} not found next to {__file__}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a)")
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i, sz, ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_ulonglong
        lib.nvfp4_last_error.restype = ctypes.c_char_p
        lib.nvfp4_last_error.argtypes = []
        lib.nvfp4_abi_version.restype = i
        lib.nvfp4_set_timeout_ns.argtypes = [ull]
        lib.nvfp4_status_get.argtypes = [ctypes.POINTER(i)]
        lib.nvfp4_status_reset.argtypes = []
        lib.nvfp4_gemm.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp]
        lib.nvfp4_gemm_ex.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp,
                                      ctypes.POINTER(Nvfp4Options)]
        lib.nvfp4_grouped_gemm_workspace_size.restype = sz
        lib.nvfp4_grouped_gemm_workspace_size.argtypes = [i]
        lib.nvfp4_grouped_gemm.argtypes = [vp, vp, vp, i, vp, sz, vp]
        lib.nvfp4_grouped_gemm_ex.argtypes = [vp, vp, vp, i, vp, sz, vp,
                                              ctypes.POINTER(Nvfp4Options)]
        lib.nvfp4_grouped_gemm_noalloc.argtypes = [vp, vp, vp, i, vp]
        lib.nvfp4_quantize.argtypes = [vp, i, i, i, i, vp, vp, vp, vp]
        lib.nvfp4_gemm_multi.argtypes = [vp, vp, vp, vp, vp, i, ctypes.c_longlong, i, i, i, vp]
        lib.nvfp4_ipc_handle_size.argtypes = []
        lib.nvfp4_ipc_get_handle.argtypes = [vp, vp, ctypes.POINTER(ull)]
        lib.nvfp4_ipc_open_handle.argtypes = [vp, ctypes.POINTER(vp)]
        lib.nvfp4_ipc_close.argtypes = [vp]
        for name in EXPORTED:
            getattr(lib, name)  # AttributeError here means a stale build
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != NVFP4_OK:
        msg = load().nvfp4_last_error().decode(errors="replace")
        raise Nvfp4Error(f"{what} failed ({ERRORS.get(rc, rc)}): {msg}")


def status() -> int:
    """Synchronous read of the current device's status word (0 = no device-side error)."""
    v = ctypes.c_int(0)
    check(load().nvfp4_status_get(ctypes.byref(v)), "nvfp4_status_get")
    return v.value


def status_reset() -> None:
    check(load().nvfp4_status_reset(), "nvfp4_status_reset")


def raise_on_device_error() -> None:
    s = status()
    if s != 0:
        status_reset()
        raise Nvfp4Error(f"device-side error: {STATUS.get(s, s)}")


def options(operand_order=0, tile_n=0, max_ctas=0, timeout_ns=0, debug=0, dev_status=None, stage_k=0,
            cta_pair=0, stream_k=0, bias=None, activation=0, out_dtype=0):
    """Options for the ``*_ex`` entry points; ``dev_status``: device address of an int32 that
    receives this call's device-side error code instead of the per-device status word."""
    return Nvfp4Options(operand_order, tile_n, max_ctas, timeout_ns, debug, dev_status, stage_k,
                        cta_pair, stream_k, bias, activation, out_dtype)
