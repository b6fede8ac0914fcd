"""ctypes binding of libqrb200.so (the C ABI declared in include/qrb200.h).

The library is built in-tree by :mod:`gpumode_qr_b200.build`. Loading fails
loudly when it is missing or stale: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH, build_library, needs_build

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

# Every symbol the public header declares, with its ctypes signature.
_I64, _I32, _P, _SZ = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t
SIGNATURES: dict[str, tuple] = {
    "qrb_version": (ctypes.c_int, []),
    "qrb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qrb_max_n": (_I32, []),
    "qrb_workspace_bytes": (_SZ, [_I64, _I32]),
    "qrb_route": (ctypes.c_int, [_I64, _I32, _SZ]),
    "qrb_geqrf_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I32, _P, _SZ, _P]),
    "qrb_geqrf_f32_noalloc": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I32, _P]),
    "qrb_host_workspace_bytes": (_SZ, [_I64, _I32]),
    "qrb_orgqr_workspace_bytes": (_SZ, [_I64, _I32]),
    "qrb_orgqr_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _I32, _P, _I64, _I32, _P, _SZ, _P]),
    "qrb_ormqr_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32,
                                     _I32, _P, _SZ, _P]),
    "qrb_gram_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I32, _I32, _P]),
    "qrb_gram_geqrf_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I32, _I32, _P, _SZ, _P]),
    "qrb_geqrf_f32_host": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _P, _SZ, _I32, _P]),
    "qrb_fused_qr_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I32, _P]),
    "qrb_fused_max_n": (_I32, []),
    "qrb_panel_qr_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "qrb_larfb_f32": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P]),
    "qrb_set_config": (ctypes.c_int, [ctypes.c_char_p, _I64]),
    "qrb_get_config": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_I64)]),
}


class QRBError(RuntimeError):
    """A libqrb200 entry point returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def lib() -> ctypes.CDLL:
    """Return the loaded library, building it first if it is absent or stale.

    ``QRB200_NO_BUILD=1`` forbids the build step (the library must already be
    present, as on a machine without nvcc).
    """
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if os.environ.get("QRB200_NO_BUILD") != "1" and needs_build():
            build_library()
        if not LIB_PATH.exists():
            raise ImportError(
                f"libqrb200.so not found at {LIB_PATH}; run `python -m gpumode_qr_b200.build`"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
        return _lib


def status_string(status: int) -> str:
    return lib().qrb_status_string(int(status)).decode()


def check(status: int) -> None:
    if status != 0:
        raise QRBError(status, status_string(status))


def set_config(key: str, value: int) -> None:
    check(lib().qrb_set_config(key.encode(), int(value)))


def get_config(key: str) -> int:
    out = ctypes.c_int64(0)
    check(lib().qrb_get_config(key.encode(), ctypes.byref(out)))
    return int(out.value)
