"""ctypes binding of libqrb200.so (the C ABI declared in include/qrb200.h).

The shared library is built in-tree by ``build.py`` next to this file.  There is
no fallback: if the library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqrb200.so"

QRB_OK = 0
QRB_ERR_INVALID_ARG = 1
QRB_ERR_UNSUPPORTED = 2
QRB_ERR_WORKSPACE = 3
QRB_ERR_CUDA = 4
QRB_ERR_DEVICE = 5
QRB_MAX_N = 8192

# name -> (restype, argtypes); mirrors include/qrb200.h one to one.
_c_int64, _c_size, _vp, _fp = ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p
SIGNATURES = {
    "qrb_version": (ctypes.c_int, []),
    "qrb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qrb_last_error": (ctypes.c_int, [ctypes.c_char_p, _c_size]),
    "qrb_workspace_size": (_c_size, [_c_int64, ctypes.c_int]),
    "qrb_device_error": (ctypes.c_int, []),
    "qrb_kernel_launches": (_c_int64, [_c_int64, ctypes.c_int, ctypes.c_int]),
    "qrb_geqrf_f32": (ctypes.c_int, [_fp, _fp, _fp, _c_int64, ctypes.c_int, _vp, _c_size, _vp]),
    "qrb_orgqr_f32": (ctypes.c_int, [_fp, _fp, _fp, _c_int64, ctypes.c_int, _vp, _c_size, _vp]),
    "qrb_qr_f32": (ctypes.c_int, [_fp, _fp, _fp, _fp, _c_int64, ctypes.c_int, _vp, _c_size, _vp]),
    "qrb_geqrf_f32_noalloc": (ctypes.c_int, [_fp, _fp, _fp, _c_int64, ctypes.c_int, _vp]),
    "qrb_kernel_timing": (None, [ctypes.c_int]),
    "qrb_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_uint, _vp]),
    "qrb_kernel_timing_report": (_c_size, [ctypes.c_char_p, _c_size]),
    "qrb_host_workspace_size": (_c_size, [_c_int64, ctypes.c_int, ctypes.c_int]),
    "qrb_qr_f32_host": (ctypes.c_int, [_fp, _fp, _fp, _fp, _c_int64, ctypes.c_int, _vp, _c_size, _vp]),
}

_lock = threading.Lock()
_lib = None


class QRBError(RuntimeError):
    """A libqrb200 call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"libqrb200 error {status}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libqrb200.so once (raises if it is not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python build.py` in {LIB_PATH.parent.parent}")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    st = lib().qrb_last_error(buf, len(buf))
    return st, buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != QRB_OK:
        _, msg = last_error()
        raise QRBError(status, msg or lib().qrb_status_string(status).decode())


def kernel_timing_report() -> dict:
    """Per-kernel totals logged since the last report while ``qrb_kernel_timing(1)`` was on:
    ``{name: {"launches", "ms", "bytes", "flops"}}`` (CUDA-event durations)."""
    need = lib().qrb_kernel_timing_report(None, 0)
    buf = ctypes.create_string_buffer(int(need) + 64)
    lib().qrb_kernel_timing_report(buf, len(buf))
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms, by, fl = line.split()
        out[name] = {"launches": int(cnt), "ms": float(ms), "bytes": float(by), "flops": float(fl)}
    return out
