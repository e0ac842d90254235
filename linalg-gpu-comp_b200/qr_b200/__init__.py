"""qr_b200 -- B200-native batched Householder QR (sm_100a CUDA behind a C ABI).

Public API mirrors the reference's submission interface:

* ``custom_kernel(data) -> (H, tau)``   (torch.geqrf compact form)
* ``form_q(H, tau) -> Q``               (torch.linalg.householder_product)
* ``qr(A) -> (H, tau, Q)``              (both, one library call)
* ``geqrf`` / ``orgqr``                 (aliases with explicit names)

The ops (and with them ``libqrb200.so``) load on first attribute access, so that
``qr_b200.inputs`` -- the seeded input generators -- can be imported by code that
must not map the library (the CPU reference arm of ``bench.py``).
"""
from __future__ import annotations

import importlib

_OPS = ("custom_kernel", "form_q", "geqrf", "orgqr", "qr", "qr_host")
_LIB = ("QRBError", "lib")

__all__ = [*_OPS, *_LIB]


def __getattr__(name: str):
    if name in _OPS:
        return getattr(importlib.import_module(".ops", __name__), name)
    if name in _LIB:
        return getattr(importlib.import_module("._lib", __name__), name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
