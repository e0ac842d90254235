"""qr_b200 -- B200-native batched Householder QR (sm_100a CUDA behind a C ABI).

Public API mirrors the reference's submission interface:

* ``custom_kernel(data) -> (H, tau)``   (torch.geqrf compact form)
* ``form_q(H, tau) -> Q``               (torch.linalg.householder_product)
* ``qr(A) -> (H, tau, Q)``              (both, one library call)
* ``geqrf`` / ``orgqr``                 (aliases with explicit names)
"""
from .ops import custom_kernel, form_q, geqrf, orgqr, qr, qr_host  # noqa: F401
from ._lib import QRBError, lib  # noqa: F401

__all__ = ["custom_kernel", "form_q", "geqrf", "orgqr", "qr", "qr_host", "QRBError", "lib"]
