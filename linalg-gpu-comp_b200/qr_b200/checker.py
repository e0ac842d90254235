"""Fast GPU checker for (H, tau) outputs: the reference harness's gate on the device.

Restates reference_repo/reference.py:127-192 ``check_implementation`` -- the same
validations, tolerances (factor 20·n·eps·‖A‖₁, orthogonality 100·n·eps), residuals
and message text -- with one change: Q is formed by this library's orgqr
(``qrb_orgqr_f32``, fp32 like the reference's ``torch.linalg.householder_product``)
instead of householder_product, whose per-matrix cost dominates the reference
harness's per-iteration recheck (eval.py:208-212).  The residuals are then computed in
fp64 on the device exactly as the reference does.

Used by ``bench.py --suite gpumode`` to validate every timed output, and usable as a
drop-in for the harness's ``check_implementation`` on CUDA tensors.
"""
from __future__ import annotations

import torch

from .ops import form_q

_FACTOR_RTOL_FACTOR = 20.0   # reference.py:5
_ORTH_RTOL_FACTOR = 100.0    # reference.py:6
_EPS = torch.finfo(torch.float32).eps


def _l1(x: torch.Tensor) -> torch.Tensor:
    return torch.linalg.matrix_norm(x.double(), ord=1, dim=(-2, -1))


def _scaled(residual: torch.Tensor, scale: torch.Tensor, n: int) -> torch.Tensor:
    return residual / (_EPS * max(n, 1) * scale.clamp_min(1e-30))


def _check_tensor(name, value, shape, device):
    if not isinstance(value, torch.Tensor):
        return f"{name} must be a torch.Tensor"
    if value.shape != shape:
        return f"{name} shape must be {shape}, got {tuple(value.shape)}"
    if value.dtype != torch.float32:
        return f"{name} dtype must be torch.float32, got {value.dtype}"
    if value.device != device:
        return f"{name} must be on {device}, got {value.device}"
    if not torch.isfinite(value).all().item():
        return f"{name} contains NaN or Inf"
    return None


def residuals(a: torch.Tensor, h: torch.Tensor, tau: torch.Tensor) -> dict:
    """The reference checker's residuals (fp64) for a CUDA batch; Q from qrb_orgqr_f32."""
    batch, n, _ = a.shape
    q = form_q(h, tau).double()
    r = torch.triu(h).double()
    a64 = a.double()
    projected = q.transpose(-1, -2) @ a64
    f_res = _l1(r - projected).amax()
    a_scale = _l1(a64).amax()
    eye = torch.eye(n, device=a.device, dtype=torch.float64).expand(batch, n, n)
    o_res = _l1(q.transpose(-1, -2) @ q - eye).amax()
    o_scale = torch.ones((), dtype=torch.float64, device=a.device)   # ‖I‖₁
    t_res = _l1(torch.tril(projected, diagonal=-1)).amax()
    rc_res = _l1(q @ r - a64).amax()
    return {
        "factor_residual": f_res.item(), "factor_allowed": (_FACTOR_RTOL_FACTOR * max(n, 1) * _EPS * a_scale).item(),
        "orth_residual": o_res.item(), "orth_allowed": (_ORTH_RTOL_FACTOR * max(n, 1) * _EPS * o_scale).item(),
        "scaled_factor_residual": _scaled(f_res, a_scale, n).item(),
        "scaled_reconstruction_residual": _scaled(rc_res, a_scale, n).item(),
        "scaled_triangular_residual": _scaled(t_res, a_scale, n).item(),
        "scaled_orthogonality_residual": _scaled(o_res, o_scale, n).item(),
    }


def check_implementation(data: torch.Tensor, output) -> tuple[bool, str]:
    """Same contract as reference.py:127 ``check_implementation`` for CUDA tensors."""
    a = data
    batch, n, _ = a.shape
    factor_rtol = _FACTOR_RTOL_FACTOR * max(n, 1) * _EPS
    orth_rtol = _ORTH_RTOL_FACTOR * max(n, 1) * _EPS
    if not isinstance(output, tuple) or len(output) != 2:
        return False, "output must be a tuple `(H, tau)`"
    h, tau = output
    error = _check_tensor("H", h, (batch, n, n), a.device)
    if error is not None:
        return False, error
    error = _check_tensor("tau", tau, (batch, n), a.device)
    if error is not None:
        return False, error
    res = residuals(a, h, tau)
    if res["factor_residual"] > res["factor_allowed"]:
        return False, ("R - Q.T @ A is too large: "
                       f"residual={res['factor_residual']:.3g}, allowed={res['factor_allowed']:.3g}, "
                       f"scaled={res['scaled_factor_residual']:.3g}")
    if res["orth_residual"] > res["orth_allowed"]:
        return False, ("Q is not orthogonal enough: "
                       f"residual={res['orth_residual']:.3g}, allowed={res['orth_allowed']:.3g}, "
                       f"scaled={res['scaled_orthogonality_residual']:.3g}")
    return True, (f"factor_rtol={factor_rtol:.3g}; "
                  f"orth_rtol={orth_rtol:.3g}; "
                  f"scaled_factor_residual={res['scaled_factor_residual']:.3g}; "
                  f"scaled_reconstruction_residual={res['scaled_reconstruction_residual']:.3g}; "
                  f"scaled_triangular_residual={res['scaled_triangular_residual']:.3g}; "
                  f"scaled_orthogonality_residual={res['scaled_orthogonality_residual']:.3g}; "
                  f"batch={batch}; n={n}")
