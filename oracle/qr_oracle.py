"""CPU oracle for batched Householder QR -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy, the algorithm the reference submission
computes on its hot path, so the CUDA library can be checked against it.  It is
imported only by ``tests/``, by ``__graft_entry__.smoke()`` and by the CPU legs
of ``bench.py``; the product path (``qr_b200``) never imports or calls it.

Reference algorithm (nshejwalkar/linalg-gpu-comp):

* Householder step convention -- submissions/v1.py:9-38, restated in-kernel at
  submission.py:242-251 (CUDA panel) and submission.py:552-567 (fused small n):
  ``alpha = x[0]``; ``beta = -sign(alpha) * ||x||`` with sign(0) = +1;
  ``v0 = alpha - beta``; ``tau = 2 v0^2 / (v0^2 + ||x[1:]||^2)`` (0 when the
  denominator is 0); ``u = x[1:] / v0`` with ``|v0| < 1e-30 -> v0 := 1``;
  ``H[j, j] = beta``, ``H[j+1:, j] = u``.
* Compact-WY blocking -- submissions/v1.py:41-63: ``Y`` = unit lower
  trapezoidal reflectors of the block, ``T`` upper triangular with
  ``T[j, j] = tau_j`` and ``T[:j, j] = -tau_j T[:j, :j] (Y[:, :j]^T y_j)``;
  trailing update ``A -= Y (T^T (Y^T A))``.
* Output contract -- reference_repo/task.yml:12-27 and reference.py:90-92:
  ``(H, tau)`` in torch.geqrf / LAPACK SGEQRF compact form.
* Q formation -- reference.py:144 (``torch.linalg.householder_product``):
  ``Q = H_0 H_1 ... H_{n-1}`` applied to the identity.
* Correctness gate -- reference.py:5-6, 95-97, 127-192 (``check_implementation``):
  fp64 L1 norms, factor residual ``||R - Q^T A||_1 <= 20 n eps32 ||A||_1`` and
  orthogonality ``||Q^T Q - I||_1 <= 100 n eps32 ||I||_1``.

Parity status: pinned.  ``tests/golden/`` holds fixtures produced by running
the reference's own Python (``reference.generate_input``, ``ref_kernel`` =
``torch.geqrf`` and ``submissions/v1.py:_blocked_wy``) on CPU;
``tests/test_oracle.py`` checks this module against them.
"""
from __future__ import annotations

import numpy as np

EPS32 = float(np.finfo(np.float32).eps)
EPS_V0 = 1e-30  # submissions/v1.py:27 (safe_v0 guard), submission.py:68

FACTOR_RTOL_FACTOR = 20.0   # reference_repo/reference.py:5
ORTH_RTOL_FACTOR = 100.0    # reference_repo/reference.py:6


# ---------------------------------------------------------------------------
# Householder step (submissions/v1.py:9-38)
# ---------------------------------------------------------------------------
def householder_vector(x: np.ndarray):
    """Reflector for a batch of column segments ``x`` of shape (batch, m).

    Returns ``(beta, tau, u)`` where ``u`` (batch, m-1) are the sub-diagonal
    entries of the unit-leading Householder vector.  Follows
    submissions/v1.py:12-29 exactly, including sign(0) = +1 and the
    ``|v0| < 1e-30`` guard.  m == 1 gives tau = 0 (v1.py:14-16).
    """
    x = np.asarray(x)
    m = x.shape[-1]
    if m <= 1:
        return x[..., 0].copy(), np.zeros(x.shape[:-1], x.dtype), x[..., 1:].copy()
    alpha = x[..., 0]
    norm_x = np.sqrt(np.sum(x * x, axis=-1))
    sign_a = np.where(alpha >= 0, 1.0, -1.0).astype(x.dtype)
    beta = -sign_a * norm_x
    v0 = alpha - beta
    v_norm_sq = v0 * v0 + np.sum(x[..., 1:] * x[..., 1:], axis=-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        tau = np.where(v_norm_sq > 0, 2.0 * v0 * v0 / np.where(v_norm_sq > 0, v_norm_sq, 1), 0.0)
    safe_v0 = np.where(np.abs(v0) < EPS_V0, 1.0, v0)
    u = x[..., 1:] / safe_v0[..., None]
    return beta.astype(x.dtype), tau.astype(x.dtype), u.astype(x.dtype)


def geqr2(A: np.ndarray, dtype=np.float64):
    """Unblocked Householder QR of a batch (batch, m, n) -> (H, tau).

    Column-by-column restatement of submissions/v1.py:9-38 applied to every
    column (v1.py:72-76 with one block spanning the matrix).
    """
    H = np.array(A, dtype=dtype, copy=True)
    if H.ndim == 2:
        H = H[None]
    b, m, n = H.shape
    k = min(m, n)
    tau = np.zeros((b, n), dtype=dtype)
    for j in range(k):
        beta, t, u = householder_vector(H[:, j:, j])
        if j + 1 < n:
            # w = v^T A[j:, j+1:] with v = [1, u]
            w = H[:, j, j + 1:] + np.einsum("bi,bic->bc", u, H[:, j + 1:, j + 1:])
            H[:, j, j + 1:] -= t[:, None] * w
            H[:, j + 1:, j + 1:] -= t[:, None, None] * u[:, :, None] * w[:, None, :]
        H[:, j, j] = beta
        H[:, j + 1:, j] = u
        tau[:, j] = t
    return H, tau


# ---------------------------------------------------------------------------
# Compact WY (submissions/v1.py:41-63)
# ---------------------------------------------------------------------------
def unit_lower(H: np.ndarray, k: int, b: int) -> np.ndarray:
    """Y = unit lower trapezoidal block of reflectors H[k:, k:k+b] (v1.py:44-47)."""
    Y = np.tril(H[:, k:, k:k + b], -1)
    idx = np.arange(b)
    Y[:, idx, idx] = 1.0
    return Y


def larft(Y: np.ndarray, tau: np.ndarray) -> np.ndarray:
    """Forward column-wise T factor: I - Y T Y^T = H_0 ... H_{b-1} (v1.py:48-56)."""
    batch, _, b = Y.shape
    G = np.einsum("bri,brj->bij", Y, Y)
    T = np.zeros((batch, b, b), dtype=Y.dtype)
    for j in range(b):
        T[:, j, j] = tau[:, j]
        if j > 0:
            T[:, :j, j] = -tau[:, j, None] * np.einsum("bik,bk->bi", T[:, :j, :j], G[:, :j, j])
    return T


def blocked_geqrf(A: np.ndarray, nb: int = 32, dtype=np.float64):
    """Right-looking blocked Householder QR (v1.py:66-79; panel width ``nb``).

    Panel by unblocked steps, then ``A_trail -= Y (T^T (Y^T A_trail))``
    (v1.py:59-63).  Mathematically identical to :func:`geqr2`.
    """
    H = np.array(A, dtype=dtype, copy=True)
    batch, n, _ = H.shape
    tau = np.zeros((batch, n), dtype=dtype)
    for k in range(0, n, nb):
        b = min(nb, n - k)
        Hp, tp = geqr2(H[:, k:, k:k + b], dtype=dtype)
        H[:, k:, k:k + b] = Hp
        tau[:, k:k + b] = tp[:, :b]
        if k + b < n:
            Y = unit_lower(H, k, b)
            T = larft(Y, tau[:, k:k + b])
            C = np.einsum("bri,brc->bic", Y, H[:, k:, k + b:])
            W = np.einsum("bji,bjc->bic", T, C)          # T^T C
            H[:, k:, k + b:] -= np.einsum("bri,bic->brc", Y, W)
    return H, tau


def orgqr(H: np.ndarray, tau: np.ndarray, dtype=np.float64) -> np.ndarray:
    """Q = H_0 H_1 ... H_{n-1} (reference.py:144, householder_product).

    Backward accumulation on the identity, one reflector at a time.
    """
    H = np.asarray(H, dtype=dtype)
    tau = np.asarray(tau, dtype=dtype)
    batch, m, n = H.shape
    Q = np.broadcast_to(np.eye(m, dtype=dtype), (batch, m, m)).copy()
    for j in range(min(m, n) - 1, -1, -1):
        v = np.concatenate([np.ones((batch, 1), dtype), H[:, j + 1:, j]], axis=1)
        w = np.einsum("bi,bic->bc", v, Q[:, j:, j:])
        Q[:, j:, j:] -= tau[:, j, None, None] * v[:, :, None] * w[:, None, :]
    return Q


# ---------------------------------------------------------------------------
# Correctness gates
# ---------------------------------------------------------------------------
def _l1(x: np.ndarray) -> np.ndarray:
    """Matrix 1-norm (max column abs sum) per batch entry, as reference.py:109-110."""
    return np.abs(x).sum(axis=-2).max(axis=-1)


def check_implementation(A: np.ndarray, H: np.ndarray, tau: np.ndarray):
    """numpy restatement of reference_repo/reference.py:127-192.

    Returns ``(ok, info)`` where ``info`` holds the scaled residuals the
    reference prints.  Q comes from :func:`orgqr` in fp64.
    """
    A = np.asarray(A, np.float64)
    batch, n, _ = A.shape
    eps = EPS32
    factor_rtol = FACTOR_RTOL_FACTOR * max(n, 1) * eps
    orth_rtol = ORTH_RTOL_FACTOR * max(n, 1) * eps
    if not (np.all(np.isfinite(H)) and np.all(np.isfinite(tau))):
        return False, {"error": "non-finite output"}
    Q = orgqr(np.asarray(H, np.float32).astype(np.float64), np.asarray(tau, np.float32))
    R = np.triu(np.asarray(H, np.float64))
    proj = np.swapaxes(Q, -1, -2) @ A
    f_res = _l1(R - proj).max()
    f_scale = _l1(A).max()
    eye = np.eye(n)
    o_res = _l1(np.swapaxes(Q, -1, -2) @ Q - eye).max()
    o_scale = 1.0
    info = {
        "factor_residual": float(f_res),
        "factor_allowed": float(factor_rtol * f_scale),
        "scaled_factor_residual": float(f_res / (eps * max(n, 1) * max(f_scale, 1e-30))),
        "orth_residual": float(o_res),
        "orth_allowed": float(orth_rtol * o_scale),
        "scaled_orthogonality_residual": float(o_res / (eps * max(n, 1))),
    }
    ok = f_res <= factor_rtol * f_scale and o_res <= orth_rtol * o_scale
    return bool(ok), info


def north_star_metrics(A: np.ndarray, Q: np.ndarray, R: np.ndarray, R_ref: np.ndarray | None = None):
    """The three north-star measures (fp64), worst case over the batch.

    * ``recon``: ||QR - A||_F / ||A||_F
    * ``orth``: spectral ||Q^T Q - I||_2
    * ``rdiff``: ||Rs - Rs_ref||_F / ||R_ref||_F with rows sign-normalised so
      diag(R) >= 0 (only when ``R_ref`` is given).
    """
    A = np.asarray(A, np.float64)
    Q = np.asarray(Q, np.float64)
    R = np.asarray(R, np.float64)
    n = A.shape[-1]
    recon = np.linalg.norm(Q @ R - A, axis=(-2, -1)) / np.maximum(np.linalg.norm(A, axis=(-2, -1)), 1e-300)
    orth = np.linalg.norm(np.swapaxes(Q, -1, -2) @ Q - np.eye(n), ord=2, axis=(-2, -1))
    out = {"recon": float(recon.max()), "orth": float(orth.max())}
    if R_ref is not None:
        out["rdiff"] = float(r_sign_normalised_diff(R, R_ref))
    return out


def r_sign_normalised_diff(R: np.ndarray, R_ref: np.ndarray) -> float:
    """max over batch of ||D R - D' R_ref||_F / ||R_ref||_F, D = sign(diag R)."""
    R = np.asarray(R, np.float64)
    R_ref = np.asarray(R_ref, np.float64)
    s = np.where(np.diagonal(R, axis1=-2, axis2=-1) >= 0, 1.0, -1.0)
    s_ref = np.where(np.diagonal(R_ref, axis1=-2, axis2=-1) >= 0, 1.0, -1.0)
    d = np.linalg.norm(s[..., :, None] * R - s_ref[..., :, None] * R_ref, axis=(-2, -1))
    return float((d / np.maximum(np.linalg.norm(R_ref, axis=(-2, -1)), 1e-300)).max())
