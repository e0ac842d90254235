"""CPU baseline for the batched QR path -- test / benchmark infrastructure only.

The reference names CPU ``torch.linalg.qr`` as the comparator for this path
(the harness's own oracle kernel is ``torch.geqrf``, reference_repo/reference.py:90-92,
and its checker forms Q with ``torch.linalg.householder_product``,
reference.py:144).  ``bench.py --impl reference`` and the ``cpu_baseline`` leg
of the default bench time :func:`cpu_qr` on the host cores.  Never imported by
the product package.
"""
from __future__ import annotations

import os
import time

import torch


def set_threads(threads: int | None = None) -> int:
    n = int(threads or os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def cpu_qr(A: torch.Tensor):
    """Full QR on the CPU: (Q, R) = torch.linalg.qr(A) (LAPACK sgeqrf + sorgqr)."""
    return torch.linalg.qr(A, mode="reduced")


def cpu_geqrf_q(A: torch.Tensor):
    """The reference contract on CPU: (H, tau) = geqrf(A), Q = householder_product(H, tau)."""
    H, tau = torch.geqrf(A)
    return H, tau, torch.linalg.householder_product(H, tau)


def time_cpu_qr(A: torch.Tensor, min_seconds: float = 2.0, max_iters: int = 1000):
    """Time :func:`cpu_qr` on ``A`` (a CPU tensor); returns seconds per call (mean)."""
    cpu_qr(A)  # warm-up (first call initialises LAPACK workspaces)
    iters, t0 = 0, time.perf_counter()
    while True:
        cpu_qr(A)
        iters += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or iters >= max_iters:
            return el / iters
