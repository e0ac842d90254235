"""Seeded input generators for the batched QR workloads.

* :func:`config_input` -- the five benchmark configurations (dense i.i.d. N(0, 1)
  batches, plus the ill-conditioned ``U diag(sigma) V^T`` batch).
* :func:`task_input` -- the reference harness's structured test cases
  (reference_repo/reference.py:23-87 ``generate_input``: dense with column
  scaling, upper, diagonal, rankdef, nearrank, clustered, band, nearcollinear,
  rowscale), restated so GPU tests can build them without the reference tree.

Everything is generated on ``device`` from a ``torch.Generator`` seeded with
``seed``; identical (seed, device type) give identical tensors.
"""
from __future__ import annotations

import torch

# name -> (batch, n, kind); kind "dense" = i.i.d. N(0,1), "illcond" = U diag(s) V^T.
CONFIGS = {
    "b64_n32": (64, 32, "dense"),
    "b4096_n64": (4096, 64, "dense"),
    "b512_n256": (512, 256, "dense"),
    "b32_n2048": (32, 2048, "dense"),
    "b256_n512_illcond": (256, 512, "illcond"),
}


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def haar_orthogonal(batch: int, n: int, gen: torch.Generator, device) -> torch.Tensor:
    """Haar-random orthogonal matrices (fp64): Q of a Gaussian with sign(diag R) folded in."""
    g = torch.randn((batch, n, n), generator=gen, device=device, dtype=torch.float64)
    q, r = torch.linalg.qr(g)
    s = torch.sign(torch.diagonal(r, dim1=-2, dim2=-1))
    s[s == 0] = 1.0
    return q * s.unsqueeze(-2)


def illcond_input(batch: int, n: int, seed: int, device="cuda", decades: float = 6.0) -> torch.Tensor:
    """A = U diag(sigma) V^T, sigma_i = 10^(-decades * i / (n - 1)), built in fp64, cast to fp32."""
    gen = _gen(device, seed)
    u = haar_orthogonal(batch, n, gen, device)
    v = haar_orthogonal(batch, n, gen, device)
    i = torch.arange(n, device=device, dtype=torch.float64)
    sigma = torch.pow(10.0, -decades * i / max(n - 1, 1))
    return ((u * sigma) @ v.transpose(-1, -2)).to(torch.float32).contiguous()


def config_input(name: str, seed: int = 0, device="cuda", batch: int | None = None) -> torch.Tensor:
    """Input batch of benchmark configuration ``name`` (``batch`` overrides its size)."""
    b, n, kind = CONFIGS[name]
    b = b if batch is None else int(batch)
    if kind == "illcond":
        return illcond_input(b, n, seed, device)
    return torch.randn((b, n, n), generator=_gen(device, seed), device=device, dtype=torch.float32)


def _col_scale(a: torch.Tensor, cond: int) -> torch.Tensor:
    if not cond:
        return a
    n = a.shape[-1]
    return a * torch.logspace(0.0, -float(cond), n, device=a.device, dtype=torch.float32)


def task_input(batch: int, n: int, cond: int, seed: int, case: str = "dense", device="cuda") -> torch.Tensor:
    """Structured inputs of the reference harness (reference.py:23-87), same recipes and draw order."""
    if batch <= 0 or n <= 0 or cond < 0:
        raise ValueError("batch and n must be positive, cond non-negative")
    gen = _gen(device, seed)
    f32 = dict(device=device, dtype=torch.float32)
    a = torch.randn((batch, n, n), generator=gen, **f32)
    case = case.lower()
    if case == "dense":
        a = _col_scale(a, cond)
    elif case == "upper":
        a = torch.triu(a)
        a.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.25, n, **f32))
        a = _col_scale(a, cond)
    elif case == "diagonal":
        d = torch.randn((batch, n), generator=gen, **f32)
        d = torch.where(d > 0, 1.0, -1.0) * torch.logspace(0.0, -float(max(cond, 2)), n, **f32)
        a = torch.diag_embed(d)
    elif case == "rankdef":
        a[:, :, max(1, (3 * n) // 4):] = 0.0
        a = _col_scale(a, cond)
    elif case == "nearrank":
        rank = max(1, (3 * n) // 4)
        tail = n - rank
        if tail > 0:
            noise = torch.randn((batch, n, tail), generator=gen, **f32)
            a[:, :, rank:] = a[:, :, :tail] + 1.0e-5 * noise
        a = _col_scale(a, cond)
    elif case == "clustered":
        eps = torch.finfo(torch.float32).eps
        s = torch.ones((n,), **f32)
        s[n // 2:] = 4.0 * eps
        if n >= 8:
            s[max(0, n // 2 - 2):min(n, n // 2 + 2)] = torch.sqrt(torch.tensor(eps, **f32))
        a = a * s
    elif case == "band":
        bw = max(2, min(32, n // 32))
        idx = torch.arange(n, device=device)
        a = a * ((idx[:, None] - idx[None, :]).abs() <= bw)
        a.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.5, n, **f32))
        a = _col_scale(a, cond)
    elif case == "nearcollinear":
        base = torch.randn((batch, n, 1), generator=gen, **f32)
        noise = torch.randn((batch, n, n), generator=gen, **f32)
        a = _col_scale(base.expand(batch, n, n) + 1.0e-4 * noise, cond)
    elif case == "rowscale":
        a = torch.logspace(0.0, -float(max(cond, 4)), n, **f32).reshape(1, n, 1) * a
    else:
        raise ValueError(f"unknown QR test case: {case}")
    return a.contiguous()
