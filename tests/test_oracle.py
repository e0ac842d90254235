"""CPU: the numpy oracle pinned against the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from conftest import golden_cases
from oracle import qr_oracle as O

# Cases whose trailing reflectors are ill-determined (rank-deficient subspaces):
# H is not unique there, so they are compared through the property gates only.
DEGENERATE = {"nearrank", "nearcollinear"}


@pytest.mark.parametrize("name,case", golden_cases())
def test_oracle_matches_reference_v1(golden, name, case):
    A = golden[f"{name}/A"]
    H1, t1 = golden[f"{name}/H_v1"], golden[f"{name}/tau_v1"]
    H, t = O.geqr2(A)
    ok, info = O.check_implementation(A, H.astype(np.float32), t.astype(np.float32))
    assert ok, info
    if case in DEGENERATE:
        return
    scale = np.abs(A).max() + 1e-30
    assert np.abs(H - H1).max() / scale < 2e-5
    assert np.abs(t - t1).max() < 2e-5


@pytest.mark.parametrize("name,case", golden_cases())
def test_checker_agrees_with_reference_checker(golden, name, case):
    """numpy check_implementation vs the values reference.check_implementation printed."""
    A = golden[f"{name}/A"]
    ok, info = O.check_implementation(A, golden[f"{name}/H_v1"], golden[f"{name}/tau_v1"])
    assert ok
    ref = golden[f"{name}/chk_v1"]   # factor, reconstruction, triangular, orthogonality (scaled)
    for ours, theirs in ((info["scaled_factor_residual"], ref[0]),
                         (info["scaled_orthogonality_residual"], ref[3])):
        if theirs > 1e-3:
            assert 0.2 < ours / theirs < 5.0, (ours, theirs)
        else:
            assert ours < 1e-2


@pytest.mark.parametrize("n,nb", [(33, 32), (64, 32), (96, 32), (100, 16), (65, 64)])
def test_blocked_equals_unblocked(n, nb):
    A = np.random.default_rng(n).standard_normal((3, n, n))
    H0, t0 = O.geqr2(A)
    H1, t1 = O.blocked_geqrf(A, nb)
    assert np.abs(H0 - H1).max() < 1e-12
    assert np.abs(t0 - t1).max() < 1e-12


@pytest.mark.parametrize("n", [1, 2, 7, 32, 70])
def test_orgqr_matches_householder_product(n):
    A = torch.randn(2, n, n, dtype=torch.float64, generator=torch.Generator().manual_seed(n))
    H, tau = torch.geqrf(A)
    Q_ref = torch.linalg.householder_product(H, tau).numpy()
    Q = O.orgqr(H.numpy(), tau.numpy())
    assert np.abs(Q - Q_ref).max() < 1e-12


def test_larft_is_product_of_reflectors():
    A = np.random.default_rng(5).standard_normal((2, 40, 40))
    H, tau = O.geqr2(A)
    Y = O.unit_lower(H, 0, 40)
    T = O.larft(Y, tau)
    P = np.eye(40) - Y @ T @ np.swapaxes(Y, -1, -2)
    assert np.abs(P - O.orgqr(H, tau)).max() < 1e-12


@pytest.mark.parametrize("name,case", golden_cases())
def test_task_input_restates_reference_generator(golden, name, case):
    from qr_b200.inputs import task_input
    batch, n, cond, seed = (int(x) for x in golden[f"{name}/spec"])
    a = task_input(batch, n, cond, seed, case, device="cpu")
    assert np.array_equal(a.numpy(), golden[f"{name}/A"])


def test_sign_convention_is_the_reference_one(golden):
    """On an exactly upper-triangular input the reference reflects (tau = 2 where
    alpha < 0) instead of LAPACK's tau = 0; the oracle follows the reference."""
    A = golden["upper_b2_n32/A"]
    H, t = O.geqr2(A, dtype=np.float32)
    assert np.array_equal(H, golden["upper_b2_n32/H_v1"])
    assert np.array_equal(t, golden["upper_b2_n32/tau_v1"])


def test_north_star_metrics_on_oracle():
    A = np.random.default_rng(3).standard_normal((2, 48, 48))
    H, tau = O.geqr2(A)
    Q, R = O.orgqr(H, tau), np.triu(H)
    q_ref, r_ref = np.linalg.qr(A)
    m = O.north_star_metrics(A, Q, R, r_ref)
    assert m["recon"] < 1e-13 and m["orth"] < 1e-13 and m["rdiff"] < 1e-12
