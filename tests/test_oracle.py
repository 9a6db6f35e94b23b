"""CPU: the numpy oracle against the reference's own outputs (golden fixtures) and the
structural known answers of the algorithm (reflection_no_reflectors.py)."""
import numpy as np
import pytest
import torch

from oracle import checker, qr_oracle as O
from tests.golden import fixtures as F

NAMES = F.names()


def test_fixtures_present():
    assert len(NAMES) >= 25


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference(name):
    fx = F.load(name)
    A = fx["A"]
    kind = F.kind(name)
    if kind == "c5":
        # bf16 inputs of all six classes: the oracle's float32 factors pass the gates, match
        # the reference's float32 factors where they are determined (dense, upper-triangular)
        # and, rounded to bf16, its bf16 outputs there
        At = torch.from_numpy(A)
        H, tau = O.custom_kernel_np(A)
        f, o, ftol, otol, passed = checker.check(At, torch.from_numpy(H), torch.from_numpy(tau))
        assert bool(passed.all()), (f / ftol, o / otol)
        _, _, _, _, ref_pass = checker.check(At, torch.from_numpy(fx["H32"]),
                                             torch.from_numpy(fx["tau32"]))
        assert bool(ref_pass.all())
        for i in F.C5_TIGHT:
            np.testing.assert_allclose(H[i], fx["H32"][i], rtol=1e-4, atol=1e-4)
            np.testing.assert_allclose(tau[i], fx["tau32"][i], rtol=0, atol=1e-4)
            Hb = torch.from_numpy(H[i]).to(torch.bfloat16).float().numpy()
            np.testing.assert_allclose(Hb, fx["H"][i], rtol=2 ** -7, atol=1e-3)
        return
    if kind == "bf16":
        H, tau = O.custom_kernel(torch.from_numpy(A).to(torch.bfloat16))
        H, tau = H.float().numpy(), tau.float().numpy()
        # one bf16 ulp of the value (2^-7 relative) where the reference and oracle agree
        np.testing.assert_allclose(H, fx["H"], rtol=2 ** -7, atol=1e-3)
        np.testing.assert_allclose(tau, fx["tau"], rtol=2 ** -7, atol=0)
        return
    H, tau = O.custom_kernel_np(A)
    At, Ht, tt = map(torch.from_numpy, (A, H, tau))
    f, o, ftol, otol, passed = checker.check(At, Ht, tt)
    assert bool(passed.all()), (f / ftol, o / otol)
    # the reference itself passes the same gates on these inputs
    _, _, _, _, ref_pass = checker.check(At, torch.from_numpy(fx["H"]), torch.from_numpy(fx["tau"]))
    assert bool(ref_pass.all())
    if kind == "tight":
        np.testing.assert_allclose(H, fx["H"], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(tau, fx["tau"], rtol=0, atol=1e-4)
    elif kind == "loose":
        np.testing.assert_allclose(tau, fx["tau"], rtol=0, atol=F.loose_tol(A.shape[-1]))


def test_lu_pivots_match_torch():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((4, 45, 45)).astype(np.float32)
    LU, perm = O.lu_partial_pivot(A)
    P, L, U = torch.linalg.lu(torch.from_numpy(A))
    assert (P.numpy().transpose(0, 2, 1).argmax(-1) == perm).all()
    np.testing.assert_allclose(O.unit_lower(LU), L.numpy(), atol=1e-4)
    np.testing.assert_allclose(np.triu(LU), U.numpy(), atol=1e-4)


def test_cholesky_and_trsm_match_torch():
    rng = np.random.default_rng(1)
    X = rng.standard_normal((3, 70, 70)).astype(np.float32)
    G = X.transpose(0, 2, 1) @ X + 70 * np.eye(70, dtype=np.float32)
    R, ok = O.cholesky_upper(G)
    assert ok.all()
    Rt = torch.linalg.cholesky(torch.from_numpy(G), upper=True).numpy()
    np.testing.assert_allclose(R, Rt, rtol=1e-4, atol=1e-4)
    Xs = O.trsm_right_upper(X, R)
    Xt = torch.linalg.solve_triangular(torch.from_numpy(Rt), torch.from_numpy(X), upper=True,
                                       left=False).numpy()
    np.testing.assert_allclose(Xs, Xt, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("sign", [1.0, -1.0])
def test_identity_known_answer(sign):
    # A = +-I  ->  d = +-1, s = -+1, pivot 2, Y = 0: H = -+I, tau = 2
    A = sign * np.eye(9, dtype=np.float32)[None].repeat(2, 0)
    H, tau = O.custom_kernel_np(A)
    np.testing.assert_allclose(H, -A, atol=1e-6)
    np.testing.assert_array_equal(tau, 2.0)


def test_upper_triangular_known_answer():
    rng = np.random.default_rng(3)
    A = np.triu(rng.standard_normal((3, 20, 20))).astype(np.float32)
    H, tau = O.custom_kernel_np(A)
    np.testing.assert_array_equal(tau, 2.0)
    np.testing.assert_array_equal(np.tril(H, -1), 0.0)
    f, o, ftol, otol, passed = checker.check(*map(torch.from_numpy, (A, H, tau)))
    assert bool(passed.all())


def test_multiplier_bound():
    # pivot >= 1 caps every multiplier: |Y[i,k]| <= |M[i,k]| <= 1 on an orthonormal frame
    rng = np.random.default_rng(4)
    A = rng.standard_normal((4, 30, 30)).astype(np.float32)
    H, tau = O.custom_kernel_np(A)
    assert np.abs(np.tril(H, -1)).max() <= 1.0 + 1e-5
    assert ((tau >= 1 - 1e-6) & (tau <= 2 + 1e-6)).all()


def test_empty_batch():
    H, tau = O.custom_kernel_np(np.zeros((0, 5, 5), np.float32))
    assert H.shape == (0, 5, 5) and tau.shape == (0, 5)


def test_checker_flags_bad_factors():
    rng = np.random.default_rng(5)
    A = rng.standard_normal((2, 16, 16)).astype(np.float32)
    H, tau = O.custom_kernel_np(A)
    H2 = H.copy()
    H2[:, 0, 5] += 1.0
    _, _, _, _, passed = checker.check(*map(torch.from_numpy, (A, H2, tau)))
    assert not bool(passed.any())
    tau2 = tau.copy()
    tau2[:, 3] = 2.5
    _, _, _, _, passed = checker.check(*map(torch.from_numpy, (A, H, tau2)))
    assert not bool(passed.any())


def test_rect_oracle_factors_tall_matrices():
    # the rectangular restatement: Q R = A with Q = householder_product(H, tau) m x n
    # orthonormal, tau in [1, 2], |diag R| equal to torch.geqrf's; square input = square path
    rng = np.random.default_rng(6)
    for m, n in ((50, 20), (64, 64), (33, 1)):
        A = rng.standard_normal((3, m, n)).astype(np.float32)
        H, tau = O.custom_kernel_rect_np(A)
        Hd, td, Ad = (torch.from_numpy(x).double() for x in (H, tau, A))
        Q = torch.linalg.householder_product(Hd, td)
        R = torch.triu(Hd[:, :n, :])
        assert float((Q @ R - Ad).abs().max()) < 1e-4
        assert float((Q.mT @ Q - torch.eye(n, dtype=torch.float64)).abs().max()) < 1e-5
        assert ((tau >= 1 - 1e-6) & (tau <= 2 + 1e-6)).all()
        Hg, _ = torch.geqrf(torch.from_numpy(A))
        assert torch.allclose(torch.diagonal(R, dim1=-2, dim2=-1).abs().float(),
                              torch.diagonal(Hg[:, :n, :], dim1=-2, dim2=-1).abs(), atol=1e-4)
        if m == n:
            Hs, ts = O.custom_kernel_np(A)
            np.testing.assert_array_equal(H, Hs)
            np.testing.assert_array_equal(tau, ts)
