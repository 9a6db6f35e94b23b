"""fp64 gate checker for ``(H, tau)`` -- TEST INFRASTRUCTURE ONLY.

Restates the reference's checker ``common/oracle.py:156-168`` (``check``) and its
per-column variant ``common/oracle.py:171-195`` (``check_percol``):

    Q = householder_product(H, tau)            (LAPACK orgqr; fp64)
    R = triu(H)
    factor = ||R - Q^T A||_1 / ||A||_1  <  20 n eps32
    ortho  = ||Q^T Q - I||_1            < 100 n eps32

plus the tau-range gate ``tau in [1, 2] +- 1e-6`` that the sign rule guarantees
(reflection_no_reflectors.py:117).  Runs on whatever device the tensors live on.
"""
from __future__ import annotations

import torch

EPS32 = float(torch.finfo(torch.float32).eps)
TAU_SLACK = 1e-6


def _m1(X):
    return torch.linalg.matrix_norm(X, ord=1, dim=(-2, -1))


def gates(A, H, tau, chunk: int = 256):
    """Per-matrix ``(factor, ortho, tau_ok)`` as float64 / bool tensors of shape ``(b,)``.

    ``A``, ``H``: ``(..., n, n)``; ``tau``: ``(..., n)``.  Processed in chunks of ``chunk``
    matrices so that large batches fit in memory.
    """
    n = A.shape[-1]
    A3 = A.reshape(-1, n, n)
    H3 = H.reshape(-1, n, n)
    t2 = tau.reshape(-1, n)
    fs, os_, ts = [], [], []
    for i in range(0, A3.shape[0], chunk):
        Ad = A3[i:i + chunk].double()
        Hd = H3[i:i + chunk].double()
        td = t2[i:i + chunk].double()
        Q = torch.linalg.householder_product(Hd, td)
        R = torch.triu(Hd)
        fs.append(_m1(R - Q.mT @ Ad) / _m1(Ad).clamp_min(1e-300))
        I = torch.eye(n, dtype=torch.float64, device=Q.device)
        os_.append(_m1(Q.mT @ Q - I))
        ts.append(((td >= 1 - TAU_SLACK) & (td <= 2 + TAU_SLACK)).all(dim=-1))
    if not fs:
        z = torch.zeros(0, dtype=torch.float64, device=A.device)
        return z, z, torch.zeros(0, dtype=torch.bool, device=A.device)
    return torch.cat(fs), torch.cat(os_), torch.cat(ts)


def check(A, H, tau):
    """Mirror of ``common/oracle.py:156-168``: ``(max_factor, max_ortho, ftol, otol, passed)``.

    ``passed`` also requires the tau gate and finite residuals.
    """
    n = A.shape[-1]
    f, o, t = gates(A, H, tau)
    ftol, otol = 20 * n * EPS32, 100 * n * EPS32
    passed = (f < ftol) & (o < otol) & t & torch.isfinite(f) & torch.isfinite(o)
    fmax = f.max().item() if f.numel() else 0.0
    omax = o.max().item() if o.numel() else 0.0
    return fmax, omax, ftol, otol, passed


def check_percol(A, H, tau, chunk: int = 256):
    """Mirror of ``common/oracle.py:171-195``: per-column-relative factor gate.

    Returns ``(max_ratio, max_ortho, passed)``; ratio < 1 passes.
    """
    n = A.shape[-1]
    A3, H3, t2 = A.reshape(-1, n, n), H.reshape(-1, n, n), tau.reshape(-1, n)
    ftol, otol = 20 * n * EPS32, 100 * n * EPS32
    rs, os_ = [], []
    for i in range(0, A3.shape[0], chunk):
        Ad, Hd, td = A3[i:i + chunk].double(), H3[i:i + chunk].double(), t2[i:i + chunk].double()
        Q = torch.linalg.householder_product(Hd, td)
        res = (torch.triu(Hd) - Q.mT @ Ad).abs().sum(dim=-2)
        acol = Ad.abs().sum(dim=-2).clamp_min(1e-300)
        rs.append((res / (ftol * acol)).amax(dim=-1))
        I = torch.eye(n, dtype=torch.float64, device=Q.device)
        os_.append(_m1(Q.mT @ Q - I))
    r, o = torch.cat(rs), torch.cat(os_)
    passed = (r < 1.0) & (o < otol)
    return r.max().item(), o.max().item(), passed
