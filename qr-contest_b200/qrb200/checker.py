"""On-device float64 gate checker for batches of ``(H, tau)``.

The reference validates a factorization with ``common/oracle.py:156-168`` (``check``) on the
host: ``Q = householder_product(H, tau)``, ``R = triu(H)`` and the two norms

    factor = ||R - Q^T A||_1 / ||A||_1  <  20 n eps32
    ortho  = ||Q^T Q - I||_1            < 100 n eps32

This module runs the same gates in float64 on the device that holds the tensors, chunk by
chunk, so a whole benchmark batch (1536 matrices of n = 512, 65536 of n = 256) can be gated
in the same run as its timing.  It adds the tau-range gate ``tau in [1, 2] +- 1e-6`` that the
sign rule guarantees (reflection_no_reflectors.py:149-158, :192).
"""
from __future__ import annotations

import torch

EPS32 = float(torch.finfo(torch.float32).eps)
TAU_SLACK = 1e-6


def _norm1(X):
    return torch.linalg.matrix_norm(X, ord=1, dim=(-2, -1))


def gates(A, H, tau, chunk: int = 128):
    """Per-matrix ``(factor, ortho, tau_lo, tau_hi)`` float64 tensors of shape ``(b,)``.

    ``A``, ``H``: ``(..., n, n)`` of any float dtype; ``tau``: ``(..., n)``.
    """
    n = A.shape[-1]
    A3, H3, t2 = A.reshape(-1, n, n), H.reshape(-1, n, n), tau.reshape(-1, n)
    out = ([], [], [], [])
    eye = torch.eye(n, dtype=torch.float64, device=A.device)
    for i in range(0, A3.shape[0], chunk):
        Ad = A3[i:i + chunk].double()
        Hd = H3[i:i + chunk].double()
        td = t2[i:i + chunk].double()
        Q = torch.linalg.householder_product(Hd, td)
        out[0].append(_norm1(torch.triu(Hd) - Q.mT @ Ad) / _norm1(Ad).clamp_min(1e-300))
        out[1].append(_norm1(Q.mT @ Q - eye))
        out[2].append(td.amin(dim=-1))
        out[3].append(td.amax(dim=-1))
    if not out[0]:
        z = torch.zeros(0, dtype=torch.float64, device=A.device)
        return z, z, z, z
    return tuple(torch.cat(x) for x in out)


def summary(A, H, tau, chunk: int = 128) -> dict:
    """Gate summary of a batch: how many matrices pass all three gates, the worst factor and
    orthogonality residuals as multiples of their tolerances, and the tau range."""
    n = A.shape[-1]
    f, o, tlo, thi = gates(A, H, tau, chunk)
    ftol, otol = 20 * n * EPS32, 100 * n * EPS32
    ok = ((f < ftol) & (o < otol) & (tlo >= 1 - TAU_SLACK) & (thi <= 2 + TAU_SLACK)
          & torch.isfinite(f) & torch.isfinite(o))
    return {"n_pass": int(ok.sum()), "n": int(ok.numel()),
            "max_factor_ratio": float(f.max() / ftol) if f.numel() else 0.0,
            "max_ortho_ratio": float(o.max() / otol) if o.numel() else 0.0,
            "tau_min": float(tlo.min()) if tlo.numel() else None,
            "tau_max": float(thi.max()) if thi.numel() else None}
