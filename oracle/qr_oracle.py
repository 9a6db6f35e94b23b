"""CPU restatement (numpy, fp32) of the reference's "reflection without reflectors" QR.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA library: only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``qrb200.custom_kernel``) never calls into this file.

Every function follows one piece of ``reflection_no_reflectors.py`` (file:line below)
and of the LAPACK routines that ``torch.linalg`` dispatches to on CPU.  Those routines
are third-party (torch 2.11.0+cpu links Intel MKL's LAPACK: getrf, potrf, trsm); their
published algorithms are restated here:

* getrf  -- right-looking LU with partial pivoting.  Pivot = first row index holding the
            maximum |a| of the live column (i?amax semantics); an all-zero column is
            left unscaled (getf2 skips the scaling when the pivot is 0).
* potrf  -- upper Cholesky ``G = R^T R`` (column-by-column / blocked, right-looking).
* trsm   -- right, upper, non-transposed solve ``X R = M``.

Parity anchor: ``tests/golden/`` holds inputs and the reference's own outputs made by
importing ``reflection_no_reflectors.custom_kernel`` (script committed beside them);
``tests/test_oracle.py`` pins this restatement against them.

All arithmetic is float32 like the reference (``custom_kernel`` casts to float32,
reflection_no_reflectors.py:183).  Batched: every function takes ``(b, n, n)`` arrays.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _bmm(a, b):
    return np.matmul(a, b)


# --------------------------------------------------------------------------------------
# Stage I-a: partial-pivot LU  (reflection_no_reflectors.py:66, torch.linalg.lu -> getrf)
# --------------------------------------------------------------------------------------
def lu_partial_pivot(A, nb: int = 32):
    """Blocked right-looking LU with partial pivoting of a batch ``A (b,m,n)``, m >= n
    (square for the reference entry point; tall for the rectangular variant).

    Returns ``(LU, perm)``: ``LU`` packs the unit-lower ``L`` (strictly below the
    diagonal) and ``U``; ``perm[b, j]`` is the row of ``A`` that became row ``j`` of
    ``L U`` (``A[perm] = L U``, i.e. ``A = P L U`` with ``P[perm[j], j] = 1``, the
    ``P`` that ``torch.linalg.lu`` returns).
    """
    A = np.array(A, dtype=F32, copy=True)
    b, m, n = A.shape
    perm = np.tile(np.arange(m), (b, 1))
    bi = np.arange(b)
    for k0 in range(0, n, nb):
        k1 = min(k0 + nb, n)
        for k in range(k0, k1):
            col = np.abs(A[:, k:, k])
            p = k + np.argmax(col, axis=1)          # first maximal index (amax semantics)
            # swap full rows k <-> p (getrf applies the swap to the whole row)
            rk = A[bi, k, :].copy()
            A[bi, k, :] = A[bi, p, :]
            A[bi, p, :] = rk
            pk = perm[bi, k].copy()
            perm[bi, k] = perm[bi, p]
            perm[bi, p] = pk
            piv = A[:, k, k]
            nz = piv != 0
            inv = np.where(nz, F32(1.0) / np.where(nz, piv, F32(1.0)), F32(1.0)).astype(F32)
            A[:, k + 1:, k] = np.where(nz[:, None], A[:, k + 1:, k] * inv[:, None],
                                       A[:, k + 1:, k])
            if k + 1 < k1:
                A[:, k + 1:, k + 1:k1] -= A[:, k + 1:, k, None] * A[:, k, None, k + 1:k1]
        if k1 < n:
            # U12 = L11^{-1} A12 (unit-lower forward substitution), then rank-nb update.
            for k in range(k0, k1):
                if k + 1 < k1:
                    A[:, k + 1:k1, k1:] -= A[:, k + 1:k1, k, None] * A[:, k, None, k1:]
            A[:, k1:, k1:] -= _bmm(A[:, k1:, k0:k1], A[:, k0:k1, k1:])
    return A, perm


def unit_lower(LU):
    n = LU.shape[-1]           # m x n: unit lower trapezoidal
    L = np.tril(LU, -1)
    L[:, np.arange(n), np.arange(n)] = 1.0
    return L.astype(F32)


# --------------------------------------------------------------------------------------
# Stage I-c: upper Cholesky  (reflection_no_reflectors.py:76, cholesky(upper=True) -> potrf)
# --------------------------------------------------------------------------------------
def cholesky_upper(G, nb: int = 32):
    """Return ``(R, ok)`` with ``G = R^T R``; ``ok[b]`` False where a pivot was <= 0
    (torch raises ``LinAlgError`` there; the restatement reports it instead)."""
    R = np.triu(np.array(G, dtype=F32, copy=True))
    b, n, _ = R.shape
    ok = np.ones(b, dtype=bool)
    for k0 in range(0, n, nb):
        k1 = min(k0 + nb, n)
        for k in range(k0, k1):
            d = R[:, k, k]
            ok &= d > 0
            r = np.sqrt(np.maximum(d, F32(0))).astype(F32)
            R[:, k, k] = r
            rs = np.where(r > 0, r, F32(1.0))
            R[:, k, k + 1:] /= rs[:, None]
            if k + 1 < k1:
                # within-panel symmetric update (upper part only)
                R[:, k + 1:k1, k + 1:] -= R[:, k, k + 1:k1, None] * R[:, k, None, k + 1:]
        if k1 < n:
            U12 = R[:, k0:k1, k1:]
            R[:, k1:, k1:] -= np.triu(_bmm(np.swapaxes(U12, 1, 2), U12))
    return np.triu(R).astype(F32), ok


# --------------------------------------------------------------------------------------
# Stage I-d: X R = M  (reflection_no_reflectors.py:77, solve_triangular(upper, left=False))
# --------------------------------------------------------------------------------------
def trsm_right_upper(M, R, nb: int = 32):
    X = np.array(M, dtype=F32, copy=True)
    n = R.shape[-1]
    for k0 in range(0, n, nb):
        k1 = min(k0 + nb, n)
        for k in range(k0, k1):
            X[:, :, k] /= R[:, k, k][:, None]
            if k + 1 < k1:
                X[:, :, k + 1:k1] -= X[:, :, k, None] * R[:, k, None, k + 1:k1]
        if k1 < n:
            X[:, :, k1:] -= _bmm(X[:, :, k0:k1], R[:, k0:k1, k1:])
    return X


# --------------------------------------------------------------------------------------
# Stage I: the frame  (reflection_no_reflectors.py:55-81)
# --------------------------------------------------------------------------------------
def cholqr_pass(M):
    """One CholeskyQR pass with the reference's jitter (reflection_no_reflectors.py:68-77)."""
    n = M.shape[-1]
    G = _bmm(np.swapaxes(M, 1, 2), M).astype(F32)
    mu = (F32(1e-7) * np.mean(np.diagonal(G, axis1=1, axis2=2), axis=-1, dtype=F32)).astype(F32)
    idx = np.arange(n)
    G[:, idx, idx] += mu[:, None]
    R, ok = cholesky_upper(G)
    return trsm_right_upper(M, R), ok


def frame(A):
    """``A = P L U``; CholeskyQR2 on ``L``; return ``(P Q, perm, ok)``."""
    LU, perm = lu_partial_pivot(A)
    L = unit_lower(LU)
    Q1, ok1 = cholqr_pass(L)
    Q, ok2 = cholqr_pass(Q1)
    b = Q.shape[0]
    PQ = np.empty_like(Q)
    PQ[np.arange(b)[:, None], perm, :] = Q          # (P Q)[perm[j]] = Q[j]
    return PQ, perm, ok1 & ok2


# --------------------------------------------------------------------------------------
# Stage III: the chart  (reflection_no_reflectors.py:86-176)
# --------------------------------------------------------------------------------------
def chart(Q, bs: int = 32):
    """Sign-rule unpivoted elimination of ``I - Q S`` run on a copy of ``Q``.

    Sign rule (reflection_no_reflectors.py:149-155): ``s_k = +1`` when
    ``|1-d| >= |1+d|`` (so ``d = 0`` gives ``+1``), else ``-1``; pivot ``1 + |d|``;
    multipliers ``Y[i,k] = -s_k M[i,k] / piv`` (:158).  Blocked exactly as :144-174.
    """
    M = np.array(Q, dtype=F32, copy=True)
    b, m, n = M.shape          # m > n: the rectangular chart (irregular/exp1_irregular.py:106-122)
    Y = np.zeros_like(M)
    s = np.ones((b, n), dtype=F32)
    for k0 in range(0, n, bs):
        k1 = min(k0 + bs, n)
        for k in range(k0, k1):
            d = M[:, k, k]
            pp = F32(1.0) - d
            pm = F32(1.0) + d
            take_plus = np.abs(pp) >= np.abs(pm)
            sk = np.where(take_plus, F32(1.0), F32(-1.0)).astype(F32)
            piv = np.where(take_plus, pp, pm).astype(F32)
            s[:, k] = sk
            if k + 1 < m:
                mult = (-sk[:, None] * M[:, k + 1:, k]) / piv[:, None]
                Y[:, k + 1:, k] = mult
                if k + 1 < k1:
                    M[:, k + 1:, k + 1:k1] -= mult[:, :, None] * M[:, k, None, k + 1:k1]
        if k1 < n:
            for k in range(k0, k1):
                if k + 1 < k1:
                    M[:, k + 1:k1, k1:] -= Y[:, k + 1:k1, k, None] * M[:, k, None, k1:]
            M[:, k1:, k1:] -= _bmm(Y[:, k1:, k0:k1], M[:, k0:k1, k1:])
    return Y, s


# --------------------------------------------------------------------------------------
# Entry: custom_kernel  (reflection_no_reflectors.py:181-196)
# --------------------------------------------------------------------------------------
def custom_kernel_np(A, return_info: bool = False):
    """``A (..., n, n)`` -> ``(H, tau)`` in float32 (the caller casts back)."""
    A = np.asarray(A)
    lead, n = A.shape[:-2], A.shape[-1]
    A3 = A.reshape(-1, n, n).astype(F32)
    if A3.shape[0] == 0:
        H = np.zeros(A3.shape, F32)
        tau = np.zeros((0, n), F32)
    else:
        Q, _perm, ok = frame(A3)
        R = np.triu(_bmm(np.swapaxes(Q, 1, 2), A3))            # closure, :186
        Y, s = chart(Q)                                        # chart, :187
        tau = (F32(2.0) / (np.sum(np.square(np.tril(Y, -1)), axis=1) + F32(1.0))).astype(F32)
        H = (np.triu(s[:, :, None] * R) + np.tril(Y, -1)).astype(F32)   # :195
    H = H.reshape(*lead, n, n)
    tau = tau.reshape(*lead, n)
    if return_info:
        return H, tau, (~ok).astype(np.int32) if A3.shape[0] else np.zeros(0, np.int32)
    return H, tau


def custom_kernel_rect_np(A):
    """Tall ``A (b, m, n)``, m >= n -> ``(H (b, m, n), tau (b, n))``: the same frame, closure and
    chart on an m x n input.  The LU pivots over m rows, CholeskyQR2 runs on the m x n unit
    lower-trapezoidal L (jitter over its n Gram diagonal entries), the closure is the n x n
    triu(Q^T A), and the chart is the reference's rectangular elimination over the n columns
    of the frame (modlu_rect, irregular/exp1_irregular.py:106-122) with the sign rule of
    reflection_no_reflectors.py:149-158."""
    A3 = np.asarray(A, dtype=F32)
    b, m, n = A3.shape
    Q, _perm, _ok = frame(A3)
    R = np.triu(_bmm(np.swapaxes(Q, 1, 2), A3))
    Y, s = chart(Q)
    tau = (F32(2.0) / (np.sum(np.square(np.tril(Y, -1)), axis=1) + F32(1.0))).astype(F32)
    H = np.tril(Y, -1)
    H[:, :n, :] += np.triu(s[:, :, None] * R)
    return H.astype(F32), tau


def custom_kernel(data):
    """Torch-facing twin of the reference entry point: any float dtype in, same dtype out."""
    import torch
    dtype = data.dtype
    H, tau = custom_kernel_np(data.detach().to("cpu", torch.float32).numpy())
    return torch.from_numpy(H).to(dtype), torch.from_numpy(tau).to(dtype)
