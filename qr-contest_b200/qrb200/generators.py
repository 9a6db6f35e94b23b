"""Seeded synthetic batches for the conditioning classes the benchmark names.

The reference's real contest generators (gpu-mode ``reference-kernels``, ``task.py``) are
not available; its own approximations live in ``common/oracle.py:43-146``.  These
generators build the six n=512 classes of the heterogeneous batch (and the large-n and
small-n batches) from their definitions: construction in float64 on the target device,
then a cast to the requested dtype.

Classes (index -> name), in the order of the heterogeneous batch:
  0 dense        iid N(0,1)
  1 illcond      U diag(sigma) V^T, Haar U, V, sigma = logspace(0, -6, n)
  2 rankdef      B C, B n x r, C r x n Gaussian (r = n // 2)
  3 rowscaled    rows of N(0,1) scaled by 10^k, k uniform integer in [-6, 6] per row
  4 nearrank     rank-r product B C + 1e-7 N(0,1)
  5 uppertri     triu(N(0,1))
"""
from __future__ import annotations

import torch

CLASSES = ("dense", "illcond", "rankdef", "rowscaled", "nearrank", "uppertri")


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def _randn(shape, g, device):
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float64)


def haar(b: int, n: int, g, device):
    """Haar-distributed orthogonal matrices: QR of a Gaussian with the sign(diag R) fix."""
    Z = _randn((b, n, n), g, device)
    Q, R = torch.linalg.qr(Z)
    d = torch.sign(torch.diagonal(R, dim1=-2, dim2=-1))
    d = torch.where(d == 0, torch.ones_like(d), d)
    return Q * d.unsqueeze(-2)


def make_class(name: str, b: int, n: int, g, device, sigma_min_exp: float = -6.0,
               rank: int | None = None):
    """One class as a float64 ``(b, n, n)`` batch."""
    r = rank if rank is not None else max(1, n // 2)
    if name == "dense":
        return _randn((b, n, n), g, device)
    if name == "illcond":
        U = haar(b, n, g, device)
        V = haar(b, n, g, device)
        sig = torch.logspace(0.0, sigma_min_exp, n, dtype=torch.float64, device=device)
        return (U * sig) @ V.mT
    if name == "rankdef":
        return _randn((b, n, r), g, device) @ _randn((b, r, n), g, device)
    if name == "rowscaled":
        k = torch.randint(-6, 7, (b, n, 1), generator=g, device=device).to(torch.float64)
        return _randn((b, n, n), g, device) * torch.pow(10.0, k)
    if name == "nearrank":
        base = _randn((b, n, r), g, device) @ _randn((b, r, n), g, device)
        return base + 1e-7 * _randn((b, n, n), g, device)
    if name == "uppertri":
        return torch.triu(_randn((b, n, n), g, device))
    raise ValueError(f"unknown class {name!r}")


def heterogeneous(b: int, n: int, seed: int = 3, device="cpu", dtype=torch.float32,
                  layout: str = "blocks", chunk: int = 64):
    """The mixed-class batch.  ``layout='blocks'``: classes in contiguous blocks of
    ``b // 6`` (remainder to the last class); ``'roundrobin'``: class = index mod 6."""
    g = _gen(seed, device)
    out = torch.empty(b, n, n, dtype=dtype, device=device)
    if layout == "blocks":
        per = b // 6
        bounds = [(c * per, (c + 1) * per if c < 5 else b) for c in range(6)]
        for c, (lo, hi) in enumerate(bounds):
            for i in range(lo, hi, chunk):
                j = min(hi, i + chunk)
                out[i:j] = make_class(CLASSES[c], j - i, n, g, device).to(dtype)
    elif layout == "roundrobin":
        for c in range(6):
            idx = torch.arange(c, b, 6, device=device)
            for i in range(0, idx.numel(), chunk):
                sel = idx[i:i + chunk]
                out[sel] = make_class(CLASSES[c], sel.numel(), n, g, device).to(dtype)
    else:
        raise ValueError(layout)
    return out


def gaussian(shape, seed: int = 0, device="cpu", dtype=torch.float32):
    g = _gen(seed, device)
    return torch.randn(*shape, generator=g, device=device, dtype=torch.float64).to(dtype)


def large_illcond(b: int, n: int, seed: int = 4, device="cpu", dtype=torch.float32, chunk=4):
    """``U diag(sigma) V^T`` with sigma = logspace(0, -12, n) (the large-n stress batch)."""
    g = _gen(seed, device)
    out = torch.empty(b, n, n, dtype=dtype, device=device)
    for i in range(0, b, chunk):
        j = min(b, i + chunk)
        out[i:j] = make_class("illcond", j - i, n, g, device, sigma_min_exp=-12.0).to(dtype)
    return out


C5_BLOCK = 1024  # matrices per independently seeded block of the C5 sweep


def sweep_shard(global_batch: int, n: int, rank: int, world: int, seed: int = 5,
                device="cpu", dtype=torch.bfloat16, block: int = C5_BLOCK):
    """This rank's slice of the 8-GPU sweep batch (the six classes regenerated at order n,
    rank parameter n // 2, class = global index mod 6), generated on ``device``.

    Rank g owns the contiguous global slice ``[g * ceil(b / G), ...)``.  The global batch is
    cut into blocks of ``block`` matrices, block j seeded with ``seed + j * block`` (the
    seed plus the block's global offset), so every rank builds only its own slice and the
    global batch is the same for every world size.  Returns ``(shard, first_global_index)``.
    """
    per = -(-global_batch // world)
    lo = min(global_batch, rank * per)
    hi = min(global_batch, lo + per)
    out = torch.empty(hi - lo, n, n, dtype=dtype, device=device)
    j0 = lo // block
    for j in range(j0, -(-hi // block)):
        b0, b1 = j * block, min(global_batch, (j + 1) * block)
        s0, s1 = max(b0, lo), min(b1, hi)
        if s0 >= s1:
            continue
        g = _gen(seed + b0, device)
        blk = torch.empty(b1 - b0, n, n, dtype=dtype, device=device)
        for c in range(6):
            # global index i has class i mod 6: inside the block that is offset (c - b0) mod 6
            idx = torch.arange((c - b0) % 6, b1 - b0, 6, device=device)
            if idx.numel():
                blk[idx] = make_class(CLASSES[c], idx.numel(), n, g, device).to(dtype)
        out[s0 - lo:s1 - lo] = blk[s0 - b0:s1 - b0]
    return out, lo
