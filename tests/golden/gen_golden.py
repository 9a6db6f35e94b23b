"""Generate the golden fixtures that pin the CPU oracle to the reference.

Imports the reference implementation (``reflection_no_reflectors.custom_kernel``, pure
PyTorch) from a read-only checkout and runs it on CPU over small seeded inputs; stores
inputs and the reference's own outputs ``(H, tau)`` as ``.npz`` files next to this
script.  The GPU box never runs this script; tests only read the ``.npz`` files.

Usage:  python tests/golden/gen_golden.py /path/to/qr-contest-checkout [name ...]

With names, only those fixtures are (re)generated.  Fixtures at the benchmark's own orders:
``<class>_n512`` (the heterogeneous n = 512 classes; two matrices of the classes compared
elementwise or by tau, one of the gate-only ones) and ``c5_n256`` (the first six matrices
of the 8-GPU sweep's global bf16 batch, one per class, with the reference's bf16 outputs and
its float32 outputs of the same inputs).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "qr-contest_b200"))

from qrb200 import generators as G  # noqa: E402


def cases():
    """(name, tensor) pairs: every class at n in {16, 33, 64}, plus structural cases."""
    out = []
    for n in (16, 33, 64):
        for ci, cname in enumerate(G.CLASSES):
            g = G._gen(100 + 10 * n + ci, "cpu")
            A = G.make_class(cname, 6, n, g, "cpu").to(torch.float32)
            out.append((f"{cname}_n{n}", A))
    out.append(("smoke_n64", G.gaussian((64, 64, 64), seed=0)[:16].clone()))
    out.append(("small_n32", G.gaussian((8, 32, 32), seed=1)))
    out.append(("small_n128", G.gaussian((2, 128, 128), seed=2)))
    out.append(("lead_2x3_n8", G.gaussian((2, 3, 8, 8), seed=7)))
    out.append(("n1", G.gaussian((5, 1, 1), seed=8)))
    out.append(("n2", G.gaussian((5, 2, 2), seed=9)))
    n = 12
    eye = torch.eye(n).expand(2, n, n).clone()
    out.append(("identity", eye))
    out.append(("neg_identity", -eye))
    out.append(("zero_col", torch.cat([G.gaussian((3, 10, 1), seed=10),
                                       torch.zeros(3, 10, 1),
                                       G.gaussian((3, 10, 8), seed=11)], dim=-1)))
    out.append(("bf16_n32", G.gaussian((4, 32, 32), seed=12, dtype=torch.bfloat16)))
    for ci, cname in enumerate(G.CLASSES):
        g = G._gen(600 + ci, "cpu")
        b = 2 if cname in ("dense", "uppertri", "illcond") else 1
        out.append((f"{cname}_n512", G.make_class(cname, b, 512, g, "cpu").to(torch.float32)))
    c5, _ = G.sweep_shard(6, 256, 0, 1, seed=5, device="cpu", dtype=torch.bfloat16)
    out.append(("c5_n256", c5))
    return out


def main(ref_root: str, only=()):
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import reflection_no_reflectors as ref  # the reference's own entry point

    torch.manual_seed(0)
    for name, A in cases():
        if only and name not in only:
            continue
        H, tau = ref.custom_kernel(A.clone())
        payload = {
            "A": A.float().numpy(),
            "H": H.float().numpy(),
            "tau": tau.float().numpy(),
            "dtype": np.array(str(A.dtype)),
        }
        if A.dtype == torch.bfloat16:  # the reference's float32 factors of the same inputs
            H32, tau32 = ref.custom_kernel(A.float())
            payload["H32"], payload["tau32"] = H32.numpy(), tau32.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **payload)
        print(name, tuple(A.shape), A.dtype)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit(__doc__)
    main(sys.argv[1], tuple(sys.argv[2:]))
