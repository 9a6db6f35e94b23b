"""Generate the golden fixtures that pin the CPU oracle to the reference.

Imports the reference implementation (``reflection_no_reflectors.custom_kernel``, pure
PyTorch) from a read-only checkout and runs it on CPU over small seeded inputs; stores
inputs and the reference's own outputs ``(H, tau)`` as ``.npz`` files next to this
script.  The GPU box never runs this script; tests only read the ``.npz`` files.

Usage:  python tests/golden/gen_golden.py /path/to/qr-contest-checkout
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
    return out


def main(ref_root: str):
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import reflection_no_reflectors as ref  # the reference's own entry point

    torch.manual_seed(0)
    for name, A in cases():
        H, tau = ref.custom_kernel(A.clone())
        payload = {
            "A": A.float().numpy() if A.dtype != torch.bfloat16 else A.float().numpy(),
            "H": H.float().numpy(),
            "tau": tau.float().numpy(),
            "dtype": np.array(str(A.dtype)),
        }
        np.savez_compressed(HERE / f"{name}.npz", **payload)
        print(name, tuple(A.shape), A.dtype)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
