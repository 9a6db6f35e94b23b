"""Loader for the committed golden fixtures (inputs + the reference's own outputs)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# classes whose outputs are determined to float32 rounding (compared elementwise);
# rank-deficient inputs have arbitrary null-space columns and are gated only.
TIGHT = ("dense_", "smoke_", "small_", "lead_", "n1", "n2", "identity", "neg_identity",
         "uppertri_", "zero_col")
LOOSE = ("illcond_",)


def names():
    return sorted(p.stem for p in HERE.glob("*.npz"))


def load(name):
    z = np.load(HERE / f"{name}.npz")
    return {"A": z["A"], "H": z["H"], "tau": z["tau"], "dtype": str(z["dtype"])}


def kind(name):
    if name.startswith("bf16"):
        return "bf16"
    if any(name.startswith(t) for t in TIGHT):
        return "tight"
    if any(name.startswith(t) for t in LOOSE):
        return "loose"
    return "gate"
