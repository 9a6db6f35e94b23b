"""Build ``libqrb200.so`` in-tree with nvcc for sm_100a (no GPU needed to compile).

    python -m qrb200.build            (from the qr-contest_b200 directory)

The library has no PyTorch dependency: plain ``nvcc -shared`` of ``csrc/qrb_api.cu`` with
the CUDA runtime linked statically.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # qr-contest_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB = PKG / "libqrb200.so"
TESTKIT = PKG / "libqrb200_testkit.so"   # single-stage entry points for the GPU unit tests
CHECKED = PKG / "libqrb200_checked.so"   # the library with the pivot-map bounds checks

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return (sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp"))
            + sorted(INCLUDE.glob("*.h")))


def up_to_date(target: Path) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def _compile(src: Path, out: Path, verbose: bool, extra) -> None:
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", str(INCLUDE), "-o", str(out), str(src)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


OPS = PKG / "libqrb200_torch_ops.so"  # torch.ops.qrb200.geqrf (links libqrb200.so)


def _compile_ops(verbose: bool) -> None:
    """The TORCH_LIBRARY operator library: g++ against torch's headers and libraries, linked
    to libqrb200.so next to it (rpath $ORIGIN).  No CUDA code is compiled here."""
    import torch
    from torch.utils import cpp_extension as ce
    cuda_home = Path(ce.CUDA_HOME or "/usr/local/cuda")
    abi = int(torch.compiled_with_cxx11_abi())
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", str(INCLUDE), "-I", str(cuda_home / "include")]
    for d in ce.include_paths():
        cmd += ["-I", d]
    cmd += ["-o", str(OPS), str(CSRC / "qrb_torch_op.cpp"), "-L", str(PKG), "-l:libqrb200.so",
            "-Wl,-rpath,$ORIGIN"]
    for d in ce.library_paths():
        cmd += ["-L", d, f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    # the three nvcc runs are independent (minutes each): run them side by side
    from concurrent.futures import ThreadPoolExecutor
    jobs = [(src, out, defs) for src, out, defs in
            ((CSRC / "qrb_api.cu", LIB, []),
             (CSRC / "qrb_api.cu", CHECKED, ["-DQRB_BOUNDS_CHECK"]),
             (CSRC / "qrb_testkit.cu", TESTKIT, ["-DQRB_PANEL_TIMERS"]))
            if force or not up_to_date(out)]
    with ThreadPoolExecutor(max_workers=max(1, len(jobs))) as ex:
        for f in [ex.submit(_compile, src, out, verbose, [*extra, *defs]) for src, out, defs in jobs]:
            f.result()
    if force or not up_to_date(OPS) or OPS.stat().st_mtime < (CSRC / "qrb_torch_op.cpp").stat().st_mtime:
        _compile_ops(verbose)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [])
