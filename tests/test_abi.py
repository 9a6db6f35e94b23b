"""CPU: the C-ABI library loads, exports exactly what include/*.h declares, and validates
its arguments before touching the GPU (every call below returns before any CUDA call)."""
import ctypes
import re
from pathlib import Path

import pytest

from qrb200 import _lib

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    syms = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(qrb200_\w+)\s*\(", text, flags=re.M):
            syms.add(m.group(1))
    return syms


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = declared_symbols()
    assert syms, "no declarations parsed"
    assert syms == set(_lib.SIGNATURES), syms ^ set(_lib.SIGNATURES)
    for s in syms:
        assert hasattr(L, s), s


def test_version_and_limits():
    L = _lib.lib()
    assert L.qrb200_version() >= 100
    assert L.qrb200_max_n() >= 2048
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(_lib.QRB200_ERR_WORKSPACE)


def test_workspace_bytes():
    assert _lib.workspace_bytes(0, 64) == 0
    assert _lib.workspace_bytes(10, 0) == 0
    # n <= 64 (default) runs the fused one-CTA-per-matrix kernel: no workspace at all
    assert _lib.workspace_bytes(1000, 64) == 0 and _lib.workspace_bytes(7, 32) == 0
    assert _lib.workspace_bytes(7, 128) > 0
    a = _lib.workspace_bytes(1, 200)
    b = _lib.workspace_bytes(2, 200)
    assert 5 * 200 * 200 * 4 <= a < b
    # n=512, batch 1536 fits one chunk: >= 5 float32 n x n buffers per matrix
    assert _lib.workspace_bytes(1536, 512) >= 1536 * 5 * 512 * 512 * 4
    with pytest.raises(_lib.QRB200Error):
        _lib.workspace_bytes(4, 100000)
    with pytest.raises(_lib.QRB200Error):
        _lib.workspace_bytes(-1, 8)


def _call(**kw):
    args = dict(A=1, H=1, tau=1, info=1, batch=1, n=8, dtype=0, ws=None, wsb=0, stream=None)
    args.update(kw)
    return _lib.geqrf_batched(args["A"], args["H"], args["tau"], args["info"], args["batch"],
                              args["n"], args["dtype"], args["ws"], args["wsb"], args["stream"])


def test_argument_validation_without_gpu():
    assert _call(batch=-1) == _lib.QRB200_ERR_INVALID_ARG
    assert _call(n=-3) == _lib.QRB200_ERR_UNSUPPORTED_N
    assert _call(n=10 ** 6) == _lib.QRB200_ERR_UNSUPPORTED_N
    assert _call(dtype=9) == _lib.QRB200_ERR_INVALID_ARG
    assert _call(A=None) == _lib.QRB200_ERR_INVALID_ARG
    assert _call(info=None) == _lib.QRB200_ERR_INVALID_ARG
    assert _call(n=200, ws=1, wsb=16) == _lib.QRB200_ERR_WORKSPACE
    # empty problems are a successful no-op
    assert _call(batch=0, A=None, H=None, tau=None, info=None) == _lib.QRB200_OK
    assert _call(n=0) == _lib.QRB200_OK


def test_no_torch_in_the_abi():
    text = "".join(h.read_text() for h in (REPO / "include").glob("*.h"))
    assert not re.search(r"\b(at::|torch::|c10::|Tensor\b)", text)
    assert "#include <cuda" not in text


def test_library_has_no_torch_dependency():
    # the dynamic section lists no libtorch / libc10 (CUDA runtime is linked statically)
    import shutil
    import subprocess
    if not shutil.which("readelf"):
        pytest.skip("readelf not available")
    out = subprocess.run(["readelf", "-d", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    needed = [l for l in out.splitlines() if "NEEDED" in l]
    assert needed and not any(("torch" in l) or ("c10" in l) for l in needed), needed


def test_small_n_option():
    with pytest.raises(_lib.QRB200Error):
        _lib.set_small_n(129)
    with pytest.raises(_lib.QRB200Error):
        _lib.set_small_n(-1)
    try:
        _lib.set_small_n(128)
        assert _lib.workspace_bytes(7, 128) == 0
        _lib.set_small_n(0)
        assert _lib.workspace_bytes(7, 16) > 0
    finally:
        _lib.set_small_n(64)
    assert _lib.workspace_bytes(7, 64) == 0


def test_block_and_lane_options():
    """Option ranges are enforced on the host; the block widths size the panel buffers, so
    the workspace query follows them (one-level eliminations need the least)."""
    L = _lib.lib()
    for key, bad in ((_lib.OPT_CHOL_BLOCK, (1, 32, 100, 512, -1)),
                     (_lib.OPT_CHART_BLOCK, (1, 32, 100, 512, -1)),
                     (_lib.OPT_LANES, (0, 5, -1))):
        for v in bad:
            assert L.qrb200_set_option(key, v) == _lib.QRB200_ERR_INVALID_ARG, (key, v)
    try:
        default = _lib.workspace_bytes(8, 512)
        _lib.set_chol_block(0)
        _lib.set_chart_block(0)
        one_level = _lib.workspace_bytes(8, 512)
        _lib.set_chol_block(256)
        wide = _lib.workspace_bytes(8, 512)
        assert one_level < default < wide
        for lanes in (1, 2, 3, 4):
            _lib.set_lanes(lanes)
    finally:
        _lib.set_chol_block(128)
        _lib.set_chart_block(128)
        _lib.set_lanes(2)
    assert _lib.workspace_bytes(8, 512) == default


def test_noalloc_order_limit_without_gpu():
    # the allocation-free entry point checks the order against its built-in scratch before it
    # looks at the buffers or the device: with null buffers an order that fits reports an
    # invalid argument, one that does not fit reports the scratch limit
    from qrb200 import _lib
    L = _lib.lib()
    nmax = _lib.NOALLOC_MAX_N_DEFAULT
    call = lambda n: L.qrb200_geqrf_batched_noalloc(None, None, None, None, 1, n,  # noqa: E731
                                                    _lib.QRB200_F32, None)
    assert call(nmax) == _lib.QRB200_ERR_INVALID_ARG
    assert call(nmax + 1) == _lib.QRB200_ERR_SCRATCH_LIMIT
    n4 = _lib.NOALLOC_MAX_N4_DEFAULT
    assert call(n4) == _lib.QRB200_ERR_INVALID_ARG
    assert call(n4 + 4) == _lib.QRB200_ERR_SCRATCH_LIMIT
    assert call(64) == _lib.QRB200_ERR_INVALID_ARG


def test_torch_operator_registers_and_has_meta_shapes():
    # torch.ops.qrb200.geqrf loads without a GPU; its Meta kernel gives the output shapes
    import torch
    from qrb200 import api
    op = api.load_torch_ops()
    A = torch.empty(2, 3, 40, 40, device="meta", dtype=torch.bfloat16)
    H, tau, info = op(A)
    assert H.shape == (2, 3, 40, 40) and tau.shape == (2, 3, 40) and info.shape == (2, 3)
    assert H.dtype == torch.bfloat16 and tau.dtype == torch.bfloat16 and info.dtype == torch.int32
