"""ctypes binding of ``libqrb200.so`` (the C ABI declared in ``include/qrb200.h``).

The shared library is built in-tree (``qrb200/build.py``).  Loading it needs no GPU;
calling the compute entry point does.  There is no fallback: if the library is missing
the import of :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqrb200.so"
# the same library built with -DQRB_BOUNDS_CHECK (pivot-map indices checked, INFO_BOUNDS)
CHECKED_LIB_PATH = Path(__file__).resolve().parent / "libqrb200_checked.so"

QRB200_OK = 0
QRB200_ERR_INVALID_ARG = 1
QRB200_ERR_UNSUPPORTED_N = 2
QRB200_ERR_WORKSPACE = 3
QRB200_ERR_CUDA = 4
QRB200_ERR_SCRATCH_LIMIT = 5
NOALLOC_SCRATCH_BYTES = 64 << 20
# largest n the allocation-free entry point accepts with the default block options
# (n % 4 != 0: 16-wide panels; n % 4 == 0: 32-wide panels, larger panel buffers)
NOALLOC_MAX_N_DEFAULT = 1826
NOALLOC_MAX_N4_DEFAULT = 1792

QRB200_F32, QRB200_BF16, QRB200_F16 = 0, 1, 2

INFO_NONFINITE_INPUT = 1
INFO_CHOL1_NOT_PD = 2
INFO_CHOL2_NOT_PD = 4
INFO_LU_ZERO_PIVOT = 8
INFO_DEVICE_TIMEOUT = 16
INFO_BOUNDS = 32

OPT_GEMM_PATH = 1
OPT_SMALL_N = 2
OPT_CHOL_BLOCK = 3
OPT_LANES = 4
OPT_CHART_BLOCK = 5
OPT_PANEL_LOOP = 6
OPT_CLOSURE_DUAL_N = 7
GEMM_AUTO, GEMM_SIMT, GEMM_TC = 0, 1, 2

# every symbol include/qrb200.h declares, with its ctypes signature
SIGNATURES = {
    "qrb200_version": (ctypes.c_int, []),
    "qrb200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qrb200_max_n": (ctypes.c_int32, []),
    "qrb200_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "qrb200_geqrf_batched": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p]),
    "qrb200_geqrf_batched_q": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_void_p]),
    "qrb200_geqrf_batched_rect": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                 ctypes.c_int32, ctypes.c_void_p]),
    "qrb200_geqrf_batched_timed": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_void_p, ctypes.c_size_t,
                                                  ctypes.c_void_p,
                                                  ctypes.POINTER(ctypes.c_float)]),
    "qrb200_num_families": (ctypes.c_int32, []),
    "qrb200_family_name": (ctypes.c_char_p, [ctypes.c_int32]),
    "qrb200_launch_count": (ctypes.c_longlong, []),
    "qrb200_last_cuda_error": (ctypes.c_char_p, []),
    "qrb200_set_option": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int64]),
    "qrb200_geqrf_batched_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_int64, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_void_p]),
    "qrb200_geqrf_batched_host": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                 ctypes.c_int64, ctypes.c_void_p]),
    "qrb200_release_host_staging": (ctypes.c_int, []),
}

_LIB = None


class QRB200Error(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, where: str):
        self.status = status
        msg = f"{where}: {status_string(status)} (status {status})"
        if status == QRB200_ERR_CUDA:
            msg += ": " + lib().qrb200_last_cuda_error().decode()
        super().__init__(msg)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m qrb200.build` "
                              "(or __graft_entry__.build())")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def status_string(status: int) -> str:
    return lib().qrb200_status_string(int(status)).decode()


def workspace_bytes(batch: int, n: int) -> int:
    out = ctypes.c_size_t(0)
    rc = lib().qrb200_workspace_bytes(int(batch), int(n), ctypes.byref(out))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_workspace_bytes")
    return int(out.value)


def geqrf_batched(A_ptr, H_ptr, tau_ptr, info_ptr, batch, n, dtype, ws_ptr, ws_bytes,
                  stream_ptr) -> int:
    return lib().qrb200_geqrf_batched(A_ptr, H_ptr, tau_ptr, info_ptr, int(batch), int(n),
                                      int(dtype), ws_ptr, int(ws_bytes), stream_ptr)


def families():
    L = lib()
    return [L.qrb200_family_name(i).decode() for i in range(L.qrb200_num_families())]


def launch_count() -> int:
    return int(lib().qrb200_launch_count())


def geqrf_batched_timed(A_ptr, H_ptr, tau_ptr, info_ptr, batch, n, dtype, ws_ptr, ws_bytes,
                        stream_ptr):
    """Returns (status, {family: ms}); synchronises the stream."""
    nf = lib().qrb200_num_families()
    buf = (ctypes.c_float * nf)()
    rc = lib().qrb200_geqrf_batched_timed(A_ptr, H_ptr, tau_ptr, info_ptr, int(batch), int(n),
                                          int(dtype), ws_ptr, int(ws_bytes), stream_ptr, buf)
    return rc, dict(zip(families(), [float(x) for x in buf]))


def set_gemm_path(path: int) -> None:
    """0 = automatic, 1 = SIMT tiles only, 2 = tcgen05 tiles whenever n % 4 == 0."""
    rc = lib().qrb200_set_option(OPT_GEMM_PATH, int(path))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_set_option")


def set_small_n(n_max: int) -> None:
    """Largest order handled by the fused one-CTA-per-matrix kernel (0..128)."""
    rc = lib().qrb200_set_option(OPT_SMALL_N, int(n_max))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_set_option")


def set_chol_block(block: int) -> None:
    """Column block of the two-level Cholesky elimination: 0 (one level), 64, 128 or 256."""
    rc = lib().qrb200_set_option(OPT_CHOL_BLOCK, int(block))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_set_option")


def set_lanes(lanes: int) -> None:
    """Internal streams a chunk of the batch is split over (1..4)."""
    rc = lib().qrb200_set_option(OPT_LANES, int(lanes))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_set_option")


def set_chart_block(block: int) -> None:
    """Column block of the two-level chart elimination: 0 (one level), 64, 128 or 256."""
    rc = lib().qrb200_set_option(OPT_CHART_BLOCK, int(block))
    if rc != QRB200_OK:
        raise QRB200Error(rc, "qrb200_set_option")


def set_panel_loop(mode: int) -> None:
    """Column loop of the register-resident panels: 0 automatic, 1 unrolled, 2 rotating."""
    rc = lib().qrb200_set_option(OPT_PANEL_LOOP, int(mode))
    if rc != 0:
        raise QRB200Error(rc, "qrb200_set_option")


def set_closure_dual_n(n_max: int) -> None:
    """Largest n whose closure GEMM runs two CTAs per SM (0 = none)."""
    rc = lib().qrb200_set_option(OPT_CLOSURE_DUAL_N, int(n_max))
    if rc != 0:
        raise QRB200Error(rc, "qrb200_set_option")
