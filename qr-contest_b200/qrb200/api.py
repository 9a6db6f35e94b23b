"""Host-side mirror of the reference entry point over the C ABI.

``custom_kernel(data) -> (H, tau)`` follows reflection_no_reflectors.py:181-196:

* input ``(..., n, n)`` of any dtype; the factors are computed in float32
  (``A = data.to(torch.float32)``, :183) and returned in the input dtype (:196);
* ``H`` carries ``s_i * R_ij`` on and above the diagonal and the reflector tails below it,
  ``tau_k = 2 / (1 + ||Y[:, k]||^2)`` (:192-195) -- the torch.geqrf layout;
* a Gram matrix that is not positive definite after the jitter raises
  ``torch.linalg.LinAlgError``, as ``torch.linalg.cholesky`` does at :76 (NaN/Inf input
  ends there too).

The tensor may live on a CUDA device (results stay there) or in host memory (results come
back in host memory, like the reference called on a CPU tensor).  Host tensors are factored
on the current CUDA device through ``qrb200_geqrf_batched_host``, which overlaps the copies
with the kernels (page-locked tensors give the overlap).  There is no CPU compute path: without
a CUDA device or the compiled library the call raises.  float32 / bfloat16 / float16 are read
and written natively by the kernels; any other dtype is converted to float32 first.
"""
from __future__ import annotations

import torch

from . import _lib

LinAlgError = torch.linalg.LinAlgError

_NATIVE = {torch.float32: _lib.QRB200_F32, torch.bfloat16: _lib.QRB200_BF16,
           torch.float16: _lib.QRB200_F16}


def _prep(data: torch.Tensor):
    if not isinstance(data, torch.Tensor):
        raise TypeError("custom_kernel expects a torch.Tensor")
    if data.dim() < 2 or data.shape[-1] != data.shape[-2]:
        raise ValueError(f"expected a (..., n, n) tensor, got shape {tuple(data.shape)}")
    if data.device.type not in ("cuda", "cpu"):
        raise ValueError(f"qrb200 takes CUDA or host tensors (got one on {data.device})")
    A = data if data.dtype in _NATIVE else data.to(torch.float32)
    return A.contiguous()


def workspace_bytes(batch: int, n: int) -> int:
    """Device workspace one :func:`geqrf` call of this shape needs."""
    return _lib.workspace_bytes(batch, n)


def geqrf(data: torch.Tensor, workspace: torch.Tensor | None = None):
    """Asynchronous core: returns ``(H, tau, info)`` without synchronising the host.

    ``info`` is an int32 tensor of per-matrix ``QRB200_INFO_*`` bits with the leading shape
    of ``data``.  ``workspace`` (optional) is a uint8 CUDA tensor of at least
    :func:`workspace_bytes` bytes; when omitted one is taken from torch's caching allocator.
    """
    A = _prep(data)
    if A.device.type == "cpu":
        return geqrf_host(data)
    lead, n = A.shape[:-2], A.shape[-1]
    batch = 1
    for d in lead:
        batch *= int(d)
    H = torch.empty_like(A)
    tau = torch.empty(*lead, n, dtype=A.dtype, device=A.device)
    info = torch.zeros(*lead, dtype=torch.int32, device=A.device)
    if batch > 0 and n > 0:
        need = _lib.workspace_bytes(batch, n)
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=A.device)
        elif workspace.numel() * workspace.element_size() < need or workspace.device != A.device:
            raise ValueError(f"workspace must be >= {need} bytes on {A.device}")
        with torch.cuda.device(A.device):
            stream = torch.cuda.current_stream(A.device).cuda_stream
            rc = _lib.geqrf_batched(A.data_ptr(), H.data_ptr(), tau.data_ptr(), info.data_ptr(),
                                    batch, n, _NATIVE[A.dtype], workspace.data_ptr(),
                                    need, stream)
        if rc != _lib.QRB200_OK:
            raise _lib.QRB200Error(rc, "qrb200_geqrf_batched")
    if data.dtype not in _NATIVE:
        H, tau = H.to(data.dtype), tau.to(data.dtype)
    return H, tau, info


def geqrf_q(data: torch.Tensor, workspace: torch.Tensor | None = None):
    """Like :func:`geqrf`, plus the explicit orthogonal factor: returns ``(H, tau, Q, info)``
    with ``Q == torch.linalg.householder_product(H, tau)`` (to rounding), written from the
    pipeline's frame instead of being rebuilt from the reflectors by the caller."""
    A = _prep(data)
    if A.device.type != "cuda":
        raise ValueError("geqrf_q takes a CUDA tensor")
    lead, n = A.shape[:-2], A.shape[-1]
    batch = 1
    for d in lead:
        batch *= int(d)
    H = torch.empty_like(A)
    Q = torch.empty_like(A)
    tau = torch.empty(*lead, n, dtype=A.dtype, device=A.device)
    info = torch.zeros(*lead, dtype=torch.int32, device=A.device)
    if batch > 0 and n > 0:
        need = _lib.workspace_bytes(batch, n)
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=A.device)
        elif workspace.numel() * workspace.element_size() < need or workspace.device != A.device:
            raise ValueError(f"workspace must be >= {need} bytes on {A.device}")
        with torch.cuda.device(A.device):
            stream = torch.cuda.current_stream(A.device).cuda_stream
            rc = _lib.lib().qrb200_geqrf_batched_q(A.data_ptr(), H.data_ptr(), tau.data_ptr(),
                                                    Q.data_ptr(), info.data_ptr(), batch, n,
                                                    _NATIVE[A.dtype], workspace.data_ptr(),
                                                    need, stream)
        if rc != _lib.QRB200_OK:
            raise _lib.QRB200Error(rc, "qrb200_geqrf_batched_q")
    if data.dtype not in _NATIVE:
        H, tau, Q = H.to(data.dtype), tau.to(data.dtype), Q.to(data.dtype)
    return H, tau, Q, info


def geqrf_rect(data: torch.Tensor):
    """QR of a batch of tall ``(..., m, n)`` CUDA matrices (``m >= n``): returns
    ``(H, tau, info)`` with ``H (..., m, n)`` and ``tau (..., n)`` in the torch.geqrf layout,
    ``householder_product(H, tau)`` the ``m x n`` orthonormal factor.  Asynchronous."""
    if not isinstance(data, torch.Tensor) or data.dim() < 2:
        raise ValueError("expected a (..., m, n) tensor")
    m, n = data.shape[-2], data.shape[-1]
    if n > m:
        raise ValueError(f"geqrf_rect takes tall or square matrices (got {m} x {n})")
    if data.device.type != "cuda":
        raise ValueError("geqrf_rect takes a CUDA tensor")
    A = (data if data.dtype in _NATIVE else data.to(torch.float32)).contiguous()
    lead = A.shape[:-2]
    batch = 1
    for d in lead:
        batch *= int(d)
    H = torch.empty_like(A)
    tau = torch.empty(*lead, n, dtype=A.dtype, device=A.device)
    info = torch.zeros(*lead, dtype=torch.int32, device=A.device)
    if batch > 0 and n > 0:
        with torch.cuda.device(A.device):
            stream = torch.cuda.current_stream(A.device).cuda_stream
            rc = _lib.lib().qrb200_geqrf_batched_rect(A.data_ptr(), H.data_ptr(), tau.data_ptr(),
                                                       info.data_ptr(), batch, m, n,
                                                       _NATIVE[A.dtype], stream)
        if rc != _lib.QRB200_OK:
            raise _lib.QRB200Error(rc, "qrb200_geqrf_batched_rect")
    if data.dtype not in _NATIVE:
        H, tau = H.to(data.dtype), tau.to(data.dtype)
    return H, tau, info


def geqrf_host(data: torch.Tensor, out=None, sub_batch: int = 0):
    """Factor a HOST tensor on the current CUDA device; returns host ``(H, tau, info)``.

    Blocking.  ``out`` = optional preallocated host ``(H, tau, info)`` (page-locked tensors
    let the library overlap the copies with the kernels); ``sub_batch`` = matrices per
    pipelined sub-batch, 0 for the library's choice.
    """
    A = _prep(data)
    if A.device.type != "cpu":
        raise ValueError("geqrf_host takes a host tensor")
    lead, n = A.shape[:-2], A.shape[-1]
    batch = 1
    for d in lead:
        batch *= int(d)
    if out is None:
        H = torch.empty_like(A)
        tau = torch.empty(*lead, n, dtype=A.dtype)
        info = torch.zeros(*lead, dtype=torch.int32)
    else:
        H, tau, info = out
        if (H.shape != A.shape or H.dtype != A.dtype or tau.shape != (*lead, n)
                or tau.dtype != A.dtype or info.shape != lead or info.dtype != torch.int32
                or not (H.is_contiguous() and tau.is_contiguous() and info.is_contiguous())
                or H.device.type != "cpu" or tau.device.type != "cpu"
                or info.device.type != "cpu"):
            raise ValueError("out must be contiguous host (H, tau, info) matching the input")
    if batch > 0 and n > 0:
        stream = torch.cuda.current_stream().cuda_stream
        rc = _lib.lib().qrb200_geqrf_batched_host(A.data_ptr(), H.data_ptr(), tau.data_ptr(),
                                                   info.data_ptr(), batch, n,
                                                   _NATIVE[A.dtype], int(sub_batch), stream)
        if rc != _lib.QRB200_OK:
            raise _lib.QRB200Error(rc, "qrb200_geqrf_batched_host")
    if data.dtype not in _NATIVE:
        H, tau = H.to(data.dtype), tau.to(data.dtype)
    return H, tau, info


_OPS_LOADED = False


def load_torch_ops():
    """Register ``torch.ops.qrb200.geqrf(A) -> (H, tau, info)`` (the TORCH_LIBRARY operator in
    ``libqrb200_torch_ops.so``, a thin layer over the C ABI with CUDA and Meta kernels) and
    return the operator.  Raises if the library was not built."""
    global _OPS_LOADED
    from pathlib import Path
    if not _OPS_LOADED:
        path = Path(__file__).resolve().parent / "libqrb200_torch_ops.so"
        if not path.exists():
            raise ImportError(f"{path} is not built; run `python -m qrb200.build`")
        _lib.lib()  # the C ABI library the operator links to
        torch.ops.load_library(str(path))
        _OPS_LOADED = True
    return torch.ops.qrb200.geqrf


def raise_on_info(info: torch.Tensor) -> None:
    """Raise ``LinAlgError`` like torch.linalg.cholesky would (one device->host read)."""
    bad = (info & (_lib.INFO_CHOL1_NOT_PD | _lib.INFO_CHOL2_NOT_PD)) != 0
    if info.numel() and bool(bad.any()):
        idx = int(bad.reshape(-1).nonzero()[0])
        raise LinAlgError(
            f"qrb200: (Batch element {idx}): the Gram matrix of the CholeskyQR frame is not "
            "positive-definite (non-finite or degenerate input)")


def custom_kernel(data: torch.Tensor):
    """Drop-in for reflection_no_reflectors.custom_kernel: ``(H, tau)`` in data's dtype."""
    H, tau, info = geqrf(data)
    raise_on_info(info)
    return H, tau
