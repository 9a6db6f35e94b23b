"""qrb200 -- B200-native batched square QR with the reference's drop-in API.

    from qrb200 import custom_kernel
    H, tau = custom_kernel(A)          # A: (..., n, n) CUDA tensor, any float dtype

Mirrors ``custom_kernel`` of reflection_no_reflectors.py:181-196 (johnzfitch/qr-contest):
same signature, same output layout (torch.geqrf compact form), same dtype semantics,
same error on a Gram that is not positive definite.  The compute path is the CUDA library
``libqrb200.so`` (C ABI in ``include/qrb200.h``); there is no CPU fallback.
"""
from .api import custom_kernel, geqrf, geqrf_q, geqrf_rect, LinAlgError  # noqa: F401
from . import api  # noqa: F401

__all__ = ["custom_kernel", "geqrf", "geqrf_q", "geqrf_rect", "LinAlgError"]
