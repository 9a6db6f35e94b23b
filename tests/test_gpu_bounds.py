"""GPU: the bounds-check build (libqrb200_checked.so, compiled with -DQRB_BOUNDS_CHECK).

The LU's pivot maps are the only data-dependent indices of the pipeline.  In this build every
row index read from them is checked; an out-of-range one would raise QRB200_INFO_BOUNDS and be
redirected inside its buffer instead of faulting.  This test runs the checked build through the
C ABI on every kernel path (warp, one-CTA, staged register panels, cluster panels, shared-memory
panels, float32 tiles for n % 4 != 0, bf16 input) and requires clean info words and results
identical to the regular library's.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _checked():
    from qrb200 import _lib
    h = ctypes.CDLL(str(_lib.CHECKED_LIB_PATH))
    for name, (res, args) in _lib.SIGNATURES.items():
        fn = getattr(h, name)
        fn.restype, fn.argtypes = res, args
    return h


@pytest.mark.parametrize("n,b,dtype", [(16, 64, torch.float32), (33, 40, torch.float32),
                                       (64, 40, torch.float32), (96, 30, torch.float32),
                                       (130, 12, torch.float32), (200, 12, torch.bfloat16),
                                       (512, 12, torch.float32), (1040, 2, torch.float32)])
def test_bounds_checked_build_is_clean_and_identical(n, b, dtype):
    import qrb200
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(b, n, seed=91, device="cuda").to(dtype)
    H0, t0, i0 = qrb200.geqrf(A)
    h = _checked()
    H, tau = torch.empty_like(A), torch.empty(b, n, dtype=dtype, device="cuda")
    info = torch.full((b,), -1, dtype=torch.int32, device="cuda")
    code = {torch.float32: _lib.QRB200_F32, torch.bfloat16: _lib.QRB200_BF16}[dtype]
    rc = h.qrb200_geqrf_batched(A.data_ptr(), H.data_ptr(), tau.data_ptr(), info.data_ptr(), b, n,
                                code, None, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == _lib.QRB200_OK
    assert not bool((info & _lib.INFO_BOUNDS).any())
    assert torch.equal(info, i0)
    assert torch.equal(H, H0) and torch.equal(tau, t0)
