"""GPU unit tests of the GEMM-shaped stages, tcgen05 3xTF32 tiles (register loader = 1,
TMA-fed = 2, TMA-fed in the two-CTAs-per-SM shape = 4, rank-w = 2/3 for the trailing update) and
SIMT tiles (0), each against a float64 product of the same operands.

Tolerance: |C - C64| <= 2e-5 * (|A| |B|)_ij + 1e-30 elementwise -- the float32 error bound
of a K-term dot product (3xTF32 products are accurate to ~2^-21 relative, float32 sums add
K * 2^-24).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def kit():
    from qrb200 import build
    h = ctypes.CDLL(str(build.TESTKIT))
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    h.qrbt_gram.argtypes = [P, P, P, I64, I, I, P]
    h.qrbt_trailw.argtypes = [P, P, P, P, P, I64, I, I, I, I, I, P]
    h.qrbt_syrk.argtypes = [P, P, P, I64, I, I, I, I, P]
    h.qrbt_closure.argtypes = [P, P, P, P, P, I64, I, I, P]
    h.qrbt_qapply.argtypes = [P, P, P, P, P, I64, I, I, I, P]
    return h


def stream():
    return torch.cuda.current_stream().cuda_stream


def close(C, C64, bound):
    err = (C.double() - C64).abs()
    ratio = (err / (2e-5 * bound + 1e-30)).max().item()
    assert ratio <= 1.0, f"error {ratio:.3g} x bound"


@pytest.mark.parametrize("tc", [0, 1, 2, 4])
@pytest.mark.parametrize("n", [128, 256, 384, 132])
def test_gram(tc, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    X = torch.randn(3, n, n, device="cuda", generator=g)
    G = torch.full_like(X, float("nan"))
    info = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert kit().qrbt_gram(X.data_ptr(), G.data_ptr(), info.data_ptr(), 3, n, tc, stream()) == 0
    torch.cuda.synchronize()
    X64 = X.double()
    ref = X64.mT @ X64
    bound = X64.abs().mT @ X64.abs()
    low = torch.tril(torch.ones(n, n, dtype=torch.bool, device="cuda"))
    close(torch.where(low, G, 0).nan_to_num(), torch.where(low, ref, 0), bound)
    assert int(info.sum()) == 0


@pytest.mark.parametrize("tc", [0, 1, 2, 3])
@pytest.mark.parametrize("gather", [False, True])
@pytest.mark.parametrize("n,k0,k1", [(256, 32, 64), (512, 0, 32), (192, 160, 176)])
def test_trailw(tc, gather, n, k0, k1):
    b = 2
    g = torch.Generator(device="cuda").manual_seed(7 + n + k0)
    Cold = torch.randn(b, n, n, device="cuda", generator=g)
    Cnew = torch.full_like(Cold, float("nan"))
    ldw = 32
    W = torch.randn(b, n, ldw, device="cuda", generator=g)
    if gather:
        src = torch.stack([torch.randperm(n, device="cuda", generator=g) for _ in range(b)])
        src = src.to(torch.int32).contiguous()
        sp = src.data_ptr()
    else:
        src = torch.arange(n, device="cuda", dtype=torch.int32).expand(b, n).contiguous()
        sp = None
    info = torch.zeros(b, dtype=torch.int32, device="cuda")
    rc = kit().qrbt_trailw(Cold.data_ptr(), Cnew.data_ptr(), W.data_ptr(), sp, info.data_ptr(),
                           b, n, k0, k1, ldw, tc, stream())
    assert rc == 0
    torch.cuda.synchronize()
    w = k1 - k0
    bi = torch.arange(b, device="cuda")[:, None]
    C64 = Cold.double()
    Cg = C64[bi, src.long()]                        # rows in the new order
    Wt = W[:, k1:, :w].double()
    Bm = Cg[:, k0:k1, k1:]
    ref = Cg[:, k1:, k1:] - Wt @ Bm
    bound = Cg[:, k1:, k1:].abs() + Wt.abs() @ Bm.abs()
    close(Cnew[:, k1:, k1:], ref, bound)


@pytest.mark.parametrize("tc", [0, 1])
@pytest.mark.parametrize("n,k0,k1", [(256, 32, 64), (512, 96, 128)])
def test_syrk(tc, n, k0, k1):
    b = 2
    g = torch.Generator(device="cuda").manual_seed(11 + n)
    G = torch.randn(b, n, n, device="cuda", generator=g)
    R = torch.randn(b, n, n, device="cuda", generator=g)
    G0 = G.double().clone()
    info = torch.zeros(b, dtype=torch.int32, device="cuda")
    assert kit().qrbt_syrk(G.data_ptr(), R.data_ptr(), info.data_ptr(), b, n, k0, k1, tc,
                           stream()) == 0
    torch.cuda.synchronize()
    R12 = R[:, k0:k1, k1:].double()
    ref = G0[:, k1:, k1:] - R12.mT @ R12
    bound = G0[:, k1:, k1:].abs() + R12.abs().mT @ R12.abs()
    m = n - k1
    low = torch.tril(torch.ones(m, m, dtype=torch.bool, device="cuda"))
    close(torch.where(low, G[:, k1:, k1:], 0), torch.where(low, ref, 0), bound)


@pytest.mark.parametrize("tc", [0, 1, 2, 4])
@pytest.mark.parametrize("n", [128, 256, 260])
def test_closure(tc, n):
    b = 2
    g = torch.Generator(device="cuda").manual_seed(13 + n)
    Q = torch.randn(b, n, n, device="cuda", generator=g)
    A = torch.randn(b, n, n, device="cuda", generator=g)
    sgn = torch.where(torch.rand(b, n, device="cuda", generator=g) > 0.5, 1.0, -1.0)
    H = torch.zeros(b, n, n, device="cuda")
    info = torch.zeros(b, dtype=torch.int32, device="cuda")
    assert kit().qrbt_closure(Q.data_ptr(), A.data_ptr(), sgn.data_ptr(), H.data_ptr(),
                              info.data_ptr(), b, n, tc, stream()) == 0
    torch.cuda.synchronize()
    Q64, A64 = Q.double(), A.double()
    ref = torch.triu(sgn.double()[:, :, None] * (Q64.mT @ A64))
    bound = Q64.abs().mT @ A64.abs()
    close(torch.triu(H), ref, bound)
    assert float(torch.tril(H, -1).abs().max()) == 0.0


@pytest.mark.parametrize("tc", [0, 1, 2, 4])
@pytest.mark.parametrize("pass2", [0, 1])
@pytest.mark.parametrize("n", [128, 384])
def test_qapply(tc, pass2, n):
    b = 2
    g = torch.Generator(device="cuda").manual_seed(17 + n)
    X = torch.randn(b, n, n, device="cuda", generator=g)
    # strict lower part = L^{-1} entries; upper part holds unrelated data that must be ignored
    RL = torch.randn(b, n, n, device="cuda", generator=g) * 0.1
    D = 1.0 + 0.5 * torch.rand(b, n, device="cuda", generator=g)
    Q = torch.full_like(X, float("nan"))
    info = torch.zeros(b, dtype=torch.int32, device="cuda")
    assert kit().qrbt_qapply(X.data_ptr(), RL.data_ptr(), D.data_ptr(), Q.data_ptr(),
                             info.data_ptr(), b, n, pass2, tc, stream()) == 0
    torch.cuda.synchronize()
    Linv = torch.tril(RL.double(), -1) + torch.eye(n, dtype=torch.float64, device="cuda")
    Rinv = Linv.mT / D.double().sqrt()[:, None, :]
    X64 = X.double()
    if pass2:
        F = torch.eye(n, dtype=torch.float64, device="cuda") - Rinv
        ref = X64 - X64 @ F
        bound = X64.abs() + X64.abs() @ F.abs()
    else:
        ref = X64 @ Rinv
        bound = X64.abs() @ Rinv.abs()
    close(Q, ref, bound)


@pytest.mark.parametrize("tc", [0, 2])
def test_gram_long_k(tc):
    # K = 2048: the TMA tile drains its TMEM accumulator into float32 registers every 256 k,
    # which keeps the error inside the float32 bound (a single TMEM accumulation does not)
    test_gram(tc, 2048)


def test_bounded_wait_times_out_cleanly():
    # Failure detection without a GPU fault: a short bounded wait on an mbarrier that nothing
    # completes runs out in every CTA; each one reports INFO_DEVICE_TIMEOUT, frees its tensor
    # memory and returns.  The context stays usable: tensor-core work runs right after it
    # (2 x 148 CTAs so that every SM's TMEM is taken and freed at least once).
    from qrb200 import _lib
    h = kit()
    h.qrbt_timeout_probe.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_void_p]
    blocks = 296
    info = torch.zeros(blocks, dtype=torch.int32, device="cuda")
    assert h.qrbt_timeout_probe(info.data_ptr(), blocks, 4096, stream()) == 0
    torch.cuda.synchronize()
    assert bool((info == _lib.INFO_DEVICE_TIMEOUT).all())
    test_gram(2, 256)
