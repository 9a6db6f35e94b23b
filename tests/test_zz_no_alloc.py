"""GPU: the allocation-free entry point ``qrb200_geqrf_batched_noalloc``.

It exists for callers that cannot allocate device memory at the moment they factor
(host callbacks and allocator hooks where cudaMalloc would re-enter or deadlock, embedders
whose memory is fully pre-partitioned): its working buffers live in a 64 MiB device array
built into the library.  These tests call it through the C ABI twice in a row (the array
keeps the first call's contents) and compare every output with the regular entry point
``qrb200_geqrf_batched`` under the same tolerance as the other parity tests
(|dH| <= 2e-4 (1 + |H|), |dtau| <= 2e-4), plus the fp64 gates.

This file is named so that pytest collects it last.
"""
import pytest
import torch

from oracle import checker

pytestmark = pytest.mark.gpu


def _noalloc(A):
    from qrb200 import _lib
    n = A.shape[-1]
    batch = A.numel() // (n * n) if n else 0
    H = torch.empty_like(A)
    tau = torch.empty(*A.shape[:-1], dtype=A.dtype, device=A.device)
    info = torch.full(A.shape[:-2], -1, dtype=torch.int32, device=A.device)
    dt = {torch.float32: _lib.QRB200_F32, torch.bfloat16: _lib.QRB200_BF16,
          torch.float16: _lib.QRB200_F16}[A.dtype]
    rc = _lib.lib().qrb200_geqrf_batched_noalloc(
        A.data_ptr(), H.data_ptr(), tau.data_ptr(), info.data_ptr(), batch, n, dt,
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.QRB200_OK, _lib.status_string(rc)
    return H, tau, info


def _regular(A):
    import qrb200
    return qrb200.geqrf(A)


def _close(H1, t1, H2, t2):
    err = ((H1.float() - H2.float()).abs() / (1 + H2.float().abs())).max().item()
    terr = (t1.float() - t2.float()).abs().max().item()
    assert err <= 2e-4 and terr <= 2e-4, (err, terr)


@pytest.mark.parametrize("n,batch", [(512, 20), (64, 100)])
def test_noalloc_matches_regular_entry_point_twice(n, batch):
    g = torch.Generator(device="cuda").manual_seed(77 + n)
    A1 = torch.randn(batch, n, n, device="cuda", generator=g)
    A2 = torch.randn(batch, n, n, device="cuda", generator=g) * 3.0
    outs = []
    for A in (A1, A2):   # two calls in a row on the shared scratch
        outs.append(_noalloc(A))
    torch.cuda.synchronize()
    for A, (H, tau, info) in zip((A1, A2), outs):
        Hr, tr, ir = _regular(A)
        torch.cuda.synchronize()
        _close(H, tau, Hr, tr)
        assert torch.equal(info, ir) and int(info.abs().sum()) == 0
        _, _, _, _, passed = checker.check(A[:4], H[:4], tau[:4])
        assert bool(passed.all())


def test_noalloc_bf16_and_limit():
    from qrb200 import _lib
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(8, 96, 96, device="cuda", generator=g).to(torch.bfloat16)
    H, tau, info = _noalloc(A)
    Hr, tr, _ = _regular(A)
    torch.cuda.synchronize()
    _close(H, tau, Hr, tr)
    # one 2048 x 2048 problem does not fit the 64 MiB array: rejected up front, no launch
    rc = _lib.lib().qrb200_geqrf_batched_noalloc(1, 1, 1, 1, 1, 2048, _lib.QRB200_F32, None)
    assert rc == _lib.QRB200_ERR_SCRATCH_LIMIT
    assert "scratch" in _lib.status_string(rc)


def test_noalloc_largest_order_runs():
    # n = 1826 is the largest order whose working set fits the array with the default block
    # options (1827 is rejected, see tests/test_abi.py); one such matrix factors and passes
    from qrb200 import _lib
    n = _lib.NOALLOC_MAX_N_DEFAULT
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(1, n, n, device="cuda", generator=g)
    H, tau, info = _noalloc(A)
    torch.cuda.synchronize()
    assert int(info.sum()) == 0
    _, _, _, _, passed = checker.check(A, H, tau)
    assert bool(passed.all())


def test_noalloc_allocates_nothing():
    # after a warm-up call (which may load kernel modules), a call changes neither the
    # device's free memory nor torch's allocator statistics
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(24, 256, 256, device="cuda", generator=g)
    out = _noalloc(A)
    torch.cuda.synchronize()
    del out
    from qrb200 import _lib
    n, batch = 256, 24
    H = torch.empty_like(A)
    tau = torch.empty(batch, n, device="cuda")
    info = torch.empty(batch, dtype=torch.int32, device="cuda")
    free1, _ = torch.cuda.mem_get_info()
    st1 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    rc = _lib.lib().qrb200_geqrf_batched_noalloc(
        A.data_ptr(), H.data_ptr(), tau.data_ptr(), info.data_ptr(), batch, n, _lib.QRB200_F32,
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == _lib.QRB200_OK
    free2, _ = torch.cuda.mem_get_info()
    st2 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    assert free2 == free1, (free1, free2)
    assert st2 == st1
    assert int(info.sum()) == 0
