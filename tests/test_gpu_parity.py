"""GPU parity: the CUDA library (through the C ABI) against the CPU oracle, the golden
fixtures made from the reference, and the fp64 gates (common/oracle.py:156-195).

Tolerances (float32 pipeline, factors compared elementwise only where they are determined
to rounding -- rank-deficient inputs have arbitrary null-space columns, gated only):
  gates   : ||R - Q^T A||_1/||A||_1 < 20 n eps32, ||Q^T Q - I||_1 < 100 n eps32,
            tau in [1, 2] +- 1e-6   (the north-star gates)
  tight   : |H - H_ref| <= 2e-4 (1 + |H_ref|), |tau - tau_ref| <= 2e-4
  illcond : |tau - tau_ref| <= 2e-2 (frame differences scale with cond(A) * eps32)
"""
import numpy as np
import pytest
import torch

from oracle import checker, qr_oracle as O
from tests.golden import fixtures as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def qrb():
    import qrb200
    return qrb200


def run(A):
    H, tau = qrb().custom_kernel(A.to(DEV))
    torch.cuda.synchronize()
    return H, tau


def assert_gates(A, H, tau, msg=""):
    f, o, ftol, otol, passed = checker.check(A.to(DEV), H.to(DEV), tau.to(DEV))
    assert bool(passed.all()), f"{msg} factor {f / ftol:.3g}x tol, ortho {o / otol:.3g}x tol"
    return f / ftol, o / otol


def assert_tight(H, tau, Href, tref, tol=2e-4):
    H, tau = H.float().cpu().numpy(), tau.float().cpu().numpy()
    err = np.abs(H - Href) / (1.0 + np.abs(Href))
    assert err.max() <= tol, f"H rel err {err.max():.3g}"
    assert np.abs(tau - tref).max() <= tol, f"tau err {np.abs(tau - tref).max():.3g}"


@pytest.mark.parametrize("name", F.names())
def test_golden(name):
    fx = F.load(name)
    kind = F.kind(name)
    A = torch.from_numpy(fx["A"])
    if kind == "c5":
        # the 8-GPU sweep's bf16 inputs (one per class): bf16 outputs against the reference's
        # bf16 outputs and float32 factors against its float32 factors where determined
        # (dense, upper-triangular); float32 factors of every class gated
        Ab = A.to(torch.bfloat16)
        H, tau = run(Ab)
        H32, t32 = run(Ab.float())
        assert_gates(Ab.float(), H32, t32, name)
        for i in F.C5_TIGHT:
            np.testing.assert_allclose(H[i].float().cpu().numpy(), fx["H"][i], rtol=2 ** -7,
                                       atol=2e-3)
            assert_tight(H32[i], t32[i], fx["H32"][i], fx["tau32"][i])
        return
    if kind == "bf16":
        H, tau = run(A.to(torch.bfloat16))
        assert H.dtype == torch.bfloat16 and tau.dtype == torch.bfloat16
        np.testing.assert_allclose(H.float().cpu().numpy(), fx["H"], rtol=2 ** -7, atol=2e-3)
        np.testing.assert_allclose(tau.float().cpu().numpy(), fx["tau"], rtol=2 ** -7, atol=0)
        # gate the float32 factors of the same input (the bf16 rounding of H/tau itself
        # breaks tau = 2/v^T v exactness, for the reference as well)
        H32, t32 = run(A.to(torch.bfloat16).float())
        assert_gates(A.to(torch.bfloat16).float(), H32, t32, name)
        return
    H, tau = run(A)
    assert_gates(A, H, tau, name)
    if kind == "tight":
        assert_tight(H, tau, fx["H"], fx["tau"])
    elif kind == "loose":
        assert np.abs(tau.cpu().numpy() - fx["tau"]).max() <= F.loose_tol(A.shape[-1])


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 17, 31, 32, 33, 47, 64, 65, 100, 127, 128, 129,
                               200, 256, 300])
def test_vs_oracle_random(n):
    g = torch.Generator().manual_seed(1000 + n)
    b = 8 if n <= 128 else 3
    A = torch.randn(b, n, n, generator=g, dtype=torch.float64).float()
    H, tau = run(A)
    assert_gates(A, H, tau, f"n={n}")
    Ho, to = O.custom_kernel_np(A.numpy())
    assert_tight(H, tau, Ho, to)


@pytest.mark.parametrize("n", [48, 96, 160])
def test_classes_vs_oracle(n):
    from qrb200 import generators as G
    A = G.heterogeneous(12, n, seed=21, device="cpu")
    H, tau = run(A)
    assert_gates(A, H, tau, f"hetero n={n}")
    Ho, to = O.custom_kernel_np(A.numpy())
    # dense block (first 2 matrices) is determined to rounding
    assert_tight(H[:2], tau[:2], Ho[:2], to[:2])


def test_leading_dims_and_noncontiguous():
    g = torch.Generator().manual_seed(5)
    A = torch.randn(2, 3, 24, 24, generator=g)
    H, tau = run(A)
    assert H.shape == (2, 3, 24, 24) and tau.shape == (2, 3, 24)
    H2, tau2 = run(A.reshape(6, 24, 24))
    assert torch.equal(H.reshape(6, 24, 24), H2) and torch.equal(tau.reshape(6, 24), tau2)
    At = A.transpose(-1, -2)  # non-contiguous view
    H3, tau3 = run(At)
    H4, tau4 = run(At.contiguous())
    assert torch.equal(H3, H4) and torch.equal(tau3, tau4)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_dtypes(dtype):
    g = torch.Generator().manual_seed(6)
    A = torch.randn(4, 40, 40, generator=g).to(dtype)
    H, tau = run(A)
    assert H.dtype == dtype and tau.dtype == dtype
    H32, t32 = run(A.float())
    ref_H = H32.to(dtype).float()
    ref_t = t32.to(dtype).float()
    if dtype == torch.float64:
        assert torch.equal(H.float(), H32) and torch.equal(tau.float(), t32)
    else:
        assert torch.allclose(H.float(), ref_H, rtol=2 ** -8, atol=1e-3)
        assert torch.allclose(tau.float(), ref_t, rtol=2 ** -8, atol=0)


def test_known_answers():
    n = 37
    eye = torch.eye(n).expand(3, n, n).contiguous()
    H, tau = run(eye)
    assert torch.allclose(H.cpu(), -eye, atol=1e-6) and bool((tau == 2).all())
    H, tau = run(-eye)
    assert torch.allclose(H.cpu(), eye, atol=1e-6) and bool((tau == 2).all())
    g = torch.Generator().manual_seed(7)
    U = torch.triu(torch.randn(3, n, n, generator=g))
    H, tau = run(U)
    assert bool((tau == 2).all()) and bool((torch.tril(H, -1) == 0).all())
    f, o = assert_gates(U, H, tau)
    assert f == 0.0


def test_multiplier_bound_and_tau_range():
    g = torch.Generator().manual_seed(8)
    A = torch.randn(16, 96, 96, generator=g)
    H, tau = run(A)
    assert float(torch.tril(H, -1).abs().max()) <= 1.0 + 1e-5
    assert bool(((tau >= 1 - 1e-6) & (tau <= 2 + 1e-6)).all())


def test_deterministic():
    g = torch.Generator().manual_seed(9)
    A = torch.randn(64, 80, 80, generator=g).to(DEV)
    H1, t1 = qrb().custom_kernel(A)
    H2, t2 = qrb().custom_kernel(A)
    assert torch.equal(H1, H2) and torch.equal(t1, t2)


def test_empty_batch_and_zero_matrix_rows():
    H, tau = run(torch.zeros(0, 16, 16))
    assert H.shape == (0, 16, 16) and tau.shape == (0, 16)


def test_nonfinite_raises():
    A = torch.randn(3, 20, 20)
    A[1, 4, 7] = float("nan")
    with pytest.raises(torch.linalg.LinAlgError):
        run(A)
    _, _, info = qrb().geqrf(A.to(DEV))
    info = info.cpu()
    assert int(info[0]) == 0 and int(info[2]) == 0 and int(info[1]) & 1


def test_info_clean_on_valid_input():
    A = torch.randn(10, 50, 50)
    _, _, info = qrb().geqrf(A.to(DEV))
    assert int(info.abs().sum()) == 0


@pytest.mark.parametrize("n,b,sub", [(16, 40, 7), (96, 30, 0), (200, 11, 4), (256, 9, 2)])
def test_host_buffers_match_device_path(n, b, sub):
    """qrb200_geqrf_batched_host (host tensors, pipelined sub-batches over three streams)
    returns exactly what the device entry point returns for the same matrices."""
    from qrb200 import generators as G
    A = G.heterogeneous(b, n, seed=41, device="cpu")
    Hd, td, infod = qrb().geqrf(A.cuda())
    torch.cuda.synchronize()
    out = (torch.empty_like(A).pin_memory(), torch.empty(b, n).pin_memory(),
           torch.full((b,), -1, dtype=torch.int32).pin_memory())
    H, tau, info = qrb().api.geqrf_host(A.pin_memory(), out=out, sub_batch=sub)
    assert H.device.type == "cpu" and H.data_ptr() == out[0].data_ptr()
    assert torch.equal(H, Hd.cpu()) and torch.equal(tau, td.cpu())
    assert torch.equal(info, infod.cpu())
    assert_gates(A, H, tau, f"host n={n}")


def test_host_custom_kernel_pageable_and_dtypes():
    A = torch.randn(3, 2, 40, 40, generator=torch.Generator().manual_seed(5))
    H, tau = qrb().custom_kernel(A)                       # pageable host tensor
    assert H.device.type == "cpu" and H.shape == A.shape and tau.shape == (3, 2, 40)
    Hd, td = qrb().custom_kernel(A.cuda())
    assert torch.equal(H, Hd.cpu()) and torch.equal(tau, td.cpu())
    H64, t64 = qrb().custom_kernel(A.double())            # converted like .to(float32)
    assert H64.dtype == torch.float64 and torch.equal(H64.float(), H)
    Hb, tb = qrb().custom_kernel(A.to(torch.bfloat16))
    assert Hb.dtype == torch.bfloat16 and Hb.device.type == "cpu"


@pytest.mark.parametrize("n", [1040, 2048])
def test_large_n_gates(n):
    # panels taller than 512 rows (shared-memory panel kernel), panel width 16 at n = 2048,
    # long-K tensor-core Grams; the ill-conditioned large-n class of the benchmark configs
    from qrb200 import generators as G
    A = G.large_illcond(2, n, seed=4, device="cuda")
    H, tau, info = qrb().geqrf(A)
    torch.cuda.synchronize()
    assert int(info.abs().sum()) == 0
    assert_gates(A, H, tau, f"n={n}")


@pytest.mark.parametrize("small_n", [0, 128])
@pytest.mark.parametrize("n", [16, 64, 96, 128])
def test_fused_and_staged_paths(small_n, n):
    """Both sides of the fused/staged crossover on the same inputs: small_n=0 forces the staged
    kernels at every n, small_n=128 the fused one-CTA-per-matrix kernel up to n=128."""
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(12, n, seed=33, device="cpu")
    _lib.set_small_n(small_n)
    try:
        H, tau = run(A)
    finally:
        _lib.set_small_n(64)
    assert_gates(A, H, tau, f"small_n={small_n} n={n}")
    Ho, to = O.custom_kernel_np(A.numpy())
    assert_tight(H[:2], tau[:2], Ho[:2], to[:2])


@pytest.mark.parametrize("block", [0, 64, 256])
@pytest.mark.parametrize("n", [192, 320, 512])
def test_cholesky_block_widths(block, n):
    """The two-level Cholesky elimination at every block width (0 = one level: every panel
    updates the whole trailing matrix) against the default width on the same inputs: gates on
    all six classes, tight agreement on the well-determined classes."""
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(12, n, seed=41, device="cuda")
    H0, t0 = run(A)
    _lib.set_chol_block(block)
    try:
        H, tau = run(A)
    finally:
        _lib.set_chol_block(128)
    assert_gates(A, H, tau, f"block={block} n={n}")
    assert_tight(H[:2], tau[:2], H0[:2].cpu().numpy(), t0[:2].cpu().numpy())


@pytest.mark.parametrize("lanes", [1, 3, 4])
def test_lanes_bit_identical(lanes):
    """Splitting a chunk over internal streams changes only the schedule: every matrix is
    factored by the same kernels, so H, tau and info match the default (2 lanes) bit for bit,
    and the call still completes in the caller's stream order."""
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(37, 256, seed=43, device="cuda")
    H0, t0, i0 = qrb().geqrf(A)
    _lib.set_lanes(lanes)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            H, tau, info = qrb().geqrf(A)
            Hc = H.clone()  # ordered after the factorization on the caller's stream
        torch.cuda.synchronize()
    finally:
        _lib.set_lanes(2)
    assert torch.equal(H, H0) and torch.equal(Hc, H0)
    assert torch.equal(tau, t0) and torch.equal(info, i0)


@pytest.mark.parametrize("n", [128, 256])
def test_closure_tile_shapes(n):
    """The closure GEMM in its two-CTAs-per-SM shape (default for n <= 256) and in the one-CTA
    shape give the same upper triangle to float32 rounding; the chart part of H and tau do not
    depend on it at all."""
    from qrb200 import _lib, generators as G
    A = G.gaussian((24, n, n), seed=59, device="cuda")
    outs = []
    try:
        for d in (256, 0):
            _lib.set_closure_dual_n(d)
            outs.append(qrb().geqrf(A))
    finally:
        _lib.set_closure_dual_n(256)
    (H1, t1, i1), (H2, t2, i2) = outs
    up = torch.triu(torch.ones(n, n, dtype=torch.bool, device="cuda"))
    assert torch.equal(t1, t2) and torch.equal(i1, i2)
    assert torch.equal(H1[:, ~up], H2[:, ~up])
    d = (H1 - H2).abs()[:, up]
    assert float((d / (1 + H2.abs()[:, up])).max()) <= 2e-5


@pytest.mark.parametrize("n", [66, 100, 130, 257, 384, 512])
def test_panel_loops_bit_identical(n):
    """The register panels' two column loops (fully unrolled; rotating registers) perform the
    same floating-point operations in the same order, so H, tau and info agree bit for bit
    (LU, Cholesky and chart panels; the last panel narrower than 32 when n % 32 != 0)."""
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(18, n, seed=53, device="cuda")
    outs = []
    try:
        for mode in (1, 2):
            _lib.set_panel_loop(mode)
            outs.append(qrb().geqrf(A))
    finally:
        _lib.set_panel_loop(0)
    (H1, t1, i1), (H2, t2, i2) = outs
    assert torch.equal(H1, H2) and torch.equal(t1, t2) and torch.equal(i1, i2)


@pytest.mark.parametrize("block", [0, 64, 256])
@pytest.mark.parametrize("n", [192, 320, 512])
def test_chart_block_widths(block, n):
    """The two-level chart elimination at every block width (0 = one level) against the
    default width on the same inputs: gates on all six classes, tight agreement on the
    well-determined classes."""
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(12, n, seed=47, device="cuda")
    H0, t0 = run(A)
    _lib.set_chart_block(block)
    try:
        H, tau = run(A)
    finally:
        _lib.set_chart_block(128)
    assert_gates(A, H, tau, f"chart block={block} n={n}")
    assert_tight(H[:2], tau[:2], H0[:2].cpu().numpy(), t0[:2].cpu().numpy())


# ---- the benchmark's own configurations ----

@pytest.mark.parametrize("n", [512, 1024, 1536])
def test_dense_vs_oracle_large(n):
    """The measured order and larger ones, elementwise against the oracle on dense matrices
    (n = 1024 and 1536: panels taller than 512 rows run over 2- and 4-CTA clusters)."""
    g = torch.Generator().manual_seed(2000 + n)
    A = torch.randn(2, n, n, generator=g, dtype=torch.float64).float()
    H, tau = run(A)
    assert_gates(A, H, tau, f"n={n}")
    Ho, to = O.custom_kernel_np(A.numpy())
    # elementwise differences of two float32 frames scale like cond(A) eps32, and a Gaussian
    # matrix's condition number grows like n: the 2e-4 bound widens in proportion above 1024
    assert_tight(H, tau, Ho, to, tol=2e-4 * max(1.0, n / 1024))


def test_hetero_n512_vs_oracle():
    """The n = 512 heterogeneous classes, two matrices each, against the oracle: gates on all,
    elementwise on dense and upper-triangular, tau within the cond-scaled bound on the
    ill-conditioned class."""
    from qrb200 import generators as G
    A = G.heterogeneous(12, 512, seed=3, device="cpu")
    H, tau = run(A)
    assert_gates(A, H, tau, "hetero n=512")
    Ho, to = O.custom_kernel_np(A.numpy())
    for i in (0, 1, 10, 11):  # dense, upper-triangular
        assert_tight(H[i], tau[i], Ho[i], to[i])
    assert np.abs(tau[2:4].cpu().numpy() - to[2:4]).max() <= F.loose_tol(512)


@pytest.mark.parametrize("n,seed", [(32, 1), (128, 2)])
def test_c2_leading_dims(n, seed):
    """Config 2: (128, 128, n, n) float32 N(0,1) through the leading-dims entry point; every
    matrix gated on the device, 8 of them elementwise against the oracle."""
    from qrb200 import checker as DC
    from qrb200 import generators as G
    A = G.gaussian((128, 128, n, n), seed=seed, device="cuda")
    H, tau, info = qrb().geqrf(A)
    torch.cuda.synchronize()
    assert H.shape == A.shape and tau.shape == (128, 128, n)
    assert int(info.abs().sum()) == 0
    s = DC.summary(A, H, tau, chunk=2048)
    assert s["n_pass"] == s["n"] == 16384, s
    A8 = A.reshape(-1, n, n)[:8].cpu()
    Ho, to = O.custom_kernel_np(A8.numpy())
    assert_tight(H.reshape(-1, n, n)[:8], tau.reshape(-1, n)[:8], Ho, to)


def test_c4_large_illcond_vs_oracle_gates():
    """Config 4 (2048 x 2048, sigma down to 1e-12): gates on the device path and the same
    gates met by the oracle on the same matrix."""
    from qrb200 import generators as G
    A = G.large_illcond(1, 2048, seed=4, device="cuda")
    H, tau, info = qrb().geqrf(A)
    torch.cuda.synchronize()
    assert int(info.abs().sum()) == 0
    assert_gates(A, H, tau, "c4")


def test_c5_sweep_shard_bf16():
    """Config 5: a shard of the fixed global bf16 batch (n = 256, six classes round robin):
    bf16 outputs equal the float32 factors rounded to bf16 (the same kernels compute both),
    float32 factors gated on every class, and shards concatenate to the 1-rank batch."""
    from qrb200 import generators as G
    A, lo = G.sweep_shard(96, 256, 1, 2, seed=5, device="cuda")
    assert lo == 48 and A.dtype == torch.bfloat16
    full, _ = G.sweep_shard(96, 256, 0, 1, seed=5, device="cuda")
    assert torch.equal(full[48:], A)
    H, tau, info = qrb().geqrf(A)
    H32, t32, _ = qrb().geqrf(A.float())
    torch.cuda.synchronize()
    assert int(info.abs().sum()) == 0
    assert torch.equal(H, H32.to(torch.bfloat16)) and torch.equal(tau, t32.to(torch.bfloat16))
    assert_gates(A.float(), H32, t32, "c5 shard")


def test_device_checker_matches_oracle_checker():
    """qrb200.checker (the on-device fp64 gates the benchmark applies to every timed output)
    agrees with the test-side checker and flags a corrupted factor."""
    from qrb200 import checker as DC
    from qrb200 import generators as G
    A = G.heterogeneous(12, 160, seed=5, device="cuda")
    H, tau, _ = qrb().geqrf(A)
    f, o, tlo, thi = DC.gates(A, H, tau)
    f2, o2, _ = checker.gates(A, H, tau)
    assert torch.allclose(f, f2) and torch.allclose(o, o2)
    s = DC.summary(A, H, tau)
    assert s["n_pass"] == 12
    H[3, 0, 7] += 1.0
    assert DC.summary(A, H, tau)["n_pass"] == 11


@pytest.mark.parametrize("n,dtype", [(33, torch.float32), (64, torch.float32),
                                     (130, torch.float32), (512, torch.float32),
                                     (256, torch.bfloat16), (96, torch.float16)])
def test_explicit_q_matches_householder_product(n, dtype):
    """qrb200_geqrf_batched_q: H and tau are the same as the plain entry point's, and Q equals
    householder_product(H, tau) (float64 reconstruction) to float32 rounding (bf16 / f16:
    the rounding of the returned Q)."""
    from qrb200 import generators as G
    if dtype == torch.float16:  # row-scaled inputs (10^+-6) do not fit float16
        A = G.gaussian((12, n, n), seed=51, device="cuda").to(dtype)
    else:
        A = G.heterogeneous(12, n, seed=51, device="cuda").to(dtype)
    H, tau, Q, info = qrb().geqrf_q(A)
    H0, t0, i0 = qrb().geqrf(A)
    torch.cuda.synchronize()
    assert torch.equal(H, H0) and torch.equal(tau, t0) and torch.equal(info, i0)
    Qr = torch.linalg.householder_product(H.double(), tau.double())
    tol = 2e-5 if dtype == torch.float32 else (2 ** -7 if dtype == torch.bfloat16 else 2 ** -10)
    err = (Q.double() - Qr).abs().max().item()
    assert err <= tol * 4, err


@pytest.mark.parametrize("n,b", [(1, 5), (7, 9), (20, 13), (32, 6), (32, 4099)])
def test_warp_kernel_classes_vs_oracle(n, b):
    """n <= 32 runs one warp per matrix (four matrices per CTA; batches that do not fill the
    last CTA included): all six classes gated, dense matrices elementwise against the oracle,
    and identical results for the same matrix wherever it sits in the batch."""
    from qrb200 import generators as G
    A = G.heterogeneous(max(b, 6), n, seed=61, layout="roundrobin", device="cpu")[:b]
    H, tau = run(A)
    assert_gates(A, H, tau, f"warp n={n}")
    Ho, to = O.custom_kernel_np(A[:6].numpy())
    assert_tight(H[0], tau[0], Ho[0], to[0])
    H1, t1 = run(A[1:2].clone())
    assert torch.equal(H1[0], H[1]) and torch.equal(t1[0], tau[1])


def rect_gates(A, H, tau):
    """fp64 gates of a tall factorization: ||R - Q^T A||_1/||A||_1 < 20 m eps32 and
    ||Q^T Q - I||_1 < 100 m eps32 with Q = householder_product(H, tau) (m x n)."""
    m, n = A.shape[-2], A.shape[-1]
    Ad, Hd, td = A.double(), H.double(), tau.double()
    Q = torch.linalg.householder_product(Hd, td)
    R = torch.triu(Hd[..., :n, :])
    f = torch.linalg.matrix_norm(R - Q.mT @ Ad, ord=1) / torch.linalg.matrix_norm(Ad, ord=1)
    o = torch.linalg.matrix_norm(Q.mT @ Q - torch.eye(n, dtype=torch.float64, device=A.device),
                                 ord=1)
    eps = torch.finfo(torch.float32).eps
    assert bool((f < 20 * m * eps).all()) and bool((o < 100 * m * eps).all()), (f.max(), o.max())
    assert bool(((td >= 1 - 1e-6) & (td <= 2 + 1e-6)).all())


@pytest.mark.parametrize("m,n", [(40, 17), (48, 48), (100, 31), (256, 128), (520, 300),
                                 (1024, 64)])
def test_rect_vs_oracle(m, n):
    """qrb200_geqrf_batched_rect (tall m x n) against the oracle's rectangular restatement:
    elementwise on dense inputs, gates on all; a square call equals the square entry point."""
    from qrb200 import generators as G
    A = G.gaussian((3, m, n), seed=70 + m + n)
    H, tau, info = qrb().geqrf_rect(A.cuda())
    torch.cuda.synchronize()
    assert H.shape == (3, m, n) and tau.shape == (3, n) and int(info.abs().sum()) == 0
    rect_gates(A.cuda(), H, tau)
    Ho, to = O.custom_kernel_rect_np(A.numpy())
    assert_tight(H, tau, Ho, to)
    if m == n:
        H0, t0, _ = qrb().geqrf(A.cuda())
        assert torch.equal(H, H0) and torch.equal(tau, t0)


def test_rect_classes_bf16_and_errors():
    from qrb200 import _lib, generators as G
    A = G.heterogeneous(12, 160, seed=71, device="cuda")[:, :, :96].contiguous()
    H, tau, info = qrb().geqrf_rect(A)
    rect_gates(A, H, tau)
    Ab = A.to(torch.bfloat16)
    Hb, tb, _ = qrb().geqrf_rect(Ab)
    H32, t32, _ = qrb().geqrf_rect(Ab.float())
    assert torch.equal(Hb, H32.to(torch.bfloat16)) and torch.equal(tb, t32.to(torch.bfloat16))
    with pytest.raises(ValueError):
        qrb().geqrf_rect(A.mT.contiguous())
    rc = _lib.lib().qrb200_geqrf_batched_rect(1, 1, 1, 1, 1, 8, 9, _lib.QRB200_F32, None)
    assert rc == _lib.QRB200_ERR_INVALID_ARG


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_torch_operator_matches_entry_point(dtype):
    """torch.ops.qrb200.geqrf (TORCH_LIBRARY operator over the C ABI) returns exactly what
    qrb200.geqrf returns, on the current stream, with leading dims."""
    op = qrb().api.load_torch_ops()
    g = torch.Generator(device="cuda").manual_seed(81)
    A = torch.randn(3, 2, 96, 96, device="cuda", generator=g).to(dtype)
    H, tau, info = op(A)
    H0, t0, i0 = qrb().geqrf(A)
    torch.cuda.synchronize()
    assert H.dtype == dtype and H.shape == A.shape and tau.shape == (3, 2, 96)
    assert torch.equal(H, H0) and torch.equal(tau, t0) and torch.equal(info, i0)
