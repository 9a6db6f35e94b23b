#!/usr/bin/env python
"""Benchmark: batched fp32 QR matrices/s at n=512 on the heterogeneous batch.

Workload (one "step"): one call of the library on the heterogeneous n=512 batch of 1536
float32 matrices (256 each of dense / ill-conditioned / rank-deficient / row-scaled /
near-rank-deficient / upper-triangular; seeded synthetic data, seed 3 + rank).  Inputs are
1.5 GiB per step, larger than the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qrb200|reference] [--quick]

N > 1 is launched by torchrun (one rank per GPU, NCCL); every rank factors its own 1536
matrices (weak scaling, no collective on the data path) and the time is the max over ranks.
Every output of the timed steps is gated afterwards in float64 on the device.

Besides the headline the line carries the other BASELINE.json configurations, each measured
on the device: ``c2`` (small n, leading dims (128, 128, n, n)), ``c4`` (64 matrices of
2048 x 2048, sigma down to 1e-12) and ``c5`` (the fixed global batch of 65536 bf16
256 x 256 matrices sharded over the ranks, factorization and NCCL all-gather timed apart),
the host-link roof of the end-to-end path, the reference's own ``custom_kernel`` and
``torch.geqrf`` on the host cores and on the GPU (context), and the roofline.

``--impl reference`` times the reference's own ``custom_kernel`` (pure PyTorch, installed
unmodified under baseline/_ref) on the host cores of this node, rank 0 only; without that
install it falls back to the numpy restatement under oracle/ (kind "port").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "qr-contest_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "batched fp32 QR matrices/s at n=512 (heterogeneous 6-class batch)"
UNIT = "matrices/s"
REF_DIR = REPO / "baseline" / "_ref"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of every kernel of one library
# call, per matrix, from an ncu capture of the n = 512 heterogeneous configuration at 256
# matrices (profiles/dram_traffic_all_kernels_n512_b256.md); None until captured
TRAFFIC_PER_MATRIX = {512: 35.80e6}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["qrb200", "reference"], default="qrb200")
    p.add_argument("--n", type=int, default=512)
    p.add_argument("--batch", type=int, default=1536)
    p.add_argument("--cpu-sample", type=int, default=16, help="matrices per class (CPU leg)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--quick", action="store_true",
                   help="headline only: no extra configurations, GPU context or gates")
    p.add_argument("--ref-kernels", action="store_true",
                   help="context only: time the reference's own CUDA stage kernels "
                        "(kan_metric/kqr_fused.py fused_qr, kan_metric/kqr_cluster_kan.py "
                        "cluster_qr; JIT-compiled from baseline/_ref) against qrb200 on the same "
                        "inputs, print one JSON line and exit")
    p.add_argument("--profile-run", action="store_true",
                   help="one warm-up call and one measured call of the library, nothing else "
                        "(the command the ncu summaries under profiles/ are taken on)")
    return p.parse_args()


# ----------------------------------------------------------------------------------------
# algorithmic work model (per matrix)
# ----------------------------------------------------------------------------------------
def algo_flops(n: int) -> float:
    """7 n^3: LU 2n^3/3 + 2 x (Gram n^3 + Cholesky n^3/3 + TRSM n^3) + closure n^3 + chart
    2n^3/3 (the permutation is free; split-precision extra products are not counted)."""
    return 7.0 * n ** 3


def algo_bytes(n: int, elem: int = 4) -> float:
    """Read A once, write H and tau once."""
    return elem * (2 * n * n + n)


def nb_for(n: int) -> int:
    for w in (32, 16, 8):
        if n * (w + 1) * 4 + 3 * n * 4 + (w + 16) * 4 + 64 <= 200 * 1024:
            return w
    return 8


def family_flops(n: int) -> dict:
    """Algorithmic flops each kernel family performs on one matrix."""
    nb = nb_for(n)
    f = {k: 0.0 for k in ("lu_panel", "lu_trail", "gram", "chol_panel", "chol_trail", "q_apply",
                          "chart_panel", "chart_trail", "closure", "small_fused")}
    for k0 in range(0, n, nb):
        w = min(nb, n - k0)
        m = n - k0
        k1 = k0 + w
        panel = sum(2.0 * (m - c - 1) * (w - c - 1) + (m - c - 1) for c in range(w))
        wcalc = max(0, m - w) * w * (w - 1)  # W = L21 L11^{-1}
        f["lu_panel"] += panel + wcalc
        f["chart_panel"] += panel + wcalc
        f["chol_panel"] += 2 * panel
        t = n - k1
        f["lu_trail"] += 2.0 * t * t * w
        f["chart_trail"] += 2.0 * t * t * w
        f["chol_trail"] += 2 * (t * t * w + 2.0 * t * k1 * w)  # two passes: SYRK half + L_G^-1
    f["gram"] = 2.0 * n ** 3            # two Grams, symmetric half each
    f["q_apply"] = 2.0 * n ** 3         # two passes of X R^{-1} (R^{-1} upper triangular)
    f["closure"] = 1.0 * n ** 3         # upper triangle of Q^T A
    return f


# ----------------------------------------------------------------------------------------
def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.f = None
        try:
            u = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            u = ""
        self.uuid = u.lower().replace("gpu-", "")

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        mine = [r for r in rows if len(r) >= 10 and r[1].lower().replace("gpu-", "") == self.uuid]
        if not mine:
            mine = [r for r in rows if len(r) >= 10]
        sm = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in mine if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in mine for i in range(4) if r[6 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(mine)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local



def load_reference():
    """The reference's own module (reflection_no_reflectors, pure PyTorch) from its unmodified
    install under baseline/_ref, or None when it is not installed."""
    if not (REF_DIR / "reflection_no_reflectors.py").exists():
        return None
    sys.dont_write_bytecode = True
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import reflection_no_reflectors as ref
    return ref


def cpu_sample(n: int, per_class: int, seed: int = 3):
    from qrb200 import generators as G
    g = G._gen(seed, "cpu")
    parts = [G.make_class(c, per_class, n, g, "cpu").float() for c in G.CLASSES]
    return torch.cat(parts)


def cpu_rate(fn, A, reps: int = 1):
    """matrices/s of ``fn(A)`` on the host (one untimed call first)."""
    fn(A)
    t0 = time.perf_counter()
    for _ in range(reps):
        fn(A)
    return reps * A.shape[0] / (time.perf_counter() - t0)


def cpu_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def config(args, world):
    return {"workload": f"heterogeneous n={args.n} fp32, {args.batch} matrices per GPU "
                        "(6 classes x 256)",
            "n": args.n, "batch_per_gpu": args.batch, "global_batch": args.batch * world,
            "parallelism": f"batch-sharded x{world} (no data-path collective)",
            "l2": "inputs larger than L2 (1.5 GiB per step), no flush"}


def dev_time(fn, dev, reps: int, warm: int = 1, world: int = 1):
    """Mean device milliseconds of ``fn()`` over ``reps`` calls (CUDA events on the current
    stream, barrier + synchronize on both sides, max over ranks)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        fn()
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


# ----------------------------------------------------------------------------------------
def run_reference(args):
    """The reference arm: the reference's own custom_kernel on the host cores (rank 0)."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    # torch's default thread count is every core of the host; calling torch.set_num_threads
    # (even with the same value) makes MKL's batched LU under torch.linalg.lu fail here
    cores = torch.get_num_threads()
    per = 2
    A = cpu_sample(args.n, per, seed=3)
    ref = load_reference()
    if ref is not None:
        kind = "reference"

        def fn(X):
            return ref.custom_kernel(X.clone())
        what = ("the reference's own reflection_no_reflectors.custom_kernel (unmodified, "
                "baseline/_ref) on torch CPU")
    else:
        from oracle import qr_oracle
        kind = "port"

        def fn(X):
            return qr_oracle.custom_kernel_np(X.numpy())
        what = "the numpy restatement of reflection_no_reflectors.custom_kernel (oracle/)"
    for _ in range(args.warmup):
        fn(A)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn(A)
        times.append(time.perf_counter() - t0)
    rate = A.shape[0] * len(times) / sum(times)
    line = {"metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config(args, world),
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": kind,
                             "cpu": cpu_name(),
                             "scope": "the host CPU of this node, run once (rank 0 only "
                                      "under torchrun; the other ranks do no work)",
                             "sample": f"{A.shape[0]} matrices per step ({per} per class, "
                                       f"n={args.n}, seed 3) through {what}"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------
def roofline(value_per_gpu: float, n: int, fams: dict, B: int) -> dict:
    """Roofline of the headline: the whole call's 7 n^3 flops per matrix against the 3xTF32
    tensor roof (n = 512 runs at ~447 flop per algorithmic byte, far above the ridge), with
    every kernel family's own algorithmic flops against the same roof beside it."""
    hbm, bf16, src = measured_peaks()
    sus = None
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        sus = json.loads(p.read_text()).get("bf16_tflops_sustained")
    tc_peak = bf16 / 2 / 3  # TF32 runs at half the bf16 rate; 3 products per float32 product
    achieved = value_per_gpu * algo_flops(n) / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
            "frac": achieved / tc_peak,
            "kernel": "whole qrb200_geqrf_batched call (all kernel families, 7 n^3 per matrix)",
            "peak_source": (f"{src} MEASURED_PEAKS.json bf16 {bf16} TF/s (burst) / 2 (TF32) "
                            "/ 3 (3xTF32 products)")}
    if sus:
        roof["frac_of_sustained"] = achieved / (float(sus) / 6)
    alg_bytes = algo_bytes(n) * B
    tpm = TRAFFIC_PER_MATRIX.get(n)
    roof["algorithmic_bytes_per_step"] = alg_bytes
    roof["traffic"] = tpm * B if tpm else None
    if tpm:
        roof["traffic_unit"] = ("DRAM bytes per step: ncu dram__bytes_read.sum + "
                                "dram__bytes_write.sum over every kernel of a 256-matrix call, "
                                "scaled to the batch")
        roof["waste"] = tpm / algo_bytes(n)
    roof["hbm_frac_of_algorithmic_bytes"] = value_per_gpu * algo_bytes(n) / 1e9 / hbm
    ff = family_flops(n)
    total = sum(fams.values()) or 1.0
    per = {}
    for k, ms in fams.items():
        if ms <= 0:
            continue
        tf = ff.get(k, 0.0) * B / (ms / 1000.0) / 1e12
        per[k] = {"ms": round(ms, 4), "share": round(ms / total, 4),
                  "tflops": round(tf, 3), "frac": round(tf / tc_peak, 4)}
    roof["families"] = per
    dom = max(per, key=lambda k: per[k]["ms"]) if per else None
    roof["dominant_family"] = dict(per[dom], name=dom) if dom else None
    return roof


def measure_host_link(Ah, out, dev, world):
    """Copy-engine roof of the end-to-end path: the step's upload and download bytes copied
    between the same pinned host buffers and the device, alone and both directions at once,
    on every rank at the same time (max over ranks)."""
    import torch.distributed as dist
    dA = torch.empty(Ah.shape, dtype=Ah.dtype, device=dev)
    dO = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in out]
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(up: bool, down: bool):
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        if up:
            with torch.cuda.stream(s1):
                dA.copy_(Ah, non_blocking=True)
        if down:
            with torch.cuda.stream(s2):
                for h, d in zip(out, dO):
                    h.copy_(d, non_blocking=True)
        torch.cuda.synchronize(dev)
        ms = (time.perf_counter() - t0) * 1e3
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    timed(True, True)
    up, down, both = timed(True, False), timed(False, True), timed(True, True)
    ub = Ah.numel() * Ah.element_size()
    db = sum(t.numel() * t.element_size() for t in out)
    del dA, dO
    return {"h2d_gbs_per_rank": ub / up / 1e6, "d2h_gbs_per_rank": db / down / 1e6,
            "both_directions_ms": both, "ranks_copying_at_once": world,
            "matrices_per_s_bound": world * Ah.shape[0] / (both / 1e3),
            "method": "host wall clock around cudaMemcpyAsync between the pinned step buffers "
                      "and device memory, after a barrier, max over ranks"}


def measure_c2(dev):
    """(128, 128, n, n) float32 iid N(0,1), n = 32 (seed 1) and 128 (seed 2)."""
    import qrb200
    from qrb200 import checker
    from qrb200 import generators as G
    hbm, bf16, _ = measured_peaks()
    res = {}
    for n, seed in ((32, 1), (128, 2)):
        A = G.gaussian((128, 128, n, n), seed=seed, device=dev)
        ws = torch.empty(qrb200.api.workspace_bytes(A.numel() // (n * n), n), dtype=torch.uint8,
                         device=dev)
        out = {}

        def step():
            out["r"] = qrb200.geqrf(A, workspace=ws)
        ms = dev_time(step, dev, reps=5, warm=3)
        H, tau, info = out["r"]
        b = A.numel() // (n * n)
        rate = b / (ms / 1e3)
        gbs = rate * algo_bytes(n) / 1e9
        tf = rate * algo_flops(n) / 1e12
        gates = checker.summary(A.reshape(-1, n, n)[:512], H.reshape(-1, n, n)[:512],
                                tau.reshape(-1, n)[:512])
        res[f"n{n}"] = {"shape": [128, 128, n, n], "matrices_per_s": rate, "ms": ms,
                        "hbm_gbs_algorithmic": gbs, "hbm_frac": gbs / hbm,
                        "tflops_7n3": tf, "tensor_frac": tf / (bf16 / 6),
                        "info_nonzero": int((info != 0).sum()), "gates_first_512": gates}
        # the other side of the fused / staged crossover on the same batch (evidence for it)
        from qrb200 import _lib
        small = 64
        _lib.set_small_n(0 if n <= small else 128)
        try:
            ws2 = torch.empty(qrb200.api.workspace_bytes(b, n), dtype=torch.uint8, device=dev)
            ms2 = dev_time(lambda: qrb200.geqrf(A, workspace=ws2), dev, reps=3, warm=1)
        finally:
            _lib.set_small_n(small)
        res[f"n{n}"]["other_path"] = {"path": "staged kernels" if n <= small else
                                      "fused one-CTA-per-matrix kernel",
                                      "ms": ms2, "matrices_per_s": b / (ms2 / 1e3)}
        res[f"n{n}"]["path"] = "fused one-CTA-per-matrix kernel" if n <= small else "staged kernels"
        Hh = torch.empty_like(A)
        th = torch.empty(b, n, device=dev)
        inf = torch.zeros(b, dtype=torch.int32, device=dev)
        rc, f = _lib.geqrf_batched_timed(A.data_ptr(), Hh.data_ptr(), th.data_ptr(),
                                         inf.data_ptr(), b, n, _lib.QRB200_F32, ws.data_ptr(),
                                         ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
        res[f"n{n}"]["family_ms"] = {k: round(v, 4) for k, v in f.items() if v > 0}
        del ws2, Hh, th, inf
        del A, ws, H, tau, info, out
    return res


def measure_c4(dev):
    """64 matrices of 2048 x 2048, U diag(sigma) V^T, sigma to 1e-12."""
    import qrb200
    from qrb200 import checker
    from qrb200 import generators as G
    _, bf16, _ = measured_peaks()
    n, b = 2048, 64
    A = G.large_illcond(b, n, seed=4, device=dev)
    ws = torch.empty(qrb200.api.workspace_bytes(b, n), dtype=torch.uint8, device=dev)
    out = {}

    def step():
        out["r"] = qrb200.geqrf(A, workspace=ws)
    ms = dev_time(step, dev, reps=2, warm=1)
    H, tau, info = out["r"]
    rate = b / (ms / 1e3)
    tf = rate * algo_flops(n) / 1e12
    gates = checker.summary(A[:4], H[:4], tau[:4], chunk=2)
    from qrb200 import _lib
    Hh, th = torch.empty_like(A), torch.empty(b, n, device=dev)
    inf = torch.zeros(b, dtype=torch.int32, device=dev)
    _, fam = _lib.geqrf_batched_timed(A.data_ptr(), Hh.data_ptr(), th.data_ptr(), inf.data_ptr(),
                                      b, n, _lib.QRB200_F32, ws.data_ptr(), ws.numel(),
                                      torch.cuda.current_stream(dev).cuda_stream)
    del Hh, th, inf
    r = {"matrices": b, "n": n, "ms": ms, "matrices_per_s": rate, "tflops_7n3": tf,
         "family_ms": {k: round(v, 3) for k, v in fam.items() if v > 0},
         "tensor_frac": tf / (bf16 / 6), "info_nonzero": int((info != 0).sum()),
         "gates_first_4": gates}
    del A, ws, H, tau, info, out
    return r


def measure_c5(dev, rank, world):
    """a fixed global batch of 65536 bf16 256 x 256 matrices (six classes,
    round robin, rank parameter 128), sharded contiguously over the ranks; factors computed in
    float32 and returned in bf16; then H and tau all-gathered over NCCL (timed apart)."""
    import qrb200
    from qrb200 import checker
    from qrb200 import generators as G
    _, bf16, _ = measured_peaks()
    n, gb = 256, 65536
    A, lo = G.sweep_shard(gb, n, rank, world, seed=5, device=dev, dtype=torch.bfloat16)
    b = A.shape[0]
    ws = torch.empty(qrb200.api.workspace_bytes(b, n), dtype=torch.uint8, device=dev)
    out = {}

    def step():
        out["r"] = qrb200.geqrf(A, workspace=ws)
    ms = dev_time(step, dev, reps=4, warm=1, world=world)
    H, tau, info = out["r"]
    del ws
    # per-family CUDA-event timings of the library on the first 8192 matrices of the shard
    from qrb200 import _lib
    bs = min(b, 8192)
    As = A[:bs].contiguous()
    wss = torch.empty(qrb200.api.workspace_bytes(bs, n), dtype=torch.uint8, device=dev)
    Hh, th = torch.empty_like(As), torch.empty(bs, n, dtype=As.dtype, device=dev)
    inf = torch.zeros(bs, dtype=torch.int32, device=dev)
    _, fam = _lib.geqrf_batched_timed(As.data_ptr(), Hh.data_ptr(), th.data_ptr(), inf.data_ptr(),
                                      bs, n, _lib.QRB200_BF16, wss.data_ptr(), wss.numel(),
                                      torch.cuda.current_stream(dev).cuda_stream)
    del As, wss, Hh, th, inf
    bad = int((info != 0).sum())
    # float32 factors of a sample of this shard's (bf16) inputs, gated in float64
    As = A[:96].float()
    Hs, ts, _ = qrb200.geqrf(As)
    gates = checker.summary(As, Hs, ts)
    r = {"global_batch": gb, "n": n, "dtype": "bf16 in/out, float32 compute",
         "per_rank": b, "factor_ms_max_over_ranks": ms,
         "matrices_per_s": gb / (ms / 1e3), "tflops_7n3": gb / (ms / 1e3) * algo_flops(n) / 1e12,
         "tensor_frac_per_gpu": gb / world / (ms / 1e3) * algo_flops(n) / 1e12 / (bf16 / 6),
         "info_nonzero_rank0": bad, "gates_rank0_sample96_fp32": gates,
         "scaling": "strong (fixed global batch)",
         "family_ms_first_8192": {k: round(v, 3) for k, v in fam.items() if v > 0}}
    if world > 1:
        import torch.distributed as dist
        Hall = torch.empty(gb, n, n, dtype=H.dtype, device=dev)
        tall = torch.empty(gb, n, dtype=tau.dtype, device=dev)

        def gather():
            dist.all_gather_into_tensor(Hall, H)
            dist.all_gather_into_tensor(tall, tau)
        gms = dev_time(gather, dev, reps=2, warm=1, world=world)
        moved = (world - 1) * b * (n * n + n) * 2
        r.update({"allgather_ms_max_over_ranks": gms,
                  "allgather_bytes_received_per_rank": moved,
                  "allgather_gbs_per_rank": moved / (gms / 1e3) / 1e9,
                  "limiter": "all-gather" if gms > ms else "factorization"})
        del Hall, tall
    else:
        r["allgather_ms_max_over_ranks"] = None
    del A, H, tau, info, out, As, Hs, ts
    return r


def gpu_context(A, dev):
    """Context (not a baseline arm): the reference's own custom_kernel and torch.geqrf run on
    this B200 on the first 256 matrices of the headline batch."""
    res = {}
    S = A[:256].contiguous()
    ref = load_reference()
    if ref is not None:
        ms = dev_time(lambda: ref.custom_kernel(S), dev, reps=1, warm=1)
        res["reference_custom_kernel_gpu"] = {"matrices_per_s": S.shape[0] / (ms / 1e3),
                                              "ms": ms, "matrices": S.shape[0]}
    ms = dev_time(lambda: torch.geqrf(S), dev, reps=1, warm=1)
    res["torch_geqrf_gpu"] = {"matrices_per_s": S.shape[0] / (ms / 1e3), "ms": ms,
                              "matrices": S.shape[0]}
    return res


def cpu_context(n: int, per_class: int):
    """The reference's own custom_kernel (cpu_baseline) and torch.geqrf on the host cores."""
    cores = torch.get_num_threads()  # the default: every core (see run_reference)
    As = cpu_sample(n, per_class, seed=3)
    sample = f"{As.shape[0]} matrices ({per_class} per class, n={n}, seed 3)"
    ref = load_reference()
    if ref is not None:
        rate = cpu_rate(lambda X: ref.custom_kernel(X.clone()), As)
        base = {"value": rate, "unit": UNIT, "cores": cores, "kind": "reference",
                "cpu": cpu_name(),
                "sample": sample + " through the reference's own "
                          "reflection_no_reflectors.custom_kernel (unmodified, baseline/_ref)"}
    else:
        from oracle import qr_oracle
        rate = cpu_rate(lambda X: qr_oracle.custom_kernel_np(X.numpy()), As)
        base = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port", "cpu": cpu_name(),
                "sample": sample + " through the numpy restatement of the reference pipeline"}
    geq = cpu_rate(lambda X: torch.geqrf(X), As, reps=2)
    return base, {"value": geq, "unit": UNIT, "cores": cores, "sample": sample}


def run_qrb(args):
    import qrb200
    from qrb200 import _lib, checker
    from qrb200 import generators as G

    world, rank, local = dist_setup()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    n, B = args.n, args.batch
    A = G.heterogeneous(B, n, seed=3 + rank, device=dev)
    ws = torch.empty(qrb200.api.workspace_bytes(B, n), dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def step():
        return qrb200.geqrf(A, workspace=ws)

    if args.profile_run:
        step()
        torch.cuda.synchronize(dev)
        step()
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_run": True, "launches_per_call": _lib.launch_count() // 2}))
        return

    for _ in range(max(3, args.warmup)):
        H, tau, info = step()
    torch.cuda.synchronize(dev)
    assert int(info.abs().sum()) == 0, "info flags raised on the benchmark batch"

    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    l0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        H, tau, info = step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    launches = _lib.launch_count() - l0
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * B * args.steps / (ms / 1000.0)

    # ---- every output of the last timed step, gated in float64 on the device ----
    gates = None
    if not args.quick:
        gates = checker.summary(A, H, tau)
        gates["info_nonzero"] = int((info != 0).sum())
        gates["what"] = ("all matrices of the last timed step on this rank: fp64 "
                         "householder_product, ||R - Q^T A||_1/||A||_1 / (20 n eps32), "
                         "||Q^T Q - I||_1 / (100 n eps32), tau in [1, 2] +- 1e-6")
    del H, tau, info

    # ---- per-family device time with CUDA events on the launch stream ----
    fams = {}
    reps = 2
    for _ in range(reps):
        Hh = torch.empty_like(A)
        th = torch.empty(B, n, device=dev)
        inf = torch.zeros(B, dtype=torch.int32, device=dev)
        rc, f = _lib.geqrf_batched_timed(A.data_ptr(), Hh.data_ptr(), th.data_ptr(),
                                         inf.data_ptr(), B, n, _lib.QRB200_F32, ws.data_ptr(),
                                         ws.numel(), stream.cuda_stream)
        assert rc == 0, rc
        for k, v in f.items():
            fams[k] = fams.get(k, 0.0) + v / reps
    del Hh, th, inf
    roof = roofline(value / world, n, fams, B)

    # ---- e2e through the public API with pinned host buffers ----
    e2e = None
    if not args.no_e2e:
        Ah = A.cpu().pin_memory()
        out = (torch.empty(B, n, n, dtype=torch.float32).pin_memory(),
               torch.empty(B, n, dtype=torch.float32).pin_memory(),
               torch.empty(B, dtype=torch.int32).pin_memory())
        e2e_steps = max(2, min(args.steps, 5))

        def e2e_step():
            # host buffers in, host buffers out: qrb200_geqrf_batched_host pipelines the
            # uploads, kernels and downloads of its sub-batches; blocks until H/tau/info land
            qrb200.api.geqrf_host(Ah, out=out)

        e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize(dev)
        ems = f0.elapsed_time(f1)
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": world * B * e2e_steps / (ems / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": Ah.numel() * 4,
               "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in out),
               "steps": e2e_steps,
               "path": "pinned host A -> qrb200.api.geqrf_host (C ABI "
                       "qrb200_geqrf_batched_host: sub-batches over 3 streams, copies overlapped "
                       "with kernels) -> pinned host H/tau/info"}
        if not args.quick:
            link = measure_host_link(Ah, out, dev, world)
            link["e2e_frac_of_link_bound"] = e2e["value"] / link["matrices_per_s_bound"]
            e2e["host_link"] = link
        del Ah, out

    extra = {}
    if not args.quick:
        del ws
        torch.cuda.empty_cache()
        if world == 1:
            # the single-GPU configs run before the sweep: after the sweep's ~40 GB of
            # allocations the n = 2048 batch measured 40 % slower in the same process
            extra["c2"] = measure_c2(dev)
            torch.cuda.empty_cache()
            extra["c4"] = measure_c4(dev)
            torch.cuda.empty_cache()
            extra["gpu_context"] = gpu_context(A, dev)
            torch.cuda.empty_cache()
        extra["c5"] = measure_c5(dev, rank, world)
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, geq = cpu_context(n, args.cpu_sample)
        extra["geqrf_cpu"] = geq

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": max(3, args.warmup),
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config(args, world), "roofline": roof, "cpu_baseline": cpu,
                "e2e": e2e, "gpu_launches": launches, "clocks": clk, "gates": gates,
                "gflops_4n3_per_s": value * 4 * n ** 3 / 3 / 1e9,
                "device": torch.cuda.get_device_name(dev)}
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_ref_kernels(args):
    """Same-box comparison with the reference's hand-written CUDA kernels for this pipeline:
    its fully fused one-block-per-matrix kernel (kan_metric/kqr_fused.py:230-305, FP32 Gram
    build GRAM_MODE=0) on the small-n batches of config 2, and its 16-CTA cluster kernel
    (kan_metric/kqr_cluster_kan.py:308-365, cluster_qr with C = 16) on n = 512.  Both are
    JIT-compiled by the reference's own load_inline calls from the unmodified copies under
    baseline/_ref.  Timed with CUDA events after a warm-up call; gated on the device."""
    import qrb200
    from qrb200 import checker
    from qrb200 import generators as G
    dev = torch.device("cuda", 0)
    sys.dont_write_bytecode = True
    sys.path[:0] = [str(REF_DIR / "kan_metric"), str(REF_DIR)]
    out = {"ref_kernels": {}}
    import kqr_fused  # the reference module (compiles kqr.py's modlu kernel on import)
    fused = kqr_fused._build(0)
    for n, seed in ((32, 1), (64, 1), (128, 2)):
        A = G.gaussian((16384, n, n), seed=seed, device=dev)
        r = {}
        ms_ref = dev_time(lambda: fused.fused_qr(A, 1), dev, reps=3, warm=1)
        H, tau = fused.fused_qr(A, 1)
        r["reference_fused_qr"] = {"ms": ms_ref, "matrices_per_s": A.shape[0] / (ms_ref / 1e3),
                                   "gates_first_512": checker.summary(A[:512], H[:512], tau[:512])}
        ms_q = dev_time(lambda: qrb200.geqrf(A), dev, reps=3, warm=1)
        Hq, tq, _ = qrb200.geqrf(A)
        r["qrb200"] = {"ms": ms_q, "matrices_per_s": A.shape[0] / (ms_q / 1e3),
                       "gates_first_512": checker.summary(A[:512], Hq[:512], tq[:512])}
        out["ref_kernels"][f"fused_n{n}_b16384"] = r
        del A, H, tau, Hq, tq
    import kqr_cluster_kan
    cl = kqr_cluster_kan._build(4, 3)
    A = G.heterogeneous(1536, 512, seed=3, device=dev)
    r = {}
    ms_ref = dev_time(lambda: cl.cluster_qr(A, 16), dev, reps=1, warm=1)
    H, tau = cl.cluster_qr(A, 16)
    r["reference_cluster_qr_C16"] = {"ms": ms_ref, "matrices_per_s": A.shape[0] / (ms_ref / 1e3),
                                     "gates": checker.summary(A, H, tau)}
    ms_q = dev_time(lambda: qrb200.geqrf(A), dev, reps=3, warm=1)
    Hq, tq, _ = qrb200.geqrf(A)
    r["qrb200"] = {"ms": ms_q, "matrices_per_s": A.shape[0] / (ms_q / 1e3),
                   "gates": checker.summary(A, Hq, tq)}
    out["ref_kernels"]["hetero_n512_b1536"] = r
    out["note"] = ("context, not a benchmark arm: the reference's CUDA stage kernels against "
                   "qrb200 on the same inputs on one B200; the cluster kernel's timing includes "
                   "the cudaDeviceSynchronize inside its host wrapper")
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.ref_kernels:
        run_ref_kernels(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_qrb(args)


if __name__ == "__main__":
    main()
