#!/usr/bin/env python
"""Benchmark: batched fp32 QR matrices/s at n=512 on the heterogeneous batch.

Workload (one "step"): one call of the library on the heterogeneous n=512 batch of 1536
float32 matrices (256 each of dense / ill-conditioned / rank-deficient / row-scaled /
near-rank-deficient / upper-triangular; seeded synthetic data, seed 3 + rank).  Inputs are
1.5 GiB per step, larger than the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qrb200|reference]

N > 1 is launched by torchrun (one rank per GPU, NCCL); every rank factors its own 1536
matrices (weak scaling, no collective on the data path) and the time is the max over ranks.
``--impl reference`` times the reference algorithm's CPU restatement (oracle port) on the
host cores, rank 0 only.
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

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "batched fp32 QR matrices/s at n=512 (heterogeneous 6-class batch)"
UNIT = "matrices/s"


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


def family_bytes(n: int) -> dict:
    """Algorithmic HBM bytes of each family per matrix (float32 working set)."""
    nb = nb_for(n)
    b = {k: 0.0 for k in family_flops(n)}
    for k0 in range(0, n, nb):
        w = min(nb, n - k0)
        m = n - k0
        t = n - k0 - w
        k1 = k0 + w
        b["lu_panel"] += 4.0 * (m * w + n * w + t * w)
        b["chart_panel"] += 4.0 * (m * w + m * w + t * w)
        b["chol_panel"] += 2 * 4.0 * (m * w + m * w)
        b["lu_trail"] += 4.0 * (2 * t * t + t * w + w * t)
        b["chart_trail"] += 4.0 * (2 * t * t + t * w + w * t)
        b["chol_trail"] += 2 * 4.0 * (t * t + 2 * t * w + 2 * t * k1)  # G lower half, L_G^-1
    # two-level Cholesky and chart eliminations (the library's default block of 128 columns
    # when 32-wide panels are used and n > 128): C moves once per panel only inside the block
    # strips, and once per block for the rest
    blk = 128
    if nb == 32 and n > blk and n % 4 == 0:
        chol = chart = 8.0 * n * n  # chart: the frame copied into the working buffer once
        for kb in range(0, n, blk):
            ke = min(n, kb + blk)
            for k0 in range(kb, ke, nb):
                w = min(nb, n - k0)
                k1 = k0 + w
                c = ke - k1
                # Cholesky: block columns of every row below (lower part), L_G^-1 rows in block
                chol += 8.0 * ((n - k1) * c - c * (c - 1) / 2) + 4.0 * ((n - k1) * w + w * c)
                chol += 4.0 * ((ke - k1) * k0 + (ke - k0) * k1 + (ke - k0) * w + w * k1)
                # chart: block columns of every row below, block rows right of the block
                chart += 8.0 * ((n - k1) * c + c * (n - ke)) + 4.0 * ((n - k1) * w + w * (n - k1))
            t2, K = n - ke, ke - kb
            if t2 > 0:
                chol += 8.0 * t2 * (t2 + 1) / 2 + 4.0 * 2 * K * t2           # trailing triangle
                chol += 4.0 * (t2 * kb + t2 * ke + t2 * K + K * ke)          # L_G^-1 rows below
                chart += 8.0 * t2 * t2 + 4.0 * 2 * K * t2
        b["chol_trail"] = 2 * chol
        b["chart_trail"] = chart
    b["gram"] = 2 * 4.0 * (n * n + n * n / 2)
    b["q_apply"] = 4.0 * (2 * n * n + n * n / 2) + 4.0 * (3 * n * n + n * n / 2)
    b["closure"] = 4.0 * (2 * n * n + n * n / 2)
    return b


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


def cpu_port_rate(A_cpu: torch.Tensor, threads: int):
    """Time the numpy oracle (the reference algorithm restated) on host cores."""
    from oracle import qr_oracle
    torch.set_num_threads(threads)
    A = A_cpu.numpy()
    t0 = time.perf_counter()
    qr_oracle.custom_kernel_np(A)
    return A.shape[0] / (time.perf_counter() - t0)


def cpu_sample(n: int, per_class: int, seed: int = 3):
    from qrb200 import generators as G
    g = G._gen(seed, "cpu")
    parts = [G.make_class(c, per_class, n, g, "cpu").float() for c in G.CLASSES]
    return torch.cat(parts)


def config(args, world):
    return {"workload": f"heterogeneous n={args.n} fp32, {args.batch} matrices per GPU "
                        "(6 classes x 256)",
            "n": args.n, "batch_per_gpu": args.batch, "global_batch": args.batch * world,
            "parallelism": f"batch-sharded x{world} (no data-path collective)",
            "l2": "inputs larger than L2 (1.5 GiB per step), no flush"}


# ----------------------------------------------------------------------------------------
def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    per = 2
    A = cpu_sample(args.n, per, seed=3)
    from oracle import qr_oracle
    torch.set_num_threads(cores)
    for _ in range(args.warmup):
        qr_oracle.custom_kernel_np(A.numpy())
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        qr_oracle.custom_kernel_np(A.numpy())
        times.append(time.perf_counter() - t0)
    rate = A.shape[0] * len(times) / sum(times)
    line = {"metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config(args, world),
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{A.shape[0]} matrices per step ({per} per class, "
                                       f"n={args.n}, seed 3) through the numpy restatement "
                                       "of reflection_no_reflectors.custom_kernel"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_qrb(args):
    import qrb200
    from qrb200 import _lib, api
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
    ws = torch.empty(api.workspace_bytes(B, n), dtype=torch.uint8, device=dev)
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

    # ---- roofline: per-family device time with CUDA events on the launch stream ----
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
    dom = max(fams, key=fams.get)
    hbm, bf16, src = measured_peaks()
    ff = family_flops(n)[dom] * B
    fb = family_bytes(n)[dom] * B
    t_dom = fams[dom] / 1000.0
    tc_peak = bf16 / 2 / 3  # 3xTF32 roof: TF32 rate is half the bf16 rate, three products
    t_tc, t_hbm = ff / (tc_peak * 1e12), fb / (hbm * 1e9)
    if t_tc >= t_hbm:
        roof = {"bound": "tensor", "achieved": ff / t_dom / 1e12, "peak": tc_peak,
                "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": fb / t_dom / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    # DRAM bytes per matrix of the chol_trail kernels from an ncu capture of the same
    # configuration at 256 matrices (dram__bytes_read.sum + dram__bytes_write.sum summed over
    # the family's launches), scaled to the batch; writes that were still in L2 when each
    # profiled launch ended are not in it
    traffic_per_matrix = {("chol_trail", 512): 9.54e6}.get((dom, n))
    roof["traffic"] = traffic_per_matrix * B if traffic_per_matrix else None
    if traffic_per_matrix:
        roof["traffic_unit"] = "bytes per step (ncu, 256-matrix capture scaled to the batch)"
    roof["kernel"] = dom
    roof["peak_source"] = (f"{src} MEASURED_PEAKS.json: bf16 {bf16} TF/s / 2 (TF32) / 3 "
                           f"(3xTF32), HBM {hbm} GB/s")
    roof["family_ms_per_step"] = {k: round(v, 4) for k, v in fams.items()}
    roof["family_share"] = {k: round(v / sum(fams.values()), 4) for k, v in fams.items()}
    whole_tflops = value / world * algo_flops(n) / 1e12
    roof["pipeline_tflops_7n3"] = whole_tflops
    roof["pipeline_frac_of_3xtf32_roof"] = whole_tflops / tc_peak

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

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        As = cpu_sample(n, args.cpu_sample, seed=3)
        rate = cpu_port_rate(As, cores)
        cpu = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{As.shape[0]} matrices ({args.cpu_sample} per class, n={n}, "
                         "seed 3) through the numpy restatement of the reference pipeline"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": max(3, args.warmup),
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config(args, world), "roofline": roof, "cpu_baseline": cpu,
                "e2e": e2e, "gpu_launches": launches, "clocks": clk,
                "gflops_4n3_per_s": value * 4 * n ** 3 / 3 / 1e9,
                "device": torch.cuda.get_device_name(dev)}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_qrb(args)


if __name__ == "__main__":
    main()
