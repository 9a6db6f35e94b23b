"""CPU: the N > 1 path -- batch sharding and result gathering over world_size-2 gloo ranks,
and a failing rank that the others observe on a bounded timeout (no GPU involved)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]

from qrb200.shard import shard_range  # noqa: E402


def test_shard_range_covers_batch():
    for batch in (0, 1, 7, 16, 1536, 65537):
        for world in (1, 2, 3, 8):
            got = [shard_range(batch, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [h - l for l, h in got]
            assert max(sizes) - min(sizes) <= max(1, -(-batch // world))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, batch, n, out, fail_rank):
    sys.path[:0] = [str(REPO), str(REPO / "qr-contest_b200")]
    import datetime
    import torch.distributed as dist
    from oracle import qr_oracle
    from qrb200.shard import gather_results, shard_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(123)
        A = torch.randn(batch, n, n, generator=g)
        lo, hi = shard_range(batch, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host")
        H, tau = qr_oracle.custom_kernel(A[lo:hi])   # per-rank worker (CPU stand-in)
        Hall, tall = gather_results(H, tau, batch)
        if rank == 0:
            out["H"] = Hall.numpy()
            out["tau"] = tall.numpy()
        out[f"ok{rank}"] = True
    except Exception as e:  # the surviving rank sees its collective fail within the timeout
        out[f"err{rank}"] = type(e).__name__
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, batch, n, fail_rank=-1):
    mgr = mp.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [mp.get_context("spawn").Process(target=_worker,
                                             args=(r, world, port, batch, n, out, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
        if p.is_alive():
            p.kill()
    return dict(out)


def test_two_rank_shard_gather_matches_single_process():
    from oracle import qr_oracle
    batch, n = 7, 12
    out = _run(2, batch, n)
    assert out.get("ok0") and out.get("ok1"), out
    g = torch.Generator().manual_seed(123)
    A = torch.randn(batch, n, n, generator=g)
    H, tau = qr_oracle.custom_kernel_np(A.numpy())
    np.testing.assert_array_equal(out["H"], H)
    np.testing.assert_array_equal(out["tau"], tau)


def test_failing_rank_is_observed_on_bounded_timeout():
    out = _run(2, 6, 8, fail_rank=1)
    assert out.get("err1") == "RuntimeError"
    assert "err0" in out and not out.get("ok0")
