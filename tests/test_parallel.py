"""Multi-process (gloo, CPU) tests of the data-parallel host logic.

The shard + one all-reduce step must reproduce the full-batch gradients; a
rank that fails before the collective must surface as an error on the others
(process-group timeout), never as a hang.  GPU kernels are not involved: the
per-shard gradients come from the CPU oracle."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from piecewiselinearembeddings_optimized_b200.parallel import GradientBucket, shard_bounds


def test_shard_bounds_cover_batch():
    for n in (1, 7, 1024, 1_048_576):
        for ws in (1, 2, 3, 8):
            spans = [shard_bounds(n, ws, r) for r in range(ws)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, ws, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=10))
    try:
        from oracle import ple_oracle as o
        from piecewiselinearembeddings_optimized_b200 import workloads

        wl = workloads.make_workload("c1", n=512)
        g = workloads.make_grad(wl)
        edges, inv_w, nb = o.pad_bins(wl.bins)
        lo, hi = shard_bounds(wl.n, ws, rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the collective")
        part = o.embeddings_backward(g[lo:hi], wl.x[lo:hi], edges, inv_w, nb, wl.weight, version="B",
                                     activation=True, w0=wl.w0, b0=wl.b0)
        params = [torch.nn.Parameter(torch.zeros(s)) for s in (wl.weight.shape, wl.w0.shape, wl.b0.shape)]
        for p, key in zip(params, ("grad_W", "grad_w0", "grad_b0")):
            p.grad = torch.from_numpy(part[key].astype(np.float32))
        bucket = GradientBucket(params)
        bucket.gather()
        bucket.all_reduce()
        bucket.scatter()
        q.put((rank, "ok", [p.grad.numpy().copy() for p in params]))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(ws, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q, mode)) for r in range(ws)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_sharded_allreduce_equals_full_batch():
    from oracle import ple_oracle as o
    from piecewiselinearembeddings_optimized_b200 import workloads

    res = _run(2, "ok")
    assert all(r[1] == "ok" for r in res), res
    wl = workloads.make_workload("c1", n=512)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    full = o.embeddings_backward(g, wl.x, edges, inv_w, nb, wl.weight, version="B", activation=True,
                                 w0=wl.w0, b0=wl.b0)
    for rank, _, grads in res:
        for got, key in zip(grads, ("grad_W", "grad_w0", "grad_b0")):
            np.testing.assert_allclose(got, full[key], rtol=1e-5, atol=1e-5, err_msg=f"rank {rank} {key}")


def test_failed_rank_surfaces_as_error():
    res = _run(2, "fail")
    status = {r[0]: r[1] for r in res}
    assert status[1] == "error"
    assert status[0] == "error"  # the survivor's collective times out instead of hanging
