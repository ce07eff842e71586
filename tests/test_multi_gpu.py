"""Data-parallel step on 2+ GPUs: each rank runs the fused backward on its
batch shard and one NCCL all-reduce of the packed parameter gradients.  The
reduced gradients must match the CPU oracle's full-batch gradients (and the
single-GPU full-batch kernel), and each rank's grad_x rows the oracle's rows
of its shard.  Skipped with fewer than two visible GPUs."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, ws, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import rtdl_num_embeddings_cuda  # noqa: F401
        from oracle import ple_oracle as o
        from piecewiselinearembeddings_optimized_b200 import workloads
        from piecewiselinearembeddings_optimized_b200.parallel import GradientBucket, shard_bounds

        ops = torch.ops.rtdl_num_embeddings_cuda
        wl = workloads.make_workload("c5", n=8192, f=64)
        g = workloads.make_grad(wl)
        edges, inv_w, nb = o.pad_bins(wl.bins)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        te, tr, tn, tw, tw0, tb0 = map(T, (edges, inv_w, nb, wl.weight, wl.w0, wl.b0))
        lo, hi = shard_bounds(wl.n, ws, rank)
        tx, tg = T(wl.x[lo:hi]), T(g[lo:hi])
        params = [torch.nn.Parameter(torch.empty_like(t)) for t in (tw, tw0, tb0)]
        bucket = GradientBucket(params)
        gxs, gw, _, gw0, gb0 = ops.embeddings_backward(tg, tx, te, tr, tn, tw, None, tw0, tb0, None, 2, True,
                                                        torch.float32, True, True, False, True)
        shard_gx = gxs.cpu().numpy()
        for v, src in zip(bucket.views, (gw, gw0, gb0)):
            v.copy_(src)
        bucket.all_reduce()
        reduced = [v.cpu().numpy() for v in bucket.views]
        full = None
        if rank == 0:
            fx, fg = T(wl.x), T(g)
            _, fw, _, fw0, fb0 = ops.embeddings_backward(fg, fx, te, tr, tn, tw, None, tw0, tb0, None, 2, True,
                                                          torch.float32, False, True, False, True)
            full = [t.cpu().numpy() for t in (fw, fw0, fb0)]
            absg = np.abs(g).sum(0)
            k = o.bin_index(wl.x, edges, nb)
            tmax = max(1.0, float(np.abs(o.position(wl.x, k, edges, inv_w)).max()))
            bounds = [np.broadcast_to(absg[:, None, :] * tmax, fw.shape), np.einsum("nfd,nf->fd", np.abs(g),
                      np.abs(wl.x)), absg]
            q.put((rank, "ok", (reduced, shard_gx, lo, hi), full, bounds))
        else:
            q.put((rank, "ok", (reduced, shard_gx, lo, hi), None, None))
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_allreduce_matches_full_batch():
    from oracle import ple_oracle as o

    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ws = 2
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(ws)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    assert all(r[1] == "ok" for r in res), [r[2] for r in res if r[1] != "ok"]
    full, bounds = res[0][3], res[0][4]
    # the CPU oracle's full-batch gradients (dense upstream formulation, float64 accumulation)
    from piecewiselinearembeddings_optimized_b200 import workloads

    wl = workloads.make_workload("c5", n=8192, f=64)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    ref = o.embeddings_backward(g, wl.x, edges, inv_w, nb, wl.weight, version="B", activation=True, w0=wl.w0,
                                b0=wl.b0)
    oracle = (ref["grad_W"], ref["grad_w0"], ref["grad_b0"])
    for rank, _, (reduced, shard_gx, lo, hi), _, _ in res:
        for got, one_gpu, want, bd, name in zip(reduced, full, oracle, bounds, ("grad_W", "grad_w0", "grad_b0")):
            o.assert_reduction_close(got, want, 2 * bd, err_msg=f"rank {rank} {name} vs the oracle")
            o.assert_reduction_close(got, one_gpu, 2 * bd, err_msg=f"rank {rank} {name} vs one GPU")
        np.testing.assert_allclose(shard_gx, ref["grad_x"][lo:hi], rtol=1e-4, atol=1e-5,
                                   err_msg=f"rank {rank} grad_x rows {lo}..{hi}")
