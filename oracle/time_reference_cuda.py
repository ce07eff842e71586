"""Time the REFERENCE's own CUDA ops on this GPU (a secondary, GPU-side baseline).

TEST / MEASUREMENT INFRASTRUCTURE ONLY: the ops come from
``oracle/_ref/rtdl_ref_ops.so``, compiled from the reference's sources by
``oracle/build_ref.py``; nothing here is part of the product.  The library
registers the same op namespace as this project (``rtdl_num_embeddings_cuda``),
so this script runs in its own process and never loads this project's native
library.

One step is the reference module's training step on the path
(``src/rtdl_num_embeddings_cuda/module.py:207-248`` and ``_autograd.py:42-96``):
``::forward`` (``csrc/ops.cpp:35-44``) for x_ple and the bin indices, the
PyTorch epilogue the module composes (``+ bias`` for version A, ReLU,
``linear0(x) + ...`` for version B), autograd through that epilogue, then
``::backward`` (``csrc/ops.cpp:46-58``) with the gradient of x_ple.  Inputs are
seeded synthetic draws with the configuration's shapes (as ``bench.py``), all
resident on the device; CUDA events, median of the timed steps.

    python oracle/time_reference_cuda.py --config c4 [--batch N] [--steps K] [--warmup W]

Prints one JSON line: step / forward-op / backward-op milliseconds and
feature-embeddings per second.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

REF_LIB = ROOT / "oracle" / "_ref" / "rtdl_ref_ops.so"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c4")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    if not REF_LIB.exists():
        print(json.dumps({"unavailable": f"{REF_LIB.name} not built (oracle/build_ref.py needs the reference sources)"}))
        return 0

    import torch

    from oracle.ple_oracle import pad_bins
    from piecewiselinearembeddings_optimized_b200 import workloads

    torch.ops.load_library(str(REF_LIB))
    ops = torch.ops.rtdl_num_embeddings_cuda
    dev = torch.device("cuda", 0)
    n0, F, D, version, relu, mode, out_mode = workloads.SPECS[args.config]
    N = args.batch or n0
    wl = workloads.make_workload(args.config, n=8)
    edges, inv_w, n_bins = [torch.from_numpy(a).to(dev) for a in pad_bins(wl.bins)]
    W = torch.from_numpy(wl.weight).to(dev)
    dt = {"f32": torch.float32, "bf16": torch.bfloat16}
    gen = torch.Generator(device=dev).manual_seed(4000)
    x = torch.randn(N, F, device=dev, generator=gen)
    if args.config == "c4":
        m = torch.rand(N, F, device=dev, generator=gen) < 0.01
        x[m] = torch.where(torch.rand(N, F, device=dev, generator=gen) < 0.5, -10.0, 10.0)[m]
    g = torch.randn(N, F, D, device=dev, generator=gen).to(dt[out_mode])
    bias = None if wl.bias is None else torch.from_numpy(wl.bias).to(dev).requires_grad_(True)
    w0 = None if wl.w0 is None else torch.from_numpy(wl.w0).to(dev).requires_grad_(True)
    b0 = None if wl.b0 is None else torch.from_numpy(wl.b0).to(dev).requires_grad_(True)
    x_leaf = x.detach().clone().requires_grad_(version == "B")
    ev = {}

    def step(record=False):
        def mark(name):
            if record:
                ev[name].record()
        mark("f0")
        xp, k = ops.forward(x, edges, inv_w, n_bins, W, dt[mode])
        mark("f1")
        xp_leaf = xp.detach().requires_grad_(True)
        z = xp_leaf + bias if version == "A" else xp_leaf
        y = torch.relu(z) if relu else z
        if version == "B":
            y = torch.addcmul(b0, w0, x_leaf[..., None]) + y
        for p in (bias, w0, b0, x_leaf):
            if p is not None:
                p.grad = None
        y.backward(g)
        mark("b0")
        ops.backward(xp_leaf.grad.contiguous(), x, edges, inv_w, n_bins, W, k, True, True)
        mark("b1")

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    times = {"step": [], "forward_op": [], "backward_op": []}
    for _ in range(args.steps):
        ev = {n: torch.cuda.Event(enable_timing=True) for n in ("f0", "f1", "b0", "b1")}
        step(record=True)
        torch.cuda.synchronize(dev)
        times["step"].append(ev["f0"].elapsed_time(ev["b1"]))
        times["forward_op"].append(ev["f0"].elapsed_time(ev["f1"]))
        times["backward_op"].append(ev["b0"].elapsed_time(ev["b1"]))
    med = {k: float(np.median(v)) for k, v in times.items()}
    print(json.dumps({
        "what": "reference CUDA ops built from its sources (oracle/_ref) + the module's PyTorch epilogue and autograd",
        "config": args.config, "batch": N, "ms_per_step": med["step"], "forward_op_ms": med["forward_op"],
        "backward_op_ms": med["backward_op"], "feature_embeddings_per_s": N * F / (med["step"] * 1e-3),
        "steps": args.steps, "warmup": args.warmup,
        "gpu": torch.cuda.get_device_name(dev),
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
