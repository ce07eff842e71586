"""Generate golden vectors by running the REFERENCE's own CUDA ops.

Run on a GPU host, in a process that has NOT loaded this project's native
library (both register the ``rtdl_num_embeddings_cuda`` op namespace):

    python tests/golden/make_golden.py --out tests/golden

The reference ops come from ``oracle/_ref/rtdl_ref_ops.so``, compiled from the
reference sources by ``oracle/build_ref.py``.  For every case this script

1. calls ``rtdl_num_embeddings_cuda::forward`` (reference ``ops.cpp:35-44``)
   for ``x_ple`` and ``bin_indices``;
2. applies the reference module's epilogue exactly as ``module.py:230-248``
   composes it (``+ linear.bias`` for version A, ReLU, ``linear0(x) + ...``
   for version B with ``linear0(x) = addcmul(b0, w0, x[..., None])``), with
   torch autograd to obtain the epilogue gradients and ``dL/dx_ple``;
3. calls ``rtdl_num_embeddings_cuda::backward`` (reference ``ops.cpp:46-58``)
   with ``dL/dx_ple`` for ``grad_x`` (x_ple part) and ``grad_weight``.

Outputs are written as one ``.npz`` per case with the inputs (or, for the
seeded large cases, the recipe and a digest of the inputs) and the results.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.ple_oracle import pad_bins, quantize  # noqa: E402
from tests import cases  # noqa: E402
from piecewiselinearembeddings_optimized_b200 import workloads  # noqa: E402

REF_LIB = ROOT / "oracle" / "_ref" / "rtdl_ref_ops.so"

# name, bin case, n, d, version, relu, mode, sampler options, with backward
SMALL_CASES = [
    ("equal_A_f32_d10", "equal", 64, 10, "A", False, "f32", {}, True),
    ("equal_B_relu_f32_d15", "equal", 64, 15, "B", True, "f32", {}, True),
    ("ragged_A_relu_f32_d20", "ragged", 64, 20, "A", True, "f32", {}, True),
    ("ragged_B_f32_d16", "ragged", 64, 16, "B", False, "f32", {}, True),
    ("single_B_relu_f32_d12", "single_bin", 64, 12, "B", True, "f32", {}, True),
    ("allsingle_A_f32_d8", "all_single_bin", 64, 8, "A", False, "f32", {}, True),
    ("ties_B_relu_f32_d16", "ties", 64, 16, "B", True, "f32", {"integer": True}, True),
    ("specials_A_f32_d4", "ragged", 64, 4, "A", False, "f32", {"specials": True}, False),
    ("equal_A_relu_bf16_d16", "equal", 64, 16, "A", True, "bf16", {}, True),
    ("ragged_B_relu_bf16_d24", "ragged", 64, 24, "B", True, "bf16", {}, True),
    ("single_A_f16_d8", "single_bin", 64, 8, "A", False, "f16", {}, True),
    ("wide_B_relu_bf16_d24", "wide", 128, 24, "B", True, "bf16", {}, True),
    ("ties_A_relu_bf16_d8", "ties", 64, 8, "A", True, "bf16", {"integer": True}, True),
]

# seeded larger cases (inputs regenerated from the recipe; only a digest is stored)
LARGE_CASES = [
    # name, workload, n override, f override, sampled rows
    ("c1_full", "c1", None, None, 128),
    ("c2_sorted_path", "c2", None, None, 64),
    ("c3_slice", "c3", 2048, 16, 64),
]

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def run_reference(ops, bins, x, w, bias, w0, b0, g, version, relu, mode, backward=True):
    dev = torch.device("cuda")
    edges, inv_w, n_bins = pad_bins(bins)
    te = torch.from_numpy(edges).to(dev)
    tr = torch.from_numpy(inv_w).to(dev)
    tn = torch.from_numpy(n_bins).to(dev)
    tx = torch.from_numpy(x).to(dev)
    tw = torch.from_numpy(w).to(dev)
    xp, k = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    xp_leaf = xp.detach().requires_grad_(True)
    x_leaf = tx.detach().clone().requires_grad_(True)
    leaves = {}
    z = xp_leaf
    if version == "A":
        leaves["bias"] = torch.from_numpy(bias).to(dev).requires_grad_(True)
        z = z + leaves["bias"]
    y = torch.relu(z) if relu else z
    if version == "B":
        leaves["w0"] = torch.from_numpy(w0).to(dev).requires_grad_(True)
        leaves["b0"] = torch.from_numpy(b0).to(dev).requires_grad_(True)
        y = torch.addcmul(leaves["b0"], leaves["w0"], x_leaf[..., None]) + y
    out = {
        "x_ple": xp.float().cpu().numpy(),
        "bin_indices": k.cpu().numpy(),
        "y": y.detach().float().cpu().numpy(),
    }
    if not backward:
        return out
    tg = torch.from_numpy(g).to(dev)
    y.backward(tg)
    g_ple = xp_leaf.grad
    gx_ple, gw = ops.backward(g_ple.contiguous(), tx, te, tr, tn, tw, k, True, True)
    gx = gx_ple + (x_leaf.grad if x_leaf.grad is not None else 0)
    out.update({
        "g_ple": g_ple.float().cpu().numpy(),
        "grad_x_ple": gx_ple.cpu().numpy(),
        "grad_x": gx.cpu().numpy(),
        "grad_W": gw.cpu().numpy(),
    })
    for name, leaf in leaves.items():
        out["grad_" + name] = leaf.grad.cpu().numpy()
    torch.cuda.synchronize()
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", type=Path, default=ROOT / "tests" / "golden")
    args = ap.parse_args(argv)
    torch.ops.load_library(str(REF_LIB))
    ops = torch.ops.rtdl_num_embeddings_cuda
    args.out.mkdir(parents=True, exist_ok=True)

    for name, bcase, n, d, version, relu, mode, opts, with_bwd in SMALL_CASES:
        bins = cases.make_bins(bcase)
        x = cases.sample_x(bins, n, seed=1000 + n + d, **opts)
        b = max(len(e) - 1 for e in bins)
        w, bias, w0, b0 = cases.init_params(len(bins), b, d, version, seed=d)
        g = np.random.default_rng(3000 + d).standard_normal((n, len(bins), d)).astype(np.float32)
        g = quantize(g, mode)
        res = run_reference(ops, bins, x, w, bias, w0, b0, g, version, relu, mode, with_bwd)
        edges, inv_w, n_bins = pad_bins(bins)
        payload = dict(edges=edges, inv_w=inv_w, n_bins=n_bins, x=x, weight=w, g=g,
                       version=version, activation=relu, mode=mode, backward=with_bwd)
        for key, val in (("bias", bias), ("w0", w0), ("b0", b0)):
            if val is not None:
                payload[key] = val
        payload.update({"ref_" + k: v for k, v in res.items()})
        np.savez_compressed(args.out / f"{name}.npz", **payload)
        print("wrote", name)

    for name, cfg, n, f, n_rows in LARGE_CASES:
        wl = workloads.make_workload(cfg, n=n, f=f)
        g = workloads.make_grad(wl)
        res = run_reference(ops, wl.bins, wl.x, wl.weight, wl.bias, wl.w0, wl.b0, g,
                            wl.version, wl.activation, wl.mode, True)
        rows = np.random.default_rng(5).choice(wl.n, size=n_rows, replace=False)
        rows.sort()
        payload = dict(workload=cfg, n=wl.n, f=wl.f, rows=rows,
                       input_digest=digest(wl.x, wl.weight, wl.bias, wl.w0, wl.b0, g),
                       ref_x_ple_rows=res["x_ple"][rows], ref_y_rows=res["y"][rows],
                       ref_bin_indices=res["bin_indices"], ref_grad_x=res["grad_x"],
                       ref_grad_x_ple=res["grad_x_ple"], ref_grad_W=res["grad_W"])
        for key in ("grad_bias", "grad_w0", "grad_b0"):
            if key in res:
                payload["ref_" + key] = res[key]
        np.savez_compressed(args.out / f"{name}.npz", **payload)
        print("wrote", name)
    return 0


if __name__ == "__main__":
    sys.exit(main())
