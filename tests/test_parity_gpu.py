"""GPU parity of the sm_100a kernels against the CPU oracle.

Tolerances (from the task's acceptance bar): bin indices bit-exact; fp32
outputs rtol 1e-5 / atol 1e-6; gradients rtol 1e-4 / atol 1e-5; bf16 / fp16
mode rtol 1e-2 (atol 1e-2; gradients 2e-2).  Every call goes through the
``rtdl_num_embeddings_cuda`` torch ops, which call the C ABI.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import ple_oracle as o  # noqa: E402
from piecewiselinearembeddings_optimized_b200 import workloads  # noqa: E402
from tests import cases  # noqa: E402

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-6)
GRAD_TOL = dict(rtol=1e-4, atol=1e-5)
LOW_TOL = dict(rtol=1e-2, atol=1e-2)
LOW_GRAD_TOL = dict(rtol=2e-2, atol=2e-2)
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
EPI = {"A": 1, "B": 2}
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def ops(cuda_device):
    import rtdl_num_embeddings_cuda  # noqa: F401  (registers the ops)

    return torch.ops.rtdl_num_embeddings_cuda


def to_dev(dev, *arrays):
    return [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays]


def run_fused(ops, dev, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, mode, out_mode=None,
              reuse_bins=False):
    out_mode = out_mode or "f32"
    tx, te, tr, tn, tw, tb, tw0, tb0 = to_dev(dev, x, edges, inv_w, nb, w, bias, w0, b0)
    y = ops.embeddings_forward(tx, te, tr, tn, tw, tb, tw0, tb0, EPI[version], relu, TORCH_DT[mode],
                               TORCH_DT[out_mode])
    res = {"y": y.float().cpu().numpy()}
    if g is not None:
        # the bin indices of the x_ple op (reference contract) are also accepted by the fused backward
        idx = ops.forward(tx, te, tr, tn, tw, torch.float32)[1] if reuse_bins else None
        tg = torch.from_numpy(g).to(dev).to(TORCH_DT[out_mode])
        gx, gw, gb, gw0, gb0 = ops.embeddings_backward(tg, tx, te, tr, tn, tw, tb, tw0, tb0,
                                                       idx, EPI[version], relu,
                                                       TORCH_DT[mode], True, True, True, True)
        res.update(grad_x=gx.cpu().numpy(), grad_W=gw.cpu().numpy())
        if version == "A":
            res["grad_bias"] = gb.cpu().numpy()
        else:
            res["grad_w0"], res["grad_b0"] = gw0.cpu().numpy(), gb0.cpu().numpy()
    return res


def compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, mode, out_mode="f32"):
    y_ref, _, _ = o.embeddings_forward(x, edges, inv_w, nb, w, version=version, activation=relu, bias=bias,
                                       w0=w0, b0=b0, mode=mode, out_mode=out_mode)
    low = mode != "f32" or out_mode != "f32"
    np.testing.assert_allclose(res["y"], y_ref, **(LOW_TOL if low else FWD_TOL))
    if g is None:
        return
    ref = o.embeddings_backward(g, x, edges, inv_w, nb, w, version=version, activation=relu, bias=bias, w0=w0,
                                b0=b0, mode=mode)
    check_grads(res, ref, ref["abs"], low)


def check_grads(res, ref, abs_sums, low):
    """grad_x element-wise; batch reductions with the fp32 summation allowance."""
    tol = LOW_GRAD_TOL if low else GRAD_TOL
    np.testing.assert_allclose(res["grad_x"], ref["grad_x"], err_msg="grad_x", **tol)
    for key in ("grad_W", "grad_bias", "grad_w0", "grad_b0"):
        if key in ref and key in res:
            o.assert_reduction_close(res[key], ref[key], abs_sums[key], err_msg=key, **tol)


# ---------------------------------------------------------------- structural cases

@pytest.mark.parametrize("case", cases.BIN_CASES)
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("d", [8, 10, 15, 16, 20, 24])
def test_fused_fp32_matches_oracle(ops, cuda_device, case, version, relu, d):
    bins = cases.make_bins(case)
    x = cases.sample_x(bins, 128, 1000 + d, integer=(case == "ties"))
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, d)
    g = np.random.default_rng(3000 + d).standard_normal((128, len(bins), d)).astype(np.float32)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, "f32",
                    reuse_bins=(d % 2 == 0))
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, "f32")


@pytest.mark.parametrize("case", ["equal", "ragged", "single_bin", "ties", "wide"])
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("mode,out_mode", [("bf16", "f32"), ("bf16", "bf16"), ("f16", "f32"), ("f16", "f16")])
def test_fused_low_precision_matches_oracle(ops, cuda_device, case, version, mode, out_mode):
    bins = cases.make_bins(case)
    d = 16
    x = cases.sample_x(bins, 128, 7, integer=(case == "ties"))
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, 9)
    g = np.random.default_rng(5).standard_normal((128, len(bins), d)).astype(np.float32)
    g = o.quantize(g, out_mode)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode)
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode)


# odd d_embedding above 32: the C ABI's backward refuses it and the torch ops pad one zero column
@pytest.mark.parametrize("case", ["equal", "ragged", "single_bin"])
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("d,mode,out_mode", [(33, "f32", "f32"), (63, "f32", "f32"), (45, "bf16", "bf16")])
def test_fused_odd_wide_d_matches_oracle(ops, cuda_device, case, version, d, mode, out_mode):
    bins = cases.make_bins(case)
    x = cases.sample_x(bins, 96, 4000 + d)
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, d)
    g = o.quantize(np.random.default_rng(5000 + d).standard_normal((96, len(bins), d)).astype(np.float32), out_mode)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode,
                    reuse_bins=(version == "A"))
    assert res["grad_W"].shape == w.shape
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode)


@pytest.mark.parametrize("d", [33, 63])
def test_reference_backward_odd_wide_d(ops, cuda_device, d):
    bins = cases.make_bins("ragged")
    x = cases.sample_x(bins, 80, 60 + d)
    edges, inv_w, nb = o.pad_bins(bins)
    w, *_ = cases.init_params(len(bins), edges.shape[1] - 1, d, "A", 5)
    g = np.random.default_rng(70 + d).standard_normal((80, len(bins), d)).astype(np.float32)
    tx, te, tr, tn, tw, tg = to_dev(cuda_device, x, edges, inv_w, nb, w, g)
    _, idx = ops.forward(tx, te, tr, tn, tw, torch.float32)
    gx, gw = ops.backward(tg, tx, te, tr, tn, tw, idx, True, True)
    assert gw.shape == (len(bins), edges.shape[1] - 1, d) and gw.is_contiguous()
    rgx, rgw, rabs = o.x_ple_backward(g, x, edges, inv_w, nb, w, "f32", with_abs=True)
    np.testing.assert_allclose(gx.cpu().numpy(), rgx, **GRAD_TOL)
    o.assert_reduction_close(gw.cpu().numpy(), rgw, rabs, err_msg="grad_W", **GRAD_TOL)
    gx2, gw2 = ops.backward(tg, tx, te, tr, tn, tw, idx, False, True)
    assert gx2.numel() == 0 and torch.equal(gw2, gw)


# more than 256 bins: int16 / int32 bin indices, the global-memory kernels of the bare x_ple op, and the
# module's epilogue composed around it

def _wide_bins(n_bins, seed):
    rng = np.random.default_rng(seed)
    return [(np.cumsum(rng.random(n + 1) + 0.01) - 0.3 * n).astype(np.float32) for n in n_bins]


def _wide_x(bins, n, seed):
    x = cases.sample_x(bins, n, seed)
    x[:8, 0] = bins[0][10:18]  # exact interior edges: the boundary sub-gradient
    return x


@pytest.mark.parametrize("n_bins,idx_dtype", [((300, 5, 1, 120), torch.int16), ((40000, 3), torch.int32)])
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_reference_ops_wide_bins(ops, cuda_device, n_bins, idx_dtype, mode):
    bins = _wide_bins(n_bins, 31)
    d = 6
    x = _wide_x(bins, 64, 32)
    edges, inv_w, nb = o.pad_bins(bins)
    w, *_ = cases.init_params(len(bins), edges.shape[1] - 1, d, "A", 33)
    tx, te, tr, tn, tw = to_dev(cuda_device, x, edges, inv_w, nb, w)
    xp, idx = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    assert idx.dtype == idx_dtype
    ref_xp, ref_k = o.x_ple_forward(x, edges, inv_w, nb, w, mode)
    np.testing.assert_array_equal(idx.cpu().numpy().astype(np.int64), ref_k)
    np.testing.assert_allclose(xp.float().cpu().numpy(), ref_xp, **(FWD_TOL if mode == "f32" else LOW_TOL))
    g = o.quantize(np.random.default_rng(34).standard_normal((64, len(bins), d)).astype(np.float32), mode)
    tg = torch.from_numpy(g).to(cuda_device).to(TORCH_DT[mode])
    gx, gw = ops.backward(tg, tx, te, tr, tn, tw, idx, True, True)
    rgx, rgw, rabs = o.x_ple_backward(g, x, edges, inv_w, nb, w, mode, with_abs=True)
    tol = GRAD_TOL if mode == "f32" else LOW_GRAD_TOL
    np.testing.assert_allclose(gx.cpu().numpy(), rgx, **tol)
    o.assert_reduction_close(gw.cpu().numpy(), rgw, rabs, err_msg="grad_W", **tol)
    gx2, gw2 = ops.backward(tg, tx, te, tr, tn, tw, idx, True, False)
    assert gw2.numel() == 0 and torch.equal(gx2, gx)


@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("mode,out_mode", [("f32", "f32"), ("bf16", "f32"), ("bf16", "bf16")])
def test_fused_wide_bins_match_oracle(ops, cuda_device, version, relu, mode, out_mode):
    bins = _wide_bins((260, 7, 2, 512), 41)
    d = 10
    x = _wide_x(bins, 96, 42)
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, 43)
    g = o.quantize(np.random.default_rng(44).standard_normal((96, len(bins), d)).astype(np.float32), out_mode)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, mode, out_mode,
                    reuse_bins=relu)
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, mode, out_mode)


# ---------------------------------------------------------------- reference-interface ops

@pytest.mark.parametrize("case", cases.BIN_CASES)
@pytest.mark.parametrize("mode", ["f32", "bf16", "f16"])
def test_reference_ops_match_oracle(ops, cuda_device, case, mode):
    bins = cases.make_bins(case)
    d = 12
    x = cases.sample_x(bins, 64, 21, specials=True)
    edges, inv_w, nb = o.pad_bins(bins)
    w, *_ = cases.init_params(len(bins), edges.shape[1] - 1, d, "A", 2)
    tx, te, tr, tn, tw = to_dev(cuda_device, x, edges, inv_w, nb, w)
    xp, idx = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    assert xp.dtype == TORCH_DT[mode] and idx.dtype == torch.uint8
    ref_xp, ref_k = o.x_ple_forward(x, edges, inv_w, nb, w, mode)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_k)
    got = xp.float().cpu().numpy()
    fin = np.isfinite(ref_xp)
    np.testing.assert_array_equal(np.isfinite(got), fin)
    np.testing.assert_allclose(got[fin], ref_xp[fin], **(FWD_TOL if mode == "f32" else LOW_TOL))
    # backward on finite rows only (the +-inf samples make t infinite)
    keep = np.isfinite(x).all(axis=1)
    xk = np.ascontiguousarray(x[keep])
    g = o.quantize(np.random.default_rng(8).standard_normal((xk.shape[0], len(bins), d)).astype(np.float32), mode)
    tx, tg = to_dev(cuda_device, xk, g)
    tg = tg.to(TORCH_DT[mode])
    _, idx = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    gx, gw = ops.backward(tg, tx, te, tr, tn, tw, idx, True, True)
    rgx, rgw, rabs = o.x_ple_backward(g, xk, edges, inv_w, nb, w, mode, with_abs=True)
    tol = GRAD_TOL if mode == "f32" else LOW_GRAD_TOL
    np.testing.assert_allclose(gx.cpu().numpy(), rgx, **tol)
    o.assert_reduction_close(gw.cpu().numpy(), rgw, rabs, err_msg="grad_W", **tol)
    gx2, gw2 = ops.backward(tg, tx, te, tr, tn, tw, idx, False, True)
    assert gx2.numel() == 0 and torch.equal(gw2, gw)
    gx3, gw3 = ops.backward(tg, tx, te, tr, tn, tw, idx, True, False)
    assert gw3.numel() == 0 and torch.equal(gx3, gx)


def test_empty_batch(ops, cuda_device):
    bins = cases.make_bins("equal")
    edges, inv_w, nb = o.pad_bins(bins)
    w, *_ = cases.init_params(3, 4, 8, "A", 0)
    te, tr, tn, tw = to_dev(cuda_device, edges, inv_w, nb, w)
    x = torch.empty(0, 3, device=cuda_device)
    y, idx = ops.forward(x, te, tr, tn, tw, torch.float32)
    assert y.shape == (0, 3, 8) and idx.shape == (0, 3)
    gx, gw = ops.backward(torch.empty(0, 3, 8, device=cuda_device), x, te, tr, tn, tw, idx, True, True)
    assert gx.shape == (0, 3) and torch.count_nonzero(gw) == 0


# ---------------------------------------------------------------- golden fixtures of the reference

def _golden():
    return sorted(GOLDEN.glob("*.npz"))


@pytest.mark.skipif(not _golden(), reason="golden fixtures not generated")
@pytest.mark.parametrize("path", _golden(), ids=lambda p: p.stem)
def test_kernels_match_reference_golden(ops, cuda_device, path):
    z = np.load(path)
    if "workload" in z.files:
        n, f, name = int(z["n"]), int(z["f"]), str(z["workload"])
        spec = workloads.SPECS[name]
        wl = workloads.make_workload(name, n=None if n == spec[0] else n, f=None if f == spec[1] else f)
        g = workloads.make_grad(wl)
        edges, inv_w, nb = o.pad_bins(wl.bins)
        res = run_fused(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0, g,
                        wl.version, wl.activation, wl.mode)
        rows = z["rows"]
        np.testing.assert_allclose(res["y"][rows], z["ref_y_rows"], **FWD_TOL)
        ora = o.embeddings_backward(g, wl.x, edges, inv_w, nb, wl.weight, version=wl.version,
                                    activation=wl.activation, bias=wl.bias, w0=wl.w0, b0=wl.b0, mode=wl.mode)
        ref = {k: z["ref_" + k] for k in ("grad_x", "grad_W", "grad_bias", "grad_w0", "grad_b0")
               if "ref_" + k in z.files}
        check_grads(res, ref, {k: 2 * v for k, v in ora["abs"].items()}, False)
        return
    mode, version, relu = str(z["mode"]), str(z["version"]), bool(z["activation"])
    bias = z["bias"] if "bias" in z.files else None
    w0 = z["w0"] if "w0" in z.files else None
    b0 = z["b0"] if "b0" in z.files else None
    tx, te, tr, tn, tw = to_dev(cuda_device, z["x"], z["edges"], z["inv_w"], z["n_bins"], z["weight"])
    xp, idx = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    np.testing.assert_array_equal(idx.cpu().numpy(), z["ref_bin_indices"])
    low = mode != "f32"
    got, ref = xp.float().cpu().numpy(), z["ref_x_ple"]
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(np.isfinite(got), fin)
    np.testing.assert_allclose(got[fin], ref[fin], **(LOW_TOL if low else FWD_TOL))
    g = z["g"] if bool(z["backward"]) else None
    if g is None:
        res = run_fused(ops, cuda_device, z["x"], z["edges"], z["inv_w"], z["n_bins"], z["weight"], bias, w0, b0,
                        None, version, relu, mode)
        fin = np.isfinite(z["ref_y"])
        np.testing.assert_allclose(res["y"][fin], z["ref_y"][fin], **(LOW_TOL if low else FWD_TOL))
        return
    res = run_fused(ops, cuda_device, z["x"], z["edges"], z["inv_w"], z["n_bins"], z["weight"], bias, w0, b0, g,
                    version, relu, mode)
    np.testing.assert_allclose(res["y"], z["ref_y"], **(LOW_TOL if low else FWD_TOL))
    tol = LOW_GRAD_TOL if low else GRAD_TOL
    ora = o.embeddings_backward(g, z["x"], z["edges"], z["inv_w"], z["n_bins"], z["weight"], version=version,
                                activation=relu, bias=bias, w0=w0, b0=b0, mode=mode)
    allow = {k: 2 * v for k, v in ora["abs"].items()}
    ref = {k: z["ref_" + k] for k in ("grad_x", "grad_W", "grad_bias", "grad_w0", "grad_b0") if "ref_" + k in z.files}
    check_grads(res, ref, allow, low)
    tg = torch.from_numpy(z["ref_g_ple"]).to(cuda_device).to(TORCH_DT[mode])
    gx, gw = ops.backward(tg, tx, te, tr, tn, tw, idx, True, True)
    np.testing.assert_allclose(gx.cpu().numpy(), z["ref_grad_x_ple"], **tol)
    o.assert_reduction_close(gw.cpu().numpy(), z["ref_grad_W"], allow["grad_W"], err_msg="grad_W (x_ple op)", **tol)


# ---------------------------------------------------------------- benchmark configurations

@pytest.mark.parametrize("name,n,f", [("c1", None, None), ("c2", None, None), ("c3", None, None),
                                      ("c4", 4096, None), ("c5", 2048, None), ("c5", 512, 48), ("c4", 512, 40)])
def test_configs_match_oracle(ops, cuda_device, name, n, f):
    """c1, c2 and c3 at their full batch (c3: 16,384 rows, ragged and deduplicated bins, D = 64 on the sorted
    kernel), c4 and c5 on a slice (their full batches are checked by test_full_size_properties).  48 features
    of c5 (3 forward chunks of 16 in slots of 2 CTAs) and 40 of c4 (5 chunks of 8 in slots of 4) leave the
    last forward slot partly idle."""
    wl = workloads.make_workload(name, n=n, f=f)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    res = run_fused(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0, g, wl.version,
                    wl.activation, wl.mode, wl.out_mode)
    compare_fused(res, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0, g, wl.version, wl.activation,
                  wl.mode, wl.out_mode)


def test_backward_is_bitwise_deterministic(ops, cuda_device):
    wl = workloads.make_workload("c4", n=8192, f=64)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    a = run_fused(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0, g, wl.version,
                  wl.activation, wl.mode, wl.out_mode)
    b = run_fused(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0, g, wl.version,
                  wl.activation, wl.mode, wl.out_mode)
    for k in a:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)


@pytest.mark.parametrize("name", ["c4", "c5"])
def test_full_size_properties(ops, cuda_device, name):
    """Full benchmark batch (c5: one rank's shard of 8): forward rows and
    grad_x rows against the oracle on a row sample; grad_W equals the sum of
    the grad_W of four batch shards (the data-parallel identity)."""
    n = None if name == "c4" else workloads.SPECS["c5"][0] // 8
    wl = workloads.make_workload(name, n=n)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    dev = cuda_device
    tx, te, tr, tn, tw, tb, tw0, tb0 = to_dev(dev, wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0)
    od = TORCH_DT[wl.out_mode]
    y = ops.embeddings_forward(tx, te, tr, tn, tw, tb, tw0, tb0, EPI[wl.version], wl.activation,
                               TORCH_DT[wl.mode], od)
    idx = ops.forward(tx, te, tr, tn, tw, torch.float32)[1]
    rows = np.random.default_rng(0).choice(wl.n, 256, replace=False)
    rows.sort()
    y_ref, _, _ = o.embeddings_forward(wl.x[rows], edges, inv_w, nb, wl.weight, version=wl.version,
                                       activation=wl.activation, bias=wl.bias, w0=wl.w0, b0=wl.b0, mode=wl.mode,
                                       out_mode=wl.out_mode)
    low = wl.mode != "f32"
    np.testing.assert_allclose(y[torch.from_numpy(rows).to(dev)].float().cpu().numpy(), y_ref,
                               **(LOW_TOL if low else FWD_TOL))
    del y
    tg = torch.from_numpy(g).to(dev).to(od)
    full = ops.embeddings_backward(tg, tx, te, tr, tn, tw, tb, tw0, tb0, idx, EPI[wl.version], wl.activation,
                                   TORCH_DT[wl.mode], True, True, True, True)
    ref_rows = o.embeddings_backward(g[rows], wl.x[rows], edges, inv_w, nb, wl.weight, version=wl.version,
                                     activation=wl.activation, bias=wl.bias, w0=wl.w0, b0=wl.b0, mode=wl.mode)
    np.testing.assert_allclose(full[0][torch.from_numpy(rows).to(dev)].cpu().numpy(), ref_rows["grad_x"],
                               **(LOW_GRAD_TOL if low else GRAD_TOL))
    shards = torch.tensor_split(torch.arange(wl.n, device=dev), 4)
    acc = [torch.zeros_like(t) for t in full[1:]]
    for sel in shards:
        part = ops.embeddings_backward(tg[sel].contiguous(), tx[sel].contiguous(), te, tr, tn, tw, tb, tw0, tb0,
                                       None, EPI[wl.version], wl.activation, TORCH_DT[wl.mode], False, True, True,
                                       True)
        for a_, p_ in zip(acc, part[1:]):
            if p_.numel():
                a_ += p_
    # allowance: sum over the batch of |g| * max(1, |t|) bounds sum|terms| of every grad_W element
    k = o.bin_index(wl.x, edges, nb)
    t = torch.from_numpy(np.abs(o.position(wl.x, k, edges, inv_w))).to(dev).clamp_min(1.0)
    ag = tg.float().abs()
    bound_w = (ag * t[..., None]).sum(0)[:, None, :].expand_as(full[1])
    bounds = [bound_w, ag.sum(0), (ag * tx.abs()[..., None]).sum(0), ag.sum(0)]
    for a_, f_, b_ in zip(acc, full[1:], bounds):
        if f_.numel():
            o.assert_reduction_close(a_.cpu().numpy(), f_.cpu().numpy(), 2 * b_.cpu().numpy(), err_msg="shards")


# ---------------------------------------------------------------- the two fused backward kernels

def test_backward_kernel_kind(cuda_device):
    """D = 8 / 16 / 24 run the histogram kernel where its private sums fit in shared memory (unless
    PLE_BACKWARD_KERNEL=sorted); other widths, and D = 24 with 64 bins (16 warps x 64 x 24 x 2 floats of sums
    alone take 192 KB), the sorted one."""
    from piecewiselinearembeddings_optimized_b200 import _native

    lib = _native.capi()
    sorted_only = os.environ.get("PLE_BACKWARD_KERNEL") == "sorted"
    for f, b, d in ((512, 64, 8), (512, 64, 16), (256, 32, 24)):
        assert lib.ple_backward_kernel_kind(f, b, d) == (0 if sorted_only else 1), d
    assert lib.ple_backward_kernel_kind(512, 64, 24) == 0
    for d in (4, 10, 32, 64):
        assert lib.ple_backward_kernel_kind(512, 64, d) == 0, d
    assert lib.ple_backward_kernel_kind(8, 300, 16) == 2


def test_sorted_backward_kernel_matches_oracle(cuda_device):
    """The sorted kernel on the shapes the histogram kernel takes by default (so that both stay checked):
    the configuration, low-precision and determinism cases again in a child process with
    PLE_BACKWARD_KERNEL=sorted."""
    if os.environ.get("PLE_BACKWARD_KERNEL") == "sorted":
        pytest.skip("already the sorted kernel")
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, PLE_BACKWARD_KERNEL="sorted")
    sel = ("test_configs_match_oracle or test_fused_low_precision_matches_oracle or "
           "test_backward_is_bitwise_deterministic or test_backward_kernel_kind")
    r = subprocess.run([sys.executable, "-m", "pytest", str(Path(__file__)), "-q", "-x", "-m", "gpu",
                        "-p", "no:cacheprovider", "-k", sel], cwd=root, env=env, capture_output=True, text=True,
                       timeout=1800)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]

