"""The tensor-core (tcgen05 one-hot GEMM) backward, selected with
``PLE_BACKWARD_KERNEL=tensor``: parity with the CPU oracle under the same
tolerances as the default sorted backward (fp32 and the low-precision modes,
both epilogues, ReLU, ragged / single-bin / tied / 64-bin edge tables, several
tiles and flush periods, the reference op with the forward's bin indices),
agreement with the sorted kernel where gradients or t are non-finite (those
contributions are summed outside the MMAs), bitwise determinism, a clean
status word, and PLE_ERR_UNSUPPORTED for shapes outside its geometry."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import ple_oracle as o  # noqa: E402
from tests import cases  # noqa: E402
from tests.test_parity_gpu import EPI, TORCH_DT, compare_fused, run_fused, to_dev  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    import rtdl_num_embeddings_cuda  # noqa: F401

    return torch.ops.rtdl_num_embeddings_cuda


@pytest.fixture
def tensor_kernel(monkeypatch):
    monkeypatch.setenv("PLE_BACKWARD_KERNEL", "tensor")


def _status():
    from piecewiselinearembeddings_optimized_b200 import _native

    return _native.capi().ple_tensor_core_status()


def _problem(case, n, d, version, seed):
    bins = cases.make_bins(case)
    x = cases.sample_x(bins, n, seed, integer=(case == "ties"))
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, seed)
    g = np.random.default_rng(seed + 1).standard_normal((n, len(bins), d)).astype(np.float32)
    return x, edges, inv_w, nb, w, bias, w0, b0, g


@pytest.mark.parametrize("case", cases.BIN_CASES)
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("d", [8, 16, 32])
def test_tensor_core_fp32_matches_oracle(ops, cuda_device, tensor_kernel, case, version, relu, d):
    # 1000 samples: several 64-row tiles, a partial last tile, flush points every 256 rows
    x, edges, inv_w, nb, w, bias, w0, b0, g = _problem(case, 1000, d, version, 40 + d)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, "f32",
                    reuse_bins=(d == 16))
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, relu, "f32")
    assert _status() == 0


@pytest.mark.parametrize("case", ["equal", "ragged", "ties", "wide"])
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("mode,out_mode,d", [("bf16", "f32", 16), ("bf16", "bf16", 16), ("bf16", "bf16", 24),
                                              ("f16", "f32", 16), ("f16", "f16", 16)])
def test_tensor_core_low_precision_matches_oracle(ops, cuda_device, tensor_kernel, case, version, mode, out_mode,
                                                  d):
    x, edges, inv_w, nb, w, bias, w0, b0, g = _problem(case, 512, d, version, 7)
    g = o.quantize(g, out_mode)
    res = run_fused(ops, cuda_device, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode)
    compare_fused(res, x, edges, inv_w, nb, w, bias, w0, b0, g, version, True, mode, out_mode)
    assert _status() == 0


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_tensor_core_reference_op_matches_oracle(ops, cuda_device, tensor_kernel, mode):
    """``ops.backward`` (the reference x_ple contract) with the forward's bin indices."""
    bins = cases.make_bins("wide")
    d = 16
    x = cases.sample_x(bins, 640, 5)
    edges, inv_w, nb = o.pad_bins(bins)
    w, *_ = cases.init_params(len(bins), edges.shape[1] - 1, d, "A", 2)
    g = o.quantize(np.random.default_rng(8).standard_normal((640, len(bins), d)).astype(np.float32), mode)
    tx, te, tr, tn, tw, tg = to_dev(cuda_device, x, edges, inv_w, nb, w, g)
    _, idx = ops.forward(tx, te, tr, tn, tw, TORCH_DT[mode])
    gx, gw = ops.backward(tg.to(TORCH_DT[mode]), tx, te, tr, tn, tw, idx, True, True)
    rgx, rgw, rabs = o.x_ple_backward(g, x, edges, inv_w, nb, w, mode, with_abs=True)
    tol = dict(rtol=1e-4, atol=1e-5) if mode == "f32" else dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(gx.cpu().numpy(), rgx, **tol)
    o.assert_reduction_close(gw.cpu().numpy(), rgw, rabs, err_msg="grad_W", **tol)


def _backward(ops, dev, x, edges, inv_w, nb, w, w0, b0, g):
    tx, te, tr, tn, tw, tw0, tb0, tg = to_dev(dev, x, edges, inv_w, nb, w, w0, b0, g)
    out = ops.embeddings_backward(tg, tx, te, tr, tn, tw, None, tw0, tb0, None, EPI["B"], True, torch.float32,
                                  True, True, False, True)
    return [t.cpu().numpy() for t in (out[0], out[1], out[3], out[4])]


def test_tensor_core_non_finite_matches_sorted(ops, cuda_device, monkeypatch):
    """NaN / +-Inf gradients and x = +-inf (infinite t): the same non-finite pattern as the sorted kernel,
    finite values within the fp32 reduction tolerance."""
    bins = cases.make_bins("wide")
    d = 16
    x = cases.sample_x(bins, 512, 3, specials=True)
    edges, inv_w, nb = o.pad_bins(bins)
    w, _, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, "B", 4)
    g = np.random.default_rng(6).standard_normal((512, len(bins), d)).astype(np.float32)
    g[17, 1, 3] = np.nan
    g[200, 3, 0] = np.inf
    g[201, 3, 0] = -np.inf
    g[300, 4, 9] = np.inf
    monkeypatch.setenv("PLE_BACKWARD_KERNEL", "sorted")
    ref = _backward(ops, cuda_device, x, edges, inv_w, nb, w, w0, b0, g)
    monkeypatch.setenv("PLE_BACKWARD_KERNEL", "tensor")
    got = _backward(ops, cuda_device, x, edges, inv_w, nb, w, w0, b0, g)
    assert _status() == 0
    for name, a, b in zip(("grad_x", "grad_W", "grad_w0", "grad_b0"), got, ref):
        np.testing.assert_array_equal(np.isnan(a), np.isnan(b), err_msg=f"{name}: NaN pattern")
        np.testing.assert_array_equal(np.isposinf(a), np.isposinf(b), err_msg=f"{name}: +inf pattern")
        np.testing.assert_array_equal(np.isneginf(a), np.isneginf(b), err_msg=f"{name}: -inf pattern")
        fin = np.isfinite(b)
        np.testing.assert_allclose(a[fin], b[fin], rtol=1e-4, atol=1e-4, err_msg=name)


def test_tensor_core_is_deterministic_and_sizes_match_config(ops, cuda_device, tensor_kernel):
    """c5-shaped slice (512 features, 64 bins, D = 16): two runs are bitwise equal and match the oracle."""
    from piecewiselinearembeddings_optimized_b200 import workloads

    wl = workloads.make_workload("c5", n=2048, f=64)
    g = workloads.make_grad(wl)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    a = _backward(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.w0, wl.b0, g)
    b = _backward(ops, cuda_device, wl.x, edges, inv_w, nb, wl.weight, wl.w0, wl.b0, g)
    for u, v in zip(a, b):
        assert np.array_equal(u, v, equal_nan=True)
    ref = o.embeddings_backward(g, wl.x, edges, inv_w, nb, wl.weight, version="B", activation=True, w0=wl.w0,
                                b0=wl.b0, mode="f32")
    np.testing.assert_allclose(a[0], ref["grad_x"], rtol=1e-4, atol=1e-5)
    o.assert_reduction_close(a[1], ref["grad_W"], ref["abs"]["grad_W"], err_msg="grad_W")
    o.assert_reduction_close(a[2], ref["grad_w0"], ref["abs"]["grad_w0"], err_msg="grad_w0")
    o.assert_reduction_close(a[3], ref["grad_b0"], ref["abs"]["grad_b0"], err_msg="grad_b0")
    assert _status() == 0


def test_tensor_core_rejects_unsupported_shape(ops, cuda_device, tensor_kernel):
    bins = cases.make_bins("equal")
    x, edges, inv_w, nb, w, _, w0, b0, g = _problem("equal", 64, 10, "B", 1)  # D = 10: not a multiple of 8
    with pytest.raises(RuntimeError, match="tensor-core backward: shape not supported"):
        _backward(ops, cuda_device, x, edges, inv_w, nb, w, w0, b0, g)
    assert len(bins) == 3
