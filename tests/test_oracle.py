"""CPU checks of the oracle itself (no GPU): its two formulations agree, the
bin search follows the reference's rules, and - when the golden fixtures are
present - it reproduces the reference's own CUDA outputs."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import ple_oracle as o
from tests import cases

GOLDEN = Path(__file__).resolve().parent / "golden"


def _setup(case, n=64, d=12, version="A", seed=3, **opts):
    bins = cases.make_bins(case)
    x = cases.sample_x(bins, n, seed, **opts)
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, seed)
    return x, edges, inv_w, nb, w, bias, w0, b0


@pytest.mark.parametrize("case", cases.BIN_CASES)
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("relu", [False, True])
def test_pairwise_matches_dense(case, version, relu):
    x, edges, inv_w, nb, w, bias, w0, b0 = _setup(case, version=version)
    y, _, _ = o.embeddings_forward(x, edges, inv_w, nb, w, version=version, activation=relu,
                                   bias=bias, w0=w0, b0=b0)
    yd = o.dense_forward(x, edges, inv_w, nb, w, version=version, activation=relu, bias=bias, w0=w0, b0=b0)
    np.testing.assert_allclose(y, yd, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_zero_column_padding_leaves_gradients_unchanged(version, mode):
    """The torch ops serve an odd d_embedding above 32 by appending one zero
    column to g', W, bias, w0 and b0 and dropping its gradients; every other
    gradient must come out the same."""
    d = 33
    x, edges, inv_w, nb, w, bias, w0, b0 = _setup("ragged", n=48, d=d, version=version, seed=11)
    g = np.random.default_rng(12).standard_normal((48, x.shape[1], d)).astype(np.float32)
    pad = lambda a: None if a is None else np.concatenate(  # noqa: E731
        [a, np.zeros(a.shape[:-1] + (1,), np.float32)], axis=-1)
    kw = dict(version=version, activation=True, mode=mode)
    ref = o.embeddings_backward(g, x, edges, inv_w, nb, w, bias=bias, w0=w0, b0=b0, **kw)
    got = o.embeddings_backward(pad(g), x, edges, inv_w, nb, pad(w), bias=pad(bias), w0=pad(w0), b0=pad(b0), **kw)
    np.testing.assert_allclose(got["grad_x"], ref["grad_x"], rtol=1e-6, atol=1e-7)
    for key in ("grad_W", "grad_bias", "grad_w0", "grad_b0"):
        if ref.get(key) is not None:
            assert not np.any(got[key][..., d]), key
            np.testing.assert_array_equal(got[key][..., :d], ref[key], err_msg=key)


def test_bin_index_rules():
    edges, inv_w, nb = o.pad_bins([np.array([0.0, 1.0, 2.0, 4.0], np.float32), np.array([-1.0, 1.0], np.float32)])
    x = np.array([[-5, -5], [0, -1], [1, 0], [1.5, 1], [2, 7], [4, np.nan], [9, np.inf],
                  [np.nan, -np.inf], [np.inf, 0.5]], np.float32)
    k = o.bin_index(x, edges, nb)
    assert k[:, 0].tolist() == [0, 0, 1, 1, 2, 2, 2, 2, 2]
    assert k[:, 1].tolist() == [0, 0, 0, 0, 0, 0, 0, 0, 0]
    assert o.physical_bin(np.array([0, 1, 2]), 3, 3).tolist() == [0, 1, 2]
    assert o.physical_bin(np.array([0, 1]), 2, 5).tolist() == [0, 4]


def test_boundary_subgradient_finite_difference():
    """At an interior edge the reference adds both adjacent slopes; away from
    edges grad_x matches a central finite difference of the dense form."""
    bins = [np.array([0.0, 1.0, 3.0, 4.0], np.float32)]
    edges, inv_w, nb = o.pad_bins(bins)
    w = np.random.default_rng(0).uniform(0.05, 0.25, size=(1, 3, 4)).astype(np.float32)
    g = np.ones((1, 1, 4), np.float32)
    x_in = np.array([[2.0]], np.float32)
    gx, _ = o.x_ple_backward(g, x_in, edges, inv_w, nb, w)
    h = 1e-3
    x64 = x_in.astype(np.float64)
    fd = (o.dense_forward(x64 + h, edges, inv_w, nb, w) - o.dense_forward(x64 - h, edges, inv_w, nb, w)) / (2 * h)
    np.testing.assert_allclose(gx, fd.sum(-1), rtol=1e-6)
    x_tie = np.array([[1.0]], np.float32)
    gx_tie, _ = o.x_ple_backward(g, x_tie, edges, inv_w, nb, w)
    left = w[0, 0].sum() * inv_w[0, 0]
    right = w[0, 1].sum() * inv_w[0, 1]
    np.testing.assert_allclose(gx_tie[0, 0], left + right, rtol=1e-6)


def test_grad_w_matches_dense_autograd():
    torch = pytest.importorskip("torch")
    x, edges, inv_w, nb, w, bias, w0, b0 = _setup("ragged", n=128, d=6, version="A")
    g = np.random.default_rng(1).standard_normal((128, 4, 6)).astype(np.float32)
    _, gw = o.x_ple_backward(g, x, edges, inv_w, nb, w)
    enc = torch.from_numpy(o.dense_encoding(x, edges, inv_w, nb))
    gw_dense = torch.einsum("nfb,nfd->fbd", enc, torch.from_numpy(g).double()).numpy()
    np.testing.assert_allclose(gw, gw_dense, rtol=1e-5, atol=1e-6)  # fp32 t vs float64 encoding


def test_bf16_round_matches_torch():
    torch = pytest.importorskip("torch")
    v = np.random.default_rng(2).standard_normal(10000).astype(np.float32) * 100
    ours = o.bf16_round(v)
    ref = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, ref)


def test_algorithmic_bytes_match_survey():
    from piecewiselinearembeddings_optimized_b200 import workloads as w

    expect = {"c1": 1_175_616, "c2": 71_483_904, "c3": 1_105_462_272, "c4": 1_814_513_664}
    for name, b in expect.items():
        wl = w.make_workload(name, n=8)  # bins/params only matter; bytes scale with n
        full = w.algorithmic_bytes(wl, n_local=w.SPECS[name][0])
        assert full["step"] == b, name


# ---------------------------------------------------------------- golden pinning

def _golden_files():
    return sorted(GOLDEN.glob("*.npz"))


@pytest.mark.skipif(not _golden_files(), reason="golden fixtures not generated")
@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_golden(path):
    """The oracle reproduces the reference's own CUDA ops (x_ple, bin indices,
    grad_x, grad_W) and the module composition on the same inputs."""
    z = np.load(path, allow_pickle=False)
    if "workload" in z.files:
        from piecewiselinearembeddings_optimized_b200 import workloads
        from tests.golden.make_golden import digest

        n = int(z["n"])
        f = int(z["f"])
        name = str(z["workload"])
        spec_n, spec_f = workloads.SPECS[name][0], workloads.SPECS[name][1]
        wl = workloads.make_workload(name, n=None if n == spec_n else n, f=None if f == spec_f else f)
        g = workloads.make_grad(wl)
        assert digest(wl.x, wl.weight, wl.bias, wl.w0, wl.b0, g) == str(z["input_digest"])
        edges, inv_w, nb = o.pad_bins(wl.bins)
        x, w, bias, w0, b0 = wl.x, wl.weight, wl.bias, wl.w0, wl.b0
        version, relu, mode = wl.version, wl.activation, wl.mode
        rows = z["rows"]
        xs = x[rows]
        xp, k = o.x_ple_forward(xs, edges, inv_w, nb, w, mode)
        np.testing.assert_array_equal(k, z["ref_bin_indices"][rows])
        np.testing.assert_allclose(xp, z["ref_x_ple_rows"], rtol=1e-5, atol=1e-6)
        grads = o.embeddings_backward(g, x, edges, inv_w, nb, w, version=version, activation=relu,
                                      bias=bias, w0=w0, b0=b0, mode=mode)
        np.testing.assert_allclose(grads["grad_x"], z["ref_grad_x"], rtol=1e-4, atol=1e-5)
        for key in ("grad_W", "grad_bias", "grad_w0", "grad_b0"):
            if "ref_" + key in z.files:
                o.assert_reduction_close(grads[key], z["ref_" + key], grads["abs"][key], err_msg=key)
        return

    mode = str(z["mode"])
    version = str(z["version"])
    relu = bool(z["activation"])
    edges, inv_w, nb, x, w, g = z["edges"], z["inv_w"], z["n_bins"], z["x"], z["weight"], z["g"]
    bias = z["bias"] if "bias" in z.files else None
    w0 = z["w0"] if "w0" in z.files else None
    b0 = z["b0"] if "b0" in z.files else None
    xp, k = o.x_ple_forward(x, edges, inv_w, nb, w, mode)
    np.testing.assert_array_equal(k, z["ref_bin_indices"])
    tol = dict(rtol=1e-5, atol=1e-6) if mode == "f32" else dict(rtol=1e-2, atol=1e-2)
    finite = np.isfinite(z["ref_x_ple"])
    np.testing.assert_array_equal(finite, np.isfinite(xp))
    np.testing.assert_allclose(xp[finite], z["ref_x_ple"][finite], **tol)
    y, _, _ = o.embeddings_forward(x, edges, inv_w, nb, w, version=version, activation=relu,
                                   bias=bias, w0=w0, b0=b0, mode=mode)
    finite = np.isfinite(z["ref_y"])
    np.testing.assert_allclose(y[finite], z["ref_y"][finite], **tol)
    if not bool(z["backward"]):
        return
    gtol = dict(rtol=1e-4, atol=1e-5) if mode == "f32" else dict(rtol=2e-2, atol=2e-2)
    gx_ple, gw_ple, abs_w = o.x_ple_backward(z["ref_g_ple"], x, edges, inv_w, nb, w, mode, with_abs=True)
    np.testing.assert_allclose(gx_ple, z["ref_grad_x_ple"], **gtol)
    o.assert_reduction_close(gw_ple, z["ref_grad_W"], abs_w, err_msg="grad_W (x_ple op)", **gtol)
    grads = o.embeddings_backward(g, x, edges, inv_w, nb, w, version=version, activation=relu,
                                  bias=bias, w0=w0, b0=b0, mode=mode)
    np.testing.assert_allclose(grads["grad_x"], z["ref_grad_x"], **gtol)
    for key in ("grad_W", "grad_bias", "grad_w0", "grad_b0"):
        if "ref_" + key in z.files:
            o.assert_reduction_close(grads[key], z["ref_" + key], grads["abs"][key], err_msg=key, **gtol)
