"""Quantile bin edges on the device (upstream ``compute_bins`` without a tree):
distinct-edge counts equal the oracle's, edges within fp32 rounding of the
float64 quantiles, padded tables bitwise equal to ``pad_bin_tables`` of the
edge list; constant columns and bad inputs are refused."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ple_oracle as o

torch = pytest.importorskip("torch")


def _columns(n, seed):
    rng = np.random.default_rng(seed)
    return np.stack([
        rng.standard_normal(n),                      # continuous
        rng.poisson(3.0, n).astype(np.float64),      # integer values: many equal quantiles
        rng.lognormal(0.0, 1.0, n),                  # skewed
        np.repeat(np.arange(5.0), n // 5 + 1)[:n],   # five values only
        rng.uniform(-5, 5, n),
    ], axis=1).astype(np.float32)


def test_oracle_quantile_bins_dedup():
    X = _columns(1000, 0)
    bins = o.quantile_bins(X, 48)
    assert len(bins[0]) == 49 and len(bins[3]) == 5
    assert all(np.all(np.diff(b) > 0) for b in bins)


def test_compute_bins_refuses_cpu_and_bad_shapes():
    from rtdl_num_embeddings_cuda import compute_bins

    with pytest.raises(RuntimeError, match="CUDA"):
        compute_bins(torch.zeros(10, 3), 8)
    with pytest.raises(ValueError):
        compute_bins(torch.zeros(10), 8)
    with pytest.raises(ValueError):
        compute_bins(torch.zeros(10, 2), 0)


@pytest.mark.gpu
@pytest.mark.parametrize("n,n_bins", [(1000, 48), (4096, 16), (257, 64), (50_000, 100)])
def test_compute_bins_matches_oracle(cuda_device, n, n_bins):
    from piecewiselinearembeddings_optimized_b200.module import pad_bin_tables
    from rtdl_num_embeddings_cuda import bin_tables, compute_bins

    X = _columns(n, n)
    ref = o.quantile_bins(X, n_bins)
    got = compute_bins(torch.from_numpy(X).to(cuda_device), n_bins)
    assert [len(b) for b in got] == [len(b) for b in ref]
    for g, r in zip(got, ref):
        np.testing.assert_allclose(g.cpu().numpy(), r, rtol=2e-7, atol=1e-6)
        assert bool((g[1:] > g[:-1]).all())
    e, w, nb = bin_tables(torch.from_numpy(X).to(cuda_device), n_bins)
    e2, w2, nb2 = pad_bin_tables(got)
    assert torch.equal(e, e2) and torch.equal(w, w2) and torch.equal(nb, nb2)


@pytest.mark.gpu
def test_compute_bins_refuses_constant_columns(cuda_device):
    from rtdl_num_embeddings_cuda import compute_bins

    X = torch.randn(100, 3, device=cuda_device)
    X[:, 1] = 2.5
    with pytest.raises(ValueError, match="constant"):
        compute_bins(X, 8)
    X[0, 1] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        compute_bins(X, 8)


@pytest.mark.gpu
def test_modules_from_device_bins(cuda_device):
    """Both modules accept the device-computed edges (the usual construction)."""
    from rtdl_num_embeddings_cuda import CudaPiecewiseLinearEmbeddings, CudaPiecewiseLinearEncoding, compute_bins

    X = torch.from_numpy(_columns(2048, 7)).to(cuda_device)
    bins = compute_bins(X, 32)
    m = CudaPiecewiseLinearEmbeddings(bins, 8, activation=True, version="B").to(cuda_device)
    y = m(X)
    assert y.shape == (2048, 5, 8) and bool(torch.isfinite(y).all())
    enc = CudaPiecewiseLinearEncoding(bins).to(cuda_device)
    assert enc(X).shape == (2048, sum(len(b) - 1 for b in bins))
