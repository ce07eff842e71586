"""Bin edges on the device: upstream ``rtdl_num_embeddings.compute_bins`` for
quantile bins (no tree), computed by ``rtdl_num_embeddings_cuda::compute_bins``.

Per feature the ``n_bins + 1`` quantiles at ``j / n_bins`` of the training
column (linear interpolation between order statistics, as ``torch.quantile``)
with repeated values removed; the reference builds these on the host and pads
them in a Python loop (``module.py:58-109``).
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _native

_native.load_ops()
from . import _meta as _meta  # noqa: E402,F401


def _checked_tables(X: Tensor, n_bins: int):
    if X.ndim != 2:
        raise ValueError(f"X must have two dimensions, got {X.ndim}")
    if X.shape[0] < 2:
        raise ValueError("X must have at least two rows")
    if not 1 <= n_bins <= 1023:
        raise ValueError("n_bins must lie in [1, 1023]")
    if X.device.type != "cuda":
        raise RuntimeError("compute_bins runs on CUDA tensors only (this package has no CPU path)")
    X = X.to(torch.float32)
    if not bool(torch.isfinite(X).all()):
        raise ValueError("X must contain only finite values")
    edges, inv_w, nb = torch.ops.rtdl_num_embeddings_cuda.compute_bins(X, int(n_bins))
    counts = nb.tolist()
    bad = [i for i, c in enumerate(counts) if c < 1]
    if bad:
        raise ValueError(f"features {bad[:10]} have fewer than two distinct quantiles (constant columns)")
    return edges, inv_w, nb, counts


def compute_bins(X: Tensor, n_bins: int = 48) -> list[Tensor]:
    """Bin edges per feature (a list of 1-D float32 tensors on X's device)."""
    edges, _, _, counts = _checked_tables(X, n_bins)
    return [edges[i, : c + 1].clone() for i, c in enumerate(counts)]


def bin_tables(X: Tensor, n_bins: int = 48):
    """The padded tables of ``compute_bins(X, n_bins)`` directly: edges
    ``[F, B+1]`` (+inf padded), reciprocal widths ``[F, B]`` (0 padded) and
    ``n_bins [F]`` int32 with ``B = max_i n_i`` (what ``pad_bin_tables`` builds
    from the edge list)."""
    edges, inv_w, nb, counts = _checked_tables(X, n_bins)
    b = max(counts)
    return edges[:, : b + 1].contiguous(), inv_w[:, :b].contiguous(), nb
