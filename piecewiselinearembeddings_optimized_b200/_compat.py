"""Base class of the drop-in module.

When the upstream package ``rtdl_num_embeddings`` (the dependency the
reference subclasses, ``pyproject.toml:17``) is importable, its
``PiecewiseLinearEmbeddings`` is the base class, exactly as in the reference
(``module.py:6-11``).  Otherwise a minimal base with the same trainable
parameter names, shapes and initialisation is used, so checkpoints
(``state_dict``) stay interchangeable:

* ``linear.weight [F, B, D]`` and, for version A, ``linear.bias [F, D]``,
  both ``U(-B**-0.5, B**-0.5)``; version B zero-initialises ``linear.weight``;
* version B: ``linear0.weight [F, D]`` and ``linear0.bias [F, D]``,
  ``U(-D**-0.5, D**-0.5)``;
* ``activation`` is ``nn.ReLU()`` or ``None``; ``version=None`` means "A"
  (with a warning, as upstream).

The minimal base has no CPU implementation: the CUDA kernels are the only
compute path of this package.
"""
from __future__ import annotations

import warnings

import torch
from torch import Tensor, nn

try:  # pragma: no cover - exercised only where upstream is installed
    from rtdl_num_embeddings import PiecewiseLinearEmbeddings as _UpstreamBase

    HAVE_UPSTREAM = True
except ImportError:  # the usual case in this environment
    _UpstreamBase = None
    HAVE_UPSTREAM = False


def check_bins(bins: list[Tensor]) -> None:
    """Validation of the bin edges (one 1-D, finite, strictly increasing tensor
    of at least two edges per feature)."""
    if not bins:
        raise ValueError("The list of bins must not be empty")
    for i, b in enumerate(bins):
        if not isinstance(b, Tensor):
            raise ValueError(f"bins[{i}] must be a torch.Tensor")
        if b.ndim != 1:
            raise ValueError(f"bins[{i}] must be one-dimensional, got shape {tuple(b.shape)}")
        if b.numel() < 2:
            raise ValueError(f"bins[{i}] must have at least two edges")
        if not torch.isfinite(b).all():
            raise ValueError(f"bins[{i}] must contain only finite values")
        if b.numel() > 1 and not (b[1:] > b[:-1]).all():
            raise ValueError(f"bins[{i}] must be sorted in strictly increasing order")


class _NLinear(nn.Module):
    """``n`` independent linear layers: weight ``[n, in, out]``, bias ``[n, out]``."""

    def __init__(self, n: int, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(n, in_features, out_features))
        self.bias = nn.Parameter(torch.empty(n, out_features)) if bias else None
        bound = in_features ** -0.5
        nn.init.uniform_(self.weight, -bound, bound)
        if self.bias is not None:
            nn.init.uniform_(self.bias, -bound, bound)


class _LinearEmbeddings(nn.Module):
    """Per-feature affine map ``x[..., None] * weight + bias`` with ``[F, D]`` parameters."""

    def __init__(self, n_features: int, d_embedding: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(n_features, d_embedding))
        self.bias = nn.Parameter(torch.empty(n_features, d_embedding))
        bound = d_embedding ** -0.5
        nn.init.uniform_(self.weight, -bound, bound)
        nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x: Tensor) -> Tensor:
        return torch.addcmul(self.bias, self.weight, x[..., None])


class _MinimalBase(nn.Module):
    def __init__(self, bins: list[Tensor], d_embedding: int, *, activation: bool, version=None) -> None:
        if d_embedding <= 0:
            raise ValueError(f"d_embedding must be a positive integer, got {d_embedding}")
        check_bins(bins)
        if version is None:
            warnings.warn(
                'The `version` argument is not provided, so version="A" will be used '
                "for backward compatibility.",
                stacklevel=3,
            )
            version = "A"
        if version not in ("A", "B"):
            raise ValueError(f'version must be "A" or "B", got {version!r}')
        super().__init__()
        n_features = len(bins)
        max_n_bins = max(len(b) - 1 for b in bins)
        is_b = version == "B"
        self.linear0 = _LinearEmbeddings(n_features, d_embedding) if is_b else None
        self.linear = _NLinear(n_features, max_n_bins, d_embedding, bias=not is_b)
        if is_b:
            nn.init.zeros_(self.linear.weight)
        self.activation = nn.ReLU() if activation else None

    def get_output_shape(self) -> torch.Size:
        return torch.Size((self.linear.weight.shape[0], self.linear.weight.shape[2]))

    def forward(self, x: Tensor) -> Tensor:  # only reached for non-CUDA inputs
        raise RuntimeError(
            "CudaPiecewiseLinearEmbeddings computes on CUDA tensors only; CPU execution is "
            "delegated to the upstream rtdl_num_embeddings package, which is not installed"
        )


Base = _UpstreamBase if HAVE_UPSTREAM else _MinimalBase

