"""``CudaPiecewiseLinearEmbeddings``: the drop-in module (reference ``module.py``).

Same constructor (``bins, d_embedding, *, activation, version``), same
trainable parameters and ``state_dict`` as the upstream
``PiecewiseLinearEmbeddings``, same non-persistent helper buffers
``_cuda_bin_edges [F, B+1]`` (+inf padded), ``_cuda_inv_bin_widths [F, B]``
(fp32 reciprocal widths, 0 padded) and ``_cuda_n_bins [F]`` int32
(reference ``module.py:58-131``).

On CUDA the whole forward - ``[linear0(x)] + act(x_ple + [bias])`` - is one
fused kernel (``rtdl_num_embeddings_cuda::embeddings_forward``) and the whole
backward is one fused kernel plus a tiny finalize; the reference runs the
``x_ple`` op plus 1-3 separate PyTorch passes.  Autocast semantics follow the
reference: under CUDA fp16/bf16 autocast ``x_ple`` is computed from weights
and positions rounded to that type with fp32 accumulation and rounded to it,
then the fp32 epilogue produces an fp32 result.  ``output_dtype`` (default
``None`` = the reference's result dtype) may be set to store the result
directly in bf16/fp16.

Non-CUDA inputs are delegated to the base class (upstream's implementation
when installed); this package itself has no CPU compute path.
"""
from __future__ import annotations

from typing import Literal

import torch
from torch import Tensor

from . import _native
from ._compat import Base

_native.load_ops()
from . import _meta as _meta  # noqa: E402,F401  (fake registrations)
from . import _autograd as _autograd  # noqa: E402,F401  (autograd registrations)

EPILOGUE_NONE, EPILOGUE_A, EPILOGUE_B = 0, 1, 2


def pad_bin_tables(bins: list[Tensor]):
    """Padded edges ``[F, B+1]`` (+inf), fp32 reciprocal widths ``[F, B]`` (0) and
    ``n_bins [F]`` int32 (reference ``module.py:58-109``)."""
    n_bins = [int(e.numel() - 1) for e in bins]
    f, b = len(bins), max(n_bins)
    device = bins[0].device
    for i, e in enumerate(bins):
        if e.device != device:
            raise ValueError(
                "All bin tensors must be on the same device. "
                f"bins[0].device={device}, bins[{i}].device={e.device}"
            )
    edges = torch.full((f, b + 1), torch.inf, dtype=torch.float32, device=device)
    inv_w = torch.zeros((f, b), dtype=torch.float32, device=device)
    for i, e in enumerate(bins):
        e32 = e.to(device=device, dtype=torch.float32)
        edges[i, : e32.numel()].copy_(e32)
        inv_w[i, : e32.numel() - 1].copy_(torch.reciprocal(e32[1:] - e32[:-1]))
    return edges, inv_w, torch.tensor(n_bins, dtype=torch.int32, device=device)


class CudaPiecewiseLinearEmbeddings(Base):
    """Drop-in CUDA implementation of ``PiecewiseLinearEmbeddings``.

    CUDA contract (as the reference's): ``x`` contiguous float32 ``[N, F]``,
    float32 parameters, first-order autograd, ``torch.compile(fullgraph=True)``
    through the fake registrations; double backward is not implemented.
    """

    def __init__(self, bins: list[Tensor], d_embedding: int, *, activation: bool,
                 version: Literal[None, "A", "B"] = None) -> None:
        assert d_embedding <= 64, "d_embedding must be less than or equal to 64"
        super().__init__(bins, d_embedding, activation=activation, version=version)
        edges, inv_w, n_bins = pad_bin_tables(bins)
        # non-persistent: state_dict stays identical to upstream's
        self.register_buffer("_cuda_bin_edges", edges, persistent=False)
        self.register_buffer("_cuda_inv_bin_widths", inv_w, persistent=False)
        self.register_buffer("_cuda_n_bins", n_bins, persistent=False)
        self.output_dtype: torch.dtype | None = None

    @property
    def n_features(self) -> int:
        return int(self.linear.weight.shape[0])

    @property
    def max_n_bins(self) -> int:
        return int(self.linear.weight.shape[1])

    @property
    def d_embedding(self) -> int:
        return int(self.linear.weight.shape[2])

    def _cuda_output_dtype(self) -> torch.dtype:
        """Type of ``x_ple``: fp32, or the CUDA autocast dtype (reference ``module.py:145-158``)."""
        if torch.is_autocast_enabled("cuda"):
            dtype = torch.get_autocast_dtype("cuda")
            if dtype not in (torch.float16, torch.bfloat16):
                raise RuntimeError(f"CUDA autocast dtype must be float16 or bfloat16, got {dtype}")
            return dtype
        return torch.float32

    def _check_cuda_inputs(self, x: Tensor) -> None:
        if x.dtype != torch.float32:
            raise TypeError(f"The fused CUDA path requires float32 x. Got {x.dtype}.")
        if self.linear.weight.dtype != torch.float32:
            raise TypeError(
                f"The fused CUDA path requires float32 parameters. Got weight dtype {self.linear.weight.dtype}."
            )
        if not x.is_contiguous():
            raise ValueError("The fused CUDA path requires contiguous x.")
        for name in ("_cuda_bin_edges", "_cuda_inv_bin_widths", "_cuda_n_bins"):
            if not getattr(self, name).is_contiguous():
                raise RuntimeError(f"{name} must be contiguous")
        if not self.linear.weight.is_contiguous():
            raise RuntimeError("linear.weight must be contiguous")

    def _forward_cuda_x_ple(self, x: Tensor) -> Tensor:
        """``x_ple`` alone through the reference op ``rtdl_num_embeddings_cuda::forward``."""
        self._check_cuda_inputs(x)
        x_ple, _ = torch.ops.rtdl_num_embeddings_cuda.forward(
            x, self._cuda_bin_edges, self._cuda_inv_bin_widths, self._cuda_n_bins, self.linear.weight,
            self._cuda_output_dtype(),
        )
        return x_ple

    def forward(self, x: Tensor) -> Tensor:
        if x.ndim != 2:
            raise ValueError("Only inputs with shape [batch_size, n_features] are supported")
        if x.shape[1] != self.n_features:
            raise ValueError(f"Expected {self.n_features} numerical features, got {x.shape[1]}")
        if x.device.type != "cuda":
            return super().forward(x)
        if x.device != self._cuda_bin_edges.device:
            raise RuntimeError("x and the module must be on the same CUDA device")
        self._check_cuda_inputs(x)
        compute = self._cuda_output_dtype()
        out_dtype = self.output_dtype or torch.float32
        if self.linear0 is not None:
            epilogue, bias, w0, b0 = EPILOGUE_B, None, self.linear0.weight, self.linear0.bias
        elif self.linear.bias is not None:
            epilogue, bias, w0, b0 = EPILOGUE_A, self.linear.bias, None, None
        else:
            epilogue, bias, w0, b0 = EPILOGUE_NONE, None, None, None
        return torch.ops.rtdl_num_embeddings_cuda.embeddings_forward(
            x, self._cuda_bin_edges, self._cuda_inv_bin_widths, self._cuda_n_bins, self.linear.weight,
            bias, w0, b0, epilogue, self.activation is not None, compute, out_dtype,
        )


class CudaPiecewiseLinearEmbeddingsLinear(torch.nn.Module):
    """``linear(embeddings(x).flatten(1))`` with the embeddings fused into the Linear.

    Wraps an existing ``CudaPiecewiseLinearEmbeddings`` and the
    ``nn.Linear(F * D, H)`` that consumes its flattened output (parameters are
    shared, not copied), so it replaces ``nn.Sequential(embeddings,
    nn.Flatten(), linear)`` in an MLP.  With ``fused=True``, on CUDA under bf16
    autocast the three run as one tensor-core kernel (``rtdl_num_embeddings_cuda::
    embeddings_linear_forward``) whose ``[N, F, D]`` intermediate never reaches
    memory; the result is bf16, as autocast's Linear returns.  With
    ``bf16_linear=True`` and no autocast the fp32 module output is rounded to
    bf16 for the product and the result is fp32.  Everything else (CPU inputs,
    fp16 autocast, plain fp32, d_embedding not a multiple of 8, more than 256
    bins) runs the composition: the module's own kernel followed by ``linear``.

    The fused kernel is opt-in (``fused=True``); by default the module runs
    the composition.  The trade-off: the fused kernel never allocates the
    ``[N, F, D]`` activation (805 MB at 65,536 rows × 256 features × D = 24 in
    bf16), but on one B200 it is slower than the composition at the measured
    shapes (e.g. 0.55 ms against 0.43 ms for Linear(6144, 256) over 65,536
    rows), so it pays only where that activation does not fit in memory.
    """

    def __init__(self, embeddings: CudaPiecewiseLinearEmbeddings, linear: torch.nn.Linear, *,
                 bf16_linear: bool = False, fused: bool = False) -> None:
        super().__init__()
        d_in = embeddings.n_features * embeddings.d_embedding
        if linear.in_features != d_in:
            raise ValueError(f"linear.in_features must be n_features * d_embedding = {d_in}, "
                             f"got {linear.in_features}")
        self.embeddings = embeddings
        self.linear = linear
        self.bf16_linear = bf16_linear
        self.fused = fused

    def _fused_dtypes(self, x: Tensor):
        if not self.fused or x.device.type != "cuda" or self.embeddings.d_embedding % 8 != 0:
            return None
        if self.embeddings.linear.weight.shape[1] > 256:  # the fused kernel's tables hold up to 256 bins
            return None
        if torch.is_autocast_enabled("cuda"):
            if torch.get_autocast_dtype("cuda") != torch.bfloat16:
                return None
            return torch.bfloat16, torch.bfloat16
        return (torch.float32, torch.float32) if self.bf16_linear else None

    def forward(self, x: Tensor) -> Tensor:
        dtypes = self._fused_dtypes(x)
        if dtypes is None:
            return self.linear(self.embeddings(x).flatten(1))
        emb = self.embeddings
        if x.ndim != 2 or x.shape[1] != emb.n_features:
            raise ValueError(f"Expected x of shape [batch_size, {emb.n_features}]")
        if x.device != emb._cuda_bin_edges.device:
            raise RuntimeError("x and the module must be on the same CUDA device")
        emb._check_cuda_inputs(x)
        compute, out_dtype = dtypes
        if emb.linear0 is not None:
            epilogue, bias, w0, b0 = EPILOGUE_B, None, emb.linear0.weight, emb.linear0.bias
        elif emb.linear.bias is not None:
            epilogue, bias, w0, b0 = EPILOGUE_A, emb.linear.bias, None, None
        else:
            epilogue, bias, w0, b0 = EPILOGUE_NONE, None, None, None
        w1 = self.linear.weight.to(torch.bfloat16).contiguous()
        b1 = self.linear.bias
        if b1 is not None and compute == torch.bfloat16:
            b1 = b1.to(torch.bfloat16).float()  # autocast's Linear adds a bf16 bias
        return torch.ops.rtdl_num_embeddings_cuda.embeddings_linear_forward(
            x, emb._cuda_bin_edges, emb._cuda_inv_bin_widths, emb._cuda_n_bins, emb.linear.weight,
            bias, w0, b0, epilogue, emb.activation is not None, compute, w1, b1, out_dtype,
        )


ENCODING_RAGGED, ENCODING_PADDED = 0, 1


class CudaPiecewiseLinearEncoding(torch.nn.Module):
    """Drop-in CUDA counterpart of upstream ``PiecewiseLinearEncoding(bins)``.

    ``forward(x [..., F] float32) -> [..., sum_i n_i]``: for each feature i the
    ``n_i`` columns of its bins in logical order (feature-major, no padding),
    column j holding ``t_j = (x - e_j) / w_j`` clamped to ``<= 1`` (first bin),
    ``[0, 1]`` (middle bins), ``>= 0`` (last bin), unclamped for a single-bin
    feature; NaN propagates.  ``padded=True`` returns ``[..., F, B]`` in the
    embedding weights' physical layout instead (last real bin at column
    ``B - 1``, zero padding).  The gradient with respect to x passes the clamps
    at their bounds (``torch.clamp``'s rule).  The reference package has no
    CUDA path for this module; here both directions are sm_100a kernels.
    Non-CUDA inputs go to upstream's class when it is installed.
    """

    def __init__(self, bins: list[Tensor], *, padded: bool = False) -> None:
        super().__init__()
        from ._compat import check_bins

        check_bins(bins)
        edges, inv_w, n_bins = pad_bin_tables(bins)
        counts = [int(e.numel() - 1) for e in bins]
        offsets = [0]
        for c in counts:
            offsets.append(offsets[-1] + c)
        self.register_buffer("_cuda_bin_edges", edges, persistent=False)
        self.register_buffer("_cuda_inv_bin_widths", inv_w, persistent=False)
        self.register_buffer("_cuda_n_bins", n_bins, persistent=False)
        self.register_buffer("_cuda_col_offsets", torch.tensor(offsets, dtype=torch.int64, device=edges.device),
                             persistent=False)
        self.padded = bool(padded)
        self.total_n_bins = offsets[-1]
        self.max_n_bins = int(inv_w.shape[1])
        self.output_dtype: torch.dtype = torch.float32
        self._upstream = None
        self._bins = [b.detach().clone() for b in bins]

    @property
    def n_features(self) -> int:
        return int(self._cuda_n_bins.shape[0])

    def _cpu_forward(self, x: Tensor) -> Tensor:
        from . import _compat

        if not getattr(_compat, "HAVE_UPSTREAM", False):
            raise RuntimeError(
                "CudaPiecewiseLinearEncoding has no CPU implementation; install rtdl_num_embeddings for CPU inputs"
            )
        if self._upstream is None:
            from rtdl_num_embeddings import PiecewiseLinearEncoding  # pragma: no cover

            self._upstream = PiecewiseLinearEncoding([b.to(x.device) for b in self._bins])  # pragma: no cover
        return self._upstream(x)  # pragma: no cover

    def forward(self, x: Tensor) -> Tensor:
        if x.ndim < 2:
            raise ValueError("The input must have at least two dimensions: [..., n_features]")
        if x.shape[-1] != self.n_features:
            raise ValueError(f"Expected {self.n_features} numerical features, got {x.shape[-1]}")
        if x.device.type != "cuda":
            return self._cpu_forward(x)
        if x.device != self._cuda_bin_edges.device:
            raise RuntimeError("x and the module must be on the same CUDA device")
        if x.dtype != torch.float32:
            raise TypeError(f"The CUDA encoding requires float32 x. Got {x.dtype}.")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.n_features).contiguous()
        layout = ENCODING_PADDED if self.padded else ENCODING_RAGGED
        total = self.n_features * self.max_n_bins if self.padded else self.total_n_bins
        y = torch.ops.rtdl_num_embeddings_cuda.encoding_forward(
            x2, self._cuda_bin_edges, self._cuda_inv_bin_widths, self._cuda_n_bins, self._cuda_col_offsets, layout,
            total, self.output_dtype,
        )
        return y.reshape(*lead, *y.shape[1:])
