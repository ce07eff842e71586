"""Fake (meta) implementations of the ``rtdl_num_embeddings_cuda`` ops.

Shape and dtype propagation for FakeTensor / ``torch.compile(fullgraph=True)``;
the checks follow the reference's ``_meta.py:22-188`` for ``forward`` and
``backward`` and extend them to the fused ``embeddings_*`` ops.
"""
from __future__ import annotations

import torch
from torch import Tensor

SUPPORTED_FLOAT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def bin_indices_dtype(max_n_bins: int) -> torch.dtype:
    """u8 up to 256 bins, i16 up to 32768, i32 beyond (reference ``_meta.py:14-19``)."""
    if max_n_bins <= 256:
        return torch.uint8
    if max_n_bins <= 32768:
        return torch.int16
    return torch.int32


def _check_tables(x, bin_edges, inv_bin_widths, n_bins, weight) -> None:
    torch._check(x.ndim == 2, lambda: "x must have shape [N, F]")
    torch._check(bin_edges.ndim == 2, lambda: "bin_edges must have shape [F, B + 1]")
    torch._check(inv_bin_widths.ndim == 2, lambda: "inv_bin_widths must have shape [F, B]")
    torch._check(n_bins.ndim == 1, lambda: "n_bins must have shape [F]")
    torch._check(weight.ndim == 3, lambda: "weight must have shape [F, B, D]")
    torch._check(x.shape[1] == weight.shape[0], lambda: "x.shape[1] must equal weight.shape[0]")
    torch._check(bin_edges.shape[0] == weight.shape[0], lambda: "bin_edges.shape[0] must equal weight.shape[0]")
    torch._check(bin_edges.shape[1] == weight.shape[1] + 1,
                 lambda: "bin_edges.shape[1] must equal weight.shape[1] + 1")
    torch._check(inv_bin_widths.shape[0] == weight.shape[0],
                 lambda: "inv_bin_widths.shape[0] must equal weight.shape[0]")
    torch._check(inv_bin_widths.shape[1] == weight.shape[1],
                 lambda: "inv_bin_widths.shape[1] must equal weight.shape[1]")
    torch._check(n_bins.shape[0] == weight.shape[0], lambda: "n_bins.shape[0] must equal weight.shape[0]")
    torch._check(x.dtype == torch.float32, lambda: "x must be float32")
    torch._check(bin_edges.dtype == torch.float32, lambda: "bin_edges must be float32")
    torch._check(inv_bin_widths.dtype == torch.float32, lambda: "inv_bin_widths must be float32")
    torch._check(n_bins.dtype == torch.int32, lambda: "n_bins must be int32")
    torch._check(weight.dtype == torch.float32, lambda: "weight must be float32")


@torch.library.register_fake("rtdl_num_embeddings_cuda::forward")
def _forward_fake(x: Tensor, bin_edges: Tensor, inv_bin_widths: Tensor, n_bins: Tensor, weight: Tensor,
                  output_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    _check_tables(x, bin_edges, inv_bin_widths, n_bins, weight)
    torch._check(output_dtype in SUPPORTED_FLOAT_DTYPES, lambda: "Unsupported output dtype")
    return (
        torch.empty((x.shape[0], x.shape[1], weight.shape[2]), dtype=output_dtype, device=x.device),
        torch.empty((x.shape[0], x.shape[1]), dtype=bin_indices_dtype(weight.shape[1]), device=x.device),
    )


@torch.library.register_fake("rtdl_num_embeddings_cuda::backward")
def _backward_fake(grad_output: Tensor, x: Tensor, bin_edges: Tensor, inv_bin_widths: Tensor, n_bins: Tensor,
                   weight: Tensor, bin_indices: Tensor, compute_grad_x: bool,
                   compute_grad_weight: bool) -> tuple[Tensor, Tensor]:
    torch._check(grad_output.ndim == 3, lambda: "grad_output must have shape [N, F, D]")
    torch._check(grad_output.shape[0] == x.shape[0], lambda: "grad_output N mismatch")
    torch._check(grad_output.shape[1] == x.shape[1], lambda: "grad_output F mismatch")
    torch._check(grad_output.shape[2] == weight.shape[2], lambda: "grad_output D mismatch")
    torch._check(bin_indices.shape[0] == x.shape[0], lambda: "bin_indices N mismatch")
    torch._check(bin_indices.shape[1] == x.shape[1], lambda: "bin_indices F mismatch")
    torch._check(bin_indices.dtype == bin_indices_dtype(weight.shape[1]),
                 lambda: "bin_indices has an invalid dtype")
    torch._check(grad_output.dtype in SUPPORTED_FLOAT_DTYPES, lambda: "Unsupported grad_output dtype")
    grad_x = torch.empty_like(x) if compute_grad_x else torch.empty((0,), dtype=x.dtype, device=x.device)
    grad_w = (torch.empty_like(weight) if compute_grad_weight
              else torch.empty((0,), dtype=weight.dtype, device=weight.device))
    return grad_x, grad_w


@torch.library.register_fake("rtdl_num_embeddings_cuda::embeddings_forward")
def _embeddings_forward_fake(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue: int,
                             activation: bool, compute_dtype: torch.dtype, output_dtype: torch.dtype) -> Tensor:
    _check_tables(x, bin_edges, inv_bin_widths, n_bins, weight)
    torch._check(output_dtype in SUPPORTED_FLOAT_DTYPES, lambda: "Unsupported output dtype")
    torch._check(compute_dtype in SUPPORTED_FLOAT_DTYPES, lambda: "Unsupported compute dtype")
    torch._check(epilogue in (0, 1, 2), lambda: "epilogue must be 0 (none), 1 (A) or 2 (B)")
    return torch.empty((x.shape[0], x.shape[1], weight.shape[2]), dtype=output_dtype, device=x.device)


@torch.library.register_fake("rtdl_num_embeddings_cuda::embeddings_backward")
def _embeddings_backward_fake(grad_output, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0,
                              bin_indices, epilogue: int, activation: bool, compute_dtype: torch.dtype,
                              compute_grad_x: bool, compute_grad_weight: bool, compute_grad_bias: bool,
                              compute_grad_linear0: bool):
    torch._check(grad_output.ndim == 3, lambda: "grad_output must have shape [N, F, D]")
    f, d = weight.shape[0], weight.shape[2]

    def empty(shape, on: bool):
        return torch.empty(shape if on else (0,), dtype=torch.float32, device=x.device)

    return (
        empty(tuple(x.shape), compute_grad_x),
        empty(tuple(weight.shape), compute_grad_weight),
        empty((f, d), compute_grad_bias and epilogue == 1),
        empty((f, d), compute_grad_linear0 and epilogue == 2),
        empty((f, d), compute_grad_linear0 and epilogue == 2),
    )


ENC_RAGGED, ENC_PADDED = 0, 1


@torch.library.register_fake("rtdl_num_embeddings_cuda::encoding_forward")
def _encoding_forward_fake(x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout: int, total_bins: int,
                           output_dtype: torch.dtype) -> Tensor:
    torch._check(x.ndim == 2, lambda: "x must have shape [N, F]")
    torch._check(x.dtype == torch.float32, lambda: "x must be float32")
    torch._check(output_dtype in SUPPORTED_FLOAT_DTYPES, lambda: "Unsupported output dtype")
    torch._check(layout in (ENC_RAGGED, ENC_PADDED), lambda: "layout must be 0 (ragged) or 1 (padded)")
    if layout == ENC_PADDED:
        return torch.empty((x.shape[0], x.shape[1], inv_bin_widths.shape[1]), dtype=output_dtype, device=x.device)
    torch._check(col_offsets is not None, lambda: "the ragged layout needs col_offsets")
    return torch.empty((x.shape[0], total_bins), dtype=output_dtype, device=x.device)


@torch.library.register_fake("rtdl_num_embeddings_cuda::encoding_backward")
def _encoding_backward_fake(grad_output, x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout: int,
                            total_bins: int) -> Tensor:
    torch._check(grad_output.shape[0] == x.shape[0], lambda: "grad_output N mismatch")
    return torch.empty_like(x)


@torch.library.register_fake("rtdl_num_embeddings_cuda::compute_bins")
def _compute_bins_fake(x, n_bins: int):
    torch._check(x.ndim == 2, lambda: "x must have shape [N, F]")
    f = x.shape[1]
    return (torch.empty((f, n_bins + 1), dtype=torch.float32, device=x.device),
            torch.empty((f, n_bins), dtype=torch.float32, device=x.device),
            torch.empty((f,), dtype=torch.int32, device=x.device))


@torch.library.register_fake("rtdl_num_embeddings_cuda::embeddings_linear_forward")
def _embeddings_linear_forward_fake(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue: int,
                                    activation: bool, compute_dtype: torch.dtype, linear_weight, linear_bias,
                                    output_dtype: torch.dtype):
    _check_tables(x, bin_edges, inv_bin_widths, n_bins, weight)
    torch._check(linear_weight.ndim == 2, lambda: "linear_weight must have shape [H, F * D]")
    torch._check(linear_weight.shape[1] == weight.shape[0] * weight.shape[2],
                 lambda: "linear_weight.shape[1] must equal n_features * d_embedding")
    torch._check(linear_weight.dtype == torch.bfloat16, lambda: "linear_weight must be bfloat16")
    torch._check(output_dtype in (torch.float32, torch.bfloat16), lambda: "output_dtype must be float32 or bfloat16")
    torch._check(compute_dtype in (torch.float32, torch.bfloat16), lambda: "compute_dtype must be float32 or bfloat16")
    return torch.empty((x.shape[0], linear_weight.shape[0]), dtype=output_dtype, device=x.device)
