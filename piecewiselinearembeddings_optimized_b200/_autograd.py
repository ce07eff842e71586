"""Autograd registration for the ``rtdl_num_embeddings_cuda`` ops.

``forward`` keeps the reference contract (``_autograd.py:9-96``): it saves
the inputs and the bin indices, marks ``bin_indices`` non-differentiable,
does not materialise missing gradients, and calls ``backward`` only for the
gradients that are needed.  ``embeddings_forward`` (the fused module path)
calls ``embeddings_backward``, which finds the bins again and returns every
gradient of the fused forward (x, weight, bias or linear0) in one pass over
``grad_output``.
Double backward is not implemented.
"""
from __future__ import annotations

from typing import Any

import torch

# ---------------------------------------------------------------- forward / backward


def _setup_forward_context(ctx: Any, inputs, output) -> None:
    x, bin_edges, inv_bin_widths, n_bins, weight, _output_dtype = inputs
    _x_ple, bin_indices = output
    ctx.save_for_backward(x, bin_edges, inv_bin_widths, n_bins, weight, bin_indices)
    ctx.mark_non_differentiable(bin_indices)
    ctx.set_materialize_grads(False)


def _forward_backward(ctx: Any, grad_output, _grad_bin_indices):
    if grad_output is None:
        return None, None, None, None, None, None
    x, bin_edges, inv_bin_widths, n_bins, weight, bin_indices = ctx.saved_tensors
    compute_grad_x = bool(ctx.needs_input_grad[0])
    compute_grad_weight = bool(ctx.needs_input_grad[4])
    grad_x, grad_weight = torch.ops.rtdl_num_embeddings_cuda.backward(
        grad_output.contiguous(), x, bin_edges, inv_bin_widths, n_bins, weight, bin_indices,
        compute_grad_x, compute_grad_weight,
    )
    return (
        grad_x if compute_grad_x else None, None, None, None,
        grad_weight if compute_grad_weight else None, None,
    )


torch.library.register_autograd(
    "rtdl_num_embeddings_cuda::forward", _forward_backward, setup_context=_setup_forward_context
)

# ---------------------------------------------------------------- fused embeddings


def _setup_embeddings_context(ctx: Any, inputs, output) -> None:
    (x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue, activation, compute_dtype,
     output_dtype) = inputs
    ctx.save_for_backward(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0)
    ctx.epilogue = int(epilogue)
    ctx.activation = bool(activation)
    ctx.compute_dtype = compute_dtype
    ctx.set_materialize_grads(False)


def _embeddings_backward(ctx: Any, grad_output):
    none = (None,) * 12
    if grad_output is None:
        return none
    x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0 = ctx.saved_tensors
    need = ctx.needs_input_grad
    g = grad_output.contiguous()
    if g.dtype != ctx.compute_dtype and g.dtype != torch.float32:
        g = g.float()
    gx, gw, gb, gw0, gb0 = torch.ops.rtdl_num_embeddings_cuda.embeddings_backward(
        g, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, None, ctx.epilogue, ctx.activation,
        ctx.compute_dtype, bool(need[0]), bool(need[4]), bool(need[5]), bool(need[6] or need[7]),
    )
    return (
        gx if need[0] else None, None, None, None,
        gw if need[4] else None,
        gb if need[5] else None,
        gw0 if need[6] else None,
        gb0 if need[7] else None,
        None, None, None, None,
    )


torch.library.register_autograd(
    "rtdl_num_embeddings_cuda::embeddings_forward", _embeddings_backward,
    setup_context=_setup_embeddings_context,
)

# ---------------------------------------------------------------- standalone encoding


def _setup_encoding_context(ctx: Any, inputs, output) -> None:
    x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout, total_bins, _output_dtype = inputs
    ctx.save_for_backward(x, bin_edges, inv_bin_widths, n_bins, col_offsets)
    ctx.layout = int(layout)
    ctx.total_bins = int(total_bins)
    ctx.set_materialize_grads(False)


def _encoding_backward(ctx: Any, grad_output):
    if grad_output is None or not ctx.needs_input_grad[0]:
        return (None,) * 8
    x, bin_edges, inv_bin_widths, n_bins, col_offsets = ctx.saved_tensors
    grad_x = torch.ops.rtdl_num_embeddings_cuda.encoding_backward(
        grad_output.contiguous(), x, bin_edges, inv_bin_widths, n_bins, col_offsets, ctx.layout, ctx.total_bins,
    )
    return (grad_x,) + (None,) * 7


torch.library.register_autograd(
    "rtdl_num_embeddings_cuda::encoding_forward", _encoding_backward, setup_context=_setup_encoding_context,
)
