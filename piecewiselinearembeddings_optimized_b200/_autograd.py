"""Autograd registration for the ``rtdl_num_embeddings_cuda`` ops.

``forward`` keeps the reference contract (``_autograd.py:9-96``): it saves
the inputs and the bin indices, marks ``bin_indices`` non-differentiable,
does not materialise missing gradients, and calls ``backward`` only for the
gradients that are needed.  ``embeddings_forward`` (the fused module path)
calls ``embeddings_backward``, which finds the bins again and returns every
gradient of the fused forward (x, weight, bias or linear0) in one pass over
``grad_output``.  ``embeddings_linear_forward`` (the module fused into its
consumer's first Linear) differentiates as ``linear(flatten(module(x)))`` under
autocast: the linear's gradients by two bf16 matmuls (the weight gradient
against the embeddings recomputed by ``embeddings_forward``), the module's by
``embeddings_backward`` on ``grad_z @ linear_weight``.
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

# ---------------------------------------------------------------- module fused into a consumer Linear


def _setup_embeddings_linear_context(ctx: Any, inputs, output) -> None:
    (x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue, activation, compute_dtype,
     linear_weight, linear_bias, _output_dtype) = inputs
    ctx.save_for_backward(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, linear_weight)
    ctx.epilogue = int(epilogue)
    ctx.activation = bool(activation)
    ctx.compute_dtype = compute_dtype
    ctx.has_linear_bias = linear_bias is not None
    ctx.set_materialize_grads(False)


def _embeddings_linear_backward(ctx: Any, grad_output):
    out = [None] * 14
    if grad_output is None:
        return tuple(out)
    x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, linear_weight = ctx.saved_tensors
    need = ctx.needs_input_grad
    ops = torch.ops.rtdl_num_embeddings_cuda
    n = x.shape[0]
    gz = grad_output.contiguous()
    if ctx.has_linear_bias and need[12]:
        out[12] = gz.float().sum(0)
    if need[11]:
        emb = ops.embeddings_forward(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, ctx.epilogue,
                                     ctx.activation, ctx.compute_dtype, torch.bfloat16)
        out[11] = torch.mm(gz.to(torch.bfloat16).t(), emb.view(n, -1))
    if need[0] or need[4] or need[5] or need[6] or need[7]:
        if ctx.compute_dtype == torch.bfloat16:
            g = torch.mm(gz.to(torch.bfloat16), linear_weight)
        else:
            g = torch.mm(gz.float(), linear_weight.float())
        g = g.view(n, weight.shape[0], weight.shape[2])
        gx, gw, gb, gw0, gb0 = ops.embeddings_backward(
            g, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, None, ctx.epilogue, ctx.activation,
            ctx.compute_dtype, bool(need[0]), bool(need[4]), bool(need[5]), bool(need[6] or need[7]),
        )
        out[0] = gx if need[0] else None
        out[4] = gw if need[4] else None
        out[5] = gb if need[5] else None
        out[6] = gw0 if need[6] else None
        out[7] = gb0 if need[7] else None
    return tuple(out)


torch.library.register_autograd(
    "rtdl_num_embeddings_cuda::embeddings_linear_forward", _embeddings_linear_backward,
    setup_context=_setup_embeddings_linear_context,
)
