// ops.cpp - torch op registration for rtdl_num_embeddings_cuda (the only
// torch-facing layer).  Validates like the reference (TORCH_CHECK with the
// same conditions), allocates outputs and the backward workspace from the
// ATen caching allocator on the input's device, and calls the C ABI of
// libple_b200.so on the current CUDA stream.
//
// Schemas kept verbatim from the reference (ops.cpp:35-58):
//   forward(x, bin_edges, inv_bin_widths, n_bins, weight, output_dtype) -> (output, bin_indices)
//   backward(grad_output, x, bin_edges, inv_bin_widths, n_bins, weight, bin_indices,
//            compute_grad_x, compute_grad_weight) -> (grad_x, grad_weight)
// Added (the fused module path):
//   embeddings_forward / embeddings_backward.
// Added (the standalone encoding, upstream PiecewiseLinearEncoding):
//   encoding_forward / encoding_backward.
// Added (the module fused into its consumer's first Linear layer):
//   embeddings_linear_forward.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>
#include <tuple>

#include "ple_capi.h"

namespace {

int to_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return PLE_DTYPE_F32;
    case at::kHalf: return PLE_DTYPE_F16;
    case at::kBFloat16: return PLE_DTYPE_BF16;
    case at::kByte: return PLE_DTYPE_U8;
    case at::kShort: return PLE_DTYPE_I16;
    case at::kInt: return PLE_DTYPE_I32;
    default: return -1;
  }
}

at::ScalarType bin_index_dtype(int64_t max_n_bins) {
  return max_n_bins <= 256 ? at::kByte : (max_n_bins <= 32768 ? at::kShort : at::kInt);
}

void check_status(int st, const char* what) {
  TORCH_CHECK(st == PLE_OK, what, " failed: ", ple_status_string(st), ": ", ple_last_error_message());
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

void check_tables(const at::Tensor& x, const at::Tensor& bin_edges, const at::Tensor& inv_bin_widths,
                  const at::Tensor& n_bins, const at::Tensor& weight) {
  TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor");
  TORCH_CHECK(bin_edges.is_cuda(), "bin_edges must be a CUDA tensor");
  TORCH_CHECK(inv_bin_widths.is_cuda(), "inv_bin_widths must be a CUDA tensor");
  TORCH_CHECK(n_bins.is_cuda(), "n_bins must be a CUDA tensor");
  TORCH_CHECK(weight.is_cuda(), "weight must be a CUDA tensor");
  TORCH_CHECK(x.device() == bin_edges.device() && x.device() == inv_bin_widths.device() &&
                  x.device() == n_bins.device() && x.device() == weight.device(),
              "All forward tensors must be on the same CUDA device");
  TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
  TORCH_CHECK(bin_edges.is_contiguous(), "bin_edges must be contiguous");
  TORCH_CHECK(inv_bin_widths.is_contiguous(), "inv_bin_widths must be contiguous");
  TORCH_CHECK(n_bins.is_contiguous(), "n_bins must be contiguous");
  TORCH_CHECK(weight.is_contiguous(), "weight must be contiguous");
  TORCH_CHECK(x.dim() == 2, "x must have shape [N, F]");
  TORCH_CHECK(bin_edges.dim() == 2, "bin_edges must have shape [F, B + 1]");
  TORCH_CHECK(inv_bin_widths.dim() == 2, "inv_bin_widths must have shape [F, B]");
  TORCH_CHECK(n_bins.dim() == 1, "n_bins must have shape [F]");
  TORCH_CHECK(weight.dim() == 3, "weight must have shape [F, B, D]");
  TORCH_CHECK(x.scalar_type() == at::kFloat, "x must be float32");
  TORCH_CHECK(bin_edges.scalar_type() == at::kFloat, "bin_edges must be float32");
  TORCH_CHECK(inv_bin_widths.scalar_type() == at::kFloat, "inv_bin_widths must be float32");
  TORCH_CHECK(n_bins.scalar_type() == at::kInt, "n_bins must be int32");
  TORCH_CHECK(weight.scalar_type() == at::kFloat, "weight parameters must be float32");
  const int64_t F = x.size(1), B = weight.size(1);
  TORCH_CHECK(F > 0, "n_features must be positive");
  TORCH_CHECK(B > 0, "max_n_bins must be positive");
  TORCH_CHECK(weight.size(2) > 0, "d_embedding must be positive");
  TORCH_CHECK(weight.size(0) == F, "weight.size(0) must equal x.size(1)");
  TORCH_CHECK(bin_edges.size(0) == F, "bin_edges.size(0) must equal x.size(1)");
  TORCH_CHECK(bin_edges.size(1) == B + 1, "bin_edges.size(1) must equal max_n_bins + 1");
  TORCH_CHECK(inv_bin_widths.size(0) == F, "inv_bin_widths.size(0) must equal x.size(1)");
  TORCH_CHECK(inv_bin_widths.size(1) == B, "inv_bin_widths.size(1) must equal max_n_bins");
  TORCH_CHECK(n_bins.size(0) == F, "n_bins.size(0) must equal x.size(1)");
}

void check_param(const std::optional<at::Tensor>& p, const at::Tensor& weight, const char* name) {
  if (!p.has_value()) return;
  TORCH_CHECK(p->is_cuda() && p->device() == weight.device(), name, " must be on the weight's CUDA device");
  TORCH_CHECK(p->scalar_type() == at::kFloat, name, " must be float32");
  TORCH_CHECK(p->is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(p->dim() == 2 && p->size(0) == weight.size(0) && p->size(1) == weight.size(2), name,
              " must have shape [F, D]");
}

const float* ptr_or_null(const std::optional<at::Tensor>& p) {
  return p.has_value() ? p->data_ptr<float>() : nullptr;
}

std::tuple<at::Tensor, at::Tensor> ple_forward_op(const at::Tensor& x, const at::Tensor& bin_edges,
                                                  const at::Tensor& inv_bin_widths, const at::Tensor& n_bins,
                                                  const at::Tensor& weight, at::ScalarType output_dtype) {
  check_tables(x, bin_edges, inv_bin_widths, n_bins, weight);
  TORCH_CHECK(output_dtype == at::kFloat || output_dtype == at::kHalf || output_dtype == at::kBFloat16,
              "output_dtype must be float32, float16, or bfloat16");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  at::Tensor out = at::empty({N, F, D}, weight.options().dtype(output_dtype));
  const at::ScalarType idx_t = bin_index_dtype(B);
  at::Tensor idx = at::empty({N, F}, weight.options().dtype(idx_t));
  if (out.numel() == 0) return {out, idx};
  check_status(ple_forward(x.data_ptr<float>(), bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                           n_bins.data_ptr<int32_t>(), weight.data_ptr<float>(), N, F, B, D,
                           to_code(output_dtype), out.data_ptr(), to_code(idx_t), idx.data_ptr(),
                           stream_of(x)),
               "rtdl_num_embeddings_cuda::forward");
  return {out, idx};
}

at::Tensor workspace_for(const at::Tensor& like, int64_t N, int64_t F, int64_t B, int64_t D) {
  const size_t bytes = ple_backward_workspace_size(N, F, B, D);
  return at::empty({(int64_t)bytes}, like.options().dtype(at::kByte));
}

// The backward kernels hold one D row in at most one warp (D / vec <= 32 lanes with vec | D), so the
// C ABI refuses an odd d_embedding above 32, which the reference's module accepts (D <= 64).  The
// ops below serve those shapes by appending one zero column to grad_output, weight and the epilogue
// parameters: with W, bias, w0, b0 and g' all zero there, the column adds exactly +0 to grad_x and
// leaves every other column's gradients unchanged; its own gradients are dropped.
bool backward_needs_even_d(int64_t B, int64_t D) { return (D & 1) != 0 && D > 32 && B <= 256; }

at::Tensor pad_d(const at::Tensor& t) { return at::constant_pad_nd(t, {0, 1}, 0).contiguous(); }

std::optional<at::Tensor> pad_d(const std::optional<at::Tensor>& t) {
  if (!t.has_value()) return t;
  return pad_d(*t);
}

at::Tensor drop_pad_d(const at::Tensor& t, int64_t D) {
  return t.numel() == 0 ? t : t.narrow(t.dim() - 1, 0, D).contiguous();
}

std::tuple<at::Tensor, at::Tensor> ple_backward_op(const at::Tensor& grad_output, const at::Tensor& x,
                                                   const at::Tensor& bin_edges, const at::Tensor& inv_bin_widths,
                                                   const at::Tensor& n_bins, const at::Tensor& weight,
                                                   const at::Tensor& bin_indices, bool compute_grad_x,
                                                   bool compute_grad_weight) {
  TORCH_CHECK(grad_output.is_cuda(), "grad_output must be CUDA");
  TORCH_CHECK(bin_indices.is_cuda(), "bin_indices must be CUDA");
  check_tables(x, bin_edges, inv_bin_widths, n_bins, weight);
  TORCH_CHECK(grad_output.device() == x.device() && bin_indices.device() == x.device(),
              "All backward tensors must be on the same CUDA device");
  TORCH_CHECK(grad_output.is_contiguous(), "grad_output must be contiguous");
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  TORCH_CHECK(grad_output.scalar_type() == at::kFloat || grad_output.scalar_type() == at::kHalf ||
                  grad_output.scalar_type() == at::kBFloat16,
              "grad_output must be float32, float16, or bfloat16");
  TORCH_CHECK(bin_indices.scalar_type() == bin_index_dtype(B), "bin_indices has an invalid dtype");
  TORCH_CHECK(grad_output.dim() == 3 && grad_output.size(0) == N && grad_output.size(1) == F &&
                  grad_output.size(2) == D,
              "grad_output shape must be [N, F, D]");
  TORCH_CHECK(bin_indices.dim() == 2 && bin_indices.size(0) == N && bin_indices.size(1) == F,
              "bin_indices shape must be [N, F]");
  c10::cuda::CUDAGuard guard(x.device());
  if (backward_needs_even_d(B, D) && N > 0 && (compute_grad_x || compute_grad_weight)) {
    auto r = ple_backward_op(pad_d(grad_output), x, bin_edges, inv_bin_widths, n_bins, pad_d(weight), bin_indices,
                             compute_grad_x, compute_grad_weight);
    return {std::get<0>(r), drop_pad_d(std::get<1>(r), D)};
  }
  at::Tensor grad_x = compute_grad_x ? at::empty_like(x) : at::empty({0}, x.options());
  at::Tensor grad_w = compute_grad_weight ? at::empty_like(weight) : at::empty({0}, weight.options());
  if (!compute_grad_x && !compute_grad_weight) return {grad_x, grad_w};
  at::Tensor ws = workspace_for(x, N, F, B, D);
  check_status(ple_backward(grad_output.data_ptr(), to_code(grad_output.scalar_type()), x.data_ptr<float>(),
                            bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                            n_bins.data_ptr<int32_t>(), weight.data_ptr<float>(), bin_indices.data_ptr(),
                            to_code(bin_indices.scalar_type()), N, F, B, D,
                            compute_grad_x ? grad_x.data_ptr<float>() : nullptr,
                            compute_grad_weight ? grad_w.data_ptr<float>() : nullptr, ws.data_ptr(),
                            (size_t)ws.numel(), stream_of(x)),
               "rtdl_num_embeddings_cuda::backward");
  return {grad_x, grad_w};
}

// max_n_bins above 256: the C ABI serves only the bare x_ple op there (ple_wide.cu), so the module's
// epilogue runs as ATen ops around it, in the module's order and types (module.py:230-248): x_ple in
// the compute type, then + bias, ReLU and + linear0 in fp32; the x_ple branch of the backward gets
// q(g' * mask) in the compute type (_autograd.py:68-80), the parameter gradients are fp32 sums.
at::Tensor wide_pre_activation(const at::Tensor& x, const at::Tensor& bin_edges, const at::Tensor& inv_bin_widths,
                               const at::Tensor& n_bins, const at::Tensor& weight,
                               const std::optional<at::Tensor>& bias, int64_t epilogue,
                               at::ScalarType compute_dtype) {
  at::Tensor z = std::get<0>(ple_forward_op(x, bin_edges, inv_bin_widths, n_bins, weight, compute_dtype))
                     .to(at::kFloat);
  if (epilogue == PLE_EPILOGUE_A) {
    TORCH_CHECK(bias.has_value(), "epilogue A needs bias");
    z = z + *bias;
  }
  return z;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> wide_embeddings_backward(
    const at::Tensor& grad_output, const at::Tensor& x, const at::Tensor& bin_edges,
    const at::Tensor& inv_bin_widths, const at::Tensor& n_bins, const at::Tensor& weight,
    const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& w0,
    const std::optional<at::Tensor>& b0, int64_t epilogue, bool activation, at::ScalarType compute_dtype,
    bool compute_grad_x, bool compute_grad_weight, bool want_bias, bool want_l0) {
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  auto opt = weight.options();
  at::Tensor g32 = grad_output.to(at::kFloat);
  at::Tensor gm = g32;
  if (activation) {
    at::Tensor z = wide_pre_activation(x, bin_edges, inv_bin_widths, n_bins, weight, bias, epilogue, compute_dtype);
    gm = g32.masked_fill(z <= 0, 0.0);  // threshold_backward: NaN inputs pass the gradient
  }
  at::Tensor gx = compute_grad_x ? at::empty_like(x) : at::empty({0}, x.options());
  at::Tensor gw = compute_grad_weight ? at::empty_like(weight) : at::empty({0}, opt);
  if (compute_grad_x || compute_grad_weight) {
    at::Tensor gq = gm.to(compute_dtype).contiguous();
    at::Tensor ws = workspace_for(x, N, F, B, D);
    check_status(ple_backward(gq.data_ptr(), to_code(compute_dtype), x.data_ptr<float>(),
                              bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                              n_bins.data_ptr<int32_t>(), weight.data_ptr<float>(), nullptr, PLE_DTYPE_I32, N, F,
                              B, D, compute_grad_x ? gx.data_ptr<float>() : nullptr,
                              compute_grad_weight ? gw.data_ptr<float>() : nullptr, ws.data_ptr(),
                              (size_t)ws.numel(), stream_of(x)),
                 "rtdl_num_embeddings_cuda::embeddings_backward");
  }
  at::Tensor gb = want_bias ? gm.sum(0) : at::empty({0}, opt);
  at::Tensor gw0 = want_l0 ? (g32 * x.unsqueeze(-1)).sum(0) : at::empty({0}, opt);
  at::Tensor gb0 = want_l0 ? g32.sum(0) : at::empty({0}, opt);
  if (compute_grad_x && epilogue == PLE_EPILOGUE_B) {
    TORCH_CHECK(w0.has_value(), "epilogue B needs w0");
    gx.add_((g32 * *w0).sum(-1));
  }
  return {gx, gw, gb.contiguous(), gw0.contiguous(), gb0.contiguous()};
}

at::Tensor ple_embeddings_forward_op(const at::Tensor& x, const at::Tensor& bin_edges,
                                     const at::Tensor& inv_bin_widths, const at::Tensor& n_bins,
                                     const at::Tensor& weight, const std::optional<at::Tensor>& bias,
                                     const std::optional<at::Tensor>& w0, const std::optional<at::Tensor>& b0,
                                     int64_t epilogue, bool activation, at::ScalarType compute_dtype,
                                     at::ScalarType output_dtype) {
  check_tables(x, bin_edges, inv_bin_widths, n_bins, weight);
  check_param(bias, weight, "bias");
  check_param(w0, weight, "w0");
  check_param(b0, weight, "b0");
  TORCH_CHECK(to_code(output_dtype) >= 0 && to_code(output_dtype) <= PLE_DTYPE_BF16,
              "output_dtype must be float32, float16, or bfloat16");
  TORCH_CHECK(to_code(compute_dtype) >= 0 && to_code(compute_dtype) <= PLE_DTYPE_BF16,
              "compute_dtype must be float32, float16, or bfloat16");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  if (B > 256) {
    at::Tensor z = wide_pre_activation(x, bin_edges, inv_bin_widths, n_bins, weight, bias, epilogue, compute_dtype);
    at::Tensor y = activation ? at::relu(z) : z;
    if (epilogue == PLE_EPILOGUE_B) {
      TORCH_CHECK(w0.has_value() && b0.has_value(), "epilogue B needs w0 and b0");
      y = at::addcmul(*b0, x.unsqueeze(-1), *w0) + y;
    }
    return y.to(output_dtype).contiguous();
  }
  at::Tensor out = at::empty({N, F, D}, weight.options().dtype(output_dtype));
  if (out.numel() == 0) return out;
  // bin indices are not requested: the fused backward finds the bins itself, which costs less than
  // writing and re-reading a byte per (sample, feature)
  check_status(ple_embeddings_forward(x.data_ptr<float>(), bin_edges.data_ptr<float>(),
                                      inv_bin_widths.data_ptr<float>(), n_bins.data_ptr<int32_t>(),
                                      weight.data_ptr<float>(), ptr_or_null(bias), ptr_or_null(w0),
                                      ptr_or_null(b0), (int)epilogue, activation ? 1 : 0,
                                      to_code(compute_dtype), N, F, B, D, to_code(output_dtype), out.data_ptr(),
                                      PLE_DTYPE_U8, nullptr, stream_of(x)),
               "rtdl_num_embeddings_cuda::embeddings_forward");
  return out;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> ple_embeddings_backward_op(
    const at::Tensor& grad_output, const at::Tensor& x, const at::Tensor& bin_edges,
    const at::Tensor& inv_bin_widths, const at::Tensor& n_bins, const at::Tensor& weight,
    const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& w0,
    const std::optional<at::Tensor>& b0, const std::optional<at::Tensor>& bin_indices, int64_t epilogue,
    bool activation, at::ScalarType compute_dtype, bool compute_grad_x, bool compute_grad_weight,
    bool compute_grad_bias, bool compute_grad_linear0) {
  check_tables(x, bin_edges, inv_bin_widths, n_bins, weight);
  check_param(bias, weight, "bias");
  check_param(w0, weight, "w0");
  check_param(b0, weight, "b0");
  TORCH_CHECK(grad_output.is_cuda() && grad_output.device() == x.device(),
              "grad_output must be on x's CUDA device");
  TORCH_CHECK(grad_output.is_contiguous(), "grad_output must be contiguous");
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  TORCH_CHECK(grad_output.dim() == 3 && grad_output.size(0) == N && grad_output.size(1) == F &&
                  grad_output.size(2) == D,
              "grad_output shape must be [N, F, D]");
  TORCH_CHECK(to_code(grad_output.scalar_type()) >= 0 && to_code(grad_output.scalar_type()) <= PLE_DTYPE_BF16,
              "grad_output must be float32, float16, or bfloat16");
  if (bin_indices.has_value()) {
    TORCH_CHECK(bin_indices->is_cuda() && bin_indices->device() == x.device(), "bin_indices must be on x's device");
    TORCH_CHECK(bin_indices->is_contiguous(), "bin_indices must be contiguous");
    TORCH_CHECK(bin_indices->scalar_type() == bin_index_dtype(B), "bin_indices has an invalid dtype");
    TORCH_CHECK(bin_indices->dim() == 2 && bin_indices->size(0) == N && bin_indices->size(1) == F,
                "bin_indices shape must be [N, F]");
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto opt = weight.options();
  const bool want_bias = compute_grad_bias && epilogue == PLE_EPILOGUE_A;
  const bool want_l0 = compute_grad_linear0 && epilogue == PLE_EPILOGUE_B;
  if (B > 256)
    return wide_embeddings_backward(grad_output, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue,
                                    activation, compute_dtype, compute_grad_x, compute_grad_weight, want_bias, want_l0);
  if (backward_needs_even_d(B, D) && N > 0 && (compute_grad_x || compute_grad_weight || want_bias || want_l0)) {
    auto r = ple_embeddings_backward_op(pad_d(grad_output), x, bin_edges, inv_bin_widths, n_bins, pad_d(weight),
                                        pad_d(bias), pad_d(w0), pad_d(b0), bin_indices, epilogue, activation,
                                        compute_dtype, compute_grad_x, compute_grad_weight, compute_grad_bias,
                                        compute_grad_linear0);
    return {std::get<0>(r), drop_pad_d(std::get<1>(r), D), drop_pad_d(std::get<2>(r), D),
            drop_pad_d(std::get<3>(r), D), drop_pad_d(std::get<4>(r), D)};
  }
  at::Tensor gx = compute_grad_x ? at::empty_like(x) : at::empty({0}, x.options());
  at::Tensor gw = compute_grad_weight ? at::empty_like(weight) : at::empty({0}, opt);
  at::Tensor gb = want_bias ? at::empty({F, D}, opt) : at::empty({0}, opt);
  at::Tensor gw0 = want_l0 ? at::empty({F, D}, opt) : at::empty({0}, opt);
  at::Tensor gb0 = want_l0 ? at::empty({F, D}, opt) : at::empty({0}, opt);
  if (!compute_grad_x && !compute_grad_weight && !want_bias && !want_l0) return {gx, gw, gb, gw0, gb0};
  at::Tensor ws = workspace_for(x, N, F, B, D);
  check_status(ple_embeddings_backward(
                   grad_output.data_ptr(), to_code(grad_output.scalar_type()), x.data_ptr<float>(),
                   bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(), n_bins.data_ptr<int32_t>(),
                   weight.data_ptr<float>(), ptr_or_null(bias), ptr_or_null(w0), ptr_or_null(b0), (int)epilogue,
                   activation ? 1 : 0, to_code(compute_dtype), N, F, B, D,
                   bin_indices.has_value() ? bin_indices->data_ptr() : nullptr,
                   bin_indices.has_value() ? to_code(bin_indices->scalar_type()) : PLE_DTYPE_U8,
                   compute_grad_x ? gx.data_ptr<float>() : nullptr,
                   compute_grad_weight ? gw.data_ptr<float>() : nullptr, want_bias ? gb.data_ptr<float>() : nullptr,
                   want_l0 ? gw0.data_ptr<float>() : nullptr, want_l0 ? gb0.data_ptr<float>() : nullptr,
                   ws.data_ptr(), (size_t)ws.numel(), stream_of(x)),
               "rtdl_num_embeddings_cuda::embeddings_backward");
  return {gx, gw, gb, gw0, gb0};
}

at::Tensor ple_embeddings_linear_forward_op(const at::Tensor& x, const at::Tensor& bin_edges,
                                            const at::Tensor& inv_bin_widths, const at::Tensor& n_bins,
                                            const at::Tensor& weight, const std::optional<at::Tensor>& bias,
                                            const std::optional<at::Tensor>& w0,
                                            const std::optional<at::Tensor>& b0, int64_t epilogue, bool activation,
                                            at::ScalarType compute_dtype, const at::Tensor& linear_weight,
                                            const std::optional<at::Tensor>& linear_bias,
                                            at::ScalarType output_dtype) {
  check_tables(x, bin_edges, inv_bin_widths, n_bins, weight);
  check_param(bias, weight, "bias");
  check_param(w0, weight, "w0");
  check_param(b0, weight, "b0");
  const int64_t N = x.size(0), F = x.size(1), B = weight.size(1), D = weight.size(2);
  TORCH_CHECK(linear_weight.is_cuda() && linear_weight.device() == x.device(),
              "linear_weight must be on x's CUDA device");
  TORCH_CHECK(linear_weight.scalar_type() == at::kBFloat16, "linear_weight must be bfloat16");
  TORCH_CHECK(linear_weight.dim() == 2 && linear_weight.size(1) == F * D,
              "linear_weight must have shape [out_features, n_features * d_embedding]");
  TORCH_CHECK(linear_weight.is_contiguous(), "linear_weight must be contiguous");
  const int64_t H = linear_weight.size(0);
  if (linear_bias.has_value()) {
    TORCH_CHECK(linear_bias->is_cuda() && linear_bias->device() == x.device(), "linear_bias must be on x's device");
    TORCH_CHECK(linear_bias->scalar_type() == at::kFloat, "linear_bias must be float32");
    TORCH_CHECK(linear_bias->dim() == 1 && linear_bias->size(0) == H, "linear_bias must have shape [out_features]");
    TORCH_CHECK(linear_bias->is_contiguous(), "linear_bias must be contiguous");
  }
  TORCH_CHECK(output_dtype == at::kFloat || output_dtype == at::kBFloat16,
              "output_dtype must be float32 or bfloat16");
  TORCH_CHECK(compute_dtype == at::kFloat || compute_dtype == at::kBFloat16,
              "compute_dtype must be float32 or bfloat16");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty({N, H}, x.options().dtype(output_dtype));
  if (N == 0) return out;
  const size_t need = ple_embeddings_linear_workspace_size(F, B, D, H, to_code(compute_dtype));
  TORCH_CHECK(need > 0, "rtdl_num_embeddings_cuda::embeddings_linear_forward: unsupported shape (d_embedding must "
              "be a multiple of 8)");
  at::Tensor ws = at::empty({(int64_t)need + 256}, x.options().dtype(at::kByte));
  void* wp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~(uintptr_t)255);
  check_status(ple_embeddings_linear_forward(
                   x.data_ptr<float>(), bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                   n_bins.data_ptr<int32_t>(), weight.data_ptr<float>(), ptr_or_null(bias), ptr_or_null(w0),
                   ptr_or_null(b0), (int)epilogue, activation ? 1 : 0, to_code(compute_dtype), N, F, B, D,
                   linear_weight.data_ptr(), PLE_DTYPE_BF16,
                   linear_bias.has_value() ? linear_bias->data_ptr<float>() : nullptr, H, to_code(output_dtype),
                   out.data_ptr(), wp, need, stream_of(x)),
               "rtdl_num_embeddings_cuda::embeddings_linear_forward");
  return out;
}

void check_encoding(const at::Tensor& x, const at::Tensor& bin_edges, const at::Tensor& inv_bin_widths,
                    const at::Tensor& n_bins, const std::optional<at::Tensor>& col_offsets, int64_t layout,
                    int64_t total_bins) {
  TORCH_CHECK(x.is_cuda() && bin_edges.is_cuda() && inv_bin_widths.is_cuda() && n_bins.is_cuda(),
              "encoding tensors must be CUDA tensors");
  TORCH_CHECK(x.device() == bin_edges.device() && x.device() == inv_bin_widths.device() &&
                  x.device() == n_bins.device(),
              "All encoding tensors must be on the same CUDA device");
  TORCH_CHECK(x.dim() == 2, "x must have shape [N, F]");
  TORCH_CHECK(x.scalar_type() == at::kFloat, "x must be float32");
  TORCH_CHECK(x.is_contiguous() && bin_edges.is_contiguous() && inv_bin_widths.is_contiguous() &&
                  n_bins.is_contiguous(),
              "encoding tensors must be contiguous");
  TORCH_CHECK(bin_edges.dim() == 2 && bin_edges.scalar_type() == at::kFloat, "bin_edges must be float32 [F, B + 1]");
  TORCH_CHECK(inv_bin_widths.dim() == 2 && inv_bin_widths.scalar_type() == at::kFloat,
              "inv_bin_widths must be float32 [F, B]");
  TORCH_CHECK(n_bins.dim() == 1 && n_bins.scalar_type() == at::kInt, "n_bins must be int32 [F]");
  const int64_t F = x.size(1), B = inv_bin_widths.size(1);
  TORCH_CHECK(bin_edges.size(0) == F && inv_bin_widths.size(0) == F && n_bins.size(0) == F,
              "bin tables must have n_features rows");
  TORCH_CHECK(bin_edges.size(1) == B + 1, "bin_edges.size(1) must equal inv_bin_widths.size(1) + 1");
  TORCH_CHECK(layout == PLE_ENC_RAGGED || layout == PLE_ENC_PADDED, "layout must be 0 (ragged) or 1 (padded)");
  if (layout == PLE_ENC_RAGGED) {
    TORCH_CHECK(col_offsets.has_value(), "the ragged layout needs col_offsets");
    TORCH_CHECK(col_offsets->is_cuda() && col_offsets->device() == x.device(), "col_offsets must be on x's device");
    TORCH_CHECK(col_offsets->scalar_type() == at::kLong && col_offsets->dim() == 1 && col_offsets->size(0) == F + 1 &&
                    col_offsets->is_contiguous(),
                "col_offsets must be a contiguous int64 tensor of shape [F + 1]");
  } else {
    TORCH_CHECK(total_bins == F * B, "the padded layout has n_features * max_n_bins columns");
  }
}

at::Tensor ple_encoding_forward_op(const at::Tensor& x, const at::Tensor& bin_edges, const at::Tensor& inv_bin_widths,
                                   const at::Tensor& n_bins, const std::optional<at::Tensor>& col_offsets,
                                   int64_t layout, int64_t total_bins, at::ScalarType output_dtype) {
  check_encoding(x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout, total_bins);
  TORCH_CHECK(to_code(output_dtype) >= 0 && to_code(output_dtype) <= PLE_DTYPE_BF16,
              "output_dtype must be float32, float16, or bfloat16");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), F = x.size(1), B = inv_bin_widths.size(1);
  at::Tensor out = layout == PLE_ENC_PADDED ? at::empty({N, F, B}, x.options().dtype(output_dtype))
                                            : at::empty({N, total_bins}, x.options().dtype(output_dtype));
  if (N == 0) return out;
  check_status(ple_encoding_forward(x.data_ptr<float>(), bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                                    n_bins.data_ptr<int32_t>(),
                                    col_offsets.has_value() ? col_offsets->data_ptr<int64_t>() : nullptr, (int)layout,
                                    N, F, B, total_bins, to_code(output_dtype), out.data_ptr(), stream_of(x)),
               "rtdl_num_embeddings_cuda::encoding_forward");
  return out;
}

at::Tensor ple_encoding_backward_op(const at::Tensor& grad_output, const at::Tensor& x, const at::Tensor& bin_edges,
                                    const at::Tensor& inv_bin_widths, const at::Tensor& n_bins,
                                    const std::optional<at::Tensor>& col_offsets, int64_t layout, int64_t total_bins) {
  check_encoding(x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout, total_bins);
  TORCH_CHECK(grad_output.is_cuda() && grad_output.device() == x.device(), "grad_output must be on x's device");
  TORCH_CHECK(grad_output.is_contiguous(), "grad_output must be contiguous");
  TORCH_CHECK(to_code(grad_output.scalar_type()) >= 0 && to_code(grad_output.scalar_type()) <= PLE_DTYPE_BF16,
              "grad_output must be float32, float16, or bfloat16");
  const int64_t N = x.size(0), F = x.size(1), B = inv_bin_widths.size(1);
  TORCH_CHECK(grad_output.numel() == N * total_bins && grad_output.size(0) == N,
              "grad_output must have the encoding's shape");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor grad_x = at::empty({N, F}, x.options());
  if (N == 0) return grad_x;
  check_status(ple_encoding_backward(grad_output.data_ptr(), to_code(grad_output.scalar_type()), x.data_ptr<float>(),
                                     bin_edges.data_ptr<float>(), inv_bin_widths.data_ptr<float>(),
                                     n_bins.data_ptr<int32_t>(),
                                     col_offsets.has_value() ? col_offsets->data_ptr<int64_t>() : nullptr,
                                     (int)layout, N, F, B, total_bins, grad_x.data_ptr<float>(), stream_of(x)),
               "rtdl_num_embeddings_cuda::encoding_backward");
  return grad_x;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> ple_compute_bins_op(const at::Tensor& x, int64_t n_bins) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kFloat, "x must be a float32 CUDA tensor [N, F]");
  TORCH_CHECK(x.size(0) >= 2, "compute_bins needs at least two rows");
  TORCH_CHECK(n_bins >= 1 && n_bins <= 1023, "n_bins must lie in [1, 1023]");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), F = x.size(1);
  at::Tensor sorted = std::get<0>(at::sort(x.t().contiguous(), 1));  // [F, N], each column ascending
  at::Tensor edges = at::empty({F, n_bins + 1}, x.options());
  at::Tensor inv_w = at::empty({F, n_bins}, x.options());
  at::Tensor nb = at::empty({F}, x.options().dtype(at::kInt));
  check_status(ple_compute_bins(sorted.data_ptr<float>(), N, F, (int)n_bins, edges.data_ptr<float>(),
                                inv_w.data_ptr<float>(), nb.data_ptr<int32_t>(), stream_of(x)),
               "rtdl_num_embeddings_cuda::compute_bins");
  return {edges, inv_w, nb};
}

}  // namespace

TORCH_LIBRARY(rtdl_num_embeddings_cuda, m) {
  m.def(
      "forward(Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, Tensor weight, "
      "ScalarType output_dtype) -> (Tensor output, Tensor bin_indices)");
  m.def(
      "backward(Tensor grad_output, Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, "
      "Tensor weight, Tensor bin_indices, bool compute_grad_x, bool compute_grad_weight) -> "
      "(Tensor grad_x, Tensor grad_weight)");
  m.def(
      "embeddings_forward(Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, Tensor weight, "
      "Tensor? bias, Tensor? w0, Tensor? b0, int epilogue, bool activation, ScalarType compute_dtype, "
      "ScalarType output_dtype) -> Tensor");
  m.def(
      "embeddings_backward(Tensor grad_output, Tensor x, Tensor bin_edges, Tensor inv_bin_widths, "
      "Tensor n_bins, Tensor weight, Tensor? bias, Tensor? w0, Tensor? b0, Tensor? bin_indices, "
      "int epilogue, bool activation, ScalarType compute_dtype, bool compute_grad_x, bool compute_grad_weight, bool compute_grad_bias, "
      "bool compute_grad_linear0) -> (Tensor grad_x, Tensor grad_weight, Tensor grad_bias, Tensor grad_w0, "
      "Tensor grad_b0)");
  m.def(
      "encoding_forward(Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, Tensor? col_offsets, "
      "int layout, int total_bins, ScalarType output_dtype) -> Tensor");
  m.def(
      "encoding_backward(Tensor grad_output, Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, "
      "Tensor? col_offsets, int layout, int total_bins) -> Tensor");
  m.def("compute_bins(Tensor x, int n_bins) -> (Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins)");
  m.def(
      "embeddings_linear_forward(Tensor x, Tensor bin_edges, Tensor inv_bin_widths, Tensor n_bins, Tensor weight, "
      "Tensor? bias, Tensor? w0, Tensor? b0, int epilogue, bool activation, ScalarType compute_dtype, "
      "Tensor linear_weight, Tensor? linear_bias, ScalarType output_dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(rtdl_num_embeddings_cuda, CUDA, m) {
  m.impl("forward", &ple_forward_op);
  m.impl("backward", &ple_backward_op);
  m.impl("embeddings_forward", &ple_embeddings_forward_op);
  m.impl("embeddings_backward", &ple_embeddings_backward_op);
  m.impl("encoding_forward", &ple_encoding_forward_op);
  m.impl("encoding_backward", &ple_encoding_backward_op);
  m.impl("compute_bins", &ple_compute_bins_op);
  m.impl("embeddings_linear_forward", &ple_embeddings_linear_forward_op);
}
