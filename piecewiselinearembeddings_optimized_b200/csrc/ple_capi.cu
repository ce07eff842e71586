// ple_capi.cu - extern "C" entry points of libple_b200.so.
//
// Validation mirrors the reference's TORCH_CHECKs (forward_cuda.cu:695-790,
// backward_cuda.cu:1539-1657) as status codes; the torch adapter (ops.cpp)
// turns a non-zero status into a RuntimeError with ple_last_error_message().
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

static thread_local char g_msg[512] = "";

int set_error(int code, const char* msg) {
  snprintf(g_msg, sizeof(g_msg), "%s", msg);
  return code;
}

int set_cuda_error(cudaError_t e, const char* what) {
  snprintf(g_msg, sizeof(g_msg), "%s: %s", what, cudaGetErrorString(e));
  return PLE_ERR_CUDA;
}

namespace {
struct DevProps {
  int sms = 0;
  size_t smem_optin = 0;
};
constexpr int kMaxDevices = 64;
DevProps g_props[kMaxDevices];
std::once_flag g_once[kMaxDevices];

// Without a visible device (host-side size queries on a machine with no GPU) the
// properties of the B200 this library is built for: 148 SMs, 227 KiB of opt-in
// shared memory per block.
constexpr int kDefaultSms = 148;
constexpr size_t kDefaultSmemOptin = 232448;

const DevProps& props() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  std::call_once(g_once[dev], [dev] {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 0;
    g_props[dev].sms = v > 0 ? v : kDefaultSms;
    v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 0;
    g_props[dev].smem_optin = v > 0 ? (size_t)v : kDefaultSmemOptin;
  });
  return g_props[dev];
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int dtype_size(int dt) {
  switch (dt) {
    case PLE_DTYPE_F32: return 4;
    case PLE_DTYPE_F16: case PLE_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// max_bins: 256 for the main kernels; the bare x_ple ops also take wider features (ple_wide.cu).
int check_sizes(int64_t N, int64_t F, int64_t B, int64_t D, int64_t max_bins = 256) {
  if (N < 0) return set_error(PLE_ERR_SHAPE, "batch must be >= 0");
  if (F <= 0) return set_error(PLE_ERR_SHAPE, "n_features must be positive");
  if (B <= 0) return set_error(PLE_ERR_SHAPE, "max_n_bins must be positive");
  if (D <= 0) return set_error(PLE_ERR_SHAPE, "d_embedding must be positive");
  if (D > kMaxD) return set_error(PLE_ERR_UNSUPPORTED, "d_embedding must be <= 64");
  if (B > max_bins)
    return set_error(PLE_ERR_UNSUPPORTED, B > kWideMaxBins ? "max_n_bins above 2^20 is not supported"
                                                          : "max_n_bins > 256 needs the bare x_ple op (no epilogue, "
                                                            "no activation)");
  if (F > (int64_t)1 << 30) return set_error(PLE_ERR_OVERFLOW, "n_features too large");
  if (N > 0 && F > INT64_MAX / N / D) return set_error(PLE_ERR_OVERFLOW, "N * F * D overflows int64");
  return PLE_OK;
}

int check_tables(const float* edges, const float* inv_w, const int32_t* n_bins, const float* W) {
  if (!edges || !inv_w || !n_bins || !W)
    return set_error(PLE_ERR_INVALID_ARGUMENT, "bin_edges, inv_bin_widths, n_bins and weight are required");
  return PLE_OK;
}

// Widest vector width (elements) such that D is a multiple and every listed
// pointer is aligned for it.
int pick_vec(int64_t D, int max_vec, std::initializer_list<std::pair<const void*, int>> ptrs) {
  for (int v = max_vec; v > 1; v >>= 1) {
    if (D % v) continue;
    bool ok = true;
    for (auto& pe : ptrs)
      if (pe.first && !aligned(pe.first, (size_t)v * pe.second)) ok = false;
    if (ok) return v;
  }
  return 1;
}
}  // namespace

int device_sm_count() { return props().sms; }
size_t device_max_smem_optin() { return props().smem_optin; }

// ---------------------------------------------------------------- no-allocation backward
// The scratch lives in this module's static device memory; its device address
// is looked up with the device current and cached per device.  Only a
// successful lookup is cached: a call that failed (for example one made
// during a stream capture) leaves the slot empty and the next call retries.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PLE_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu[kMaxDevices];
void* g_scratch_ptr[kMaxDevices] = {};
}  // namespace

static int noalloc_scratch(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(PLE_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_scratch_mu[dev]);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGetSymbolAddress(no-allocation scratch)");
    if (p == nullptr) return set_error(PLE_ERR_CUDA, "cudaGetSymbolAddress(no-allocation scratch) returned null");
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return PLE_OK;
}

}  // namespace ple

using namespace ple;

extern "C" {

int ple_abi_version(void) { return PLE_ABI_VERSION; }

int ple_linear_status(void) { return linear_status(); }

const char* ple_status_string(int status) {
  switch (status) {
    case PLE_OK: return "ok";
    case PLE_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PLE_ERR_SHAPE: return "invalid shape";
    case PLE_ERR_OVERFLOW: return "size overflow";
    case PLE_ERR_UNSUPPORTED: return "unsupported configuration";
    case PLE_ERR_WORKSPACE: return "workspace missing or too small";
    case PLE_ERR_CUDA: return "CUDA error";
    case PLE_ERR_ALIGNMENT: return "misaligned pointer";
    default: return "unknown status";
  }
}

const char* ple_last_error_message(void) { return g_msg; }

static int forward_impl(const float* x, const float* edges, const float* inv_w, const int32_t* n_bins,
                        const float* W, const float* bias, const float* w0, const float* b0, int epi,
                        int relu, int compute_dtype, int64_t N, int64_t F, int64_t B, int64_t D,
                        int out_dtype, void* out, int bin_idx_dtype, void* bin_idx, void* stream) {
  g_msg[0] = 0;
  int st = check_sizes(N, F, B, D, epi == kEpiNone && !relu ? kWideMaxBins : 256);
  if (st) return st;
  if ((st = check_tables(edges, inv_w, n_bins, W))) return st;
  if (dtype_size(out_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "output dtype must be F32, F16 or BF16");
  if (dtype_size(compute_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "compute dtype must be F32, F16 or BF16");
  if (epi != kEpiNone && epi != kEpiA && epi != kEpiB) return set_error(PLE_ERR_INVALID_ARGUMENT, "bad epilogue");
  if (epi == kEpiA && !bias) return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue A needs bias");
  if (epi == kEpiB && (!w0 || !b0)) return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue B needs w0 and b0");
  int idx_bytes = 0;
  if (bin_idx) {
    switch (bin_idx_dtype) {
      case PLE_DTYPE_U8: idx_bytes = 1; break;
      case PLE_DTYPE_I16: idx_bytes = 2; break;
      case PLE_DTYPE_I32: idx_bytes = 4; break;
      default: return set_error(PLE_ERR_INVALID_ARGUMENT, "bin index dtype must be U8, I16 or I32");
    }
    if (idx_bytes == 1 && B > 256) return set_error(PLE_ERR_INVALID_ARGUMENT, "U8 bin indices need max_n_bins <= 256");
  }
  if (N == 0) return PLE_OK;
  if (!x || !out) return set_error(PLE_ERR_INVALID_ARGUMENT, "x and output are required");
  FwdArgs a{};
  a.x = x; a.edges = edges; a.inv_w = inv_w; a.n_bins = n_bins; a.W = W;
  a.bias = bias; a.w0 = w0; a.b0 = b0; a.out = out; a.bin_idx = bin_idx; a.bin_idx_bytes = idx_bytes;
  a.N = N; a.F = (int)F; a.B = (int)B; a.D = (int)D; a.epi = epi; a.relu = relu ? 1 : 0;
  if (B > 256) return launch_forward_wide(a, compute_dtype, out_dtype, static_cast<cudaStream_t>(stream));
  const int vec = pick_vec(D, 4, {{out, dtype_size(out_dtype)}, {bias, 4}, {w0, 4}, {b0, 4}});
  return launch_forward(a, compute_dtype, out_dtype, vec, static_cast<cudaStream_t>(stream));
}

int ple_forward(const float* x, const float* bin_edges, const float* inv_bin_widths, const int32_t* n_bins,
                const float* weight, int64_t batch, int64_t n_features, int64_t max_n_bins,
                int64_t d_embedding, int output_dtype, void* output, int bin_index_dtype,
                void* bin_indices, void* stream) {
  return forward_impl(x, bin_edges, inv_bin_widths, n_bins, weight, nullptr, nullptr, nullptr, kEpiNone, 0,
                      output_dtype, batch, n_features, max_n_bins, d_embedding, output_dtype, output,
                      bin_index_dtype, bin_indices, stream);
}

int ple_embeddings_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                           const int32_t* n_bins, const float* weight, const float* bias, const float* w0,
                           const float* b0, int epilogue, int activation, int compute_dtype, int64_t batch,
                           int64_t n_features, int64_t max_n_bins, int64_t d_embedding, int output_dtype,
                           void* output, int bin_index_dtype, void* bin_indices, void* stream) {
  return forward_impl(x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0, epilogue, activation,
                      compute_dtype, batch, n_features, max_n_bins, d_embedding, output_dtype, output,
                      bin_index_dtype, bin_indices, stream);
}

size_t ple_backward_workspace_size(int64_t batch, int64_t n_features, int64_t max_n_bins,
                                   int64_t d_embedding) {
  if (check_sizes(batch, n_features, max_n_bins, d_embedding, kWideMaxBins) != PLE_OK) return 0;
  if (max_n_bins > 256) return wide_workspace_bytes(n_features, max_n_bins, d_embedding);
  size_t b = backward_workspace_bytes(batch < 1 ? 1 : batch, n_features, max_n_bins, d_embedding);
  return b ? b : 16;
}

int ple_backward_kernel_kind(int64_t n_features, int64_t max_n_bins, int64_t d_embedding) {
  const int rc = check_sizes(1, n_features, max_n_bins, d_embedding, kWideMaxBins);
  if (rc != PLE_OK) return -rc;
  if (max_n_bins > 256) return PLE_BACKWARD_WIDE;
  return backward_uses_hist(n_features, max_n_bins, d_embedding) ? PLE_BACKWARD_HISTOGRAM : PLE_BACKWARD_SORTED;
}

static int backward_impl(const void* g, int grad_dtype, const float* x, const float* edges, const float* inv_w,
                         const int32_t* n_bins, const float* W, const float* bias, const float* w0,
                         const float* b0, int epi, int relu, int compute_dtype, int64_t N, int64_t F,
                         int64_t B, int64_t D, const void* bin_idx, int bin_idx_dtype, float* grad_x,
                         float* grad_W, float* grad_bias, float* grad_w0, float* grad_b0, void* ws,
                         size_t ws_bytes, void* stream) {
  g_msg[0] = 0;
  int st = check_sizes(N, F, B, D, epi == kEpiNone && !relu ? kWideMaxBins : 256);
  if (st) return st;
  if ((st = check_tables(edges, inv_w, n_bins, W))) return st;
  if (dtype_size(grad_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "grad dtype must be F32, F16 or BF16");
  if (dtype_size(compute_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "compute dtype must be F32, F16 or BF16");
  if (epi != kEpiNone && epi != kEpiA && epi != kEpiB) return set_error(PLE_ERR_INVALID_ARGUMENT, "bad epilogue");
  if (epi == kEpiA && relu && !bias) return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue A with ReLU needs bias");
  if (epi == kEpiB && (grad_x || grad_w0 || grad_b0) && !w0)
    return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue B needs w0");
  if (epi != kEpiA) grad_bias = nullptr;
  if (epi != kEpiB) { grad_w0 = nullptr; grad_b0 = nullptr; }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool any_param = grad_W || grad_bias || grad_w0 || grad_b0;
  if (!grad_x && !any_param) return PLE_OK;
  if (N == 0) {
    // no samples: parameter gradients are zero (reference zeros_like, backward_cuda.cu:1661-1670)
    cudaError_t e = cudaSuccess;
    if (grad_W) e = cudaMemsetAsync(grad_W, 0, (size_t)F * B * D * 4, s);
    if (e == cudaSuccess && grad_bias) e = cudaMemsetAsync(grad_bias, 0, (size_t)F * D * 4, s);
    if (e == cudaSuccess && grad_w0) e = cudaMemsetAsync(grad_w0, 0, (size_t)F * D * 4, s);
    if (e == cudaSuccess && grad_b0) e = cudaMemsetAsync(grad_b0, 0, (size_t)F * D * 4, s);
    return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "cudaMemsetAsync");
  }
  if (!g || !x) return set_error(PLE_ERR_INVALID_ARGUMENT, "grad_output and x are required");
  if (!ws) return set_error(PLE_ERR_WORKSPACE, "backward needs a workspace (ple_backward_workspace_size)");
  if (!aligned(ws, 16)) return set_error(PLE_ERR_WORKSPACE, "workspace must be 16-byte aligned");
  if (B > 256) {  // bare x_ple op over wide features: bins are recomputed, bin_indices are not read
    if (!aligned(g, dtype_size(grad_dtype))) return set_error(PLE_ERR_ALIGNMENT, "grad_output is misaligned");
    BwdArgs a{};
    a.g = g; a.x = x; a.edges = edges; a.inv_w = inv_w; a.n_bins = n_bins; a.W = W;
    a.grad_x = grad_x; a.grad_W = grad_W;
    a.ws = static_cast<float*>(ws); a.ws_bytes = ws_bytes;
    a.N = N; a.F = (int)F; a.B = (int)B; a.D = (int)D; a.epi = kEpiNone;
    return launch_backward_wide(a, compute_dtype, grad_dtype, s);
  }
  const int vec = backward_vec(D, dtype_size(grad_dtype));
  if (D / vec > 32) return set_error(PLE_ERR_UNSUPPORTED, "backward: odd d_embedding above 32 is not supported");
  // widest power of two (<= 16 bytes) dividing a lane's chunk of grad_output / of an fp32 parameter row
  const size_t chunk = (size_t)vec * dtype_size(grad_dtype);
  const size_t g_align = chunk % 16 == 0 ? 16 : chunk % 8 == 0 ? 8 : chunk % 4 == 0 ? 4 : 2;
  const size_t p_align = vec % 4 == 0 ? 16 : (size_t)vec * 4;
  if (!aligned(g, g_align) || !aligned(w0, p_align) || !aligned(bias, p_align))
    return set_error(PLE_ERR_ALIGNMENT, "grad_output / bias / w0 must be aligned to the vector width");
  int idx_bytes = 0;
  if (bin_idx) {
    switch (bin_idx_dtype) {
      case PLE_DTYPE_U8: idx_bytes = 1; break;
      case PLE_DTYPE_I16: idx_bytes = 2; break;
      case PLE_DTYPE_I32: idx_bytes = 4; break;
      default: return set_error(PLE_ERR_INVALID_ARGUMENT, "bin index dtype must be U8, I16 or I32");
    }
  }
  BwdArgs a{};
  a.bin_idx = bin_idx;
  a.bin_idx_bytes = idx_bytes;
  a.g = g; a.x = x; a.edges = edges; a.inv_w = inv_w; a.n_bins = n_bins; a.W = W;
  a.bias = bias; a.w0 = w0; a.b0 = b0;
  a.grad_x = grad_x; a.grad_W = grad_W; a.grad_bias = grad_bias; a.grad_w0 = grad_w0; a.grad_b0 = grad_b0;
  a.ws = static_cast<float*>(ws); a.ws_bytes = ws_bytes;
  a.N = N; a.F = (int)F; a.B = (int)B; a.D = (int)D; a.epi = epi; a.relu = relu ? 1 : 0;
  a.g_wide = aligned(g, 32) ? 1 : 0;  // 32-byte gradient chunks (a whole sector) may be read at once
  a.gx_vec4 = (grad_x != nullptr && aligned(grad_x, 16) && F % 4 == 0) ? 1 : 0;
  return launch_backward(a, compute_dtype, grad_dtype, vec, s);
}

int ple_backward(const void* grad_output, int grad_dtype, const float* x, const float* bin_edges,
                 const float* inv_bin_widths, const int32_t* n_bins, const float* weight,
                 const void* bin_indices, int bin_index_dtype, int64_t batch, int64_t n_features,
                 int64_t max_n_bins, int64_t d_embedding, float* grad_x, float* grad_weight, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return backward_impl(grad_output, grad_dtype, x, bin_edges, inv_bin_widths, n_bins, weight, nullptr, nullptr,
                       nullptr, kEpiNone, 0, grad_dtype, batch, n_features, max_n_bins, d_embedding, bin_indices,
                       bin_index_dtype, grad_x, grad_weight, nullptr, nullptr, nullptr, workspace, workspace_bytes,
                       stream);
}

int ple_embeddings_backward(const void* grad_output, int grad_dtype, const float* x, const float* bin_edges,
                            const float* inv_bin_widths, const int32_t* n_bins, const float* weight,
                            const float* bias, const float* w0, const float* b0, int epilogue, int activation,
                            int compute_dtype, int64_t batch, int64_t n_features, int64_t max_n_bins,
                            int64_t d_embedding, const void* bin_indices, int bin_index_dtype, float* grad_x,
                            float* grad_weight, float* grad_bias, float* grad_w0, float* grad_b0, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return backward_impl(grad_output, grad_dtype, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0,
                       epilogue, activation, compute_dtype, batch, n_features, max_n_bins, d_embedding, bin_indices,
                       bin_index_dtype, grad_x, grad_weight, grad_bias, grad_w0, grad_b0, workspace,
                       workspace_bytes, stream);
}

// ---------------------------------------------------------------- standalone encoding
static int encoding_args(EncArgs& a, const float* x, const float* edges, const float* inv_w, const int32_t* n_bins,
                         const int64_t* col_offsets, int layout, int64_t N, int64_t F, int64_t B,
                         int64_t total_cols) {
  if (N < 0) return set_error(PLE_ERR_SHAPE, "batch must be >= 0");
  if (F <= 0) return set_error(PLE_ERR_SHAPE, "n_features must be positive");
  if (B <= 0) return set_error(PLE_ERR_SHAPE, "max_n_bins must be positive");
  if (F > (int64_t)1 << 30 || B > (int64_t)1 << 20) return set_error(PLE_ERR_OVERFLOW, "n_features or max_n_bins too large");
  if (!edges || !inv_w || !n_bins) return set_error(PLE_ERR_INVALID_ARGUMENT, "bin_edges, inv_bin_widths and n_bins are required");
  if (layout == PLE_ENC_PADDED) {
    if (total_cols != F * B) return set_error(PLE_ERR_SHAPE, "padded layout: total_cols must equal n_features * max_n_bins");
  } else if (layout == PLE_ENC_RAGGED) {
    if (!col_offsets) return set_error(PLE_ERR_INVALID_ARGUMENT, "ragged layout needs col_offsets");
    if (total_cols < F || total_cols > F * B)
      return set_error(PLE_ERR_SHAPE, "ragged layout: total_cols must lie in [n_features, n_features * max_n_bins]");
  } else {
    return set_error(PLE_ERR_INVALID_ARGUMENT, "layout must be PLE_ENC_RAGGED or PLE_ENC_PADDED");
  }
  if (N > 0 && total_cols > INT64_MAX / N) return set_error(PLE_ERR_OVERFLOW, "N * total_cols overflows int64");
  a = EncArgs{};
  a.x = x; a.edges = edges; a.inv_w = inv_w; a.n_bins = n_bins; a.col_off = col_offsets;
  a.N = N; a.total_cols = total_cols; a.F = (int)F; a.B = (int)B; a.layout = layout;
  return PLE_OK;
}

int ple_encoding_forward(const float* x, const float* bin_edges, const float* inv_bin_widths, const int32_t* n_bins,
                         const int64_t* col_offsets, int layout, int64_t batch, int64_t n_features,
                         int64_t max_n_bins, int64_t total_cols, int output_dtype, void* output, void* stream) {
  g_msg[0] = 0;
  EncArgs a;
  int st = encoding_args(a, x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout, batch, n_features, max_n_bins,
                         total_cols);
  if (st) return st;
  if (dtype_size(output_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "output dtype must be F32, F16 or BF16");
  if (batch == 0) return PLE_OK;
  if (!x || !output) return set_error(PLE_ERR_INVALID_ARGUMENT, "x and output are required");
  a.out = output;
  return launch_encoding_forward(a, output_dtype, static_cast<cudaStream_t>(stream));
}

int ple_encoding_backward(const void* grad_output, int grad_dtype, const float* x, const float* bin_edges,
                          const float* inv_bin_widths, const int32_t* n_bins, const int64_t* col_offsets, int layout,
                          int64_t batch, int64_t n_features, int64_t max_n_bins, int64_t total_cols, float* grad_x,
                          void* stream) {
  g_msg[0] = 0;
  EncArgs a;
  int st = encoding_args(a, x, bin_edges, inv_bin_widths, n_bins, col_offsets, layout, batch, n_features, max_n_bins,
                         total_cols);
  if (st) return st;
  if (dtype_size(grad_dtype) == 0) return set_error(PLE_ERR_INVALID_ARGUMENT, "grad dtype must be F32, F16 or BF16");
  if (batch == 0) return PLE_OK;
  if (!grad_output || !x || !grad_x) return set_error(PLE_ERR_INVALID_ARGUMENT, "grad_output, x and grad_x are required");
  a.g = grad_output;
  a.grad_x = grad_x;
  return launch_encoding_backward(a, grad_dtype, static_cast<cudaStream_t>(stream));
}

int ple_compute_bins(const float* sorted_columns, int64_t n_rows, int64_t n_features, int n_bins, float* bin_edges,
                     float* inv_bin_widths, int32_t* n_bins_out, void* stream) {
  g_msg[0] = 0;
  if (n_rows < 2) return set_error(PLE_ERR_SHAPE, "compute_bins needs at least two rows");
  if (n_features <= 0) return set_error(PLE_ERR_SHAPE, "n_features must be positive");
  if (n_features > 0x7fffffff) return set_error(PLE_ERR_OVERFLOW, "n_features too large");
  if (n_bins < 1 || n_bins > 1023) return set_error(PLE_ERR_UNSUPPORTED, "n_bins must lie in [1, 1023]");
  if (!sorted_columns || !bin_edges || !inv_bin_widths || !n_bins_out)
    return set_error(PLE_ERR_INVALID_ARGUMENT, "compute_bins: every pointer is required");
  return launch_bins(sorted_columns, n_rows, n_features, n_bins + 1, bin_edges, inv_bin_widths, n_bins_out, n_bins + 1,
                     static_cast<cudaStream_t>(stream));
}

int ple_embeddings_backward_noalloc(const void* grad_output, int grad_dtype, const float* x,
                                    const float* bin_edges, const float* inv_bin_widths, const int32_t* n_bins,
                                    const float* weight, const float* bias, const float* w0, const float* b0,
                                    int epilogue, int activation, int compute_dtype, int64_t batch,
                                    int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                                    const void* bin_indices, int bin_index_dtype, float* grad_x,
                                    float* grad_weight, float* grad_bias, float* grad_w0, float* grad_b0,
                                    void* stream) {
  g_msg[0] = 0;
  // the same size limits as ple_embeddings_backward (more than 256 bins only for the bare x_ple op)
  int st = check_sizes(batch, n_features, max_n_bins, d_embedding,
                       epilogue == kEpiNone && !activation ? kWideMaxBins : 256);
  if (st) return st;
  const size_t need = ple_backward_workspace_size(batch, n_features, max_n_bins, d_embedding);
  if (need > PLE_NOALLOC_SCRATCH_BYTES) {
    snprintf(g_msg, sizeof(g_msg),
             "ple_embeddings_backward_noalloc: this shape needs %zu bytes of workspace, more than the %zu-byte "
             "built-in scratch; call ple_embeddings_backward with a workspace of ple_backward_workspace_size() "
             "bytes",
             need, (size_t)PLE_NOALLOC_SCRATCH_BYTES);
    return PLE_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch))) return st;
  return backward_impl(grad_output, grad_dtype, x, bin_edges, inv_bin_widths, n_bins, weight, bias, w0, b0,
                       epilogue, activation, compute_dtype, batch, n_features, max_n_bins, d_embedding, bin_indices,
                       bin_index_dtype, grad_x, grad_weight, grad_bias, grad_w0, grad_b0, scratch,
                       (size_t)PLE_NOALLOC_SCRATCH_BYTES, stream);
}

size_t ple_embeddings_linear_workspace_size(int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                                            int64_t out_features, int compute_dtype) {
  if (n_features <= 0 || max_n_bins <= 0 || max_n_bins > 256 || d_embedding <= 0 || d_embedding > kMaxD ||
      out_features <= 0 || n_features > ((int64_t)1 << 30))
    return 0;
  if (compute_dtype != PLE_DTYPE_F32 && compute_dtype != PLE_DTYPE_BF16) return 0;
  return linear_workspace_bytes(n_features, max_n_bins, d_embedding, out_features, compute_dtype);
}

int ple_embeddings_linear_forward(const float* x, const float* bin_edges, const float* inv_bin_widths,
                                  const int32_t* n_bins, const float* weight, const float* bias, const float* w0,
                                  const float* b0, int epilogue, int activation, int compute_dtype, int64_t batch,
                                  int64_t n_features, int64_t max_n_bins, int64_t d_embedding,
                                  const void* linear_weight, int linear_weight_dtype, const float* linear_bias,
                                  int64_t out_features, int output_dtype, void* output, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  g_msg[0] = 0;
  int st = check_sizes(batch, n_features, max_n_bins, d_embedding);
  if (st) return st;
  if ((st = check_tables(bin_edges, inv_bin_widths, n_bins, weight))) return st;
  if (epilogue != kEpiNone && epilogue != kEpiA && epilogue != kEpiB)
    return set_error(PLE_ERR_INVALID_ARGUMENT, "bad epilogue");
  if (epilogue == kEpiA && !bias) return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue A needs bias");
  if (epilogue == kEpiB && (!w0 || !b0)) return set_error(PLE_ERR_INVALID_ARGUMENT, "epilogue B needs w0 and b0");
  if (compute_dtype != PLE_DTYPE_F32 && compute_dtype != PLE_DTYPE_BF16)
    return set_error(PLE_ERR_UNSUPPORTED, "embeddings-linear: compute dtype must be F32 or BF16");
  if (linear_weight_dtype != PLE_DTYPE_BF16)
    return set_error(PLE_ERR_UNSUPPORTED, "embeddings-linear: the linear weight must be BF16");
  if (output_dtype != PLE_DTYPE_F32 && output_dtype != PLE_DTYPE_BF16)
    return set_error(PLE_ERR_UNSUPPORTED, "embeddings-linear: output dtype must be F32 or BF16");
  if (out_features <= 0) return set_error(PLE_ERR_SHAPE, "out_features must be positive");
  if (out_features > ((int64_t)1 << 20)) return set_error(PLE_ERR_UNSUPPORTED, "out_features above 2^20");
  if (batch > 0 && out_features > INT64_MAX / batch) return set_error(PLE_ERR_OVERFLOW, "N * out_features overflows");
  if (!linear_weight) return set_error(PLE_ERR_INVALID_ARGUMENT, "linear_weight is required");
  if (batch == 0) return PLE_OK;
  if (!x || !output) return set_error(PLE_ERR_INVALID_ARGUMENT, "x and output are required");
  if (!aligned(output, 16)) return set_error(PLE_ERR_ALIGNMENT, "output must be 16-byte aligned");
  LinearCall c{};
  c.x = x; c.edges = bin_edges; c.inv_w = inv_bin_widths; c.n_bins = n_bins; c.W = weight;
  c.bias = bias; c.w0 = w0; c.b0 = b0; c.W1 = linear_weight; c.b1 = linear_bias; c.z = output;
  c.ws = workspace; c.ws_bytes = workspace_bytes; c.N = batch; c.H = out_features;
  c.F = (int)n_features; c.B = (int)max_n_bins; c.D = (int)d_embedding;
  c.epi = epilogue; c.relu = activation ? 1 : 0; c.compute_dtype = compute_dtype; c.out_dtype = output_dtype;
  return launch_linear(c, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
