// ple_wide.cu - the reference's x_ple forward / backward ops for max_n_bins above 256.
//
// The main kernels stage a feature chunk's tables in shared memory and pack
// bins into 8 bits of their sort keys, which caps them at 256 bins.  The
// reference keeps serving wider features through its generic paths (int16 bin
// indices up to 32,768 bins, int32 beyond: _meta.py:14-19,
// ple_backward_generic_weight_kernel backward_cuda.cu:495-593).  These kernels
// are that path here: plain global-memory kernels with the same arithmetic as
// the main ones, for correctness at any bin count rather than speed.
//   forward   one thread per output element (sample, feature, d): bin search
//             over e_0 .. e_n in global memory, the fp32 prefix
//             sum_{j<k} q(W[j, d]) left to right, q(fma(q(t), q(W[phys k, d]), prefix))
//             (forward_cuda.cu:135-176, 258-273);
//   backward  one thread per (sample, feature): grad_x from the two dots
//             (backward_cuda.cu:385-483) and, per bin, fp32 atomics of g' and
//             q(t) g' into a workspace [2][F][B][D]; then one thread per
//             (feature, d) turns them into grad_W by a reverse prefix over the
//             bins (backward_cuda.cu:889-923), zeroing the padding rows.
// grad_W sums in atomic order here, so this path is not bitwise reproducible
// (the reference's atomic paths are not either).
#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

__device__ __forceinline__ int wide_n(int32_t n, int B) { return n < 1 ? 1 : (n > B ? B : n); }

// k = clamp(#{j <= n : !(x < e_j)} - 1, 0, n - 1); NaN counts every edge (common.cuh:27-63).
__device__ __forceinline__ int wide_bin(const float* e, int n, float xv) {
  int lo = 0, hi = n + 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (!(xv < e[mid])) lo = mid + 1;
    else hi = mid;
  }
  int k = lo - 1;
  k = k < 0 ? 0 : k;
  return k > n - 1 ? n - 1 : k;
}

template <typename QT, typename OT>
__global__ void __launch_bounds__(256) ple_wide_fwd_kernel(const FwdArgs a) {
  const int B = a.B, D = a.D, F = a.F;
  const int64_t total = a.N * F * D;
  OT* out = static_cast<OT*>(a.out);
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = u / D;
    const int d = (int)(u - p * D);
    const int i = (int)(p % F);
    const float xv = a.x[p];
    const float* e = a.edges + (int64_t)i * (B + 1);
    const int n = wide_n(a.n_bins[i], B);
    const int k = wide_bin(e, n, xv);
    const float qt = quantize<QT>((xv - e[k]) * a.inv_w[(int64_t)i * B + k]);
    const float* Wc = a.W + (int64_t)i * B * D + d;
    float acc = 0.0f;
    for (int j = 0; j < k; ++j) acc += quantize<QT>(Wc[(int64_t)j * D]);  // j < k <= n - 1: physical row j
    const int phys = (k == n - 1) ? B - 1 : k;
    out[u] = Dt<OT>::from_f(quantize<QT>(fmaf(qt, quantize<QT>(Wc[(int64_t)phys * D]), acc)));
    if (d == 0 && a.bin_idx != nullptr) {
      if (a.bin_idx_bytes == 2) static_cast<int16_t*>(a.bin_idx)[p] = (int16_t)k;
      else if (a.bin_idx_bytes == 4) static_cast<int32_t*>(a.bin_idx)[p] = k;
      else static_cast<uint8_t*>(a.bin_idx)[p] = (uint8_t)k;
    }
  }
}

template <typename QT, typename GT>
__global__ void __launch_bounds__(256) ple_wide_bwd_kernel(const BwdArgs a, float* U, float* H) {
  const int B = a.B, D = a.D, F = a.F;
  const int64_t pairs = a.N * F;
  const GT* gall = static_cast<const GT*>(a.g);
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < pairs; p += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(p % F);
    const float xv = a.x[p];
    const float* e = a.edges + (int64_t)i * (B + 1);
    const float* r = a.inv_w + (int64_t)i * B;
    const int n = wide_n(a.n_bins[i], B);
    const int k = wide_bin(e, n, xv);
    const float qt = quantize<QT>((xv - e[k]) * r[k]);
    const int phys = (k == n - 1) ? B - 1 : k;
    const bool edge = k > 0 && xv == e[k];
    const float* Wk = a.W + ((int64_t)i * B + phys) * D;
    const float* Wp = a.W + ((int64_t)i * B + (k > 0 ? k - 1 : 0)) * D;  // bin k - 1 < n - 1: physical row k - 1
    const GT* g = gall + p * D;
    float* Uk = U + ((int64_t)i * B + k) * D;
    float* Hk = H + ((int64_t)i * B + k) * D;
    float dot = 0.0f, dotp = 0.0f;
    for (int d = 0; d < D; ++d) {
      const float gd = Dt<GT>::to_f(g[d]);
      if (a.grad_x != nullptr) {
        dot = fmaf(gd, quantize<QT>(Wk[d]), dot);
        if (edge) dotp = fmaf(gd, quantize<QT>(Wp[d]), dotp);
      }
      if (a.grad_W != nullptr) {
        atomicAdd(Uk + d, qt * gd);
        atomicAdd(Hk + d, gd);
      }
    }
    if (a.grad_x != nullptr) a.grad_x[p] = r[k] * dot + (edge ? r[k - 1] * dotp : 0.0f);
  }
}

__global__ void __launch_bounds__(256) ple_wide_finalize_kernel(const BwdArgs a, const float* U, const float* H) {
  const int B = a.B, D = a.D;
  const int64_t cols = (int64_t)a.F * D;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(c / D);
    const int d = (int)(c - (int64_t)i * D);
    const int n = wide_n(a.n_bins[i], B);
    float* gw = a.grad_W + (int64_t)i * B * D + d;
    for (int j = n - 1; j < B - 1; ++j) gw[(int64_t)j * D] = 0.0f;  // padding rows
    float suffix = 0.0f;
    for (int j = n - 1; j >= 0; --j) {
      const int64_t o = ((int64_t)i * B + j) * D + d;
      const int phys = (j == n - 1) ? B - 1 : j;
      gw[(int64_t)phys * D] = U[o] + suffix;
      suffix += H[o];
    }
  }
}

size_t wide_workspace_bytes(int64_t F, int64_t B, int64_t D) { return (size_t)2 * F * B * D * sizeof(float); }

static int wide_grid(int64_t items) {
  const int64_t cap = (int64_t)device_sm_count() * 8;
  int64_t g = (items + 255) / 256;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

template <typename QT, typename OT>
static int fwd_wide_t(const FwdArgs& a, cudaStream_t st) {
  ple_wide_fwd_kernel<QT, OT><<<wide_grid(a.N * a.F * a.D), 256, 0, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "ple_wide_fwd_kernel");
}

int launch_forward_wide(const FwdArgs& a, int compute_dtype, int output_dtype, cudaStream_t st) {
  const int q = compute_dtype, o = output_dtype;
  if (q == PLE_DTYPE_F32 && o == PLE_DTYPE_F32) return fwd_wide_t<float, float>(a, st);
  if (q == PLE_DTYPE_BF16 && o == PLE_DTYPE_BF16) return fwd_wide_t<__nv_bfloat16, __nv_bfloat16>(a, st);
  if (q == PLE_DTYPE_BF16 && o == PLE_DTYPE_F32) return fwd_wide_t<__nv_bfloat16, float>(a, st);
  if (q == PLE_DTYPE_F16 && o == PLE_DTYPE_F16) return fwd_wide_t<__half, __half>(a, st);
  if (q == PLE_DTYPE_F16 && o == PLE_DTYPE_F32) return fwd_wide_t<__half, float>(a, st);
  if (q == PLE_DTYPE_F32 && o == PLE_DTYPE_BF16) return fwd_wide_t<float, __nv_bfloat16>(a, st);
  return set_error(PLE_ERR_UNSUPPORTED, "forward: unsupported (compute, output) dtype pair");
}

template <typename QT, typename GT>
static int bwd_wide_t(const BwdArgs& a, float* U, float* H, cudaStream_t st) {
  ple_wide_bwd_kernel<QT, GT><<<wide_grid(a.N * a.F), 256, 0, st>>>(a, U, H);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "ple_wide_bwd_kernel");
  if (a.grad_W == nullptr) return PLE_OK;
  ple_wide_finalize_kernel<<<wide_grid((int64_t)a.F * a.D), 256, 0, st>>>(a, U, H);
  e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "ple_wide_finalize_kernel");
}

template <typename QT>
static int bwd_wide_g(const BwdArgs& a, int grad_dtype, float* U, float* H, cudaStream_t st) {
  if (grad_dtype == PLE_DTYPE_F32) return bwd_wide_t<QT, float>(a, U, H, st);
  if (grad_dtype == PLE_DTYPE_BF16) return bwd_wide_t<QT, __nv_bfloat16>(a, U, H, st);
  if (grad_dtype == PLE_DTYPE_F16) return bwd_wide_t<QT, __half>(a, U, H, st);
  return set_error(PLE_ERR_UNSUPPORTED, "backward: unsupported gradient dtype");
}

int launch_backward_wide(const BwdArgs& a, int compute_dtype, int grad_dtype, cudaStream_t st) {
  const size_t cells = (size_t)a.F * a.B * a.D;
  float* U = a.ws;
  float* H = a.ws + cells;
  if (a.grad_W != nullptr) {
    if (a.ws_bytes < wide_workspace_bytes(a.F, a.B, a.D))
      return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
    const cudaError_t e = cudaMemsetAsync(a.ws, 0, 2 * cells * sizeof(float), st);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaMemsetAsync");
  }
  if (compute_dtype == PLE_DTYPE_F32) return bwd_wide_g<float>(a, grad_dtype, U, H, st);
  if (compute_dtype == PLE_DTYPE_BF16) return bwd_wide_g<__nv_bfloat16>(a, grad_dtype, U, H, st);
  if (compute_dtype == PLE_DTYPE_F16) return bwd_wide_g<__half>(a, grad_dtype, U, H, st);
  return set_error(PLE_ERR_UNSUPPORTED, "backward: unsupported compute dtype");
}

}  // namespace ple
