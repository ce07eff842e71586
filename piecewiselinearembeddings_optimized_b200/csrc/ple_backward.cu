// ple_backward.cu - planning, workspace and finalize of the fused PLE backward
// (the kernel itself is in ple_backward_impl.cuh, instantiated per dtype pair
// in ple_backward_<dtypes>.cu so that the instantiations compile in parallel).
#include "ple_backward_impl.cuh"

namespace ple {

int launch_bwd_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16_f32(const BwdArgs& a, int vec, cudaStream_t st);

// Sum, per feature, the partials of the CTAs whose ranges cover its chunk, in
// CTA order (deterministic).  Rows whose gradient was not requested are
// neither read nor written.
__global__ void ple_bwd_finalize_kernel(const BwdArgs a, int grid) {
  const int B = a.B, D = a.D, lgFc = a.lgFc, Fc = 1 << lgFc;
  const int64_t rows = (int64_t)a.F * (B + 3) * D;
  const int64_t total = (int64_t)a.n_chunks * a.N;
  const int64_t slot = (int64_t)Fc * (B + 3) * D;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = idx / ((int64_t)(B + 3) * D);
    const int64_t rem = idx - f * (B + 3) * D;
    const int row = (int)(rem / D), d = (int)(rem - (int64_t)row * D);
    float* dst = row < B ? (a.grad_W ? a.grad_W + (f * B + row) * D + d : nullptr)
               : row == B ? (a.grad_bias ? a.grad_bias + f * D + d : nullptr)
               : row == B + 1 ? (a.grad_w0 ? a.grad_w0 + f * D + d : nullptr)
                              : (a.grad_b0 ? a.grad_b0 + f * D + d : nullptr);
    if (dst == nullptr) continue;
    const int chunk = (int)(f >> lgFc), i = (int)(f & (Fc - 1));
    const int64_t c_lo = (int64_t)chunk * a.N, c_hi = c_lo + a.N;
    // first CTA whose range [total*j/grid, total*(j+1)/grid) ends past the chunk start
    int64_t j = c_lo * grid / total;
    while (j > 0 && total * j / grid > c_lo) --j;
    while (j < grid && total * (j + 1) / grid <= c_lo) ++j;
    float s = 0.f;
    for (; j < grid; ++j) {
      const int64_t lo = total * j / grid;
      const int64_t hi = total * (j + 1) / grid;
      if (lo >= c_hi) break;
      if (hi <= lo) continue;
      const int seg = chunk - (int)(lo / a.N);  // segments of CTA j are consecutive chunks
      s += a.ws[(j * a.max_segs + seg) * slot + (int64_t)i * (B + 3) * D + rem];
    }
    *dst = s;
  }
}

// ------------------------------------------------------------------ planning
// Elements per lane of a D row: the widest of 8, 4, 2, 1 that divides D (a row
// never spans more than a warp).
int backward_vec(int64_t D, int /*grad_bytes*/) {
  for (int v : {8, 4, 2})
    if (D % v == 0 && D / v <= 32) return v;
  return 1;
}

// Features per CTA (power of two) and tile length: the largest tile in
// (feature, sample) pairs whose layout fits, preferring more features; false
// if even one feature does not fit.
static bool bwd_plan(BwdArgs& a, int vec, size_t* smem_out) {
  const int nc = a.D / vec;
  if (nc > 32) return false;
  int pow2 = 1;
  while (pow2 < a.B + 1) pow2 <<= 1;
  a.pow2 = pow2;
  const size_t optin = device_max_smem_optin();
  constexpr int kWarps = kBwdThreads / 32;
  int lgWarps = 0;
  while ((1 << lgWarps) < kWarps) ++lgWarps;
  int best = -1;
  for (int lgFc = 2; lgFc >= 0; --lgFc) {
    if (lgFc > lgWarps) continue;
    if (lgFc > 0 && (1 << (lgFc - 1)) >= a.F) continue;
    const int Fc = 1 << lgFc;
    const int lgWf = lgWarps - lgFc;
    const int G = (1 << lgWf) * (32 / nc);
    for (int lgSt = 12; lgSt >= 7; --lgSt) {
      if (lgSt < lgWf) break;
      BwdDims m{Fc, 1 << lgWf, 1 << lgSt, G, nc};
      const size_t bytes = bwd_layout_bytes(a.B, a.D, pow2, m, nullptr, nullptr);
      if (bytes > optin) continue;
      const int score = lgFc + lgSt;
      if (score > best) {
        best = score;
        a.lgFc = lgFc;
        a.lgWf = lgWf;
        a.lgSt = lgSt;
        a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
        *smem_out = bytes;
      }
      break;
    }
  }
  return best >= 0;
}

static void bwd_grid(BwdArgs& a, int* grid) {
  const int64_t total = (int64_t)a.n_chunks * a.N;
  int64_t g = device_sm_count();
  const int64_t min_units = 64;  // at least 64 (chunk, sample) rows per CTA
  if (g > total / min_units) g = total / min_units;
  if (g < 1) g = 1;
  *grid = (int)g;
  const int64_t len = ceil_div<int64_t>(total, g);
  a.max_segs = (int)(ceil_div<int64_t>(len, a.N) + 1);  // chunks one range can touch
}

static size_t ws_bytes_for(const BwdArgs& a, int grid) {
  return (size_t)grid * a.max_segs * ((size_t)(1 << a.lgFc) * (a.B + 3) * a.D) * sizeof(float);
}

size_t backward_workspace_bytes(int64_t N, int64_t F, int64_t B, int64_t D) {
  BwdArgs b{};
  b.N = N; b.F = (int)F; b.B = (int)B; b.D = (int)D;
  size_t smem = 0;
  if (!bwd_plan(b, backward_vec(D, 4), &smem)) return 0;
  int grid = 0;
  bwd_grid(b, &grid);
  return ws_bytes_for(b, grid);
}

int bwd_prepare(BwdArgs& a, int vec, size_t* smem, int* grid) {
  if (!bwd_plan(a, vec, smem)) return set_error(PLE_ERR_UNSUPPORTED, "backward: tables do not fit in shared memory");
  bwd_grid(a, grid);
  if (ws_bytes_for(a, *grid) > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  a.x_vec4 = ((1 << a.lgFc) >= 4) && (a.F % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  return PLE_OK;
}

int bwd_finalize(const BwdArgs& a, int grid, cudaStream_t st) {
  const int64_t rows = (int64_t)a.F * (a.B + 3) * a.D;
  const int blocks = (int)min64(ceil_div<int64_t>(rows, 256), 4L * device_sm_count());
  ple_bwd_finalize_kernel<<<blocks, 256, 0, st>>>(a, grid);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "backward finalize launch");
}

int launch_backward(BwdArgs a, int compute_dtype, int grad_dtype, int vec, cudaStream_t st) {
  const int q = compute_dtype, g = grad_dtype;
  if (a.epi == kEpiNone) a.relu = 0;
  if (q == PLE_DTYPE_F32 && g == PLE_DTYPE_F32) return launch_bwd_f32(a, vec, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_BF16) return launch_bwd_bf16(a, vec, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_F32) return launch_bwd_bf16_f32(a, vec, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F16) return launch_bwd_f16(a, vec, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F32) return launch_bwd_f16_f32(a, vec, st);
  return set_error(PLE_ERR_UNSUPPORTED, "backward: unsupported (compute, grad) dtype pair");
}

}  // namespace ple
