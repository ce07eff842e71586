// ple_backward.cu - planning, workspace and finalize of the fused PLE backward
// (the kernel itself is in ple_backward_impl.cuh, instantiated per dtype pair
// in ple_backward_<dtypes>.cu so that the instantiations compile in parallel).
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "ple_backward_tc.cuh"

namespace ple {

// Set to 1 by a tensor-core backward whose wait expired (ple_tensor_core_status reads and clears it).
__device__ int g_tc_dev_err = 0;

int launch_bwd_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16_f32(const BwdArgs& a, int vec, cudaStream_t st);

// Sum, per feature, the partials of the CTAs whose ranges cover its chunk, in
// CTA order (deterministic).  Rows whose gradient was not requested are
// neither read nor written.
__global__ void ple_bwd_finalize_kernel(const BwdArgs a, int grid) {
  const int B = a.B, D = a.D, Fc = a.Fc;
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
    const int chunk = (int)(f / Fc), i = (int)(f - (int64_t)chunk * Fc);
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
  a.lgk = 0;
  while ((1 << a.lgk) < a.B) ++a.lgk;
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
      const size_t bytes = bwd_layout_bytes(a.B, a.D, 1 << a.lgk, m, nullptr, nullptr);
      if (bytes > optin) continue;
      const int score = lgFc + lgSt;
      if (score > best) {
        best = score;
        a.lgFc = lgFc;
        a.lgWf = lgWf;
        a.lgSt = lgSt;
        a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
        a.Fc = Fc;
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
  size_t bytes = ws_bytes_for(b, grid);
  // the tensor-core kernel's needs for each compute type (parts of q(g') and of q(t) q(g'))
  // (bf16 parts of H, of U, register cap) per (compute, gradient) type pair
  const int parts[5][3] = {{3, 3, tc_max_regs<float>()}, {1, 2, tc_max_regs<__nv_bfloat16>()},
                           {1, 2, tc_max_regs<float>()}, {2, 3, tc_max_regs<__half>()}, {2, 3, tc_max_regs<float>()}};
  for (const auto& pp : parts) {
    BwdArgs t{};
    t.N = N; t.F = (int)F; t.B = (int)B; t.D = (int)D;
    TcGeom m{};
    int threads = 0, tg = 0;
    if (tc_plan(t, pp[0], pp[1], tc_max_warps(pp[2]), &m, &threads, &smem)) bytes = std::max(bytes, tc_ws_floats(t, m, threads, &tg) * 4);
  }
  return bytes;
}

int bwd_prepare(BwdArgs& a, int vec, size_t* smem, int* grid) {
  if (!bwd_plan(a, vec, smem)) return set_error(PLE_ERR_UNSUPPORTED, "backward: tables do not fit in shared memory");
  bwd_grid(a, grid);
  if (ws_bytes_for(a, *grid) > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  a.x_vec4 = ((1 << a.lgFc) >= 4) && (a.F % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  return PLE_OK;
}

// ------------------------------------------------------------ tensor-core kernel planning
static int pow2_at_least(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

static size_t tc_layout(TcGeom& m, int B, int D, int pow2) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 127) & ~(size_t)127;
    return (int)o;
  };
  const int units = m.nG * m.nh;
  m.oA = take((size_t)2 * m.nG * 128 * m.R * 2);
  m.oB = take((size_t)2 * m.nG * m.R * m.cols * 2);  // directly after A (zeroed together)
  m.oT = take((size_t)B * m.ts * 4);
  m.oS = take((size_t)B * m.ts * 4);
  m.oE = take((size_t)pow2 * m.Fc * 4);
  m.oR = take((size_t)B * m.Fc * 4);
  m.oN = take((size_t)m.Fc * 4);
  m.oGX = take((size_t)2 * m.R * m.Fc * m.nh * 4);  // [2][Fc * nh][R]
  m.oTot = take((size_t)units * 4 * 8 * 4);
  m.oKey = take((size_t)2 * m.R * m.Fc);
  m.oBar = take(64);  // full[2], empty[2], TMEM address, non-finite flag, abort flag
  (void)D;
  return off;
}

// Geometry of the tensor-core kernel, false where it does not apply: bins <= 128 (padded to Bp = 32,
// 64 or 128; FM = 128 / Bp features share an MMA's M = 128 rows), D a multiple of 8 up to 32 (one
// warp of flush lanes per 8-column block and group), one feature's parts * D columns <= 256 (one MMA).
bool tc_plan(const BwdArgs& a, int parts_h, int parts_u, int max_warps, TcGeom* m, int* threads, size_t* smem) {
  const int B = a.B, D = a.D;
  if (B < 1 || B > 128 || D % 8 != 0 || D > 32 || a.F < 1) return false;
  int Bp = 32;
  while (Bp < B) Bp <<= 1;
  const int Cf = (parts_h + parts_u) * D;
  if (Cf > 256) return false;
  const int nh = D / 8;
  const int pow2 = pow2_at_least(B + 1);
  int lgp = 0;
  while ((1 << lgp) < pow2) ++lgp;
  const size_t optin = device_max_smem_optin();
  // FM features stacked in the M = 128 rows (up to 128 / Bp; rows past FM * Bp stay zero), nG groups of
  // accumulators plus 16 running-sum columns per unit (group, column block) in TMEM: the most of both whose
  // producer warps and shared memory fit
  for (int FM = 128 / Bp; FM >= 1; FM >>= 1) {
    int fpm = FM;
    while (fpm > 1 && fpm * Cf > 256) fpm >>= 1;
    const int Nmma = (fpm * Cf + 15) & ~15;
    const int n_mma = FM / fpm, cols = n_mma * Nmma;
    int nG = kTcTmemCols / (cols + 16 * nh);
    nG = std::min<int>(nG, (int)ceil_div<int64_t>(a.F, FM));
    for (; nG >= 1; --nG) {
      TcGeom g{};
      g.Bp = Bp; g.FM = FM; g.fpm = fpm; g.Nmma = Nmma; g.n_mma = n_mma; g.cols = cols; g.nG = nG; g.nh = nh;
      g.Fc = nG * FM;
      g.ts = table_stride(g.Fc, D);
      g.lgp = lgp;
      // producer warps: a multiple of the (feature, column block) count C (each warp keeps one) and of 4
      // (the TMEM lane quarters); each warp drains nu of the nG * nh units
      const int C = g.Fc * nh;
      int WP = C;
      while (WP % 4) WP += C;
      if (WP * 32 > kTcMaxProducers || WP + 1 > max_warps || (4 * nG * nh) % WP != 0) continue;
      g.nu = 4 * nG * nh / WP;
      g.R = 32 * kTcItems * WP / C;
      size_t bytes = tc_layout(g, B, D, pow2);
      // more than half of an SM's shared memory: one CTA per SM, so the 512-column TMEM allocation never waits
      bytes = std::max<size_t>(bytes, 116 * 1024);
      if (bytes > optin) continue;
      g.flush_tiles = std::max(1, 256 / g.R);  // the accumulators are drained every 256 samples
      *m = g;
      *threads = 32 * WP;
      *smem = bytes;
      return true;
    }
  }
  return false;
}

// Workspace floats of the tensor-core kernel: partials [grid][max_segs][Fc][B + 3][D], non-finite sums
// [grid][Fc][Bp][2][D], epilogue scratch [grid][threads][16]; fills a's chunking and m's offsets.
size_t tc_ws_floats(BwdArgs& a, TcGeom& m, int threads, int* grid) {
  a.Fc = m.Fc;
  a.n_chunks = (int)ceil_div<int64_t>(a.F, m.Fc);
  const int64_t total = (int64_t)a.n_chunks * a.N;
  int64_t g = device_sm_count();
  const int64_t min_units = 64;
  if (g > total / min_units) g = total / min_units;
  if (g < 1) g = 1;
  *grid = (int)g;
  const int64_t len = ceil_div<int64_t>(total, g);
  a.max_segs = (int)(ceil_div<int64_t>(len, a.N) + 1);
  const int64_t partials = g * a.max_segs * (int64_t)m.Fc * (a.B + 3) * a.D;
  m.spec_off = (partials + 63) & ~(int64_t)63;
  const int64_t spec = g * (int64_t)m.Fc * m.Bp * 2 * a.D;
  m.escr_off = (m.spec_off + spec + 63) & ~(int64_t)63;
  return (size_t)(m.escr_off + g * (int64_t)threads * 16);
}

static int* tc_err_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  static int* cache[64] = {};
  if (dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_dev_err) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

int tc_prepare(BwdArgs& a, TcGeom& m, int threads, int* grid) {
  a.pow2 = pow2_at_least(a.B + 1);
  const size_t floats = tc_ws_floats(a, m, threads, grid);
  if (floats * 4 > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  m.dev_err = tc_err_ptr();
  if (!m.dev_err) return set_error(PLE_ERR_CUDA, "tensor-core backward: status word not addressable");
  return PLE_OK;
}

int tensor_core_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_dev_err, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_tc_dev_err, &zero, sizeof(int));
  }
  return v;
}

// PLE_BACKWARD_KERNEL: "tensor" selects the tensor-core backward, anything else the sorted one.
int backward_kernel_mode() {
  const char* v = getenv("PLE_BACKWARD_KERNEL");
  return (v != nullptr && strcmp(v, "tensor") == 0) ? 2 : 1;
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
