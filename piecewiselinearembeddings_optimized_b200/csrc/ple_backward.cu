// ple_backward.cu - planning, workspace and finalize of the fused PLE backward
// (the kernel itself is in ple_backward_impl.cuh, instantiated per dtype pair
// in ple_backward_<dtypes>.cu so that the instantiations compile in parallel).
//
// Workspace: one partial [Fc][B + 3][D] fp32 block per (slot, segment of the
// slot's range, member CTA of the slot); rows 0..B-1 grad_W in the physical
// layout, B the bias, B + 1 w0, B + 2 b0.  The finalize kernel sums, per
// feature, the blocks of the slots whose ranges cover the feature's group,
// in slot order (deterministic).
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include <cudaTypedefs.h>

#include "ple_backward_hist.cuh"
#include "ple_backward_impl.cuh"

namespace ple {

int launch_bwd_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_bf16_f32(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16(const BwdArgs& a, int vec, cudaStream_t st);
int launch_bwd_f16_f32(const BwdArgs& a, int vec, cudaStream_t st);

__global__ void ple_bwd_finalize_kernel(const BwdArgs a, int n_slots) {
  const int B = a.B, D = a.D, Fc = a.Fc, m = a.group;
  const int64_t rows = (int64_t)a.F * (B + 3) * D;
  const int64_t total = (int64_t)a.n_groups * a.N;
  const int64_t block = (int64_t)Fc * (B + 3) * D;
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
    const int grp = chunk / m, member = chunk - grp * m;
    const int64_t c_lo = (int64_t)grp * a.N, c_hi = c_lo + a.N;
    // first slot whose range [total*j/n_slots, total*(j+1)/n_slots) ends past the group start
    int64_t j = c_lo * n_slots / total;
    while (j > 0 && total * j / n_slots > c_lo) --j;
    while (j < n_slots && total * (j + 1) / n_slots <= c_lo) ++j;
    float s = 0.f;
    for (; j < n_slots; ++j) {
      const int64_t lo = total * j / n_slots;
      const int64_t hi = total * (j + 1) / n_slots;
      if (lo >= c_hi) break;
      if (hi <= lo) continue;
      const int seg = grp - (int)(lo / a.N);  // segments of slot j are consecutive groups
      s += a.ws[((j * a.max_segs + seg) * m + member) * block + (int64_t)i * (B + 3) * D + rem];
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

// Features per CTA (power of two, up to 4) and tile length: the largest tile in (feature, sample) pairs
// whose layout fits, preferring more features (wider gradient rows per sample for DRAM: measured, one
// feature per CTA with 4096-sample tiles read 114 bytes of DRAM per 68-byte pair at c5 and ran 30%
// slower than four features with 1024-sample tiles).  False if even one feature does not fit.
static bool bwd_plan(BwdArgs& a, int vec, size_t* smem_out) {
  const int nc = a.D / vec;
  if (nc > 32) return false;
  a.lgk = 0;
  while ((1 << a.lgk) < a.B) ++a.lgk;
  const size_t optin = device_max_smem_optin();
  int lgWarps = 0;
  while ((1 << lgWarps) < kBwdWarps) ++lgWarps;
  int best = -1;
  for (int lgFc = 2; lgFc >= 0; --lgFc) {
    if (lgFc > lgWarps) continue;
    if (lgFc > 0 && (1 << (lgFc - 1)) >= a.F) continue;
    const int Fc = 1 << lgFc;
    const int lgWf = lgWarps - lgFc;
    const int G = (1 << lgWf) * (32 / nc);
    for (int lgSt = 11; lgSt >= 7; --lgSt) {
      if (lgSt < lgWf + 5) break;    // every warp ranks at least 32 samples of its quarter
      if (lgSt - lgWf > 11) continue;  // ranks within a quarter take 11 bits of the entry
      BwdDims m{Fc, 1 << lgWf, 1 << lgSt, G, nc, 1 << a.lgk};
      const size_t bytes = bwd_layout_bytes(a.B, a.D, m, nullptr, nullptr);
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

// Slots of `group` CTAs: the CTAs of a slot cover consecutive chunks whose x / grad_x rows together fill
// 64 bytes, over the same samples, so that the pieces of a row the members read and write meet in L2
// (measured: 32-byte groups left about 13 bytes per pair of extra DRAM reads at c5).
static void bwd_grid(BwdArgs& a, int* grid) {
  int m = 64 / (4 * a.Fc);
  if (m < 1) m = 1;
  if (m > a.n_chunks) m = a.n_chunks;
  a.group = m;
  a.n_groups = (int)ceil_div<int64_t>(a.n_chunks, m);
  const int64_t total = (int64_t)a.n_groups * a.N;
  int64_t slots = device_sm_count() / m;
  const int64_t min_units = 64;  // at least 64 (group, sample) rows per slot
  if (slots > total / min_units) slots = total / min_units;
  if (slots < 1) slots = 1;
  *grid = (int)(slots * m);
  const int64_t len = ceil_div<int64_t>(total, slots);
  a.max_segs = (int)(ceil_div<int64_t>(len, a.N) + 1);  // groups one range can touch
}

static size_t ws_bytes_for(const BwdArgs& a, int grid) {
  return (size_t)grid * a.max_segs * ((size_t)a.Fc * (a.B + 3) * a.D) * sizeof(float);
}

// Histogram kernel: D = 4 VEC with VEC in {2, 4, 6}, at most 256 bins; features per CTA (4, 2, 1, preferred
// in that order: whole 16-byte x / grad_x pieces per sample) and the longest tile (2 to 16 batches of 32
// samples per warp) whose layout fits.
static bool hist_plan(BwdArgs& a, size_t* smem_out) {
  const int vec = a.D / kHistNC;
  if (a.D % kHistNC != 0 || (vec != 2 && vec != 4 && vec != 6) || a.B > 256 || a.B < 1) return false;
  a.lgk = 0;
  while ((1 << a.lgk) < a.B) ++a.lgk;
  const size_t optin = device_max_smem_optin();
  for (int lgFc = 2; lgFc >= 0; --lgFc) {
    if (lgFc > 0 && (1 << (lgFc - 1)) >= a.F) continue;
    const int Fc = 1 << lgFc, Wf = kHistWarps / Fc;
    for (int batches = 16; batches >= 2; batches /= 2) {  // batches per warp per tile
      const int St = 32 * Wf * batches;
      const size_t bytes = hist_layout_bytes(a.B, a.D, Fc, St, 1 << a.lgk, nullptr, nullptr);
      if (bytes > optin) continue;
      a.lgFc = lgFc;
      a.Fc = Fc;
      a.hist_St = St;
      a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
      *smem_out = bytes;
      return true;
    }
  }
  return false;
}

// The kernel a backward of this shape runs: the histogram kernel where its plan fits, unless
// PLE_BACKWARD_KERNEL=sorted (read once) asks for the sorted kernel everywhere.
static bool use_hist() {
  static const bool hist = [] {
    const char* v = getenv("PLE_BACKWARD_KERNEL");
    return !(v != nullptr && strcmp(v, "sorted") == 0);
  }();
  return hist;
}

size_t backward_workspace_bytes(int64_t N, int64_t F, int64_t B, int64_t D) {
  size_t best = 0;
  BwdArgs b{};
  b.N = N; b.F = (int)F; b.B = (int)B; b.D = (int)D;
  size_t smem = 0;
  int grid = 0;
  if (bwd_plan(b, backward_vec(D, 4), &smem)) {
    bwd_grid(b, &grid);
    best = ws_bytes_for(b, grid);
  }
  BwdArgs h{};
  h.N = N; h.F = (int)F; h.B = (int)B; h.D = (int)D;
  if (hist_plan(h, &smem)) {
    bwd_grid(h, &grid);
    best = std::max(best, ws_bytes_for(h, grid));
  }
  return best;
}

bool backward_uses_hist(int64_t F, int64_t B, int64_t D) {
  BwdArgs h{};
  h.N = 1; h.F = (int)F; h.B = (int)B; h.D = (int)D;
  size_t smem = 0;
  return use_hist() && hist_plan(h, &smem);
}

int hist_prepare(BwdArgs& a, size_t* smem, int* grid) {
  if (!hist_plan(a, smem)) return set_error(PLE_ERR_UNSUPPORTED, "backward: shape outside the histogram kernel");
  bwd_grid(a, grid);
  if (ws_bytes_for(a, *grid) > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  return PLE_OK;
}

int bwd_prepare(BwdArgs& a, int vec, size_t* smem, int* grid) {
  if (!bwd_plan(a, vec, smem)) return set_error(PLE_ERR_UNSUPPORTED, "backward: tables do not fit in shared memory");
  // sample offsets inside a tile are 32-bit: (tile length) * F * D elements must fit
  if ((int64_t)(1 << a.lgSt) * a.F * a.D >= ((int64_t)1 << 32))
    return set_error(PLE_ERR_UNSUPPORTED, "backward: n_features * d_embedding too large");
  bwd_grid(a, grid);
  if (ws_bytes_for(a, *grid) > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  return PLE_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool bwd_grad_map(const BwdArgs& a, int elem, CUtensorMap* map) {
  memset(map, 0, sizeof(*map));
  const int gbytes = elem == 0 ? 4 : 2;
  const int64_t cols = (int64_t)a.F * a.D;
  const int box_cols = a.Fc * a.D;
  if (a.N < 1 || a.N > 0x7fffffff || cols > 0x7fffffff) return false;
  if (box_cols > 256 || (box_cols * gbytes) % 16 != 0 || (cols * gbytes) % 16 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(a.g) & 15) != 0) return false;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const CUtensorMapDataType dt = elem == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                               : elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)a.N};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * gbytes)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, 256u};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = enc(map, dt, 2, const_cast<void*>(a.g), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    memset(map, 0, sizeof(*map));
    return false;
  }
  return true;
}

int bwd_finalize(const BwdArgs& a, int grid, cudaStream_t st) {
  const int64_t rows = (int64_t)a.F * (a.B + 3) * a.D;
  const int blocks = (int)min64(ceil_div<int64_t>(rows, 256), 4L * device_sm_count());
  ple_bwd_finalize_kernel<<<blocks, 256, 0, st>>>(a, grid / a.group);
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
