// ple_bins.cu - quantile bin edges on the device (upstream
// rtdl_num_embeddings.compute_bins without a tree: per feature the
// n_bins + 1 quantiles at j / n_bins, j = 0..n_bins, of the training column,
// linearly interpolated between order statistics (torch.quantile's default),
// duplicates removed), written straight into the padded tables the kernels
// consume (module.py:58-109 of the reference: +inf padded edges, fp32
// reciprocal widths, int32 bin counts).
//
// Input: the columns sorted ascending, feature-major [F][N] (any sort; the
// caller uses torch.sort).  One CTA per feature, one thread per quantile.
#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

namespace {

constexpr int kBinsThreads = 1024;

__global__ void __launch_bounds__(kBinsThreads) ple_bins_kernel(const float* sorted, int64_t N, int n_q,
                                                                 float* edges, float* inv_w, int32_t* n_bins,
                                                                 int ld_e) {
  __shared__ float sq[kBinsThreads];
  __shared__ int spos[kBinsThreads];
  __shared__ int s_warp[kBinsThreads / 32];
  const int f = blockIdx.x, j = threadIdx.x;
  const float* col = sorted + (int64_t)f * N;
  const bool live = j < n_q;
  float q = 0.f;
  if (live) {
    // position j / (n_q - 1) * (N - 1), split into an order statistic and a fraction (float64 for exactness
    // of the split on large N)
    const double pos = (double)j * (double)(N - 1) / (double)(n_q - 1);
    int64_t lo = (int64_t)floor(pos);
    if (lo > N - 1) lo = N - 1;
    const int64_t hi = lo + 1 < N ? lo + 1 : N - 1;
    const float w = (float)(pos - (double)lo);
    const float a = col[lo], b = col[hi];
    q = w == 0.f ? a : fmaf(w, b - a, a);  // linear interpolation (exact endpoints)
    sq[j] = q;
  }
  __syncthreads();
  // keep the first of every run of equal values (the column is sorted, so the quantiles are too)
  const bool keep = live && (j == 0 || sq[j - 1] != q);
  const unsigned m = __ballot_sync(0xffffffffu, keep);
  const int lane = j & 31, wid = j >> 5;
  if (lane == 0) s_warp[wid] = __popc(m);
  __syncthreads();
  if (wid == 0) {
    int v = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += u;
    }
    if (lane < (int)(blockDim.x >> 5)) s_warp[lane] = v;  // inclusive prefix over warps
  }
  __syncthreads();
  const int before = (wid > 0 ? s_warp[wid - 1] : 0) + __popc(m & ((1u << lane) - 1u));
  const int n_unique = s_warp[(blockDim.x >> 5) - 1];
  if (keep) spos[before] = j;
  __syncthreads();
  // compacted edges, +inf padding; reciprocal widths of consecutive kept edges, 0 padding
  float* er = edges + (int64_t)f * ld_e;
  float* rw = inv_w + (int64_t)f * (ld_e - 1);
  const float inf = __int_as_float(0x7f800000);
  for (int t = j; t < ld_e; t += blockDim.x) er[t] = t < n_unique ? sq[spos[t]] : inf;
  for (int t = j; t < ld_e - 1; t += blockDim.x)
    rw[t] = t + 1 < n_unique ? 1.0f / (sq[spos[t + 1]] - sq[spos[t]]) : 0.0f;
  if (j == 0) n_bins[f] = n_unique - 1;
}

}  // namespace

int launch_bins(const float* sorted, int64_t N, int64_t F, int n_q, float* edges, float* inv_w, int32_t* n_bins,
                int ld_e, cudaStream_t st) {
  ple_bins_kernel<<<(unsigned)F, kBinsThreads, 0, st>>>(sorted, N, n_q, edges, inv_w, n_bins, ld_e);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "bins launch");
}

}  // namespace ple
