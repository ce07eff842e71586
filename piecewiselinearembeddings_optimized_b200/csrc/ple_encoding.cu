// ple_encoding.cu - standalone piecewise-linear encoding (upstream
// rtdl_num_embeddings.PiecewiseLinearEncoding): the materialised encoding and
// the gradient with respect to x.  The reference package has no CUDA path for
// it (it only exists implicitly inside its x_ple op).
//
// Column j of feature i (logical bin j < n_i) holds
//   t_j = (x - e_j) * r_j clamped to <= 1 (j = 0), [0, 1] (0 < j < n_i - 1),
//   >= 0 (j = n_i - 1); a single-bin feature is unclamped; NaN propagates.
// (position as backward_cuda.cu:194-196 / forward_cuda.cu:223-225; the
// clamps are upstream's column clamps.)
// grad_x = sum_j g_j * r_j * [lo_j <= t_j <= hi_j]   (the clamp's gradient
// passes at its bounds, as torch.clamp's backward does; NaN t passes none).
//
// Layouts of the encoding row of a sample:
//   PLE_ENC_RAGGED  [sum_i n_i]: feature-major, logical bin order, no padding
//                   (column offsets col_off[F + 1] = prefix of n_i);
//   PLE_ENC_PADDED  [F, B]: the physical layout of the embedding weights
//                   (bin j < n_i - 1 at column j, the last bin at B - 1,
//                   zero padding between).
#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

namespace {

constexpr int kEncThreads = 256;
constexpr int kEncTileCols = kEncThreads * 4;  // forward: four columns per thread

struct ColInfo {
  int f;  // feature, or -1 for a padding column
  float e, r, lo, hi;
};

// Feature and logical bin of column c of the encoding row.
__device__ __forceinline__ ColInfo column_info(const EncArgs& a, int64_t c) {
  ColInfo ci{-1, 0.f, 0.f, 0.f, 0.f};
  int f, j;
  if (a.layout == PLE_ENC_PADDED) {
    f = (int)(c / a.B);
    const int p = (int)(c - (int64_t)f * a.B);
    const int n = a.n_bins[f];
    j = p == a.B - 1 ? n - 1 : (p < n - 1 ? p : -1);
    if (j < 0) return ci;
  } else {
    // last feature whose first column is <= c (n_i >= 1, so offsets are strictly increasing)
    int lo = 0, hi = a.F - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.col_off[mid] <= c) lo = mid;
      else hi = mid - 1;
    }
    f = lo;
    j = (int)(c - a.col_off[f]);
  }
  const int n = a.n_bins[f];
  if (j < 0 || j >= n || n > a.B) return ci;  // offsets inconsistent with n_bins: written as padding
  ci.f = f;
  ci.e = a.edges[(int64_t)f * (a.B + 1) + j];
  ci.r = a.inv_w[(int64_t)f * a.B + j];
  const float inf = __int_as_float(0x7f800000);
  ci.lo = (n == 1 || j == 0) ? -inf : 0.f;
  ci.hi = (n == 1 || j == n - 1) ? inf : 1.f;
  return ci;
}

// clamp that keeps NaN (comparisons with NaN are false)
__device__ __forceinline__ float clamp_keep_nan(float v, float lo, float hi) {
  v = v < lo ? lo : v;
  return v > hi ? hi : v;
}

template <typename OT>
__device__ __forceinline__ void store4(OT* p, const float (&v)[4], bool vec_ok, int valid) {
  if constexpr (std::is_same<OT, float>::value) {
    if (vec_ok && valid == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
      return;
    }
  } else {
    if (vec_ok && valid == 4) {
      uint2 w;
      OT h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = Dt<OT>::from_f(v[e]);
      w.x = *reinterpret_cast<unsigned short*>(&h[0]) | ((unsigned)*reinterpret_cast<unsigned short*>(&h[1]) << 16);
      w.y = *reinterpret_cast<unsigned short*>(&h[2]) | ((unsigned)*reinterpret_cast<unsigned short*>(&h[3]) << 16);
      *reinterpret_cast<uint2*>(p) = w;
      return;
    }
  }
  for (int e = 0; e < valid; ++e) p[e] = Dt<OT>::from_f(v[e]);
}

// Forward: blockIdx.x = column tile of kEncTileCols columns (its column table
// is built once), blockIdx.y strides over the rows.  A warp stores 512
// contiguous bytes of a row per instruction.
template <typename OT>
__global__ void __launch_bounds__(kEncThreads) ple_enc_fwd_kernel(const EncArgs a) {
  __shared__ ColInfo sc[kEncTileCols];
  const int64_t C = a.total_cols;
  OT* out = reinterpret_cast<OT*>(a.out);
  // 16-byte (f32) / 8-byte (16-bit) stores need every row to start aligned
  const bool vec_ok = (C % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & (4 * sizeof(OT) - 1)) == 0);
  const int64_t c0 = (int64_t)blockIdx.x * kEncTileCols;
  for (int q = threadIdx.x; q < kEncTileCols; q += blockDim.x) {
    const int64_t c = c0 + q;
    sc[q] = c < C ? column_info(a, c) : ColInfo{-1, 0.f, 0.f, 0.f, 0.f};
  }
  __syncthreads();
  const int q0 = threadIdx.x * 4;
  const int valid = (int)min64(4, C - (c0 + q0));
  if (valid <= 0) return;
  ColInfo ci[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) ci[e] = sc[q0 + e];
  for (int64_t s = blockIdx.y; s < a.N; s += gridDim.y) {
    const float* xrow = a.x + s * a.F;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[e] = 0.f;
      if (ci[e].f >= 0) v[e] = clamp_keep_nan((__ldg(xrow + ci[e].f) - ci[e].e) * ci[e].r, ci[e].lo, ci[e].hi);
    }
    store4<OT>(out + s * C + c0 + q0, v, vec_ok, valid);
  }
}

// Backward: CTA = (kBwdRows rows) x (feature group of fg features).  The rows'
// gradient segment of the group is staged in shared memory with coalesced
// loads, then each (row, feature) pair sums its columns.
constexpr int kEncBwdRows = 8;

template <typename GT>
__global__ void __launch_bounds__(kEncThreads) ple_enc_bwd_kernel(const EncArgs a, int fg, int pitch) {
  extern __shared__ float sg[];  // [kEncBwdRows][pitch]
  const int64_t C = a.total_cols;
  const GT* g = reinterpret_cast<const GT*>(a.g);
  const int n_groups = (a.F + fg - 1) / fg;
  const int64_t row_blocks = (a.N + kEncBwdRows - 1) / kEncBwdRows;
  for (int64_t work = blockIdx.x; work < (int64_t)n_groups * row_blocks; work += gridDim.x) {
    const int grp = (int)(work % n_groups);
    const int64_t rb = work / n_groups;
    const int f_lo = grp * fg, f_hi = min(a.F, f_lo + fg);
    const int64_t cb = a.layout == PLE_ENC_PADDED ? (int64_t)f_lo * a.B : a.col_off[f_lo];
    const int64_t ce = a.layout == PLE_ENC_PADDED ? (int64_t)f_hi * a.B : a.col_off[f_hi];
    // staged width, bounded by the buffer and the row even if the offsets disagree with n_bins
    const int w = (cb < 0 || cb > C) ? 0 : (int)min64(min64(ce - cb, (int64_t)pitch - 1), C - cb);
    const int64_t s0 = rb * kEncBwdRows;
    const int nr = (int)min64(kEncBwdRows, a.N - s0);
    __syncthreads();  // previous work item finished with the staged rows
    for (int rr = 0; rr < nr; ++rr) {
      const GT* grow = g + (s0 + rr) * C + cb;
      for (int c = threadIdx.x; c < w; c += blockDim.x) sg[rr * pitch + c] = Dt<GT>::to_f(grow[c]);
    }
    __syncthreads();
    const int nf = f_hi - f_lo;
    for (int p = threadIdx.x; p < nr * nf; p += blockDim.x) {
      const int rr = p % nr, i = f_lo + p / nr;  // rows fastest: lanes of a feature read different rows
      const float xv = a.x[(s0 + rr) * a.F + i];
      const int n = a.n_bins[i];
      const float* er = a.edges + (int64_t)i * (a.B + 1);
      const float* rw = a.inv_w + (int64_t)i * a.B;
      const int off = (int)((a.layout == PLE_ENC_PADDED ? (int64_t)i * a.B : a.col_off[i]) - cb);
      const float* row = sg + rr * pitch + off;
      // columns of this feature inside the staged width (all of them for consistent offsets)
      const int span = a.layout == PLE_ENC_PADDED ? a.B : n;
      const int nn = (off < 0 || off + span > w || n > a.B) ? 0 : n;
      const float inf = __int_as_float(0x7f800000);
      float acc = 0.f;
      for (int j = 0; j < nn; ++j) {
        const int col = (a.layout == PLE_ENC_PADDED && j == n - 1) ? a.B - 1 : j;
        const float r = rw[j];
        const float t = (xv - er[j]) * r;
        const float lo = (n == 1 || j == 0) ? -inf : 0.f;
        const float hi = (n == 1 || j == n - 1) ? inf : 1.f;
        if (t >= lo && t <= hi) acc = fmaf(row[col], r, acc);
      }
      a.grad_x[(s0 + rr) * a.F + i] = acc;
    }
  }
}

template <typename OT>
int launch_enc_fwd_t(const EncArgs& a, cudaStream_t st) {
  const int64_t n_tiles = (a.total_cols + kEncTileCols - 1) / kEncTileCols;
  if (n_tiles > 0x7fffffff) return set_error(PLE_ERR_OVERFLOW, "encoding: too many columns");
  const int64_t per_tile = min64(min64(a.N, 65535), ceil_div<int64_t>(8L * device_sm_count(), n_tiles));
  dim3 grid((unsigned)n_tiles, (unsigned)(per_tile < 1 ? 1 : per_tile));
  ple_enc_fwd_kernel<OT><<<grid, kEncThreads, 0, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "encoding forward launch");
}

template <typename GT>
int launch_enc_bwd_t(const EncArgs& a, cudaStream_t st) {
  // feature groups of at most 2048 staged columns (B bounds a feature's columns)
  const int fg = (int)(a.B >= 2048 ? 1 : 2048 / a.B);
  const int64_t wmax = (int64_t)fg * a.B;
  const int pitch = (int)(wmax | 1);  // odd pitch: rows start on different banks
  const size_t smem = (size_t)kEncBwdRows * pitch * sizeof(float);
  auto kern = ple_enc_bwd_kernel<GT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(encoding backward)");
  const int64_t work = (int64_t)((a.F + fg - 1) / fg) * ((a.N + kEncBwdRows - 1) / kEncBwdRows);
  const int grid = (int)min64(work, 4L * device_sm_count());
  kern<<<grid, kEncThreads, smem, st>>>(a, fg, pitch);
  e = cudaGetLastError();
  return e == cudaSuccess ? PLE_OK : set_cuda_error(e, "encoding backward launch");
}

}  // namespace

int launch_encoding_forward(const EncArgs& a, int output_dtype, cudaStream_t st) {
  switch (output_dtype) {
    case PLE_DTYPE_F32: return launch_enc_fwd_t<float>(a, st);
    case PLE_DTYPE_BF16: return launch_enc_fwd_t<__nv_bfloat16>(a, st);
    case PLE_DTYPE_F16: return launch_enc_fwd_t<__half>(a, st);
    default: return set_error(PLE_ERR_INVALID_ARGUMENT, "encoding: output dtype must be F32, F16 or BF16");
  }
}

int launch_encoding_backward(const EncArgs& a, int grad_dtype, cudaStream_t st) {
  switch (grad_dtype) {
    case PLE_DTYPE_F32: return launch_enc_bwd_t<float>(a, st);
    case PLE_DTYPE_BF16: return launch_enc_bwd_t<__nv_bfloat16>(a, st);
    case PLE_DTYPE_F16: return launch_enc_bwd_t<__half>(a, st);
    default: return set_error(PLE_ERR_INVALID_ARGUMENT, "encoding: grad dtype must be F32, F16 or BF16");
  }
}

}  // namespace ple
