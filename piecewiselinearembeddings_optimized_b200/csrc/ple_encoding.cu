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
  // the common case: the four columns belong to one feature (n_i >= 4), so one x per row; four rows per
  // iteration with their loads issued first
  const bool one_f = ci[0].f >= 0 && ci[1].f == ci[0].f && ci[2].f == ci[0].f && ci[3].f == ci[0].f;
  for (int64_t s = (int64_t)blockIdx.y * 4; s < a.N; s += (int64_t)gridDim.y * 4) {
    const int nrow = (int)min64(4, a.N - s);
    if (one_f) {
      float xv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) xv[r] = r < nrow ? __ldg(a.x + (s + r) * a.F + ci[0].f) : 0.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (r < nrow) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = clamp_keep_nan((xv[r] - ci[e].e) * ci[e].r, ci[e].lo, ci[e].hi);
          store4<OT>(out + (s + r) * C + c0 + q0, v, vec_ok, valid);
        }
      }
    } else {
      for (int r = 0; r < nrow; ++r) {
        const float* xrow = a.x + (s + r) * a.F;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[e] = 0.f;
          if (ci[e].f >= 0) v[e] = clamp_keep_nan((__ldg(xrow + ci[e].f) - ci[e].e) * ci[e].r, ci[e].lo, ci[e].hi);
        }
        store4<OT>(out + (s + r) * C + c0 + q0, v, vec_ok, valid);
      }
    }
  }
}

// Four consecutive gradients (aligned to four elements) as fp32.
template <typename GT>
__device__ __forceinline__ void load4(const GT* p, float (&v)[4]) {
  if constexpr (std::is_same<GT, float>::value) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
    const GT* h = reinterpret_cast<const GT*>(&q);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = Dt<GT>::to_f(h[e]);
  }
}

// Backward: blockIdx.x = feature group (at most kEncGroupCols columns; its
// column table is built once), blockIdx.y strides over blocks of kEncBwdRows
// rows.  Per block, threads take the group's columns of each row in order
// (coalesced gradient loads) and stage each column's contribution
// g * r * [lo <= t <= hi] in shared memory; then each (row, feature) sums its
// columns.
constexpr int kEncBwdRows = 8;
constexpr int kEncGroupCols = 2048;

template <typename GT>
__global__ void __launch_bounds__(kEncThreads) ple_enc_bwd_kernel(const EncArgs a, int fg, int pitch) {
  extern __shared__ float smem_f[];
  ColInfo* sc = reinterpret_cast<ColInfo*>(smem_f);                // [pitch] column table of the group
  float* sv = smem_f + (size_t)pitch * (sizeof(ColInfo) / 4);       // [kEncBwdRows][pitch] contributions
  float* sx = sv + (size_t)kEncBwdRows * pitch;                     // [kEncBwdRows][fg] x of the block
  const int64_t C = a.total_cols;
  const GT* g = reinterpret_cast<const GT*>(a.g);
  const int grp = blockIdx.x;
  const int f_lo = grp * fg, f_hi = min(a.F, f_lo + fg);
  const int64_t cb = a.layout == PLE_ENC_PADDED ? (int64_t)f_lo * a.B : a.col_off[f_lo];
  const int64_t ce = a.layout == PLE_ENC_PADDED ? (int64_t)f_hi * a.B : a.col_off[f_hi];
  // width bounded by the buffers and the row even if the offsets disagree with n_bins
  const int w = (cb < 0 || cb > C) ? 0 : (int)min64(min64(ce - cb, (int64_t)pitch - 1), C - cb);
  for (int c = threadIdx.x; c < w; c += blockDim.x) {
    ColInfo ci = column_info(a, cb + c);
    if (ci.f < f_lo || ci.f >= f_hi) ci.f = -1;  // (only with inconsistent offsets)
    sc[c] = ci;
  }
  const int nf = f_hi - f_lo;
  // vector loads of four gradients need every chunk start aligned: row length, group start and base
  const bool vec_g = ((C | cb) & 3) == 0 && (reinterpret_cast<uintptr_t>(g) & (4 * sizeof(GT) - 1)) == 0;
  const int64_t row_blocks = (a.N + kEncBwdRows - 1) / kEncBwdRows;
  for (int64_t rb = blockIdx.y; rb < row_blocks; rb += gridDim.y) {
    const int64_t s0 = rb * kEncBwdRows;
    const int nr = (int)min64(kEncBwdRows, a.N - s0);
    __syncthreads();  // column table ready / previous block's sums done
    for (int p = threadIdx.x; p < nr * nf; p += blockDim.x) {
      const int rr = p / nf, i = p - rr * nf;
      sx[rr * fg + i] = a.x[(s0 + rr) * a.F + f_lo + i];
    }
    __syncthreads();
    // four columns per thread and chunk; the chunk's gradients of all the block's rows are loaded before any
    // is used (the loads would otherwise serialise behind the shared-memory stores)
    const int nchunks = (w + 3) >> 2;
    for (int q = threadIdx.x; q < nchunks; q += blockDim.x) {
      const int c = q << 2;
      const int cn = min(4, w - c);
      float gv[kEncBwdRows][4];
#pragma unroll
      for (int rr = 0; rr < kEncBwdRows; ++rr) {
        if (rr < nr) {
          const GT* gp = g + (s0 + rr) * C + cb + c;
          if (vec_g && cn == 4) {
            load4<GT>(gp, gv[rr]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) gv[rr][e] = e < cn ? Dt<GT>::to_f(gp[e]) : 0.f;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (e < cn) {
          const ColInfo ci = sc[c + e];
#pragma unroll
          for (int rr = 0; rr < kEncBwdRows; ++rr) {
            if (rr < nr) {
              float v = 0.f;
              if (ci.f >= 0) {
                const float t = (sx[rr * fg + ci.f - f_lo] - ci.e) * ci.r;
                if (t >= ci.lo && t <= ci.hi) v = gv[rr][e] * ci.r;
              }
              sv[rr * pitch + c + e] = v;
            }
          }
        }
      }
    }
    __syncthreads();
    for (int p = threadIdx.x; p < nr * nf; p += blockDim.x) {
      const int rr = p % nr, i = f_lo + p / nr;  // rows fastest: lanes of a feature read different rows
      const int64_t c_i = a.layout == PLE_ENC_PADDED ? (int64_t)i * a.B : a.col_off[i];
      const int64_t c_n = a.layout == PLE_ENC_PADDED ? c_i + a.B : a.col_off[i + 1];
      const int lo = (int)max64(0, c_i - cb), hi = (int)min64(w, c_n - cb);
      const float* row = sv + rr * pitch;
      float acc = 0.f;
      for (int c = lo; c < hi; ++c) acc += row[c];
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
  // feature groups of at most kEncGroupCols columns (B bounds a feature's columns)
  const int fg = (int)(a.B >= kEncGroupCols ? 1 : kEncGroupCols / a.B);
  const int64_t wmax = (int64_t)fg * a.B;
  const int pitch = (int)(wmax | 1);  // odd pitch: rows start on different banks
  const size_t smem = (size_t)pitch * (sizeof(ColInfo) + kEncBwdRows * sizeof(float)) +
                      (size_t)kEncBwdRows * fg * sizeof(float);
  auto kern = ple_enc_bwd_kernel<GT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(encoding backward)");
  const int n_groups = (a.F + fg - 1) / fg;
  const int64_t row_blocks = (a.N + kEncBwdRows - 1) / kEncBwdRows;
  const int64_t per_group = min64(min64(row_blocks, 65535), ceil_div<int64_t>(4L * device_sm_count(), n_groups));
  dim3 grid((unsigned)n_groups, (unsigned)(per_group < 1 ? 1 : per_group));
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
