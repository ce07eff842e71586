// ple_forward.cu - fused PLE forward for sm_100a.
//
// One persistent CTA owns a chunk of Fc (power of two) consecutive features
// and a contiguous range of samples.  It stages, once, the chunk's edges
// (transposed, +inf-padded to a power of two), inverse widths and two tables
// in shared memory, laid out bin-major [k][feature][d]:
//     T[k][i][:] = sum_{j<k} q(W[i, j, :])          (prefix of full bins)
//     S[k][i][:] = q(W[i, phys(k), :])              (slope of the active bin)
// so that x_ple = q(fma(q(t), S[k], T[k])) (reference forward_cuda.cu:135-176,
// 258-273).  Then, per tile of samples:
//   x tile   [S_t][Fc] arrives by cp.async, double-buffered one tile ahead;
//   phase 1  one thread per (sample, feature): bin search and q(t) -> smem
//            (+ bin-index store for the reference op);
//   phase 2  one thread per VEC-wide chunk of an output row, each thread on a
//            fixed column (its epilogue parameters live in registers), two
//            samples per iteration: T/S lookup, epilogue, streaming store.
// The epilogue (none / A / B) and ReLU are template parameters, the math
// uses packed fp32x2 instructions and packed bf16/fp16 conversions.  With
// the bin-major layout and Fc*D a multiple of 32, the table reads of
// consecutive threads land in distinct banks whatever their bins.
#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"

namespace ple {

// y = epilogue(q(fma(tq, S, T))) for VEC elements; rounding through QT emulates
// the reference's low-precision x_ple (its output cast), then the fp32 epilogue.
template <typename QT, int VEC, int EPI, bool RELU>
__device__ __forceinline__ FV<VEC> fwd_chunk(float tq, const FV<VEC>& T, const FV<VEC>& S, float xv,
                                             const FV<VEC>& ep0, const FV<VEC>& ep1) {
  FV<VEC> y;
  if constexpr (VEC >= 2) {
    const f2_t t2 = pack2(tq, tq);
    const f2_t x2 = pack2(xv, xv);
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      f2_t p = fma2(t2, pack2(S.v[e], S.v[e + 1]), pack2(T.v[e], T.v[e + 1]));
      float lo, hi;
      unpack2(p, lo, hi);
      round2<QT>(lo, hi);
      if constexpr (EPI == kEpiA) {
        p = add2(pack2(lo, hi), pack2(ep0.v[e], ep0.v[e + 1]));
        unpack2(p, lo, hi);
      }
      if constexpr (RELU) {
        lo = relu_nan(lo);
        hi = relu_nan(hi);
      }
      if constexpr (EPI == kEpiB) {
        const f2_t lin = fma2(x2, pack2(ep0.v[e], ep0.v[e + 1]), pack2(ep1.v[e], ep1.v[e + 1]));
        unpack2(add2(lin, pack2(lo, hi)), lo, hi);
      }
      y.v[e] = lo;
      y.v[e + 1] = hi;
    }
  } else {
    float v = quantize<QT>(fmaf(tq, S.v[0], T.v[0]));
    if constexpr (EPI == kEpiA) v += ep0.v[0];
    if constexpr (RELU) v = relu_nan(v);
    if constexpr (EPI == kEpiB) v = fmaf(xv, ep0.v[0], ep1.v[0]) + v;
    y.v[0] = v;
  }
  return y;
}

template <typename OT, int VEC>
__device__ __forceinline__ void store_out(OT* p, const FV<VEC>& y) {
  if constexpr (!std::is_same<OT, float>::value && VEC == 4) {
    uint2 u = make_uint2(cvt_pack<OT>(y.v[0], y.v[1]), cvt_pack<OT>(y.v[2], y.v[3]));
    __stcs(reinterpret_cast<uint2*>(p), u);
  } else {
    stg_stream<OT, VEC>(p, y);
  }
}

template <typename QT, typename OT, int VEC, int EPI, bool RELU>
__global__ void __launch_bounds__(kFwdMaxThreads)
ple_fwd_kernel(const FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lgFc = a.lgFc;
  const int Fc = 1 << lgFc, B = a.B, D = a.D, pow2 = a.pow2, S_t = a.S_t;
  const int nc = D / VEC;
  const int R = Fc * nc;
  float* sT = reinterpret_cast<float*>(smem_raw);
  float* sS = sT + B * Fc * D;
  float2* sKT = reinterpret_cast<float2*>(sS + B * Fc * D);
  float* sXb = reinterpret_cast<float*>(sKT + S_t * Fc);  // [2][S_t][Fc]
  float* sE = sXb + 2 * S_t * Fc;
  float* sR = sE + pow2 * Fc;
  int* sN = reinterpret_cast<int*>(sR + B * Fc);

  const int chunk = blockIdx.x % a.n_chunks;
  const int part = blockIdx.x / a.n_chunks;
  const int f0 = chunk << lgFc;
  const int fc = min(Fc, a.F - f0);
  const int64_t s_begin = a.N * part / a.n_parts;
  const int64_t s_end = a.N * (part + 1) / a.n_parts;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const bool x_vec4 = a.x_vec4 && fc == Fc;

  // x tile loader: rows [t0, t0 + ns) x features [f0, f0 + Fc) -> dst[s][i]
  auto load_x = [&](int64_t t0, int ns, float* dst) {
    if (x_vec4) {
      const int per_row = Fc >> 2;
      for (int q = tid; q < ns * per_row; q += nthr) {
        const int s = q / per_row, c4 = q - s * per_row;
        cp_async16(dst + s * Fc + 4 * c4, a.x + (t0 + s) * a.F + f0 + 4 * c4);
      }
    } else {
      for (int q = tid; q < (ns << lgFc); q += nthr) {
        const int s = q >> lgFc, i = q & (Fc - 1);
        if (i < fc) cp_async4(dst + q, a.x + (t0 + s) * a.F + f0 + i);
        else dst[q] = 0.0f;
      }
    }
    cp_async_commit();
  };
  if (s_begin < s_end) load_x(s_begin, (int)min64(S_t, s_end - s_begin), sXb);

  // ---- prologue: per-feature tables (overlaps the first x tile copy)
  for (int i = tid; i < Fc; i += nthr) {
    int n = i < fc ? a.n_bins[f0 + i] : 1;
    sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  __syncthreads();
  for (int idx = tid; idx < pow2 * Fc; idx += nthr) {
    const int j = idx >> lgFc, i = idx & (Fc - 1);
    float e = __int_as_float(0x7f800000);
    if (i < fc && j <= sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j];
    sE[idx] = e;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {
    const int j = idx >> lgFc, i = idx & (Fc - 1);
    sR[idx] = (i < fc && j < sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
  }
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int idx = tid; idx < fc * B * D; idx += nthr) {
    const int i = idx / (B * D);
    const int rem = idx - i * B * D;
    const int p = rem / D, d = rem - p * D;
    const int n = sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) sS[((lg << lgFc) + i) * D + d] = quantize<QT>(Wc[idx]);
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = sN[i];
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int o = ((j << lgFc) + i) * D + d;
      sT[o] = acc;
      acc += sS[o];
    }
  }

  // ---- this thread's fixed output column (nthr is a multiple of R)
  const int col = tid % R;
  const int ci = col / nc;
  const int cd = (col - ci * nc) * VEC;
  const int s_step = nthr / R;
  const bool col_live = ci < fc;
  FV<VEC> ep0, ep1;
#pragma unroll
  for (int e = 0; e < VEC; ++e) { ep0.v[e] = 0.0f; ep1.v[e] = 0.0f; }
  if (col_live) {
    const int64_t po = (int64_t)(f0 + ci) * D + cd;
    if constexpr (EPI == kEpiA) ep0 = ldg_f32vec<float, VEC>(a.bias + po);
    if constexpr (EPI == kEpiB) {
      ep0 = ldg_f32vec<float, VEC>(a.w0 + po);
      ep1 = ldg_f32vec<float, VEC>(a.b0 + po);
    }
  }

  OT* out = reinterpret_cast<OT*>(a.out);
  int buf = 0;
  for (int64_t t0 = s_begin; t0 < s_end; t0 += S_t, buf ^= 1) {
    const int ns = (int)min64(S_t, s_end - t0);
    const float* sX = sXb + buf * S_t * Fc;
    cp_async_wait_all();
    __syncthreads();  // x tile visible; previous phase 2 done with sKT and the other buffer
    if (t0 + S_t < s_end) load_x(t0 + S_t, (int)min64(S_t, s_end - t0 - S_t), sXb + (buf ^ 1) * S_t * Fc);
    // ---- phase 1: bins and positions
    for (int p = tid; p < (ns << lgFc); p += nthr) {
      const int i = p & (Fc - 1);
      float2 kt = make_float2(0.0f, 0.0f);
      if (i < fc) {
        const float xv = sX[p];
        const int k = logical_bin(edge_count(xv, sE, Fc, i, pow2), sN[i]);
        const float t = (xv - sE[(k << lgFc) + i]) * sR[(k << lgFc) + i];
        kt = make_float2(__int_as_float(k), quantize<QT>(t));
        if (a.bin_idx != nullptr) {
          const int64_t pair = (t0 + (p >> lgFc)) * a.F + f0 + i;
          if (a.bin_idx_bytes == 1) reinterpret_cast<uint8_t*>(a.bin_idx)[pair] = (uint8_t)k;
          else if (a.bin_idx_bytes == 2) reinterpret_cast<int16_t*>(a.bin_idx)[pair] = (int16_t)k;
          else reinterpret_cast<int32_t*>(a.bin_idx)[pair] = k;
        }
      }
      sKT[p] = kt;
    }
    __syncthreads();
    // ---- phase 2: output chunks, two samples per iteration
    if (col_live) {
      OT* orow = out + ((t0 * a.F) + f0 + ci) * (int64_t)D + cd;
      const int64_t ostride = (int64_t)a.F * D;
      for (int s = tid / R; s < ns; s += 2 * s_step) {
        const int s2 = s + s_step;
        const bool two = s2 < ns;
        const float2 kt = sKT[(s << lgFc) + ci];
        const float2 kt2 = two ? sKT[(s2 << lgFc) + ci] : kt;
        const int to = ((__float_as_int(kt.x) << lgFc) + ci) * D + cd;
        const int to2 = ((__float_as_int(kt2.x) << lgFc) + ci) * D + cd;
        const FV<VEC> tv = lds<VEC>(sT + to), sv = lds<VEC>(sS + to);
        const FV<VEC> tv2 = lds<VEC>(sT + to2), sv2 = lds<VEC>(sS + to2);
        const float xv = EPI == kEpiB ? sX[(s << lgFc) + ci] : 0.0f;
        const float xv2 = (EPI == kEpiB && two) ? sX[(s2 << lgFc) + ci] : 0.0f;
        const FV<VEC> y = fwd_chunk<QT, VEC, EPI, RELU>(kt.y, tv, sv, xv, ep0, ep1);
        const FV<VEC> y2 = fwd_chunk<QT, VEC, EPI, RELU>(kt2.y, tv2, sv2, xv2, ep0, ep1);
        store_out<OT, VEC>(orow + s * ostride, y);
        if (two) store_out<OT, VEC>(orow + s2 * ostride, y2);
      }
    }
  }
}

// ------------------------------------------------------------------ launch
template <typename QT, typename OT, int VEC, int EPI, bool RELU>
static int launch_fwd_t(const FwdArgs& a, size_t smem, int threads, cudaStream_t st) {
  auto kern = ple_fwd_kernel<QT, OT, VEC, EPI, RELU>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(forward)");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess) return set_cuda_error(e, "occupancy(forward)");
  if (per_sm < 1) return set_error(PLE_ERR_UNSUPPORTED, "forward: tables do not fit in shared memory");
  FwdArgs b = a;
  const int64_t slots = (int64_t)device_sm_count() * per_sm;
  int64_t parts = slots / b.n_chunks;
  const int64_t max_parts = ceil_div<int64_t>(b.N, 32);
  parts = parts < 1 ? 1 : (parts > max_parts ? max_parts : parts);
  b.n_parts = (int)parts;
  const int64_t grid = (int64_t)b.n_chunks * parts;
  if (grid > 0x7fffffff) return set_error(PLE_ERR_OVERFLOW, "forward grid too large");
  kern<<<(unsigned)grid, threads, smem, st>>>(b);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "forward launch");
  return PLE_OK;
}

template <typename QT, typename OT, int VEC>
static int launch_fwd_epi(const FwdArgs& a, size_t smem, int threads, cudaStream_t st) {
  if (a.epi == kEpiB) {
    return a.relu ? launch_fwd_t<QT, OT, VEC, kEpiB, true>(a, smem, threads, st)
                  : launch_fwd_t<QT, OT, VEC, kEpiB, false>(a, smem, threads, st);
  }
  if (a.epi == kEpiA) {
    return a.relu ? launch_fwd_t<QT, OT, VEC, kEpiA, true>(a, smem, threads, st)
                  : launch_fwd_t<QT, OT, VEC, kEpiA, false>(a, smem, threads, st);
  }
  return a.relu ? launch_fwd_t<QT, OT, VEC, kEpiNone, true>(a, smem, threads, st)
                : launch_fwd_t<QT, OT, VEC, kEpiNone, false>(a, smem, threads, st);
}

template <typename QT, typename OT>
static int launch_fwd_vec(const FwdArgs& a, int vec, size_t smem, int threads, cudaStream_t st) {
  if (vec == 4) return launch_fwd_epi<QT, OT, 4>(a, smem, threads, st);
  return launch_fwd_epi<QT, OT, 1>(a, smem, threads, st);
}

int launch_forward(FwdArgs a, int compute_dtype, int output_dtype, int vec, cudaStream_t st) {
  if (vec != 4) vec = 1;
  // feature chunk: power of two, tables <= kFwdTableBudget, R = Fc * D / vec <= kFwdMaxThreads
  const int nc = a.D / vec;
  int lg = 4;
  auto tables = [&](int fc) { return (size_t)2 * a.B * fc * a.D * sizeof(float); };
  while (lg > 0 && (tables(1 << lg) > kFwdTableBudget || (1 << lg) * nc > kFwdMaxThreads ||
                    (1 << (lg - 1)) >= a.F))
    --lg;
  const int Fc = 1 << lg;
  if (Fc * nc > kFwdMaxThreads) return set_error(PLE_ERR_UNSUPPORTED, "forward: d_embedding too large");
  a.lgFc = lg;
  a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
  int pow2 = 1;
  while (pow2 < a.B + 1) pow2 <<= 1;
  a.pow2 = pow2;
  const int R = Fc * nc;
  const int threads = R * (kFwdMaxThreads / R);
  a.S_t = kFwdPairsPerTile / Fc;
  if (a.S_t < 1) a.S_t = 1;
  a.x_vec4 = (Fc >= 4) && (a.F % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  const size_t smem = tables(Fc) + (size_t)a.S_t * Fc * (sizeof(float2) + 2 * sizeof(float)) +
                      (size_t)pow2 * Fc * sizeof(float) + (size_t)a.B * Fc * sizeof(float) +
                      (size_t)Fc * sizeof(int);
  if (smem > device_max_smem_optin())
    return set_error(PLE_ERR_UNSUPPORTED, "forward: shared memory budget exceeded");
  const int q = compute_dtype, o = output_dtype;
  if (q == PLE_DTYPE_F32 && o == PLE_DTYPE_F32) return launch_fwd_vec<float, float>(a, vec, smem, threads, st);
  if (q == PLE_DTYPE_BF16 && o == PLE_DTYPE_BF16) return launch_fwd_vec<__nv_bfloat16, __nv_bfloat16>(a, vec, smem, threads, st);
  if (q == PLE_DTYPE_BF16 && o == PLE_DTYPE_F32) return launch_fwd_vec<__nv_bfloat16, float>(a, vec, smem, threads, st);
  if (q == PLE_DTYPE_F16 && o == PLE_DTYPE_F16) return launch_fwd_vec<__half, __half>(a, vec, smem, threads, st);
  if (q == PLE_DTYPE_F16 && o == PLE_DTYPE_F32) return launch_fwd_vec<__half, float>(a, vec, smem, threads, st);
  if (q == PLE_DTYPE_F32 && o == PLE_DTYPE_BF16) return launch_fwd_vec<float, __nv_bfloat16>(a, vec, smem, threads, st);
  return set_error(PLE_ERR_UNSUPPORTED, "forward: unsupported (compute, output) dtype pair");
}

}  // namespace ple
