// ple_forward.cu - fused PLE forward for sm_100a.
//
// One persistent CTA owns a chunk of Fc consecutive features and a contiguous
// range of samples.  It stages, once, the chunk's edges (transposed,
// +inf-padded to a power of two), inverse widths and two tables in shared
// memory, laid out bin-major [k][feature][d]:
//     T[k][i][:] = sum_{j<k} q(W[i, j, :])          (prefix of full bins)
//     S[k][i][:] = q(W[i, phys(k), :])              (slope of the active bin)
// so that x_ple = fma(q(t), S[k], T[k]) (reference forward_cuda.cu:135-176,
// 258-273).  Then, per tile of samples:
//   phase 1 (one thread per (sample, feature) pair): coalesced x load, bin
//            search, position t, optional bin-index store;
//   phase 2 (one thread per VEC-wide chunk of an output row): T/S lookup,
//            epilogue (bias / ReLU / linear0), coalesced streaming store.
// With the bin-major layout and Fc*D a multiple of 32, the VEC-wide table
// reads of consecutive threads land in distinct banks whatever their bins.
// Each thread keeps one (feature, chunk) column for the whole kernel, so its
// epilogue parameters live in registers.
#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

template <typename QT, typename OT, int VEC>
__global__ void __launch_bounds__(kFwdMaxThreads)
ple_fwd_kernel(const FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int Fc = a.Fc, B = a.B, D = a.D, pow2 = a.pow2;
  const int nc = D / VEC;
  const int R = Fc * nc;
  float* sT = reinterpret_cast<float*>(smem_raw);
  float* sS = sT + B * Fc * D;
  float2* sKT = reinterpret_cast<float2*>(sS + B * Fc * D);
  float* sX = reinterpret_cast<float*>(sKT + a.S_t * Fc);
  float* sE = sX + a.S_t * Fc;
  float* sR = sE + pow2 * Fc;
  int* sN = reinterpret_cast<int*>(sR + B * Fc);

  const int chunk = blockIdx.x % a.n_chunks;
  const int part = blockIdx.x / a.n_chunks;
  const int f0 = chunk * Fc;
  const int fc = min(Fc, a.F - f0);
  const int64_t s_begin = a.N * part / a.n_parts;
  const int64_t s_end = a.N * (part + 1) / a.n_parts;
  const int tid = threadIdx.x, nthr = blockDim.x;

  // ---- prologue: per-feature tables
  for (int i = tid; i < Fc; i += nthr) {
    int n = i < fc ? a.n_bins[f0 + i] : 1;
    sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  __syncthreads();
  for (int idx = tid; idx < pow2 * Fc; idx += nthr) {
    const int j = idx / Fc, i = idx - j * Fc;
    float e = __int_as_float(0x7f800000);
    if (i < fc && j <= sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j];
    sE[idx] = e;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {
    const int j = idx / Fc, i = idx - j * Fc;
    sR[idx] = (i < fc && j < sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
  }
  // W rows of the chunk are contiguous: [fc][B][D]; scatter to logical order.
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int idx = tid; idx < fc * B * D; idx += nthr) {
    const int i = idx / (B * D);
    const int rem = idx - i * B * D;
    const int p = rem / D, d = rem - p * D;
    const int n = sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) sS[(lg * Fc + i) * D + d] = quantize<QT>(Wc[idx]);
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = sN[i];
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int o = (j * Fc + i) * D + d;
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
    if (a.epi == kEpiA) {
      ep0 = ldg_f32vec<float, VEC>(a.bias + po);
    } else if (a.epi == kEpiB) {
      ep0 = ldg_f32vec<float, VEC>(a.w0 + po);
      ep1 = ldg_f32vec<float, VEC>(a.b0 + po);
    }
  }
  __syncthreads();

  OT* out = reinterpret_cast<OT*>(a.out);
  for (int64_t t0 = s_begin; t0 < s_end; t0 += a.S_t) {
    const int ns = (int)min64(a.S_t, s_end - t0);
    // ---- phase 1: bins and positions for ns x Fc pairs
    for (int p = tid; p < ns * Fc; p += nthr) {
      const int s = p / Fc, i = p - s * Fc;
      float2 kt = make_float2(0.0f, 0.0f);
      if (i < fc) {
        const int64_t pair = (t0 + s) * a.F + f0 + i;
        const float xv = a.x[pair];
        const int k = logical_bin(edge_count(xv, sE, Fc, i, pow2), sN[i]);
        const float t = (xv - sE[k * Fc + i]) * sR[k * Fc + i];
        kt = make_float2(__int_as_float(k), quantize<QT>(t));
        sX[p] = xv;
        if (a.bin_idx != nullptr) {
          if (a.bin_idx_bytes == 1) reinterpret_cast<uint8_t*>(a.bin_idx)[pair] = (uint8_t)k;
          else if (a.bin_idx_bytes == 2) reinterpret_cast<int16_t*>(a.bin_idx)[pair] = (int16_t)k;
          else reinterpret_cast<int32_t*>(a.bin_idx)[pair] = k;
        }
      }
      sKT[p] = kt;
    }
    __syncthreads();
    // ---- phase 2: output chunks
    if (col_live) {
      for (int s = tid / R; s < ns; s += s_step) {
        const float2 kt = sKT[s * Fc + ci];
        const int k = __float_as_int(kt.x);
        const float tq = kt.y;
        const int to = (k * Fc + ci) * D + cd;
        const FV<VEC> tv = lds<VEC>(sT + to);
        const FV<VEC> sv = lds<VEC>(sS + to);
        FV<VEC> y;
        const float xv = a.epi == kEpiB ? sX[s * Fc + ci] : 0.0f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          float v = quantize<QT>(fmaf(tq, sv.v[e], tv.v[e]));
          if (a.epi == kEpiA) v += ep0.v[e];
          if (a.relu) v = relu_f(v);
          if (a.epi == kEpiB) v = fmaf(xv, ep0.v[e], ep1.v[e]) + v;
          y.v[e] = v;
        }
        stg_stream<OT, VEC>(out + ((t0 + s) * a.F + f0 + ci) * D + cd, y);
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ launch
template <typename QT, typename OT, int VEC>
static int launch_fwd_t(const FwdArgs& a, size_t smem, int threads, cudaStream_t st) {
  auto kern = ple_fwd_kernel<QT, OT, VEC>;
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

template <typename QT, typename OT>
static int launch_fwd_vec(const FwdArgs& a, int vec, size_t smem, int threads, cudaStream_t st) {
  switch (vec) {
    case 4: return launch_fwd_t<QT, OT, 4>(a, smem, threads, st);
    case 2: return launch_fwd_t<QT, OT, 2>(a, smem, threads, st);
    default: return launch_fwd_t<QT, OT, 1>(a, smem, threads, st);
  }
}

int launch_forward(FwdArgs a, int compute_dtype, int output_dtype, int vec, cudaStream_t st) {
  // feature chunk: power of two, tables <= kFwdTableBudget, R = Fc * D / vec <= kFwdMaxThreads
  const int nc = a.D / vec;
  int Fc = 16;
  auto tables = [&](int fc) { return (size_t)2 * a.B * fc * a.D * sizeof(float); };
  while (Fc > 1 && (tables(Fc) > kFwdTableBudget || Fc * nc > kFwdMaxThreads || Fc / 2 >= a.F))
    Fc >>= 1;
  if (Fc * nc > kFwdMaxThreads) return set_error(PLE_ERR_UNSUPPORTED, "forward: d_embedding too large");
  a.Fc = Fc;
  a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
  int pow2 = 1;
  while (pow2 < a.B + 1) pow2 <<= 1;
  a.pow2 = pow2;
  const int R = Fc * nc;
  const int threads = R * (kFwdMaxThreads / R);
  a.S_t = kFwdPairsPerTile / Fc;
  if (a.S_t < 1) a.S_t = 1;
  const size_t smem = tables(Fc) + (size_t)a.S_t * Fc * (sizeof(float2) + sizeof(float)) +
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
