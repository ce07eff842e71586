// ple_forward.cu - fused PLE forward for sm_100a.
//
// The grid is persistent (SMs x resident CTAs) and cut into slots of m CTAs;
// slot j owns an equal contiguous range of the flattened (chunk group, sample)
// space, and member i of the slot takes chunk g m + i of group g, so that the
// members read the x pieces of one 128-byte line together.  A CTA has one or a
// few (chunk of Fc consecutive features, sample range) segments.  Per segment it
// stages the chunk's search keys (interior edges e_1 .. e_{n-1}, +inf padded
// to 2^L - 1), {e_k, r_k} pairs and two tables in shared memory, the tables
// laid out bin-major [k][feature][d]:
//     T[k][i][:] = sum_{j<k} q(W[i, j, :])          (prefix of full bins)
//     S[k][i][:] = q(W[i, phys(k), :])              (slope of the active bin)
// so that x_ple = q(fma(q(t), S[k], T[k])) (reference forward_cuda.cu:135-176,
// 258-273).  Then, per tile of samples:
//   x tile   [S_t][Fc] arrives by cp.async, double-buffered one tile ahead;
//   phase 1  one thread per (sample, feature), two pairs of one feature at a time so
//            that their searches overlap: L-probe bin search, {k, q(t), x} -> smem
//            (+ bin-index store for the reference op);
//   phase 2  one thread per VEC-wide chunk of an output row, each thread on a
//            fixed column (its epilogue parameters live in registers): one
//            16-byte record (read one sample ahead), two table reads, epilogue,
//            streaming store.
// The epilogue (none / A / B) and ReLU are template parameters; the inner
// loop is kept to a minimum of instructions (the kernel is issue-bound
// before it is bandwidth-bound).  With
// the bin-major layout and Fc*D a multiple of 32, the table reads of
// consecutive threads land in distinct banks whatever their bins.
#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"
#include "ple_fwd_math.cuh"

namespace ple {

template <typename OT, int VEC>
__device__ __forceinline__ void store_out(OT* p, const FV<VEC>& y) {
  if constexpr (!std::is_same<OT, float>::value && VEC == 4) {
    uint2 u = make_uint2(cvt_pack<OT>(y.v[0], y.v[1]), cvt_pack<OT>(y.v[2], y.v[3]));
    __stcs(reinterpret_cast<uint2*>(p), u);
  } else {
    stg_stream<OT, VEC>(p, y);
  }
}

// Shared-memory layout of one CTA (sizes from FwdArgs).
struct FwdLayout {
  float *sT, *sS, *sXb, *sK;
  float2* sL;
  float4* sQ;
  int* sN;
};

__host__ __device__ __forceinline__ size_t fwd_layout(const FwdArgs& a, FwdLayout* L, unsigned char* base) {
  const int Fc = 1 << a.lgFc;
  const size_t tab = (size_t)a.B * Fc * a.D;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 15) & ~(size_t)15;
    return base + o;
  };
  unsigned char* pT = take(2 * tab * 4);
  unsigned char* pQ = take((size_t)a.S_t * Fc * 16);
  unsigned char* pX = take((size_t)2 * a.S_t * Fc * 4);
  unsigned char* pE = take((size_t)Fc * a.ldK * 4);
  unsigned char* pR = take((size_t)Fc * a.B * 8);
  unsigned char* pN = take((size_t)Fc * 4);
  if (L) {
    L->sT = reinterpret_cast<float*>(pT);
    L->sS = L->sT + tab;
    L->sQ = reinterpret_cast<float4*>(pQ);
    L->sXb = reinterpret_cast<float*>(pX);
    L->sK = reinterpret_cast<float*>(pE);
    L->sL = reinterpret_cast<float2*>(pR);
    L->sN = reinterpret_cast<int*>(pN);
  }
  return off;
}

// Bin index k of one (sample, feature) pair into the reference op's bin-index output.
__device__ __forceinline__ void store_bin(const FwdArgs& a, int64_t pair, int k) {
  if (a.bin_idx_bytes == 1) reinterpret_cast<uint8_t*>(a.bin_idx)[pair] = (uint8_t)k;
  else if (a.bin_idx_bytes == 2) reinterpret_cast<int16_t*>(a.bin_idx)[pair] = (int16_t)k;
  else reinterpret_cast<int32_t*>(a.bin_idx)[pair] = k;
}

// Phase 1 of a tile: per (sample, feature) the bin (L-probe search over the
// feature's interior edges), the position and the record {k * kstride, q(t), x}.
template <int L, typename QT>
__device__ __forceinline__ void fwd_phase1(const FwdArgs& a, const FwdLayout& Ly, const float* sX, int ns, int fc,
                                           int kstride, int64_t t0, int f0, int tid, int nthr) {
  const int lgFc = a.lgFc, Fc = 1 << lgFc, ldK = a.ldK, B = a.B;
  const int np = ns << lgFc;
  // two pairs a thread at a time (p and p + nthr: the same feature, nthr being a multiple of Fc), so that
  // their searches overlap
  for (int p = tid; p < np; p += 2 * nthr) {
    const int i = p & (Fc - 1);
    const int p1 = p + nthr;
    const bool has1 = p1 < np;
    const float x0 = sX[p];
    const float x1 = has1 ? sX[p1] : 0.0f;
    float4 q0 = make_float4(0.0f, 0.0f, x0, 0.0f), q1 = make_float4(0.0f, 0.0f, x1, 0.0f);
    if (i < fc) {
      const float* keys = Ly.sK + i * ldK;
      const int c0 = key_count<L>(x0, keys);
      const int c1 = key_count<L>(x1, keys);
      const int n1 = Ly.sN[i] - 1;
      const int k0 = c0 < n1 ? c0 : n1, k1 = c1 < n1 ? c1 : n1;
      const float2 er0 = Ly.sL[i * B + k0], er1 = Ly.sL[i * B + k1];
      q0.x = __int_as_float(k0 * kstride);
      q0.y = quantize<QT>((x0 - er0.x) * er0.y);
      q1.x = __int_as_float(k1 * kstride);
      q1.y = quantize<QT>((x1 - er1.x) * er1.y);
      if (a.bin_idx != nullptr) {
        store_bin(a, (t0 + (p >> lgFc)) * a.F + f0 + i, k0);
        if (has1) store_bin(a, (t0 + (p1 >> lgFc)) * a.F + f0 + i, k1);
      }
    }
    Ly.sQ[p] = q0;
    if (has1) Ly.sQ[p1] = q1;
  }
}

template <typename QT, typename OT, int VEC, int EPI, bool RELU>
__global__ void __launch_bounds__(kFwdMaxThreads, 2)
ple_fwd_kernel(const FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lgFc = a.lgFc;
  const int Fc = 1 << lgFc, B = a.B, D = a.D, S_t = a.S_t, ldK = a.ldK;
  const int nc = D / VEC;
  const int R = Fc * nc;
  FwdLayout L;
  fwd_layout(a, &L, smem_raw);
  const int tid = threadIdx.x, nthr = blockDim.x;
  // this thread's fixed output column (nthr is a multiple of R)
  const int col = tid % R;
  const int ci = col / nc;
  const int cd = (col - ci * nc) * VEC;
  const int s_step = nthr / R;
  const int s_first = tid / R;
  const int kstride = D << lgFc;  // floats between consecutive bin rows of the tables
  OT* out = reinterpret_cast<OT*>(a.out);

  // this CTA's slot range of the flattened (chunk group, sample) space; the members of a slot take
  // consecutive chunks of the same samples, so that their x pieces of one 128-byte line are read together
  const int m = a.group;
  const int slot = blockIdx.x / m, member = blockIdx.x - slot * m;
  const int n_slots = gridDim.x / m;
  const int64_t total = (int64_t)a.n_groups * a.N;
  int64_t u_lo = total * slot / n_slots;
  const int64_t u_hi = total * (slot + 1) / n_slots;

  while (u_lo < u_hi) {
    const int grp = (int)(u_lo / a.N);
    const int64_t s_begin = u_lo - (int64_t)grp * a.N;
    const int64_t s_end = min64(a.N, s_begin + (u_hi - u_lo));
    u_lo += s_end - s_begin;
    const int chunk = grp * m + member;
    if (chunk >= a.n_chunks) continue;  // uniform over the CTA
    const int f0 = chunk << lgFc;
    const int fc = min(Fc, a.F - f0);
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
    __syncthreads();  // the previous segment is done with every buffer
    load_x(s_begin, (int)min64(S_t, s_end - s_begin), L.sXb);

    // ---- per-segment tables (overlap the first x tile copy)
    for (int i = tid; i < Fc; i += nthr) {
      int n = i < fc ? a.n_bins[f0 + i] : 1;
      L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
    }
    __syncthreads();
    for (int idx = tid; idx < Fc * ldK; idx += nthr) {  // feature-major key rows: e_1 .. e_{n-1}, +inf
      const int i = idx / ldK, j = idx - i * ldK;
      float e = __int_as_float(0x7f800000);
      if (i < fc && j + 1 < L.sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j + 1];
      L.sK[idx] = e;
    }
    for (int idx = tid; idx < Fc * B; idx += nthr) {  // {e_k, r_k}
      const int i = idx / B, j = idx - i * B;
      float2 v = make_float2(0.0f, 0.0f);
      if (i < fc && j < L.sN[i])
        v = make_float2(a.edges[(int64_t)(f0 + i) * (B + 1) + j], a.inv_w[(int64_t)(f0 + i) * B + j]);
      L.sL[idx] = v;
    }
    const float* Wc = a.W + (int64_t)f0 * B * D;
    for (int idx = tid; idx < fc * B * D; idx += nthr) {
      const int i = idx / (B * D);
      const int rem = idx - i * B * D;
      const int p = rem / D, d = rem - p * D;
      const int n = L.sN[i];
      const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
      if (lg >= 0) L.sS[((lg << lgFc) + i) * D + d] = quantize<QT>(Wc[idx]);
    }
    __syncthreads();
    for (int c2 = tid; c2 < Fc * D; c2 += nthr) {
      const int i = c2 / D, d = c2 - i * D;
      const int n = L.sN[i];
      float acc = 0.0f;
      for (int j = 0; j < n; ++j) {
        const int o = ((j << lgFc) + i) * D + d;
        L.sT[o] = acc;
        acc += L.sS[o];
      }
    }
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
    const float* sTc = L.sT + ci * D + cd;
    const float* sSc = L.sS + ci * D + cd;

    int buf = 0;
    for (int64_t t0 = s_begin; t0 < s_end; t0 += S_t, buf ^= 1) {
      const int ns = (int)min64(S_t, s_end - t0);
      const float* sX = L.sXb + buf * S_t * Fc;
      cp_async_wait_all();
      __syncthreads();  // x tile visible; previous phase 2 done with sQ and the other buffer
      if (t0 + S_t < s_end) load_x(t0 + S_t, (int)min64(S_t, s_end - t0 - S_t), L.sXb + (buf ^ 1) * S_t * Fc);
      // ---- phase 1: bins, positions -> sQ[s][i] = {k, q(t), x}
      switch (a.lgk) {
#define PLE_FWD_P1(LL) \
  case LL: fwd_phase1<LL, QT>(a, L, sX, ns, fc, kstride, t0, f0, tid, nthr); break;
        PLE_FWD_P1(0) PLE_FWD_P1(1) PLE_FWD_P1(2) PLE_FWD_P1(3) PLE_FWD_P1(4)
        PLE_FWD_P1(5) PLE_FWD_P1(6) PLE_FWD_P1(7) PLE_FWD_P1(8)
#undef PLE_FWD_P1
        default: break;
      }
      __syncthreads();
      // ---- phase 2: output chunks of this thread's column
      if (col_live) {
        const int64_t ostride = (int64_t)a.F * D;
        OT* optr = out + ((t0 + s_first) * a.F + f0 + ci) * (int64_t)D + cd;
        const int64_t ostep = ostride * s_step;
        const float4* qptr = L.sQ + (s_first << lgFc) + ci;
        const int qstep = s_step << lgFc;
        // the record of the next sample is read one iteration ahead, so that only the table reads
        // wait on a shared-memory round trip
        float4 q = s_first < ns ? *qptr : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 2
        for (int s = s_first; s < ns; s += s_step, optr += ostep) {
          const int off = __float_as_int(q.x);
          const FV<VEC> tv = lds<VEC>(sTc + off);
          const FV<VEC> sv = lds<VEC>(sSc + off);
          qptr += qstep;
          const float4 qn = s + s_step < ns ? *qptr : q;
          store_out<OT, VEC>(optr, fwd_chunk<QT, OT, VEC, EPI, RELU>(q.y, tv, sv, q.z, ep0, ep1));
          q = qn;
        }
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
  // slots of m CTAs on consecutive chunks whose x pieces fill a 128-byte line (measured: with one CTA per
  // chunk range the forward read 2x (16 features) to 4x (8 features) the bytes of x from DRAM)
  FwdArgs g = a;
  int m = 128 / (4 << a.lgFc);
  if (m < 1) m = 1;
  if (m > a.n_chunks) m = a.n_chunks;
  g.group = m;
  g.n_groups = (int)ceil_div<int64_t>(a.n_chunks, m);
  const int64_t total = (int64_t)g.n_groups * a.N;
  int64_t slots = (int64_t)device_sm_count() * per_sm / m;
  if (slots > total / 32) slots = total / 32;  // at least 32 (chunk group, sample) rows per slot
  if (slots < 1) slots = 1;
  const int64_t grid = slots * m;
  kern<<<(unsigned)grid, threads, smem, st>>>(g);
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
  // feature chunk: power of two, tables within the budget, R = Fc * D / vec <= kFwdMaxThreads.  The larger
  // budget (wider chunks, one CTA per SM) only for fp32 outputs with D <= 16, where it measured faster (c5
  // shard: 16 features 0.92 ms, 8 features 1.05) before the CTA slots and ties with them (full c5: 6.733 vs
  // 6.725 ms); elsewhere it measured slower (c4, bf16: 0.30 vs 0.26 ms; c2, D = 32: 0.126 vs 0.122; c3,
  // D = 64: 0.125 vs 0.117)
  const int nc = a.D / vec;
  int lg = 4;
  const size_t budget = output_dtype == PLE_DTYPE_F32 && a.D <= 16 ? kFwdTableBudgetF32 : kFwdTableBudget;
  auto tables = [&](int fc) { return (size_t)2 * a.B * fc * a.D * sizeof(float); };
  while (lg > 0 && (tables(1 << lg) > budget || (1 << lg) * nc > kFwdMaxThreads ||
                    (1 << (lg - 1)) >= a.F))
    --lg;
  const int Fc = 1 << lg;
  if (Fc * nc > kFwdMaxThreads) return set_error(PLE_ERR_UNSUPPORTED, "forward: d_embedding too large");
  a.lgFc = lg;
  a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
  int lgk = 0;
  while ((1 << lgk) < a.B) ++lgk;  // 2^lgk - 1 >= B - 1 interior edges
  a.lgk = lgk;
  const int R = Fc * nc;
  const int threads = R * (kFwdMaxThreads / R);
  a.S_t = kFwdPairsPerTile / Fc;
  if (a.S_t < 1) a.S_t = 1;
  a.ldK = (1 << lgk) + 1;  // odd row stride: the first probes of different features hit different banks
  a.x_vec4 = (Fc >= 4) && (a.F % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  const size_t smem = fwd_layout(a, nullptr, nullptr);
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
