// ple_backward_impl.cuh - the fused PLE backward kernel (templates), shared by
// the per-dtype instantiation files ple_backward_<dtypes>.cu.
//
// Gradients (reference backward_cuda.cu:343-492 for grad_x, :268-336 and
// :859-925 for grad_W; the epilogue gradients follow autograd of
// module.py:230-248):
//   g'       = 0 where the ReLU input z <= 0, else g   (torch threshold_backward;
//              NaN inputs pass the gradient); g' = g without ReLU
//   grad_W[i, phys(j)] = U[j] + sum_{j' > j} H[j']  with
//       H[j] = sum_{b: k_b = j} q(g'_b),  U[j] = sum_{b: k_b = j} q(t_b) q(g'_b)
//   grad_x   = r_k <q(g'), S[k]> + [k > 0, x == e_k] r_{k-1} <q(g'), S[k-1]>
//              (+ <g, w0> for epilogue B)
//   grad_bias = sum_b g'  (A);  grad_w0 = sum_b g x, grad_b0 = sum_b g  (B)
//
// Work decomposition.  One persistent CTA of 16 warps per SM.  Features are
// cut into chunks of Fc; m consecutive chunks form a group whose x / grad_x
// rows fill whole 32-byte sectors (m = 32 / (4 Fc)), and the m CTAs of a slot
// walk the same sample range of a group, one chunk each, so the sectors they
// share meet in L2.  Each slot owns an equal contiguous range of the
// flattened (group, sample) space.  A chunk's warps split evenly over its Fc
// features (Wf warps per feature); a lane group (nc lanes x VEC elements =
// one D row) is one walk slot.  Per segment the chunk's tables are staged
// and H / U zeroed; per tile of S_t samples (x arrives by cp.async one tile
// ahead and the next tile's gradient rows are bulk-prefetched into L2 with an
// evict-last policy):
//   A  warp (feature, quarter): bin of 32 samples at a time (the forward's
//      bin indices when given, else an L-level search over the feature's
//      interior edges in breadth-first order, conflict-free in shared
//      memory), the rank of each sample among the warp's equal bins
//      (ballots of the bin bits), per-(feature, bin, quarter) counts kept by the warp
//      itself (no atomics: the counts and ranks are a function of the input),
//      q(t), the tie flag, one draft entry per pair;
//   B  exclusive scan of the counts (bin-major, quarter-minor);
//   C  each draft moves to its sorted position, stored segment-major (entry
//      p of segment g at p * G + g) so the slots of a warp read adjacent
//      entries;
//   D  walk: a feature's sorted list is cut into at most G equal segments,
//      one per slot.  The slot keeps the active bin's T / S rows and the run's
//      H / U sums in registers and adds a run to the shared histogram once,
//      at its end; the first run of a segment (which may continue the
//      previous segment's last run) goes to a carry slot.  Gradient rows are
//      read from L2 two entries ahead, a whole 32-byte sector per lane where
//      the row allows.  A bin whose ReLU input is positive for every t the
//      bin admits ("open": the input is monotone in t, so its two end values
//      decide) needs no mask; when every slot of a warp is in an open bin the
//      step skips the mask, bit-identically;
//   E  carries are added per chain of equal bins (one start per chain,
//      segment order within it); grad_x rows are stored in natural order.
// At the end of a segment a suffix scan over bins turns H / U into grad_W
// and the partial goes to the workspace; ple_bwd_finalize_kernel sums the
// partials of each feature in slot order.  No floating-point atomics: the
// result is bitwise deterministic for a given shape and device.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"

namespace ple {

enum { kMaskNone = 0, kMaskRelu = 1, kMaskReluBias = 2 };
// epilogue terms accumulated along the walk: none, sum g' (epilogue A bias), or linear0 (<g, w0>, sum g x,
// sum g; epilogue B)
enum { kEpvNone = 0, kEpvBias = 1, kEpvLin = 2 };

constexpr int kBwdWarps = kBwdThreads / 32;

// Floats between bin rows of the tables: Fc * D rounded up to 4, plus 4 when
// that is a multiple of 8, so that consecutive bins shift by 16 bytes modulo
// the 128-byte bank window.
__host__ __device__ __forceinline__ int table_stride(int Fc, int D) {
  int ts = (Fc * D + 3) & ~3;
  if (((ts >> 2) & 1) == 0) ts += 4;
  return ts;
}

struct BwdDims {
  int Fc, Wf, S_t, G, nc, nkeys;
};

struct BwdLayout {
  float *sT, *sS, *sH, *sU;  // [B][ts]: feature i's row of bin k at k * ts + i * D (bin-major, padded)
  float* sKey;               // [Fc][nkeys] interior edges in breadth-first order (node 1 = root; slot 0 unused)
  float2* sER;               // [Fc][B] {e_k, r_k}
  float2* sRO;               // [Fc][B] {r_k, open_k}
  float* sX;                 // [2][Fc][S_t] x tiles (transposed)
  float2* sDraft;            // [Fc][S_t] natural-order drafts (q(t), s | k << 12 | rank << 20 | tie << 31)
  float* sGX;                // [S_t][Fc][nc] grad_x shares (aliases sDraft: drafts die in phase C)
  float2* sEnt;              // [Fc][S_t + G] sorted (q(t), s | k << 12 | tie << 31), segment-major
  float* sCarry;             // [Fc][G][2][D]
  int* sCnt;                 // [Fc][B][Wf]
  int* sCarryBin;            // [Fc][G]
  int* sN;                   // [Fc]
  int* sTie;                 // [Fc]: the tile has an edge tie (x == e_k, k > 0) in feature i
  uint8_t* sBin;             // [Fc][S_t] the forward's bins of the tile (when given)
};

__host__ __device__ __forceinline__ size_t bwd_layout_bytes(int B, int D, const BwdDims& m, BwdLayout* L,
                                                            unsigned char* base) {
  const size_t tab = (size_t)B * table_stride(m.Fc, D);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 15) & ~(size_t)15;
    return base + o;
  };
  unsigned char* pT = take(4 * tab * 4);
  unsigned char* pGX = take((size_t)m.Fc * m.S_t * 8);  // drafts (8 bytes per pair), then grad_x (4)
  unsigned char* pEnt = take((size_t)m.Fc * (m.S_t + m.G) * 8);
  unsigned char* pCarry = take((size_t)m.Fc * m.G * 2 * D * 4);
  unsigned char* pX = take((size_t)2 * m.S_t * m.Fc * 4);
  unsigned char* pER = take((size_t)m.Fc * B * 8);
  unsigned char* pRO = take((size_t)m.Fc * B * 8);
  unsigned char* pK = take((size_t)m.Fc * m.nkeys * 4);
  unsigned char* pCnt = take((size_t)m.Fc * B * m.Wf * 4);
  unsigned char* pCB = take((size_t)m.Fc * m.G * 4);
  unsigned char* pN = take((size_t)m.Fc * 4);
  unsigned char* pTie = take((size_t)m.Fc * 4);
  unsigned char* pBin = take((size_t)m.Fc * m.S_t);
  if (L) {
    L->sT = reinterpret_cast<float*>(pT);
    L->sS = L->sT + tab;
    L->sH = L->sS + tab;
    L->sU = L->sH + tab;
    L->sGX = reinterpret_cast<float*>(pGX);
    L->sDraft = reinterpret_cast<float2*>(pGX);
    L->sEnt = reinterpret_cast<float2*>(pEnt);
    L->sCarry = reinterpret_cast<float*>(pCarry);
    L->sX = reinterpret_cast<float*>(pX);
    L->sER = reinterpret_cast<float2*>(pER);
    L->sRO = reinterpret_cast<float2*>(pRO);
    L->sKey = reinterpret_cast<float*>(pK);
    L->sCnt = reinterpret_cast<int*>(pCnt);
    L->sCarryBin = reinterpret_cast<int*>(pCB);
    L->sN = reinterpret_cast<int*>(pN);
    L->sTie = reinterpret_cast<int*>(pTie);
    L->sBin = reinterpret_cast<uint8_t*>(pBin);
  }
  return off;
}

// Exclusive scan of cnt[0..m) in place by one warp.
__device__ __forceinline__ void warp_exclusive_scan(int* cnt, int m, int lane) {
  const int per = (m + 31) >> 5;
  const int lo = min(lane * per, m), hi = min(lo + per, m);
  int local = 0;
  for (int j = lo; j < hi; ++j) local += cnt[j];
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  int run = incl - local;
  for (int j = lo; j < hi; ++j) {
    const int c = cnt[j];
    cnt[j] = run;
    run += c;
  }
}

// Sum of v over the nc lanes of a slot row (lanes r * nc .. r * nc + nc - 1, active together), complete in
// lane c == 0 (the others hold partial sums).
__device__ __forceinline__ float row_sum(float v, int c, int nc) {
  if (nc == 1) return v;
  const unsigned m = __activemask();
  if ((nc & (nc - 1)) == 0) {
    for (int off = nc >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(m, v, off);
    return v;
  }
  float t = v;
  for (int j = 1; j < nc; ++j) t += __shfl_down_sync(m, v, j);
  return t;
}

// ------------------------------------------------------------------ rows
// VEC fp32 values of one D-row chunk held as packed pairs (VEC >= 2, even) or
// a scalar (VEC == 1), so the arithmetic maps onto fp32x2 instructions;
// shared / global accesses are 16 bytes wide when VEC % 4 == 0, else 8.
template <int VEC> struct Row {
  static constexpr int NP = VEC >= 2 ? VEC / 2 : 1;
  f2_t p[NP];  // VEC == 1 uses the low half of p[0]
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int e = 0; e < NP; ++e) p[e] = 0ull;
  }
  __device__ __forceinline__ void lds(const float* src) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int e = 0; e < NP; e += 2) {
        const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(src + 2 * e);
        p[e] = v.x;
        p[e + 1] = v.y;
      }
    } else if constexpr (VEC % 2 == 0) {
#pragma unroll
      for (int e = 0; e < NP; ++e) p[e] = *reinterpret_cast<const unsigned long long*>(src + 2 * e);
    } else {
      p[0] = (f2_t)__float_as_uint(*src);
    }
  }
  __device__ __forceinline__ void ldg(const float* src) {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int e = 0; e < NP; e += 2) {
        const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(src + 2 * e));
        p[e] = v.x;
        p[e + 1] = v.y;
      }
    } else if constexpr (VEC % 2 == 0) {
#pragma unroll
      for (int e = 0; e < NP; ++e) p[e] = __ldg(reinterpret_cast<const unsigned long long*>(src + 2 * e));
    } else {
      p[0] = (f2_t)__float_as_uint(__ldg(src));
    }
  }
  __device__ __forceinline__ void sts(float* dst) const {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int e = 0; e < NP; e += 2)
        *reinterpret_cast<ulonglong2*>(dst + 2 * e) = make_ulonglong2(p[e], p[e + 1]);
    } else if constexpr (VEC % 2 == 0) {
#pragma unroll
      for (int e = 0; e < NP; ++e) *reinterpret_cast<unsigned long long*>(dst + 2 * e) = p[e];
    } else {
      *dst = __uint_as_float((unsigned)p[0]);
    }
  }
  __device__ __forceinline__ void add_from(const float* src) {  // this += src (shared memory)
    Row<VEC> o;
    o.lds(src);
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      if constexpr (VEC >= 2) p[e] = add2(p[e], o.p[e]);
      else p[e] = (f2_t)__float_as_uint(lo(e) + o.lo(e));
    }
  }
  __device__ __forceinline__ float lo(int e) const {
    float a, b;
    unpack2(p[e], a, b);
    return a;
  }
};

// Raw gradient chunk of VEC elements of GT, loaded with the widest access the
// chunk allows (the host checks the base pointer): 32 bytes at once when
// `wide` (a whole sector), through L2 only, with the given cache policy.
template <typename GT, int VEC> struct GRaw {
  static constexpr int kBytes = (int)sizeof(GT) * VEC;
  static constexpr int kWords = (kBytes + 3) / 4;
  unsigned w[kWords];
};

template <typename GT, int VEC> constexpr int chunk_align() {
  return (sizeof(GT) * VEC) % 16 == 0 ? 16 : (sizeof(GT) * VEC) % 8 == 0 ? 8 : (sizeof(GT) * VEC) % 4 == 0 ? 4 : 2;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// L2 prefetch of one box of the gradient tensor (2-D tensor map over [N][F * D]: box of the chunk's
// columns x up to 256 sample rows starting at element column c0, row r0), with a cache policy.
__device__ __forceinline__ void prefetch_tile_l2(const CUtensorMap* map, int c0, int r0, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile.L2::cache_hint [%0, {%1, %2}], %3;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(r0), "l"(pol)
               : "memory");
}

template <typename GT, int VEC>
__device__ __forceinline__ void ldg_raw(GRaw<GT, VEC>& r, const GT* p, bool wide, uint64_t pol) {
  constexpr int bytes = GRaw<GT, VEC>::kBytes;
  constexpr int al = chunk_align<GT, VEC>();
  if constexpr (bytes == 32) {
    if (wide) {
      asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
                   : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]), "=r"(r.w[4]), "=r"(r.w[5]),
                     "=r"(r.w[6]), "=r"(r.w[7])
                   : "l"(p), "l"(pol));
      return;
    }
  }
  if constexpr (al == 16) {
#pragma unroll
    for (int j = 0; j < bytes / 16; ++j)
      asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                   : "=r"(r.w[4 * j]), "=r"(r.w[4 * j + 1]), "=r"(r.w[4 * j + 2]), "=r"(r.w[4 * j + 3])
                   : "l"(reinterpret_cast<const char*>(p) + 16 * j), "l"(pol));
  } else if constexpr (al == 8) {
#pragma unroll
    for (int j = 0; j < bytes / 8; ++j)
      asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
                   : "=r"(r.w[2 * j]), "=r"(r.w[2 * j + 1])
                   : "l"(reinterpret_cast<const char*>(p) + 8 * j), "l"(pol));
  } else if constexpr (al == 4) {
#pragma unroll
    for (int j = 0; j < bytes / 4; ++j) r.w[j] = __ldg(reinterpret_cast<const unsigned*>(p) + j);
  } else {
    r.w[0] = (unsigned)__ldg(reinterpret_cast<const unsigned short*>(p));
  }
}

// Elements 2e, 2e + 1 of a raw chunk as a packed fp32 pair (VEC >= 2).
template <typename GT, int VEC>
__device__ __forceinline__ f2_t raw_pair(const GRaw<GT, VEC>& r, int e) {
  if constexpr (std::is_same<GT, float>::value) {
    return from_bits2(r.w[2 * e], r.w[2 * e + 1]);
  } else if constexpr (std::is_same<GT, __nv_bfloat16>::value) {
    return from_bits2(r.w[e] << 16, r.w[e] & 0xffff0000u);
  } else {
    float lo, hi;
    widen_pack<GT>(r.w[e], lo, hi);
    return pack2(lo, hi);
  }
}
template <typename GT, int VEC>
__device__ __forceinline__ float raw_one(const GRaw<GT, VEC>& r) {
  if constexpr (std::is_same<GT, float>::value) return __uint_as_float(r.w[0]);
  else return Dt<GT>::to_f(*reinterpret_cast<const GT*>(&r.w[0]));
}

// Largest value that rounds to zero in QT: with no bias after the rounding,
// q(p) <= 0 exactly when p <= threshold (ties round to the even zero).
template <typename QT> __host__ __device__ __forceinline__ float zero_round_threshold() {
  if constexpr (std::is_same<QT, float>::value) return 0.0f;
  else if constexpr (std::is_same<QT, __nv_bfloat16>::value) return 1.4012984643e-45f * 0x8000;  // 2^-134
  else return 2.98023223876953125e-08f;                                                     // 2^-25
}

// The ReLU passes the gradient of an input p (torch threshold_backward: NaN passes).
template <typename QT, int MASK>
__device__ __forceinline__ bool relu_passes(float p, float bias) {
  if constexpr (MASK == kMaskReluBias) return !(quantize<QT>(p) + bias <= 0.0f);
  else return !(p <= zero_round_threshold<QT>());
}

// ------------------------------------------------------------------ tables
// The chunk's tables for one segment: search keys (breadth-first interior
// edges), {e_k, r_k}, S = q(W) in logical bin order, its exclusive prefix T,
// the open flags (MASK variants), H / U zeroed.
template <typename QT, int MASK>
__device__ __forceinline__ void stage_tables(const BwdArgs& a, const BwdLayout& L, int f0, int fc, int Fc, int ts,
                                             int nkeys, int lgk, int tid, int nthr) {
  const int B = a.B, D = a.D;
  for (int i = tid; i < Fc; i += nthr) {
    const int n = i < fc ? a.n_bins[f0 + i] : 1;
    L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  for (int idx = tid; idx < B * ts; idx += nthr) {
    L.sH[idx] = 0.0f;
    L.sU[idx] = 0.0f;
    L.sS[idx] = 0.0f;
  }
  __syncthreads();
  // breadth-first keys: node v (1 <= v < nkeys) at level l = floor(log2 v), position p = v - 2^l holds sorted
  // key (2p + 1) * 2^(lgk - 1 - l) - 1 of e_1 .. e_{n-1}, +inf beyond (the search count is capped at n - 1)
  for (int idx = tid; idx < Fc * nkeys; idx += nthr) {
    const int i = idx / nkeys, v = idx - i * nkeys;
    float e = __int_as_float(0x7f800000);
    if (v > 0 && i < fc) {
      const int l = 31 - __clz(v);
      const int j = ((2 * (v - (1 << l)) + 1) << (lgk - 1 - l)) - 1;
      if (j + 1 < L.sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j + 1];
    }
    L.sKey[idx] = e;
  }
  for (int idx = tid; idx < Fc * B; idx += nthr) {
    const int i = idx / B, k = idx - i * B;
    float e = 0.0f, r = 0.0f;
    if (i < fc && k < L.sN[i]) {
      e = a.edges[(int64_t)(f0 + i) * (B + 1) + k];
      r = a.inv_w[(int64_t)(f0 + i) * B + k];
    }
    L.sER[idx] = make_float2(e, r);
  }
  // S[logical bin][i][d] = q(W[i][physical bin][d]); W rows are walked per (i, p) to avoid divisions
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int row = tid; row < fc * B; row += nthr) {
    const int i = row / B, p = row - i * B;
    const int n = L.sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) {
      const float* src = Wc + (int64_t)row * D;
      float* dst = L.sS + lg * ts + i * D;
      for (int d = 0; d < D; ++d) dst[d] = quantize<QT>(src[d]);
    }
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = L.sN[i];
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int o = j * ts + i * D + d;
      L.sT[o] = acc;
      acc += L.sS[o];
    }
  }
  __syncthreads();
  // open flags: the ReLU input fma(t, S, T) (+ bias) is monotone in t, so it is positive for every t of
  // the bin when it is at both ends of the bin's t range: [0, tmax] for a middle bin (tmax from the
  // right edge, computed as the kernel computes t); [0, inf) for the last bin, where it suffices that
  // S >= 0 and the value at t = 0 passes (t = inf or NaN then passes too); never for bin 0
  for (int idx = tid; idx < Fc * B; idx += nthr) {
    const int i = idx / B, k = idx - i * B;
    const float2 er = L.sER[idx];
    bool open = false;
    if constexpr (MASK != kMaskNone) {
      const int n = L.sN[i];
      // bins given by the caller need not contain x: their t range is unknown, so the exact path
      if (a.bin_idx == nullptr && i < fc && k > 0 && k < n) {
        const bool last = k == n - 1;
        const float tmax = last ? 0.0f : quantize<QT>((a.edges[(int64_t)(f0 + i) * (B + 1) + k + 1] - er.x) * er.y);
        open = true;
        for (int d = 0; d < D && open; ++d) {
          const float S = L.sS[k * ts + i * D + d], T = L.sT[k * ts + i * D + d];
          const float bias = MASK == kMaskReluBias ? a.bias[(int64_t)(f0 + i) * D + d] : 0.0f;
          const float p0 = fmaf(0.0f, S, T), p1 = fmaf(tmax, S, T);
          // a NaN end value (non-finite tables or edges) leaves the bin on the exact path
          if (p0 != p0 || p1 != p1 || !relu_passes<QT, MASK>(p0, bias) || !relu_passes<QT, MASK>(p1, bias)) open = false;
          if (last && !(S >= 0.0f)) open = false;
        }
      }
    }
    L.sRO[idx] = make_float2(er.y, open ? 1.0f : 0.0f);
  }
}

// ------------------------------------------------------------------ phase A
// Warp (feature my_i, quarter my_w): bins, per-warp ranks, counts, drafts.
template <int LGK, typename QT>
__device__ __forceinline__ void phase_a(const BwdArgs& a, const BwdLayout& L, const float* sX, int my_i, int my_w,
                                        int lgWf, int lgSt, int lg_q, int ns, int lane) {
  const int B = a.B, S_t = 1 << lgSt;
  const float* keys = L.sKey + (my_i << LGK);
  const float* xs = sX + my_i * S_t;
  const float2* er = L.sER + my_i * B;
  int* cnt = L.sCnt + ((my_i * B) << lgWf) + my_w;
  float2* drafts = L.sDraft + my_i * S_t;
  const int n1 = L.sN[my_i] - 1;
  const uint8_t* bins = a.bin_idx != nullptr ? L.sBin + my_i * S_t : nullptr;
  const int lo = my_w << lg_q, hi = min(lo + (1 << lg_q), ns);
  unsigned any_tie = 0;
  for (int base = lo; base < hi; base += 32) {
    const int s = base + lane;
    const bool v = s < hi;
    const float x = xs[v ? s : lo];
    int k;
    if (bins != nullptr) {
      k = bins[v ? s : lo];
    } else {
      int node = 1;
#pragma unroll
      for (int l = 0; l < LGK; ++l) node = 2 * node + (x < keys[node] ? 0 : 1);
      k = min(node - (1 << LGK), n1);
    }
    // lanes with the same bin: the intersection of the ballots of the bin bits (every lane takes part; idle
    // lanes keep only themselves); measured faster here than match.any
    unsigned peers = __ballot_sync(0xffffffffu, v);
#pragma unroll
    for (int bit = 0; bit < LGK; ++bit) {
      const unsigned bal = __ballot_sync(0xffffffffu, (k >> bit) & 1);
      peers &= ((k >> bit) & 1) ? bal : ~bal;
    }
    if (!v) peers = 1u << lane;
    const int leader = __ffs(peers) - 1;
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool lead = v && lane == leader;
    int old = 0;
    if (lead) old = cnt[k << lgWf];
    old = __shfl_sync(0xffffffffu, old, leader);
    if (lead) cnt[k << lgWf] = old + __popc(peers);
    const float2 e = er[k];
    const float t = quantize<QT>((x - e.x) * e.y);
    const bool tie = v && k > 0 && x == e.x;
    any_tie |= __ballot_sync(0xffffffffu, tie);
    if (v)
      drafts[s] = make_float2(t, __uint_as_float((unsigned)s | ((unsigned)k << 12) | ((unsigned)(old + rank) << 20) |
                                                 (tie ? 0x80000000u : 0u)));
  }
  if (any_tie != 0 && lane == 0) L.sTie[my_i] = 1;
}

// ------------------------------------------------------------------ phase D
// Per-slot state of the walk.
template <int VEC> struct WalkState {
  Row<VEC> Sk, Hr, Ur;
  float r_k;
  int k_cur;
  bool first, open;
};

// One walk step of one slot: returns the slot's share of grad_x (without the
// edge term) and leaves q(g') in q for it.
template <typename QT, typename GT, int VEC, int MASK, int EPIV, bool EXACT>
__device__ __forceinline__ float walk_step(const GRaw<GT, VEC>& g, float tq, float xv, WalkState<VEC>& st,
                                           const float* trow, const Row<VEC>& pbias, const Row<VEC>& w0r,
                                           Row<VEC>& aw, Row<VEC>& ab, f2_t (&q)[Row<VEC>::NP]) {
  constexpr int NP = Row<VEC>::NP;
  Row<VEC> Tk;  // prefix row of the active bin: only the exact (masked) path needs it
  if constexpr (MASK != kMaskNone && EXACT) Tk.lds(trow);
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ROUND_G = !std::is_same<GT, QT>::value && !std::is_same<QT, float>::value;
  const float thr = zero_round_threshold<QT>();
  if constexpr (VEC >= 2) {
    const f2_t t2 = pack2(tq, tq);
    const f2_t x2 = pack2(xv, xv);
    f2_t d2 = 0ull, dw2 = 0ull;
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      const f2_t g2 = raw_pair<GT, VEC>(g, e);
      if constexpr (LIN) {
        dw2 = fma2(g2, w0r.p[e], dw2);
        aw.p[e] = fma2(g2, x2, aw.p[e]);
        ab.p[e] = add2(ab.p[e], g2);
      }
      f2_t qq = g2;
      if constexpr (MASK != kMaskNone && EXACT) {
        float p0, p1, g0, g1;
        unpack2(fma2(t2, st.Sk.p[e], Tk.p[e]), p0, p1);
        unpack2(g2, g0, g1);
        if constexpr (MASK == kMaskReluBias) {
          round2<QT>(p0, p1);
          float b0, b1;
          unpack2(pbias.p[e], b0, b1);
          p0 += b0;
          p1 += b1;
          qq = pack2(p0 <= 0.f ? 0.f : g0, p1 <= 0.f ? 0.f : g1);
        } else {
          qq = pack2(p0 <= thr ? 0.f : g0, p1 <= thr ? 0.f : g1);
        }
      }
      if constexpr (EPIV == kEpvBias) aw.p[e] = add2(aw.p[e], qq);  // sum g' (before the QT rounding)
      if constexpr (ROUND_G) {
        float q0, q1;
        unpack2(qq, q0, q1);
        round2<QT>(q0, q1);
        qq = pack2(q0, q1);
      }
      q[e] = qq;
      st.Hr.p[e] = add2(st.Hr.p[e], qq);
      st.Ur.p[e] = fma2(t2, qq, st.Ur.p[e]);
      d2 = fma2(qq, st.Sk.p[e], d2);
    }
    float lo, hi;
    unpack2(d2, lo, hi);
    float gx = st.r_k * (lo + hi);
    if constexpr (LIN) {
      unpack2(dw2, lo, hi);
      gx += lo + hi;
    }
    return gx;
  } else {
    const float g0 = raw_one<GT, VEC>(g);
    if constexpr (LIN) {
      aw.p[0] = (f2_t)__float_as_uint(fmaf(g0, xv, aw.lo(0)));
      ab.p[0] = (f2_t)__float_as_uint(ab.lo(0) + g0);
    }
    float q0 = g0;
    const float s0 = st.Sk.lo(0);
    if constexpr (MASK != kMaskNone && EXACT) {
      float p0 = fmaf(tq, s0, Tk.lo(0));
      if constexpr (MASK == kMaskReluBias) {
        p0 = quantize<QT>(p0) + pbias.lo(0);
        q0 = p0 <= 0.f ? 0.f : g0;
      } else {
        q0 = p0 <= thr ? 0.f : g0;
      }
    }
    if constexpr (EPIV == kEpvBias) aw.p[0] = (f2_t)__float_as_uint(aw.lo(0) + q0);
    if constexpr (!std::is_same<GT, QT>::value) q0 = quantize<QT>(q0);
    q[0] = (f2_t)__float_as_uint(q0);
    st.Hr.p[0] = (f2_t)__float_as_uint(st.Hr.lo(0) + q0);
    st.Ur.p[0] = (f2_t)__float_as_uint(fmaf(tq, q0, st.Ur.lo(0)));
    float gx = st.r_k * (q0 * s0);
    if constexpr (LIN) gx += g0 * w0r.lo(0);
    return gx;
  }
}

// ------------------------------------------------------------------ kernel
template <typename QT, typename GT, int VEC, int MASK, int EPIV>
__global__ void __launch_bounds__(kBwdThreads, 1) ple_bwd_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap gmap) {
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ACC = EPIV != kEpvNone;  // per-slot epilogue sums (sum g x or sum g', and sum g)
  constexpr int NP = Row<VEC>::NP;
  extern __shared__ __align__(128) unsigned char smem_raw[];  // one declaration per file: the strictest
  const int lgFc = a.lgFc, lgWf = a.lgWf, lgSt = a.lgSt;
  const int Fc = 1 << lgFc, Wf = 1 << lgWf, S_t = 1 << lgSt;
  const int B = a.B, D = a.D;
  const int nc = D / VEC;
  const int Rint = 32 / nc;
  const int G = Wf * Rint;
  const int ES = S_t + G;
  const int ts = table_stride(Fc, D);
  const int nkeys = 1 << a.lgk;
  BwdLayout L;
  bwd_layout_bytes(B, D, BwdDims{Fc, Wf, S_t, G, nc, nkeys}, &L, smem_raw);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int r = lane / nc, c = lane - r * nc;
  const int cd = c * VEC;
  // warp wid serves feature my_i; its slots are segments g_seg of that feature
  const int my_i = wid >> lgWf;
  const int my_w = wid & (Wf - 1);
  const int g_seg = my_w * Rint + r;
  const bool do_gx = a.grad_x != nullptr;
  const GT* gptr = reinterpret_cast<const GT*>(a.g);
  const int lg_q = lgSt - lgWf;  // quarter length (log2)
  const uint64_t pol_first = l2_policy_evict_first();
  const uint64_t pol_last = l2_policy_evict_last();
  const unsigned gstride = (unsigned)a.F * (unsigned)D;  // elements between samples (checked to fit)

  const int m = a.group;
  const int slot = blockIdx.x / m, member = blockIdx.x - slot * m;
  const int n_slots = gridDim.x / m;
  const int64_t total = (int64_t)a.n_groups * a.N;
  int64_t u_lo = total * slot / n_slots;
  const int64_t u_hi = total * (slot + 1) / n_slots;

  for (int seg = 0; u_lo < u_hi; ++seg) {
    const int grp = (int)(u_lo / a.N);
    const int64_t s_begin = u_lo - (int64_t)grp * a.N;
    const int64_t s_end = min64(a.N, s_begin + (u_hi - u_lo));
    u_lo += s_end - s_begin;
    const int chunk = grp * m + member;
    if (chunk >= a.n_chunks) continue;  // uniform over the CTA
    const int f0 = chunk << lgFc;
    const int fc = min(Fc, a.F - f0);
    const bool walk_live = r < Rint && my_i < fc;

    // x tile, transposed to [Fc][S_t]: one 4-byte async copy per pair (features past fc read as 0)
    auto load_x = [&](int64_t t0, int ns, float* dst) {
      for (int q = tid; q < (ns << lgFc); q += nthr) {
        const int s = q >> lgFc, i = q & (Fc - 1);
        if (i < fc) cp_async4(dst + i * S_t + s, a.x + (t0 + s) * a.F + f0 + i);
        else dst[i * S_t + s] = 0.0f;
      }
      cp_async_commit();
    };
    // the tile's gradient rows of this chunk into L2, one box of up to 256 rows per instruction
    auto prefetch_g = [&](int64_t t0, int ns) {
      if (!a.g_prefetch || tid != 0) return;
      for (int r0 = 0; r0 < ns; r0 += 256) prefetch_tile_l2(&gmap, f0 * D, (int)(t0 + r0), pol_last);
    };

    __syncthreads();  // previous segment finished with every shared buffer
    load_x(s_begin, (int)min64(S_t, s_end - s_begin), L.sX);
    prefetch_g(s_begin, (int)min64(S_t, s_end - s_begin));
    stage_tables<QT, MASK>(a, L, f0, fc, Fc, ts, nkeys, a.lgk, tid, nthr);

    // per-slot parameters and accumulators that live across the segment's tiles
    Row<VEC> pbias, w0r, aw, ab;  // aw: sum g x (B) or sum g' (A); ab: sum g (B)
    pbias.zero();
    w0r.zero();
    aw.zero();
    ab.zero();
    if constexpr (MASK == kMaskReluBias) {
      if (walk_live) pbias.ldg(a.bias + (int64_t)(f0 + my_i) * D + cd);
    }
    if constexpr (LIN) {
      if (walk_live) w0r.ldg(a.w0 + (int64_t)(f0 + my_i) * D + cd);
    }

    int buf = 0;
    for (int64_t t0 = s_begin; t0 < s_end; t0 += S_t, buf ^= 1) {
      const int ns = (int)min64(S_t, s_end - t0);
      const float* sX = L.sX + buf * S_t * Fc;
      // segments of this tile: Lseg entries each, ceil(ns / Lseg) <= G of them non-empty, all at the front
      const int Ge = min(G, ns);
      const int Lseg = (ns + Ge - 1) / Ge;
      int lgL = 0;
      while ((1 << lgL) < Lseg) ++lgL;
      const bool pow2L = (1 << lgL) == Lseg;
      const unsigned mL = pow2L ? 0u : (unsigned)(0xffffffffu / (unsigned)Lseg) + 1u;
      for (int idx = tid; idx < ((Fc * B) << lgWf); idx += nthr) L.sCnt[idx] = 0;
      if (tid < Fc) L.sTie[tid] = 0;
      if (a.bin_idx != nullptr) {  // the forward's bins of this tile, clamped to [0, n_i - 1], as u8 [Fc][S_t]
        for (int q = tid; q < (ns << lgFc); q += nthr) {
          const int s = q >> lgFc, i = q & (Fc - 1);
          if (i < fc) {
            const int64_t pair = (t0 + s) * a.F + f0 + i;
            int k = a.bin_idx_bytes == 1 ? (int)reinterpret_cast<const uint8_t*>(a.bin_idx)[pair]
                  : a.bin_idx_bytes == 2 ? (int)reinterpret_cast<const int16_t*>(a.bin_idx)[pair]
                                         : reinterpret_cast<const int32_t*>(a.bin_idx)[pair];
            const int n1 = L.sN[i] - 1;
            L.sBin[i * S_t + s] = (uint8_t)(k < 0 ? 0 : (k > n1 ? n1 : k));
          }
        }
      }
      cp_async_wait_all();
      __syncthreads();  // x tile landed, counters reset, previous tile finished
      if (t0 + S_t < s_end) {
        const int ns2 = (int)min64(S_t, s_end - t0 - S_t);
        load_x(t0 + S_t, ns2, L.sX + (buf ^ 1) * S_t * Fc);
        prefetch_g(t0 + S_t, ns2);
      }

      // ---- A: bins, ranks, counts, drafts
      if (my_i < fc) {
        switch (a.lgk) {
#define PLE_BWD_PHASE_A(LL)                                                                                 \
  case LL:                                                                                                  \
    phase_a<LL, QT>(a, L, sX, my_i, my_w, lgWf, lgSt, lg_q, ns, lane);                              \
    break;
          PLE_BWD_PHASE_A(0) PLE_BWD_PHASE_A(1) PLE_BWD_PHASE_A(2) PLE_BWD_PHASE_A(3) PLE_BWD_PHASE_A(4)
          PLE_BWD_PHASE_A(5) PLE_BWD_PHASE_A(6) PLE_BWD_PHASE_A(7) PLE_BWD_PHASE_A(8)
#undef PLE_BWD_PHASE_A
          default: break;
        }
      }
      __syncthreads();
      // ---- B: exclusive scan per feature (bin-major, quarter-minor)
      // carry slots emptied (the previous tile's carries were consumed before this tile's first barrier)
      if (my_w == 0 && my_i < fc) warp_exclusive_scan(L.sCnt + ((my_i * B) << lgWf), B << lgWf, lane);
      for (int idx = tid; idx < Fc * G; idx += nthr) L.sCarryBin[idx] = -1;
      __syncthreads();
      // ---- C: drafts to their sorted positions; sorted position p is stored at (p % Lseg) * G + p / Lseg
      for (int p = tid; p < (fc << lgSt); p += nthr) {
        const int i = p >> lgSt, s = p & (S_t - 1);
        if (s < ns) {
          const float2 d = L.sDraft[p];
          const unsigned meta = __float_as_uint(d.y);
          const int k = (meta >> 12) & 0xff;
          const unsigned pos = (unsigned)L.sCnt[((i * B + k) << lgWf) + (s >> lg_q)] + ((meta >> 20) & 0x7ffu);
          const unsigned gq = pow2L ? pos >> lgL : __umulhi(pos, mL);
          L.sEnt[i * ES + (int)(pos - gq * (unsigned)Lseg) * G + (int)gq] =
              make_float2(d.x, __uint_as_float(meta & 0x800fffffu));
        }
      }
      __syncthreads();
      // ---- D: segmented walk
      if (my_i < fc) {
        int len = 0;
        if (walk_live) {
          const int rest = ns - g_seg * Lseg;
          len = rest < 0 ? 0 : (rest < Lseg ? rest : Lseg);
        }
        int trips = len;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) trips = max(trips, __shfl_xor_sync(0xffffffffu, trips, off));
        const int toff = my_i * D + cd;
        float* tH = L.sH + toff;
        float* tU = L.sU + toff;
        const float* tS = L.sS + toff;
        const float* tT = L.sT + toff;
        const float2* ro = L.sRO + my_i * B;
        float* gxs = L.sGX + my_i;  // grad_x of sample s at gxs[s * Fc]
        float* carry = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        int* carry_bin = L.sCarryBin + my_i * G + g_seg;
        const float* xcol = sX + my_i * S_t;
        const float2* ents = L.sEnt + my_i * ES + (g_seg < G ? g_seg : 0);
        const GT* grow = gptr + (t0 * a.F + f0 + my_i) * (int64_t)D + cd;
        const bool ties = L.sTie[my_i] != 0;
        const bool wide = a.g_wide != 0;
        WalkState<VEC> st;
        st.Sk.zero();
        st.Hr.zero();
        st.Ur.zero();
        st.r_k = 0.f;
        st.k_cur = -1;
        st.first = true;
        st.open = false;
        // entry and gradient row of step j in buffer j & 1, loaded two steps ahead (ping-pong, no copies)
        float2 eb0 = make_float2(0.f, 0.f), eb1 = make_float2(0.f, 0.f);
        GRaw<GT, VEC> gb0, gb1;
        auto fetch = [&](float2& e, GRaw<GT, VEC>& g, int j) {
          if (j < len) {
            e = ents[j * G];
            ldg_raw<GT, VEC>(g, grow + (__float_as_uint(e.y) & 0xfffu) * gstride, wide, pol_first);
          }
        };
        auto step = [&](const float2& e0, const GRaw<GT, VEC>& g0, bool live) {
          const unsigned meta = __float_as_uint(e0.y);
          const int k = (int)((meta >> 12) & 0xffu);
          const bool chg = live && k != st.k_cur;
          // bin switches are handled in one warp-uniform block: each part is predicated per slot (finished
          // run to its carry slot or added to its bin's rows; the new bin's slope row loaded)
          if (__any_sync(0xffffffffu, chg)) {
            const bool has = chg && st.k_cur >= 0;
            const bool to_carry = has && st.first;
            const bool to_rows = has && !st.first;
            const int kc = st.k_cur < 0 ? 0 : st.k_cur;
            float* h = tH + kc * ts;
            float* u = tU + kc * ts;
            Row<VEC> hv, uv;
            hv.zero();
            uv.zero();
            if (to_rows) {
              hv.lds(h);
              uv.lds(u);
            }
#pragma unroll
            for (int e = 0; e < NP; ++e) {
              if constexpr (VEC >= 2) {
                hv.p[e] = add2(hv.p[e], st.Hr.p[e]);
                uv.p[e] = add2(uv.p[e], st.Ur.p[e]);
              } else {
                hv.p[e] = (f2_t)__float_as_uint(hv.lo(e) + st.Hr.lo(e));
                uv.p[e] = (f2_t)__float_as_uint(uv.lo(e) + st.Ur.lo(e));
              }
            }
            if (to_rows) {
              hv.sts(h);
              uv.sts(u);
            }
            if (to_carry) {
              st.Hr.sts(carry);
              st.Ur.sts(carry + D);
              if (c == 0) *carry_bin = st.k_cur;
            }
            if (has) st.first = false;
            if (chg) {
              st.k_cur = k;
              st.Sk.lds(tS + k * ts);
              const float2 rv = ro[k];
              st.r_k = rv.x;
              st.open = rv.y != 0.0f;
              st.Hr.zero();
              st.Ur.zero();
            }
          }
          // every slot of the warp in an open bin (or idle): the step needs no ReLU mask (warp-uniform)
          bool fast = true;
          if constexpr (MASK != kMaskNone) fast = __all_sync(0xffffffffu, !live || st.open);
          if (!live) return;  // a slot past its segment (whole rows are idle together)
          const int s = (int)(meta & 0xfffu);
          const float xv = LIN ? xcol[s] : 0.0f;
          f2_t q[NP];
          const float* trow = tT + st.k_cur * ts;
          float gx = fast ? walk_step<QT, GT, VEC, MASK, EPIV, false>(g0, e0.x, xv, st, trow, pbias, w0r, aw, ab, q)
                          : walk_step<QT, GT, VEC, MASK, EPIV, true>(g0, e0.x, xv, st, trow, pbias, w0r, aw, ab, q);
          const bool tie = (meta >> 31) != 0;
          if (ties && __any_sync(__activemask(), tie)) {  // edge sub-gradient (x == e_k, k > 0): rare
            const int km1 = st.k_cur > 0 ? st.k_cur - 1 : 0;
            Row<VEC> Skm1;
            Skm1.lds(tS + km1 * ts);
            const float r_km1 = ro[km1].x;
            float dp;
            if constexpr (VEC >= 2) {
              f2_t dp2 = 0ull;
#pragma unroll
              for (int e = 0; e < NP; ++e) dp2 = fma2(q[e], Skm1.p[e], dp2);
              float lo, hi;
              unpack2(dp2, lo, hi);
              dp = lo + hi;
            } else {
              dp = __uint_as_float((unsigned)q[0]) * Skm1.lo(0);
            }
            if (tie) gx += r_km1 * dp;
          }
          if (do_gx) {  // the row's nc lane shares summed in lane order; lane c == 0 stores the pair's grad_x
            gx = row_sum(gx, c, nc);
            if (c == 0) gxs[s * Fc] = gx;
          }
        };
        fetch(eb0, gb0, 0);
        fetch(eb1, gb1, 1);
#pragma unroll 1
        for (int j = 0; j < trips; j += 2) {
          step(eb0, gb0, j < len);
          fetch(eb0, gb0, j + 2);
          step(eb1, gb1, j + 1 < len);
          fetch(eb1, gb1, j + 3);
        }
        if (st.k_cur >= 0) {
          if (st.first) {
            st.Hr.sts(carry);
            st.Ur.sts(carry + D);
            if (c == 0) *carry_bin = st.k_cur;
          } else {
            float* h = tH + st.k_cur * ts;
            float* u = tU + st.k_cur * ts;
            st.Hr.add_from(h);
            st.Ur.add_from(u);
            st.Hr.sts(h);
            st.Ur.sts(u);
          }
        }
      }
      __syncthreads();
      // ---- E1: carries, one thread per (feature, segment): a segment whose carry starts a chain of equal
      // carry bins (a chain has one start: empty segments are only at the end) adds the chain's carries to
      // its bin's row, in segment order, 4 columns at a time
      for (int idx = tid; idx < fc * G; idx += nthr) {
        const int i = idx / G, g = idx - i * G;
        const int* cb = L.sCarryBin + i * G;
        const int kb = cb[g];
        if (kb < 0 || (g > 0 && cb[g - 1] == kb)) continue;
        int gend = g + 1;
        while (gend < G && cb[gend] == kb) ++gend;
        float* h = L.sH + kb * ts + i * D;
        float* u = L.sU + kb * ts + i * D;
        const float* cp0 = L.sCarry + ((i * G + g) * 2) * D;
        if ((D & 3) == 0) {
          for (int d = 0; d < D; d += 4) {
            float4 hs = *reinterpret_cast<const float4*>(h + d), us = *reinterpret_cast<const float4*>(u + d);
            for (int g2 = g; g2 < gend; ++g2) {
              const float* cp = cp0 + (g2 - g) * 2 * D + d;
              const float4 ch = *reinterpret_cast<const float4*>(cp), cu = *reinterpret_cast<const float4*>(cp + D);
              hs.x += ch.x; hs.y += ch.y; hs.z += ch.z; hs.w += ch.w;
              us.x += cu.x; us.y += cu.y; us.z += cu.z; us.w += cu.w;
            }
            *reinterpret_cast<float4*>(h + d) = hs;
            *reinterpret_cast<float4*>(u + d) = us;
          }
        } else {
          for (int d = 0; d < D; ++d) {
            float hs = h[d], us = u[d];
            for (int g2 = g; g2 < gend; ++g2) {
              hs += cp0[(g2 - g) * 2 * D + d];
              us += cp0[(g2 - g) * 2 * D + D + d];
            }
            h[d] = hs;
            u[d] = us;
          }
        }
      }
      // ---- E2: grad_x rows of the tile, stored in natural order (a 16-byte row per sample when Fc = 4)
      if (do_gx) {
        float* gdst = a.grad_x + t0 * a.F + f0;
        if (Fc == 4 && fc == 4 && a.gx_vec4) {
          for (int s = tid; s < ns; s += nthr)
            *reinterpret_cast<float4*>(gdst + (int64_t)s * a.F) = *reinterpret_cast<const float4*>(L.sGX + s * 4);
        } else {
          for (int p = tid; p < (ns << lgFc); p += nthr) {
            const int s = p >> lgFc, i = p & (Fc - 1);
            if (i < fc) gdst[(int64_t)s * a.F + i] = L.sGX[p];
          }
        }
      }
    }

    // ---- F: epilogue partials (fixed slot order) and grad_W suffix scan
    __syncthreads();
    float* ws = a.ws + (((int64_t)slot * a.max_segs + seg) * m + member) * ((int64_t)Fc * (B + 3) * D);
    if constexpr (ACC) {
      if (walk_live) {
        float* cp = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        aw.sts(cp);  // sum g x, or sum g' (epilogue A)
        if constexpr (LIN) ab.sts(cp + D);
      }
      __syncthreads();
      for (int colx = tid; colx < fc * D; colx += nthr) {
        const int i = colx / D, d = colx - i * D;
        float s0 = 0.f, s1 = 0.f;
        for (int g = 0; g < G; ++g) {
          const float* cp = L.sCarry + ((i * G + g) * 2) * D + d;
          s0 += cp[0];
          if constexpr (LIN) s1 += cp[D];
        }
        float* row = ws + (int64_t)i * (B + 3) * D;
        if constexpr (LIN) {
          row[(B + 1) * D + d] = s0;
          row[(B + 2) * D + d] = s1;
        } else {
          row[B * D + d] = s0;
        }
      }
    }
    for (int colx = tid; colx < fc * D; colx += nthr) {
      const int i = colx / D, d = colx - i * D;
      const int n = L.sN[i];
      float* row = ws + (int64_t)i * (B + 3) * D;
      float suffix = 0.f;
      for (int j = n - 1; j >= 0; --j) {
        const int o = j * ts + i * D + d;
        row[physical_bin(j, n, B) * D + d] = L.sU[o] + suffix;
        suffix += L.sH[o];
      }
      for (int p = n - 1; p < B - 1; ++p) row[p * D + d] = 0.f;  // padding rows
      if (EPIV != kEpvBias) row[B * D + d] = suffix;
    }
  }
}

// Host: plan + launch (ple_backward.cu) and the per-dtype dispatch.
int bwd_prepare(BwdArgs& a, int vec, size_t* smem, int* grid);
// 2-D tensor map over the gradient [N][F * D] (element type 0 f32, 1 f16, 2 bf16; boxes of the chunk's
// columns x 256 rows) for the L2 prefetch; false when the shape or the alignment allows none (the kernel
// then runs without the prefetch; *map is zeroed).
bool bwd_grad_map(const BwdArgs& a, int elem, CUtensorMap* map);
int bwd_finalize(const BwdArgs& a, int grid, cudaStream_t st);

template <typename QT, typename GT, int VEC, int MASK, int EPIV>
int launch_bwd_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  int grid = 0;
  const int prep = bwd_prepare(a, VEC, &smem, &grid);
  if (prep != PLE_OK) return prep;
  a.g_wide = (GRaw<GT, VEC>::kBytes == 32) && a.g_wide;
  CUtensorMap map;
  a.g_prefetch = bwd_grad_map(a, std::is_same<GT, float>::value ? 0 : std::is_same<GT, __nv_bfloat16>::value ? 2 : 1,
                              &map) ? 1 : 0;
  auto kern = ple_bwd_kernel<QT, GT, VEC, MASK, EPIV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  kern<<<grid, kBwdThreads, smem, st>>>(a, map);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward launch");
  return bwd_finalize(a, grid, st);
}

// Mask variant (ReLU with bias is epilogue A, plain ReLU is epilogue B) and the epilogue terms the requested
// gradients need.
template <typename QT, typename GT, int VEC>
int launch_bwd_mask(const BwdArgs& a, cudaStream_t st) {
  const bool lin = a.epi == kEpiB && (a.grad_x || a.grad_w0 || a.grad_b0);
  const bool bias = a.epi == kEpiA && a.grad_bias;
  if (a.relu && a.epi == kEpiA)
    return bias ? launch_bwd_t<QT, GT, VEC, kMaskReluBias, kEpvBias>(a, st)
                : launch_bwd_t<QT, GT, VEC, kMaskReluBias, kEpvNone>(a, st);
  if (a.relu)
    return lin ? launch_bwd_t<QT, GT, VEC, kMaskRelu, kEpvLin>(a, st) : launch_bwd_t<QT, GT, VEC, kMaskRelu, kEpvNone>(a, st);
  if (lin) return launch_bwd_t<QT, GT, VEC, kMaskNone, kEpvLin>(a, st);
  return bias ? launch_bwd_t<QT, GT, VEC, kMaskNone, kEpvBias>(a, st) : launch_bwd_t<QT, GT, VEC, kMaskNone, kEpvNone>(a, st);
}

template <typename QT, typename GT>
int launch_bwd_dtype(const BwdArgs& a, int vec, cudaStream_t st) {
  switch (vec) {
    case 8: return launch_bwd_mask<QT, GT, 8>(a, st);
    case 4: return launch_bwd_mask<QT, GT, 4>(a, st);
    case 2: return launch_bwd_mask<QT, GT, 2>(a, st);
    default: return launch_bwd_mask<QT, GT, 1>(a, st);
  }
}

}  // namespace ple
