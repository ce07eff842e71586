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
// Work decomposition.  One persistent CTA of kBwdThreads threads per SM owns
// an equal contiguous range of the flattened (feature chunk, sample) space:
// one or a few (chunk, sample range) segments.  A chunk is Fc features; the
// CTA's warps split evenly over them.  A lane group (nc lanes x VEC elements =
// one D row) is the unit of the walk.  Per segment the chunk's tables are
// staged and H/U zeroed; per tile of S_t samples (x arrives by cp.async one
// tile ahead, the tile's gradient rows are bulk-prefetched into L2):
//   A  bin of every pair (the forward's bin indices when given, else a bin
//      search, four searches interleaved per thread) and per-(feature,
//      quarter, bin) counts (integer shared atomics: order independent);
//   B  exclusive scan of the counts (bin-major, quarter-minor);
//   C  stable counting sort: each warp ranks its quarter (lanes with equal
//      bins found from ballots of the bin bits), so the sorted order is a pure
//      function of the input.  The sorted list is stored segment-major (entry
//      p of segment g at p * G + g) so that the lane groups of a warp read
//      adjacent entries;
//   D  walk: a feature's sorted list is cut into at most G equal segments,
//      one per lane group, empty groups only at the end.  The group keeps the
//      current bin's T/S rows and the run's H/U sums in registers and adds a
//      run to the shared histogram once, at its end; the first run of a
//      segment (it may continue the previous segment's last run) goes to a
//      carry slot instead.  Epilogue-B terms (<g, w0>, sum g x, sum g) are
//      taken from the same gradient row.  The group writes its grad_x share to
//      a per-(sample, lane) slot;
//   E  carries are added per chain of equal bins (parallel over chains, in
//      segment order within a chain; a chain has one start because equal
//      carry bins are contiguous); grad_x rows are stored coalesced.
// At the end of a segment a suffix scan over bins turns H/U into grad_W and
// the partial goes to the workspace; ple_bwd_finalize_kernel sums the
// partials of each feature in CTA order.  No floating-point atomics: the
// result is bitwise deterministic for a given shape and device.
// Table rows are padded so that consecutive bins start on different shared
// memory banks (lanes of a warp read rows of different bins).
#pragma once

#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"

namespace ple {

enum { kMaskNone = 0, kMaskRelu = 1, kMaskReluBias = 2 };
// epilogue terms accumulated along the walk: none, sum g' (epilogue A bias), or linear0 (<g, w0>, sum g x,
// sum g; epilogue B)
enum { kEpvNone = 0, kEpvBias = 1, kEpvLin = 2 };

struct BwdDims {
  int Fc, Wf, S_t, G, nc;  // G = lane groups per feature
};

// Floats between bin rows of the tables: Fc * D rounded up to 4, plus 4 when
// that is a multiple of 8, so that consecutive bins shift by 16 bytes modulo
// the 128-byte bank window.
__host__ __device__ __forceinline__ int table_stride(int Fc, int D) {
  int ts = (Fc * D + 3) & ~3;
  if (((ts >> 2) & 1) == 0) ts += 4;
  return ts;
}

struct BwdLayout {
  float *sT, *sS, *sH, *sU;  // [B][ts] rows, feature i at i * D (bin-major, padded)
  float *sK, *sE, *sR;       // [2^lgk][Fc] search keys (interior edges), [B][Fc] left edges e_k,
                             // [B][Fc] inverse widths
  float *sX;                 // [2][S_t][Fc] x tiles
  float *sGX;                // [Fc][S_t][nc] grad_x shares
  float *sCarry;             // [Fc][G][2][D]
  float2* sEnt;              // [Fc][S_t + G] sorted (q(t), meta bits: s | k << 16 | tie << 31), segment-major
  uint8_t* sKey;             // [Fc][S_t] bins of the tile
  int *sN, *sCnt, *sCarryBin, *sTie;  // sTie[Fc]: the tile has an edge tie in feature i
};

__host__ __device__ __forceinline__ size_t bwd_layout_bytes(int B, int D, int key_rows, const BwdDims& m,
                                                            BwdLayout* L, unsigned char* base) {
  const size_t tab = (size_t)B * table_stride(m.Fc, D);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 15) & ~(size_t)15;
    return base + o;
  };
  unsigned char* pT = take(4 * tab * 4);
  unsigned char* pCarry = take((size_t)m.Fc * m.G * 2 * D * 4);
  unsigned char* pGX = take((size_t)m.Fc * m.S_t * m.nc * 4);
  unsigned char* pEnt = take((size_t)m.Fc * (m.S_t + m.G) * 8);
  unsigned char* pX = take((size_t)2 * m.S_t * m.Fc * 4);
  unsigned char* pK = take((size_t)key_rows * m.Fc * 4);
  unsigned char* pE = take((size_t)B * m.Fc * 4);
  unsigned char* pR = take((size_t)B * m.Fc * 4);
  unsigned char* pN = take((size_t)m.Fc * 4);
  unsigned char* pCnt = take((size_t)m.Fc * B * m.Wf * 4);
  unsigned char* pCB = take((size_t)m.Fc * m.G * 4);
  unsigned char* pTie = take((size_t)m.Fc * 4);
  unsigned char* pKey = take((size_t)m.Fc * m.S_t);
  if (L) {
    L->sT = reinterpret_cast<float*>(pT);
    L->sS = L->sT + tab;
    L->sH = L->sS + tab;
    L->sU = L->sH + tab;
    L->sCarry = reinterpret_cast<float*>(pCarry);
    L->sGX = reinterpret_cast<float*>(pGX);
    L->sEnt = reinterpret_cast<float2*>(pEnt);
    L->sX = reinterpret_cast<float*>(pX);
    L->sK = reinterpret_cast<float*>(pK);
    L->sE = reinterpret_cast<float*>(pE);
    L->sR = reinterpret_cast<float*>(pR);
    L->sN = reinterpret_cast<int*>(pN);
    L->sCnt = reinterpret_cast<int*>(pCnt);
    L->sCarryBin = reinterpret_cast<int*>(pCB);
    L->sTie = reinterpret_cast<int*>(pTie);
    L->sKey = reinterpret_cast<uint8_t*>(pKey);
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

// Raw gradient chunk of VEC elements of GT, kept packed until use.
template <typename GT, int VEC> struct GRaw {
  static constexpr int kBytes = (int)sizeof(GT) * VEC;
  static constexpr int kWords = (kBytes + 3) / 4;
  unsigned w[kWords];
};

// Widest access that divides the chunk: rows are D = nc * VEC elements, so
// every chunk start is a multiple of it (the host checks the base pointer).
template <typename GT, int VEC> constexpr int chunk_align() {
  return (sizeof(GT) * VEC) % 16 == 0 ? 16 : (sizeof(GT) * VEC) % 8 == 0 ? 8 : (sizeof(GT) * VEC) % 4 == 0 ? 4 : 2;
}

template <typename GT, int VEC>
__device__ __forceinline__ void ldg_raw(GRaw<GT, VEC>& r, const GT* p) {
  constexpr int bytes = GRaw<GT, VEC>::kBytes;
  constexpr int al = chunk_align<GT, VEC>();
  if constexpr (al == 16) {
#pragma unroll
    for (int j = 0; j < bytes / 16; ++j) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p) + j);
      r.w[4 * j] = a.x; r.w[4 * j + 1] = a.y; r.w[4 * j + 2] = a.z; r.w[4 * j + 3] = a.w;
    }
  } else if constexpr (al == 8) {
#pragma unroll
    for (int j = 0; j < bytes / 8; ++j) {
      const uint2 a = __ldg(reinterpret_cast<const uint2*>(p) + j);
      r.w[2 * j] = a.x; r.w[2 * j + 1] = a.y;
    }
  } else if constexpr (al == 4) {
#pragma unroll
    for (int j = 0; j < bytes / 4; ++j) r.w[j] = __ldg(reinterpret_cast<const unsigned*>(p) + j);
  } else {
    r.w[0] = (unsigned)__ldg(reinterpret_cast<const unsigned short*>(p));
  }
}

// Elements e, e + 1 (e even) of a raw chunk as fp32.
template <typename GT, int VEC>
__device__ __forceinline__ void raw_pair(const GRaw<GT, VEC>& r, int e, float& lo, float& hi) {
  if constexpr (std::is_same<GT, float>::value) {
    lo = __uint_as_float(r.w[e]);
    hi = __uint_as_float(r.w[e + 1]);
  } else {
    widen_pack<GT>(r.w[e >> 1], lo, hi);
  }
}
template <typename GT, int VEC>
__device__ __forceinline__ float raw_one(const GRaw<GT, VEC>& r) {
  if constexpr (std::is_same<GT, float>::value) return __uint_as_float(r.w[0]);
  else return Dt<GT>::to_f(*reinterpret_cast<const GT*>(&r.w[0]));
}

// Largest value that rounds to zero in QT: with no bias after the rounding,
// q(p) <= 0 exactly when p <= threshold (ties round to the even zero).
template <typename QT> __device__ __forceinline__ float zero_round_threshold() {
  if constexpr (std::is_same<QT, float>::value) return 0.0f;
  else if constexpr (std::is_same<QT, __nv_bfloat16>::value) return __uint_as_float(0x00008000u);  // 2^-134
  else return 2.98023223876953125e-08f;                                                           // 2^-25
}

// VEC fp32 values of one D-row chunk held as packed pairs (VEC >= 2) or a
// scalar (VEC == 1), so the arithmetic maps onto fp32x2 instructions.
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
    } else if constexpr (VEC == 2) {
      p[0] = *reinterpret_cast<const unsigned long long*>(src);
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
    } else if constexpr (VEC == 2) {
      p[0] = __ldg(reinterpret_cast<const unsigned long long*>(src));
    } else {
      p[0] = (f2_t)__float_as_uint(__ldg(src));
    }
  }
  __device__ __forceinline__ void sts(float* dst) const {
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int e = 0; e < NP; e += 2)
        *reinterpret_cast<ulonglong2*>(dst + 2 * e) = make_ulonglong2(p[e], p[e + 1]);
    } else if constexpr (VEC == 2) {
      *reinterpret_cast<unsigned long long*>(dst) = p[0];
    } else {
      *dst = __uint_as_float((unsigned)p[0]);
    }
  }
  __device__ __forceinline__ float lo(int e) const {
    float a, b;
    unpack2(p[e], a, b);
    return a;
  }
};

// Gradient rows per block of the walk; two blocks are in flight per lane.
template <typename GT, int VEC> constexpr int walk_depth() {
  return GRaw<GT, VEC>::kBytes >= 32 ? 1 : (GRaw<GT, VEC>::kBytes >= 16 ? 2 : 4);
}

// Add a finished run to the shared histogram or, for the segment's first run
// (which may continue the previous segment's last run), to the carry slot.
template <int VEC>
__device__ __forceinline__ void flush_run(const Row<VEC>& H, const Row<VEC>& U, bool& first_run, int k_cur,
                                          float* carry, int* carry_bin, int D, int c, float* h, float* u) {
  if (first_run) {
    H.sts(carry);
    U.sts(carry + D);
    if (c == 0) *carry_bin = k_cur;
    first_run = false;
  } else {
    Row<VEC> hv, uv;
    hv.lds(h);
    uv.lds(u);
#pragma unroll
    for (int e = 0; e < Row<VEC>::NP; ++e) {
      hv.p[e] = add2(hv.p[e], H.p[e]);
      uv.p[e] = add2(uv.p[e], U.p[e]);
    }
    hv.sts(h);
    uv.sts(u);
  }
}

// Per-lane inputs of one walk step.
template <typename GT, int VEC> struct WalkIn {
  float2 ent;
  GRaw<GT, VEC> g;
};

template <typename GT, int VEC, int DEPTH>
__device__ __forceinline__ void walk_fetch(WalkIn<GT, VEC> (&in)[DEPTH], const float2* ents, int estride, int base,
                                           int len, const GT* grow, unsigned gstride) {
#pragma unroll
  for (int u = 0; u < DEPTH; ++u) {
    const int step = base + u;
    if (step < len) {
      in[u].ent = ents[step * estride];
      ldg_raw<GT, VEC>(in[u].g, grow + (unsigned long long)(__float_as_uint(in[u].ent.y) & 0xffffu) * gstride);
    }
  }
}

struct WalkCtx {
  const float* tS;  // S[0] row chunk of this lane: S[k] at tS + k * kstride (T, H, U likewise)
  const float* tT;
  float* tH;
  float* tU;
  const float* rK;  // r[0] of this feature: r[k] at rK[k << lgFc]
  float* gx;        // this lane's grad_x share of sample s at gx[s * nc]
  float* carry;
  int* carry_bin;
  const float* xcol;  // x of sample s at xcol[s << lgFc]
  int kstride, lgFc, nc, D, c;
};

template <typename QT, typename GT, int VEC, int MASK, int EPIV, int DEPTH>
__device__ __forceinline__ void walk_block(const WalkCtx& w, WalkIn<GT, VEC> (&in)[DEPTH], int base, int len,
                                           int& k_cur, bool& first_run, float& r_k, Row<VEC>& Tk, Row<VEC>& Sk,
                                           Row<VEC>& Hrun, Row<VEC>& Urun, const Row<VEC>& pbias, Row<VEC>& braw,
                                           const Row<VEC>& w0r, Row<VEC>& acc_w0, Row<VEC>& acc_b0, bool ties,
                                           bool do_gx) {
  constexpr int NP = Row<VEC>::NP;
  constexpr bool LIN = EPIV == kEpvLin;
  const float thr = zero_round_threshold<QT>();
#pragma unroll
  for (int u = 0; u < DEPTH; ++u) {
    const bool live = base + u < len;
    const unsigned meta = __float_as_uint(in[u].ent.y);
    const int k = (int)((meta >> 16) & 0x7fffu);
    if (live && k != k_cur) {
      if (k_cur >= 0)
        flush_run<VEC>(Hrun, Urun, first_run, k_cur, w.carry, w.carry_bin, w.D, w.c, w.tH + k_cur * w.kstride,
                       w.tU + k_cur * w.kstride);
      k_cur = k;
      Tk.lds(w.tT + k * w.kstride);
      Sk.lds(w.tS + k * w.kstride);
      r_k = w.rK[k << w.lgFc];
      Hrun.zero();
      Urun.zero();
    }
    const bool tie = live && (meta >> 31);
    if (live) {
      const float tq = in[u].ent.x;
      float gx;
      f2_t q[NP];
      if constexpr (VEC >= 2) {
        const f2_t t2 = pack2(tq, tq);
        f2_t d2 = 0ull, dw2 = 0ull, x2 = 0ull;
        if constexpr (LIN) {
          const float xv = w.xcol[(int)(meta & 0xffffu) << w.lgFc];
          x2 = pack2(xv, xv);
        }
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          float g0, g1;
          raw_pair<GT, VEC>(in[u].g, 2 * e, g0, g1);
          if constexpr (LIN) {
            const f2_t gg = pack2(g0, g1);
            dw2 = fma2(gg, w0r.p[e], dw2);
            acc_w0.p[e] = fma2(gg, x2, acc_w0.p[e]);
            acc_b0.p[e] = add2(acc_b0.p[e], gg);
          }
          float q0 = g0, q1 = g1;
          if constexpr (MASK != kMaskNone) {
            float p0, p1;
            unpack2(fma2(t2, Sk.p[e], Tk.p[e]), p0, p1);
            if constexpr (MASK == kMaskReluBias) {
              round2<QT>(p0, p1);
              float b0, b1;
              unpack2(pbias.p[e], b0, b1);
              p0 += b0;
              p1 += b1;
              q0 = p0 <= 0.f ? 0.f : g0;
              q1 = p1 <= 0.f ? 0.f : g1;
            } else {
              q0 = p0 <= thr ? 0.f : g0;
              q1 = p1 <= thr ? 0.f : g1;
            }
          }
          if constexpr (EPIV == kEpvBias) braw.p[e] = add2(braw.p[e], pack2(q0, q1));
          if constexpr (!std::is_same<GT, QT>::value && !std::is_same<QT, float>::value) round2<QT>(q0, q1);
          q[e] = pack2(q0, q1);
          Hrun.p[e] = add2(Hrun.p[e], q[e]);
          Urun.p[e] = fma2(t2, q[e], Urun.p[e]);
          d2 = fma2(q[e], Sk.p[e], d2);
        }
        float lo, hi;
        unpack2(d2, lo, hi);
        gx = r_k * (lo + hi);
        if constexpr (LIN) {
          unpack2(dw2, lo, hi);
          gx += lo + hi;
        }
      } else {
        const float g0 = raw_one<GT, VEC>(in[u].g);
        if constexpr (LIN) {
          const float xv = w.xcol[(int)(meta & 0xffffu) << w.lgFc];
          acc_w0.p[0] = (f2_t)__float_as_uint(fmaf(g0, xv, acc_w0.lo(0)));
          acc_b0.p[0] = (f2_t)__float_as_uint(acc_b0.lo(0) + g0);
        }
        float q0 = g0;
        const float s0 = Sk.lo(0);
        if constexpr (MASK != kMaskNone) {
          float p0 = fmaf(tq, s0, Tk.lo(0));
          if constexpr (MASK == kMaskReluBias) {
            p0 = quantize<QT>(p0) + pbias.lo(0);
            q0 = p0 <= 0.f ? 0.f : g0;
          } else {
            q0 = p0 <= thr ? 0.f : g0;
          }
        }
        if constexpr (EPIV == kEpvBias) braw.p[0] = (f2_t)__float_as_uint(braw.lo(0) + q0);
        if constexpr (!std::is_same<GT, QT>::value) q0 = quantize<QT>(q0);
        q[0] = (f2_t)__float_as_uint(q0);
        Hrun.p[0] = (f2_t)__float_as_uint(Hrun.lo(0) + q0);
        Urun.p[0] = (f2_t)__float_as_uint(fmaf(tq, q0, Urun.lo(0)));
        gx = r_k * (q0 * s0);
        if constexpr (LIN) gx += g0 * w0r.lo(0);
      }
      if (ties && __any_sync(__activemask(), tie)) {  // edge sub-gradient (x == e_k, k > 0): rare
        const int km1 = k_cur > 0 ? k_cur - 1 : 0;
        Row<VEC> Skm1;
        Skm1.lds(w.tS + km1 * w.kstride);
        const float r_km1 = w.rK[km1 << w.lgFc];
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
      if (do_gx) w.gx[(int)(meta & 0xffffu) * w.nc] = gx;
    }
  }
}

// The chunk's tables for one segment: edges (transposed for the search),
// inverse widths, S = q(W) in logical bin order and its exclusive prefix T;
// H/U zeroed.
// Four interleaved key counts (key_count over the transposed key table [2^LG][Fc], column ii[j]).
template <int LG>
__device__ __forceinline__ void key_count4(const float (&xs)[4], int (&c)[4], const float* sK, const int (&ii)[4],
                                           int lgFc) {
#pragma unroll
  for (int j = 0; j < 4; ++j) c[j] = 0;
#pragma unroll
  for (int h = (1 << LG) >> 1; h > 0; h >>= 1) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(xs[j] < sK[((c[j] + h - 1) << lgFc) + ii[j]])) c[j] += h;
  }
}

template <typename QT>
__device__ __forceinline__ void stage_tables(const BwdArgs& a, const BwdLayout& L, int f0, int fc, int lgFc, int ts,
                                             int tid, int nthr) {
  const int Fc = 1 << lgFc, B = a.B, D = a.D, nkeys = 1 << a.lgk;
  for (int i = tid; i < Fc; i += nthr) {
    int n = i < fc ? a.n_bins[f0 + i] : 1;
    L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  for (int idx = tid; idx < B * ts; idx += nthr) {
    L.sH[idx] = 0.0f;
    L.sU[idx] = 0.0f;
    L.sS[idx] = 0.0f;
  }
  __syncthreads();
  // search keys: interior edges e_1 .. e_{n-1}, then +inf (key_count capped at n - 1 = the clamped bin)
  for (int idx = tid; idx < nkeys * Fc; idx += nthr) {
    const int j = idx >> lgFc, i = idx & (Fc - 1);
    float e = __int_as_float(0x7f800000);
    if (i < fc && j + 1 < L.sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j + 1];
    L.sK[idx] = e;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {  // left edges e_k of the real bins
    const int j = idx >> lgFc, i = idx & (Fc - 1);
    L.sE[idx] = (i < fc && j < L.sN[i]) ? a.edges[(int64_t)(f0 + i) * (B + 1) + j] : 0.0f;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {
    const int j = idx >> lgFc, i = idx & (Fc - 1);
    L.sR[idx] = (i < fc && j < L.sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
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
}

template <typename QT, typename GT, int VEC, int MASK, int EPIV>
__global__ void __launch_bounds__(kBwdThreads, 1) ple_bwd_kernel(const BwdArgs a) {
  constexpr bool LIN = EPIV == kEpvLin;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int DEPTH = walk_depth<GT, VEC>();
  const int lgFc = a.lgFc, lgWf = a.lgWf, lgSt = a.lgSt;
  const int Fc = 1 << lgFc, Wf = 1 << lgWf, S_t = 1 << lgSt;
  const int B = a.B, D = a.D;
  const int nc = D / VEC;
  const int Rint = 32 / nc;
  const int G = Wf * Rint;
  const int ES = S_t + G;  // entries per feature (segment-major, see phase C)
  const int ts = table_stride(Fc, D);
  BwdLayout L;
  bwd_layout_bytes(B, D, 1 << a.lgk, BwdDims{Fc, Wf, S_t, G, nc}, &L, smem_raw);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int r = lane / nc, c = lane - r * nc;
  const int cd = c * VEC;
  // warp wid serves feature my_i; its lane groups are segments g_seg of that feature
  const int my_i = wid >> lgWf;
  const int my_w = wid & (Wf - 1);
  const int g_seg = my_w * Rint + r;
  const bool do_gx = a.grad_x != nullptr;
  constexpr bool acc_bias = EPIV == kEpvBias;  // sum g' for the epilogue-A bias gradient
  const GT* gptr = reinterpret_cast<const GT*>(a.g);
  const int lg_q = lgSt - lgWf;  // quarter length (log2)

  const int64_t total = (int64_t)a.n_chunks * a.N;
  int64_t u_lo = total * blockIdx.x / gridDim.x;
  const int64_t u_hi = total * (blockIdx.x + 1) / gridDim.x;

  for (int seg = 0; u_lo < u_hi; ++seg) {
    const int chunk = (int)(u_lo / a.N);
    const int64_t s_begin = u_lo - (int64_t)chunk * a.N;
    const int64_t s_end = min64(a.N, s_begin + (u_hi - u_lo));
    u_lo += s_end - s_begin;
    const int f0 = chunk << lgFc;
    const int fc = min(Fc, a.F - f0);
    const bool walk_live = r < Rint && my_i < fc;
    const bool x_vec4 = a.x_vec4 && fc == Fc;
    // bulk L2 prefetch of a sample's fc gradient rows: 16-byte aligned start and length
    const int64_t row_bytes_all = (int64_t)a.F * D * (int64_t)sizeof(GT);
    const unsigned pf_bytes = (unsigned)(fc * D * (int)sizeof(GT));
    const bool pf_rows = (pf_bytes & 15u) == 0 && (row_bytes_all & 15) == 0 &&
                         ((reinterpret_cast<uintptr_t>(gptr + (int64_t)f0 * D)) & 15) == 0;

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

    __syncthreads();  // previous segment finished with every shared buffer
    load_x(s_begin, (int)min64(S_t, s_end - s_begin), L.sX);
    stage_tables<QT>(a, L, f0, fc, lgFc, ts, tid, nthr);

    // per-lane parameters and accumulators that live across the segment's tiles; sum g' (epilogue A)
    // shares acc_w0's registers
    Row<VEC> pbias, w0r, acc_w0, acc_b0;
    Row<VEC>& braw = acc_w0;
    pbias.zero();
    w0r.zero();
    acc_w0.zero();
    acc_b0.zero();
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
      for (int idx = tid; idx < Fc * B * Wf; idx += nthr) L.sCnt[idx] = 0;
      cp_async_wait_all();
      __syncthreads();  // x tile landed, counts zeroed, previous tile finished
      if (t0 + S_t < s_end) load_x(t0 + S_t, (int)min64(S_t, s_end - t0 - S_t), L.sX + (buf ^ 1) * S_t * Fc);
      // the walk reads this tile's gradient rows in bin order: start streaming them into L2 now
      if (pf_rows) {
        const char* g0 = reinterpret_cast<const char*>(gptr + (t0 * a.F + f0) * (int64_t)D);
        for (int s = tid; s < ns; s += nthr) prefetch_l2_bulk(g0 + (int64_t)s * row_bytes_all, pf_bytes);
      }

      // ---- A: bins and counts
      {
        const int npairs = ns << lgFc;
        for (int p0 = tid; p0 < npairs; p0 += 4 * nthr) {
          int kk[4], ii[4];
          bool ok[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int p = p0 + j * nthr;
            ii[j] = p & (Fc - 1);
            ok[j] = p < npairs && ii[j] < fc;
          }
          if (a.bin_idx != nullptr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              kk[j] = 0;
              if (ok[j]) {
                const int64_t pair = (t0 + ((p0 + j * nthr) >> lgFc)) * a.F + f0 + ii[j];
                const int k = a.bin_idx_bytes == 1 ? (int)reinterpret_cast<const uint8_t*>(a.bin_idx)[pair]
                            : a.bin_idx_bytes == 2 ? (int)reinterpret_cast<const int16_t*>(a.bin_idx)[pair]
                                                   : reinterpret_cast<const int32_t*>(a.bin_idx)[pair];
                kk[j] = k < 0 ? 0 : (k >= L.sN[ii[j]] ? L.sN[ii[j]] - 1 : k);
              }
            }
          } else {
            // count of interior edges <= x (capped at n - 1: the clamped bin), four searches interleaved
            float xs[4];
            int cnt[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) xs[j] = ok[j] ? sX[p0 + j * nthr] : 0.f;
            switch (a.lgk) {
#define PLE_BWD_COUNT(LL) \
  case LL: key_count4<LL>(xs, cnt, L.sK, ii, lgFc); break;
              PLE_BWD_COUNT(0) PLE_BWD_COUNT(1) PLE_BWD_COUNT(2) PLE_BWD_COUNT(3) PLE_BWD_COUNT(4)
              PLE_BWD_COUNT(5) PLE_BWD_COUNT(6) PLE_BWD_COUNT(7) PLE_BWD_COUNT(8)
#undef PLE_BWD_COUNT
              default:
#pragma unroll
                for (int j = 0; j < 4; ++j) cnt[j] = 0;
                break;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int n1 = L.sN[ii[j]] - 1;
              kk[j] = cnt[j] < n1 ? cnt[j] : n1;
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (ok[j]) {
              const int s = (p0 + j * nthr) >> lgFc;
              L.sKey[(ii[j] << lgSt) + s] = (uint8_t)kk[j];
              atomicAdd(&L.sCnt[((ii[j] * B + kk[j]) << lgWf) + (s >> lg_q)], 1);
            }
          }
        }
      }
      __syncthreads();
      // ---- B: exclusive scan per feature (bin-major, quarter-minor); carry slots emptied (the previous
      // tile's carries were consumed before this tile's first barrier)
      for (int i = wid; i < fc; i += nthr >> 5) warp_exclusive_scan(L.sCnt + ((i * B) << lgWf), B << lgWf, lane);
      for (int idx = tid; idx < Fc * G; idx += nthr) L.sCarryBin[idx] = -1;
      for (int idx = tid; idx < Fc; idx += nthr) L.sTie[idx] = 0;
      __syncthreads();
      // ---- C: stable scatter of each quarter into sorted order; sorted position p is stored at
      // (p % Lseg) * G + p / Lseg
      if (my_i < fc) {
        const int lo = my_w << lg_q, hi = min(lo + (1 << lg_q), ns);
        for (int base = lo; base < hi; base += 32) {
          const int s = base + lane;
          const bool v = s < hi;
          const unsigned act = __ballot_sync(0xffffffffu, v);
          if (v) {
            const int k = L.sKey[(my_i << lgSt) + s];
            // lanes with the same bin: intersect the ballots of every bin bit (bins are < B)
            unsigned peers = act;
            for (int bit = 1; bit < B; bit <<= 1) {
              const unsigned bal = __ballot_sync(act, k & bit);
              peers &= (k & bit) ? bal : ~bal;
            }
            const int leader = __ffs(peers) - 1;
            const int rank = __popc(peers & ((1u << lane) - 1u));
            int* cur = &L.sCnt[((my_i * B + k) << lgWf) + my_w];
            int pos0 = 0;
            if (lane == leader) pos0 = *cur;
            pos0 = __shfl_sync(peers, pos0, leader);
            if (lane == leader) *cur = pos0 + __popc(peers);
            const float xv = sX[(s << lgFc) + my_i];
            const float e_k = L.sE[(k << lgFc) + my_i];
            const float t = (xv - e_k) * L.sR[(k << lgFc) + my_i];
            const unsigned tie = (k > 0 && xv == e_k) ? 0x80000000u : 0u;
            if (tie) L.sTie[my_i] = 1;
            const unsigned pos = (unsigned)(pos0 + rank);
            const unsigned gq = pow2L ? pos >> lgL : __umulhi(pos, mL);
            L.sEnt[my_i * ES + (int)(pos - gq * (unsigned)Lseg) * G + (int)gq] =
                make_float2(quantize<QT>(t), __uint_as_float((unsigned)s | ((unsigned)k << 16) | tie));
          }
          __syncwarp();
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
        WalkCtx w;
        const int toff = my_i * D + cd;
        w.tS = L.sS + toff;
        w.tT = L.sT + toff;
        w.tH = L.sH + toff;
        w.tU = L.sU + toff;
        w.rK = L.sR + my_i;
        w.gx = L.sGX + (my_i << lgSt) * nc + c;
        w.carry = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        w.carry_bin = L.sCarryBin + my_i * G + g_seg;
        w.xcol = sX + my_i;
        w.kstride = ts;
        w.lgFc = lgFc;
        w.nc = nc;
        w.D = D;
        w.c = c;
        const float2* ents = L.sEnt + my_i * ES + (g_seg < G ? g_seg : 0);
        const GT* grow = gptr + (t0 * a.F + f0 + my_i) * (int64_t)D + cd;
        const unsigned gstride = (unsigned)a.F * (unsigned)D;
        const bool ties = L.sTie[my_i] != 0;
        int k_cur = -1;
        bool first_run = true;
        float r_k = 0.f;
        Row<VEC> Tk, Sk, Hrun, Urun;
        Tk.zero();
        Sk.zero();
        Hrun.zero();
        Urun.zero();
        WalkIn<GT, VEC> ia[DEPTH], ib[DEPTH];
        walk_fetch<GT, VEC, DEPTH>(ia, ents, G, 0, len, grow, gstride);
        for (int base = 0; base < trips; base += 2 * DEPTH) {
          walk_fetch<GT, VEC, DEPTH>(ib, ents, G, base + DEPTH, len, grow, gstride);
          walk_block<QT, GT, VEC, MASK, EPIV, DEPTH>(w, ia, base, len, k_cur, first_run, r_k, Tk, Sk, Hrun, Urun,
                                                     pbias, braw, w0r, acc_w0, acc_b0, ties, do_gx);
          walk_fetch<GT, VEC, DEPTH>(ia, ents, G, base + 2 * DEPTH, len, grow, gstride);
          walk_block<QT, GT, VEC, MASK, EPIV, DEPTH>(w, ib, base + DEPTH, len, k_cur, first_run, r_k, Tk, Sk, Hrun,
                                                     Urun, pbias, braw, w0r, acc_w0, acc_b0, ties, do_gx);
        }
        if (k_cur >= 0)
          flush_run<VEC>(Hrun, Urun, first_run, k_cur, w.carry, w.carry_bin, D, c, w.tH + k_cur * ts,
                         w.tU + k_cur * ts);
      }
      __syncthreads();
      // ---- E1: carries, one thread per (feature, chain start, 4-element column block)
      {
        const int dq = (D & 3) == 0 ? 4 : 1;
        const int nd = D / dq;
        for (int item = tid; item < fc * G * nd; item += nthr) {
          const int i = item / (G * nd);
          const int rem = item - i * G * nd;
          const int g = rem / nd, dd = (rem - g * nd) * dq;
          const int* cb = L.sCarryBin + i * G;
          const int kb = cb[g];
          if (kb < 0 || (g > 0 && cb[g - 1] == kb)) continue;
          float hs[4] = {0.f, 0.f, 0.f, 0.f}, us[4] = {0.f, 0.f, 0.f, 0.f};
          for (int g2 = g; g2 < G && cb[g2] == kb; ++g2) {
            const float* cp = L.sCarry + ((i * G + g2) * 2) * D + dd;
            for (int e = 0; e < dq; ++e) {
              hs[e] += cp[e];
              us[e] += cp[D + e];
            }
          }
          float* h = L.sH + kb * ts + i * D + dd;
          float* u = L.sU + kb * ts + i * D + dd;
          for (int e = 0; e < dq; ++e) {
            h[e] += hs[e];
            u[e] += us[e];
          }
        }
      }
      // ---- E2: grad_x = sum of the lanes' shares, stored in natural order
      if (do_gx) {
        for (int p = tid; p < (ns << lgFc); p += nthr) {
          const int s = p >> lgFc, i = p & (Fc - 1);
          if (i < fc) {
            const float* part = L.sGX + ((i << lgSt) + s) * nc;
            float v = 0.f;
            for (int cc = 0; cc < nc; ++cc) v += part[cc];
            a.grad_x[(t0 + s) * a.F + f0 + i] = v;
          }
        }
      }
    }

    // ---- F: epilogue partials (fixed group order) and grad_W suffix scan
    __syncthreads();
    float* ws = a.ws + ((int64_t)blockIdx.x * a.max_segs + seg) * ((int64_t)Fc * (B + 3) * D);
    if constexpr (LIN || acc_bias) {
      if (walk_live) {
        float* cp = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        acc_w0.sts(cp);  // sum g x, or sum g' (epilogue A)
        if constexpr (LIN) acc_b0.sts(cp + D);
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
      if (!acc_bias) row[B * D + d] = suffix;
    }
  }
}

// Host: plan + launch (ple_backward.cu) and the per-dtype dispatch.
int bwd_prepare(BwdArgs& a, int vec, size_t* smem, int* grid);
int bwd_finalize(const BwdArgs& a, int grid, cudaStream_t st);

template <typename QT, typename GT, int VEC, int MASK, int EPIV>
int launch_bwd_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  int grid = 0;
  const int prep = bwd_prepare(a, VEC, &smem, &grid);
  if (prep != PLE_OK) return prep;
  auto kern = ple_bwd_kernel<QT, GT, VEC, MASK, EPIV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  kern<<<grid, kBwdThreads, smem, st>>>(a);
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
