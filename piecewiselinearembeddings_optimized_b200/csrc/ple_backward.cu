// ple_backward.cu - fused, deterministic PLE backward for sm_100a.
//
// Gradients (reference backward_cuda.cu:343-492 for grad_x, :268-336 and
// :859-925 for grad_W; the epilogue gradients follow autograd of
// module.py:230-248):
//   g'       = g * [pre-activation > 0]            (ReLU; g' = g without it)
//   grad_W[i, phys(j)] = U[j] + sum_{j' > j} H[j']  with
//       H[j] = sum_{b: k_b = j} q(g'_b),  U[j] = sum_{b: k_b = j} q(t_b) q(g'_b)
//   grad_x   = r_k <q(g'), S[k]> + [k > 0, x == e_k] r_{k-1} <q(g'), S[k-1]>
//              (+ <g, w0> for epilogue B)
//   grad_bias = sum_b g'  (A);  grad_w0 = sum_b g x, grad_b0 = sum_b g  (B)
//
// Work decomposition.  The grid is one persistent CTA per SM; CTA j owns an
// equal contiguous range of the flattened (feature chunk, sample) space, i.e.
// one or a few (chunk, sample range) segments.  16 warps = Fc features x Wf
// warps.  Per segment the chunk's tables are staged and H/U zeroed; per tile
// of S_t samples (x arrives by cp.async one tile ahead):
//   A  bin of every pair (the forward's bin indices when given, else a bin
//      search), per-(feature, quarter, bin) counts (integer shared atomics:
//      order independent);
//   B  exclusive scan of the counts (bin-major, quarter-minor);
//   C  stable counting sort: each warp ranks its quarter with __match_any_sync,
//      so the sorted order is a pure function of the input;
//   D  walk: a feature's sorted list is cut into G equal contiguous segments;
//      each lane group (nc lanes x VEC elements = one D row) walks one segment
//      four samples at a time (four gradient-row gathers in flight), keeping
//      the active bin's T/S rows and running H/U sums in registers and
//      flushing a run to the shared H/U histogram once, by its only owner (the
//      segment in which it starts); a segment's first run goes to a carry
//      slot.  Each lane writes its share of grad_x to a per-(sample, lane)
//      partial slot;
//   E  carries are added in segment order; grad_x partials are summed and
//      stored coalesced.
// At the end of a segment a suffix scan over bins turns H/U into grad_W and
// the partial goes to the workspace; ple_bwd_finalize_kernel sums the
// partials of each feature in CTA order.  No floating-point atomics:
// bitwise deterministic for a given shape and device.
#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"

namespace ple {

struct BwdLayout {
  float *sT, *sS, *sH, *sU, *sE, *sR, *sGX, *sCarry, *sXb;
  float2* sEnt;     // sorted (x, q(t))
  unsigned* sMeta;  // sorted s | k << 16 | tie << 31
  uint8_t* sKey;
  int *sN, *sCnt, *sCarryBin;
};

struct BwdDims {
  int Fc, Wf, S_t, G, nc;
};

__host__ __device__ __forceinline__ size_t bwd_layout_bytes(const BwdArgs& a, const BwdDims& m, BwdLayout* L,
                                                            unsigned char* base) {
  const size_t tab = (size_t)a.B * m.Fc * a.D;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 15) & ~(size_t)15;
    return base + o;
  };
  unsigned char* pT = take(4 * tab * 4);
  unsigned char* pCarry = take((size_t)m.Fc * m.G * 2 * a.D * 4);
  unsigned char* pGX = take((size_t)m.Fc * m.S_t * m.nc * 4);  // grad_x partials [Fc][S_t][nc]
  unsigned char* pEnt = take((size_t)m.Fc * m.S_t * 8);
  unsigned char* pMeta = take((size_t)m.Fc * m.S_t * 4);
  unsigned char* pXb = take((size_t)2 * m.S_t * m.Fc * 4);
  unsigned char* pE = take((size_t)a.pow2 * m.Fc * 4);
  unsigned char* pR = take((size_t)a.B * m.Fc * 4);
  unsigned char* pN = take((size_t)m.Fc * 4);
  unsigned char* pCnt = take((size_t)m.Fc * a.B * m.Wf * 4);
  unsigned char* pCB = take((size_t)m.Fc * m.G * 4);
  unsigned char* pKey = take((size_t)m.Fc * m.S_t);
  if (L) {
    L->sT = reinterpret_cast<float*>(pT);
    L->sS = L->sT + tab;
    L->sH = L->sS + tab;
    L->sU = L->sH + tab;
    L->sCarry = reinterpret_cast<float*>(pCarry);
    L->sGX = reinterpret_cast<float*>(pGX);
    L->sEnt = reinterpret_cast<float2*>(pEnt);
    L->sMeta = reinterpret_cast<unsigned*>(pMeta);
    L->sXb = reinterpret_cast<float*>(pXb);
    L->sE = reinterpret_cast<float*>(pE);
    L->sR = reinterpret_cast<float*>(pR);
    L->sN = reinterpret_cast<int*>(pN);
    L->sCnt = reinterpret_cast<int*>(pCnt);
    L->sCarryBin = reinterpret_cast<int*>(pCB);
    L->sKey = reinterpret_cast<uint8_t*>(pKey);
  }
  return off;
}

// Exclusive scan of cnt[0..m) in place by one warp.
__device__ __forceinline__ void warp_exclusive_scan(int* cnt, int m, int lane) {
  const int per = (m + 31) / 32;
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

// Raw gradient chunk of VEC elements of GT (kept packed until use).
template <typename GT, int VEC> struct GRaw {
  static constexpr int kWords = (int)(sizeof(GT) * VEC + 3) / 4;
  unsigned w[kWords];
};

template <typename GT, int VEC>
__device__ __forceinline__ void ldg_raw(GRaw<GT, VEC>& r, const GT* p) {
  constexpr int bytes = (int)sizeof(GT) * VEC;
  if constexpr (bytes == 32) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    r.w[0] = a.x; r.w[1] = a.y; r.w[2] = a.z; r.w[3] = a.w;
    r.w[4] = b.x; r.w[5] = b.y; r.w[6] = b.z; r.w[7] = b.w;
  } else if constexpr (bytes == 16) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    r.w[0] = a.x; r.w[1] = a.y; r.w[2] = a.z; r.w[3] = a.w;
  } else if constexpr (bytes == 8) {
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(p));
    r.w[0] = a.x; r.w[1] = a.y;
  } else if constexpr (bytes == 4) {
    r.w[0] = __ldg(reinterpret_cast<const unsigned*>(p));
  } else {
    r.w[0] = (unsigned)__ldg(reinterpret_cast<const unsigned short*>(p));
  }
}

// Elements e, e+1 (e even) of a raw chunk as fp32.
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
// q(p) > 0 exactly when p > threshold (ties round to the even zero).
template <typename QT> __device__ __forceinline__ float zero_round_threshold() {
  if constexpr (std::is_same<QT, float>::value) return 0.0f;
  else if constexpr (std::is_same<QT, __nv_bfloat16>::value) return __uint_as_float(0x00008000u);  // 2^-134
  else return 2.98023223876953125e-08f;                                                           // 2^-25
}

// gradient rows gathered ahead per lane group: 4 for chunks up to 16 bytes, 2 for 32-byte chunks
template <typename GT, int VEC> constexpr int walk_unroll() { return sizeof(GT) * VEC >= 32 ? 2 : (sizeof(GT) * VEC >= 16 && VEC >= 8 ? 2 : 4); }

// VEC fp32 values of one D-row chunk held as packed pairs (VEC >= 2) or a
// scalar (VEC == 1), so the walk's arithmetic maps onto fp32x2 instructions.
template <int VEC> struct Row {
  static constexpr int NP = VEC >= 2 ? VEC / 2 : 1;
  f2_t p[NP];  // VEC == 1 uses the low half of p[0]
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int e = 0; e < NP; ++e) p[e] = 0ull;
  }
  __device__ __forceinline__ void lds(const float* src) {
    if constexpr (VEC >= 4) {
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
    if constexpr (VEC >= 4) {
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
    if constexpr (VEC >= 4) {
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

// Add a run's sums into the shared histogram (H, U) or, for the first run of
// the segment (which may have started in the previous segment), into the
// segment's carry slot.
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

// One lane group's walk over its segment of a feature's bin-sorted samples.
template <typename QT, typename GT, int VEC, int EPI, bool RELU>
__device__ __forceinline__ void walk_segment(
    const BwdLayout& L, const float2* ents, const unsigned* metas, int my_len, int trips, const GT* grow,
    int64_t gstride, int my_i, int lgFc, int D, int cd, int c, int nc, float* carry, int* carry_bin, float* gx_row,
    bool do_gx, const Row<VEC>& pw0, const Row<VEC>& pbias, Row<VEC>& acc_w0, Row<VEC>& acc_b0) {
  constexpr int NP = Row<VEC>::NP;
  int k_cur = -1;
  bool first_run = true;
  float r_k = 0.f, r_km1 = 0.f;
  Row<VEC> Tk, Sk, Skm1, Hrun, Urun;
  Tk.zero(); Sk.zero(); Skm1.zero(); Hrun.zero(); Urun.zero();
  const float thr = zero_round_threshold<QT>();
  const int kstride = D << lgFc;
  float* hbase = L.sH + my_i * D + cd;
  float* ubase = L.sU + my_i * D + cd;

  constexpr int kWalkUnroll = walk_unroll<GT, VEC>();
  for (int base = 0; base < trips; base += kWalkUnroll) {
    float2 ent[kWalkUnroll];
    unsigned meta[kWalkUnroll];
    GRaw<GT, VEC> graw[kWalkUnroll];
#pragma unroll
    for (int u = 0; u < kWalkUnroll; ++u) {
      const int step = base + u;
      meta[u] = 0xffffu << 16;  // bin sentinel for lanes past their segment
      if (step < my_len) {
        ent[u] = ents[step];
        meta[u] = metas[step];
        ldg_raw<GT, VEC>(graw[u], grow + (int64_t)(meta[u] & 0xffffu) * gstride);
      }
    }
#pragma unroll
    for (int u = 0; u < kWalkUnroll; ++u) {
      const bool live = base + u < my_len;
      const int k = (meta[u] >> 16) & 0x7fff;
      if (live && k != k_cur) {
        if (k_cur >= 0)
          flush_run<VEC>(Hrun, Urun, first_run, k_cur, carry, carry_bin, D, c, hbase + k_cur * kstride,
                         ubase + k_cur * kstride);
        k_cur = k;
        const int to = (k << lgFc) * D + my_i * D + cd;
        Tk.lds(L.sT + to);
        Sk.lds(L.sS + to);
        r_k = L.sR[(k << lgFc) + my_i];
        Hrun.zero();
        Urun.zero();
      }
      const bool tie = live && (meta[u] >> 31);
      float gx = 0.f;
      if (live) {
        const float xv = ent[u].x, tq = ent[u].y;
        if constexpr (VEC >= 2) {
          const f2_t t2 = pack2(tq, tq), x2 = pack2(xv, xv);
          f2_t d2 = 0ull, dw2 = 0ull;
          f2_t q[NP];
#pragma unroll
          for (int e = 0; e < NP; ++e) {
            float g0, g1;
            raw_pair<GT, VEC>(graw[u], 2 * e, g0, g1);
            float q0 = g0, q1 = g1;
            if constexpr (RELU) {
              float p0, p1;
              unpack2(fma2(t2, Sk.p[e], Tk.p[e]), p0, p1);
              if constexpr (EPI == kEpiA) {
                round2<QT>(p0, p1);
                float b0, b1;
                unpack2(pbias.p[e], b0, b1);
                p0 += b0;
                p1 += b1;
                q0 = p0 > 0.f ? g0 : 0.f;
                q1 = p1 > 0.f ? g1 : 0.f;
              } else {
                q0 = p0 > thr ? g0 : 0.f;
                q1 = p1 > thr ? g1 : 0.f;
              }
            }
            if constexpr (!std::is_same<GT, QT>::value && !std::is_same<QT, float>::value) round2<QT>(q0, q1);
            q[e] = pack2(q0, q1);
            Hrun.p[e] = add2(Hrun.p[e], q[e]);
            Urun.p[e] = fma2(t2, q[e], Urun.p[e]);
            d2 = fma2(q[e], Sk.p[e], d2);
            if constexpr (EPI == kEpiB) {
              const f2_t gg = pack2(g0, g1);
              acc_w0.p[e] = fma2(gg, x2, acc_w0.p[e]);
              acc_b0.p[e] = add2(acc_b0.p[e], gg);
              dw2 = fma2(gg, pw0.p[e], dw2);
            }
          }
          float lo, hi;
          unpack2(d2, lo, hi);
          gx = r_k * (lo + hi);
          if constexpr (EPI == kEpiB) {
            unpack2(dw2, lo, hi);
            gx += lo + hi;
          }
          if (__any_sync(__activemask(), tie)) {  // edge sub-gradient (x == e_k), rare for continuous x
            const int km1 = k_cur > 0 ? k_cur - 1 : 0;
            Skm1.lds(L.sS + (km1 << lgFc) * D + my_i * D + cd);
            r_km1 = L.sR[(km1 << lgFc) + my_i];
            f2_t dp2 = 0ull;
#pragma unroll
            for (int e = 0; e < NP; ++e) dp2 = fma2(q[e], Skm1.p[e], dp2);
            unpack2(dp2, lo, hi);
            if (tie) gx += r_km1 * (lo + hi);
          }
        } else {
          const float g0 = raw_one<GT, VEC>(graw[u]);
          float q0 = g0;
          const float s0 = Sk.lo(0), t0v = Tk.lo(0);
          if constexpr (RELU) {
            float p0 = fmaf(tq, s0, t0v);
            if constexpr (EPI == kEpiA) {
              p0 = quantize<QT>(p0) + pbias.lo(0);
              q0 = p0 > 0.f ? g0 : 0.f;
            } else {
              q0 = p0 > thr ? g0 : 0.f;
            }
          }
          if constexpr (!std::is_same<GT, QT>::value) q0 = quantize<QT>(q0);
          Hrun.p[0] = (f2_t)__float_as_uint(Hrun.lo(0) + q0);
          Urun.p[0] = (f2_t)__float_as_uint(fmaf(tq, q0, Urun.lo(0)));
          gx = r_k * (q0 * s0);
          if (tie) {
            const int km1 = k_cur - 1;
            gx += L.sR[(km1 << lgFc) + my_i] * (q0 * L.sS[(km1 << lgFc) * D + my_i * D + cd]);
          }
          if constexpr (EPI == kEpiB) {
            acc_w0.p[0] = (f2_t)__float_as_uint(fmaf(g0, xv, acc_w0.lo(0)));
            acc_b0.p[0] = (f2_t)__float_as_uint(acc_b0.lo(0) + g0);
            gx += g0 * pw0.lo(0);
          }
        }
      }
      if (do_gx && live) gx_row[(meta[u] & 0xffffu) * nc] = gx;  // this lane's partial of the row
    }
  }
  if (my_len > 0 && k_cur >= 0)
    flush_run<VEC>(Hrun, Urun, first_run, k_cur, carry, carry_bin, D, c, hbase + k_cur * kstride,
                   ubase + k_cur * kstride);
}


template <typename QT, typename GT, int VEC, int EPI, bool RELU>
__global__ void __launch_bounds__(kBwdThreads, 1)
ple_bwd_kernel(const BwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lgFc = a.lgFc, lgWf = a.lgWf, lgSt = a.lgSt;
  const int Fc = 1 << lgFc, Wf = 1 << lgWf, S_t = 1 << lgSt;
  const int B = a.B, D = a.D, pow2 = a.pow2;
  const int nc = D / VEC;
  const int Rint = 32 / nc;
  const int G = Wf * Rint;
  BwdLayout L;
  bwd_layout_bytes(a, BwdDims{Fc, Wf, S_t, G, nc}, &L, smem_raw);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int my_i = wid >> lgWf;         // feature slot of this warp
  const int my_w = wid & (Wf - 1);      // warp rank within the feature
  const int r = lane / nc, c = lane - r * nc;
  const int g_seg = my_w * Rint + r;    // walk segment of this lane group
  const int cd = c * VEC;
  const bool do_gx = a.grad_x != nullptr;
  const GT* gptr = reinterpret_cast<const GT*>(a.g);
  const int lg_q = lgSt - lgWf;         // quarter length (log2)

  // this CTA's range of the flattened (chunk, sample) space
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
    const bool grp_live = r < Rint && my_i < fc;
    const bool x_vec4 = a.x_vec4 && fc == Fc;

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
    load_x(s_begin, (int)min64(S_t, s_end - s_begin), L.sXb);

    // ---- tables (as the forward) and zeroed H/U
    for (int i = tid; i < Fc; i += nthr) {
      int n = i < fc ? a.n_bins[f0 + i] : 1;
      L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
    }
    for (int idx = tid; idx < B * Fc * D; idx += nthr) {
      L.sH[idx] = 0.0f;
      L.sU[idx] = 0.0f;
      L.sS[idx] = 0.0f;
    }
    __syncthreads();
    for (int idx = tid; idx < pow2 * Fc; idx += nthr) {
      const int j = idx >> lgFc, i = idx & (Fc - 1);
      float e = __int_as_float(0x7f800000);
      if (i < fc && j <= L.sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j];
      L.sE[idx] = e;
    }
    for (int idx = tid; idx < B * Fc; idx += nthr) {
      const int j = idx >> lgFc, i = idx & (Fc - 1);
      L.sR[idx] = (i < fc && j < L.sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
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
    for (int col = tid; col < Fc * D; col += nthr) {
      const int i = col / D, d = col - i * D;
      const int n = L.sN[i];
      float acc = 0.0f;
      for (int j = 0; j < n; ++j) {
        const int o = ((j << lgFc) + i) * D + d;
        L.sT[o] = acc;
        acc += L.sS[o];
      }
    }

    // per-lane epilogue parameters and linear0 accumulators (packed pairs)
    Row<VEC> pw0, pbias, acc_w0, acc_b0;
    pw0.zero();
    pbias.zero();
    acc_w0.zero();
    acc_b0.zero();
    if (grp_live) {
      const int64_t po = (int64_t)(f0 + my_i) * D + cd;
      if constexpr (EPI == kEpiA && RELU) pbias.ldg(a.bias + po);
      if constexpr (EPI == kEpiB) pw0.ldg(a.w0 + po);
    }

    int buf = 0;
    for (int64_t t0 = s_begin; t0 < s_end; t0 += S_t, buf ^= 1) {
      const int ns = (int)min64(S_t, s_end - t0);
      const float* sX = L.sXb + buf * S_t * Fc;
      for (int idx = tid; idx < Fc * B * Wf; idx += nthr) L.sCnt[idx] = 0;
      cp_async_wait_all();
      __syncthreads();  // x tile landed, counts zeroed, previous tile finished
      if (t0 + S_t < s_end) load_x(t0 + S_t, (int)min64(S_t, s_end - t0 - S_t), L.sXb + (buf ^ 1) * S_t * Fc);
      // ---- A: bins and counts
      for (int p = tid; p < (ns << lgFc); p += nthr) {
        const int s = p >> lgFc, i = p & (Fc - 1);
        if (i < fc) {
          int k;
          if (a.bin_idx != nullptr) {
            const int64_t pair = (t0 + s) * a.F + f0 + i;
            k = a.bin_idx_bytes == 1 ? (int)reinterpret_cast<const uint8_t*>(a.bin_idx)[pair]
              : a.bin_idx_bytes == 2 ? (int)reinterpret_cast<const int16_t*>(a.bin_idx)[pair]
                                     : reinterpret_cast<const int32_t*>(a.bin_idx)[pair];
            k = k < 0 ? 0 : (k >= L.sN[i] ? L.sN[i] - 1 : k);
          } else {
            k = logical_bin(edge_count(sX[p], L.sE, Fc, i, pow2), L.sN[i]);
          }
          L.sKey[(i << lgSt) + s] = (uint8_t)k;
          atomicAdd(&L.sCnt[((i * B + k) << lgWf) + (s >> lg_q)], 1);
        }
      }
      __syncthreads();
      // ---- B: exclusive scan per feature (bin-major, quarter-minor)
      for (int i = wid; i < fc; i += nthr / 32) warp_exclusive_scan(L.sCnt + ((i * B) << lgWf), B << lgWf, lane);
      __syncthreads();
      // ---- C: stable scatter of each quarter into sorted order
      if (my_i < fc) {
        const int lo = my_w << lg_q, hi = min(lo + (1 << lg_q), ns);
        for (int base = lo; base < hi; base += 32) {
          const int s = base + lane;
          const bool v = s < hi;
          const unsigned act = __ballot_sync(0xffffffffu, v);
          if (v) {
            const int k = L.sKey[(my_i << lgSt) + s];
            const unsigned peers = __match_any_sync(act, k);
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
            const int pos = (my_i << lgSt) + pos0 + rank;
            L.sEnt[pos] = make_float2(xv, quantize<QT>(t));
            L.sMeta[pos] = (unsigned)s | ((unsigned)k << 16) | tie;
          }
          __syncwarp();
        }
      }
      __syncthreads();
      // ---- D: segmented walk
      if (my_i < fc) {
        const int seg_lo = (int)(((int64_t)g_seg * ns) / G);
        const int seg_hi = (int)(((int64_t)(g_seg + 1) * ns) / G);
        const int my_len = grp_live ? seg_hi - seg_lo : 0;
        int trips = my_len;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) trips = max(trips, __shfl_xor_sync(0xffffffffu, trips, off));
        float* carry = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        if (grp_live && c == 0) L.sCarryBin[my_i * G + g_seg] = -1;
        walk_segment<QT, GT, VEC, EPI, RELU>(
            L, L.sEnt + (my_i << lgSt) + seg_lo, L.sMeta + (my_i << lgSt) + seg_lo, my_len, trips,
            gptr + (t0 * a.F + f0 + my_i) * (int64_t)D + cd, (int64_t)a.F * D, my_i, lgFc, D, cd, c, nc,
            carry, L.sCarryBin + my_i * G + g_seg, L.sGX + (my_i << lgSt) * nc + c, do_gx, pw0, pbias, acc_w0,
            acc_b0);
      }
      __syncthreads();
      // ---- E: carries in segment order; grad_x rows
      for (int colx = tid; colx < fc * D; colx += nthr) {
        const int i = colx / D, d = colx - i * D;
        for (int g = 0; g < G; ++g) {
          const int kb = L.sCarryBin[i * G + g];
          if (kb >= 0) {
            const float* cp = L.sCarry + ((i * G + g) * 2) * D + d;
            L.sH[((kb << lgFc) + i) * D + d] += cp[0];
            L.sU[((kb << lgFc) + i) * D + d] += cp[D];
          }
        }
      }
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

    // ---- F: linear0 partials (fixed segment order) and grad_W suffix scan
    __syncthreads();
    float* ws = a.ws + ((int64_t)blockIdx.x * a.max_segs + seg) * ((int64_t)Fc * (B + 3) * D);
    if constexpr (EPI == kEpiB) {
      if (grp_live) {
        float* cp = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
        acc_w0.sts(cp);
        acc_b0.sts(cp + D);
      }
      __syncthreads();
      for (int colx = tid; colx < fc * D; colx += nthr) {
        const int i = colx / D, d = colx - i * D;
        float sw = 0.f, sb = 0.f;
        for (int g = 0; g < G; ++g) {
          const float* cp = L.sCarry + ((i * G + g) * 2) * D + d;
          sw += cp[0];
          sb += cp[D];
        }
        float* row = ws + (int64_t)i * (B + 3) * D;
        row[(B + 1) * D + d] = sw;
        row[(B + 2) * D + d] = sb;
      }
    }
    for (int colx = tid; colx < fc * D; colx += nthr) {
      const int i = colx / D, d = colx - i * D;
      const int n = L.sN[i];
      float* row = ws + (int64_t)i * (B + 3) * D;
      float suffix = 0.f;
      for (int j = n - 1; j >= 0; --j) {
        const int o = ((j << lgFc) + i) * D + d;
        row[physical_bin(j, n, B) * D + d] = L.sU[o] + suffix;
        suffix += L.sH[o];
      }
      for (int p = n - 1; p < B - 1; ++p) row[p * D + d] = 0.f;  // padding rows
      row[B * D + d] = suffix;                                    // sum_b g' (bias grad)
    }
  }
}

// Sum, per feature, the partials of the CTAs whose ranges cover its chunk, in
// CTA order (deterministic).
__global__ void ple_bwd_finalize_kernel(const BwdArgs a, int grid) {
  const int B = a.B, D = a.D, lgFc = a.lgFc, Fc = 1 << lgFc;
  const int64_t rows = (int64_t)a.F * (B + 3) * D;
  const int64_t total = (int64_t)a.n_chunks * a.N;
  const int64_t slot = (int64_t)Fc * (B + 3) * D;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = idx / ((int64_t)(B + 3) * D);
    const int64_t rem = idx - f * (B + 3) * D;
    const int chunk = (int)(f >> lgFc), i = (int)(f & (Fc - 1));
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
    const int row = (int)(rem / D), d = (int)(rem - (int64_t)row * D);
    if (row < B) {
      if (a.grad_W) a.grad_W[(f * B + row) * D + d] = s;
    } else if (row == B) {
      if (a.grad_bias) a.grad_bias[f * D + d] = s;
    } else if (row == B + 1) {
      if (a.grad_w0) a.grad_w0[f * D + d] = s;
    } else {
      if (a.grad_b0) a.grad_b0[f * D + d] = s;
    }
  }
}

// ------------------------------------------------------------------ planning
// Chunk width of the walk: 8 elements for 16-bit gradients (16-byte rows),
// 4 for fp32 unless D is large (a row group must fit in a warp).
int backward_vec(int64_t D, int gbytes) {
  int v = D % 8 == 0 ? 8 : (D % 4 == 0 ? 4 : (D % 2 == 0 ? 2 : 1));
  if (gbytes == 4 && v == 8 && D <= 32) v = 4;
  return v;
}

// Features per CTA (power of two), tile length and the layout size; false if
// even one feature does not fit.
static bool bwd_plan(BwdArgs& a, int vec, size_t* smem_out) {
  const int nc = a.D / vec;
  if (nc > 32) return false;
  int pow2 = 1;
  while (pow2 < a.B + 1) pow2 <<= 1;
  a.pow2 = pow2;
  const size_t optin = device_max_smem_optin();
  for (int lgFc = 2; lgFc >= 0; --lgFc) {
    if (lgFc > 0 && (1 << (lgFc - 1)) >= a.F) continue;
    const int Fc = 1 << lgFc;
    const int lgWf = 4 - lgFc;  // 16 warps
    const int G = (1 << lgWf) * (32 / nc);
    for (int lgSt = 10; lgSt >= 7; --lgSt) {
      BwdDims m{Fc, 1 << lgWf, 1 << lgSt, G, nc};
      const size_t bytes = bwd_layout_bytes(a, m, nullptr, nullptr);
      if (bytes <= optin) {
        a.lgFc = lgFc;
        a.lgWf = lgWf;
        a.lgSt = lgSt;
        a.n_chunks = (int)ceil_div<int64_t>(a.F, Fc);
        *smem_out = bytes;
        return true;
      }
    }
  }
  return false;
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

size_t backward_workspace_bytes(int64_t N, int64_t F, int64_t B, int64_t D) {
  size_t best = 0;
  for (int gbytes : {2, 4}) {  // large enough for either gradient width
    BwdArgs b{};
    b.N = N; b.F = (int)F; b.B = (int)B; b.D = (int)D;
    size_t smem = 0;
    if (!bwd_plan(b, backward_vec(D, gbytes), &smem)) continue;
    int grid = 0;
    bwd_grid(b, &grid);
    const size_t bytes = (size_t)grid * b.max_segs * ((size_t)(1 << b.lgFc) * (B + 3) * D) * sizeof(float);
    if (bytes > best) best = bytes;
  }
  return best;
}

template <typename QT, typename GT, int VEC, int EPI, bool RELU>
static int launch_bwd_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  if (!bwd_plan(a, VEC, &smem))
    return set_error(PLE_ERR_UNSUPPORTED, "backward: tables do not fit in shared memory");
  int grid = 0;
  bwd_grid(a, &grid);
  const size_t need = (size_t)grid * a.max_segs * ((size_t)(1 << a.lgFc) * (a.B + 3) * a.D) * sizeof(float);
  if (need > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  a.x_vec4 = ((1 << a.lgFc) >= 4) && (a.F % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  auto kern = ple_bwd_kernel<QT, GT, VEC, EPI, RELU>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  kern<<<grid, kBwdThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward launch");
  const int64_t rows = (int64_t)a.F * (a.B + 3) * a.D;
  const int fin_blocks = (int)min64(ceil_div<int64_t>(rows, 256), 4L * device_sm_count());
  ple_bwd_finalize_kernel<<<fin_blocks, 256, 0, st>>>(a, grid);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward finalize launch");
  return PLE_OK;
}

template <typename QT, typename GT, int VEC>
static int launch_bwd_epi(const BwdArgs& a, cudaStream_t st) {
  if (a.epi == kEpiB)
    return a.relu ? launch_bwd_t<QT, GT, VEC, kEpiB, true>(a, st) : launch_bwd_t<QT, GT, VEC, kEpiB, false>(a, st);
  if (a.epi == kEpiA)
    return a.relu ? launch_bwd_t<QT, GT, VEC, kEpiA, true>(a, st) : launch_bwd_t<QT, GT, VEC, kEpiA, false>(a, st);
  return launch_bwd_t<QT, GT, VEC, kEpiNone, false>(a, st);
}

template <typename QT, typename GT>
static int launch_bwd_vec(const BwdArgs& a, int vec, cudaStream_t st) {
  switch (vec) {
    case 8: return launch_bwd_epi<QT, GT, 8>(a, st);
    case 4: return launch_bwd_epi<QT, GT, 4>(a, st);
    case 2: return launch_bwd_epi<QT, GT, 2>(a, st);
    default: return launch_bwd_epi<QT, GT, 1>(a, st);
  }
}

int launch_backward(BwdArgs a, int compute_dtype, int grad_dtype, int vec, cudaStream_t st) {
  (void)vec;
  const int q = compute_dtype, g = grad_dtype;
  const int v = backward_vec(a.D, g == PLE_DTYPE_F32 ? 4 : 2);
  if (a.epi == kEpiNone) a.relu = 0;
  if (q == PLE_DTYPE_F32 && g == PLE_DTYPE_F32) return launch_bwd_vec<float, float>(a, v, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_BF16) return launch_bwd_vec<__nv_bfloat16, __nv_bfloat16>(a, v, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_F32) return launch_bwd_vec<__nv_bfloat16, float>(a, v, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F16) return launch_bwd_vec<__half, __half>(a, v, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F32) return launch_bwd_vec<__half, float>(a, v, st);
  return set_error(PLE_ERR_UNSUPPORTED, "backward: unsupported (compute, grad) dtype pair");
}

}  // namespace ple
