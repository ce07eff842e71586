// ple_backward_hist.cuh - the histogram form of the fused PLE backward: samples
// in natural order, per-warp private bin sums in shared memory, no sort.
//
// Same gradients as the sorted kernel (ple_backward_impl.cuh; reference
// backward_cuda.cu:343-492 for grad_x, :268-336 for grad_W):
//   H[j] = sum_{b: k_b = j} q(g'_b),  U[j] = sum_{b: k_b = j} q(t_b) q(g'_b),
//   grad_W[phys(j)] = U[j] + sum_{j' > j} H[j'],
//   grad_x = <q(g'), Q[k]> (+ <q(g'), Q[k - 1]> at an interior edge tie)
//            (+ <g, w0> for epilogue B),  Q[k] = r_k S[k].
//
// Work decomposition.  One persistent CTA of 16 warps per SM; chunks of Fc
// features, slots of `group` CTAs over the same sample ranges and the
// workspace blocks are those of the sorted kernel (the finalize is shared).
// A chunk's warps split evenly over its features (Wf = 16 / Fc per feature).
// Each warp owns a private copy of its feature's H / U sums ([B][4][2 VEC]
// floats: lane chunk c of bin k holds H[c VEC ..] then U[c VEC ..]), so no
// two warps ever write the same word.  Per tile of S_t samples (x arrives by
// cp.async one tile ahead, the next tile's gradient rows are prefetched into
// L2 by one tensor-map instruction per 256 rows) each warp takes batches of
// 32 samples of its feature, interleaved with the feature's other warps:
//   * search: one sample per lane (the forward's bin indices when given,
//     else an L-level descent over the interior edges in breadth-first
//     order), q(t), the tie flag;
//   * 4 steps of 8 samples, 4 lanes x VEC elements per D row: the gradient
//     chunk (loaded one batch ahead), the ReLU mask (skipped, bit-identically,
//     when every sample of the step is in an "open" bin, one whose ReLU input
//     is positive for every t the bin admits), grad_x shares (summed over the
//     row's 4 lanes by shuffles), the epilogue sums, then H += q(g'),
//     U += q(t) q(g') into the warp's copy.  Samples of one step that share a
//     bin (found by match.any) update it in rounds, in sample order.  Lanes
//     of odd samples read and write the U half of a chunk before the H half,
//     so the two samples of a quarter-warp never meet in a bank.
// At the end of a segment the Wf copies of a feature are summed in warp order,
// a suffix scan over bins turns H / U into grad_W and the partial goes to the
// workspace.  No floating-point atomics: bitwise deterministic for a given
// shape and device.
#pragma once

#include "ple_backward_impl.cuh"

namespace ple {

constexpr int kHistNC = 4;  // lanes per D row: 8 samples per warp step, 4 steps per batch of 32

struct HistLayout {
  float* sAcc;      // [16 warps][B][kHistNC][2 VEC] private H / U sums
  float* sQ;        // [Fc][B][2][D] Q = r_k S_k, twice per bin (odd samples read the second copy)
  float* sS;        // [Fc][B][D] S = q(W) in logical bin order (masked path)
  float* sT;        // [Fc][B][D] exclusive prefix of S (masked path)
  float* sX;        // [2][Fc][S_t] x tiles (transposed)
  float* sGX;       // [2][S_t][Fc] grad_x tiles
  float* sKey;      // [Fc][nkeys] interior edges in breadth-first order (node 1 = root)
  float2* sER;      // [Fc][B] {e_k, r_k}
  unsigned* sOpen;  // [Fc][ceil(B / 32)] open-bin bits
  float* sEpi;      // [Fc][Wf][2][D] per-warp epilogue sums
  int* sN;          // [Fc] real bins per feature
};

__host__ __device__ __forceinline__ size_t hist_layout_bytes(int B, int D, int Fc, int S_t, int nkeys, HistLayout* L,
                                                             unsigned char* base) {
  const int Wf = kBwdWarps / Fc;
  const int ow = (B + 31) / 32;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 15) & ~(size_t)15;
    return base + o;
  };
  unsigned char* pAcc = take((size_t)kBwdWarps * B * D * 2 * 4);
  unsigned char* pQ = take((size_t)Fc * B * 2 * D * 4);
  unsigned char* pS = take((size_t)Fc * B * D * 4);
  unsigned char* pT = take((size_t)Fc * B * D * 4);
  unsigned char* pX = take((size_t)2 * Fc * S_t * 4);
  unsigned char* pGX = take((size_t)2 * S_t * Fc * 4);
  unsigned char* pK = take((size_t)Fc * nkeys * 4);
  unsigned char* pER = take((size_t)Fc * B * 8);
  unsigned char* pO = take((size_t)Fc * ow * 4);
  unsigned char* pE = take((size_t)Fc * Wf * 2 * D * 4);
  unsigned char* pN = take((size_t)Fc * 4);
  if (L) {
    L->sAcc = reinterpret_cast<float*>(pAcc);
    L->sQ = reinterpret_cast<float*>(pQ);
    L->sS = reinterpret_cast<float*>(pS);
    L->sT = reinterpret_cast<float*>(pT);
    L->sX = reinterpret_cast<float*>(pX);
    L->sGX = reinterpret_cast<float*>(pGX);
    L->sKey = reinterpret_cast<float*>(pK);
    L->sER = reinterpret_cast<float2*>(pER);
    L->sOpen = reinterpret_cast<unsigned*>(pO);
    L->sEpi = reinterpret_cast<float*>(pE);
    L->sN = reinterpret_cast<int*>(pN);
  }
  return off;
}

// The chunk's tables for one segment and zeroed private sums: search keys, {e_k, r_k}, S = q(W) in
// logical bin order, its exclusive prefix T, Q = r S (twice per bin), the open bits.
template <typename QT, int MASK>
__device__ __forceinline__ void stage_hist_tables(const BwdArgs& a, const HistLayout& L, int f0, int fc, int Fc,
                                                  int D, int nkeys, int lgk, int tid, int nthr) {
  const int B = a.B;
  const int ow = (B + 31) / 32;
  for (int i = tid; i < Fc; i += nthr) {
    const int n = i < fc ? a.n_bins[f0 + i] : 1;
    L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  {
    float4* acc = reinterpret_cast<float4*>(L.sAcc);
    const int n4 = kBwdWarps * B * D * 2 / 4;
    for (int idx = tid; idx < n4; idx += nthr) acc[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int idx = tid; idx < Fc * B * D; idx += nthr) L.sS[idx] = 0.0f;
  }
  __syncthreads();
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
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int row = tid; row < fc * B; row += nthr) {
    const int i = row / B, p = row - i * B;
    const int n = L.sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) {
      const float* src = Wc + (int64_t)row * D;
      float* dst = L.sS + (i * B + lg) * D;
      for (int d = 0; d < D; ++d) dst[d] = quantize<QT>(src[d]);
    }
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = L.sN[i];
    float acc = 0.0f;
    for (int j = 0; j < B; ++j) {
      const int o = (i * B + j) * D + d;
      const float S = L.sS[o];
      L.sT[o] = j < n ? acc : 0.0f;
      acc += j < n ? S : 0.0f;
      const float q = S * L.sER[i * B + j].y;
      L.sQ[(2 * (i * B + j)) * D + d] = q;
      L.sQ[(2 * (i * B + j) + 1) * D + d] = q;
    }
  }
  __syncthreads();
  // open bits (see stage_tables in ple_backward_impl.cuh: the ReLU input is monotone in t, so a middle bin
  // is open when it passes at t = 0 and t = tmax; the last bin when S >= 0 and t = 0 passes; never bin 0,
  // never bins given by the caller); one ballot per 32 bins
  for (int idx = tid; idx < Fc * ow * 32; idx += nthr) {
    const int i = idx / (ow * 32), k = idx - i * (ow * 32);
    bool open = false;
    if constexpr (MASK != kMaskNone) {
      const int n = L.sN[i];
      if (a.bin_idx == nullptr && i < fc && k > 0 && k < n) {
        const float2 er = L.sER[i * B + k];
        const bool last = k == n - 1;
        const float tmax = last ? 0.0f : quantize<QT>((a.edges[(int64_t)(f0 + i) * (B + 1) + k + 1] - er.x) * er.y);
        open = true;
        for (int d = 0; d < D && open; ++d) {
          const float S = L.sS[(i * B + k) * D + d], T = L.sT[(i * B + k) * D + d];
          const float bias = MASK == kMaskReluBias ? a.bias[(int64_t)(f0 + i) * D + d] : 0.0f;
          const float p0 = fmaf(0.0f, S, T), p1 = fmaf(tmax, S, T);
          if (p0 != p0 || p1 != p1 || !relu_passes<QT, MASK>(p0, bias) || !relu_passes<QT, MASK>(p1, bias))
            open = false;
          if (last && !(S >= 0.0f)) open = false;
        }
      }
    }
    const unsigned word = __ballot_sync(0xffffffffu, open);
    if ((tid & 31) == 0) L.sOpen[idx >> 5] = word;
  }
  __syncthreads();
}

// Step word of a sample: bin in bits 0-7, then the flags; dead lanes (past the tile) carry their lane in
// bits 12-16 so that no two of them match.
constexpr int kTieBit = 1 << 8, kOpenBit = 1 << 9, kDeadBit = 1 << 10;

// Count of interior edges e_1 .. e_{2^L - 1} (breadth-first in keys[1 ..]) with !(x < e): the L-level
// descent, unrolled per level count.
template <int LGK> __device__ __forceinline__ int hist_search_l(const float* keys, float x) {
  int node = 1;
#pragma unroll
  for (int l = 0; l < LGK; ++l) node = 2 * node + (x < keys[node] ? 0 : 1);
  return node - (1 << LGK);
}
__device__ __forceinline__ int hist_search(const float* keys, float x, int lgk) {
  switch (lgk) {
    case 0: return hist_search_l<0>(keys, x);
    case 1: return hist_search_l<1>(keys, x);
    case 2: return hist_search_l<2>(keys, x);
    case 3: return hist_search_l<3>(keys, x);
    case 4: return hist_search_l<4>(keys, x);
    case 5: return hist_search_l<5>(keys, x);
    case 6: return hist_search_l<6>(keys, x);
    case 7: return hist_search_l<7>(keys, x);
    default: return hist_search_l<8>(keys, x);
  }
}

// One step of one lane: q(g') of its VEC elements (the ReLU mask on the EXACT path only: every sample
// of the step in an open bin makes it a no-op), the epilogue sums, and the lane's share of grad_x
// (<q(g'), Q[k]>, plus <g, w0> for epilogue B).  Same arithmetic as walk_step of the sorted kernel.
template <typename QT, typename GT, int VEC, int MASK, int EPIV, bool EXACT>
__device__ __forceinline__ float hist_body(const GRaw<GT, VEC>& g, float tv, float xv, const Row<VEC>& Qr,
                                           uint32_t st_addr, uint32_t tt_addr, const Row<VEC>& pbias,
                                           const Row<VEC>& w0r, Row<VEC>& aw, Row<VEC>& ab,
                                           f2_t (&qv)[Row<VEC>::NP]) {
  constexpr int NP = Row<VEC>::NP;
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ROUND_G = !std::is_same<GT, QT>::value && !std::is_same<QT, float>::value;
  constexpr bool WIDE = VEC % 4 == 0;
  const float thr = zero_round_threshold<QT>();
  const f2_t t2 = pack2(tv, tv);
  f2_t Sk[NP], Tk[NP];
  if constexpr (EXACT && MASK != kMaskNone) {
    lds_pairs<NP, WIDE>(Sk, st_addr);
    lds_pairs<NP, WIDE>(Tk, tt_addr);
  }
  f2_t d2 = 0ull, dw2 = 0ull;
  f2_t x2 = 0ull;
  if constexpr (LIN) x2 = pack2(xv, xv);
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    const f2_t g2 = raw_pair<GT, VEC>(g, e);
    if constexpr (LIN) {
      dw2 = fma2(g2, w0r.p[e], dw2);
      aw.p[e] = fma2(g2, x2, aw.p[e]);
      ab.p[e] = add2(ab.p[e], g2);
    }
    f2_t qq = g2;
    if constexpr (EXACT && MASK != kMaskNone) {
      float p0, p1, g0, g1;
      unpack2(fma2(t2, Sk[e], Tk[e]), p0, p1);
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
    qv[e] = qq;
    d2 = fma2(qq, Qr.p[e], d2);
  }
  float lo, hi;
  unpack2(d2, lo, hi);
  float gx = lo + hi;
  if constexpr (LIN) {
    unpack2(dw2, lo, hi);
    gx += lo + hi;
  }
  return gx;
}

template <typename QT, typename GT, int VEC, int MASK, int EPIV>
__global__ void __launch_bounds__(kBwdThreads, 1)
    ple_bwd_hist_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap gmap) {
  constexpr int NC = kHistNC, R = 32 / NC, J = NC;  // lanes per row, samples per step, steps per batch
  constexpr int D = NC * VEC;
  constexpr int CH = 2 * VEC;  // floats of one lane chunk of a bin row (H, then U)
  constexpr int NP = Row<VEC>::NP;
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ACC = EPIV != kEpvNone;
  constexpr bool WIDE = VEC % 4 == 0;
  constexpr uint32_t kRow = 2 * D * 4;  // bytes of a Q row and of a bin row of the sums
  static_assert(VEC >= 2 && VEC % 2 == 0, "the histogram kernel packs fp32 pairs");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int B = a.B;
  const int Fc = a.Fc, S_t = 1 << a.lgSt;
  const int Wf = kBwdWarps / Fc;
  const int nkeys = 1 << a.lgk;
  const int ow = (B + 31) / 32;
  const int BD2 = B * D * 2;
  HistLayout L;
  hist_layout_bytes(B, D, Fc, S_t, nkeys, &L, smem_raw);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int r = lane / NC, c = lane - r * NC, cd = c * VEC;
  const int par = r & 1;
  const int my_i = wid / Wf, my_w = wid - my_i * Wf;
  const unsigned cmask = 0x11111111u << c;  // lanes holding chunk c of their row (NC == 4)
  const unsigned lt = (1u << lane) - 1u;
  const int JB = S_t / (32 * Wf);  // batches per warp per tile (even: the host plans it so)
  const bool do_gx = a.grad_x != nullptr;
  const GT* gptr = reinterpret_cast<const GT*>(a.g);
  const uint64_t pol_first = l2_policy_evict_first();
  const uint64_t pol_last = l2_policy_evict_last();
  float* acc_w = L.sAcc + (size_t)wid * BD2 + c * CH;  // this lane's chunk column of the warp's copy

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
    const int f0 = chunk * Fc;
    const int fc = min(Fc, a.F - f0);
    const bool live_w = my_i < fc;
    const int n_tiles = (int)ceil_div<int64_t>(s_end - s_begin, S_t);

    auto load_x = [&](int T) {
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      float* dst = L.sX + (T & 1) * Fc * S_t;
      for (int q = tid; q < ns * Fc; q += nthr) {
        const int s = q / Fc, i = q - s * Fc;
        if (i < fc) cp_async4(dst + i * S_t + s, a.x + (t0 + s) * a.F + f0 + i);
        else dst[i * S_t + s] = 0.0f;
      }
      cp_async_commit();
    };
    auto prefetch_g = [&](int T) {
      if (!a.g_prefetch || tid != 0) return;
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      for (int r0 = 0; r0 < ns; r0 += 256) prefetch_tile_l2(&gmap, f0 * D, (int)(t0 + r0), pol_last);
    };
    auto store_gx = [&](int T) {
      if (!do_gx) return;
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      const float* src = L.sGX + (T & 1) * S_t * Fc;
      float* gdst = a.grad_x + t0 * a.F + f0;
      if (Fc == 4 && fc == 4 && a.gx_vec4) {
        for (int s = tid; s < ns; s += nthr)
          *reinterpret_cast<float4*>(gdst + (int64_t)s * a.F) = *reinterpret_cast<const float4*>(src + s * 4);
      } else {
        for (int p = tid; p < ns * Fc; p += nthr) {
          const int s = p / Fc, i = p - s * Fc;
          if (i < fc) gdst[(int64_t)s * a.F + i] = src[p];
        }
      }
    };

    __syncthreads();  // previous segment finished with every shared buffer
    load_x(0);
    prefetch_g(0);
    stage_hist_tables<QT, MASK>(a, L, f0, fc, Fc, D, nkeys, a.lgk, tid, nthr);

    Row<VEC> pbias, w0r, aw, ab;  // aw: sum g x (B) or sum g' (A); ab: sum g (B)
    pbias.zero();
    w0r.zero();
    aw.zero();
    ab.zero();
    if constexpr (MASK == kMaskReluBias) {
      if (live_w) pbias.ldg(a.bias + (int64_t)(f0 + my_i) * D + cd);
    }
    if constexpr (LIN) {
      if (live_w) w0r.ldg(a.w0 + (int64_t)(f0 + my_i) * D + cd);
    }
    const float* keys = L.sKey + my_i * nkeys;
    const float2* er = L.sER + my_i * B;
    const unsigned* openw = L.sOpen + my_i * ow;
    const int n1 = L.sN[my_i] - 1;
    // lane-constant shared-memory bases; a bin adds kofs bytes (Q and H / U rows are both 2 D floats)
    const uint32_t qb = shared_addr(L.sQ + (my_i * B * 2 + par) * D + cd);
    const uint32_t sb = shared_addr(L.sS + my_i * B * D + cd);
    const uint32_t tb = shared_addr(L.sT + my_i * B * D + cd);
    const uint32_t aA = shared_addr(acc_w + par * VEC);        // first half this lane touches
    const uint32_t aB = shared_addr(acc_w + (par ^ 1) * VEC);  // second half
    // this lane's gradient row of step 0 of the warp's first batch; batches advance by 32 Wf samples
    const int64_t FD = (int64_t)a.F * D;
    const GT* gp = gptr + (s_begin + 32 * my_w + r) * FD + (int64_t)(f0 + my_i) * D + cd;
    int64_t srem = s_end - (s_begin + 32 * my_w + r);  // step j of the next batch to load is live iff j R < srem
    const int64_t gstep = (int64_t)R * FD, gbatch = (int64_t)32 * Wf * FD;
    const bool wide = a.g_wide != 0;

    auto load_batch = [&](GRaw<GT, VEC> (&g)[J]) {
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (live_w && j * R < srem) {
          ldg_raw<GT, VEC>(g[j], gp + j * gstep, wide, pol_first);
        } else {
#pragma unroll
          for (int w = 0; w < GRaw<GT, VEC>::kWords; ++w) g[j].w[w] = 0u;
        }
      }
      gp += gbatch;
      srem -= 32 * Wf;
    };

    // batch jb of tile T (samples sb0 .. sb0 + 31 of the tile).  The 4 steps go phase by phase (their
    // parameters and Q rows, their arithmetic, their grad_x, their duplicate masks, and last the ordered
    // read-modify-writes of the sums), so that the independent work of the steps overlaps.
    auto run_batch = [&](const GRaw<GT, VEC> (&g)[J], int T, int jb) {
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      const int sb0 = 32 * (my_w + Wf * jb);
      const float* xs = L.sX + (T & 1) * Fc * S_t + my_i * S_t;
      const uint32_t gxa = shared_addr(L.sGX + (T & 1) * S_t * Fc + (sb0 + r) * Fc + my_i);  // + j R Fc floats
      // ---- search: one sample per lane; the step word packs bin (bits 0-7), tie, open, dead (+ lane)
      const int s_l = sb0 + lane;
      const bool v = live_w && s_l < ns;
      const float x = v ? xs[s_l] : 0.0f;
      int k = 0;
      if (v) {
        if (a.bin_idx != nullptr) {
          const int64_t pair = (t0 + s_l) * a.F + f0 + my_i;
          k = a.bin_idx_bytes == 1 ? (int)reinterpret_cast<const uint8_t*>(a.bin_idx)[pair]
            : a.bin_idx_bytes == 2 ? (int)reinterpret_cast<const int16_t*>(a.bin_idx)[pair]
                                   : reinterpret_cast<const int32_t*>(a.bin_idx)[pair];
          k = k < 0 ? 0 : (k > n1 ? n1 : k);
        } else {
          k = min(hist_search(keys, x, a.lgk), n1);
        }
      }
      const float2 e = er[k];
      const float t = quantize<QT>((x - e.x) * e.y);
      const bool tie = v && k > 0 && x == e.x;
      const bool open = ((openw[k >> 5] >> (k & 31)) & 1u) != 0u;
      const int kk = v ? (k | (tie ? kTieBit : 0) | (open ? kOpenBit : 0)) : (kDeadBit | kOpenBit | (lane << 12));
      const bool any_tie = __any_sync(0xffffffffu, tie);
      // ---- phase 1: the steps' words, t, x and Q rows
      int kv[J];
      float tv[J], xv[J];
      Row<VEC> Qr[J];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int sj = j * R + r;
        kv[j] = __shfl_sync(0xffffffffu, kk, sj);
        tv[j] = __shfl_sync(0xffffffffu, t, sj);
        xv[j] = LIN ? __shfl_sync(0xffffffffu, x, sj) : 0.0f;
        lds_pairs<NP, WIDE>(Qr[j].p, qb + (uint32_t)(kv[j] & 0xff) * kRow);
      }
      // ---- phase 2: q(g'), the epilogue sums and the grad_x shares
      f2_t qv[J][NP];
      float gx[J];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        bool exact = false;
        if constexpr (MASK != kMaskNone) exact = !__all_sync(0xffffffffu, (kv[j] & kOpenBit) != 0);
        const uint32_t ho = (uint32_t)(kv[j] & 0xff) * (kRow / 2);
        gx[j] = exact ? hist_body<QT, GT, VEC, MASK, EPIV, true>(g[j], tv[j], xv[j], Qr[j], sb + ho, tb + ho, pbias,
                                                                 w0r, aw, ab, qv[j])
                      : hist_body<QT, GT, VEC, MASK, EPIV, false>(g[j], tv[j], xv[j], Qr[j], 0u, 0u, pbias, w0r,
                                                                  aw, ab, qv[j]);
      }
      // ---- phase 3: grad_x of the samples (edge sub-gradient where x == e_k, k > 0), the row's 4 lane
      // shares summed by shuffles
      if (do_gx) {
        if (any_tie) {
#pragma unroll
          for (int j = 0; j < J; ++j) {
            const bool tj = (kv[j] & kTieBit) != 0;
            if (__any_sync(0xffffffffu, tj)) {
              const uint32_t kofs = (uint32_t)(kv[j] & 0xff) * kRow;
              f2_t Qm[NP];
              lds_pairs<NP, WIDE>(Qm, qb + (kofs != 0u ? kofs - kRow : 0u));
              f2_t dp2 = 0ull;
#pragma unroll
              for (int e2 = 0; e2 < NP; ++e2) dp2 = fma2(qv[j][e2], Qm[e2], dp2);
              float lo, hi;
              unpack2(dp2, lo, hi);
              if (tj) gx[j] += lo + hi;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < J; ++j) gx[j] += __shfl_xor_sync(0xffffffffu, gx[j], 1);
#pragma unroll
        for (int j = 0; j < J; ++j) gx[j] += __shfl_xor_sync(0xffffffffu, gx[j], 2);
#pragma unroll
        for (int j = 0; j < J; ++j)
          if ((kv[j] & kDeadBit) == 0 && c == 0) sts_f32(gxa + j * R * Fc * 4, gx[j]);
      }
      // ---- phase 4: samples of a step that share a bin
      unsigned dup[J];
      bool any_dup = false;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        dup[j] = __match_any_sync(0xffffffffu, kv[j] & ~kTieBit) & cmask & lt;
        any_dup |= dup[j] != 0u;
      }
      any_dup = __any_sync(0xffffffffu, any_dup);
      // ---- phase 5: H += q(g'), U += q(t) q(g') into the warp's copy, step by step
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const bool live = (kv[j] & kDeadBit) == 0;
        const uint32_t kofs = (uint32_t)(kv[j] & 0xff) * kRow;
        const float ta = par ? tv[j] : 1.0f, tb2 = par ? 1.0f : tv[j];
        const f2_t wa = pack2(ta, ta), wb = pack2(tb2, tb2);
        const uint32_t pa = aA + kofs, pb = aB + kofs;
        auto rmw = [&]() {
          f2_t A[NP], Bh[NP];
          lds_pairs_ordered<NP, WIDE>(A, pa);
          lds_pairs_ordered<NP, WIDE>(Bh, pb);
#pragma unroll
          for (int e2 = 0; e2 < NP; ++e2) {
            A[e2] = fma2(wa, qv[j][e2], A[e2]);
            Bh[e2] = fma2(wb, qv[j][e2], Bh[e2]);
          }
          sts_pairs_ordered<NP, WIDE>(pa, A);
          sts_pairs_ordered<NP, WIDE>(pb, Bh);
        };
        if (!any_dup || !__any_sync(0xffffffffu, dup[j] != 0u)) {
          if (live) rmw();
        } else {
          const int rank = __popc(dup[j]);
          for (int rd = 0;; ++rd) {
            if (live && rank == rd) rmw();
            if (!__any_sync(0xffffffffu, rank > rd)) break;
            __syncwarp();
          }
        }
      }
    };

    // tiles of S_t samples, JB (even) batches per warp per tile; gradient rows one batch ahead
    GRaw<GT, VEC> gA[J], gB[J];
    load_batch(gA);
#pragma unroll 1
    for (int T = 0; T < n_tiles; ++T) {
      cp_async_wait_all();
      __syncthreads();  // x of tile T landed; every warp finished tile T - 1
      if (T > 0) store_gx(T - 1);
      if (T + 1 < n_tiles) {
        load_x(T + 1);
        prefetch_g(T + 1);
      }
#pragma unroll 1
      for (int jb = 0; jb < JB; jb += 2) {
        load_batch(gB);
        run_batch(gA, T, jb);
        load_batch(gA);
        run_batch(gB, T, jb + 1);
      }
    }
    __syncthreads();  // every warp's sums and grad_x shares are in shared memory
    store_gx(n_tiles - 1);

    // ---- epilogue sums: over the warp's 8 sample rows in row order, then the warps of a feature in order
    if constexpr (ACC) {
      Row<VEC> sw = aw, sb = ab;
#pragma unroll
      for (int r2 = 1; r2 < R; ++r2) {
#pragma unroll
        for (int e2 = 0; e2 < NP; ++e2) {
          uint32_t lo, hi;
          bits2(aw.p[e2], lo, hi);
          const f2_t ow2 = from_bits2(__shfl_sync(0xffffffffu, lo, r2 * NC + c), __shfl_sync(0xffffffffu, hi, r2 * NC + c));
          sw.p[e2] = add2(sw.p[e2], ow2);
          if constexpr (LIN) {
            bits2(ab.p[e2], lo, hi);
            const f2_t ob2 = from_bits2(__shfl_sync(0xffffffffu, lo, r2 * NC + c), __shfl_sync(0xffffffffu, hi, r2 * NC + c));
            sb.p[e2] = add2(sb.p[e2], ob2);
          }
        }
      }
      if (live_w && r == 0) {
        float* ep = L.sEpi + ((my_i * Wf + my_w) * 2) * D + cd;
        sw.sts(ep);
        if constexpr (LIN) sb.sts(ep + D);
      }
    }
    // ---- the Wf copies of each feature summed in warp order into the first
    for (int o = tid; o < fc * (BD2 / 4); o += nthr) {
      const int i = o / (BD2 / 4), off = o - i * (BD2 / 4);
      float4* base = reinterpret_cast<float4*>(L.sAcc + (size_t)i * Wf * BD2) + off;
      float4 s = base[0];
      for (int w = 1; w < Wf; ++w) {
        const float4 v4 = base[(size_t)w * (BD2 / 4)];
        s.x += v4.x;
        s.y += v4.y;
        s.z += v4.z;
        s.w += v4.w;
      }
      base[0] = s;
    }
    __syncthreads();
    // ---- partial of this segment: epilogue rows and the grad_W suffix scan
    float* ws = a.ws + (((int64_t)slot * a.max_segs + seg) * m + member) * ((int64_t)Fc * (B + 3) * D);
    for (int col = tid; col < fc * D; col += nthr) {
      const int i = col / D, d = col - i * D;
      const int n = L.sN[i];
      const int cc = d / VEC, e = d - cc * VEC;
      const float* h = L.sAcc + (size_t)i * Wf * BD2 + cc * CH + e;
      float* row = ws + (int64_t)i * (B + 3) * D;
      if constexpr (ACC) {
        float s0 = 0.f, s1 = 0.f;
        for (int w = 0; w < Wf; ++w) {
          const float* ep = L.sEpi + ((i * Wf + w) * 2) * D + d;
          s0 += ep[0];
          if constexpr (LIN) s1 += ep[D];
        }
        if constexpr (LIN) {
          row[(B + 1) * D + d] = s0;
          row[(B + 2) * D + d] = s1;
        } else {
          row[B * D + d] = s0;
        }
      }
      float suffix = 0.f;
      for (int j = n - 1; j >= 0; --j) {
        const float* hj = h + j * (NC * CH);
        row[physical_bin(j, n, B) * D + d] = hj[VEC] + suffix;
        suffix += hj[0];
      }
      for (int p = n - 1; p < B - 1; ++p) row[p * D + d] = 0.f;  // padding rows
      if (EPIV != kEpvBias) row[B * D + d] = suffix;
    }
  }
}

// Host: plan (ple_backward.cu) and launch.
int hist_prepare(BwdArgs& a, size_t* smem, int* grid);

template <typename QT, typename GT, int VEC, int MASK, int EPIV>
int launch_hist_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  int grid = 0;
  const int prep = hist_prepare(a, &smem, &grid);
  if (prep != PLE_OK) return prep;
  a.g_wide = (GRaw<GT, VEC>::kBytes == 32) && a.g_wide;
  CUtensorMap map;
  a.g_prefetch = bwd_grad_map(a, std::is_same<GT, float>::value ? 0 : std::is_same<GT, __nv_bfloat16>::value ? 2 : 1,
                              &map) ? 1 : 0;
  auto kern = ple_bwd_hist_kernel<QT, GT, VEC, MASK, EPIV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  kern<<<grid, kBwdThreads, smem, st>>>(a, map);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward launch");
  return bwd_finalize(a, grid, st);
}

// Mask variant and epilogue terms (as launch_bwd_mask of the sorted kernel).
template <typename QT, typename GT, int VEC>
int launch_hist_mask(const BwdArgs& a, cudaStream_t st) {
  const bool lin = a.epi == kEpiB && (a.grad_x || a.grad_w0 || a.grad_b0);
  const bool bias = a.epi == kEpiA && a.grad_bias;
  if (a.relu && a.epi == kEpiA)
    return bias ? launch_hist_t<QT, GT, VEC, kMaskReluBias, kEpvBias>(a, st)
                : launch_hist_t<QT, GT, VEC, kMaskReluBias, kEpvNone>(a, st);
  if (a.relu)
    return lin ? launch_hist_t<QT, GT, VEC, kMaskRelu, kEpvLin>(a, st) : launch_hist_t<QT, GT, VEC, kMaskRelu, kEpvNone>(a, st);
  if (lin) return launch_hist_t<QT, GT, VEC, kMaskNone, kEpvLin>(a, st);
  return bias ? launch_hist_t<QT, GT, VEC, kMaskNone, kEpvBias>(a, st) : launch_hist_t<QT, GT, VEC, kMaskNone, kEpvNone>(a, st);
}

// True when the histogram kernel serves a backward of this shape (ple_backward.cu).
bool backward_uses_hist(int64_t F, int64_t B, int64_t D);

// The backward of one dtype pair: the histogram kernel where it applies (D = 8, 16 or 24, at most 256 bins,
// tables that fit), else the sorted kernel with `vec` elements per lane.
template <typename QT, typename GT>
int launch_backward_dtype(const BwdArgs& a, int vec, cudaStream_t st) {
  if (backward_uses_hist(a.F, a.B, a.D)) {
    switch (a.D) {
      case 8: return launch_hist_mask<QT, GT, 2>(a, st);
      case 16: return launch_hist_mask<QT, GT, 4>(a, st);
      case 24: return launch_hist_mask<QT, GT, 6>(a, st);
      default: break;
    }
  }
  return launch_bwd_dtype<QT, GT>(a, vec, st);
}

}  // namespace ple
