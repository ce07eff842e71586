// ple_backward_hist.cuh - the histogram form of the fused PLE backward: samples
// in natural order, per-warp private bin sums in shared memory, no sort.
//
// Same gradients as the sorted kernel (ple_backward_impl.cuh; reference
// backward_cuda.cu:343-492 for grad_x, :268-336 for grad_W):
//   H[j] = sum_{b: k_b = j} q(g'_b),  U[j] = sum_{b: k_b = j} q(t_b) q(g'_b),
//   grad_W[phys(j)] = U[j] + sum_{j' > j} H[j'],
//   grad_x = r_k <q(g'), S[k]> (+ r_{k-1} <q(g'), S[k - 1]> at an interior edge tie)
//            (+ <g, w0> for epilogue B).
//
// Work decomposition.  One persistent CTA of 16 warps per SM; chunks of Fc
// features, slots of `group` CTAs over the same sample ranges and the
// workspace blocks are those of the sorted kernel (the finalize is shared).
// A chunk's warps split evenly over its features (Wf = 16 / Fc per feature)
// and each warp owns a private copy of its feature's H / U sums, so no two
// warps ever write the same word.  A D row is 4 lanes x VEC elements (D = 8,
// 16: a warp step is 8 samples) or, for D = 24, 8 lane slots of which 6 hold
// 4 elements each (a warp step is 4 samples).  Per tile of S_t samples (x arrives by cp.async
// one tile ahead, the next tile's gradient rows are prefetched into L2 by one
// tensor-map instruction per 256 rows) each warp takes batches of 32 samples
// of its feature, interleaved with the feature's other warps:
//   * search: one sample per lane (the forward's bin indices when given, else
//     an L-level descent over the interior edges in breadth-first order); the
//     sample's record {bin row offset | flags, q(t), x, r_k} goes to the
//     warp's record buffer;
//   * 4 steps of 8 samples (8 of 4 at D = 24): each lane reads its row's record
//     (one 16-byte load, shared by the row's lanes), the S / T units of the sample's bin,
//     computes q(g') (the ReLU mask; skipped, bit-identically, when every
//     sample of the step is in an "open" bin, one whose ReLU input is positive
//     for every t it admits), the epilogue sums, its share of grad_x (summed
//     over the row's lanes by shuffles);
//   * then, step by step, H += q(g'), U += q(t) q(g') into the warp's copy
//     (one predicated 16-byte read-modify-write per element pair).  Samples of
//     one step that share a bin (found by match.any) update it in rounds, in
//     sample order.
// Shared-memory layout: every bin row of the S / T table and of the H / U sums
// is a sequence of 16-byte units, one per element pair ({S_2m, S_2m+1,
// T_2m, T_2m+1}, {H_2m, H_2m+1, U_2m, U_2m+1}), lane c owning units
// c NP .. c NP + NP - 1 (NP = VEC / 2).  With NP = 2 (D = 16) a bin row is 128
// bytes and the lanes of odd rows take their two units in the opposite order
// (their gradient pairs swapped to match), so the two rows that share a
// 128-byte wavefront read disjoint bank groups whatever their bins.  With D = 24
// a bin row is 256 bytes laid out unit-major (unit u of lane c at u 8 + c), so
// a 128-byte wavefront serves one row and has no conflict at all (a 192-byte
// lane-major row conflicts whenever two rows' bins have the same parity).
// At the end of a segment the Wf copies of a feature are summed in warp order,
// a suffix scan over bins turns H / U into grad_W and the partial goes to the
// workspace.  No floating-point atomics: bitwise deterministic for a given
// shape and device.
#pragma once

#include "ple_backward_impl.cuh"

namespace ple {

constexpr int kHistNC = 4;  // lanes per D row (d_embedding 8 / 16): 8 samples per warp step, 4 steps per batch of 32

// Lane slots per sample row (the kernel's NCL): 4 for d_embedding 8 and 16 (VEC = D / 4 elements each); 8
// for d_embedding 24 (6 active lanes of 4 elements, 2 idle), whose bin rows are laid out unit-major so that
// one 128-byte wavefront serves one row and never meets a bank conflict.
// Bytes of one bin row of pair units (S / T table, H / U sums).
__host__ __device__ constexpr int hist_row_bytes(int D) { return D == 24 ? 256 : 8 * D; }
// 16 warps per CTA (128 registers a thread; measured faster than 12 warps with 168 registers)
constexpr int kHistWarps = 16, kHistThreads = 32 * kHistWarps;

// record flags (low bits of the bin row offset, which is a multiple of 64): tie, open bin, dead row, and the
// sample's rank among the samples of its step that share its bin (bits 3-5)
constexpr int kRecTie = 1, kRecOpen = 2, kRecDead = 4, kRecRankShift = 3, kRecRank = 7 << kRecRankShift;
constexpr int kRecFlags = 63;

struct HistLayout {
  float* sAcc;      // [16 warps][B][row] private H / U units
  float* sST;       // [Fc][B][row] S / T units, logical bin order
  float* sX;        // [2][Fc][S_t + 8] x tiles (transposed; the pad spreads the cp.async stores over banks)
  float* sGX;       // [2][S_t][Fc] grad_x tiles
  float4* sRec;     // [16 warps][32] sample records of the current batch
  float* sKey;      // [Fc][nkeys] interior edges in breadth-first order (node 1 = root)
  float2* sER;      // [Fc][B] {e_k, r_k}
  unsigned* sOpen;  // [Fc][ceil(B / 32)] open-bin bits
  float* sEpi;      // [Fc][Wf][2][D] per-warp epilogue sums
  int* sN;          // [Fc] real bins per feature
};

__host__ __device__ __forceinline__ int hist_xld(int S_t) { return S_t + 8; }

__host__ __device__ __forceinline__ size_t hist_layout_bytes(int B, int D, int Fc, int S_t, int nkeys, HistLayout* L,
                                                             unsigned char* base) {
  const int Wf = kHistWarps / Fc;
  const int ow = (B + 31) / 32;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 127) & ~(size_t)127;  // 128-byte aligned: bin rows start on a bank-window boundary
    return base + o;
  };
  unsigned char* pAcc = take((size_t)kHistWarps * B * hist_row_bytes(D));
  unsigned char* pST = take((size_t)Fc * B * hist_row_bytes(D));
  unsigned char* pX = take((size_t)2 * Fc * hist_xld(S_t) * 4);
  unsigned char* pGX = take((size_t)2 * S_t * Fc * 4);
  unsigned char* pRec = take((size_t)kHistWarps * 32 * 16);
  unsigned char* pK = take((size_t)Fc * nkeys * 4);
  unsigned char* pER = take((size_t)Fc * B * 8);
  unsigned char* pO = take((size_t)Fc * ow * 4);
  unsigned char* pE = take((size_t)Fc * Wf * 2 * D * 4);
  unsigned char* pN = take((size_t)Fc * 4);
  if (L) {
    L->sAcc = reinterpret_cast<float*>(pAcc);
    L->sST = reinterpret_cast<float*>(pST);
    L->sX = reinterpret_cast<float*>(pX);
    L->sGX = reinterpret_cast<float*>(pGX);
    L->sRec = reinterpret_cast<float4*>(pRec);
    L->sKey = reinterpret_cast<float*>(pK);
    L->sER = reinterpret_cast<float2*>(pER);
    L->sOpen = reinterpret_cast<unsigned*>(pO);
    L->sEpi = reinterpret_cast<float*>(pE);
    L->sN = reinterpret_cast<int*>(pN);
  }
  return off;
}

// Float offset of element d inside a bin row of 16-byte pair units (S or H at +0, T or U at +2): lane-major
// with 4 lanes a row (lane c's units at c NP + u), unit-major with 8 (unit u of lane c at u 8 + c).
template <int VEC, int NCL>
__device__ __forceinline__ int unit_float(int d) {
  constexpr int NP = VEC / 2;
  const int c = d / VEC, e = d - c * VEC;
  if constexpr (NCL == 8) return ((e >> 1) * NCL + c) * 4 + (e & 1);
  else return (c * NP + (e >> 1)) * 4 + (e & 1);
}

// The chunk's tables for one segment and zeroed private sums: search keys, {e_k, r_k}, S = q(W) and its
// exclusive prefix T in logical bin order (pair units), the open bits.
template <typename QT, int MASK, int VEC, int NCL>
__device__ __forceinline__ void stage_hist_tables(const BwdArgs& a, const HistLayout& L, int f0, int fc, int Fc,
                                                  int nkeys, int lgk, int tid, int nthr) {
  const int B = a.B, D = a.D, D2 = hist_row_bytes(D) / 4;  // floats of a bin row
  const int ow = (B + 31) / 32;
  for (int i = tid; i < Fc; i += nthr) {
    const int n = i < fc ? a.n_bins[f0 + i] : 1;
    L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  {
    float4* acc = reinterpret_cast<float4*>(L.sAcc);
    const int n4 = kHistWarps * B * D2 / 4;
    for (int idx = tid; idx < n4; idx += nthr) acc[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4* st = reinterpret_cast<float4*>(L.sST);
    for (int idx = tid; idx < Fc * B * D2 / 4; idx += nthr) st[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
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
  // S[i][logical bin] = q(W[i][physical bin]); one thread per (row, element)
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int idx = tid; idx < fc * B * D; idx += nthr) {
    const int row = idx / D, d = idx - row * D;
    const int i = row / B, p = row - i * B;
    const int n = L.sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) L.sST[(i * B + lg) * D2 + unit_float<VEC, NCL>(d)] = quantize<QT>(Wc[idx]);
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = L.sN[i];
    const int uo = unit_float<VEC, NCL>(d);
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      float* u = L.sST + (i * B + j) * D2 + uo;
      u[2] = acc;
      acc += u[0];
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
          const float* u = L.sST + (i * B + k) * D2 + unit_float<VEC, NCL>(d);
          const float S = u[0], T = u[2];
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

// ---------------------------------------------------------------- shared-memory access of pair units
__device__ __forceinline__ float4 lds_rec(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_rec(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
// {first pair, second pair} of a table unit (tables do not change while a tile is walked)
__device__ __forceinline__ void lds_unit(uint32_t addr, f2_t& a, f2_t& b) {
  asm("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

// Unit u of a lane's NP units, given the address of its first one; with NP == 2 the lane's first unit is
// the one its row parity reads first and the second is d1 = +16 or -16 bytes away.
template <int NP>
__device__ __forceinline__ uint32_t unit_addr(uint32_t a0, int u, uint32_t d1) {
  if constexpr (NP == 2) return u == 0 ? a0 : a0 + d1;
  else return a0 + 16u * u;
}

// H += g', U += t g' for the lane's NP units of one sample, when `live` (predicated loads and stores; the
// arithmetic in between runs on every lane).
template <int NP>
__device__ __forceinline__ void hist_rmw(uint32_t live, uint32_t a0, uint32_t d1, const f2_t (&g)[NP], f2_t t2) {
  f2_t h[NP], u[NP];
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    const uint32_t ad = e == 0 ? a0 : (NP == 2 ? a0 + d1 : a0 + 16u * e);
    // lanes that do not take part read zeros (their arithmetic is discarded by the store's predicate); the
    // registers are written on every lane, which keeps a predicated-off load from extending their live range
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\tmov.b64 %0, 0;\n\tmov.b64 %1, 0;\n\t"
                 "@p ld.shared.v2.b64 {%0, %1}, [%3];\n\t}"
                 : "=l"(h[e]), "=l"(u[e]) : "r"(live), "r"(ad) : "memory");
  }
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    h[e] = add2(h[e], g[e]);
    u[e] = fma2(t2, g[e], u[e]);
  }
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    const uint32_t ad = e == 0 ? a0 : (NP == 2 ? a0 + d1 : a0 + 16u * e);
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %0, 0;\n\t@p st.shared.v2.b64 [%1], {%2, %3};\n\t}"
                 ::"r"(live), "r"(ad), "l"(h[e]), "l"(u[e]) : "memory");
  }
}

// Rounds 2, 3, ... of the ordered read-modify-writes of one step (a bin shared by three or more of its
// samples; rare, so kept out of line).
template <int NP>
__device__ __noinline__ void hist_rmw_rounds(uint32_t live, int rank, uint32_t a0, uint32_t d1, f2_t q0, f2_t q1,
                                             f2_t q2, f2_t t2) {
  f2_t q[NP];
  q[0] = q0;
  if constexpr (NP > 1) q[1] = q1;
  if constexpr (NP > 2) q[2] = q2;
  for (int rd = 2;; ++rd) {
    __syncwarp();
    hist_rmw<NP>(live && rank == rd ? 1u : 0u, a0, d1, q, t2);
    if (!__any_sync(0xffffffffu, rank > rd)) break;
  }
}
template <int NP>
__device__ __forceinline__ void hist_rmw_rounds(uint32_t live, int rank, uint32_t a0, uint32_t d1,
                                                const f2_t (&q)[NP], f2_t t2) {
  hist_rmw_rounds<NP>(live, rank, a0, d1, q[0], NP > 1 ? q[NP > 1 ? 1 : 0] : 0ull, NP > 2 ? q[NP > 2 ? 2 : 0] : 0ull,
                      t2);
}

// The lane's NP gradient pairs of one sample in unit order (NP == 2 and an odd row: swapped).
template <typename GT, int VEC>
__device__ __forceinline__ void grad_pairs(const GRaw<GT, VEC>& g, bool swap, f2_t (&out)[VEC / 2]) {
  constexpr int NP = VEC / 2;
#pragma unroll
  for (int e = 0; e < NP; ++e) out[e] = raw_pair<GT, VEC>(g, e);
  if constexpr (NP == 2) {
    const f2_t p0 = out[0], p1 = out[1];
    out[0] = swap ? p1 : p0;
    out[1] = swap ? p0 : p1;
  }
}

template <typename QT, typename GT, int VEC, int MASK, int EPIV, int NCL>
__global__ void __launch_bounds__(kHistThreads, 1)
    ple_bwd_hist_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap gmap) {
  constexpr int NC = NCL, R = 32 / NC, J = NC;  // lane slots per row, samples per step, steps per batch
  // steps processed together (registers: a group's records, units and sums are live together)
  constexpr int JG = 2;
  constexpr int NG = J / JG;  // groups per batch (even)
  constexpr int D = NC == 8 ? 24 : NC * VEC;
  constexpr int NA = D / VEC;  // active lanes of a row
  static_assert(NC == 4 || (NC == 8 && VEC == 4), "8 lane slots only for d_embedding 24");
  constexpr int NP = VEC / 2;
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ACC = EPIV != kEpvNone;
  constexpr bool ROUND_G = !std::is_same<GT, QT>::value && !std::is_same<QT, float>::value;
  constexpr uint32_t kRow = hist_row_bytes(D);  // bytes of a bin row (S / T units, H / U units)
  static_assert(kRow == (uint32_t)NP * NC * 16, "pair units of a row");
  static_assert(VEC == 2 || VEC == 4 || VEC == 6, "the histogram kernel packs 1 to 3 fp32 pairs per lane");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int B = a.B;
  const int Fc = a.Fc, S_t = a.hist_St;
  const int Wf = kHistWarps / Fc;
  const int nkeys = 1 << a.lgk;
  const int ow = (B + 31) / 32;
  const int xld = hist_xld(S_t);
  HistLayout L;
  hist_layout_bytes(B, D, Fc, S_t, nkeys, &L, smem_raw);

  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int r = lane / NC, c = lane - r * NC;
  const bool active = c < NA;  // idle lanes (8 slots at D = 24) load nothing and add zeros to the row's pad
  const bool swap = NP == 2 && NC == 4 && (r & 1) != 0;
  const int my_i = wid / Wf, my_w = wid - my_i * Wf;
  const unsigned lt = (1u << lane) - 1u;
  const int JB = S_t / (32 * Wf);  // batches per warp per tile (even: the host plans it so)
  const bool do_gx = a.grad_x != nullptr;
  const GT* gptr = reinterpret_cast<const GT*>(a.g);
  const uint64_t pol_first = l2_policy_evict_first();
  const float thr = zero_round_threshold<QT>();
  // this lane's first unit inside a bin row (odd rows of D = 16 start with the second pair)
  // this lane's first unit inside a bin row and the step to its second (NP == 2): lane-major rows (odd rows
  // of D = 16 start with the second pair) or unit-major rows (D = 24)
  const uint32_t lane_unit = NC == 8 ? (uint32_t)c * 16u : (uint32_t)(c * NP + (swap ? 1 : 0)) * 16u;
  const uint32_t d1 = NC == 8 ? (uint32_t)NC * 16u : swap ? (uint32_t)-16 : 16u;
  const uint32_t acc_base = shared_addr(L.sAcc) + (uint32_t)wid * B * kRow + lane_unit;
  const uint32_t rec_w = shared_addr(L.sRec + wid * 32);
  const uint32_t rec_r = rec_w + (uint32_t)r * 16u;

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
      float* dst = L.sX + (T & 1) * Fc * xld;
      for (int q = tid; q < ns * Fc; q += nthr) {
        const int s = q / Fc, i = q - s * Fc;
        if (i < fc) cp_async4(dst + i * xld + s, a.x + (t0 + s) * a.F + f0 + i);
        else dst[i * xld + s] = 0.0f;
      }
      cp_async_commit();
    };
    auto prefetch_g = [&](int T) {
      if (!a.g_prefetch || tid != 0) return;
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      const uint64_t pol_last = l2_policy_evict_last();
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
    stage_hist_tables<QT, MASK, VEC, NCL>(a, L, f0, fc, Fc, nkeys, a.lgk, tid, nthr);

    // per-lane epilogue parameters and sums, in this lane's unit order
    f2_t pbias[NP], w0r[NP], aw[NP], ab[NP];  // aw: sum g x (B) or sum g' (A); ab: sum g (B)
#pragma unroll
    for (int u = 0; u < NP; ++u) {
      pbias[u] = 0ull;
      w0r[u] = 0ull;
      aw[u] = 0ull;
      ab[u] = 0ull;
      const int e0 = c * VEC + 2 * ((NP == 2 && swap) ? 1 - u : u);
      if constexpr (MASK == kMaskReluBias) {
        if (live_w && active) pbias[u] = pack2(a.bias[(int64_t)(f0 + my_i) * D + e0], a.bias[(int64_t)(f0 + my_i) * D + e0 + 1]);
      }
      if constexpr (LIN) {
        if (live_w && active) w0r[u] = pack2(a.w0[(int64_t)(f0 + my_i) * D + e0], a.w0[(int64_t)(f0 + my_i) * D + e0 + 1]);
      }
    }
    const float* keys = L.sKey + my_i * nkeys;
    const float2* er = L.sER + my_i * B;
    const unsigned* openw = L.sOpen + my_i * ow;
    const int n1 = L.sN[my_i] - 1;
    const uint32_t st_base = shared_addr(L.sST) + (uint32_t)my_i * B * kRow + lane_unit;
    // this lane's gradient row of step 0 of the warp's first batch; batches advance by 32 Wf samples
    const int64_t FD = (int64_t)a.F * D;
    const GT* gp = gptr + (s_begin + 32 * my_w + r) * FD + (int64_t)(f0 + my_i) * D + c * VEC;
    int64_t srem = s_end - (s_begin + 32 * my_w + r);  // step j of the next batch to load is live iff j R < srem
    const int64_t gstep = (int64_t)R * FD, gbatch = (int64_t)32 * Wf * FD;
    const bool wide = a.g_wide != 0;

    // gradient rows of steps h JG .. h JG + JG - 1 of the warp's next batch; after the last group the batch
    // pointer moves on
    auto load_group = [&](GRaw<GT, VEC> (&g)[JG], int h) {
#pragma unroll
      for (int jj = 0; jj < JG; ++jj) {
        const int j = h * JG + jj;
        if (live_w && active && j * R < srem) {
          ldg_raw<GT, VEC>(g[jj], gp + j * gstep, wide, pol_first);
        } else {
#pragma unroll
          for (int w = 0; w < GRaw<GT, VEC>::kWords; ++w) g[jj].w[w] = 0u;
        }
      }
      if (h == NG - 1) {
        gp += gbatch;
        srem -= 32 * Wf;
      }
    };

    // search of batch jb of tile T (samples 32 (my_w + Wf jb) + lane of the tile), one sample per lane: its
    // record {bin row offset | flags, q(t), x, r_k}; returns the ballot (bit j 8 + r) of the samples with rank
    // >= 1 among the samples of their step in their bin, and in dup2 that of rank >= 2
    auto search = [&](int T, int jb, unsigned& dup2) -> unsigned {
      const int64_t t0 = s_begin + (int64_t)T * S_t;
      const int ns = (int)min64(S_t, s_end - t0);
      const float* xs = L.sX + (T & 1) * Fc * xld + my_i * xld;
      const int s_l = 32 * (my_w + Wf * jb) + lane;
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
      // rank among the earlier samples of the same step (lanes 8 j .. 8 j + 7) in the same bin
      const unsigned same = __match_any_sync(0xffffffffu, v ? (k | ((lane / R) << 16)) : (int)(0x40000000u | lane));
      const int rank = __popc(same & lt);
      const float2 e = er[k];
      const bool tie = v && k > 0 && x == e.x;
      const bool open = ((openw[k >> 5] >> (k & 31)) & 1u) != 0u;
      const int hf = k * (int)kRow | (tie ? kRecTie : 0) | (open || !v ? kRecOpen : 0) | (v ? 0 : kRecDead) |
                     (rank << kRecRankShift);
      const float t = v ? quantize<QT>((x - e.x) * e.y) : 0.0f;
      sts_rec(rec_w + (uint32_t)lane * 16u, make_float4(__int_as_float(hf), t, x, e.y));
      dup2 = __ballot_sync(0xffffffffu, rank >= 2);
      return __ballot_sync(0xffffffffu, rank >= 1);
    };

    // batch jb of tile T from the records: groups of JG steps, each phase by phase (records, tables and
    // arithmetic; grad_x; last the ordered read-modify-writes of the sums), so that the independent work of
    // the steps overlaps.  The gradient rows of a group are loaded one group ahead (g0: even groups, g1: odd).
    auto run_batch = [&](GRaw<GT, VEC> (&g0)[JG], GRaw<GT, VEC> (&g1)[JG], int T, int jb, unsigned dup1,
                         unsigned dup2) {
      const int sb0 = 32 * (my_w + Wf * jb);
      const uint32_t gxa = shared_addr(L.sGX + (T & 1) * S_t * Fc + (sb0 + r) * Fc + my_i);  // + j R Fc floats
      // the steps go in groups of JG (registers: a group's records, units and sums are live together)
      auto run_group = [&](const GRaw<GT, VEC> (&g)[JG], int h) {
        // ---- phase 1: records, S / T units, q(g'), the epilogue sums and the grad_x shares
        int hv[JG];
        float tv[JG];
        f2_t qv[JG][NP];
        float gx[JG];
        bool any_tie = false;
#pragma unroll
        for (int jj = 0; jj < JG; ++jj) {
          const int j = h * JG + jj;
          const float4 rec = lds_rec(rec_r + (uint32_t)(j * R * 16));
          hv[jj] = __float_as_int(rec.x);
          tv[jj] = rec.y;
          const float xv = rec.z;
          any_tie |= (hv[jj] & kRecTie) != 0;
          const uint32_t sa = st_base + (uint32_t)(hv[jj] & ~kRecFlags);
          f2_t S[NP], Tt[NP], gs[NP];
#pragma unroll
          for (int u = 0; u < NP; ++u) lds_unit(unit_addr<NP>(sa, u, d1), S[u], Tt[u]);
          grad_pairs<GT, VEC>(g[jj], swap, gs);
          bool exact = false;
          if constexpr (MASK != kMaskNone) exact = !__all_sync(0xffffffffu, (hv[jj] & kRecOpen) != 0);
          const f2_t t2 = pack2(tv[jj], tv[jj]);
          f2_t d2 = 0ull, dw2 = 0ull;
          const f2_t x2 = LIN ? pack2(xv, xv) : 0ull;
#pragma unroll
          for (int u = 0; u < NP; ++u) {
            const f2_t g2 = gs[u];
            if constexpr (LIN) {
              dw2 = fma2(g2, w0r[u], dw2);
              aw[u] = fma2(g2, x2, aw[u]);
              ab[u] = add2(ab[u], g2);
            }
            f2_t qq = g2;
            if constexpr (MASK != kMaskNone) {
              if (exact) {
                float p0, p1, g0, g1;
                unpack2(fma2(t2, S[u], Tt[u]), p0, p1);
                unpack2(g2, g0, g1);
                if constexpr (MASK == kMaskReluBias) {
                  round2<QT>(p0, p1);
                  float b0, b1;
                  unpack2(pbias[u], b0, b1);
                  p0 += b0;
                  p1 += b1;
                  qq = pack2(p0 <= 0.f ? 0.f : g0, p1 <= 0.f ? 0.f : g1);
                } else {
                  qq = pack2(p0 <= thr ? 0.f : g0, p1 <= thr ? 0.f : g1);
                }
              }
            }
            if constexpr (EPIV == kEpvBias) aw[u] = add2(aw[u], qq);  // sum g' (before the QT rounding)
            if constexpr (ROUND_G) {
              float q0, q1;
              unpack2(qq, q0, q1);
              round2<QT>(q0, q1);
              qq = pack2(q0, q1);
            }
            qv[jj][u] = qq;
            d2 = fma2(qq, S[u], d2);
          }
          float lo, hi;
          unpack2(d2, lo, hi);
          float gxl = rec.w * (lo + hi);
          if constexpr (LIN) {
            unpack2(dw2, lo, hi);
            gxl += lo + hi;
          }
          gx[jj] = gxl;
        }
        // ---- phase 2: grad_x (edge sub-gradient where x == e_k, k > 0), the row's 4 lane shares summed
        if (do_gx) {
          if (__any_sync(0xffffffffu, any_tie)) {
#pragma unroll
            for (int jj = 0; jj < JG; ++jj) {
              const bool tj = (hv[jj] & kRecTie) != 0;
              if (__any_sync(0xffffffffu, tj)) {
                const int hk = hv[jj] & ~kRecFlags;
                const int km = hk / (int)kRow;  // bin k of the sample
                const uint32_t sa = st_base + (uint32_t)(hk != 0 ? hk - (int)kRow : 0);
                f2_t dp2 = 0ull;
#pragma unroll
                for (int u = 0; u < NP; ++u) {
                  f2_t Sm, Tm;
                  lds_unit(unit_addr<NP>(sa, u, d1), Sm, Tm);
                  dp2 = fma2(qv[jj][u], Sm, dp2);
                }
                float lo, hi;
                unpack2(dp2, lo, hi);
                if (tj) gx[jj] += er[km > 0 ? km - 1 : 0].y * (lo + hi);
              }
            }
          }
          static_assert(JG == 2, "the two steps' row sums share one reduction");
          // even lanes carry step 0's sum, odd lanes step 1's, so every shuffled share is used; the pairs
          // are summed in the same order as two separate reductions would sum them (bit-identical)
          const bool odd = (c & 1) != 0;
          float s1 = (odd ? gx[1] : gx[0]) + __shfl_xor_sync(0xffffffffu, odd ? gx[0] : gx[1], 1);
          s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
          if constexpr (NC == 8) s1 += __shfl_xor_sync(0xffffffffu, s1, 4);
          const int hs = odd ? hv[1] : hv[0];
          if ((hs & kRecDead) == 0 && c < 2) sts_f32(gxa + (h * JG + c) * R * Fc * 4, s1);
        }
        // ---- phase 3: H += q(g'), U += q(t) q(g') into the warp's copy, step by step: the first samples of
        // their bin, then, in a step with a shared bin, the second ones, then, rarely (a bin shared by three
        // or more samples of the step), the rest out of line
#pragma unroll
        for (int jj = 0; jj < JG; ++jj) {
          const int j = h * JG + jj;
          const int sel = hv[jj] & (kRecDead | kRecRank);
          const uint32_t a0 = acc_base + (uint32_t)(hv[jj] & ~kRecFlags);
          const f2_t t2 = pack2(tv[jj], tv[jj]);
          hist_rmw<NP>(sel == 0 ? 1u : 0u, a0, d1, qv[jj], t2);
          if ((dup1 >> (R * j)) & ((1u << R) - 1u)) {  // uniform: the step has a shared bin
            __syncwarp();
            hist_rmw<NP>(sel == (1 << kRecRankShift) ? 1u : 0u, a0, d1, qv[jj], t2);
            if ((dup2 >> (R * j)) & ((1u << R) - 1u)) {
              const uint32_t live = (hv[jj] & kRecDead) ? 0u : 1u;
              hist_rmw_rounds<NP>(live, (hv[jj] & kRecRank) >> kRecRankShift, a0, d1, qv[jj], t2);
            }
          }
        }
      };
      // even groups run on g0 (the first loaded during the previous batch) while the next group loads into
      // g1, odd groups on g1 while the group after them (the next batch's first after the last) loads into g0
#pragma unroll
      for (int h = 0; h < NG; h += 2) {
        load_group(g1, h + 1);
        run_group(g0, h);
        load_group(g0, (h + 2) % NG);
        run_group(g1, h + 1);
      }
    };

    // tiles of S_t samples, JB batches per warp per tile
    GRaw<GT, VEC> g0[JG], g1[JG];
    load_group(g0, 0);
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
      for (int jb = 0; jb < JB; ++jb) {
        unsigned dup2;
        const unsigned dup1 = search(T, jb, dup2);
        __syncwarp();
        run_batch(g0, g1, T, jb, dup1, dup2);
        __syncwarp();  // every lane's reads of these records precede the next batch's search
      }
    }
    __syncthreads();  // every warp's sums and grad_x shares are in shared memory
    store_gx(n_tiles - 1);

    // ---- epilogue sums: back to element order, over the warp's 8 sample rows in row order, then the
    // warps of a feature in order
    if constexpr (ACC) {
      if constexpr (NP == 2) {
        const f2_t w0_ = aw[0], w1_ = aw[1], b0_ = ab[0], b1_ = ab[1];
        aw[0] = swap ? w1_ : w0_;
        aw[1] = swap ? w0_ : w1_;
        ab[0] = swap ? b1_ : b0_;
        ab[1] = swap ? b0_ : b1_;
      }
      f2_t sw[NP], sb[NP];
#pragma unroll
      for (int u = 0; u < NP; ++u) {
        sw[u] = aw[u];
        sb[u] = ab[u];
      }
#pragma unroll
      for (int r2 = 1; r2 < R; ++r2) {
#pragma unroll
        for (int u = 0; u < NP; ++u) {
          uint32_t lo, hi;
          bits2(aw[u], lo, hi);
          sw[u] = add2(sw[u], from_bits2(__shfl_sync(0xffffffffu, lo, r2 * NC + c),
                                         __shfl_sync(0xffffffffu, hi, r2 * NC + c)));
          if constexpr (LIN) {
            bits2(ab[u], lo, hi);
            sb[u] = add2(sb[u], from_bits2(__shfl_sync(0xffffffffu, lo, r2 * NC + c),
                                           __shfl_sync(0xffffffffu, hi, r2 * NC + c)));
          }
        }
      }
      if (live_w && r == 0 && active) {
        float* ep = L.sEpi + ((my_i * Wf + my_w) * 2) * D + c * VEC;
#pragma unroll
        for (int u = 0; u < NP; ++u) {
          float lo, hi;
          unpack2(sw[u], lo, hi);
          ep[2 * u] = lo;
          ep[2 * u + 1] = hi;
          if constexpr (LIN) {
            unpack2(sb[u], lo, hi);
            ep[D + 2 * u] = lo;
            ep[D + 2 * u + 1] = hi;
          }
        }
      }
    }
    // ---- the Wf copies of each feature summed in warp order into the first
    const int BD2 = B * (int)(kRow / 4);  // floats of one warp's copy
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
      const float* h = L.sAcc + (size_t)i * Wf * BD2 + unit_float<VEC, NCL>(d);
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
        const float* hj = h + j * (int)(kRow / 4);
        row[physical_bin(j, n, B) * D + d] = hj[2] + suffix;
        suffix += hj[0];
      }
      for (int p = n - 1; p < B - 1; ++p) row[p * D + d] = 0.f;  // padding rows
      if (EPIV != kEpvBias) row[B * D + d] = suffix;
    }
  }
}

// Host: plan (ple_backward.cu) and launch.
int hist_prepare(BwdArgs& a, size_t* smem, int* grid);

template <typename QT, typename GT, int VEC, int MASK, int EPIV, int NCL>
int launch_hist_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  int grid = 0;
  const int prep = hist_prepare(a, &smem, &grid);
  if (prep != PLE_OK) return prep;
  a.g_wide = (GRaw<GT, VEC>::kBytes == 32) && a.g_wide;
  CUtensorMap map;
  a.g_prefetch = bwd_grad_map(a, std::is_same<GT, float>::value ? 0 : std::is_same<GT, __nv_bfloat16>::value ? 2 : 1,
                              &map) ? 1 : 0;
  auto kern = ple_bwd_hist_kernel<QT, GT, VEC, MASK, EPIV, NCL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  kern<<<grid, kHistThreads, smem, st>>>(a, map);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward launch");
  return bwd_finalize(a, grid, st);
}

// Mask variant and epilogue terms (as launch_bwd_mask of the sorted kernel).
template <typename QT, typename GT, int VEC, int NCL>
int launch_hist_mask(const BwdArgs& a, cudaStream_t st) {
  const bool lin = a.epi == kEpiB && (a.grad_x || a.grad_w0 || a.grad_b0);
  const bool bias = a.epi == kEpiA && a.grad_bias;
  if (a.relu && a.epi == kEpiA)
    return bias ? launch_hist_t<QT, GT, VEC, kMaskReluBias, kEpvBias, NCL>(a, st)
                : launch_hist_t<QT, GT, VEC, kMaskReluBias, kEpvNone, NCL>(a, st);
  if (a.relu)
    return lin ? launch_hist_t<QT, GT, VEC, kMaskRelu, kEpvLin, NCL>(a, st)
               : launch_hist_t<QT, GT, VEC, kMaskRelu, kEpvNone, NCL>(a, st);
  if (lin) return launch_hist_t<QT, GT, VEC, kMaskNone, kEpvLin, NCL>(a, st);
  return bias ? launch_hist_t<QT, GT, VEC, kMaskNone, kEpvBias, NCL>(a, st)
              : launch_hist_t<QT, GT, VEC, kMaskNone, kEpvNone, NCL>(a, st);
}

// True when the histogram kernel serves a backward of this shape (ple_backward.cu).
bool backward_uses_hist(int64_t F, int64_t B, int64_t D);

// The backward of one dtype pair: the histogram kernel where it applies (D = 8, 16 or 24, at most 256 bins,
// tables that fit), else the sorted kernel with `vec` elements per lane.
template <typename QT, typename GT>
int launch_backward_dtype(const BwdArgs& a, int vec, cudaStream_t st) {
  if (backward_uses_hist(a.F, a.B, a.D)) {
    switch (a.D) {
      case 8: return launch_hist_mask<QT, GT, 2, 4>(a, st);
      case 16: return launch_hist_mask<QT, GT, 4, 4>(a, st);
      case 24: return launch_hist_mask<QT, GT, 4, 8>(a, st);
      default: break;
    }
  }
  return launch_bwd_dtype<QT, GT>(a, vec, st);
}

}  // namespace ple
