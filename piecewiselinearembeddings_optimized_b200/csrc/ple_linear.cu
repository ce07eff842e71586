// ple_linear.cu - the embeddings forward fused into the first Linear layer of
// its consumer: z[N, H] = flatten(y)[N, F*D] @ W1[H, F*D]^T + b1, where y is
// the fused embeddings forward (x_ple, epilogue A / B, optional ReLU) of
// ple_embeddings_forward.  y is never written to global memory: it is produced
// tile by tile in shared memory as the A operand of tcgen05 MMAs whose fp32
// accumulators live in tensor memory.  The reference stops at the [N, F, D]
// output (module.py:207-248); this is the consumer step after it, written for
// the autocast case, where the consumer's matmul runs on bf16 operands with
// fp32 accumulation.
//
// One CTA computes `rows` = 128 * RS output rows (RS row sub-tiles of 128, one
// M = 128 MMA each) by HG output columns (one column group of the H outputs).
// The K dimension (F * D) is walked in feature groups of G features (K slice
// KA = G * D, a multiple of 16).  Warp roles:
//   producers (P warps)  per group: wait for the group's tables; the work is
//       cut into items of 32 consecutive rows (one per lane) of one feature;
//       per item each lane runs one L-probe bin search over the feature's
//       interior edges, reads {e_k, r_k}, then for each 8-column chunk of the
//       feature two table rows, applies the epilogue, converts to bf16 and
//       stores 16 bytes into the A slot of the stage ring (canonical K-major
//       no-swizzle layout: the 32 lanes' stores of one chunk fill four whole
//       128-byte core-matrix rows); then fence.proxy.async and one arrive per
//       warp.  No barrier ties the producer warps together; the table rows
//       are skewed by 16 bytes per bin so that lanes on different bins
//       spread over the banks; x arrives in registers one group ahead.
//   loader (1 thread)    per group: bulk-copies the group's table image and the
//       group's W1 slice (pre-arranged in the MMA's core-matrix layout by a
//       pre-pass) into the table ring and the stage ring.
//   MMA (1 thread)       per group: waits for both halves of the stage, issues
//       KA / 16 x RS x n_nm MMAs, commits the stage back to the producers and
//       loader; after the last group commits the accumulator barrier.
// The producers then read the accumulators (tcgen05.ld), add b1 and store z.
// Every wait is bounded in time: an expired wait sets a shared abort flag
// (the other roles stop at their next wait) and the device status word, the
// CTA waits for its own copies and MMAs in flight, frees its tensor memory and
// returns; ple_linear_status() reads the word.
//
// Table image of a feature group (built per call from W by a pre-pass, the
// same prefix / slope tables as the fused forward):
//   n[G] i32 | keys[G][2^L] f32 | left[G][B] {e_k, r_k} f32x2 |
//   epi[2][KA] f32 (bias, or w0 and b0) | T[B][ldT] f32 | S[B][ldS] ST
// with keys = the interior edges e_1 .. e_{n-1} then +inf (2^L - 1 used, 2^L >= B),
// T[k][f*D + d] = sum_{j<k} q(W[f, j, d]) and S[k][..] = q(W[f, phys k, d]).
// The count of keys <= x, capped at n - 1, is the clamped right-sided bin
// (x below e_0 counts no key, x at or above e_n counts n - 1, NaN counts every
// key): an L-probe search instead of L + 2 over all B + 1 edges.  The T and S
// row strides (ldT = KA + 4 floats, ldS padded likewise) are an odd number of
// 16-byte units, so the reads of lanes on different bins start in different
// bank groups.
#include <stdio.h>
#include <string.h>

#include <type_traits>

#include "ple_common.cuh"
#include "ple_fwd_math.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"
#include "ple_tc.cuh"

namespace ple {

// Set to 1 by a fused-linear launch whose wait expired (ple_linear_status reads and clears it).
__device__ int g_lin_dev_err = 0;

constexpr int kLinLBO = 128;             // A slot: byte step between k-blocks (canonical, packed)
constexpr int kLinWaitLimit = 1 << 22;   // polls of the final drain waits
constexpr uint32_t kLinSuspendNs = 2000; // suspend-time hint of one poll
constexpr long long kLinWaitCycles = 4000000000LL;  // time bound of one wait (SM cycles)
constexpr int kLinMaxItems = 4;          // 32-row items per producer warp and group
constexpr int kLinMaxThreads = 576;      // up to 16 producer warps + loader + MMA
// Planning budget: the sm_100 opt-in maximum of dynamic shared memory per CTA (a
// constant, so that workspace sizes do not depend on which device is queried).
constexpr size_t kLinSmemBudget = 227 * 1024;

struct LinGeom {
  int G, KA, P, RS, rows, HG, n_hg, Nm, n_nm, SA, ST, n_items;
  int n_groups, lgk, ldK, ldT, ldS;   // keys per feature 2^lgk; ldT floats, ldS elements of the slope type
  int TB, WB, AB, SBO_A;              // bytes
  int oN, oK, oL, oEp, oT, oS;        // byte offsets inside a table slot
  int oTab, oStage, oBar, smem;       // byte offsets in dynamic shared memory
  int tmem_cols;
};

struct LinArgs {
  const float* x;
  const unsigned char* tab_img;  // [n_groups][TB]
  const unsigned char* w_img;    // [n_hg][n_groups][WB]
  const float* b1;               // [H] or null
  void* z;                       // [N, H]
  int64_t N;
  int F, B, D, H;
  LinGeom g;
  int* dev_err;
};

template <typename QT>
using SlopeT = typename std::conditional<std::is_same<QT, float>::value, float, __nv_bfloat16>::type;

// ------------------------------------------------------------------ pre-passes
// Table image of each feature group (one CTA per group).
template <typename QT>
__global__ void ple_lin_tables_kernel(const float* __restrict__ edges, const float* __restrict__ inv_w,
                                      const int32_t* __restrict__ n_bins, const float* __restrict__ W,
                                      const float* __restrict__ bias, const float* __restrict__ w0,
                                      const float* __restrict__ b0, int epi, int F, int B, int D,
                                      const LinGeom g, unsigned char* __restrict__ img) {
  using ST = SlopeT<QT>;
  const int gi = blockIdx.x, G = g.G, KA = g.KA;
  const int f0 = gi * G;
  unsigned char* base = img + (int64_t)gi * g.TB;
  int* sN = reinterpret_cast<int*>(base + g.oN);
  float* sK = reinterpret_cast<float*>(base + g.oK);
  float2* sL = reinterpret_cast<float2*>(base + g.oL);
  float* sEp = reinterpret_cast<float*>(base + g.oEp);
  float* sT = reinterpret_cast<float*>(base + g.oT);
  ST* sS = reinterpret_cast<ST*>(base + g.oS);
  auto nb = [&](int f) {
    if (f >= F) return 1;
    const int n = n_bins[f];
    return n < 1 ? 1 : (n > B ? B : n);
  };
  for (int i = threadIdx.x; i < (g.oK - g.oN) / 4; i += blockDim.x) sN[i] = i < G ? nb(f0 + i) : 0;
  // keys: interior edges e_1 .. e_{n-1}, +inf after (padding features: no keys)
  for (int idx = threadIdx.x; idx < G * g.ldK; idx += blockDim.x) {
    const int i = idx / g.ldK, j = idx - i * g.ldK, f = f0 + i;
    float e = __int_as_float(0x7f800000);
    if (f < F && j + 1 < nb(f)) e = edges[(int64_t)f * (B + 1) + j + 1];
    sK[idx] = e;
  }
  // {e_k, r_k} of each real bin; padding features and bins {0, 0}, so x = 0 gives t = 0 there
  for (int idx = threadIdx.x; idx < G * B; idx += blockDim.x) {
    const int i = idx / B, j = idx - i * B, f = f0 + i;
    float2 v = make_float2(0.0f, 0.0f);
    if (f < F && j < nb(f)) v = make_float2(edges[(int64_t)f * (B + 1) + j], inv_w[(int64_t)f * B + j]);
    sL[idx] = v;
  }
  for (int c = threadIdx.x; c < KA; c += blockDim.x) {
    const int i = c / D, d = c - i * D, f = f0 + i;
    float e0 = 0.0f, e1 = 0.0f;
    if (f < F) {
      if (epi == kEpiA) e0 = bias[(int64_t)f * D + d];
      if (epi == kEpiB) {
        e0 = w0[(int64_t)f * D + d];
        e1 = b0[(int64_t)f * D + d];
      }
    }
    sEp[c] = e0;
    sEp[KA + c] = e1;
  }
  const int ncol = g.ldT > g.ldS ? g.ldT : g.ldS;
  for (int c = threadIdx.x; c < ncol; c += blockDim.x) {
    const int i = c / D, d = c - i * D, f = f0 + i;
    const bool live = c < KA && f < F;
    const int n = live ? nb(f) : 0;
    float acc = 0.0f;
    for (int k = 0; k < B; ++k) {
      float s = 0.0f, tv = 0.0f;
      if (k < n) {
        s = quantize<QT>(W[((int64_t)f * B + physical_bin(k, n, B)) * D + d]);
        tv = acc;
        acc += s;
      }
      if (c < g.ldT) sT[(int64_t)k * g.ldT + c] = tv;
      if (c < g.ldS) sS[(int64_t)k * g.ldS + c] = Dt<ST>::from_f(s);
    }
  }
}

// W1 [H][K] (bf16, row-major, K = F * D) -> per (column group, feature group) slot
// of HG x KA in the K-major core-matrix layout [n / 8][k / 8][n % 8][k % 8]
// (16-byte lines), zero outside [0, H) x [0, K).
__global__ void ple_lin_wimg_kernel(const __nv_bfloat16* __restrict__ W1, int64_t H, int64_t K, const LinGeom g,
                                    uint4* __restrict__ img) {
  const int kb_n = g.KA / 8;
  const int64_t lines_per_slot = (int64_t)g.HG * kb_n;
  const int64_t total = lines_per_slot * g.n_hg * g.n_groups;
  const bool vec = (K % 8) == 0 && (reinterpret_cast<uintptr_t>(W1) & 15) == 0;
  for (int64_t L = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; L < total; L += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slot = L / lines_per_slot;
    const int li = (int)(L - slot * lines_per_slot);
    const int hg = (int)(slot / g.n_groups), gi = (int)(slot - (int64_t)hg * g.n_groups);
    const int n8 = li / (8 * kb_n), rem = li - n8 * 8 * kb_n;
    const int kb = rem >> 3, nr = rem & 7;
    const int64_t h = (int64_t)hg * g.HG + n8 * 8 + nr;
    const int64_t k0 = (int64_t)gi * g.KA + kb * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (h < H) {
      const __nv_bfloat16* src = W1 + h * K + k0;
      if (vec && k0 + 8 <= K) {
        v = __ldg(reinterpret_cast<const uint4*>(src));
      } else {
        unsigned short u[8];
        for (int e = 0; e < 8; ++e) u[e] = (k0 + e < K) ? __bfloat16_as_ushort(src[e]) : (unsigned short)0;
        v = make_uint4(u[0] | (u[1] << 16), u[2] | (u[3] << 16), u[4] | (u[5] << 16), u[6] | (u[7] << 16));
      }
    }
    img[L] = v;
  }
}

// ------------------------------------------------------------------ main kernel
// Wait for the phase of `parity` of an mbarrier.  Each poll may suspend the
// thread in hardware for up to kLinSuspendNs (it resumes when the phase
// completes), so waiting threads do not spin on the issue slots the producer
// warps need.  Bounded by time: after kLinWaitCycles SM cycles (about two
// seconds) the wait gives up and raises the CTA's abort flag; it also returns
// early once another role has raised it.
__device__ __forceinline__ bool lin_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t a = tc::smem_addr(bar);
  long long t0 = 0;
  for (int i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(kLinSuspendNs)
        : "memory");
    if (done) return true;
    if (i == 0) t0 = clock64();
    if ((i & 7) == 7) {
      if (*abort) return false;
      if (clock64() - t0 > kLinWaitCycles) break;
    }
  }
  *abort = 1;
  return false;
}

template <typename ZT>
__device__ __forceinline__ void store_z8(ZT* p, int64_t h, int64_t H, const float (&v)[8]) {
  if (h + 8 <= H && (H & 7) == 0) {
    if constexpr (std::is_same<ZT, float>::value) {
      reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      *reinterpret_cast<uint4*>(p) = make_uint4(cvt_pack<ZT>(v[0], v[1]), cvt_pack<ZT>(v[2], v[3]),
                                                cvt_pack<ZT>(v[4], v[5]), cvt_pack<ZT>(v[6], v[7]));
    }
  } else {
    for (int e = 0; e < 8; ++e)
      if (h + e < H) p[e] = Dt<ZT>::from_f(v[e]);
  }
}

// key_count with a pointer walk: each probe is a load at an immediate offset,
// a compare and a select.
template <int L>
__device__ __forceinline__ int key_count_ptr(float x, const float* keys) {
  const float* p = keys;
#pragma unroll
  for (int h = (1 << L) >> 1; h > 0; h >>= 1) p = !(x < p[h - 1]) ? p + h : p;
  return (int)(p - keys);
}

// One item of a producer warp: this lane's row of one feature of the group.
// Bin search over the feature's interior edges, position, then per 8-column
// chunk the prefix / slope rows, the epilogue, bf16 conversion and a 16-byte
// store into the A slot (chunk cc at aS + cc * 128).  sT, sS, sEp point at the
// feature's first column.
template <int L, typename QT, typename OTe, int EPI, bool RELU, typename ST>
__device__ __forceinline__ void lin_item(float xv, int n_f, const float* keys, const float2* left, const float* sT,
                                         const ST* sS, const float* sEp, int ldT, int ldS, int KA, int nd,
                                         unsigned char* aS) {
  const int c = key_count_ptr<L>(xv, keys);
  const int k = c < n_f - 1 ? c : n_f - 1;
  const float2 er = left[k];
  const float tq = quantize<QT>((xv - er.x) * er.y);
  const float* tr = sT + k * ldT;
  const ST* sr = sS + k * ldS;
  for (int cc = 0; cc < nd; ++cc) {
    FV<8> ep0, ep1;
#pragma unroll
    for (int e = 0; e < 8; ++e) { ep0.v[e] = 0.0f; ep1.v[e] = 0.0f; }
    if constexpr (EPI != kEpiNone) ep0 = lds<8>(sEp + cc * 8);
    if constexpr (EPI == kEpiB) ep1 = lds<8>(sEp + KA + cc * 8);
    const FV<8> tv = lds<8>(tr + cc * 8);
    FV<8> sv;
    if constexpr (std::is_same<ST, float>::value) {
      sv = lds<8>(sr + cc * 8);
    } else {
      const uint4 u = *reinterpret_cast<const uint4*>(sr + cc * 8);
      widen_pack<__nv_bfloat16>(u.x, sv.v[0], sv.v[1]);
      widen_pack<__nv_bfloat16>(u.y, sv.v[2], sv.v[3]);
      widen_pack<__nv_bfloat16>(u.z, sv.v[4], sv.v[5]);
      widen_pack<__nv_bfloat16>(u.w, sv.v[6], sv.v[7]);
    }
    const FV<8> y = fwd_chunk<QT, OTe, 8, EPI, RELU>(tq, tv, sv, xv, ep0, ep1);
    const uint4 pk = make_uint4(cvt_pack<__nv_bfloat16>(y.v[0], y.v[1]), cvt_pack<__nv_bfloat16>(y.v[2], y.v[3]),
                                cvt_pack<__nv_bfloat16>(y.v[4], y.v[5]), cvt_pack<__nv_bfloat16>(y.v[6], y.v[7]));
    *reinterpret_cast<uint4*>(aS + cc * kLinLBO) = pk;
  }
}

template <typename QT, int EPI, bool RELU, typename ZT>
__global__ void __launch_bounds__(kLinMaxThreads, 1) ple_linear_kernel(const __grid_constant__ LinArgs a) {
  using ST = SlopeT<QT>;
  using OTe = typename std::conditional<std::is_same<QT, float>::value, float, QT>::type;
  extern __shared__ __align__(1024) unsigned char smem[];
  const LinGeom& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = g.P, SA = g.SA, STn = g.ST, n_groups = g.n_groups;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + g.oBar);
  uint64_t* full = bars;              // [SA] producer warps wrote the A slot
  uint64_t* wfull = bars + SA;        // [SA] W1 slice landed
  uint64_t* empty = bars + 2 * SA;    // [SA] MMAs of the stage done
  uint64_t* tfull = bars + 3 * SA;    // [ST] table image landed
  uint64_t* tempty = tfull + STn;     // [ST] producers done with the tables
  uint64_t* accb = tempty + STn;      // accumulators final
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(accb + 1);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

  if (tid == 0) {
    for (int s = 0; s < SA; ++s) {
      tc::mbar_init(&full[s], P);
      tc::mbar_init(&wfull[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < STn; ++t) {
      tc::mbar_init(&tfull[t], 1);
      tc::mbar_init(&tempty[t], P);
    }
    tc::mbar_init(accb, 1);
    *sAbort = 0;
  }
  if (warp == 0) tc::tmem_alloc(sTmem, g.tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *sTmem;
  const int64_t row0 = (int64_t)blockIdx.x * g.rows;
  const int hg = blockIdx.y;

  if (warp < P) {
    // ------------------------------------------------------------ producers
    const int G = g.G, KA = g.KA, B = a.B, F = a.F, D = a.D, lgk = g.lgk;
    const int ldK = g.ldK, ldT = g.ldT, ldS = g.ldS, TB = g.TB, stage_bytes = g.AB + g.WB;
    const int64_t N = a.N;
    // items of this warp: it = warp + j * P -> rows rb * 32 + lane of feature f = it % G of the group
    const int nd = D / 8, n_items = g.n_items, SBO_A = g.SBO_A;
    const int my_items = warp < n_items ? (n_items - warp + P - 1) / P : 0;
    const unsigned char* tab0 = smem + g.oTab;
    unsigned char* stage0 = smem + g.oStage;
    // x of this lane's rows, one group ahead
    float xc[kLinMaxItems], xn[kLinMaxItems];
    auto load_x = [&](int gi, float (&dst)[kLinMaxItems]) {
#pragma unroll
      for (int j = 0; j < kLinMaxItems; ++j) {
        dst[j] = 0.0f;
        if (j < my_items && gi < n_groups) {
          const int it = warp + j * P, rb = it / G, f = it - rb * G;
          const int64_t row = row0 + rb * 32 + lane;
          const int fg = gi * G + f;
          if (row < N && fg < F) dst[j] = __ldg(a.x + row * F + fg);
        }
      }
    };
    load_x(0, xc);
    load_x(1, xn);
    bool fail = false;
    int s = 0, s_round = 0, t = 0;
    uint32_t t_par = 0;
    for (int gi = 0; gi < n_groups; ++gi) {
      const unsigned char* tb = tab0 + t * TB;
      bool ok = lin_wait(&tfull[t], t_par, sAbort);
      if (ok && s_round > 0) ok = lin_wait(&empty[s], (s_round - 1) & 1, sAbort);
      if (__any_sync(0xffffffffu, !ok)) {  // warp-uniform exit
        fail = true;
        break;
      }
      unsigned char* slot = stage0 + s * stage_bytes;
#pragma unroll
      for (int j = 0; j < kLinMaxItems; ++j) {
        if (j < my_items) {
          const int it = warp + j * P, rb = it / G, f = it - rb * G;
          const int r = rb * 32 + lane;
          const int n_f = reinterpret_cast<const int*>(tb + g.oN)[f];
          const float* keys = reinterpret_cast<const float*>(tb + g.oK) + f * ldK;
          const float2* left = reinterpret_cast<const float2*>(tb + g.oL) + f * B;
          const float* sT = reinterpret_cast<const float*>(tb + g.oT) + f * D;
          const ST* sS = reinterpret_cast<const ST*>(tb + g.oS) + f * D;
          const float* sEp = reinterpret_cast<const float*>(tb + g.oEp) + f * D;
          unsigned char* aS = slot + (r >> 3) * SBO_A + (r & 7) * 16 + f * nd * kLinLBO;
          switch (lgk) {
#define PLE_LIN_ITEM(L) \
  case L: lin_item<L, QT, OTe, EPI, RELU, ST>(xc[j], n_f, keys, left, sT, sS, sEp, ldT, ldS, KA, nd, aS); break;
            PLE_LIN_ITEM(0) PLE_LIN_ITEM(1) PLE_LIN_ITEM(2) PLE_LIN_ITEM(3) PLE_LIN_ITEM(4)
            PLE_LIN_ITEM(5) PLE_LIN_ITEM(6) PLE_LIN_ITEM(7) PLE_LIN_ITEM(8)
#undef PLE_LIN_ITEM
            default: break;
          }
        }
      }
      tc::fence_proxy_async();
#pragma unroll
      for (int j = 0; j < kLinMaxItems; ++j) xc[j] = xn[j];
      load_x(gi + 2, xn);
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&full[s]);
        tc::mbar_arrive(&tempty[t]);
      }
      if (++s == SA) { s = 0; ++s_round; }
      if (++t == STn) { t = 0; t_par ^= 1u; }
    }
    // ------------------------------------------------------------ epilogue: TMEM -> z
    if (!fail) {
      const bool ok = __all_sync(0xffffffffu, lin_wait(accb, 0, sAbort)) && *sAbort == 0;
      if (ok) {
        tc::fence_after_sync();
        const int q = warp & 3;
        const int nq = (P - q + 3) / 4, iq = warp >> 2;
        const int total = g.RS * g.HG / 8;
        const int c_lo = total * iq / nq, c_hi = total * (iq + 1) / nq;
        const int64_t H = a.H;
        ZT* z = reinterpret_cast<ZT*>(a.z);
        for (int ch = c_lo; ch < c_hi; ++ch) {
          const int c = ch * 8;
          const int r = c / g.HG, h = c - r * g.HG;
          uint32_t u[8];
          tc::tmem_ld8(tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)c, u);
          tc::wait_ld();
          tc::hold8(u);
          const int64_t row = row0 + r * 128 + 32 * q + lane;
          const int64_t hglob = (int64_t)hg * g.HG + h;
          if (row < N && hglob < H) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              v[e] = __uint_as_float(u[e]);
              if (a.b1 != nullptr && hglob + e < H) v[e] += __ldg(a.b1 + hglob + e);
            }
            store_z8<ZT>(z + row * H + hglob, hglob, H, v);
          }
        }
      }
    }
    if (fail || *sAbort) {
      if (lane == 0) atomicExch(a.dev_err, 1);
    }
  } else if (warp == P) {
    // ------------------------------------------------------------ loader
    if (lane == 0) {
      int t_issued = 0, w_issued = 0;
      for (int gi = 0; gi < n_groups; ++gi) {
        const int t = gi % STn, s = gi % SA;
        if (gi >= STn && !lin_wait(&tempty[t], ((gi / STn) - 1) & 1, sAbort)) break;
        tc::mbar_arrive_expect_tx(&tfull[t], (uint32_t)g.TB);
        tc::bulk_g2s(smem + g.oTab + t * g.TB, a.tab_img + (int64_t)gi * g.TB, (uint32_t)g.TB, &tfull[t]);
        ++t_issued;
        if (gi >= SA && !lin_wait(&empty[s], ((gi / SA) - 1) & 1, sAbort)) break;
        tc::mbar_arrive_expect_tx(&wfull[s], (uint32_t)g.WB);
        tc::bulk_g2s(smem + g.oStage + s * (g.AB + g.WB) + g.AB,
                     a.w_img + ((int64_t)hg * n_groups + gi) * g.WB, (uint32_t)g.WB, &wfull[s]);
        ++w_issued;
      }
      // the CTA must not exit with a copy in flight: wait for the last copy into every slot
      for (int t = 0; t < STn && t < t_issued; ++t) {
        const int last = t + ((t_issued - 1 - t) / STn) * STn;  // last group copied into slot t
        tc::mbar_wait(&tfull[t], (last / STn) & 1, kLinWaitLimit);
      }
      for (int s = 0; s < SA && s < w_issued; ++s) {
        const int last = s + ((w_issued - 1 - s) / SA) * SA;
        tc::mbar_wait(&wfull[s], (last / SA) & 1, kLinWaitLimit);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_kk(128, g.Nm);
      const uint32_t LBO_A = kLinLBO, SBO_A = (uint32_t)g.SBO_A;
      const uint32_t SBO_B = (uint32_t)(g.KA / 8) * 128u;
      const int ksteps = g.KA / 16;
      for (int gi = 0; gi < n_groups; ++gi) {
        const int s = gi % SA;
        const uint32_t par = (gi / SA) & 1;
        if (!lin_wait(&full[s], par, sAbort) || !lin_wait(&wfull[s], par, sAbort)) break;
        tc::fence_after_sync();
        const uint32_t aS = tc::smem_addr(smem + g.oStage + s * (g.AB + g.WB));
        const uint32_t bS = aS + (uint32_t)g.AB;
        for (int j = 0; j < ksteps; ++j) {
          for (int r = 0; r < g.RS; ++r) {
            const uint64_t ad = tc::sdesc(aS + (uint32_t)r * 16u * SBO_A + (uint32_t)j * 2u * LBO_A, LBO_A, SBO_A);
            for (int nc = 0; nc < g.n_nm; ++nc) {
              const uint64_t bd =
                  tc::sdesc(bS + (uint32_t)(nc * g.Nm / 8) * SBO_B + (uint32_t)j * 256u, 128u, SBO_B);
              tc::mma_bf16(tbase + (uint32_t)(r * g.HG + nc * g.Nm), ad, bd, idesc, (gi > 0 || j > 0) ? 1u : 0u);
            }
          }
        }
        tc::commit(&empty[s]);
      }
      // always commit: the accumulator barrier then also covers every MMA issued before an abort
      tc::commit(accb);
      tc::mbar_wait(accb, 0, kLinWaitLimit);
    }
    __syncwarp();
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, g.tmem_cols);
  }
}

// ------------------------------------------------------------------ host
static int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Geometry for (F, B, D, H) and the slope element size; false when no
// configuration fits (D not a multiple of 8, or shared memory).
static bool lin_plan(int F, int B, int D, int64_t H, int s_bytes, size_t smem_max, LinGeom* out) {
  if (D % 8 != 0 || H <= 0 || H > (1 << 20)) return false;
  LinGeom g{};
  g.lgk = 0;
  while ((1 << g.lgk) < B) ++g.lgk;  // 2^lgk - 1 >= B - 1 interior edges
  if (g.lgk > 8) return false;
  g.ldK = 1 << g.lgk;
  const int Hp = round_up((int)H, 16);
  struct Cn { int RS, HG, n_hg, n_nm; };
  Cn cands[2];
  int nc = 0;
  if (Hp <= 256) {
    cands[nc++] = {2, Hp, 1, 1};
    cands[nc++] = {1, Hp, 1, 1};
  } else {
    const int n_hg = (Hp + 511) / 512;
    const int HG = round_up((Hp + n_hg - 1) / n_hg, 32);
    cands[nc++] = {1, HG, n_hg, HG > 256 ? 2 : 1};
  }
  for (int ci = 0; ci < nc; ++ci) {
    for (int G = 8; G >= 1; G >>= 1) {
      const int KA = G * D;
      if (KA % 16 != 0 || KA > 128) continue;
      const int rows = 128 * cands[ci].RS;
      const int n_items = (rows / 32) * G;
      const int P = n_items < 16 ? (n_items < 4 ? 4 : n_items) : 16;
      if ((n_items + P - 1) / P > kLinMaxItems) continue;
      LinGeom c = g;
      c.G = G;
      c.KA = KA; c.P = P; c.RS = cands[ci].RS; c.rows = rows; c.n_items = n_items;
      c.HG = cands[ci].HG; c.n_hg = cands[ci].n_hg; c.n_nm = cands[ci].n_nm; c.Nm = c.HG / c.n_nm;
      c.n_groups = (F + G - 1) / G;
      c.ldT = KA + 4;                                   // KA + 4 floats: an odd number of 16-byte units
      c.ldS = s_bytes == 2 ? KA + 8 : KA + 4;           // likewise for the slope rows
      int off = 0;
      c.oN = off; off += round_up(G * 4, 16);
      c.oK = off; off += round_up(G * c.ldK * 4, 16);
      c.oL = off; off += round_up(G * B * 8, 16);
      c.oEp = off; off += round_up(2 * KA * 4, 16);
      c.oT = off; off += B * c.ldT * 4;
      c.oS = off; off += B * c.ldS * s_bytes;
      c.TB = round_up(off, 128);
      c.SBO_A = (KA / 8) * kLinLBO;
      c.AB = round_up((rows / 8) * c.SBO_A, 128);
      c.WB = c.HG * KA * 2;
      c.tmem_cols = 32;
      while (c.tmem_cols < c.RS * c.HG) c.tmem_cols <<= 1;
      if (c.tmem_cols > 512) continue;
      for (int SA = 3; SA >= 2; --SA) {
        for (int STn = 4; STn >= 2; --STn) {
          c.SA = SA;
          c.ST = STn;
          int o = 0;
          c.oStage = o; o += SA * (c.AB + c.WB);
          c.oTab = o; o += c.ST * c.TB;
          c.oBar = o; o += (3 * SA + 2 * c.ST + 1) * 8 + 16;
          c.smem = round_up(o, 128);
          // at least 116 KB keeps one CTA per SM (the whole tensor memory is available to it)
          if (c.smem < 116 * 1024) c.smem = 116 * 1024;
          if ((size_t)c.smem <= smem_max) {
            *out = c;
            return true;
          }
        }
      }
    }
  }
  return false;
}

static size_t lin_ws_bytes(const LinGeom& g) {
  const size_t tab = (size_t)g.n_groups * g.TB;
  return ((tab + 255) & ~(size_t)255) + (size_t)g.n_hg * g.n_groups * g.WB;
}

static int* lin_err_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_lin_dev_err) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

int linear_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_lin_dev_err, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_lin_dev_err, &zero, sizeof(int));
  }
  return v;
}

size_t linear_workspace_bytes(int64_t F, int64_t B, int64_t D, int64_t H, int compute_dtype) {
  LinGeom g;
  const int s_bytes = compute_dtype == PLE_DTYPE_F32 ? 4 : 2;
  if (!lin_plan((int)F, (int)B, (int)D, H, s_bytes, kLinSmemBudget, &g)) return 0;
  return lin_ws_bytes(g);
}

template <typename QT, int EPI, bool RELU, typename ZT>
static int launch_lin_t(const LinArgs& a, cudaStream_t st) {
  auto kern = ple_linear_kernel<QT, EPI, RELU, ZT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, a.g.smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(linear)");
  const dim3 grid((unsigned)((a.N + a.g.rows - 1) / a.g.rows), (unsigned)a.g.n_hg);
  kern<<<grid, 32 * (a.g.P + 2), a.g.smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    char msg[256];
    snprintf(msg, sizeof(msg), "linear launch (%d threads, %d smem, kernel %d regs, max %d threads)",
             32 * (a.g.P + 2), a.g.smem, fa.numRegs, fa.maxThreadsPerBlock);
    return set_cuda_error(e, msg);
  }
  return PLE_OK;
}

template <typename QT, typename ZT>
static int launch_lin_epi(const LinArgs& a, int epi, int relu, cudaStream_t st) {
  if (epi == kEpiB)
    return relu ? launch_lin_t<QT, kEpiB, true, ZT>(a, st) : launch_lin_t<QT, kEpiB, false, ZT>(a, st);
  if (epi == kEpiA)
    return relu ? launch_lin_t<QT, kEpiA, true, ZT>(a, st) : launch_lin_t<QT, kEpiA, false, ZT>(a, st);
  return relu ? launch_lin_t<QT, kEpiNone, true, ZT>(a, st) : launch_lin_t<QT, kEpiNone, false, ZT>(a, st);
}

int launch_linear(const LinearCall& c, cudaStream_t st) {
  const int s_bytes = c.compute_dtype == PLE_DTYPE_F32 ? 4 : 2;
  LinArgs a{};
  if (!lin_plan(c.F, c.B, c.D, c.H, s_bytes, kLinSmemBudget, &a.g))
    return set_error(PLE_ERR_UNSUPPORTED,
                     "embeddings-linear: d_embedding must be a multiple of 8 and the tiles must fit in shared memory");
  if ((size_t)a.g.smem > device_max_smem_optin())
    return set_error(PLE_ERR_UNSUPPORTED, "embeddings-linear: the device has less shared memory per block than planned");
  const size_t need = lin_ws_bytes(a.g);
  if (c.ws == nullptr || c.ws_bytes < need)
    return set_error(PLE_ERR_WORKSPACE, "embeddings-linear: workspace smaller than ple_embeddings_linear_workspace_size()");
  if ((reinterpret_cast<uintptr_t>(c.ws) & 255) != 0)
    return set_error(PLE_ERR_ALIGNMENT, "embeddings-linear: workspace must be 256-byte aligned");
  a.dev_err = lin_err_ptr();
  if (!a.dev_err) return set_error(PLE_ERR_CUDA, "embeddings-linear: status word not addressable");
  unsigned char* ws = static_cast<unsigned char*>(c.ws);
  unsigned char* tab = ws;
  unsigned char* wimg = ws + (((size_t)a.g.n_groups * a.g.TB + 255) & ~(size_t)255);
  // pre-passes: table image and W1 image
  if (c.compute_dtype == PLE_DTYPE_F32)
    ple_lin_tables_kernel<float><<<a.g.n_groups, 256, 0, st>>>(c.edges, c.inv_w, c.n_bins, c.W, c.bias, c.w0, c.b0,
                                                                 c.epi, c.F, c.B, c.D, a.g, tab);
  else
    ple_lin_tables_kernel<__nv_bfloat16><<<a.g.n_groups, 256, 0, st>>>(c.edges, c.inv_w, c.n_bins, c.W, c.bias, c.w0,
                                                                         c.b0, c.epi, c.F, c.B, c.D, a.g, tab);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "embeddings-linear tables launch");
  {
    const int64_t lines = (int64_t)a.g.HG * (a.g.KA / 8) * a.g.n_hg * a.g.n_groups;
    int64_t blocks = (lines + 255) / 256;
    const int64_t cap = (int64_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    ple_lin_wimg_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(c.W1), c.H,
                                                          (int64_t)c.F * c.D, a.g, reinterpret_cast<uint4*>(wimg));
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(e, "embeddings-linear weight image launch");
  }
  a.x = c.x;
  a.tab_img = tab;
  a.w_img = wimg;
  a.b1 = c.b1;
  a.z = c.z;
  a.N = c.N;
  a.F = c.F; a.B = c.B; a.D = c.D; a.H = (int)c.H;
  if (c.compute_dtype == PLE_DTYPE_F32) {
    return c.out_dtype == PLE_DTYPE_F32 ? launch_lin_epi<float, float>(a, c.epi, c.relu, st)
                                        : launch_lin_epi<float, __nv_bfloat16>(a, c.epi, c.relu, st);
  }
  return c.out_dtype == PLE_DTYPE_F32 ? launch_lin_epi<__nv_bfloat16, float>(a, c.epi, c.relu, st)
                                      : launch_lin_epi<__nv_bfloat16, __nv_bfloat16>(a, c.epi, c.relu, st);
}

}  // namespace ple
