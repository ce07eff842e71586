// ple_backward_tc.cuh - the fused PLE backward on the 5th-generation tensor
// cores (tcgen05): per-bin gradient sums as one-hot GEMMs.
//
// Same gradients as ple_bwd_kernel (reference backward_cuda.cu:268-336 and
// :859-925 for grad_W, :343-492 for grad_x; epilogue terms from autograd of
// module.py:230-248):
//   H[j] = sum_{b: k_b = j} q(g'_b),  U[j] = sum_{b: k_b = j} q(t_b) q(g'_b),
//   grad_W[phys j] = U[j] + sum_{j' > j} H[j'].
// For a tile of R samples and one feature, H and U are the product
// onehot(k)^T [q(g') | q(t) q(g')]: A = the one-hot matrix (bins x samples,
// bf16 zeros and ones, K-major), B = the gradient rows (samples x columns,
// MN-major).  fp32 values enter B as an exact sum of bf16 parts (truncation
// split: q(g') needs 3 parts for fp32, 2 for fp16, 1 for bf16; the rounded
// fp32 product q(t) q(g') 3, 3 and 2), so every product in the tensor core is
// exact.  FM = 128 / Bp features are stacked in the M = 128 rows of one MMA
// (Bp = bins padded to 32, 64 or 128), and their columns side by side in N,
// so one MMA serves FM features (the off-diagonal blocks are discarded).
//
// The tensor core adds into its fp32 accumulator by aligning the addends to
// the largest exponent and truncating (bits below ~2^-23 of it are lost), so
// the TMEM accumulators are added into fp32 running sums (round to nearest,
// kept in spare TMEM columns) every `flush_tiles` tiles; the error per flush
// period is a few units in the last place of that period's sums.  Non-finite
// contributions (NaN or Inf gradients, infinite t) never enter an MMA, where
// 0 * Inf would poison every bin of the column: they are summed separately
// (order does not matter for non-finite sums) and added at the segment end.
//
// Per CTA (persistent, one per SM): producer warps plus one MMA warp, over a
// range of the flattened (feature chunk, sample) space as in ple_bwd_kernel.
// A producer warp owns one (feature, 8-column block) and its lanes consecutive
// sample rows (one or two 32-row blocks per tile), so operand lines are written
// without bank conflicts; x and the gradient chunk of the next tile are loaded
// into registers while the current tile is processed.  Per item: bin search,
// t, ReLU mask (recomputed from the staged q(W) table and its prefix), the
// grad_x share, the epilogue sums, the bf16 parts of the B-operand line and
// (column block 0) the one in A.  The producers then meet at a named barrier
// and arrive on the stage's `full` mbarrier; the MMA warp waits for it, issues
// the tile's MMAs (MMA issue blocks while the tensor core's queue is full, so
// it has a warp of its own) and commits them to the stage's `empty` mbarrier,
// which the producers wait on before they refill that stage.  The two operand
// stages alternate, so the tensor core works on tile i while the producers fill
// tile i + 1.  Every wait has an iteration limit; on expiry the kernel records
// an error, releases its tensor memory and returns.
#pragma once

#include <stdio.h>

#include "ple_backward_impl.cuh"
#include "ple_tc.cuh"

namespace ple {

// bf16 parts of q(g') (H) and of q(t) q(g') (U) for compute type QT
template <typename QT> struct TcParts { static constexpr int H = 3, U = 3; };
template <> struct TcParts<__nv_bfloat16> { static constexpr int H = 1, U = 2; };
template <> struct TcParts<__half> { static constexpr int H = 2, U = 3; };

constexpr int kTcMaxProducers = 384;  // up to 12 producer warps, plus the MMA warp
constexpr int kTcTmemCols = 512;
constexpr int kTcWaitLimit = 1 << 22;
constexpr int kTcItems = 2;  // 32-row blocks per producer thread and tile

// Registers per thread: fp32 gradients need more live state than 16-bit ones.  The register file is split
// over the SM's four sub-partitions (16K registers each) and warps are dealt out to them in turn, so a
// block of w warps fits when ceil(w / 4) * 32 * regs <= 16384 (168 registers: up to 12 warps; 128: 16).
template <typename GT> constexpr int tc_max_regs() { return sizeof(GT) == 4 ? 168 : 128; }
inline int tc_max_warps(int regs) { return 4 * (16384 / (32 * regs)); }

// Tile geometry and shared-memory layout, computed by the host (tc_plan).
struct TcGeom {
  int Bp, FM, fpm, Nmma, n_mma, cols, nG, nh, Fc, R, ts, flush_tiles, lgp, nu;  // nu = units per warp
  int oA, oB, oT, oS, oE, oR, oN, oGX, oTot, oKey, oBar;  // byte offsets into dynamic shared memory
  int64_t spec_off, escr_off;                            // float offsets into the workspace
  int* dev_err;                                          // set to 1 when a wait expires
};

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Named barrier that also returns the OR of every participant's flag.
__device__ __forceinline__ bool named_sync_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %2, 0;\n\t"
      "bar.red.or.pred q, %1, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(id), "r"((uint32_t)v), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(bar)) : "memory");
}

// Count of edges e_j with !(x < e_j) over a feature's 2^LG ascending edges (+inf padded): a fully
// unrolled power-of-two descent.
template <int LG>
__device__ __forceinline__ int count_le(float x, const float* e) {
  const float* p = e;
#pragma unroll
  for (int h = 1 << (LG - 1); h > 0; h >>= 1)
    if (!(x < p[h - 1])) p += h;
  if (!(x < p[0])) ++p;
  return (int)(p - e);
}
__device__ __forceinline__ int count_le_any(float x, const float* e, int lg) {
  switch (lg) {
    case 8: return count_le<8>(x, e);
    case 7: return count_le<7>(x, e);
    case 6: return count_le<6>(x, e);
    case 5: return count_le<5>(x, e);
    case 4: return count_le<4>(x, e);
    case 3: return count_le<3>(x, e);
    case 2: return count_le<2>(x, e);
    default: return count_le<1>(x, e);
  }
}

// Exact split of 4 packed pairs (8 fp32 values) into NP bf16 parts by
// truncation (part p keeps the top 8 significant bits of what parts 0..p-1
// left; the subtraction is exact), stored as NP 16-byte lines `stride` bytes
// apart.  Exact for values with at most 8 * NP significant bits.
template <int NP>
__device__ __forceinline__ void store_parts(const f2_t (&v)[4], unsigned char* dst, int stride) {
  const f2_t neg1 = pack2(-1.0f, -1.0f);
  uint32_t w[NP][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f2_t x = v[e];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      uint32_t u0, u1;
      bits2(x, u0, u1);
      w[p][e] = __byte_perm(u0, u1, 0x7632);
      if (p + 1 < NP) x = fma2(from_bits2(u0 & 0xffff0000u, u1 & 0xffff0000u), neg1, x);
    }
  }
#pragma unroll
  for (int p = 0; p < NP; ++p)
    *reinterpret_cast<uint4*>(dst + p * stride) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
}

// The chunk's tables for one segment (Fc features, producer threads only):
// bin counts, edges (feature-major, 2^lgp per feature, +inf padded), inverse
// widths (feature-major), S = q(W) in logical bin order and its exclusive prefix T.
template <typename QT>
__device__ void stage_tables_tc(const BwdArgs& a, int f0, int fc, int Fc, int ts, int lgp, float* sT, float* sS,
                                float* sE, float* sR, int* sN, int tid, int nthr) {
  const int B = a.B, D = a.D, pow2 = 1 << lgp;
  for (int i = tid; i < Fc; i += nthr) {
    const int n = i < fc ? a.n_bins[f0 + i] : 1;
    sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  for (int idx = tid; idx < B * ts; idx += nthr) sS[idx] = 0.0f;
  named_sync(1, nthr);
  for (int idx = tid; idx < pow2 * Fc; idx += nthr) {
    const int i = idx >> lgp, j = idx & (pow2 - 1);
    float e = __int_as_float(0x7f800000);
    if (i < fc && j <= sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j];
    sE[idx] = e;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {  // feature-major: [Fc][B]
    const int i = idx / B, j = idx - i * B;
    sR[idx] = (i < fc && j < sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
  }
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int row = tid; row < fc * B; row += nthr) {
    const int i = row / B, p = row - i * B;
    const int n = sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) {
      const float* src = Wc + (int64_t)row * D;
      float* dst = sS + lg * ts + i * D;
      for (int d = 0; d < D; ++d) dst[d] = quantize<QT>(src[d]);
    }
  }
  named_sync(1, nthr);
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = sN[i];
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int o = j * ts + i * D + d;
      sT[o] = acc;
      acc += sS[o];
    }
  }
}

template <typename QT, typename GT, int MASK, int EPIV>
__global__ void __maxnreg__(tc_max_regs<GT>()) ple_bwd_tc_kernel(const BwdArgs a, const TcGeom m) {
  constexpr int PH = TcParts<QT>::H, PU = TcParts<QT>::U, P = PH + PU;
  constexpr int IPT = kTcItems;
  constexpr bool LIN = EPIV == kEpvLin;
  constexpr bool ACCB = EPIV == kEpvBias;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nprod = blockDim.x - 32;  // producer threads; the last warp issues the MMAs
  const int WP = nprod >> 5;
  const bool is_mma_warp = wid == WP;
  const int B = a.B, D = a.D, Fc = m.Fc, nh = m.nh, R = m.R, Bp = m.Bp, FM = m.FM, ts = m.ts;
  const int Cf = P * D;

  unsigned char* sA = smem + m.oA;  // [2][nG][128 x R] bf16, K-major
  unsigned char* sB = smem + m.oB;  // [2][nG][R x cols] bf16, MN-major
  float* sT = reinterpret_cast<float*>(smem + m.oT);
  float* sS = reinterpret_cast<float*>(smem + m.oS);
  float* sE = reinterpret_cast<float*>(smem + m.oE);
  float* sR = reinterpret_cast<float*>(smem + m.oR);
  int* sN = reinterpret_cast<int*>(smem + m.oN);
  float* sGX = reinterpret_cast<float*>(smem + m.oGX);         // [2][Fc * nh][R] grad_x shares
  float* sTot = reinterpret_cast<float*>(smem + m.oTot);       // [units][4][8] per-warp H totals
  uint8_t* sKey = smem + m.oKey;                                // [2][Fc][R] bin whose one is set, 0xff none
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + m.oBar);  // [2] operands of the stage written
  uint64_t* empty = full + 2;                                   // [2] MMAs of the stage completed
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + m.oBar + 32);
  int* sFlag = reinterpret_cast<int*>(smem + m.oBar + 36);      // a non-finite contribution this segment
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + m.oBar + 40);

  const int a_group = 128 * R * 2, b_group = R * m.cols * 2;  // bytes
  const int a_stage = m.nG * a_group, b_stage = m.nG * b_group;
  const int sbo = (R >> 3) * 128;  // bytes between row blocks of A and column blocks of B
  const int part_stride = (D >> 3) * sbo;

  if (is_mma_warp) tc::tmem_alloc(sTmem, kTcTmemCols);
  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(&empty[0], 1);
    tc::mbar_init(&empty[1], 1);
    *sAbort = 0;
  }
  // operand buffers start zero: A keeps only the ones the producers set (and clear two tiles later),
  // B padding columns are never written
  for (int i = tid * 16; i < 2 * (a_stage + b_stage); i += blockDim.x * 16)
    *reinterpret_cast<uint4*>(sA + i) = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < 2 * R * Fc; i += blockDim.x) sKey[i] = 0xff;
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *sTmem;

  const int64_t total = (int64_t)a.n_chunks * a.N;
  const int64_t u_first = total * blockIdx.x / gridDim.x;
  const int64_t u_hi = total * (blockIdx.x + 1) / gridDim.x;
  bool failed = false;

  if (is_mma_warp) {
    // ---------------------------------------------------------------- MMA warp
    const uint32_t idesc = tc::idesc_bf16_a_k_b_mn(128, m.Nmma);
    uint32_t uses0 = 0, uses1 = 0;  // tiles issued per stage
    int gtile = 0;
    for (int64_t u_lo = u_first; u_lo < u_hi && !failed;) {
      const int chunk = (int)(u_lo / a.N);
      const int64_t s_begin = u_lo - (int64_t)chunk * a.N;
      const int64_t s_end = min64(a.N, s_begin + (u_hi - u_lo));
      u_lo += s_end - s_begin;
      const int n_tiles = (int)ceil_div<int64_t>(s_end - s_begin, R);
      for (int it = 0; it < n_tiles; ++it, ++gtile) {
        const int st = gtile & 1;
        const uint32_t uses = st ? uses1 : uses0;
        // operands written (and, at a flush point, the running sums updated) by the producers
        bool ok = false;
        for (int i = 0; i < kTcWaitLimit; ++i) {
          if (tc::mbar_wait(&full[st], uses & 1, 1)) {
            ok = true;
            break;
          }
          if (*sAbort) break;
        }
        if (!__all_sync(0xffffffffu, ok)) {
          failed = true;
          break;
        }
        tc::fence_after_sync();
        if (lane == 0) {
          const bool fresh = it == 0 || (it % m.flush_tiles) == 0;
          const uint32_t aB = tc::smem_addr(sA + st * a_stage), bB = tc::smem_addr(sB + st * b_stage);
          for (int g = 0; g < m.nG; ++g) {
            for (int ks = 0; ks < (R >> 4); ++ks) {
              const uint64_t ad = tc::sdesc(aB + g * a_group + ks * 256, 128, sbo);
              for (int jm = 0; jm < m.n_mma; ++jm) {
                const uint64_t bd = tc::sdesc(bB + g * b_group + jm * (m.Nmma >> 3) * sbo + ks * 256, 128, sbo);
                tc::mma_bf16(tbase + (uint32_t)(g * m.cols + jm * m.Nmma), ad, bd, idesc,
                             (fresh && ks == 0) ? 0u : 1u);
              }
            }
          }
          tc::commit(&empty[st]);
        }
        __syncwarp();
        if (st) ++uses1;
        else ++uses0;
      }
    }
    if (failed) {
      *sAbort = 1;
      if (lane == 0) atomicExch(m.dev_err, 1);
    }
    // the last commit (if any) covers every MMA this warp issued: wait for it before the TMEM is freed
    if (gtile > 0) {
      const int stl = (gtile - 1) & 1;
      const uint32_t uses = stl ? uses1 : uses0;
      tc::mbar_wait(&empty[stl], (uses - 1) & 1, kTcWaitLimit);
    }
  } else {
    // ---------------------------------------------------------------- producer warps
    // items: warp -> fixed (feature pf, column block ph), lanes -> sample rows r_j, the same rows in every
    // tile, so their shared-memory offsets and global pointers are set up once
    const int C = Fc * nh;
    const int cidx = wid % C;
    const int pf = cidx / nh, ph = cidx - pf * nh;
    const int rb0 = wid / C, rbstep = WP / C;
    const int pg = pf / FM, pslot = pf - pg * FM;
    const int pcol = (pslot / m.fpm) * m.Nmma + (pslot % m.fpm) * Cf + 8 * ph;
    const uint32_t rb8 = (uint32_t)(R >> 3);
    const uint32_t aslot = (uint32_t)(pslot * Bp);
    const uint32_t bcol = (uint32_t)(pcol >> 3) * rb8;  // core-matrix column of my B lines
    auto row_of = [&](int j) { return 32 * (rb0 + rbstep * j) + lane; };
    // byte offset of A row (feature slot, bin k) in a (stage, group) region
    auto arow = [&](int k) -> uint32_t {
      const uint32_t mr = aslot + (uint32_t)k;
      return (((mr >> 3) * rb8) << 7) + ((mr & 7u) << 4);
    };
    const float* sTt = sT + pf * D + 8 * ph;  // table rows of (pf, ph): bin k at + k * ts
    const float* sSt = sS + pf * D + 8 * ph;
    const float* sEf = sE + (pf << m.lgp);     // feature pf's edges
    const float* sRf = sR + pf * B;            // feature pf's inverse widths
    // flush role: the warp drains units fu = (wid >> 2) + (WP >> 2) * iu, iu < nu, of its TMEM lane quarter
    // sp; a unit is (group, 8-column block); lane -> (feature slot, bin) of the quarter
    const int sp = wid & 3;
    const int fm = sp * 32 + lane;
    const int fslot = fm / Bp, fbin = fm - fslot * Bp;
    const bool slot_used = fslot < FM;  // lane quarters past FM * Bp rows hold no feature (warp-uniform)
    const uint32_t tlane = tbase + ((uint32_t)(sp * 32) << 16);
    const int nu = slot_used ? m.nu : 0;
    // accumulator column of (unit fu, part 0) for this lane quarter's feature slot
    const uint32_t scol = (uint32_t)((fslot / m.fpm) * m.Nmma + (fslot % m.fpm) * Cf);
    auto unit_col = [&](int fu) {
      const int fgp = fu / nh;
      return (uint32_t)(fgp * m.cols + 8 * (fu - fgp * nh)) + scol;
    };
    const uint32_t rbase = (uint32_t)(m.nG * m.cols);  // running sums of unit fu at rbase + 16 fu

    const float thr = zero_round_threshold<QT>();
    const GT* gptr = reinterpret_cast<const GT*>(a.g);
    float* spec = a.ws + m.spec_off + (int64_t)blockIdx.x * Fc * Bp * 2 * D;
    float* escr = a.ws + m.escr_off + (int64_t)blockIdx.x * nprod * 16;
    const int lgp = m.lgp;
    const int bb = a.bin_idx_bytes;
    uint32_t done0 = 0, done1 = 0;  // tiles filled per stage (the stage's `empty` phases to wait for)
    int gtile = 0;

    // add the TMEM accumulators of this warp's units (its lanes' bins, 8 columns of each part) to the
    // running sums (warp-collective); `first` starts the sums.  Parts of one sum are added smallest first.
    auto flush = [&](bool first) {
#pragma unroll
      for (int iu = 0; iu < 4; ++iu) {
        if (iu < nu) {
          const int fu = (wid >> 2) + (WP >> 2) * iu;
          const uint32_t fcol = unit_col(fu), rcol = rbase + 16u * (uint32_t)fu;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            constexpr int PMAX = PH > PU ? PH : PU;
            const int np = half ? PU : PH, p0 = half ? PH : 0;
            uint32_t v[PMAX][8], acc[8];
#pragma unroll
            for (int p = 0; p < PMAX; ++p)
              if (p < np) tc::tmem_ld8(tlane + fcol + (uint32_t)((p0 + p) * D), v[p]);
            if (!first) tc::tmem_ld8(tlane + rcol + 8 * half, acc);
            tc::wait_ld();
#pragma unroll
            for (int p = 0; p < PMAX; ++p)
              if (p < np) tc::hold8(v[p]);
            if (!first) tc::hold8(acc);
#pragma unroll
            for (int d = 0; d < 8; ++d) {
              float h = __uint_as_float(v[np - 1][d]);
#pragma unroll
              for (int p = PMAX - 2; p >= 0; --p)
                if (p < np - 1) h += __uint_as_float(v[p][d]);
              if (!first) h += __uint_as_float(acc[d]);
              acc[d] = __float_as_uint(h);
            }
            tc::tmem_st8(tlane + rcol + 8 * half, acc);
          }
        }
      }
      tc::wait_st();
    };
    auto wait_empty = [&](int st, uint32_t done) -> bool {  // MMAs of the stage's last tile finished
      return done == 0 || tc::mbar_wait(&empty[st], (done - 1) & 1, kTcWaitLimit);
    };

    for (int64_t u_lo = u_first, seg = 0; u_lo < u_hi; ++seg) {
      const int chunk = (int)(u_lo / a.N);
      const int64_t s_begin = u_lo - (int64_t)chunk * a.N;
      const int64_t s_end = min64(a.N, s_begin + (u_hi - u_lo));
      u_lo += s_end - s_begin;
      const int f0 = chunk * Fc;
      const int fc = min(Fc, a.F - f0);
      const bool pf_live = pf < fc;
      const int64_t row_bytes_all = (int64_t)a.F * D * (int64_t)sizeof(GT);
      const unsigned pf_bytes = (unsigned)(fc * D * (int)sizeof(GT));
      const bool pf_rows = (pf_bytes & 15u) == 0 && (row_bytes_all & 15) == 0 &&
                           ((reinterpret_cast<uintptr_t>(gptr + (int64_t)f0 * D)) & 15) == 0;
      const int n_tiles = (int)ceil_div<int64_t>(s_end - s_begin, R);

      // x and (when given) the forward's bin of my rows, one tile ahead; the gradient rows of the next tile
      // are prefetched into L2 and loaded at the start of their tile
      float xn[IPT];
      int kn[IPT];
      auto fetch = [&](int64_t tt0, int nrows) {
#pragma unroll
        for (int j = 0; j < IPT; ++j) {
          const int r = row_of(j);
          kn[j] = 0;
          xn[j] = 0.f;
          if (pf_live && r < nrows) {
            const int64_t pair = (tt0 + r) * a.F + f0 + pf;
            xn[j] = __ldg(a.x + pair);
            if (a.bin_idx != nullptr)
              kn[j] = bb == 1 ? (int)__ldg(reinterpret_cast<const uint8_t*>(a.bin_idx) + pair)
                    : bb == 2 ? (int)__ldg(reinterpret_cast<const int16_t*>(a.bin_idx) + pair)
                              : __ldg(reinterpret_cast<const int32_t*>(a.bin_idx) + pair);
          }
        }
      };
      auto prefetch_rows = [&](int64_t tt0) {  // gradient rows of the tile at tt0 into L2
        if (!pf_rows || tt0 >= s_end) return;
        const int nsr = (int)min64(R, s_end - tt0);
        const char* gr = reinterpret_cast<const char*>(gptr + (tt0 * a.F + f0) * (int64_t)D);
        for (int s = tid; s < nsr; s += nprod) prefetch_l2_bulk(gr + (int64_t)s * row_bytes_all, pf_bytes);
      };
      fetch(s_begin, (int)min64(R, s_end - s_begin));
      prefetch_rows(s_begin);

      named_sync(1, nprod);  // previous segment done with the tables
      stage_tables_tc<QT>(a, f0, fc, Fc, ts, lgp, sT, sS, sE, sR, sN, tid, nprod);
      for (int i = tid; i < Fc * Bp * 2 * D; i += nprod) spec[i] = 0.0f;
      if (tid == 0) *sFlag = 0;
      f2_t ea0[4], ea1[4];  // epilogue sums of (pf, ph): sum g x and sum g (B), or sum g' (A)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ea0[e] = 0ull;
        ea1[e] = 0ull;
      }
      const float* pvec = nullptr;  // bias (ReLU with bias) or w0 (linear0 terms) of (pf, ph)
      if constexpr (MASK == kMaskReluBias) pvec = a.bias + (int64_t)(f0 + (pf_live ? pf : 0)) * D + 8 * ph;
      if constexpr (LIN) pvec = a.w0 + (int64_t)(f0 + (pf_live ? pf : 0)) * D + 8 * ph;
      named_sync(1, nprod);  // tables staged
      const int pn = sN[pf];
      bool rs_first = true;

      for (int it = 0; it < n_tiles; ++it, ++gtile) {
        const int st = gtile & 1;
        const int64_t t0 = s_begin + (int64_t)it * R;
        const int ns = (int)min64(R, s_end - t0);
        float xc[IPT];
        GRaw<GT, 8> gc[IPT];
        int kc[IPT];
#pragma unroll
        for (int j = 0; j < IPT; ++j) {
          const int r = row_of(j);
          xc[j] = xn[j];
          kc[j] = kn[j];
          if (pf_live && r < ns) {
            ldg_raw<GT, 8>(gc[j], gptr + ((t0 + r) * a.F + f0 + pf) * (int64_t)D + 8 * ph);
          } else {
#pragma unroll
            for (int w = 0; w < GRaw<GT, 8>::kWords; ++w) gc[j].w[w] = 0u;
          }
        }
        if (it + 1 < n_tiles) {
          fetch(t0 + R, (int)min64(R, s_end - t0 - R));
          prefetch_rows(t0 + R);
        }
        // the MMAs of the tile that last used this stage must have finished reading it
        bool ok = wait_empty(st, st ? done1 : done0);
        if (ok) {
          unsigned char* aS = sA + st * a_stage + pg * a_group;
          unsigned char* bS = sB + st * b_stage + pg * b_group;
          float* gxs = sGX + st * (R * C) + cidx * R;
          uint8_t* keys = sKey + st * (R * Fc) + pf * R;
          f2_t pv2[4];
          if constexpr (MASK == kMaskReluBias || LIN) {
            const ulonglong2 v0 = __ldg(reinterpret_cast<const ulonglong2*>(pvec));
            const ulonglong2 v1 = __ldg(reinterpret_cast<const ulonglong2*>(pvec) + 1);
            pv2[0] = v0.x; pv2[1] = v0.y; pv2[2] = v1.x; pv2[3] = v1.y;
          }
#pragma unroll
          for (int j = 0; j < IPT; ++j) {
            const int r = row_of(j);
            const bool valid = r < ns && pf_live;
            const float xv = xc[j];
            int k = 0;
            if (valid) {
              if (a.bin_idx != nullptr) {
                const int kk = kc[j];
                k = kk < 0 ? 0 : (kk >= pn ? pn - 1 : kk);
              } else {
                k = logical_bin(count_le_any(xv, sEf, lgp), pn);
              }
            }
            const float ek = sEf[k], rk = sRf[k];
            const float tq = valid ? quantize<QT>((xv - ek) * rk) : 0.f;
            const bool tie = valid && k > 0 && xv == ek;
            const f2_t t2 = pack2(tq, tq), x2 = pack2(xv, xv), zero2 = 0ull;
            const float* Tk = sTt + k * ts;
            const float* Sk = sSt + k * ts;
            f2_t q2[4];
            f2_t dot2 = 0ull, dw2 = 0ull, nf2 = 0ull;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {  // two halves of 4 columns: fewer live table registers
              const ulonglong2 TT = *reinterpret_cast<const ulonglong2*>(Tk + 4 * hf);
              const ulonglong2 SS = *reinterpret_cast<const ulonglong2*>(Sk + 4 * hf);
#pragma unroll
              for (int e2 = 0; e2 < 2; ++e2) {
                const int e = 2 * hf + e2;
                const f2_t S2 = e2 ? SS.y : SS.x, T2 = e2 ? TT.y : TT.x;
                float g0, g1;
                raw_pair<GT, 8>(gc[j], 2 * e, g0, g1);
                const f2_t g2 = pack2(g0, g1);
                if constexpr (LIN) {
                  dw2 = fma2(g2, pv2[e], dw2);
                  ea0[e] = fma2(g2, x2, ea0[e]);
                  ea1[e] = add2(ea1[e], g2);
                }
                float q0 = g0, q1 = g1;
                if constexpr (MASK != kMaskNone) {
                  float p0, p1;
                  unpack2(fma2(t2, S2, T2), p0, p1);
                  if constexpr (MASK == kMaskReluBias) {
                    round2<QT>(p0, p1);
                    float b0, b1;
                    unpack2(pv2[e], b0, b1);
                    p0 += b0;
                    p1 += b1;
                    q0 = p0 <= 0.f ? 0.f : g0;
                    q1 = p1 <= 0.f ? 0.f : g1;
                  } else {
                    q0 = p0 <= thr ? 0.f : g0;
                    q1 = p1 <= thr ? 0.f : g1;
                  }
                }
                if constexpr (ACCB) ea0[e] = add2(ea0[e], pack2(q0, q1));
                if constexpr (!std::is_same<GT, QT>::value && !std::is_same<QT, float>::value) round2<QT>(q0, q1);
                q2[e] = pack2(q0, q1);
                dot2 = fma2(q2[e], S2, dot2);
                nf2 = fma2(mul2(t2, q2[e]), zero2, nf2);
              }
            }
            float lo, hi;
            unpack2(dot2, lo, hi);
            float gxv = rk * (lo + hi);
            if (tie) {  // edge sub-gradient (x == e_k, k > 0): rare
              const float* Sm = Sk - ts;
              float dm = 0.f;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float a0, a1;
                unpack2(q2[e], a0, a1);
                dm = fmaf(a0, Sm[2 * e], dm);
                dm = fmaf(a1, Sm[2 * e + 1], dm);
              }
              gxv += sRf[k - 1] * dm;
            }
            if constexpr (LIN) {
              unpack2(dw2, lo, hi);
              gxv += lo + hi;
            }
            gxs[r] = valid ? gxv : 0.f;
            f2_t tg2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) tg2[e] = mul2(t2, q2[e]);
            unpack2(nf2, lo, hi);
            if (lo != 0.f || hi != 0.f) {  // a non-finite q(g') or q(t) q(g'): summed outside the MMAs
              float* sp0 = spec + ((int64_t)(pf * Bp + k) * 2) * D + 8 * ph;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float qa[2], ta[2];
                unpack2(q2[e], qa[0], qa[1]);
                unpack2(tg2[e], ta[0], ta[1]);
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                  if (!isfinite(ta[z])) {
                    atomicAdd(sp0 + D + 2 * e + z, ta[z]);
                    ta[z] = 0.f;
                  }
                  if (!isfinite(qa[z])) {
                    atomicAdd(sp0 + 2 * e + z, qa[z]);
                    qa[z] = 0.f;
                  }
                }
                q2[e] = pack2(qa[0], qa[1]);
                tg2[e] = pack2(ta[0], ta[1]);
              }
              *sFlag = 1;
            }
            unsigned char* line = bS + (((bcol + (uint32_t)(r >> 3)) << 7) + ((uint32_t)(r & 7) << 4));
            store_parts<PH>(q2, line, part_stride);
            store_parts<PU>(tg2, line + PH * part_stride, part_stride);
            if (ph == 0) {  // the one of (feature, sample) in A; the one set two tiles ago in this stage cleared
              const uint32_t acolb = (((uint32_t)(r >> 3) << 6) + (uint32_t)(r & 7)) * 2u;
              const int kp = keys[r];
              if (kp != 0xff) *reinterpret_cast<uint16_t*>(aS + arow(kp) + acolb) = 0;
              if (valid) *reinterpret_cast<uint16_t*>(aS + arow(k) + acolb) = (uint16_t)0x3f80u;
              keys[r] = valid ? (uint8_t)k : (uint8_t)0xff;
            }
          }
        }
        tc::fence_proxy_async();
        const bool flush_now = it > 0 && (it % m.flush_tiles) == 0;
        if (flush_now) {  // accumulators hold the tiles since the last flush; the previous tile's MMAs done
          ok = __all_sync(0xffffffffu, ok && wait_empty(st ^ 1, st ? done0 : done1));
          if (ok) {
            tc::fence_after_sync();
            flush(rs_first);
            rs_first = false;
          }
        }
        tc::fence_before_sync();
        if (named_sync_or(1, nprod, !ok)) {
          failed = true;
          break;
        }
        if (tid == 0) mbar_arrive(&full[st]);
        if (st) ++done1;
        else ++done0;
        if (a.grad_x != nullptr) {  // grad_x of the tile: the column blocks' shares in fixed order
          const float* gxs = sGX + st * (R * C);
          for (int r = tid; r < ns; r += nprod) {
            float* dst = a.grad_x + (t0 + r) * a.F + f0;
            for (int f = 0; f < fc; ++f) {
              const float* s = gxs + f * nh * R + r;
              float v = s[0];
              for (int c = 1; c < nh; ++c) v += s[c * R];
              dst[f] = v;
            }
          }
        }
      }
      if (failed) break;
      if constexpr (LIN || ACCB) {  // epilogue sums of this thread, reduced per (feature, column block) below
        float* e = escr + tid * 16;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float v0, v1;
          unpack2(ea0[q], v0, v1);
          e[2 * q] = v0;
          e[2 * q + 1] = v1;
          unpack2(ea1[q], v0, v1);
          e[8 + 2 * q] = v0;
          e[8 + 2 * q + 1] = v1;
        }
      }

      // ---- segment end: last MMAs, final flush, then per unit: non-finite sums, suffix scan over bins,
      // partial rows
      {
        const int stl = (gtile - 1) & 1;
        const bool ok = __all_sync(0xffffffffu, wait_empty(stl, stl ? done1 : done0));
        if (ok) {
          tc::fence_after_sync();
          flush(rs_first);
        }
        tc::fence_before_sync();
        if (named_sync_or(1, nprod, !ok)) {
          failed = true;
          break;
        }
      }
      float* wsb = a.ws + ((int64_t)blockIdx.x * a.max_segs + seg) * ((int64_t)Fc * (B + 3) * D);
#pragma unroll 1
      for (int iu = 0; iu < m.nu; ++iu) {  // every producer thread takes part (named barrier below)
        const int fu = (wid >> 2) + (WP >> 2) * iu;
        const int fgp = fu / nh, fh = fu - fgp * nh;
        const int ffeat = fgp * FM + fslot;
        const bool f_live = slot_used && ffeat < fc;
        const uint32_t rcol = rbase + 16u * (uint32_t)fu;
        float Hacc[8], Uacc[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          Hacc[d] = 0.f;
          Uacc[d] = 0.f;
        }
        if (slot_used) {
          uint32_t h8[8], u8[8];
          tc::tmem_ld8(tlane + rcol, h8);
          tc::tmem_ld8(tlane + rcol + 8, u8);
          tc::wait_ld();
          tc::hold8(h8);
          tc::hold8(u8);
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            Hacc[d] = __uint_as_float(h8[d]);
            Uacc[d] = __uint_as_float(u8[d]);
          }
        }
        if (*sFlag && f_live) {
          const float* sp0 = spec + ((int64_t)(ffeat * Bp + fbin) * 2) * D + 8 * fh;
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            Hacc[d] += __ldcg(sp0 + d);
            Uacc[d] += __ldcg(sp0 + D + d);
          }
        }
        // sum of H over the higher bins: within the warp (lanes = consecutive bins), then the higher
        // lane quarters of the same feature
        float ex[8];
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          float v = __shfl_down_sync(0xffffffffu, Hacc[d], 1);
          if (lane == 31) v = 0.f;
#pragma unroll
          for (int off = 1; off < 32; off <<= 1) {
            const float t = __shfl_down_sync(0xffffffffu, v, off);
            if (lane + off < 32) v += t;
          }
          ex[d] = v;
        }
        if (lane == 0) {
#pragma unroll
          for (int d = 0; d < 8; ++d) sTot[(fu * 4 + sp) * 8 + d] = Hacc[d] + ex[d];
        }
        named_sync(1, nprod);
        {
          const int wps = Bp >> 5;  // lane quarters per feature slot
          const int sp_hi = (fslot + 1) * wps;
          for (int s2 = sp_hi - 1; s2 > sp; --s2) {
#pragma unroll
            for (int d = 0; d < 8; ++d) ex[d] += sTot[(fu * 4 + s2) * 8 + d];
          }
        }
        if (f_live) {
          const int n = sN[ffeat];
          float* rowbase = wsb + (int64_t)ffeat * (B + 3) * D + 8 * fh;
          if (fbin < n) {
            float* dst = rowbase + physical_bin(fbin, n, B) * D;
#pragma unroll
            for (int d = 0; d < 8; ++d) dst[d] = Uacc[d] + ex[d];
          }
          if (fbin >= n - 1 && fbin <= B - 2) {
#pragma unroll
            for (int d = 0; d < 8; ++d) rowbase[fbin * D + d] = 0.f;
          }
          if (!ACCB && fbin == 0) {
#pragma unroll
            for (int d = 0; d < 8; ++d) rowbase[B * D + d] = Hacc[d] + ex[d];
          }
        }
      }
      if constexpr (LIN || ACCB) {
        const int nq = WP / C;  // warps per (feature, column block)
        for (int idx = tid; idx < fc * D; idx += nprod) {
          const int fi = idx / D, d = idx - fi * D;
          const int ci = fi * nh + (d >> 3), dd = d & 7;
          float s0 = 0.f, s1 = 0.f;
          for (int qq = 0; qq < nq; ++qq) {
            const float* src = escr + ((ci + C * qq) * 32) * 16;
            for (int l = 0; l < 32; ++l) {
              s0 += __ldcg(src + l * 16 + dd);
              if constexpr (LIN) s1 += __ldcg(src + l * 16 + 8 + dd);
            }
          }
          float* row = wsb + (int64_t)fi * (B + 3) * D;
          if constexpr (LIN) {
            row[(B + 1) * D + d] = s0;
            row[(B + 2) * D + d] = s1;
          } else {
            row[B * D + d] = s0;
          }
        }
      }
    }
    if (failed) {
      *sAbort = 1;
      if (tid == 0) atomicExch(m.dev_err, 1);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (is_mma_warp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, kTcTmemCols);
  }
}

// Host: geometry (ple_backward.cu) and launch.
bool tc_plan(const BwdArgs& a, int parts_h, int parts_u, int max_warps, TcGeom* m, int* threads, size_t* smem);
int tc_prepare(BwdArgs& a, TcGeom& m, int threads, int* grid);
size_t tc_ws_floats(BwdArgs& a, TcGeom& m, int threads, int* grid);
int bwd_finalize(const BwdArgs& a, int grid, cudaStream_t st);
int backward_kernel_mode();  // 1 sorted kernel (default), 2 tensor-core kernel
constexpr int kTcNotApplicable = -1000;

template <typename QT, typename GT, int MASK, int EPIV>
int launch_bwd_tc_t(BwdArgs a, cudaStream_t st) {
  TcGeom m{};
  int threads = 0, grid = 0;
  size_t smem = 0;
  if (!tc_plan(a, TcParts<QT>::H, TcParts<QT>::U, tc_max_warps(tc_max_regs<GT>()), &m, &threads, &smem))
    return kTcNotApplicable;
  const int prep = tc_prepare(a, m, threads, &grid);
  if (prep != PLE_OK) return prep;
  auto kern = ple_bwd_tc_kernel<QT, GT, MASK, EPIV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(tensor-core backward)");
  kern<<<grid, threads + 32, smem, st>>>(a, m);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    char what[160];
    snprintf(what, sizeof what, "tensor-core backward launch (%d threads, %zu B shared; kernel: %d registers, %d max threads)",
             threads + 32, smem, fa.numRegs, fa.maxThreadsPerBlock);
    return set_cuda_error(e, what);
  }
  return bwd_finalize(a, grid, st);
}

template <typename QT, typename GT>
int launch_bwd_tc_mask(const BwdArgs& a, cudaStream_t st) {
  const bool lin = a.epi == kEpiB && (a.grad_x || a.grad_w0 || a.grad_b0);
  const bool bias = a.epi == kEpiA && a.grad_bias;
  if (a.relu && a.epi == kEpiA)
    return bias ? launch_bwd_tc_t<QT, GT, kMaskReluBias, kEpvBias>(a, st)
                : launch_bwd_tc_t<QT, GT, kMaskReluBias, kEpvNone>(a, st);
  if (a.relu)
    return lin ? launch_bwd_tc_t<QT, GT, kMaskRelu, kEpvLin>(a, st) : launch_bwd_tc_t<QT, GT, kMaskRelu, kEpvNone>(a, st);
  if (lin) return launch_bwd_tc_t<QT, GT, kMaskNone, kEpvLin>(a, st);
  return bias ? launch_bwd_tc_t<QT, GT, kMaskNone, kEpvBias>(a, st) : launch_bwd_tc_t<QT, GT, kMaskNone, kEpvNone>(a, st);
}

// The sorted kernel, or on request (PLE_BACKWARD_KERNEL=tensor) the tensor-core kernel, which covers
// bins <= 128, D a multiple of 8 up to 32 and one feature's parts * D columns in one MMA and fails with
// PLE_ERR_UNSUPPORTED elsewhere.  The sorted kernel is the default: it is the faster of the two on every
// measured configuration.
template <typename QT, typename GT>
int launch_bwd_any(const BwdArgs& a, int vec, cudaStream_t st) {
  if (backward_kernel_mode() == 2) {
    const int rc = launch_bwd_tc_mask<QT, GT>(a, st);
    if (rc != kTcNotApplicable) return rc;
    return set_error(PLE_ERR_UNSUPPORTED, "tensor-core backward: shape not supported");
  }
  return launch_bwd_dtype<QT, GT>(a, vec, st);
}

}  // namespace ple
