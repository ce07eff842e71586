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
// Work decomposition.  A CTA owns Fc consecutive features and a contiguous
// sample partition; W_f warps per feature.  Per tile of S_t samples:
//   A  bin search of every (sample, feature) pair, per-(feature, quarter, bin)
//      counts (integer shared atomics: order independent);
//   B  exclusive scan of the counts (bin-major, quarter-minor);
//   C  stable counting sort: each warp ranks its quarter with __match_any_sync,
//      so the sorted order is a pure function of the input;
//   D  walk: a feature's sorted list is cut into G equal contiguous segments;
//      each lane group (nc lanes x VEC elements = one row of D) walks one
//      segment, keeping the active bin's T/S rows and its running H/U sums in
//      registers.  A run that starts inside the segment is flushed to the
//      shared H/U histogram by its only owner; the segment's first run goes
//      to a carry slot.  grad_x is reduced across the nc lanes of the row and
//      scattered to a natural-order shared buffer;
//   E  carries are added in segment order (deterministic), grad_x rows are
//      stored coalesced.
// At the end, per column, a suffix scan over bins turns H/U into grad_W;
// per-partition partials go to the workspace and a finalize kernel sums them
// in partition order.  No floating-point atomics anywhere: bitwise
// deterministic for a given shape.
#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"

namespace ple {

struct BwdLayout {
  float *sT, *sS, *sH, *sU, *sE, *sR, *sGX, *sCarry;
  int2* sEnt;
  uint8_t* sKey;
  int *sN, *sCnt, *sCarryBin;
};

__device__ __forceinline__ BwdLayout bwd_layout(unsigned char* base, const BwdArgs& a, int G) {
  BwdLayout L;
  const int tab = a.B * a.Fc * a.D;
  L.sT = reinterpret_cast<float*>(base);
  L.sS = L.sT + tab;
  L.sH = L.sS + tab;
  L.sU = L.sH + tab;
  L.sCarry = L.sU + tab;                                   // [Fc][G][2][D]
  L.sGX = L.sCarry + a.Fc * G * 2 * a.D;                   // [Fc][S_t]
  L.sEnt = reinterpret_cast<int2*>(L.sGX + a.Fc * a.S_t);  // [Fc][S_t]
  L.sE = reinterpret_cast<float*>(L.sEnt + a.Fc * a.S_t);  // [pow2][Fc]
  L.sR = L.sE + a.pow2 * a.Fc;                             // [B][Fc]
  L.sN = reinterpret_cast<int*>(L.sR + a.B * a.Fc);        // [Fc]
  L.sCnt = L.sN + a.Fc;                                    // [Fc][B][Wf]
  L.sCarryBin = L.sCnt + a.Fc * a.B * a.Wf;                // [Fc][G]
  L.sKey = reinterpret_cast<uint8_t*>(L.sCarryBin + a.Fc * G);  // [Fc][S_t]
  return L;
}

size_t bwd_smem_bytes(const BwdArgs& a, int G) {
  const size_t tab = (size_t)a.B * a.Fc * a.D;
  size_t f = 4 * tab + (size_t)a.Fc * G * 2 * a.D + (size_t)a.Fc * a.S_t;
  size_t bytes = f * 4 + (size_t)a.Fc * a.S_t * 8 + (size_t)a.pow2 * a.Fc * 4 +
                 (size_t)a.B * a.Fc * 4 + (size_t)a.Fc * 4 + (size_t)a.Fc * a.B * a.Wf * 4 +
                 (size_t)a.Fc * G * 4 + (size_t)a.Fc * a.S_t;
  return (bytes + 15) & ~(size_t)15;
}

// Exclusive scan of cnt[0..m) in place by one warp; returns the total.
__device__ __forceinline__ int warp_exclusive_scan(int* cnt, int m, int lane) {
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
  return __shfl_sync(0xffffffffu, incl, 31);
}

// Sum over the nc lanes of a row group (lanes r*nc .. r*nc+nc-1); result in c == 0.
__device__ __forceinline__ float row_reduce(float v, int c, int nc) {
  for (int off = 1; off < nc; off <<= 1) {
    const float o = __shfl_down_sync(0xffffffffu, v, off);
    if (c + off < nc) v += o;
  }
  return v;
}

template <typename QT, typename GT, int VEC>
__global__ void __launch_bounds__(kBwdThreads, VEC >= 8 ? 1 : 2)
ple_bwd_kernel(const BwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int Fc = a.Fc, B = a.B, D = a.D, Wf = a.Wf, S_t = a.S_t;
  const int nc = D / VEC;
  const int Rint = 32 / nc;
  const int G = Wf * Rint;
  BwdLayout L = bwd_layout(smem_raw, a, G);

  const int chunk = blockIdx.x % a.n_chunks;
  const int part = blockIdx.x / a.n_chunks;
  const int f0 = chunk * Fc;
  const int fc = min(Fc, a.F - f0);
  const int64_t s_begin = a.N * part / a.n_parts;
  const int64_t s_end = a.N * (part + 1) / a.n_parts;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int my_i = wid / Wf;          // feature slot of this warp
  const int my_w = wid - my_i * Wf;   // warp rank within the feature
  const int r = lane / nc, c = lane - (lane / nc) * nc;
  const bool grp_live = r < Rint && my_i < fc;
  const int g_seg = my_w * Rint + r;  // segment index within the feature
  const int cd = c * VEC;
  const bool do_gx = a.grad_x != nullptr;
  const GT* gptr = reinterpret_cast<const GT*>(a.g);

  // ---- prologue: tables (same construction as the forward) and zeroed H/U
  for (int i = tid; i < Fc; i += nthr) {
    int n = i < fc ? a.n_bins[f0 + i] : 1;
    L.sN[i] = n < 1 ? 1 : (n > B ? B : n);
  }
  __syncthreads();
  for (int idx = tid; idx < a.pow2 * Fc; idx += nthr) {
    const int j = idx / Fc, i = idx - j * Fc;
    float e = __int_as_float(0x7f800000);
    if (i < fc && j <= L.sN[i]) e = a.edges[(int64_t)(f0 + i) * (B + 1) + j];
    L.sE[idx] = e;
  }
  for (int idx = tid; idx < B * Fc; idx += nthr) {
    const int j = idx / Fc, i = idx - j * Fc;
    L.sR[idx] = (i < fc && j < L.sN[i]) ? a.inv_w[(int64_t)(f0 + i) * B + j] : 0.0f;
  }
  for (int idx = tid; idx < B * Fc * D; idx += nthr) {
    L.sH[idx] = 0.0f;
    L.sU[idx] = 0.0f;
    L.sS[idx] = 0.0f;
  }
  __syncthreads();
  const float* Wc = a.W + (int64_t)f0 * B * D;
  for (int idx = tid; idx < fc * B * D; idx += nthr) {
    const int i = idx / (B * D);
    const int rem = idx - i * B * D;
    const int p = rem / D, d = rem - p * D;
    const int n = L.sN[i];
    const int lg = (p == B - 1) ? n - 1 : (p < n - 1 ? p : -1);
    if (lg >= 0) L.sS[(lg * Fc + i) * D + d] = quantize<QT>(Wc[idx]);
  }
  __syncthreads();
  for (int col = tid; col < Fc * D; col += nthr) {
    const int i = col / D, d = col - i * D;
    const int n = L.sN[i];
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int o = (j * Fc + i) * D + d;
      L.sT[o] = acc;
      acc += L.sS[o];
    }
  }

  // per-lane epilogue parameters and linear0 accumulators
  FV<VEC> pw0, pbias, acc_w0, acc_b0;
#pragma unroll
  for (int e = 0; e < VEC; ++e) { pw0.v[e] = 0.f; pbias.v[e] = 0.f; acc_w0.v[e] = 0.f; acc_b0.v[e] = 0.f; }
  if (grp_live) {
    const int64_t po = (int64_t)(f0 + my_i) * D + cd;
    if (a.epi == kEpiA) pbias = ldg_f32vec<float, VEC>(a.bias + po);
    if (a.epi == kEpiB) pw0 = ldg_f32vec<float, VEC>(a.w0 + po);
  }
  __syncthreads();

  const int n_i = grp_live ? L.sN[my_i] : 1;
  for (int64_t t0 = s_begin; t0 < s_end; t0 += S_t) {
    const int ns = (int)min64(S_t, s_end - t0);
    const int qlen = (ns + Wf - 1) / Wf;
    // prefetch the next tile's gradient rows of this chunk into L2
    {
      const int64_t nt0 = t0 + S_t;
      if (nt0 < s_end) {
        const int nns = (int)min64(S_t, s_end - nt0);
        const int row_bytes = fc * D * (int)sizeof(GT);
        const int lines = row_bytes / 128 + 2;
        for (int q = tid; q < nns * lines; q += nthr) {
          const int s = q / lines, l = q - s * lines;
          const uintptr_t rp = reinterpret_cast<uintptr_t>(gptr + ((nt0 + s) * a.F + f0) * D);
          const uintptr_t pp = (rp & ~(uintptr_t)127) + (uintptr_t)l * 128;
          if (pp < rp + row_bytes) asm volatile("prefetch.global.L2 [%0];" ::"l"(pp));
        }
      }
    }
    // ---- A: bins, counts, natural-order x
    for (int idx = tid; idx < Fc * B * Wf; idx += nthr) L.sCnt[idx] = 0;
    __syncthreads();
    for (int p = tid; p < ns * Fc; p += nthr) {
      const int s = p / Fc, i = p - s * Fc;
      if (i < fc) {
        const float xv = a.x[(t0 + s) * a.F + f0 + i];
        const int k = logical_bin(edge_count(xv, L.sE, Fc, i, a.pow2), L.sN[i]);
        L.sKey[i * S_t + s] = (uint8_t)k;
        L.sGX[i * S_t + s] = xv;
        atomicAdd(&L.sCnt[(i * B + k) * Wf + s / qlen], 1);
      }
    }
    __syncthreads();
    // ---- B: exclusive scan per feature (bin-major, quarter-minor)
    for (int i = wid; i < fc; i += nthr / 32) warp_exclusive_scan(L.sCnt + i * B * Wf, B * Wf, lane);
    __syncthreads();
    // ---- C: stable scatter of each quarter into sorted order
    if (my_i < fc) {
      const int q = my_w;
      const int lo = q * qlen, hi = min(lo + qlen, ns);
      for (int base = lo; base < hi; base += 32) {
        const int s = base + lane;
        const bool v = s < hi;
        const unsigned act = __ballot_sync(0xffffffffu, v);
        if (v) {
          const int k = L.sKey[my_i * S_t + s];
          const unsigned peers = __match_any_sync(act, k);
          const int leader = __ffs(peers) - 1;
          const int rank = __popc(peers & ((1u << lane) - 1u));
          int* cur = &L.sCnt[(my_i * B + k) * Wf + q];
          int pos0 = 0;
          if (lane == leader) pos0 = *cur;
          pos0 = __shfl_sync(peers, pos0, leader);
          if (lane == leader) *cur = pos0 + __popc(peers);
          const float xv = L.sGX[my_i * S_t + s];
          L.sEnt[my_i * S_t + pos0 + rank] = make_int2(__float_as_int(xv), s | (k << 16));
        }
        __syncwarp();
      }
    }
    __syncthreads();
    // ---- D: segmented walk
    if (my_i < fc) {
      const int seg_lo = (int)((int64_t)g_seg * ns / G);
      const int seg_hi = (int)((int64_t)(g_seg + 1) * ns / G);
      const int my_len = grp_live ? seg_hi - seg_lo : 0;
      // uniform trip count for the warp (segments differ by at most one)
      int trips = my_len;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) trips = max(trips, __shfl_xor_sync(0xffffffffu, trips, off));
      int k_cur = -1;
      bool first_run = true;
      float e_k = 0.f, r_k = 0.f, r_km1 = 0.f;
      FV<VEC> Tk, Sk, Skm1, Hrun, Urun;
#pragma unroll
      for (int e = 0; e < VEC; ++e) { Tk.v[e] = Sk.v[e] = Skm1.v[e] = Hrun.v[e] = Urun.v[e] = 0.f; }
      float* carry = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
      if (grp_live && c == 0) L.sCarryBin[my_i * G + g_seg] = -1;
      for (int step = 0; step < trips; ++step) {
        const bool live = step < my_len;
        int2 ent = make_int2(0, 0);
        int k = k_cur;
        if (live) {
          ent = L.sEnt[my_i * S_t + seg_lo + step];
          k = ent.y >> 16;
        }
        if (live && k != k_cur) {
          if (k_cur >= 0) {
            if (first_run) {
              sts<VEC>(carry, Hrun);
              sts<VEC>(carry + D, Urun);
              if (c == 0) L.sCarryBin[my_i * G + g_seg] = k_cur;
            } else {
              float* h = L.sH + (k_cur * Fc + my_i) * D + cd;
              float* u = L.sU + (k_cur * Fc + my_i) * D + cd;
              FV<VEC> hv = lds<VEC>(h), uv = lds<VEC>(u);
#pragma unroll
              for (int e = 0; e < VEC; ++e) { hv.v[e] += Hrun.v[e]; uv.v[e] += Urun.v[e]; }
              sts<VEC>(h, hv);
              sts<VEC>(u, uv);
            }
            first_run = false;
          }
          k_cur = k;
          const int to = (k * Fc + my_i) * D + cd;
          Tk = lds<VEC>(L.sT + to);
          Sk = lds<VEC>(L.sS + to);
          e_k = L.sE[k * Fc + my_i];
          r_k = L.sR[k * Fc + my_i];
          if (k > 0) {
            Skm1 = lds<VEC>(L.sS + to - Fc * D);
            r_km1 = L.sR[(k - 1) * Fc + my_i];
          }
#pragma unroll
          for (int e = 0; e < VEC; ++e) { Hrun.v[e] = 0.f; Urun.v[e] = 0.f; }
        }
        float gx = 0.f;
        int s = 0;
        if (live) {
          const float xv = __int_as_float(ent.x);
          s = ent.y & 0xffff;
          const float t = (xv - e_k) * r_k;
          const float tq = quantize<QT>(t);
          const bool edge_tie = (k > 0) && (xv == e_k);
          const FV<VEC> gv = ldg_vec<GT, VEC>(gptr + ((t0 + s) * a.F + f0 + my_i) * D + cd);
          float dot = 0.f, dot_prev = 0.f, dot_w0 = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            float gp = gv.v[e];
            if (a.relu) {
              float z = quantize<QT>(fmaf(tq, Sk.v[e], Tk.v[e]));
              if (a.epi == kEpiA) z += pbias.v[e];
              gp = z > 0.0f ? gp : 0.0f;
            }
            float gq = gp;
            if constexpr (!std::is_same<GT, QT>::value) gq = quantize<QT>(gp);
            Hrun.v[e] += gq;
            Urun.v[e] = fmaf(tq, gq, Urun.v[e]);
            dot = fmaf(gq, Sk.v[e], dot);
            dot_prev = fmaf(gq, Skm1.v[e], dot_prev);
            if (a.epi == kEpiB) {
              acc_w0.v[e] = fmaf(gv.v[e], xv, acc_w0.v[e]);
              acc_b0.v[e] += gv.v[e];
              dot_w0 = fmaf(gv.v[e], pw0.v[e], dot_w0);
            }
          }
          gx = r_k * dot + (edge_tie ? r_km1 * dot_prev : 0.f) + dot_w0;
        }
        if (do_gx) {
          gx = row_reduce(gx, c, nc);
          if (live && c == 0) L.sGX[my_i * S_t + s] = gx;
        }
      }
      // flush the segment's last run
      if (grp_live && k_cur >= 0) {
        if (first_run) {
          sts<VEC>(carry, Hrun);
          sts<VEC>(carry + D, Urun);
          if (c == 0) L.sCarryBin[my_i * G + g_seg] = k_cur;
        } else {
          float* h = L.sH + (k_cur * Fc + my_i) * D + cd;
          float* u = L.sU + (k_cur * Fc + my_i) * D + cd;
          FV<VEC> hv = lds<VEC>(h), uv = lds<VEC>(u);
#pragma unroll
          for (int e = 0; e < VEC; ++e) { hv.v[e] += Hrun.v[e]; uv.v[e] += Urun.v[e]; }
          sts<VEC>(h, hv);
          sts<VEC>(u, uv);
        }
      }
    }
    __syncthreads();
    // ---- E: carries in segment order; grad_x rows
    for (int colx = tid; colx < fc * D; colx += nthr) {
      const int i = colx / D, d = colx - i * D;
      for (int g = 0; g < G; ++g) {
        const int kb = L.sCarryBin[i * G + g];
        if (kb >= 0) {
          const float* cp = L.sCarry + ((i * G + g) * 2) * D + d;
          L.sH[(kb * Fc + i) * D + d] += cp[0];
          L.sU[(kb * Fc + i) * D + d] += cp[D];
        }
      }
    }
    if (do_gx) {
      for (int p = tid; p < ns * Fc; p += nthr) {
        const int s = p / Fc, i = p - s * Fc;
        if (i < fc) a.grad_x[(t0 + s) * a.F + f0 + i] = L.sGX[i * S_t + s];
      }
    }
    __syncthreads();
  }

  // ---- F: linear0 partials (fixed segment order) and grad_W suffix scan
  float* ws = a.ws + (int64_t)part * a.F * (B + 3) * D;
  if (a.epi == kEpiB) {
    if (grp_live) {
      float* cp = L.sCarry + ((my_i * G + g_seg) * 2) * D + cd;
      sts<VEC>(cp, acc_w0);
      sts<VEC>(cp + D, acc_b0);
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
      float* row = ws + (int64_t)(f0 + i) * (B + 3) * D;
      row[(B + 1) * D + d] = sw;
      row[(B + 2) * D + d] = sb;
    }
  }
  for (int colx = tid; colx < fc * D; colx += nthr) {
    const int i = colx / D, d = colx - i * D;
    const int n = L.sN[i];
    float* row = ws + (int64_t)(f0 + i) * (B + 3) * D;
    float suffix = 0.f;
    for (int j = n - 1; j >= 0; --j) {
      const int o = (j * Fc + i) * D + d;
      const int phys = physical_bin(j, n, B);
      row[phys * D + d] = L.sU[o] + suffix;
      suffix += L.sH[o];
    }
    for (int p = n - 1; p < B - 1; ++p) row[p * D + d] = 0.f;  // padding rows
    row[B * D + d] = suffix;                                    // sum_b g' (bias grad)
  }
  (void)n_i;
}

// Sum the per-partition partials in partition order.
__global__ void ple_bwd_finalize_kernel(const BwdArgs a) {
  const int B = a.B, D = a.D;
  const int64_t rows = (int64_t)a.F * (B + 3) * D;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < rows;
       idx += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < a.n_parts; ++p) s += a.ws[p * rows + idx];
    const int64_t f = idx / ((int64_t)(B + 3) * D);
    const int64_t rem = idx - f * (B + 3) * D;
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

// ------------------------------------------------------------------ launch
// Chunk / tile plan: 16 warps per CTA split as Fc features x Wf warps; the
// largest tile whose shared memory allows two resident CTAs (one CTA when the
// tables alone are too large).  Shared by the workspace query and the launch.
static bool bwd_plan(BwdArgs& a, int vec, size_t* smem_out, int* ctas_per_sm) {
  const int nc = a.D / vec;
  const int G_per_warp = 32 / nc;
  int pow2 = 1;
  while (pow2 < a.B + 1) pow2 <<= 1;
  a.pow2 = pow2;
  const size_t optin = device_max_smem_optin();
  for (int want = 2; want >= 1; --want) {
    const size_t budget = want == 2 ? kBwdSmemTwoCtas : optin;
    for (int Fc = 4; Fc >= 1; Fc >>= 1) {
      if (Fc / 2 >= a.F && Fc > 1) continue;
      for (int S_t = kBwdTile; S_t >= 128; S_t >>= 1) {
        a.Fc = Fc;
        a.Wf = kBwdThreads / 32 / Fc;
        a.S_t = S_t;
        const size_t smem = bwd_smem_bytes(a, a.Wf * G_per_warp);
        if (smem <= budget) {
          *smem_out = smem;
          *ctas_per_sm = want;
          a.n_chunks = (int)ceil_div<int64_t>(a.F, a.Fc);
          int64_t parts = (int64_t)device_sm_count() * want / a.n_chunks;
          const int64_t max_by_n = ceil_div<int64_t>(a.N, 64);
          parts = parts < 1 ? 1 : parts;
          parts = parts > max_by_n ? max_by_n : parts;
          a.n_parts = (int)parts;
          return true;
        }
      }
    }
  }
  return false;
}

int backward_vec(int64_t D);

size_t backward_workspace_bytes(int64_t N, int64_t F, int64_t B, int64_t D) {
  BwdArgs a{};
  a.N = N; a.F = (int)F; a.B = (int)B; a.D = (int)D;
  size_t smem = 0;
  int per = 0;
  if (!bwd_plan(a, backward_vec(D), &smem, &per)) return 0;
  return (size_t)a.n_parts * (size_t)F * (size_t)(B + 3) * (size_t)D * sizeof(float);
}

template <typename QT, typename GT, int VEC>
static int launch_bwd_t(BwdArgs a, cudaStream_t st) {
  size_t smem = 0;
  int want = 0;
  if (!bwd_plan(a, VEC, &smem, &want))
    return set_error(PLE_ERR_UNSUPPORTED, "backward: tables do not fit in shared memory");
  auto kern = ple_bwd_kernel<QT, GT, VEC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kBwdThreads, smem);
  if (e != cudaSuccess) return set_cuda_error(e, "occupancy(backward)");
  if (per_sm < 1) return set_error(PLE_ERR_UNSUPPORTED, "backward: no resident CTA fits");
  if (per_sm < want) {
    // fewer resident CTAs than planned (registers): shrink the partition count
    int64_t parts = (int64_t)device_sm_count() * per_sm / a.n_chunks;
    a.n_parts = (int)(parts < 1 ? 1 : (parts < a.n_parts ? parts : a.n_parts));
  }
  if ((size_t)a.n_parts * a.F * (a.B + 3) * a.D * sizeof(float) > a.ws_bytes)
    return set_error(PLE_ERR_WORKSPACE, "backward: workspace smaller than ple_backward_workspace_size()");
  const int64_t grid = (int64_t)a.n_chunks * a.n_parts;
  if (grid > 0x7fffffff) return set_error(PLE_ERR_OVERFLOW, "backward grid too large");
  kern<<<(unsigned)grid, kBwdThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward launch");
  const int64_t rows = (int64_t)a.F * (a.B + 3) * a.D;
  const int fin_blocks = (int)min64(ceil_div<int64_t>(rows, 256), 4L * device_sm_count());
  ple_bwd_finalize_kernel<<<fin_blocks, 256, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward finalize launch");
  return PLE_OK;
}

template <typename QT, typename GT>
static int launch_bwd_vec(const BwdArgs& a, int vec, cudaStream_t st) {
  switch (vec) {
    case 8: return launch_bwd_t<QT, GT, 8>(a, st);
    case 4: return launch_bwd_t<QT, GT, 4>(a, st);
    case 2: return launch_bwd_t<QT, GT, 2>(a, st);
    default: return launch_bwd_t<QT, GT, 1>(a, st);
  }
}

int launch_backward(BwdArgs a, int compute_dtype, int grad_dtype, int vec, cudaStream_t st) {
  const int q = compute_dtype, g = grad_dtype;
  if (q == PLE_DTYPE_F32 && g == PLE_DTYPE_F32) return launch_bwd_vec<float, float>(a, vec, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_BF16) return launch_bwd_vec<__nv_bfloat16, __nv_bfloat16>(a, vec, st);
  if (q == PLE_DTYPE_BF16 && g == PLE_DTYPE_F32) return launch_bwd_vec<__nv_bfloat16, float>(a, vec, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F16) return launch_bwd_vec<__half, __half>(a, vec, st);
  if (q == PLE_DTYPE_F16 && g == PLE_DTYPE_F32) return launch_bwd_vec<__half, float>(a, vec, st);
  return set_error(PLE_ERR_UNSUPPORTED, "backward: unsupported (compute, grad) dtype pair");
}

}  // namespace ple
