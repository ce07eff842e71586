// ple_fwd_math.cuh - the forward's per-element arithmetic, shared by the fused
// forward (ple_forward.cu) and the forward fused into a consumer Linear
// (ple_linear.cu), so that both produce bitwise-identical embeddings.
#pragma once

#include <type_traits>

#include "ple_common.cuh"
#include "ple_internal.h"
#include "ple_simd.cuh"

namespace ple {

// Count of edges e_j (j < pow2) of one feature row with !(x < e_j); the row is
// ascending with +inf past the last real edge (prefix predicate).
__device__ __forceinline__ int edge_count_row(float x, const float* row, int pow2) {
  int base = 0;
  for (int half = pow2 >> 1; half > 0; half >>= 1) base += !(x < row[base + half - 1]) ? half : 0;
  return base + (!(x < row[base]) ? 1 : 0);
}

// Count of the 2^L - 1 ascending keys with !(x < key): L unrolled probes.
// With keys = a feature's interior edges e_1 .. e_{n-1} followed by +inf, the
// count capped at n - 1 is the reference's clamped right-sided bin
// (find_logical_bin_right, common.cuh:27-63): x below e_1 (including below
// e_0) counts no key, x at or above e_{n-1} counts n - 1, and NaN counts every
// key (n - 1 after the cap), as does +inf.
template <int L>
__device__ __forceinline__ int key_count(float x, const float* keys) {
  int p = 0;
#pragma unroll
  for (int h = (1 << L) >> 1; h > 0; h >>= 1)
    if (!(x < keys[p + h - 1])) p += h;
  return p;
}

// y = epilogue(q(fma(tq, S, T))) for VEC elements.  q() rounds x_ple through
// QT as the reference's low-precision output cast does; when the result is
// itself stored in a 16-bit type after a linear0 add (epilogue B), x_ple is
// rounded only once, at the store (at most one unit in the last place of the
// 16-bit result away from rounding twice).
template <typename QT, typename OT, int VEC, int EPI, bool RELU>
__device__ __forceinline__ FV<VEC> fwd_chunk(float tq, const FV<VEC>& T, const FV<VEC>& S, float xv,
                                             const FV<VEC>& ep0, const FV<VEC>& ep1) {
  constexpr bool kInnerRound =
      !std::is_same<QT, float>::value && (EPI == kEpiA || std::is_same<OT, float>::value);
  FV<VEC> y;
  if constexpr (VEC >= 2) {
    const f2_t t2 = pack2(tq, tq);
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      float lo, hi;
      unpack2(fma2(t2, pack2(S.v[e], S.v[e + 1]), pack2(T.v[e], T.v[e + 1])), lo, hi);
      y.v[e] = lo;
      y.v[e + 1] = hi;
    }
  } else {
    y.v[0] = fmaf(tq, S.v[0], T.v[0]);
  }
  if constexpr (kInnerRound) {
    if constexpr (VEC >= 2) {
#pragma unroll
      for (int e = 0; e < VEC; e += 2) round2<QT>(y.v[e], y.v[e + 1]);
    } else {
      y.v[0] = quantize<QT>(y.v[0]);
    }
  }
  if constexpr (VEC >= 2) {
    // the epilogue on packed pairs (fma/add.rn.f32x2 round like the scalar forms)
    const f2_t x2 = pack2(xv, xv);
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      f2_t v = pack2(y.v[e], y.v[e + 1]);
      if constexpr (EPI == kEpiA) v = add2(v, pack2(ep0.v[e], ep0.v[e + 1]));
      if constexpr (RELU) {
        float lo, hi;
        unpack2(v, lo, hi);
        v = pack2(relu_nan(lo), relu_nan(hi));
      }
      if constexpr (EPI == kEpiB) v = add2(fma2(x2, pack2(ep0.v[e], ep0.v[e + 1]), pack2(ep1.v[e], ep1.v[e + 1])), v);
      unpack2(v, y.v[e], y.v[e + 1]);
    }
  } else {
    float v = y.v[0];
    if constexpr (EPI == kEpiA) v += ep0.v[0];
    if constexpr (RELU) v = relu_nan(v);
    if constexpr (EPI == kEpiB) v = fmaf(xv, ep0.v[0], ep1.v[0]) + v;
    y.v[0] = v;
  }
  return y;
}

}  // namespace ple
