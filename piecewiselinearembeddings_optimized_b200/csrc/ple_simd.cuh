// ple_simd.cuh - packed fp32x2 arithmetic, packed low-precision conversions
// and cp.async helpers for sm_100a (inline PTX).
//
// fma/add.rn.f32x2 (PTX ISA 8.6, sm_100+) process two fp32 lanes per
// instruction with the same rounding as two scalar fmaf/__fadd_rn calls, so
// results are bit-identical to the scalar formulation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ple {

typedef unsigned long long f2_t;  // two packed fp32 values (lo = first element)

__device__ __forceinline__ f2_t pack2(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(f2_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// The two 32-bit halves of a packed pair as raw bits, and back.
__device__ __forceinline__ void bits2(f2_t v, uint32_t& lo, uint32_t& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ f2_t from_bits2(uint32_t lo, uint32_t hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2_t add2(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
  f2_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// max(v, 0) propagating NaN (torch.relu semantics).
__device__ __forceinline__ float relu_nan(float v) {
  float d;
  asm("max.NaN.f32 %0, %1, 0f00000000;" : "=f"(d) : "f"(v));
  return d;
}

// Packed round-to-nearest-even conversion of (lo, hi) to a 16-bit pair.
template <typename T> __device__ __forceinline__ unsigned cvt_pack(float lo, float hi);
template <> __device__ __forceinline__ unsigned cvt_pack<__nv_bfloat16>(float lo, float hi) {
  unsigned d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
template <> __device__ __forceinline__ unsigned cvt_pack<__half>(float lo, float hi) {
  unsigned d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Widen a 16-bit pair back to fp32.
template <typename T> __device__ __forceinline__ void widen_pack(unsigned p, float& lo, float& hi);
template <> __device__ __forceinline__ void widen_pack<__nv_bfloat16>(unsigned p, float& lo, float& hi) {
  lo = __uint_as_float(p << 16);
  hi = __uint_as_float(p & 0xffff0000u);
}
template <> __device__ __forceinline__ void widen_pack<__half>(unsigned p, float& lo, float& hi) {
  const __half2 h = *reinterpret_cast<const __half2*>(&p);
  const float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

// Round two fp32 values through T (identity for float).
template <typename T>
__device__ __forceinline__ void round2(float& lo, float& hi) {
  if constexpr (!std::is_same<T, float>::value) widen_pack<T>(cvt_pack<T>(lo, hi), lo, hi);
}

// ---------------------------------------------------------------- shared memory
// 32-bit shared-window address of a pointer into dynamic shared memory.
__device__ __forceinline__ uint32_t shared_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// n packed fp32 pairs at a shared address (16-byte accesses where n is even and `wide`): plain loads for
// tables that do not change while they are read; ordered (volatile) loads and stores for sums that the
// same warp updates in place.
template <int N, bool WIDE>
__device__ __forceinline__ void lds_pairs(unsigned long long (&v)[N], uint32_t addr) {
#pragma unroll
  for (int e = 0; e < N; e += (WIDE ? 2 : 1)) {
    if constexpr (WIDE) asm("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(v[e]), "=l"(v[e + 1]) : "r"(addr + 8 * e));
    else asm("ld.shared.b64 %0, [%1];" : "=l"(v[e]) : "r"(addr + 8 * e));
  }
}
template <int N, bool WIDE>
__device__ __forceinline__ void lds_pairs_ordered(unsigned long long (&v)[N], uint32_t addr) {
#pragma unroll
  for (int e = 0; e < N; e += (WIDE ? 2 : 1)) {
    if constexpr (WIDE)
      asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(v[e]), "=l"(v[e + 1]) : "r"(addr + 8 * e) : "memory");
    else asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v[e]) : "r"(addr + 8 * e) : "memory");
  }
}
template <int N, bool WIDE>
__device__ __forceinline__ void sts_pairs_ordered(uint32_t addr, const unsigned long long (&v)[N]) {
#pragma unroll
  for (int e = 0; e < N; e += (WIDE ? 2 : 1)) {
    if constexpr (WIDE)
      asm volatile("st.shared.v2.b64 [%0], {%1, %2};" ::"r"(addr + 8 * e), "l"(v[e]), "l"(v[e + 1]) : "memory");
    else asm volatile("st.shared.b64 [%0], %1;" ::"r"(addr + 8 * e), "l"(v[e]) : "memory");
  }
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem_src) : "memory");
}
// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

}  // namespace ple
