// ple_common.cuh - device helpers shared by the PLE kernels (sm_100a).
//
// Semantics follow the reference's csrc/common.cuh:
//   * bin search: k = clamp(searchsorted(e[0..n], x, right) - 1, 0, n - 1), NaN -> n - 1
//     (find_logical_bin_right, common.cuh:27-63);
//   * physical row of logical bin k: B - 1 for the last real bin, k otherwise
//     (physical_bin_index, common.cuh:66-78);
//   * quantize<T>: round through T and back to fp32 (quantize_to_float,
//     common.cuh:81-96) to emulate autocast's low-precision matmul inputs.
// The implementations are this project's own: the search is a branchless
// power-of-two descent over a transposed shared-memory edge table.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ple {

constexpr int kMaxD = 64;  // d_embedding limit of the module (module.py:47-49)

// ---------------------------------------------------------------- dtypes
template <typename T> struct Dt;
template <> struct Dt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ float quantize(float v) {
  return Dt<T>::to_f(Dt<T>::from_f(v));
}
template <>
__device__ __forceinline__ float quantize<float>(float v) {
  return v;
}

// ---------------------------------------------------------------- vectors
template <int VEC> struct FV;
template <> struct FV<1> { float v[1]; };
template <> struct FV<2> { float v[2]; };
template <> struct FV<4> { float v[4]; };
template <> struct FV<8> { float v[8]; };

template <int VEC>
__device__ __forceinline__ FV<VEC> lds(const float* p) {
  FV<VEC> r;
  if constexpr (VEC == 8) {
    float4 t = *reinterpret_cast<const float4*>(p);
    float4 u = *reinterpret_cast<const float4*>(p + 4);
    r.v[0] = t.x; r.v[1] = t.y; r.v[2] = t.z; r.v[3] = t.w;
    r.v[4] = u.x; r.v[5] = u.y; r.v[6] = u.z; r.v[7] = u.w;
  } else if constexpr (VEC == 4) {
    float4 t = *reinterpret_cast<const float4*>(p);
    r.v[0] = t.x; r.v[1] = t.y; r.v[2] = t.z; r.v[3] = t.w;
  } else if constexpr (VEC == 2) {
    float2 t = *reinterpret_cast<const float2*>(p);
    r.v[0] = t.x; r.v[1] = t.y;
  } else {
    r.v[0] = *p;
  }
  return r;
}

template <int VEC>
__device__ __forceinline__ void sts(float* p, const FV<VEC>& r) {
  if constexpr (VEC == 8) {
    *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(r.v[4], r.v[5], r.v[6], r.v[7]);
  } else if constexpr (VEC == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r.v[0], r.v[1]);
  } else {
    *p = r.v[0];
  }
}

template <typename T, int VEC>
__device__ __forceinline__ FV<VEC> ldg_f32vec(const float* p) {
  FV<VEC> r;
  if constexpr (VEC == 8) {
    float4 t = __ldg(reinterpret_cast<const float4*>(p));
    float4 u = __ldg(reinterpret_cast<const float4*>(p + 4));
    r.v[0] = t.x; r.v[1] = t.y; r.v[2] = t.z; r.v[3] = t.w;
    r.v[4] = u.x; r.v[5] = u.y; r.v[6] = u.z; r.v[7] = u.w;
  } else if constexpr (VEC == 4) {
    float4 t = __ldg(reinterpret_cast<const float4*>(p));
    r.v[0] = t.x; r.v[1] = t.y; r.v[2] = t.z; r.v[3] = t.w;
  } else if constexpr (VEC == 2) {
    float2 t = __ldg(reinterpret_cast<const float2*>(p));
    r.v[0] = t.x; r.v[1] = t.y;
  } else {
    r.v[0] = __ldg(p);
  }
  return r;
}

// Global load of VEC elements of T, widened to fp32.
template <typename T, int VEC>
__device__ __forceinline__ FV<VEC> ldg_vec(const T* p) {
  FV<VEC> r;
  if constexpr (sizeof(T) == 4) {
    r = ldg_f32vec<T, VEC>(reinterpret_cast<const float*>(p));
  } else if constexpr (VEC == 8) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) r.v[e] = Dt<T>::to_f(h[e]);
  } else if constexpr (VEC == 4) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) r.v[e] = Dt<T>::to_f(h[e]);
  } else if constexpr (VEC == 2) {
    unsigned u = __ldg(reinterpret_cast<const unsigned*>(p));
    const T* h = reinterpret_cast<const T*>(&u);
    r.v[0] = Dt<T>::to_f(h[0]);
    r.v[1] = Dt<T>::to_f(h[1]);
  } else {
    r.v[0] = Dt<T>::to_f(p[0]);
  }
  return r;
}

// Streaming (evict-first) global store of VEC fp32 values converted to T.
template <typename T, int VEC>
__device__ __forceinline__ void stg_stream(T* p, const FV<VEC>& r) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (VEC == 4) {
      __stcs(reinterpret_cast<float4*>(p), make_float4(r.v[0], r.v[1], r.v[2], r.v[3]));
    } else if constexpr (VEC == 2) {
      __stcs(reinterpret_cast<float2*>(p), make_float2(r.v[0], r.v[1]));
    } else {
      __stcs(reinterpret_cast<float*>(p), r.v[0]);
    }
  } else if constexpr (VEC == 4) {
    T h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = Dt<T>::from_f(r.v[e]);
    __stcs(reinterpret_cast<uint2*>(p), *reinterpret_cast<uint2*>(h));
  } else if constexpr (VEC == 2) {
    T h[2] = {Dt<T>::from_f(r.v[0]), Dt<T>::from_f(r.v[1])};
    __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<unsigned*>(h));
  } else {
    p[0] = Dt<T>::from_f(r.v[0]);
  }
}

// ---------------------------------------------------------------- bins
// Count of edges e_j (j < kPow, column `i` of the transposed table sE[j * ld + i])
// with !(x < e_j); the table is ascending with +inf past each feature's last
// real edge, so the predicate holds on a prefix (all of it for NaN or +inf).
__device__ __forceinline__ int edge_count(float x, const float* sE, int ld, int i, int pow2) {
  int base = 0;
  for (int half = pow2 >> 1; half > 0; half >>= 1) {
    if (!(x < sE[(base + half - 1) * ld + i])) base += half;
  }
  if (!(x < sE[base * ld + i])) base += 1;
  return base;
}

// Logical bin: clamp(count - 1, 0, n - 1).
__device__ __forceinline__ int logical_bin(int count, int n_real) {
  int k = count - 1;
  k = k < 0 ? 0 : k;
  return k > n_real - 1 ? n_real - 1 : k;
}

__host__ __device__ __forceinline__ int physical_bin(int k, int n_real, int max_bins) {
  return k == n_real - 1 ? max_bins - 1 : k;
}

// ReLU with torch semantics (NaN passes through).
__device__ __forceinline__ float relu_f(float v) { return v <= 0.0f ? 0.0f : v; }

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

template <typename T>
__host__ __device__ __forceinline__ T ceil_div(T a, T b) {
  return (a + b - 1) / b;
}

}  // namespace ple
