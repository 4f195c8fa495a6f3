// Shared device helpers for the SSA sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ssa_b200.h"

namespace ssa {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// element loads: every kernel computes in fp32
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Load 8 consecutive elements (16 B for 16-bit types, 32 B for fp32) as fp32.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ---------------------------------------------------------------------------
// ordering keys
// ---------------------------------------------------------------------------
// Order-preserving map float -> uint32 (larger float -> larger key);
// -0.0 is folded into +0.0 so that the two compare equal, as floats do.
__device__ __forceinline__ uint32_t float_key(float x) {
  uint32_t u = __float_as_uint(x + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit ranking key of (score, index): larger score first, then lower index.
__device__ __forceinline__ uint64_t rank_key(float score, uint32_t idx) {
  return (static_cast<uint64_t>(float_key(score)) << 32) | static_cast<uint64_t>(~idx);
}
__device__ __forceinline__ uint32_t rank_key_index(uint64_t key) {
  return ~static_cast<uint32_t>(key & 0xffffffffull);
}

__device__ __forceinline__ float float_from_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

// ---------------------------------------------------------------------------
// Sorted top-K list kept in registers by one thread (K small, static indices),
// ordered by (score desc, index asc).  Entries are 64-bit ranking keys
// rank_key(score, index), compared as integers: keys are unique, so the order
// is total and the tie rule (lower index first) holds whatever the order in
// which elements are pushed.  Key 0 marks an empty slot (below every real key).
// `thr` caches the K-th score as a float for a cheap pre-filter: an element
// can enter only if score >= thr.
// ---------------------------------------------------------------------------
template <int K>
struct TopList {
  uint64_t key[K];
  float thr;
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int t = 0; t < K; ++t) key[t] = 0ull;
    thr = -INFINITY;
  }
  __device__ __forceinline__ void insert_key(uint64_t kv) {
    uint64_t c = kv;
#pragma unroll
    for (int t = 0; t < K; ++t) {
      const uint64_t cur = key[t];
      const bool take = c > cur;
      key[t] = take ? c : cur;
      c = take ? cur : c;
    }
    thr = key[K - 1] ? float_from_key(static_cast<uint32_t>(key[K - 1] >> 32)) : -INFINITY;
  }
  // Offer (score, idx); -0.0 is folded into +0.0 by rank_key.
  __device__ __forceinline__ void push(float score, uint32_t idx) {
    if (score >= thr) {
      const uint64_t kv = rank_key(score, idx);
      if (kv > key[K - 1]) insert_key(kv);
    }
  }
  __device__ __forceinline__ int32_t index(int t) const {
    return key[t] ? static_cast<int32_t>(rank_key_index(key[t])) : -1;
  }
};

__device__ __forceinline__ void set_status(int32_t* status, int32_t bits) {
  if (status) atomicOr(status, bits);
}

// Codes can come from the caller (ssa_build_index, ssa_select_candidates,
// ssa_route_with_key_codes).  One outside [0, n_codes) is flagged and read as
// code 0, so that no input can make the index kernels address memory outside
// the histogram, the offsets or the bucket table.
__device__ __forceinline__ int checked_code(int c, int n_codes, int32_t* status) {
  if (static_cast<unsigned>(c) < static_cast<unsigned>(n_codes)) return c;
  set_status(status, SSA_DEVICE_BAD_CODE);
  return 0;
}

__host__ __device__ constexpr inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace ssa
