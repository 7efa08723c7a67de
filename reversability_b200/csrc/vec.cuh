// Vector load/store helpers: V consecutive elements of T converted to/from fp32,
// moved with the widest aligned transaction (16 B where possible).
#pragma once
#include "common.cuh"

namespace rk {

template <typename T, int V>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[V]) {
  constexpr int bytes = (int)sizeof(T) * V;
  if constexpr (bytes % 16 == 0) {
    constexpr int n = bytes / 16;
    constexpr int per = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < n; ++i) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + i);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < per; ++j) out[i * per + j] = Dt<T>::to_f(e[j]);
    }
  } else if constexpr (bytes == 8) {
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = Dt<T>::to_f(e[j]);
  } else if constexpr (bytes == 4) {
    unsigned int raw = __ldg(reinterpret_cast<const unsigned int*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = Dt<T>::to_f(e[j]);
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = Dt<T>::to_f(p[j]);
  }
}

template <typename T, int V>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&in)[V]) {
  constexpr int bytes = (int)sizeof(T) * V;
  if constexpr (bytes % 16 == 0) {
    constexpr int n = bytes / 16;
    constexpr int per = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < n; ++i) {
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int j = 0; j < per; ++j) e[j] = Dt<T>::from_f(in[i * per + j]);
      reinterpret_cast<uint4*>(p)[i] = raw;
    }
  } else if constexpr (bytes == 8) {
    uint2 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int j = 0; j < V; ++j) e[j] = Dt<T>::from_f(in[j]);
    *reinterpret_cast<uint2*>(p) = raw;
  } else if constexpr (bytes == 4) {
    unsigned int raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int j = 0; j < V; ++j) e[j] = Dt<T>::from_f(in[j]);
    *reinterpret_cast<unsigned int*>(p) = raw;
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) p[j] = Dt<T>::from_f(in[j]);
  }
}

}  // namespace rk
