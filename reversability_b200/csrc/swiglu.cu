// SwiGLU forward/backward (replaces kernels.py:88-131 and MLP's silu(gate)*value).
//
// u is [rows, 2*width]: gate = u[:, :width], value = u[:, width:]. Each thread
// handles V consecutive columns of one row with 16-byte loads of gate and
// value and a 16-byte store, so the kernel streams HBM at full width. The
// arithmetic follows the reference kernels operation by operation, with FMA
// contraction suppressed (the reference compiles with enable_fp_fusion=False)
// and the exponential/divide on the approximate hardware paths (common.cuh):
//   forward : silu = round_T(g / (1 + exp(-g)));  h = silu * v
//   backward: s = 1/(1+exp(-g)); silu = round_T(g*s); t = round_T(dh*v)
//             dg = t * (s * (1 + g*(1-s)));  dv = dh * silu
#include "vec.cuh"

namespace rk {

template <typename T>
__device__ __forceinline__ float silu_fwd(float g) {
  return round_to<T>(silu_value(g));
}

template <typename T, int V>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ u, T* __restrict__ h, int64_t rows,
                                                         int64_t width) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t vecs_per_row = width / V;
  const int64_t total = rows * vecs_per_row;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / vecs_per_row;
    const int64_t c = (t - r * vecs_per_row) * V;
    const T* ur = u + r * 2 * width;
    float g[V], v[V], o[V];
    load_vec<T, V>(ur + c, g);
    load_vec<T, V>(ur + width + c, v);
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = __fmul_rn(silu_fwd<T>(g[e]), v[e]);
    store_vec<T, V>(h + r * width + c, o);
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ u, const T* __restrict__ dh,
                                                         T* __restrict__ du, int64_t rows, int64_t width) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t vecs_per_row = width / V;
  const int64_t total = rows * vecs_per_row;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / vecs_per_row;
    const int64_t c = (t - r * vecs_per_row) * V;
    const T* ur = u + r * 2 * width;
    float g[V], v[V], up[V], dg[V], dv[V];
    load_vec<T, V>(ur + c, g);
    load_vec<T, V>(ur + width + c, v);
    load_vec<T, V>(dh + r * width + c, up);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float s = sigmoid_value(g[e]);
      const float silu = round_to<T>(__fmul_rn(g[e], s));
      const float t_ = round_to<T>(__fmul_rn(up[e], v[e]));
      const float slope = __fmul_rn(s, __fadd_rn(1.f, __fmul_rn(g[e], __fsub_rn(1.f, s))));
      dg[e] = __fmul_rn(t_, slope);
      dv[e] = __fmul_rn(up[e], silu);
    }
    T* dr = du + r * 2 * width;
    store_vec<T, V>(dr + c, dg);
    store_vec<T, V>(dr + width + c, dv);
  }
}

}  // namespace rk

using namespace rk;

namespace {

unsigned grid_for(int64_t work) {
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = 148 * 16;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks > 0 ? blocks : 1);
}

template <typename T>
int fwd_typed(const void* u, void* h, int64_t rows, int64_t width, cudaStream_t s) {
  constexpr int V = 16 / (int)sizeof(T);
  auto U = static_cast<const T*>(u);
  auto H = static_cast<T*>(h);
  if (width % V == 0 && rk_host::aligned(u, 16) && rk_host::aligned(h, 16))
    rk_host::launch_k(swiglu_fwd_kernel<T, V>, grid_for(rows * width / V), 256, 0, s, U, H, rows, width);
  else
    rk_host::launch_k(swiglu_fwd_kernel<T, 1>, grid_for(rows * width), 256, 0, s, U, H, rows, width);
  return rk_host::launch_status();
}

template <typename T>
int bwd_typed(const void* u, const void* dh, void* du, int64_t rows, int64_t width, cudaStream_t s) {
  constexpr int V = 16 / (int)sizeof(T);
  auto U = static_cast<const T*>(u);
  auto G = static_cast<const T*>(dh);
  auto D = static_cast<T*>(du);
  if (width % V == 0 && rk_host::aligned(u, 16) && rk_host::aligned(dh, 16) && rk_host::aligned(du, 16))
    rk_host::launch_k(swiglu_bwd_kernel<T, V>, grid_for(rows * width / V), 256, 0, s, U, G, D, rows, width);
  else
    rk_host::launch_k(swiglu_bwd_kernel<T, 1>, grid_for(rows * width), 256, 0, s, U, G, D, rows, width);
  return rk_host::launch_status();
}

}  // namespace

extern "C" int rk_swiglu_fwd(const void* u, void* h, int dtype, int64_t rows, int64_t width, void* stream) {
  if (rows < 0 || width <= 0) return RK_ERR_ARG;
  if (rows == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!u || !h) return RK_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case RK_F32: return fwd_typed<float>(u, h, rows, width, s);
    case RK_BF16: return fwd_typed<__nv_bfloat16>(u, h, rows, width, s);
    case RK_F16: return fwd_typed<__half>(u, h, rows, width, s);
    default: return RK_ERR_DTYPE;
  }
}

extern "C" int rk_swiglu_bwd(const void* u, const void* dh, void* du, int dtype, int64_t rows, int64_t width,
                             void* stream) {
  if (rows < 0 || width <= 0) return RK_ERR_ARG;
  if (rows == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!u || !dh || !du) return RK_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case RK_F32: return bwd_typed<float>(u, dh, du, rows, width, s);
    case RK_BF16: return bwd_typed<__nv_bfloat16>(u, dh, du, rows, width, s);
    case RK_F16: return bwd_typed<__half>(u, dh, du, rows, width, s);
    default: return RK_ERR_DTYPE;
  }
}
