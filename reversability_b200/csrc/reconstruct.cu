// Reversible reconstruction (replaces inverse_pair, reversible.py:28-32).
//
// Midpoint: x_prev = x_next - round_F(coeff * F), coeff = 2h. Autocast runs
// `2 * h * force` in the force dtype (the scaled force is rounded to bf16/f16)
// and only then promotes to fp32 for the subtraction; this kernel does the
// same so that reconstruction inverts the forward update bit for bit when the
// force is recomputed identically. Euler: state_prev = state - sublayer_out.
// Pure streaming kernels: 16-byte loads of the fp32 state, 8- or 16-byte loads
// of the force, 16-byte stores.
#include "vec.cuh"

namespace rk {

template <typename TF, int V, bool SCALE>
__global__ void __launch_bounds__(256) reconstruct_kernel(const float* __restrict__ xn, const TF* __restrict__ f,
                                                          float coeff, float* __restrict__ xp, int64_t n) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t nv = n / V;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nv; t += (int64_t)gridDim.x * blockDim.x) {
    float a[V], b[V], o[V];
    load_vec<float, V>(xn + t * V, a);
    load_vec<TF, V>(f + t * V, b);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float sf = SCALE ? round_to<TF>(__fmul_rn(coeff, b[e])) : b[e];
      o[e] = __fsub_rn(a[e], sf);
    }
    store_vec<float, V>(xp + t * V, o);
  }
  // scalar tail
  const int64_t tail0 = nv * V;
  const int64_t i = tail0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float b = Dt<TF>::to_f(f[i]);
    const float sf = SCALE ? round_to<TF>(__fmul_rn(coeff, b)) : b;
    xp[i] = __fsub_rn(xn[i], sf);
  }
}


// Force assembled from its two sublayer outputs: F = round_T(a + m) (the bf16
// add of reversible.py:18), then x_prev = x_next - round_T(coeff * F).
template <typename TF, int V>
__global__ void __launch_bounds__(256) reconstruct_sum_kernel(const float* __restrict__ xn, const TF* __restrict__ a,
                                                              const TF* __restrict__ m, float coeff,
                                                              float* __restrict__ xp, int64_t n) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t nv = n / V;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nv; t += (int64_t)gridDim.x * blockDim.x) {
    float x[V], av[V], mv[V], o[V];
    load_vec<float, V>(xn + t * V, x);
    load_vec<TF, V>(a + t * V, av);
    load_vec<TF, V>(m + t * V, mv);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float f = round_to<TF>(__fadd_rn(av[e], mv[e]));
      o[e] = __fsub_rn(x[e], round_to<TF>(__fmul_rn(coeff, f)));
    }
    store_vec<float, V>(xp + t * V, o);
  }
  const int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float f = round_to<TF>(__fadd_rn(Dt<TF>::to_f(a[i]), Dt<TF>::to_f(m[i])));
    xp[i] = __fsub_rn(xn[i], round_to<TF>(__fmul_rn(coeff, f)));
  }
}

// out = round_T(round_T(x) * scale): an fp32 cotangent cast to the compute
// dtype and scaled there (autograd's cast-backward followed by the backward of
// `2 * h * F`).
template <typename T, int V>
__global__ void __launch_bounds__(256) cast_scale_kernel(const float* __restrict__ x, T* __restrict__ out, float scale,
                                                         int64_t n) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t nv = n / V;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nv; t += (int64_t)gridDim.x * blockDim.x) {
    float v[V], o[V];
    load_vec<float, V>(x + t * V, v);
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = __fmul_rn(round_to<T>(v[e]), scale);
    store_vec<T, V>(out + t * V, o);
  }
  const int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = Dt<T>::from_f(__fmul_rn(round_to<T>(x[i]), scale));
}

}  // namespace rk

using namespace rk;

namespace {
template <typename TF, bool SCALE>
int launch(const float* xn, const void* f, float coeff, float* xp, int64_t n, cudaStream_t s) {
  auto F = static_cast<const TF*>(f);
  const bool vec = rk_host::aligned(xn, 16) && rk_host::aligned(xp, 16) && rk_host::aligned(f, 4 * sizeof(TF));
  int64_t work = vec ? n / 4 : n;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  if (vec)
    rk_host::launch_k(reconstruct_kernel<TF, 4, SCALE>, (unsigned)blocks, 256, 0, s, xn, F, coeff, xp, n);
  else
    rk_host::launch_k(reconstruct_kernel<TF, 1, SCALE>, (unsigned)blocks, 256, 0, s, xn, F, coeff, xp, n);
  return rk_host::launch_status();
}

template <bool SCALE>
int dispatch(const float* xn, const void* f, int dt, float coeff, float* xp, int64_t n, cudaStream_t s) {
  switch (dt) {
    case RK_F32: return launch<float, SCALE>(xn, f, coeff, xp, n, s);
    case RK_BF16: return launch<__nv_bfloat16, SCALE>(xn, f, coeff, xp, n, s);
    case RK_F16: return launch<__half, SCALE>(xn, f, coeff, xp, n, s);
    default: return RK_ERR_DTYPE;
  }
}
}  // namespace

extern "C" int rk_reconstruct_midpoint(const float* x_next, const void* force, int force_dtype, float coeff,
                                       float* x_prev, int64_t n, void* stream) {
  if (n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!x_next || !force || !x_prev) return RK_ERR_ARG;
  return dispatch<true>(x_next, force, force_dtype, coeff, x_prev, n, static_cast<cudaStream_t>(stream));
}

extern "C" int rk_reconstruct_euler(const float* state, const void* sublayer_out, int out_dtype, float* state_prev,
                                    int64_t n, void* stream) {
  if (n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!state || !sublayer_out || !state_prev) return RK_ERR_ARG;
  return dispatch<false>(state, sublayer_out, out_dtype, 1.f, state_prev, n, static_cast<cudaStream_t>(stream));
}

namespace {
unsigned blocks_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)(b < 1 ? 1 : b);
}
template <typename TF>
int sum_launch(const float* xn, const void* a, const void* m, float coeff, float* xp, int64_t n, cudaStream_t s) {
  auto A = static_cast<const TF*>(a);
  auto Mv = static_cast<const TF*>(m);
  const size_t va = 4 * sizeof(TF) >= 16 ? 16 : 4 * sizeof(TF);
  if (rk_host::aligned(xn, 16) && rk_host::aligned(xp, 16) && rk_host::aligned(a, va) && rk_host::aligned(m, va))
    rk_host::launch_k(reconstruct_sum_kernel<TF, 4>, blocks_for(n / 4), 256, 0, s, xn, A, Mv, coeff, xp, n);
  else
    rk_host::launch_k(reconstruct_sum_kernel<TF, 1>, blocks_for(n), 256, 0, s, xn, A, Mv, coeff, xp, n);
  return rk_host::launch_status();
}
template <typename T>
int cast_launch(const float* x, void* out, float scale, int64_t n, cudaStream_t s) {
  auto O = static_cast<T*>(out);
  const size_t vo = 4 * sizeof(T) >= 16 ? 16 : 4 * sizeof(T);
  if (rk_host::aligned(x, 16) && rk_host::aligned(out, vo))
    rk_host::launch_k(cast_scale_kernel<T, 4>, blocks_for(n / 4), 256, 0, s, x, O, scale, n);
  else
    rk_host::launch_k(cast_scale_kernel<T, 1>, blocks_for(n), 256, 0, s, x, O, scale, n);
  return rk_host::launch_status();
}
}  // namespace

extern "C" int rk_reconstruct_midpoint_sum(const float* x_next, const void* a, const void* m, int dtype, float coeff,
                                           float* x_prev, int64_t n, void* stream) {
  if (n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!x_next || !a || !m || !x_prev) return RK_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case RK_F32: return sum_launch<float>(x_next, a, m, coeff, x_prev, n, s);
    case RK_BF16: return sum_launch<__nv_bfloat16>(x_next, a, m, coeff, x_prev, n, s);
    case RK_F16: return sum_launch<__half>(x_next, a, m, coeff, x_prev, n, s);
    default: return RK_ERR_DTYPE;
  }
}

extern "C" int rk_cast_scale(const float* x, void* out, int out_dtype, float scale, int64_t n, void* stream) {
  if (!x || !out || n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (out_dtype) {
    case RK_F32: return cast_launch<float>(x, out, scale, n, s);
    case RK_BF16: return cast_launch<__nv_bfloat16>(x, out, scale, n, s);
    case RK_F16: return cast_launch<__half>(x, out, scale, n, s);
    default: return RK_ERR_DTYPE;
  }
}
