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
    reconstruct_kernel<TF, 4, SCALE><<<(unsigned)blocks, 256, 0, s>>>(xn, F, coeff, xp, n);
  else
    reconstruct_kernel<TF, 1, SCALE><<<(unsigned)blocks, 256, 0, s>>>(xn, F, coeff, xp, n);
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
  if (!x_next || !force || !x_prev || n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;
  return dispatch<true>(x_next, force, force_dtype, coeff, x_prev, n, static_cast<cudaStream_t>(stream));
}

extern "C" int rk_reconstruct_euler(const float* state, const void* sublayer_out, int out_dtype, float* state_prev,
                                    int64_t n, void* stream) {
  if (!state || !sublayer_out || !state_prev || n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;
  return dispatch<false>(state, sublayer_out, out_dtype, 1.f, state_prev, n, static_cast<cudaStream_t>(stream));
}
