// Cross-entropy over the vocabulary, forward and backward in one pass pair
// (replaces F.cross_entropy(logits, y, ignore_index=-100, reduction="sum") at
// train_baseline.py:262 and its autograd backward; the reference's Triton
// variant is kernels.py:14-85).
//
// One CTA per row. Pass 1 streams the row once with 16-byte loads, keeping a
// per-thread online (max, sum of exp) pair that is merged across the CTA.
// Pass 2 re-reads the row (from L2 for rows in flight) and writes
//   dlogit = (exp(x - lse) - [col == label]) * scale
// in place or to a separate buffer, and loss[row] = lse - x[label].
// Rows whose label is ignore_index (-100) get loss 0 and a zero gradient row,
// matching PyTorch. Arithmetic is fp32 on logits read from bf16/f16/fp32, as
// autocast runs cross-entropy in fp32. A label outside [0, V) sets
// RK_DEV_CE_LABEL in the status word and the row is treated as ignored.
#include "vec.cuh"

namespace rk {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Merge (m, s) online-softmax pairs; s is a sum of exp(x - m).
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * fast_ex2((m - mn) * kLog2e)) + (m2 == -INFINITY ? 0.f : s2 * fast_ex2((m2 - mn) * kLog2e));
  m = mn;
}

template <typename T, int V>
__global__ void __launch_bounds__(512) ce_kernel(const T* logits, int64_t ld, int vocab,
                                                 const int64_t* __restrict__ labels, float scale,
                                                 const float* __restrict__ scale_dev,
                                                 float* __restrict__ loss_rows, T* dlogits,
                                                 int64_t ldd, int ignore_index, unsigned int* status) {
  pdl_wait();  // inputs are the previous kernel's outputs
  if (scale_dev) scale *= *scale_dev;
  __shared__ float sm_m[32], sm_s[32];
  __shared__ float s_lse;
  const int64_t row = blockIdx.x;
  const T* x = logits + row * ld;
  T* dx = dlogits + row * ldd;
  int64_t label = labels[row];
  const bool ignored = (label == ignore_index);
  const bool bad = !ignored && (label < 0 || label >= vocab);
  if (bad && threadIdx.x == 0) flag_error(status, RK_DEV_CE_LABEL);
  if (ignored || bad) {
    for (int c = threadIdx.x; c < vocab; c += blockDim.x) dx[c] = Dt<T>::from_f(0.f);
    if (threadIdx.x == 0) loss_rows[row] = 0.f;
    return;
  }
  const int nvec = vocab / V;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[V];
    load_vec<T, V>(x + (int64_t)i * V, v);
    float vm = v[0];
#pragma unroll
    for (int e = 1; e < V; ++e) vm = fmaxf(vm, v[e]);
    float vs = 0.f;
#pragma unroll
    for (int e = 0; e < V; ++e) vs += fast_ex2((v[e] - vm) * kLog2e);
    merge(m, s, vm, vs);
  }
  for (int c = nvec * V + threadIdx.x; c < vocab; c += blockDim.x) merge(m, s, Dt<T>::to_f(x[c]), 1.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm_m[lane] : -INFINITY;
    s = lane < nw ? sm_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m + logf(s);
      s_lse = lse;
      loss_rows[row] = lse - Dt<T>::to_f(x[label]);
    }
  }
  __syncthreads();
  const float lse = s_lse;
  const float nl = -lse * kLog2e;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[V], g[V];
    load_vec<T, V>(x + (int64_t)i * V, v);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const int c = i * V + e;
      const float p = fast_ex2(fmaf(v[e], kLog2e, nl));
      g[e] = (p - (c == label ? 1.f : 0.f)) * scale;
    }
    store_vec<T, V>(dx + (int64_t)i * V, g);
  }
  for (int c = nvec * V + threadIdx.x; c < vocab; c += blockDim.x) {
    const float p = fast_ex2(fmaf(Dt<T>::to_f(x[c]), kLog2e, nl));
    dx[c] = Dt<T>::from_f((p - (c == label ? 1.f : 0.f)) * scale);
  }
}

}  // namespace rk

using namespace rk;

namespace {
template <typename T>
int launch(const void* logits, int64_t ld, int64_t vocab, const int64_t* labels, int64_t rows, float scale,
           const float* scale_dev, float* loss_rows, void* dlogits, int64_t ldd, int ignore_index, cudaStream_t s) {
  constexpr int V = 16 / (int)sizeof(T);
  auto X = static_cast<const T*>(logits);
  auto D = static_cast<T*>(dlogits);
  unsigned int* st = rk_host::device_status_ptr();
  const bool vec = rk_host::aligned(logits, 16) && rk_host::aligned(dlogits, 16) &&
                   (ld * (int64_t)sizeof(T)) % 16 == 0 && (ldd * (int64_t)sizeof(T)) % 16 == 0;
  if (vec)
    rk_host::launch_k(ce_kernel<T, V>, (unsigned)rows, 512, 0, s, X, ld, (int)vocab, labels, scale, scale_dev, loss_rows, D, ldd, ignore_index, st);
  else
    rk_host::launch_k(ce_kernel<T, 1>, (unsigned)rows, 512, 0, s, X, ld, (int)vocab, labels, scale, scale_dev, loss_rows, D, ldd, ignore_index, st);
  return rk_host::launch_status();
}
}  // namespace

extern "C" int rk_cross_entropy_fwd_bwd(const void* logits, int64_t ld, int64_t vocab, const int64_t* labels,
                                        int64_t rows, float grad_scale, const float* grad_scale_dev,
                                        float* loss_rows, void* dlogits, int64_t ldd, int dtype, int ignore_index,
                                        void* stream) {
  if (!logits || !labels || !loss_rows || !dlogits || rows < 0 || vocab <= 0 || ld < vocab || ldd < vocab ||
      vocab >= (1ll << 31) || rows >= (1ll << 31))
    return RK_ERR_ARG;
  if (rows == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case RK_F32: return launch<float>(logits, ld, vocab, labels, rows, grad_scale, grad_scale_dev, loss_rows, dlogits, ldd, ignore_index, s);
    case RK_BF16:
      return launch<__nv_bfloat16>(logits, ld, vocab, labels, rows, grad_scale, grad_scale_dev, loss_rows, dlogits, ldd, ignore_index, s);
    case RK_F16: return launch<__half>(logits, ld, vocab, labels, rows, grad_scale, grad_scale_dev, loss_rows, dlogits, ldd, ignore_index, s);
    default: return RK_ERR_DTYPE;
  }
}
