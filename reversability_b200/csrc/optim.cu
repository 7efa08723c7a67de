// Global-norm gradient clipping and AdamW over flat fp32 buffers (replaces
// torch.nn.utils.clip_grad_norm_ + torch.optim.AdamW at
// train_baseline.py:152-154,272,280).
//
// rk_clip_adamw_prepare: sum of squares of all gradients with a fixed grid
// (one partial per CTA) and a one-CTA finalize that sums the partials in
// index order (deterministic), then writes norm, clip coefficient
// min(1, max_norm / (norm + 1e-6)), increments the step counter and derives
// the bias-corrected step size, all into a small device scalar block so that
// a captured CUDA graph replays correctly with no host involvement.
// rk_adamw_step: one streaming pass, per element (decoupled weight decay,
// Loshchilov & Hutter):
//   g = grad * coef
//   p = p * (1 - lr*wd)
//   m = m + (1 - b1) * (g - m);  v = b2*v + (1 - b2)*g*g
//   p = p - (lr / (1 - b1^t)) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// optionally writing a bf16/f16 copy of the new parameters for the GEMMs.
#include "vec.cuh"

namespace rk {

constexpr int kNormBlocks = 1184;  // 8 per SM on 148 SMs: fixed, so the reduction order is fixed

__global__ void __launch_bounds__(256) sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  pdl_wait();  // inputs are the previous kernel's outputs
  __shared__ float red[8];
  float s = 0.f;
  const int64_t n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = g4[i];
    s = fmaf(v.x, v.x, s);
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    s = fmaf(v.w, v.w, s);
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s = fmaf(g[i], g[i], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

// scalars: [0] lr, [1] step, [2] grad norm, [3] clip coef, [4] step size lr/(1-b1^t),
//          [5] sqrt(1-b2^t), [6] 1 - lr*wd
__global__ void __launch_bounds__(256) prepare_kernel(const float* __restrict__ partial, int parts, float max_norm,
                                                      float beta1, float beta2, float weight_decay,
                                                      float* __restrict__ scalars) {
  pdl_wait();  // inputs are the previous kernel's outputs
  __shared__ double red[256];
  double s = 0.0;
  for (int i = threadIdx.x; i < parts; i += blockDim.x) s += (double)partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float norm = (float)sqrt(red[0]);
    const float coef = fminf(1.f, max_norm / (norm + 1e-6f));
    const float lr = scalars[0];
    const float t = scalars[1] + 1.f;
    scalars[1] = t;
    scalars[2] = norm;
    scalars[3] = max_norm > 0.f ? coef : 1.f;
    const double bc1 = 1.0 - pow((double)beta1, (double)t);
    const double bc2 = 1.0 - pow((double)beta2, (double)t);
    scalars[4] = (float)(lr / bc1);
    scalars[5] = (float)sqrt(bc2);
    scalars[6] = 1.f - lr * weight_decay;
  }
}

template <typename TC>
__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v, TC* __restrict__ pc,
                                                    int64_t n, const float* __restrict__ scalars, float beta1,
                                                    float beta2, float eps) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const float coef = scalars[3], step_size = scalars[4], bc2s = scalars[5], decay = scalars[6];
  const float om1 = 1.f - beta1, om2 = 1.f - beta2;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float pp[4], gg[4], mm[4], vv[4];
    load_vec<float, 4>(p + 4 * i, pp);
    load_vec<float, 4>(g + 4 * i, gg);
    load_vec<float, 4>(m + 4 * i, mm);
    load_vec<float, 4>(v + 4 * i, vv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gi = gg[e] * coef;
      pp[e] *= decay;
      mm[e] = fmaf(om1, gi - mm[e], mm[e]);
      vv[e] = fmaf(beta2, vv[e], om2 * gi * gi);
      const float denom = sqrtf(vv[e]) / bc2s + eps;
      pp[e] = pp[e] - step_size * (mm[e] / denom);
    }
    store_vec<float, 4>(p + 4 * i, pp);
    store_vec<float, 4>(m + 4 * i, mm);
    store_vec<float, 4>(v + 4 * i, vv);
    if (pc) store_vec<TC, 4>(pc + 4 * i, pp);
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i] * coef;
    float pp = p[i] * decay;
    const float mm = fmaf(om1, gi - m[i], m[i]);
    const float vv = fmaf(beta2, v[i], om2 * gi * gi);
    pp = pp - step_size * (mm / (sqrtf(vv) / bc2s + eps));
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (pc) pc[i] = Dt<TC>::from_f(pp);
  }
}

}  // namespace rk

using namespace rk;

extern "C" int64_t rk_clip_adamw_workspace(void) { return (int64_t)kNormBlocks * (int64_t)sizeof(float); }

extern "C" int rk_clip_adamw_prepare(const float* grads, int64_t n, float max_norm, float beta1, float beta2,
                                     float weight_decay, float* workspace, int64_t workspace_bytes, float* scalars,
                                     void* stream) {
  if (!grads || !workspace || !scalars || n < 0) return RK_ERR_ARG;
  if (workspace_bytes < rk_clip_adamw_workspace()) return RK_ERR_WORKSPACE;
  if (!rk_host::aligned(grads, 16)) return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rk_host::launch_k(sumsq_kernel, kNormBlocks, 256, 0, s, grads, n, workspace);
  int st = rk_host::launch_status();
  if (st) return st;
  rk_host::launch_k(prepare_kernel, 1, 256, 0, s, workspace, kNormBlocks, max_norm, beta1, beta2, weight_decay, scalars);
  return rk_host::launch_status();
}

extern "C" int rk_adamw_step(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, void* params_c,
                             int c_dtype, int64_t n, const float* scalars, float beta1, float beta2, float eps,
                             void* stream) {
  if (!params || !grads || !exp_avg || !exp_avg_sq || !scalars || n < 0) return RK_ERR_ARG;
  if (n == 0) return RK_OK;
  if (!rk_host::aligned(params, 16) || !rk_host::aligned(grads, 16) || !rk_host::aligned(exp_avg, 16) ||
      !rk_host::aligned(exp_avg_sq, 16) || (params_c && !rk_host::aligned(params_c, 8)))
    return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t blocks = (n / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  if (!params_c) {
    rk_host::launch_k(adamw_kernel<float>, (unsigned)blocks, 256, 0, s, params, grads, exp_avg, exp_avg_sq, nullptr, n, scalars,
                                                        beta1, beta2, eps);
  } else if (c_dtype == RK_BF16) {
    rk_host::launch_k(adamw_kernel<__nv_bfloat16>, (unsigned)blocks, 256, 0, s, params, grads, exp_avg, exp_avg_sq,
                                                                static_cast<__nv_bfloat16*>(params_c), n, scalars,
                                                                beta1, beta2, eps);
  } else if (c_dtype == RK_F16) {
    rk_host::launch_k(adamw_kernel<__half>, (unsigned)blocks, 256, 0, s, params, grads, exp_avg, exp_avg_sq,
                                                         static_cast<__half*>(params_c), n, scalars, beta1, beta2,
                                                         eps);
  } else {
    return RK_ERR_DTYPE;
  }
  return rk_host::launch_status();
}
