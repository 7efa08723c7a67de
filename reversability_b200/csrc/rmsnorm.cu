// RMSNorm forward/backward (replaces kernels_v3.py:9-48 and nn.RMSNorm).
//
// One warp per row. Lane l owns NV vectors of V consecutive columns:
// columns [(j*32 + l)*V, +V) for j < NV, so every warp-wide load is a
// contiguous, 16-byte-per-lane transaction. The row reduction is a warp
// shuffle tree. The weight gradient is reduced first in registers (per lane,
// over the rows a warp visits), then across the 8 warps of the CTA in shared
// memory into one fp32 partial row per CTA, then by a second kernel over the
// partials in a fixed order (deterministic, no atomics).
#include <mutex>
#include "vec.cuh"

namespace rk {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Each warp handles R consecutive rows and issues all of their loads before
// reducing any of them, so enough bytes are in flight per SM to cover memory
// latency (one 512-byte bf16 row per warp would not).
template <typename Tx, typename Ty, int V, int NV, int R>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const Tx* __restrict__ x, int64_t ldx,
                                                          const float* __restrict__ w, Ty* __restrict__ y,
                                                          int64_t ldy, float* __restrict__ rstd, int64_t rows,
                                                          int width, float eps) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R;
  if (row0 >= rows) return;
  float v[R][NV][V];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = row0 + r;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (j * 32 + lane) * V;
      if (row < rows && c < width) load_vec<Tx, V>(x + row * ldx + c, v[r][j]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = row0 + r;
    if (row >= rows) break;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {  // group j: lane sums in butterfly order, groups in column order
      const int c = (j * 32 + lane) * V;
      const float sj = warp_sum(c < width ? sumsq_chain<V>(v[r][j]) : 0.f);
      ss = j == 0 ? sj : __fadd_rn(ss, sj);
    }
    const float rs = rms_rstd(ss, width, eps);
    if (rstd && lane == 0) rstd[row] = rs;
    Ty* yr = y + row * ldy;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (j * 32 + lane) * V;
      if (c < width) {
        float wv[V], o[V];
        load_vec<float, V>(w + c, wv);
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = __fmul_rn(__fmul_rn(v[r][j][e], rs), wv[e]);
        store_vec<Ty, V>(yr + c, o);
      }
    }
  }
}

template <typename Tx, typename Tg, typename Tdx, int V, int NV>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const Tx* __restrict__ x, int64_t ldx,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ rstd, const Tg* __restrict__ dy,
                                                          int64_t lddy, Tdx* __restrict__ dx, int64_t lddx,
                                                          float* __restrict__ partial, int64_t rows, int width) {
  pdl_wait();  // inputs are the previous kernel's outputs
  extern __shared__ float red[];  // [8][width]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t stride = (int64_t)gridDim.x * 8;
  float acc[NV][V];
  float wv[NV][V];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
#pragma unroll
    for (int e = 0; e < V; ++e) acc[j][e] = 0.f;
    if (c < width) load_vec<float, V>(w + c, wv[j]);
  }
  // two rows per iteration (rows `row` and `row + stride`), all loads first
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += 2 * stride) {
    float xv[2][NV][V], gv[2][NV][V], rr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t rw = row + h * stride;
      rr[h] = rw < rows ? __ldg(rstd + rw) : 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (rw < rows && c < width) {
          load_vec<Tx, V>(x + rw * ldx + c, xv[h][j]);
          load_vec<Tg, V>(dy + rw * lddy + c, gv[h][j]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t rw = row + h * stride;
      if (rw >= rows) break;
      const float r = rr[h];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (c < width) {
#pragma unroll
          for (int e = 0; e < V; ++e) {
            dot += (gv[h][j][e] * wv[j][e]) * xv[h][j][e];
            acc[j][e] += gv[h][j][e] * (xv[h][j][e] * r);
          }
        }
      }
      dot = warp_sum(dot);
      const float corr = dot / (float)width * r * r;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (c < width) {
          float o[V];
#pragma unroll
          for (int e = 0; e < V; ++e) o[e] = (gv[h][j][e] * wv[j][e] - xv[h][j][e] * corr) * r;
          store_vec<Tdx, V>(dx + rw * lddx + c, o);
        }
      }
    }
  }
  // Cross-warp reduction of the weight-gradient accumulators.
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
    if (c < width) {
#pragma unroll
      for (int e = 0; e < V; ++e) red[warp * width + c + e] = acc[j][e];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k * width + c];
    partial[(int64_t)blockIdx.x * width + c] = s;
  }
}

// dw[c] (+)= sum over parts. A CTA owns 32 columns; thread (g, c) of its 32
// groups sums parts g, g+32, ... of column c (coalesced 128-byte rows), then
// the 32 group sums are added in group order: a fixed order, so dw is
// deterministic.
__global__ void __launch_bounds__(1024) rmsnorm_dw_reduce_kernel(const float* __restrict__ partial,
                                                                 float* __restrict__ dw, int parts, int width,
                                                                 int accumulate) {
  pdl_wait();  // inputs are the previous kernel's outputs
  __shared__ float grp[32][33];
  const int lc = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lc;
  float s = 0.f;
  if (c < width) {
    // eight partials in flight per thread, added in part order
    int p = g;
    for (; p + 7 * 32 < parts; p += 8 * 32) {
      float t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = partial[(int64_t)(p + 32 * k) * width + c];
#pragma unroll
      for (int k = 0; k < 8; ++k) s += t[k];
    }
    for (; p < parts; p += 32) s += partial[(int64_t)p * width + c];
  }
  grp[g][lc] = s;
  __syncthreads();
  if (g == 0 && c < width) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) t += grp[k][lc];
    dw[c] = accumulate ? dw[c] + t : t;
  }
}

// ---------------------------------------------------------------- fused variants
// Residual add + RMSNorm: s = x + a (fp32), y = rmsnorm(s) * w. `a` is the
// low-precision sublayer output (autocast's bf16 Linear result); the sum is
// written out only when the backward needs it (sum_out != NULL).
template <typename Ta, typename Ty, int NV>
__global__ void __launch_bounds__(256) add_rmsnorm_fwd_kernel(const float* __restrict__ x, const Ta* __restrict__ a,
                                                              const float* __restrict__ w, Ty* __restrict__ y,
                                                              float* __restrict__ sum_out, float* __restrict__ rstd,
                                                              int64_t rows, int width, float eps) {
  pdl_wait();  // inputs are the previous kernel's outputs
  constexpr int V = 4;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t base = row * width;
  float v[NV][V];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
    if (c < width) {
      float xa[V], aa[V];
      load_vec<float, V>(x + base + c, xa);
      load_vec<Ta, V>(a + base + c, aa);
#pragma unroll
      for (int e = 0; e < V; ++e) v[j][e] = __fadd_rn(xa[e], aa[e]);
      if (sum_out) store_vec<float, V>(sum_out + base + c, v[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {  // the order of rmsnorm_fwd_kernel (sumsq_chain, butterfly, groups in order)
    const int c = (j * 32 + lane) * V;
    const float sj = warp_sum(c < width ? sumsq_chain<V>(v[j]) : 0.f);
    ss = j == 0 ? sj : __fadd_rn(ss, sj);
  }
  const float r = rms_rstd(ss, width, eps);
  if (rstd && lane == 0) rstd[row] = r;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
    if (c < width) {
      float wv[V], o[V];
      load_vec<float, V>(w + c, wv);
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = __fmul_rn(__fmul_rn(v[j][e], r), wv[e]);
      store_vec<Ty, V>(y + base + c, o);
    }
  }
}

// RMSNorm backward with the cotangent bookkeeping of the reversible step fused
// into its epilogue (rows contiguous, fp32 input x):
//   dx_out = dx + residual                         (fp32; residual may be NULL)
//   LP == 1: lp_out = round(lp_add + round(dx))    (the bf16 sum autograd forms
//            when a bf16 tensor feeds two consumers)
//   LP == 2: lp_out = round(round(dx_out) * lp_scale)  (rk_cast_scale of the total: the
//                                                       next layer's round(2h * dq) in the sweep)
template <typename Tg, typename Tlp, int NV, bool RES, int LP>
__global__ void __launch_bounds__(256) rmsnorm_bwd_fused_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ rstd, const Tg* __restrict__ dy,
    const float* __restrict__ residual, const Tlp* __restrict__ lp_add, float* __restrict__ dx_out,
    Tlp* __restrict__ lp_out, float* __restrict__ partial, int64_t rows, int width, float lp_scale) {
  pdl_wait();  // inputs are the previous kernel's outputs
  constexpr int V = 4;
  extern __shared__ float red[];  // [8][width]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t stride = (int64_t)gridDim.x * 8;
  float acc[NV][V];
  float wv[NV][V];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
#pragma unroll
    for (int e = 0; e < V; ++e) acc[j][e] = 0.f;
    if (c < width) load_vec<float, V>(w + c, wv[j]);
  }
  // R rows per iteration (rows `row`, `row + stride`, ..., the order of the
  // weight-gradient sums unchanged), every load of them issued first
  constexpr int R = NV <= 4 ? 2 : 1;
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += R * stride) {
    float xv[R][NV][V], gv[R][NV][V], res[R][NV][V], la[R][NV][V], rr[R];
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t rw = row + h * stride;
      rr[h] = rw < rows ? __ldg(rstd + rw) : 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (rw < rows && c < width) {
          load_vec<float, V>(x + rw * width + c, xv[h][j]);
          load_vec<Tg, V>(dy + rw * width + c, gv[h][j]);
          if constexpr (RES) load_vec<float, V>(residual + rw * width + c, res[h][j]);
          if constexpr (LP == 1) load_vec<Tlp, V>(lp_add + rw * width + c, la[h][j]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < R; ++h) {
      const int64_t rw = row + h * stride;
      if (rw >= rows) break;
      const float r = rr[h];
      const int64_t base = rw * width;
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (c < width) {
#pragma unroll
          for (int e = 0; e < V; ++e) {
            dot += (gv[h][j][e] * wv[j][e]) * xv[h][j][e];
            acc[j][e] += gv[h][j][e] * (xv[h][j][e] * r);
          }
        }
      }
      dot = warp_sum(dot);
      const float corr = dot / (float)width * r * r;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = (j * 32 + lane) * V;
        if (c < width) {
          float o[V], lp[V];
#pragma unroll
          for (int e = 0; e < V; ++e) o[e] = (gv[h][j][e] * wv[j][e] - xv[h][j][e] * corr) * r;
          if constexpr (LP == 1) {
#pragma unroll
            for (int e = 0; e < V; ++e) lp[e] = __fadd_rn(la[h][j][e], round_to<Tlp>(o[e]));
          }
          if constexpr (RES) {
#pragma unroll
            for (int e = 0; e < V; ++e) o[e] = __fadd_rn(o[e], res[h][j][e]);  // no contraction into the last multiply
          }
          if constexpr (LP == 2) {
#pragma unroll
            for (int e = 0; e < V; ++e) lp[e] = __fmul_rn(round_to<Tlp>(o[e]), lp_scale);  // as rk_cast_scale
          }
          store_vec<float, V>(dx_out + base + c, o);
          if constexpr (LP != 0) store_vec<Tlp, V>(lp_out + base + c, lp);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = (j * 32 + lane) * V;
    if (c < width) {
#pragma unroll
      for (int e = 0; e < V; ++e) red[warp * width + c + e] = acc[j][e];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k * width + c];
    partial[(int64_t)blockIdx.x * width + c] = t;
  }
}

}  // namespace rk

using namespace rk;

namespace {

// True when a V-element vector of T at any row start (stride ld elements) is
// aligned to min(16, V*sizeof(T)) bytes.
template <typename T>
bool vec_fits(const void* p, int64_t ld, int V) {
  const int64_t a = (int64_t)sizeof(T) * V >= 16 ? 16 : (int64_t)sizeof(T) * V;
  return rk_host::aligned(p, (size_t)a) && ((ld * (int64_t)sizeof(T)) % a == 0);
}

int rms_parts(int64_t rows) {
  int64_t warps_rows = (rows + 7) / 8;
  return (int)(warps_rows < 296 ? (warps_rows > 0 ? warps_rows : 1) : 296);
}

template <typename Tx, typename Ty, int V>
int fwd_nv(const void* x, int64_t ldx, const float* w, void* y, int64_t ldy, float* rstd, int64_t rows, int width,
           float eps, cudaStream_t s) {
  const int per = 32 * V;
  const int nv = (width + per - 1) / per;
  dim3 grid((unsigned)((rows + 7) / 8)), block(256);
  auto X = static_cast<const Tx*>(x);
  auto Y = static_cast<Ty*>(y);
#define RK_FWD(N) \
  rk_host::launch_k(rmsnorm_fwd_kernel<Tx, Ty, V, N, 1>, grid, block, 0, s, X, ldx, w, Y, ldy, rstd, rows, width, eps)
  if (nv <= 1) RK_FWD(1);
  else if (nv <= 2) RK_FWD(2);
  else if (nv <= 4) RK_FWD(4);
  else if (nv <= 8) RK_FWD(8);
  else if constexpr (V == 1) {
    if (nv <= 32) RK_FWD(32);
    else return RK_ERR_UNSUPPORTED;
  } else return RK_ERR_UNSUPPORTED;
#undef RK_FWD
  return rk_host::launch_status();
}

template <typename Tx, typename Ty>
int fwd_typed(const void* x, int64_t ldx, const float* w, void* y, int64_t ldy, float* rstd, int64_t rows, int width,
              float eps, cudaStream_t s) {
  constexpr int VX = 16 / (int)sizeof(Tx);
  const bool vec_ok = (width % VX == 0) && vec_fits<Tx>(x, ldx, VX) && vec_fits<float>(w, 0, VX) &&
                      vec_fits<Ty>(y, ldy, VX);
  if (vec_ok) return fwd_nv<Tx, Ty, VX>(x, ldx, w, y, ldy, rstd, rows, width, eps, s);
  return fwd_nv<Tx, Ty, 1>(x, ldx, w, y, ldy, rstd, rows, width, eps, s);
}

template <typename Tx, typename Tg, typename Tdx, int V>
int bwd_nv(const void* x, int64_t ldx, const float* w, const float* rstd, const void* dy, int64_t lddy, void* dx,
           int64_t lddx, float* partial, int parts, int64_t rows, int width, cudaStream_t s) {
  const int per = 32 * V;
  const int nv = (width + per - 1) / per;
  dim3 grid((unsigned)parts), block(256);
  size_t smem = (size_t)8 * width * sizeof(float);
  auto X = static_cast<const Tx*>(x);
  auto G = static_cast<const Tg*>(dy);
  auto D = static_cast<Tdx*>(dx);
#define RK_BWD(N)                                                                                          \
  do {                                                                                                     \
    auto k = rmsnorm_bwd_kernel<Tx, Tg, Tdx, V, N>;                                                        \
    if (smem > 48 * 1024) { if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)smem)) return e_; }         \
    rk_host::launch_k(k, grid, block, smem, s, X, ldx, w, rstd, G, lddy, D, lddx, partial, rows, width);                  \
  } while (0)
  if (nv <= 1) RK_BWD(1);
  else if (nv <= 2) RK_BWD(2);
  else if (nv <= 4) RK_BWD(4);
  else if (nv <= 8) RK_BWD(8);
  else if constexpr (V == 1) {
    if (nv <= 32) RK_BWD(32);
    else return RK_ERR_UNSUPPORTED;
  } else return RK_ERR_UNSUPPORTED;
#undef RK_BWD
  return rk_host::launch_status();
}

template <typename Tx, typename Tg, typename Tdx>
int bwd_typed(const void* x, int64_t ldx, const float* w, const float* rstd, const void* dy, int64_t lddy, void* dx,
              int64_t lddx, float* partial, int parts, int64_t rows, int width, cudaStream_t s) {
  constexpr int VX = 16 / (int)sizeof(Tx);
  const bool vec_ok = (width % VX == 0) && vec_fits<Tx>(x, ldx, VX) && vec_fits<float>(w, 0, VX) &&
                      vec_fits<Tg>(dy, lddy, VX) && vec_fits<Tdx>(dx, lddx, VX);
  if (vec_ok) return bwd_nv<Tx, Tg, Tdx, VX>(x, ldx, w, rstd, dy, lddy, dx, lddx, partial, parts, rows, width, s);
  return bwd_nv<Tx, Tg, Tdx, 1>(x, ldx, w, rstd, dy, lddy, dx, lddx, partial, parts, rows, width, s);
}

}  // namespace

extern "C" int rk_rmsnorm_fwd(const void* x, int x_dtype, int64_t ldx, const float* w, void* y, int y_dtype,
                              int64_t ldy, float* rstd, int64_t rows, int64_t width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || ldx < width || ldy < width) return RK_ERR_ARG;
  if (width > 1024) return RK_ERR_UNSUPPORTED;
  if (rows == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!x || !w || !y) return RK_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = (int)width;
  if (x_dtype == RK_F32 && y_dtype == RK_F32) return fwd_typed<float, float>(x, ldx, w, y, ldy, rstd, rows, W, eps, s);
  if (x_dtype == RK_F32 && y_dtype == RK_BF16)
    return fwd_typed<float, __nv_bfloat16>(x, ldx, w, y, ldy, rstd, rows, W, eps, s);
  if (x_dtype == RK_F32 && y_dtype == RK_F16) return fwd_typed<float, __half>(x, ldx, w, y, ldy, rstd, rows, W, eps, s);
  if (x_dtype == RK_BF16 && y_dtype == RK_BF16)
    return fwd_typed<__nv_bfloat16, __nv_bfloat16>(x, ldx, w, y, ldy, rstd, rows, W, eps, s);
  if (x_dtype == RK_F16 && y_dtype == RK_F16) return fwd_typed<__half, __half>(x, ldx, w, y, ldy, rstd, rows, W, eps, s);
  return RK_ERR_DTYPE;
}

extern "C" int64_t rk_rmsnorm_bwd_workspace(int64_t rows, int64_t width) {
  return (int64_t)rms_parts(rows) * width * (int64_t)sizeof(float);
}

extern "C" int rk_rmsnorm_bwd(const void* x, int x_dtype, int64_t ldx, const float* w, const float* rstd,
                              const void* dy, int dy_dtype, int64_t lddy, void* dx, int dx_dtype, int64_t lddx,
                              float* dw, int accumulate_dw, float* dw_partial, int64_t workspace_bytes, int64_t rows,
                              int64_t width, void* stream) {
  if (!dw || rows < 0 || width <= 0) return RK_ERR_ARG;
  if (ldx < width || lddy < width || lddx < width) return RK_ERR_ARG;
  if (width > 1024) return RK_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = (int)width;
  if (rows == 0) {  // dw = 0 (or unchanged); the row pointers and the workspace may be null
    if (accumulate_dw) return RK_OK;
    cudaMemsetAsync(dw, 0, sizeof(float) * W, s);
    return rk_host::launch_status();
  }
  if (!x || !w || !rstd || !dy || !dx || !dw_partial) return RK_ERR_ARG;
  const int parts = rms_parts(rows);
  if (workspace_bytes < (int64_t)parts * W * (int64_t)sizeof(float)) return RK_ERR_WORKSPACE;
  int st;
  if (x_dtype == RK_F32 && dy_dtype == RK_F32 && dx_dtype == RK_F32)
    st = bwd_typed<float, float, float>(x, ldx, w, rstd, dy, lddy, dx, lddx, dw_partial, parts, rows, W, s);
  else if (x_dtype == RK_F32 && dy_dtype == RK_BF16 && dx_dtype == RK_F32)
    st = bwd_typed<float, __nv_bfloat16, float>(x, ldx, w, rstd, dy, lddy, dx, lddx, dw_partial, parts, rows, W, s);
  else if (x_dtype == RK_F32 && dy_dtype == RK_F16 && dx_dtype == RK_F32)
    st = bwd_typed<float, __half, float>(x, ldx, w, rstd, dy, lddy, dx, lddx, dw_partial, parts, rows, W, s);
  else if (x_dtype == RK_BF16 && dy_dtype == RK_BF16 && dx_dtype == RK_BF16)
    st = bwd_typed<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(x, ldx, w, rstd, dy, lddy, dx, lddx, dw_partial,
                                                                 parts, rows, W, s);
  else if (x_dtype == RK_F16 && dy_dtype == RK_F16 && dx_dtype == RK_F16)
    st = bwd_typed<__half, __half, __half>(x, ldx, w, rstd, dy, lddy, dx, lddx, dw_partial, parts, rows, W, s);
  else
    return RK_ERR_DTYPE;
  if (st != RK_OK) return st;
  rk_host::launch_k(rmsnorm_dw_reduce_kernel, (W + 31) / 32, 1024, 0, s, dw_partial, dw, parts, W, accumulate_dw);
  return rk_host::launch_status();
}


// ---------------------------------------------------------------- fused entry points
namespace {
template <typename Ta, typename Ty>
int add_fwd_typed(const float* x, const void* a, const float* w, void* y, float* sum_out, float* rstd, int64_t rows,
                  int width, float eps, cudaStream_t s) {
  const int nv = (width + 127) / 128;
  dim3 grid((unsigned)((rows + 7) / 8));
  auto A = static_cast<const Ta*>(a);
  auto Y = static_cast<Ty*>(y);
#define RK_AF(N) rk_host::launch_k(add_rmsnorm_fwd_kernel<Ta, Ty, N>, grid, 256, 0, s, x, A, w, Y, sum_out, rstd, rows, width, eps)
  if (nv <= 1) RK_AF(1);
  else if (nv <= 2) RK_AF(2);
  else if (nv <= 4) RK_AF(4);
  else if (nv <= 8) RK_AF(8);
  else return RK_ERR_UNSUPPORTED;
#undef RK_AF
  return rk_host::launch_status();
}

template <typename Tg, typename Tlp, bool RES, int LP>
int bwd_fused_nv(const float* x, const float* w, const float* rstd, const void* dy, const float* residual,
                 const void* lp_add, float* dx_out, void* lp_out, float* partial, int parts, int64_t rows, int width,
                 float lp_scale, cudaStream_t s) {
  const int nv = (width + 127) / 128;
  const size_t smem = (size_t)8 * width * sizeof(float);
  auto G = static_cast<const Tg*>(dy);
  auto LA = static_cast<const Tlp*>(lp_add);
  auto LO = static_cast<Tlp*>(lp_out);
#define RK_BF(N)                                                                                            \
  do {                                                                                                      \
    auto k = rmsnorm_bwd_fused_kernel<Tg, Tlp, N, RES, LP>;                                                 \
    if (smem > 48 * 1024) { if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)smem)) return e_; }          \
    rk_host::launch_k(k, parts, 256, smem, s, x, w, rstd, G, residual, LA, dx_out, LO, partial, rows, width, lp_scale);    \
  } while (0)
  if (nv <= 1) RK_BF(1);
  else if (nv <= 2) RK_BF(2);
  else if (nv <= 4) RK_BF(4);
  else if (nv <= 8) RK_BF(8);
  else return RK_ERR_UNSUPPORTED;
#undef RK_BF
  return rk_host::launch_status();
}

template <typename Tg, typename Tlp>
int bwd_fused_modes(const float* x, const float* w, const float* rstd, const void* dy, const float* residual,
                    const void* lp_add, float* dx_out, void* lp_out, float* partial, int parts, int64_t rows,
                    int width, float lp_scale, cudaStream_t s) {
  const bool res = residual != nullptr;
  const int lp = lp_out == nullptr ? 0 : (lp_add != nullptr ? 1 : 2);
#define RK_M(R, L)                                                                                           \
  if (res == R && lp == L)                                                                                   \
    return bwd_fused_nv<Tg, Tlp, R, L>(x, w, rstd, dy, residual, lp_add, dx_out, lp_out, partial, parts, rows, \
                                       width, lp_scale, s);
  RK_M(false, 0) RK_M(false, 1) RK_M(false, 2) RK_M(true, 0) RK_M(true, 1) RK_M(true, 2)
#undef RK_M
  return RK_ERR_ARG;
}
}  // namespace

extern "C" int rk_add_rmsnorm_fwd(const float* x, const void* a, int a_dtype, const float* w, void* y, int y_dtype,
                                  float* sum_out, float* rstd, int64_t rows, int64_t width, float eps, void* stream) {
  if (rows < 0 || width <= 0) return RK_ERR_ARG;
  if (width > 1024) return RK_ERR_UNSUPPORTED;
  if (rows == 0) return RK_OK;  // nothing is read or written, so the pointers may be null
  if (!x || !a || !w || !y) return RK_ERR_ARG;
  if (width % 4 || !rk_host::aligned(x, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(a, 8) ||
      !rk_host::aligned(y, 8) || (sum_out && !rk_host::aligned(sum_out, 16)))
    return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = (int)width;
  if (a_dtype == RK_BF16 && y_dtype == RK_BF16)
    return add_fwd_typed<__nv_bfloat16, __nv_bfloat16>(x, a, w, y, sum_out, rstd, rows, W, eps, s);
  if (a_dtype == RK_F16 && y_dtype == RK_F16)
    return add_fwd_typed<__half, __half>(x, a, w, y, sum_out, rstd, rows, W, eps, s);
  if (a_dtype == RK_F32 && y_dtype == RK_F32)
    return add_fwd_typed<float, float>(x, a, w, y, sum_out, rstd, rows, W, eps, s);
  return RK_ERR_DTYPE;
}

extern "C" int rk_rmsnorm_bwd_fused(const float* x, const float* w, const float* rstd, const void* dy, int dy_dtype,
                                    const float* residual, const void* lp_add, void* lp_out, int lp_dtype,
                                    float lp_scale, float* dx_out, float* dw, int accumulate_dw, float* dw_partial,
                                    int64_t workspace_bytes, int64_t rows, int64_t width, void* stream) {
  if (rows < 0 || width <= 0) return RK_ERR_ARG;
  if (lp_add && !lp_out) return RK_ERR_ARG;
  if (width > 1024) return RK_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = (int)width;
  if (rows == 0) {  // dw = 0 (or unchanged); the row pointers and the workspace may be null
    if (!dw || accumulate_dw) return RK_OK;
    cudaMemsetAsync(dw, 0, sizeof(float) * W, s);
    return rk_host::launch_status();
  }
  if (!x || !w || !rstd || !dy || !dx_out || !dw_partial) return RK_ERR_ARG;
  if (width % 4 || !rk_host::aligned(x, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(dx_out, 16) ||
      (residual && !rk_host::aligned(residual, 16)) || !rk_host::aligned(dy, 8) ||
      (lp_add && !rk_host::aligned(lp_add, 8)) || (lp_out && !rk_host::aligned(lp_out, 8)))
    return RK_ERR_ALIGN;
  const int parts = rms_parts(rows);
  if (workspace_bytes < (int64_t)parts * W * (int64_t)sizeof(float)) return RK_ERR_WORKSPACE;
  int st;
  const int lpd = lp_out ? lp_dtype : dy_dtype;
  if (dy_dtype == RK_BF16 && lpd == RK_BF16)
    st = bwd_fused_modes<__nv_bfloat16, __nv_bfloat16>(x, w, rstd, dy, residual, lp_add, dx_out, lp_out, dw_partial,
                                                      parts, rows, W, lp_scale, s);
  else if (dy_dtype == RK_F16 && lpd == RK_F16)
    st = bwd_fused_modes<__half, __half>(x, w, rstd, dy, residual, lp_add, dx_out, lp_out, dw_partial, parts, rows, W,
                                        lp_scale, s);
  else if (dy_dtype == RK_F32 && lpd == RK_F32)
    st = bwd_fused_modes<float, float>(x, w, rstd, dy, residual, lp_add, dx_out, lp_out, dw_partial, parts, rows, W,
                                       lp_scale, s);
  else
    return RK_ERR_DTYPE;
  if (st != RK_OK) return st;
  if (!dw) return RK_OK;  // partials left for rk_rmsnorm_dw_reduce
  rk_host::launch_k(rmsnorm_dw_reduce_kernel, (W + 31) / 32, 1024, 0, s, dw_partial, dw, parts, W, accumulate_dw);
  return rk_host::launch_status();
}

extern "C" int rk_rmsnorm_dw_reduce(const float* dw_partial, int64_t rows, int64_t width, float* dw,
                                    int accumulate_dw, void* stream) {
  if (!dw || rows < 0 || width <= 0) return RK_ERR_ARG;
  if (width > 1024) return RK_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = (int)width;
  if (rows == 0) {  // no partials were written: dw = 0 (or unchanged); dw_partial may be null
    if (accumulate_dw) return RK_OK;
    cudaMemsetAsync(dw, 0, sizeof(float) * W, s);
    return rk_host::launch_status();
  }
  if (!dw_partial) return RK_ERR_ARG;
  rk_host::launch_k(rmsnorm_dw_reduce_kernel, (W + 31) / 32, 1024, 0, s, dw_partial, dw, rms_parts(rows), W,
                    accumulate_dw);
  return rk_host::launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free variant of rk_rmsnorm_bwd.
//
// Some callers cannot hand the library a workspace: a host runtime reaching
// this library through a foreign-function binding with no device allocator of
// its own, or a plugin inside a framework whose caching allocator owns all
// device memory and hands none to third-party libraries. For them the
// weight-gradient partials live in this file-scope device array instead, sized
// for the largest request the kernel accepts: up to 592 partial rows (the
// backward uses one per CTA, at most 296 today) x 1024 columns of fp32 =
// 2,424,832 bytes, held by every GPU that loads the library until the process
// exits.
namespace {
constexpr int64_t kNoallocMaxWidth = 1024;
constexpr int64_t kNoallocScratchFloats = 592 * kNoallocMaxWidth;
static __device__ __align__(256) float g_rmsnorm_noalloc_scratch[kNoallocScratchFloats];

constexpr int kNoallocMaxDevices = 64;
float* g_noalloc_ptr[kNoallocMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device. In host code the
// array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
float* noalloc_scratch(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) {
    *status = RK_ERR_LAUNCH;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    float* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_rmsnorm_noalloc_scratch) != cudaSuccess || !p) {
      *status = RK_ERR_LAUNCH;
      return nullptr;
    }
    g_noalloc_ptr[dev] = p;
  }
  *status = RK_OK;
  return g_noalloc_ptr[dev];
}
}  // namespace

extern "C" int rk_rmsnorm_bwd_noalloc(const void* x, int x_dtype, int64_t ldx, const float* w, const float* rstd,
                                      const void* dy, int dy_dtype, int64_t lddy, void* dx, int dx_dtype,
                                      int64_t lddx, float* dw, int accumulate_dw, int64_t rows, int64_t width,
                                      void* stream) {
  if (width > kNoallocMaxWidth) return RK_ERR_SCRATCH;
  if (rows < 0 || width <= 0) return RK_ERR_ARG;
  const int64_t need = rk_rmsnorm_bwd_workspace(rows, width);
  if (need > kNoallocScratchFloats * (int64_t)sizeof(float)) return RK_ERR_SCRATCH;
  int st = RK_OK;
  float* scratch = noalloc_scratch(&st);
  if (!scratch) return st;
  // Every partial row the kernel reads is written earlier in the same call, so
  // stale contents from a previous call need no clearing.
  return rk_rmsnorm_bwd(x, x_dtype, ldx, w, rstd, dy, dy_dtype, lddy, dx, dx_dtype, lddx, dw, accumulate_dw,
                        scratch, kNoallocScratchFloats * (int64_t)sizeof(float), rows, width, stream);
}
