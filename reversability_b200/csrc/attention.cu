// Causal self-attention forward/backward for the recompute (replaces
// F.scaled_dot_product_attention(q, k, v, is_causal=True) at model.py:42-44).
//
// Layout: qkv is the packed output of the qkv Linear, [B*T, 3*D] row-major
// with D = H*HD: q at columns h*HD, k at D + h*HD, v at 2D + h*HD. The output
// o is [B*T, D] (head h at columns h*HD), i.e. exactly the tensor the proj
// Linear consumes, so no transposes are needed anywhere. lse holds the
// per-row log-sum-exp in base 2 ([B, H, T], fp32) for the backward.
//
// bf16/f16 kernels: flash-style tiles of 64 queries x 64 keys per CTA
// iteration, four warps of 16 query rows, mma.sync m16n8k16 with fp32
// accumulation, online softmax in registers, K/V double-buffered through
// shared memory with cp.async. At head_dim 32 the bound is the exponential
// unit (one ex2 per score against 128 MMA flops per score), not the tensor
// pipe. The backward is deterministic: one kernel per query block produces
// dQ (and D = rowsum(dO*O) for its rows), a second kernel per key block
// produces dK and dV; no atomics.
//
// fp32 kernels: CUDA-core versions (one warp per row) for the fp32 parity
// configuration.
#include <cstdlib>
#include "common.cuh"

namespace rk {
namespace attn {

constexpr int BQ = 64;  // query rows per CTA
constexpr int BKV = 64; // keys per iteration

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Copies rows [row0, row0+64) x HD columns starting at `col` of a [Tlen, ld]
// matrix into smem (row stride LD); rows >= Tlen are zero-filled.
template <typename T, int HD, int LD, int NT>
__device__ __forceinline__ void load_tile(T* dst, const T* base, int64_t ld, int row0, int col, int Tlen) {
  constexpr int CH = HD / 8;
  for (int i = threadIdx.x; i < 64 * CH; i += NT) {
    const int r = i / CH, c = i - (i / CH) * CH;
    const int gr = row0 + r;
    const int sr = gr < Tlen ? gr : (Tlen - 1);
    cp_async16(smem_u32(dst + r * LD + c * 8), base + (int64_t)sr * ld + col + c * 8, gr < Tlen ? 16 : 0);
  }
}

// A fragments (16 rows x HD) of a row-major smem tile for warp rows [r0, r0+16).
template <typename T, int HD, int LD>
__device__ __forceinline__ void load_a_frags(uint32_t (&a)[HD / 16][4], const T* tile, int r0, int lane) {
#pragma unroll
  for (int kc = 0; kc < HD / 16; ++kc)
    ldsm_x4(a[kc], smem_u32(tile + (r0 + (lane & 7) + 8 * ((lane >> 3) & 1)) * LD + kc * 16 + 8 * (lane >> 4)));
}

// acc[8][4] (16 rows x 64 cols) += A(16 x HD) * Rows^T where Rows is a
// 64 x HD smem tile (B operand read without transpose).
template <typename T, int HD, int LD>
__device__ __forceinline__ void mma_abT(float (&acc)[8][4], const uint32_t (&a)[HD / 16][4], const T* rows,
                                        int lane) {
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int kp = 0; kp < HD / 32; ++kp) {
      uint32_t b[4];
      ldsm_x4(b, smem_u32(rows + (nt * 8 + (lane & 7)) * LD + kp * 32 + 8 * (lane >> 3)));
      Mma<T>::run(acc[nt], a[2 * kp], b[0], b[1]);
      Mma<T>::run(acc[nt], a[2 * kp + 1], b[2], b[3]);
    }
  }
}

// out[HD/8][4] (16 rows x HD) += P(16 x 64, from accumulator registers) * Tile
// where Tile is a 64 x HD smem tile (B operand read with transpose).
template <typename T, int HD, int LD>
__device__ __forceinline__ void mma_pv(float (&out)[HD / 8][4], const float (&p)[8][4], const T* tile, int lane) {
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
    uint32_t a[4];
    a[0] = Mma<T>::pack(p[2 * kc][0], p[2 * kc][1]);
    a[1] = Mma<T>::pack(p[2 * kc][2], p[2 * kc][3]);
    a[2] = Mma<T>::pack(p[2 * kc + 1][0], p[2 * kc + 1][1]);
    a[3] = Mma<T>::pack(p[2 * kc + 1][2], p[2 * kc + 1][3]);
#pragma unroll
    for (int np = 0; np < HD / 16; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, smem_u32(tile + (kc * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * LD + np * 16 + 8 * (lane >> 4)));
      Mma<T>::run(out[2 * np], a, b[0], b[1]);
      Mma<T>::run(out[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// ------------------------------------------------------------------ forward
template <typename T, int HD>
__global__ void __launch_bounds__(128) fwd_kernel(const T* __restrict__ qkv, T* __restrict__ out,
                                                  float* __restrict__ lse, int H, int Tlen, int64_t ldq, int64_t ldo,
                                                  float c_log2) {
  pdl_wait();  // inputs are the previous kernel's outputs
  constexpr int LD = HD + 8;
  __shared__ __align__(16) T Qs[BQ * LD];
  __shared__ __align__(16) T Ks[2][BKV * LD];
  __shared__ __align__(16) T Vs[2][BKV * LD];
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest rows first
  const int b = blockIdx.y / H, h = blockIdx.y - (blockIdx.y / H) * H;
  const int D = H * HD;
  const T* base = qkv + (int64_t)b * Tlen * ldq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int q0 = qb * BQ;

  load_tile<T, HD, LD, 128>(Qs, base, ldq, q0, h * HD, Tlen);
  load_tile<T, HD, LD, 128>(Ks[0], base, ldq, 0, D + h * HD, Tlen);
  load_tile<T, HD, LD, 128>(Vs[0], base, ldq, 0, 2 * D + h * HD, Tlen);
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[HD / 16][4];
  const int nkb = qb + 1;
  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<T, HD, LD, 128>(Ks[buf ^ 1], base, ldq, (j + 1) * BKV, D + h * HD, Tlen);
      load_tile<T, HD, LD, 128>(Vs[buf ^ 1], base, ldq, (j + 1) * BKV, 2 * D + h * HD, Tlen);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) load_a_frags<T, HD, LD>(qa, Qs, warp * 16, lane);
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    mma_abT<T, HD, LD>(s, qa, Ks[buf], lane);
    if (j == qb) {  // diagonal block: key > query is masked
      const int r_lo = warp * 16 + g;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int k = nt * 8 + 2 * tig;
        if (k > r_lo) s[nt][0] = -INFINITY;
        if (k + 1 > r_lo) s[nt][1] = -INFINITY;
        if (k > r_lo + 8) s[nt][2] = -INFINITY;
        if (k + 1 > r_lo + 8) s[nt][3] = -INFINITY;
      }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = ex2((m0 - mx0) * c_log2), a1 = ex2((m1 - mx1) * c_log2);
    const float mc0 = mx0 * c_log2, mc1 = mx1 * c_log2;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = ex2(fmaf(s[nt][0], c_log2, -mc0));
      s[nt][1] = ex2(fmaf(s[nt][1], c_log2, -mc0));
      s[nt][2] = ex2(fmaf(s[nt][2], c_log2, -mc1));
      s[nt][3] = ex2(fmaf(s[nt][3], c_log2, -mc1));
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
    m0 = mx0;
    m1 = mx1;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
    mma_pv<T, HD, LD>(o, s, Vs[buf], lane);
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  const int r_lo = q0 + warp * 16 + g, r_hi = r_lo + 8;
  T* ob = out + (int64_t)b * Tlen * ldo + h * HD;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int c = i * 8 + 2 * tig;
    if (r_lo < Tlen) *reinterpret_cast<uint32_t*>(ob + (int64_t)r_lo * ldo + c) = Mma<T>::pack(o[i][0] * i0, o[i][1] * i0);
    if (r_hi < Tlen) *reinterpret_cast<uint32_t*>(ob + (int64_t)r_hi * ldo + c) = Mma<T>::pack(o[i][2] * i1, o[i][3] * i1);
  }
  if (tig == 0) {
    float* lb = lse + ((int64_t)b * H + h) * Tlen;
    if (r_lo < Tlen) lb[r_lo] = m0 * c_log2 + __log2f(l0);
    if (r_hi < Tlen) lb[r_hi] = m1 * c_log2 + __log2f(l1);
  }
}

// ------------------------------------------------------------------ backward: dQ (+ D)
template <typename T, int HD>
__global__ void __launch_bounds__(128) bwd_dq_kernel(const T* __restrict__ qkv, const T* __restrict__ o,
                                                     const T* __restrict__ dout, const float* __restrict__ lse,
                                                     float* __restrict__ dsum, T* __restrict__ dqkv, int H,
                                                     int Tlen, int64_t ldq, int64_t ldo, int64_t lddq, float c_log2,
                                                     float scale, int have_dsum) {
  pdl_wait();  // inputs are the previous kernel's outputs
  constexpr int LD = HD + 8;
  extern __shared__ __align__(16) unsigned char dsm[];  // 6 tiles of 64 x LD
  T* Qs = reinterpret_cast<T*>(dsm);
  T* dOs = Qs + BQ * LD;
  T* const Ks0 = dOs + BQ * LD;       // two K buffers
  T* const Vs0 = Ks0 + 2 * BKV * LD;  // two V buffers
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y - (blockIdx.y / H) * H;
  const int D = H * HD;
  const T* base = qkv + (int64_t)b * Tlen * ldq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int q0 = qb * BQ;
  const int64_t bh = (int64_t)b * H + h;

  load_tile<T, HD, LD, 128>(Qs, base, ldq, q0, h * HD, Tlen);
  load_tile<T, HD, LD, 128>(dOs, dout + (int64_t)b * Tlen * ldo, ldo, q0, h * HD, Tlen);
  load_tile<T, HD, LD, 128>(Ks0, base, ldq, 0, D + h * HD, Tlen);
  load_tile<T, HD, LD, 128>(Vs0, base, ldq, 0, 2 * D + h * HD, Tlen);
  cp_async_commit();

  // D = rowsum(dO * O) for this CTA's rows: 2 threads per row (unless
  // dsum_kernel has written it already).
  if (!have_dsum) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    const int gr = q0 + r;
    float acc = 0.f;
    if (gr < Tlen) {
      const T* orow = o + ((int64_t)b * Tlen + gr) * ldo + h * HD + half * (HD / 2);
      const T* drow = dout + ((int64_t)b * Tlen + gr) * ldo + h * HD + half * (HD / 2);
#pragma unroll
      for (int c = 0; c < HD / 2; ++c) acc += Dt<T>::to_f(orow[c]) * Dt<T>::to_f(drow[c]);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (gr < Tlen && half == 0) dsum[bh * Tlen + gr] = acc;
  }
  __syncthreads();

  const int r_lo = warp * 16 + g;
  const int gr_lo = q0 + r_lo, gr_hi = gr_lo + 8;
  const float* lb = lse + bh * Tlen;
  const float* db = dsum + bh * Tlen;
  const float lse0 = gr_lo < Tlen ? lb[gr_lo] : 0.f, lse1 = gr_hi < Tlen ? lb[gr_hi] : 0.f;
  const float d0 = gr_lo < Tlen ? db[gr_lo] : 0.f, d1 = gr_hi < Tlen ? db[gr_hi] : 0.f;

  float dq[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  uint32_t qa[HD / 16][4], da[HD / 16][4];
  const int nkb = qb + 1;
  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<T, HD, LD, 128>(Ks0 + (buf ^ 1) * BKV * LD, base, ldq, (j + 1) * BKV, D + h * HD, Tlen);
      load_tile<T, HD, LD, 128>(Vs0 + (buf ^ 1) * BKV * LD, base, ldq, (j + 1) * BKV, 2 * D + h * HD, Tlen);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
      load_a_frags<T, HD, LD>(qa, Qs, warp * 16, lane);
      load_a_frags<T, HD, LD>(da, dOs, warp * 16, lane);
    }
    float s[8][4], dp[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      dp[nt][0] = dp[nt][1] = dp[nt][2] = dp[nt][3] = 0.f;
    }
    mma_abT<T, HD, LD>(s, qa, Ks0 + buf * BKV * LD, lane);
    mma_abT<T, HD, LD>(dp, da, Vs0 + buf * BKV * LD, lane);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int k = j * BKV + nt * 8 + 2 * tig;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kk = k + (e & 1);
        const int qq = (e < 2) ? gr_lo : gr_hi;
        const float l_ = (e < 2) ? lse0 : lse1;
        const float d_ = (e < 2) ? d0 : d1;
        const float p = (kk > qq) ? 0.f : ex2(fmaf(s[nt][e], c_log2, -l_));
        s[nt][e] = p * (dp[nt][e] - d_);  // dS
      }
    }
    // dQ += dS * K
    mma_pv<T, HD, LD>(dq, s, Ks0 + buf * BKV * LD, lane);
    __syncthreads();
  }
  T* out = dqkv + (int64_t)b * Tlen * lddq + h * HD;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int c = i * 8 + 2 * tig;
    if (gr_lo < Tlen) *reinterpret_cast<uint32_t*>(out + (int64_t)gr_lo * lddq + c) = Mma<T>::pack(dq[i][0] * scale, dq[i][1] * scale);
    if (gr_hi < Tlen) *reinterpret_cast<uint32_t*>(out + (int64_t)gr_hi * lddq + c) = Mma<T>::pack(dq[i][2] * scale, dq[i][3] * scale);
  }
}

// ------------------------------------------------------------------ backward: D alone
// D[b, h, t] = rowsum(dO * O) over the head's HD columns, one thread per
// (row, head), so the dQ and dK/dV kernels can run side by side.
template <typename T, int HD>
__global__ void __launch_bounds__(256) dsum_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                                   float* __restrict__ dsum, int H, int Tlen, int64_t rows,
                                                   int64_t ldo) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (b*T + t)*H + h
  if (i >= rows * H) return;
  const int64_t bt = i / H;
  const int h = (int)(i - bt * H);
  const T* orow = o + bt * ldo + h * HD;
  const T* drow = dout + bt * ldo + h * HD;
  // two halves summed separately, then added: the order bwd_dq_kernel uses,
  // so both ways of producing D give the same bits
  float acc[2] = {0.f, 0.f};
#pragma unroll
  for (int c = 0; c < HD; c += 8) {
    const uint4 a = *reinterpret_cast<const uint4*>(orow + c);
    const uint4 d = *reinterpret_cast<const uint4*>(drow + c);
    const T* ae = reinterpret_cast<const T*>(&a);
    const T* de = reinterpret_cast<const T*>(&d);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[c >= HD / 2] += Dt<T>::to_f(ae[e]) * Dt<T>::to_f(de[e]);
  }
  const int64_t b = bt / Tlen, t = bt - b * Tlen;
  dsum[(b * H + h) * Tlen + t] = acc[0] + acc[1];
}

// ------------------------------------------------------------------ backward: dK, dV
template <typename T, int HD>
__global__ void __launch_bounds__(128, HD <= 32 ? 4 : 1) bwd_dkv_kernel(const T* __restrict__ qkv, const T* __restrict__ dout,
                                                      const float* __restrict__ lse, const float* __restrict__ dsum,
                                                      T* __restrict__ dqkv, int H, int Tlen, int64_t ldq,
                                                      int64_t ldo, int64_t lddq, float c_log2, float scale) {
  pdl_wait();  // inputs are the previous kernel's outputs
  constexpr int LD = HD + 8;
  extern __shared__ __align__(16) unsigned char dsm[];  // 6 tiles of 64 x LD, then 4 x 64 floats
  T* Ks = reinterpret_cast<T*>(dsm);
  T* Vs = Ks + BKV * LD;
  T* const Qs0 = Vs + BKV * LD;     // two Q buffers
  T* const dOs0 = Qs0 + 2 * BQ * LD;  // two dO buffers
  float (*Ls)[BQ] = reinterpret_cast<float (*)[BQ]>(dOs0 + 2 * BQ * LD);
  float (*Ds)[BQ] = Ls + 2;
  const int nqb = gridDim.x;
  const int kb = blockIdx.x;  // small kb = most work; launched first
  const int b = blockIdx.y / H, h = blockIdx.y - (blockIdx.y / H) * H;
  const int D = H * HD;
  const T* base = qkv + (int64_t)b * Tlen * ldq;
  const T* dbase = dout + (int64_t)b * Tlen * ldo;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int k0 = kb * BKV;
  const int64_t bh = (int64_t)b * H + h;
  const float* lb = lse + bh * Tlen;
  const float* db = dsum + bh * Tlen;

  auto load_q_block = [&](int i, int buf) {
    load_tile<T, HD, LD, 128>(Qs0 + buf * BQ * LD, base, ldq, i * BQ, h * HD, Tlen);
    load_tile<T, HD, LD, 128>(dOs0 + buf * BQ * LD, dbase, ldo, i * BQ, h * HD, Tlen);
    if (threadIdx.x < BQ) {
      const int gr = i * BQ + threadIdx.x;
      Ls[buf][threadIdx.x] = gr < Tlen ? lb[gr] : INFINITY;  // rows past the end contribute nothing
      Ds[buf][threadIdx.x] = gr < Tlen ? db[gr] : 0.f;
    }
  };
  load_tile<T, HD, LD, 128>(Ks, base, ldq, k0, D + h * HD, Tlen);
  load_tile<T, HD, LD, 128>(Vs, base, ldq, k0, 2 * D + h * HD, Tlen);
  load_q_block(kb, 0);
  cp_async_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  uint32_t ka[HD / 16][4], va[HD / 16][4];
  const int key_lo = k0 + warp * 16 + g, key_hi = key_lo + 8;
  for (int i = kb; i < nqb; ++i) {
    const int buf = (i - kb) & 1;
    if (i + 1 < nqb) load_q_block(i + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (i == kb) {
      load_a_frags<T, HD, LD>(ka, Ks, warp * 16, lane);
      load_a_frags<T, HD, LD>(va, Vs, warp * 16, lane);
    }
    // S^T (16 keys x 64 queries) and dP^T.
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      st[nt][0] = st[nt][1] = st[nt][2] = st[nt][3] = 0.f;
      dpt[nt][0] = dpt[nt][1] = dpt[nt][2] = dpt[nt][3] = 0.f;
    }
    mma_abT<T, HD, LD>(st, ka, Qs0 + buf * BQ * LD, lane);
    mma_abT<T, HD, LD>(dpt, va, dOs0 + buf * BQ * LD, lane);
    // in place: st becomes P^T, dpt becomes dS^T (no third tile of registers)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int qc = nt * 8 + 2 * tig;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = qc + (e & 1);
        const int qq = i * BQ + qi;
        const int kk = (e < 2) ? key_lo : key_hi;
        const float p = (qq < kk) ? 0.f : ex2(fmaf(st[nt][e], c_log2, -Ls[buf][qi]));
        st[nt][e] = p;
        dpt[nt][e] = p * (dpt[nt][e] - Ds[buf][qi]);  // dS^T
      }
    }
    mma_pv<T, HD, LD>(dv, st, dOs0 + buf * BQ * LD, lane);
    mma_pv<T, HD, LD>(dk, dpt, Qs0 + buf * BQ * LD, lane);
    __syncthreads();
  }
  T* out = dqkv + (int64_t)b * Tlen * lddq;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int c = i * 8 + 2 * tig;
    if (key_lo < Tlen) {
      *reinterpret_cast<uint32_t*>(out + (int64_t)key_lo * lddq + D + h * HD + c) = Mma<T>::pack(dk[i][0] * scale, dk[i][1] * scale);
      *reinterpret_cast<uint32_t*>(out + (int64_t)key_lo * lddq + 2 * D + h * HD + c) = Mma<T>::pack(dv[i][0], dv[i][1]);
    }
    if (key_hi < Tlen) {
      *reinterpret_cast<uint32_t*>(out + (int64_t)key_hi * lddq + D + h * HD + c) = Mma<T>::pack(dk[i][2] * scale, dk[i][3] * scale);
      *reinterpret_cast<uint32_t*>(out + (int64_t)key_hi * lddq + 2 * D + h * HD + c) = Mma<T>::pack(dv[i][2], dv[i][3]);
    }
  }
}

// ------------------------------------------------------------------ fp32 CUDA-core kernels
// One warp per (query row, b, h): scores in a strided loop over keys, exact
// softmax (two passes), then out = sum p * v with lanes over head_dim.
__global__ void __launch_bounds__(128) fwd_f32_kernel(const float* __restrict__ qkv, float* __restrict__ out,
                                                      float* __restrict__ lse, int H, int HD, int Tlen, int64_t ldq,
                                                      int64_t ldo, float scale) {
  pdl_wait();  // inputs are the previous kernel's outputs
  extern __shared__ float sm[];  // [4 warps][Tlen] scores
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  if (row >= Tlen) return;
  const int D = H * HD;
  const float* base = qkv + (int64_t)b * Tlen * ldq;
  const float* q = base + (int64_t)row * ldq + h * HD;
  float* sc = sm + warp * Tlen;
  float mx = -INFINITY;
  for (int k = lane; k <= row; k += 32) {
    const float* kr = base + (int64_t)k * ldq + D + h * HD;
    float s = 0.f;
    for (int c = 0; c < HD; ++c) s = fmaf(q[c], kr[c], s);
    s *= scale;
    sc[k] = s;
    mx = fmaxf(mx, s);
  }
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int k = lane; k <= row; k += 32) {
    const float p = expf(sc[k] - mx);
    sc[k] = p;
    sum += p;
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncwarp();
  const float inv = 1.f / sum;
  for (int c = lane; c < HD; c += 32) {
    float acc = 0.f;
    for (int k = 0; k <= row; ++k) acc = fmaf(sc[k], base[(int64_t)k * ldq + 2 * D + h * HD + c], acc);
    out[((int64_t)b * Tlen + row) * ldo + h * HD + c] = acc * inv;
  }
  if (lane == 0) lse[((int64_t)b * H + h) * Tlen + row] = mx + logf(sum);  // natural log for the fp32 path
}

// dQ rows and D: one warp per query row.
__global__ void __launch_bounds__(128) bwd_dq_f32_kernel(const float* __restrict__ qkv, const float* __restrict__ o,
                                                         const float* __restrict__ dout,
                                                         const float* __restrict__ lse, float* __restrict__ dsum,
                                                         float* __restrict__ dqkv, int H, int HD, int Tlen,
                                                         int64_t ldq, int64_t ldo, int64_t lddq, float scale) {
  pdl_wait();  // inputs are the previous kernel's outputs
  extern __shared__ float sm[];  // [4][Tlen] dS
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  if (row >= Tlen) return;
  const int D = H * HD;
  const float* base = qkv + (int64_t)b * Tlen * ldq;
  const float* q = base + (int64_t)row * ldq + h * HD;
  const float* dor = dout + ((int64_t)b * Tlen + row) * ldo + h * HD;
  const float* orow = o + ((int64_t)b * Tlen + row) * ldo + h * HD;
  float dd = 0.f;
  for (int c = lane; c < HD; c += 32) dd += dor[c] * orow[c];
  for (int s = 16; s; s >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, s);
  const int64_t bh = (int64_t)b * H + h;
  if (lane == 0) dsum[bh * Tlen + row] = dd;
  const float L = lse[bh * Tlen + row];
  float* ds = sm + warp * Tlen;
  for (int k = lane; k <= row; k += 32) {
    const float* kr = base + (int64_t)k * ldq + D + h * HD;
    const float* vr = base + (int64_t)k * ldq + 2 * D + h * HD;
    float s = 0.f, dp = 0.f;
    for (int c = 0; c < HD; ++c) {
      s = fmaf(q[c], kr[c], s);
      dp = fmaf(dor[c], vr[c], dp);
    }
    const float p = expf(s * scale - L);
    ds[k] = p * (dp - dd);
  }
  __syncwarp();
  for (int c = lane; c < HD; c += 32) {
    float acc = 0.f;
    for (int k = 0; k <= row; ++k) acc = fmaf(ds[k], base[(int64_t)k * ldq + D + h * HD + c], acc);
    dqkv[((int64_t)b * Tlen + row) * lddq + h * HD + c] = acc * scale;
  }
}

// dK, dV rows: one warp per key row.
__global__ void __launch_bounds__(128) bwd_dkv_f32_kernel(const float* __restrict__ qkv,
                                                          const float* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          const float* __restrict__ dsum, float* __restrict__ dqkv,
                                                          int H, int HD, int Tlen, int64_t ldq, int64_t ldo,
                                                          int64_t lddq, float scale) {
  pdl_wait();  // inputs are the previous kernel's outputs
  extern __shared__ float sm[];  // [4][2][Tlen]: p and dS per query
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int key = blockIdx.x * 4 + warp;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  if (key >= Tlen) return;
  const int D = H * HD;
  const float* base = qkv + (int64_t)b * Tlen * ldq;
  const float* kr = base + (int64_t)key * ldq + D + h * HD;
  const float* vr = base + (int64_t)key * ldq + 2 * D + h * HD;
  const int64_t bh = (int64_t)b * H + h;
  float* ps = sm + warp * 2 * Tlen;
  float* dss = ps + Tlen;
  for (int qi = key + lane; qi < Tlen; qi += 32) {
    const float* q = base + (int64_t)qi * ldq + h * HD;
    const float* dor = dout + ((int64_t)b * Tlen + qi) * ldo + h * HD;
    float s = 0.f, dp = 0.f;
    for (int c = 0; c < HD; ++c) {
      s = fmaf(q[c], kr[c], s);
      dp = fmaf(dor[c], vr[c], dp);
    }
    const float p = expf(s * scale - lse[bh * Tlen + qi]);
    ps[qi] = p;
    dss[qi] = p * (dp - dsum[bh * Tlen + qi]);
  }
  __syncwarp();
  for (int c = lane; c < HD; c += 32) {
    float ak = 0.f, av = 0.f;
    for (int qi = key; qi < Tlen; ++qi) {
      ak = fmaf(dss[qi], base[(int64_t)qi * ldq + h * HD + c], ak);
      av = fmaf(ps[qi], dout[((int64_t)b * Tlen + qi) * ldo + h * HD + c], av);
    }
    dqkv[((int64_t)b * Tlen + key) * lddq + D + h * HD + c] = ak * scale;
    dqkv[((int64_t)b * Tlen + key) * lddq + 2 * D + h * HD + c] = av;
  }
}

}  // namespace attn
}  // namespace rk

using namespace rk;
using namespace rk::attn;

int rk_attn_fwd_tc(const void* qkv, int64_t ldq, void* out, int64_t ldo, float* lse, int64_t B, int64_t H,
                   int64_t HD, int64_t T, int dtype, cudaStream_t s);
int rk_attn_bwd_tc(int piece, const void* qkv, int64_t ldq, const void* dout, int64_t ldo, const float* lse,
                   const float* dsum, void* dqkv, int64_t lddq, int64_t B, int64_t H, int64_t HD, int64_t T, int dtype,
                   cudaStream_t s);

namespace {

// Tensor-core forward for head_dim 32 and 64 (attention_tc.cu). REVK_ATTN_TC=0
// in the environment selects the mma.sync kernel instead (a tuning switch).
bool attn_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("REVK_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Tensor-core backward (attention_tc.cu); REVK_ATTN_BWD_TC=0 selects the
// mma.sync kernels (a tuning switch).
bool attn_bwd_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("REVK_ATTN_BWD_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool attn_args_ok(const void* a, const void* b, int64_t B, int64_t H, int64_t HD, int64_t T) {
  return a && b && B >= 0 && H > 0 && HD > 0 && T >= 0 && B * H < 65536 && T < (1 << 24);
}

template <typename T, int HD>
int fwd_tc(const void* qkv, void* out, float* lse, int B, int H, int Tlen, int64_t ldq, int64_t ldo, cudaStream_t s) {
  dim3 grid((Tlen + BQ - 1) / BQ, B * H);
  const float c_log2 = 1.4426950408889634f / sqrtf((float)HD);
  rk_host::launch_k(fwd_kernel<T, HD>, grid, 128, 0, s, static_cast<const T*>(qkv), static_cast<T*>(out), lse, H, Tlen, ldq, ldo,
                                         c_log2);
  return rk_host::launch_status();
}

template <typename T, int HD>
int bwd_piece(int piece, const void* qkv, const void* o, const void* dout, const float* lse, float* dsum, void* dqkv,
              int B, int H, int Tlen, int64_t ldq, int64_t ldo, int64_t lddq, cudaStream_t s);

template <typename T, int HD>
int bwd_tc(const void* qkv, const void* o, const void* dout, const float* lse, float* dsum, void* dqkv, int B, int H,
           int Tlen, int64_t ldq, int64_t ldo, int64_t lddq, cudaStream_t s) {
  if (attn_bwd_tc_enabled()) {  // D, then the tensor-core dQ and dK/dV kernels
    int st = bwd_piece<T, HD>(0, qkv, o, dout, lse, dsum, dqkv, B, H, Tlen, ldq, ldo, lddq, s);
    if (st) return st;
    const int dt = std::is_same_v<T, __nv_bfloat16> ? RK_BF16 : RK_F16;
    st = rk_attn_bwd_tc(1, qkv, ldq, dout, ldo, lse, dsum, dqkv, lddq, B, H, HD, Tlen, dt, s);
    if (st != RK_ERR_UNSUPPORTED) {
      if (st) return st;
      return rk_attn_bwd_tc(2, qkv, ldq, dout, ldo, lse, dsum, dqkv, lddq, B, H, HD, Tlen, dt, s);
    }
  }
  dim3 grid((Tlen + BQ - 1) / BQ, B * H);
  const float scale = 1.f / sqrtf((float)HD);
  const float c_log2 = 1.4426950408889634f * scale;
  constexpr int tile_bytes = 64 * (HD + 8) * (int)sizeof(T);
  constexpr int smem_dq = 6 * tile_bytes;
  constexpr int smem_dkv = 6 * tile_bytes + 4 * 64 * (int)sizeof(float);
  static_assert(smem_dkv <= 227 * 1024, "attention backward tiles exceed shared memory");
  if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dq_kernel<T, HD>), smem_dq)) return e_;
  if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dkv_kernel<T, HD>), smem_dkv)) return e_;
  rk_host::launch_k(bwd_dq_kernel<T, HD>, grid, 128, smem_dq, s, static_cast<const T*>(qkv), static_cast<const T*>(o),
                                            static_cast<const T*>(dout), lse, dsum, static_cast<T*>(dqkv), H, Tlen,
                                            ldq, ldo, lddq, c_log2, scale, 0);
  int st = rk_host::launch_status();
  if (st) return st;
  rk_host::launch_k(bwd_dkv_kernel<T, HD>, grid, 128, smem_dkv, s, static_cast<const T*>(qkv), static_cast<const T*>(dout), lse, dsum,
                                             static_cast<T*>(dqkv), H, Tlen, ldq, ldo, lddq, c_log2, scale);
  return rk_host::launch_status();
}

// The backward in three pieces for callers that run dQ and dK/dV on two streams:
// 0 = D (dsum_kernel), 1 = dQ (reading D), 2 = dK/dV.
template <typename T, int HD>
int bwd_piece(int piece, const void* qkv, const void* o, const void* dout, const float* lse, float* dsum, void* dqkv,
              int B, int H, int Tlen, int64_t ldq, int64_t ldo, int64_t lddq, cudaStream_t s) {
  dim3 grid((Tlen + BQ - 1) / BQ, B * H);
  const float scale = 1.f / sqrtf((float)HD);
  const float c_log2 = 1.4426950408889634f * scale;
  constexpr int tile_bytes = 64 * (HD + 8) * (int)sizeof(T);
  constexpr int smem_dq = 6 * tile_bytes;
  constexpr int smem_dkv = 6 * tile_bytes + 4 * 64 * (int)sizeof(float);
  if (piece != 0 && attn_bwd_tc_enabled()) {
    const int dt = std::is_same_v<T, __nv_bfloat16> ? RK_BF16 : RK_F16;
    const int st = rk_attn_bwd_tc(piece, qkv, ldq, dout, ldo, lse, dsum, dqkv, lddq, B, H, HD, Tlen, dt, s);
    if (st != RK_ERR_UNSUPPORTED) return st;
  }
  if (piece == 0) {
    const int64_t n = (int64_t)B * Tlen * H;
    rk_host::launch_k(dsum_kernel<T, HD>, (unsigned)((n + 255) / 256), 256, 0, s, static_cast<const T*>(o),
                      static_cast<const T*>(dout), dsum, H, Tlen, (int64_t)B * Tlen, ldo);
  } else if (piece == 1) {
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dq_kernel<T, HD>), smem_dq)) return e_;
    rk_host::launch_k(bwd_dq_kernel<T, HD>, grid, 128, smem_dq, s, static_cast<const T*>(qkv),
                      static_cast<const T*>(o), static_cast<const T*>(dout), lse, dsum, static_cast<T*>(dqkv), H,
                      Tlen, ldq, ldo, lddq, c_log2, scale, 1);
  } else {
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dkv_kernel<T, HD>), smem_dkv)) return e_;
    rk_host::launch_k(bwd_dkv_kernel<T, HD>, grid, 128, smem_dkv, s, static_cast<const T*>(qkv),
                      static_cast<const T*>(dout), lse, dsum, static_cast<T*>(dqkv), H, Tlen, ldq, ldo, lddq,
                      c_log2, scale);
  }
  return rk_host::launch_status();
}

bool tc_layout_ok(const void* a, const void* b, const void* c, int64_t ldq, int64_t ldo, int64_t HD) {
  return rk_host::aligned(a, 16) && rk_host::aligned(b, 16) && (!c || rk_host::aligned(c, 16)) && ldq % 8 == 0 &&
         ldo % 8 == 0 && (HD == 32 || HD == 64);
}

}  // namespace

extern "C" int rk_attn_fwd(const void* qkv, int64_t ldq, void* out, int64_t ldo, float* lse, int64_t B, int64_t H,
                           int64_t HD, int64_t T, int dtype, void* stream) {
  if (!attn_args_ok(qkv, out, B, H, HD, T) || !lse || ldq < 3 * H * HD || ldo < H * HD) return RK_ERR_ARG;
  if (B == 0 || T == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_F32) {
    dim3 grid((unsigned)((T + 3) / 4), (unsigned)(B * H));
    const size_t smem = 4 * T * sizeof(float);
    if (smem > 48 * 1024) { if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(fwd_f32_kernel), (int)smem)) return e_; }
    rk_host::launch_k(fwd_f32_kernel, grid, 128, smem, s, static_cast<const float*>(qkv), static_cast<float*>(out), lse, (int)H,
                                           (int)HD, (int)T, ldq, ldo, 1.f / sqrtf((float)HD));
    return rk_host::launch_status();
  }
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (!tc_layout_ok(qkv, out, nullptr, ldq, ldo, HD)) return (HD == 32 || HD == 64) ? RK_ERR_ALIGN : RK_ERR_UNSUPPORTED;
  if (attn_tc_enabled()) {
    const int st = rk_attn_fwd_tc(qkv, ldq, out, ldo, lse, B, H, HD, T, dtype, s);
    if (st != RK_ERR_UNSUPPORTED) return st;
  }
  if (dtype == RK_BF16)
    return HD == 32 ? fwd_tc<__nv_bfloat16, 32>(qkv, out, lse, (int)B, (int)H, (int)T, ldq, ldo, s)
                    : fwd_tc<__nv_bfloat16, 64>(qkv, out, lse, (int)B, (int)H, (int)T, ldq, ldo, s);
  return HD == 32 ? fwd_tc<__half, 32>(qkv, out, lse, (int)B, (int)H, (int)T, ldq, ldo, s)
                  : fwd_tc<__half, 64>(qkv, out, lse, (int)B, (int)H, (int)T, ldq, ldo, s);
}

extern "C" int rk_attn_bwd(const void* qkv, int64_t ldq, const void* out, const void* dout, int64_t ldo,
                           const float* lse, float* dsum, void* dqkv, int64_t lddq, int64_t B, int64_t H, int64_t HD,
                           int64_t T, int dtype, void* stream) {
  if (!attn_args_ok(qkv, out, B, H, HD, T) || !dout || !lse || !dsum || !dqkv || ldq < 3 * H * HD ||
      ldo < H * HD || lddq < 3 * H * HD)
    return RK_ERR_ARG;
  if (B == 0 || T == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_F32) {
    dim3 grid((unsigned)((T + 3) / 4), (unsigned)(B * H));
    const float scale = 1.f / sqrtf((float)HD);
    size_t smem = 4 * T * sizeof(float);
    if (smem > 48 * 1024) { if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dq_f32_kernel), (int)smem)) return e_; }
    rk_host::launch_k(bwd_dq_f32_kernel, grid, 128, smem, s, static_cast<const float*>(qkv), static_cast<const float*>(out),
                                              static_cast<const float*>(dout), lse, dsum, static_cast<float*>(dqkv),
                                              (int)H, (int)HD, (int)T, ldq, ldo, lddq, scale);
    int st = rk_host::launch_status();
    if (st) return st;
    smem = 8 * T * sizeof(float);
    if (smem > 48 * 1024) { if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(bwd_dkv_f32_kernel), (int)smem)) return e_; }
    rk_host::launch_k(bwd_dkv_f32_kernel, grid, 128, smem, s, static_cast<const float*>(qkv), static_cast<const float*>(dout), lse,
                                               dsum, static_cast<float*>(dqkv), (int)H, (int)HD, (int)T, ldq, ldo,
                                               lddq, scale);
    return rk_host::launch_status();
  }
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (!tc_layout_ok(qkv, out, dqkv, ldq, ldo, HD) || !rk_host::aligned(dout, 16) || lddq % 8)
    return (HD == 32 || HD == 64) ? RK_ERR_ALIGN : RK_ERR_UNSUPPORTED;
  if (dtype == RK_BF16)
    return HD == 32 ? bwd_tc<__nv_bfloat16, 32>(qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo, lddq, s)
                    : bwd_tc<__nv_bfloat16, 64>(qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo, lddq, s);
  return HD == 32 ? bwd_tc<__half, 32>(qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo, lddq, s)
                  : bwd_tc<__half, 64>(qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo, lddq, s);
}

// Backward pieces (bf16/f16, head_dim 32 or 64): D, then dQ and dK/dV, which
// may run concurrently on two streams once D is written. Same arguments and
// layouts as rk_attn_bwd; `out` is needed by the D piece only.
extern "C" int rk_attn_bwd_piece(int piece, const void* qkv, int64_t ldq, const void* out, const void* dout,
                                 int64_t ldo, const float* lse, float* dsum, void* dqkv, int64_t lddq, int64_t B,
                                 int64_t H, int64_t HD, int64_t T, int dtype, void* stream) {
  if (piece < 0 || piece > 2 || !attn_args_ok(qkv, dout, B, H, HD, T) || !lse || !dsum || !dqkv ||
      (piece == 0 && !out) || ldq < 3 * H * HD || ldo < H * HD || lddq < 3 * H * HD)
    return RK_ERR_ARG;
  if (B == 0 || T == 0) return RK_OK;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (!tc_layout_ok(qkv, dout, dqkv, ldq, ldo, HD) || (out && !rk_host::aligned(out, 16)) || lddq % 8)
    return (HD == 32 || HD == 64) ? RK_ERR_ALIGN : RK_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_BF16)
    return HD == 32 ? bwd_piece<__nv_bfloat16, 32>(piece, qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq,
                                                   ldo, lddq, s)
                    : bwd_piece<__nv_bfloat16, 64>(piece, qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq,
                                                   ldo, lddq, s);
  return HD == 32 ? bwd_piece<__half, 32>(piece, qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo,
                                          lddq, s)
                  : bwd_piece<__half, 64>(piece, qkv, out, dout, lse, dsum, dqkv, (int)B, (int)H, (int)T, ldq, ldo,
                                          lddq, s);
}
