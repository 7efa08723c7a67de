// Dense GEMMs for the Linear layers (replaces F.linear/cuBLAS at model.py:37,45,55-56
// and its autograd backward).
//
// bf16/f16 path: a persistent, warp-specialised tcgen05 kernel.
//   warp 0      : TMA producer (one elected thread) filling a STAGES-deep ring
//                 of 128x64 A tiles and BNx64 B tiles (128-byte swizzle).
//   warp 1      : allocates 2*BN tensor-memory columns (two accumulators) and
//                 issues tcgen05.mma (M=128, N=BN, K=16) from one thread;
//                 tcgen05.commit frees smem stages and publishes accumulators.
//   warps 2..   : epilogue; warp w reads TMEM lanes 32*(w%4)..+31 (one output
//                 row per thread) of one column group of the tile ((w-2)/4)
//                 with tcgen05.ld and stores to global memory. Eight warps
//                 (two column halves, two warps per SM sub-partition) by
//                 default; sixteen (four column quarters) for the SwiGLU
//                 backward epilogue, whose per-element arithmetic bounds the
//                 tile, so that four warps per sub-partition hide each
//                 other's latency.
// The accumulator is double buffered so the epilogue of tile i overlaps the
// MMAs of tile i+1. Operands may be K-major or MN-major (the transposed views
// that dgrad and wgrad need) without any transposition pass: TMA loads
// 64-element-wide boxes along the contiguous dimension and the smem descriptor
// says which dimension is contiguous.
// Loads are plain TMA (no cluster multicast), so the kernel is safe on every
// multi-GPU configuration.
//
// fp32 path: a CUDA-core tiled kernel (fp32 FMA, k-sequential accumulation),
// used by the fp32 parity configuration where tensor-core rounding (TF32)
// would break the 1e-5 gradient tolerance.
//
// wgrad splits the token reduction into a fixed number of slices; each slice
// writes an fp32 partial tile and a second kernel sums slices in index order,
// so weight gradients are bitwise deterministic for a given shape.
#include <cudaTypedefs.h>
#include <cstdlib>
#include <type_traits>
#include <mutex>
#include <unordered_map>
#include "vec.cuh"

namespace rk {

struct GemmArgs {
  int M, N, K;           // output rows, output cols, reduction length
  int tiles_m, tiles_n;  // output tiles
  int splits;            // reduction slices (1 = none)
  int kb_per_split;      // 64-wide k blocks per slice
  int kb_total;          // ceil(K / 64)
  int split_rows;        // EPI_TMA with splits > 1: rows between split slices (M rounded up to 128)
  int ff;                // EPI_SWIGLU*: offset of the value rows in W (and of the value columns in u)
  void* out;             // EPI_STORE: [M, N] row-major (ldo); split slices: fp32 [splits][split_rows][N]
  int64_t ldo;
  int out_dtype;
  unsigned int* status;
  // Softmax head (vocabulary logits; 128-column blocks b of a row):
  float2* stats;          // EPI_LSE writes, XF reads: per (row, b) (m_b, sum of exp(x - m_b)), m_b = block max
  int stats_ld;           // float2 entries per row (2 * ceil(V / 256): 128-column blocks)
  const float4* rowc;     // XF: per token (-lse * log2(e), scale, label gradient, -); scale 0 = ignored row
  const float* fcoef;     // XF: per (block b, token) exp(m_b - lse) * scale, block-major (fcoef_ld per block)
  int64_t fcoef_ld;
  const int64_t* labels;  // EPI_LSE / XF: per token label
  float* xlabel;          // EPI_LSE: per token, the rounded logit at its label
  int vocab;              // EPI_LSE / XF: valid vocabulary entries
  int tokens;             // XF: valid token rows
  // EPI_TMA_DSUM (attention output projection's dgrad): D[b, h, t] =
  // rowsum over head h's 32 or 64 columns of round(dx) * o
  const void* dsum_o;     // o [M, N] (16-bit, row stride dsum_ldo)
  int64_t dsum_ldo;
  float* dsum;            // [B, H, T], M = B * T
  int dsum_T, dsum_H;
  int dsum_hw;            // head width: 32 (two heads per 64-column chunk) or 64 (one)
  // EPI_RECON (sublayer output projection with the reversible state update):
  // rc_out[r, c] = rc_state[r, c] - round(rc_coeff * round(round(acc) + rc_add[r, c]))
  const float* rc_state;  // fp32 [M, N], row stride rc_lds
  int64_t rc_lds;
  const void* rc_add;     // 16-bit [M, N] addend (row stride rc_lda), or null (no addend)
  int64_t rc_lda;
  float* rc_out;          // fp32 [M, N], row stride rc_ldo (may be rc_state itself)
  int64_t rc_ldo;
  float rc_coeff;
  void* rc_low;           // 16-bit [M, N] round(acc) (row stride rc_ldl), or null
  int64_t rc_ldl;
  // EPI_RECON_NORM: the following RMSNorm forward fused (N == BN):
  // rn_y = round((rc_out * rstd) * rn_w), rstd = rsqrt(mean(rc_out^2) + eps)
  const float* rn_w;      // fp32 [N] norm weight
  void* rn_y;             // 16-bit [M, N], row stride rn_ldy
  int64_t rn_ldy;
  float* rn_rstd;         // fp32 [M], or null
  float rn_eps;
};

// STORE: direct row stores; PARTIAL: fp32 split slices; ACCUM: fp32 out += acc;
// TMA: rows staged in 128-byte-swizzled shared memory, written by TMA tensor
// stores (split slices too, at row split*split_rows); TMA_ADD: the same staging
// written with TMA reduce-add (out += acc; every element has exactly one
// writing CTA, so the result is deterministic).
// SWIGLU: fprop of the MLP up projection with SwiGLU in the epilogue: the B
// tile holds W rows [n0, n0+128) (gate) and [ff+n0, ff+n0+128) (value), so the
// accumulator has gate | value for the same 128 columns and the epilogue writes
// h = round(silu(round(g))) * round(v) only; SWIGLU_SAVE also writes u itself.
// SWIGLU_BWD: dgrad of the MLP down projection with the SwiGLU backward in the
// epilogue: u's gate and value columns matching the tile are TMA-loaded into
// the staging boxes, du = swiglu_bwd(u, round(acc)) is written over them and
// TMA-stored (gate and value halves of du).
// LSE (softmax head forward): per row and 128-column block b, the rounded
// logits x give m_b = max x and e = exp(x - m_b); e is TMA-stored (16-bit)
// instead of x, (m_b, sum e) goes to g.stats and the logit at the row's label
// to g.xlabel. Columns at or past g.vocab do not count. Sixteen epilogue
// warps, one per (TMEM lane quarter, 64-column half of a block); the two
// warps of a block exchange maxima and partial sums in shared memory.
// RECON: the reversible state update from the sublayer output in the
// accumulator: out = state - round(coeff * round(round(acc) + add)) in fp32
// (the rounding points of reconstruct_sum_kernel / reconstruct_kernel), each
// thread reading and writing its own row chunks; the sublayer output itself
// never reaches global memory. RECON_NORM: the same, then the following
// RMSNorm forward of the updated state in the same pass (bitwise equal to
// rmsnorm_fwd_kernel / add_rmsnorm_fwd_kernel on it), and optionally the
// rounded sublayer output itself (rc_low).
enum {
  EPI_STORE = 0, EPI_PARTIAL = 1, EPI_ACCUM = 2, EPI_TMA = 3, EPI_TMA_ADD = 4, EPI_SWIGLU = 5, EPI_SWIGLU_SAVE = 6,
  EPI_LSE = 7, EPI_SWIGLU_BWD = 8, EPI_TMA_DSUM = 9, EPI_RECON = 10, EPI_RECON_NORM = 11
};
// A-operand transforms (XF): the A tile holds e = exp(x - m_b) from the LSE
// epilogue and is turned, in shared memory before the MMA reads it, into the
// cross-entropy gradient dlogit = e * exp(m_b - lse) * scale, with the label's
// entry replaced by its exact (exp(x_label - lse) - 1) * scale.
//   XF_ROWS : A is K-major [tokens, vocab] (head dgrad: dX = dlogits . W)
//   XF_COLS : A is MN-major, i.e. dlogits^T [vocab, tokens] (head wgrad)
enum { XF_NONE = 0, XF_ROWS = 1, XF_COLS = 2 };

__host__ __device__ constexpr bool epi_is_swiglu(int e) { return e == EPI_SWIGLU || e == EPI_SWIGLU_SAVE; }
__host__ __device__ constexpr bool epi_stages_out(int e) {
  return e == EPI_TMA || e == EPI_TMA_ADD || e == EPI_TMA_DSUM || e == EPI_LSE || e == EPI_SWIGLU_BWD ||
         epi_is_swiglu(e);
}
// Epilogue warps per CTA (a multiple of 4: one per TMEM lane quarter and
// column group) and threads per CTA (producer warp, MMA warp, epilogue).
__host__ __device__ constexpr int epi_warps(int e) { return (e == EPI_SWIGLU_BWD || e == EPI_LSE) ? 16 : 8; }
__host__ __device__ constexpr int gemm_threads(int e) { return 64 + 32 * epi_warps(e); }
constexpr int kMaxEpiWarps = 16;
// Output staging per epilogue warp: one 4 KB box (32 rows x 128 bytes); two
// for SWIGLU_SAVE (h and the gate half of u; the value half reuses the
// first); for SWIGLU_BWD two chunk slots of (gate box, value box), 2 KB each:
// u is loaded into them and du computed in place; for LSE one 2 KB box
// (32 rows x 64 bytes) per warp, then 1 KB where the two warps of a 128-column
// block exchange their row maxima and partial sums; for RECON 1 KB where the
// two warps of the same rows exchange the fused norm's half sums and rstd.
__host__ __device__ constexpr uint32_t epi_out_bytes(int e) {
  return e == EPI_SWIGLU_BWD    ? epi_warps(e) * 2 * 4096
         : e == EPI_SWIGLU_SAVE ? epi_warps(e) * 2 * 4096
         : e == EPI_LSE         ? epi_warps(e) * 2048 + 1024
         : e == EPI_RECON_NORM  ? 1024
                                : (epi_stages_out(e) ? epi_warps(e) * 4096 : 0);
}

constexpr int kBM = 128;
constexpr int kBK = 64;

// B-resident mode (RES): K <= kResK; the whole BN x K operand tile stays in
// shared memory while the CTA walks consecutive M tiles of one N block, so a
// tile streams only its 16 KB A k-blocks through the ring.
constexpr int kResKb = 4;  // 64-wide k blocks held resident (K <= 256)

template <int BN, int STAGES, uint32_t OUT_BYTES = 0, bool RES = false>
struct TcSmem {
  static constexpr uint32_t kA = kBM * kBK * 2;  // 16 KB
  static constexpr uint32_t kB = BN * kBK * 2;
  static constexpr uint32_t kStage = RES ? kA : kA + kB;
  static constexpr uint32_t kBres = RES ? kResKb * kB : 0;
  static constexpr uint32_t kOut = OUT_BYTES;  // epilogue staging (epi_out_bytes)
  static constexpr uint32_t kBarriers = (3 * STAGES + 7 + 2 * kMaxEpiWarps) * 8;
  static constexpr uint32_t kTotal = 1024 /*align slack*/ + STAGES * kStage + kBres + kOut + kBarriers + 16;
};

// Tile walk. Default: tile t = blockIdx.x + i * gridDim.x, N fastest, split
// slices outermost. RES: CTA c owns the contiguous run [c*T/G, (c+1)*T/G) of
// the M-fastest order, so consecutive tiles share the resident B block.
template <bool RES>
struct TileWalk {
  int t, end, step;
  __device__ TileWalk(int total) {
    if (RES) {
      t = (int)((int64_t)blockIdx.x * total / gridDim.x);
      end = (int)((int64_t)(blockIdx.x + 1) * total / gridDim.x);
      step = 1;
    } else {
      t = blockIdx.x;
      end = total;
      step = gridDim.x;
    }
  }
  __device__ bool more() const { return t < end; }
  __device__ void next() { t += step; }
  // split slice, first output row, n-tile index of tile t
  __device__ void coords(const GemmArgs& g, int tt, int& split, int& m0, int& nt) const {
    if (RES) {
      split = 0;
      nt = tt / g.tiles_m;
      m0 = (tt - nt * g.tiles_m) * kBM;
    } else {
      const int tiles_mn = g.tiles_m * g.tiles_n;
      split = tt / tiles_mn;
      const int mn = tt - split * tiles_mn;
      m0 = (mn / g.tiles_n) * kBM;
      nt = mn % g.tiles_n;
    }
  }
};

// Tiled TMA store of a shared-memory box to global (bulk async-group).
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap), "r"(src),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, uint32_t src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   tmap),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ void accum_row_chunk(T* dst, float (&v)[32], int valid, bool vec_ok) {
  if constexpr (sizeof(T) == 4) {
    if (valid >= 32 && vec_ok) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 o = reinterpret_cast<const float4*>(dst)[q];
        v[q * 4] += o.x;
        v[q * 4 + 1] += o.y;
        v[q * 4 + 2] += o.z;
        v[q * 4 + 3] += o.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) v[j] += dst[j];
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_row_chunk(T* dst, const float (&v)[32], int valid, bool vec_ok) {
  if (valid >= 32 && vec_ok) {
    if constexpr (sizeof(T) == 2) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = Dt<T>::from_f(v[q * 8 + j]);
        reinterpret_cast<uint4*>(dst)[q] = raw;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) dst[j] = Dt<T>::from_f(v[j]);
  }
}

constexpr float kLog2eF = 1.4426950408889634f;

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats rounded to a packed pair of 16-bit values (lo in bits 0..15), and back.
template <typename T>
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  uint32_t d;
  if constexpr (std::is_same_v<T, __nv_bfloat16>) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
template <typename T>
__device__ __forceinline__ float unpack_half(uint32_t u, int which) {
  const uint32_t b = which ? (u >> 16) : (u & 0xffffu);
  if constexpr (std::is_same_v<T, __nv_bfloat16>) return __uint_as_float(b << 16);
  else return __half2float(__ushort_as_half((unsigned short)b));
}

// Packed 16-bit max of two pairs (values are already rounded, so this is exact).
template <typename T>
__device__ __forceinline__ uint32_t max2_16(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (std::is_same_v<T, __nv_bfloat16>) asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Two values in [0, 1] rounded to 16 bits and packed. bf16: round to nearest
// (ties away) by an integer add on the ALU, leaving the exponential unit free.
template <typename T>
__device__ __forceinline__ uint32_t pack_unit2(float lo, float hi) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>)
    return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
  else return pack2_rn<T>(lo, hi);
}

// pack2_rn on the integer ALU for bf16 (round to nearest even by adding
// 0x7fff plus the kept lowest bit; identical to the conversion for every
// non-NaN value), keeping the conversion unit for the exponentials.
template <typename T>
__device__ __forceinline__ uint32_t pack2_rne_alu(float lo, float hi) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const uint32_t a = __float_as_uint(lo), b = __float_as_uint(hi);
    return __byte_perm(a + 0x7fffu + ((a >> 16) & 1u), b + 0x7fffu + ((b >> 16) & 1u), 0x7632);
  } else {
    return pack2_rn<T>(lo, hi);
  }
}

// One packed pair of the SwiGLU backward in rk_swiglu_bwd's operation order:
// gw / vw hold u's (gate, value) pair on entry and (dg, dv) on return; a0, a1
// are the fp32 dgrad accumulators, rounded to T first (the dh that the
// unfused path stores). Roundings of pairs are one packed conversion each.
template <typename T>
__device__ __forceinline__ void swiglu_bwd_word(uint32_t& gw, uint32_t& vw, uint32_t a0, uint32_t a1) {
  const uint32_t dw = pack2_rn<T>(__uint_as_float(a0), __uint_as_float(a1));
  const float g0 = unpack_half<T>(gw, 0), g1 = unpack_half<T>(gw, 1);
  const float v0 = unpack_half<T>(vw, 0), v1 = unpack_half<T>(vw, 1);
  const float d0 = unpack_half<T>(dw, 0), d1 = unpack_half<T>(dw, 1);
  const float s0 = sigmoid_value(g0), s1 = sigmoid_value(g1);
  const uint32_t sw = pack2_rn<T>(__fmul_rn(g0, s0), __fmul_rn(g1, s1));  // round(silu(g))
  const uint32_t tw = pack2_rn<T>(__fmul_rn(d0, v0), __fmul_rn(d1, v1));  // round(dh * v)
  const float sl0 = __fmul_rn(s0, __fadd_rn(1.f, __fmul_rn(g0, __fsub_rn(1.f, s0))));
  const float sl1 = __fmul_rn(s1, __fadd_rn(1.f, __fmul_rn(g1, __fsub_rn(1.f, s1))));
  gw = pack2_rne_alu<T>(__fmul_rn(unpack_half<T>(tw, 0), sl0), __fmul_rn(unpack_half<T>(tw, 1), sl1));
  vw = pack2_rne_alu<T>(__fmul_rn(d0, unpack_half<T>(sw, 0)), __fmul_rn(d1, unpack_half<T>(sw, 1)));
}

// One 16-byte chunk (8 entries of one token, vocabulary v0..v0+7) of an A
// tile, in place: e * f, and the entry at `label` (if in the chunk) set to gl.
template <typename T>
__device__ __forceinline__ uint32_t scale_pair(uint32_t wd, float f) {
  return pack2_rn<T>(unpack_half<T>(wd, 0) * f, unpack_half<T>(wd, 1) * f);
}
// bf16 pair times f, with f = f_hi + f_lo split into two bf16 values (both
// halves of fhi2 / flo2): fma(e, f_hi, e * f_lo) rounds once, so the result is
// e * f correctly rounded up to the negligible rounding of the e * f_lo term.
__device__ __forceinline__ uint32_t bf16x2_scale(uint32_t e2, uint32_t fhi2, uint32_t flo2) {
  uint32_t t, d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t) : "r"(e2), "r"(flo2));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(e2), "r"(fhi2), "r"(t));
  return d;
}
struct ChunkScale {
  float f;
  uint32_t fhi2, flo2;  // bf16: f split into high and low bf16 parts, both halves
};
template <typename T>
__device__ __forceinline__ ChunkScale chunk_scale(float f) {
  ChunkScale c;
  c.f = f;
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const uint32_t hi = pack2_rn<T>(f, f);
    const float fh = unpack_half<T>(hi, 0);
    c.fhi2 = hi;
    c.flo2 = pack2_rn<T>(f - fh, f - fh);
  } else {
    c.fhi2 = c.flo2 = 0u;
  }
  return c;
}
template <typename T>
__device__ __forceinline__ uint32_t scale_word(uint32_t wd, const ChunkScale& c) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) return bf16x2_scale(wd, c.fhi2, c.flo2);
  else return scale_pair<T>(wd, c.f);
}
template <typename T>
__device__ __forceinline__ void softmax_grad_chunk(uint8_t* p, int v0, const ChunkScale& f, int64_t label, float gl) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  raw.x = scale_word<T>(raw.x, f);
  raw.y = scale_word<T>(raw.y, f);
  raw.z = scale_word<T>(raw.z, f);
  raw.w = scale_word<T>(raw.w, f);
  const int64_t li = label - v0;
  if (li >= 0 && li < 8) {
    const uint32_t gp = pack2_rn<T>(gl, gl);
    const uint32_t mask = (li & 1) ? 0xffff0000u : 0x0000ffffu;
    const int qi = (int)(li >> 1);
    raw.x = qi == 0 ? ((raw.x & ~mask) | (gp & mask)) : raw.x;
    raw.y = qi == 1 ? ((raw.y & ~mask) | (gp & mask)) : raw.y;
    raw.z = qi == 2 ? ((raw.z & ~mask) | (gp & mask)) : raw.z;
    raw.w = qi == 3 ? ((raw.w & ~mask) | (gp & mask)) : raw.w;
  }
  *reinterpret_cast<uint4*>(p) = raw;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, typename TOut, bool RES = false, int XF = XF_NONE,
          typename TIn = __nv_bfloat16>
__global__ void __launch_bounds__(gemm_threads(EPI), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                   const GemmArgs g, const uint32_t idesc) {
  static_assert(!RES || !B_MN, "the resident B tile is K-major");
  static_assert(XF == XF_NONE || (XF == XF_ROWS) == !A_MN, "XF_ROWS needs a K-major A, XF_COLS an MN-major A");
  static_assert(XF == XF_NONE || (!RES && !epi_is_swiglu(EPI)), "transforms run on the plain schedule");
  using L = TcSmem<BN, STAGES, epi_out_bytes(EPI), RES>;
  constexpr int NSTEP = epi_is_swiglu(EPI) ? BN / 2 : BN;  // output columns per tile
  constexpr int EW = epi_warps(EPI);
  static_assert(EW == 8 || (BN == 256 && XF == XF_NONE), "16 epilogue warps: 256-column tiles, no transform");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kA;  // B ring (RES: the resident B block)
  uint8_t* sOut = smem + STAGES * L::kStage + L::kBres;  // EPI_TMA staging (1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + L::kOut);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + STAGES * 8;
  const uint32_t tfull0 = empty0 + STAGES * 8;
  const uint32_t tempty0 = tfull0 + 2 * 8;
  const uint32_t drain = tempty0 + 2 * 8;
  const uint32_t bfull = drain + 8;    // RES: resident B block loaded
  const uint32_t bempty = bfull + 8;   // RES: MMAs reading the resident B block done
  const uint32_t xready0 = bempty + 8;  // XF: stage transformed (one arrival per epilogue warp)
  const uint32_t ubar0 = xready0 + 8 * STAGES;  // SWIGLU_BWD: u chunk (warp, chunk) landed
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 7 + 2 * kMaxEpiWarps);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(s_tmem + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(xready0 + 8 * s, EW);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 32 * EW);
    }
    mbar_init(drain, 1);
    mbar_init(bfull, 1);
    mbar_init(bempty, 1);
    for (int i = 0; i < 2 * kMaxEpiWarps; ++i) mbar_init(ubar0 + 8 * i, (EPI == EPI_LSE && i % 4 == 0) ? 2 : 1);
    fence_mbar_init();
    *s_abort = 0;
    *s_consumed = 0;
    s_tmem[3] = 0;  // resident B loads consumed by the MMA warp
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  // The prologue above (barriers, tensor-map prefetch, TMEM allocation) touches
  // no global data, so it overlaps the previous kernel's tail.
  pdl_wait();

  const int total = g.tiles_m * g.tiles_n * g.splits;
  int issued = 0;
  int b_issued = 0;  // RES: resident B loads issued (producer) / consumed (MMA)
  volatile int* s_b_consumed = reinterpret_cast<volatile int*>(s_tmem + 3);

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int cur_nt = -1;
    uint32_t bphase = 0;
    for (TileWalk<RES> w(total); w.more() && ok; w.next()) {
      int split, m0, nt;
      w.coords(g, w.t, split, m0, nt);
      const int n0 = nt * NSTEP;
      const int kb0 = split * g.kb_per_split;
      int kb1 = kb0 + g.kb_per_split;
      if (kb1 > g.kb_total) kb1 = g.kb_total;
      if constexpr (RES) {
        if (nt != cur_nt) {  // load the B block of this N tile once
          if (!mbar_wait(bempty, bphase ^ 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bfull, (uint32_t)(kb1 - kb0) * L::kB);
          for (int kb = kb0; kb < kb1; ++kb) {
            const uint32_t b_dst = smem_u32(sB + (kb - kb0) * L::kB);
            if constexpr (epi_is_swiglu(EPI)) {
              tma_load_2d(b_dst, &tmB, bfull, kb * kBK, n0);
              tma_load_2d(b_dst + (BN / 2) * 128, &tmB, bfull, kb * kBK, g.ff + n0);
            } else {
              tma_load_2d(b_dst, &tmB, bfull, kb * kBK, n0);
            }
          }
          ++b_issued;
          bphase ^= 1;
          cur_nt = nt;
        }
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        const uint32_t fb = full0 + 8 * stage;
        mbar_arrive_expect_tx(fb, L::kStage);
        const uint32_t a_dst = smem_u32(sA + stage * L::kA);
        const int k0 = kb * kBK;
        if constexpr (A_MN) {
          tma_load_2d(a_dst, &tmA, fb, m0, k0);
          tma_load_2d(a_dst + 8192, &tmA, fb, m0 + 64, k0);
        } else {
          tma_load_2d(a_dst, &tmA, fb, k0, m0);
        }
        if constexpr (!RES) {
          const uint32_t b_dst = smem_u32(sB + stage * L::kB);
          if constexpr (epi_is_swiglu(EPI)) {  // gate rows, then the matching value rows
            tma_load_2d(b_dst, &tmB, fb, k0, n0);
            tma_load_2d(b_dst + (BN / 2) * 128, &tmB, fb, k0, g.ff + n0);
          } else if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * 8192, &tmB, fb, n0 + 64 * c, k0);
          } else {
            tma_load_2d(b_dst, &tmB, fb, k0, n0);
          }
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int consumed = 0;
    int b_consumed = 0;
    bool ok = true;
    bool pending = false;
    int cur_nt = -1;
    uint32_t bphase = 0;
    for (TileWalk<RES> w(total); w.more() && ok; w.next()) {
      int split, m0, nt;
      w.coords(g, w.t, split, m0, nt);
      const int kb0 = split * g.kb_per_split;
      int kb1 = kb0 + g.kb_per_split;
      if (kb1 > g.kb_total) kb1 = g.kb_total;
      if constexpr (RES) {
        if (nt != cur_nt) {
          if (!mbar_wait(bfull, bphase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          ++b_consumed;
          bphase ^= 1;
          cur_nt = nt;
        }
      }
      if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        const uint32_t ready = XF != XF_NONE ? xready0 + 8 * stage : full0 + 8 * stage;
        if (!mbar_wait(ready, phase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        ++consumed;
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + stage * L::kA);
        const uint32_t b_base = RES ? smem_u32(sB + (kb - kb0) * L::kB) : smem_u32(sB + stage * L::kB);
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {
          const uint64_t ad = A_MN ? smem_desc_sw128(a_base + j * 2048, 8192, 1024)
                                   : smem_desc_sw128(a_base + j * 32, 16, 1024);
          const uint64_t bd = B_MN ? smem_desc_sw128(b_base + j * 2048, 8192, 1024)
                                   : smem_desc_sw128(b_base + j * 32, 16, 1024);
          umma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
        }
        umma_commit(empty0 + 8 * stage);
        pending = true;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      umma_commit(tfull0 + 8 * acc);
      if constexpr (RES) {
        // last tile of this N block: the resident B block may be overwritten
        // once these MMAs complete
        if (w.t + 1 < w.end) {
          int s2, m2, nt2;
          w.coords(g, w.t + 1, s2, m2, nt2);
          if (nt2 != nt) umma_commit(bempty);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    *s_consumed = consumed;
    *s_b_consumed = b_consumed;
    if (!ok && pending) {
      // Let every MMA already issued finish before tensor memory is released.
      umma_commit(drain);
      mbar_wait(drain, 0, g.status, RK_DEV_GEMM_TIMEOUT, nullptr);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;      // TMEM lane quarter this warp may access
    const int ew = warp - 2;           // epilogue warp 0..EW-1
    const int half = ew / 4;           // column group of the tile this warp stores (a half when EW == 8)
    int acc = 0;
    uint32_t acc_phase = 0;
    int xstage = 0;                    // XF: ring position, in step with the producer
    uint32_t xphase = 0;
    uint32_t uphase = 0;               // SWIGLU_BWD: parity of each chunk's u barrier (bit ch)
    uint32_t upend = 0;                // SWIGLU_BWD: u loads issued and not yet waited on (bit ch)
    bool uwarm = false;                // SWIGLU_BWD: the first tile's u has been requested
    int xtiles = 0;                    // LSE, RECON + norm: tiles this warp finished (phase of its pair's barriers)
    for (TileWalk<RES> w(total); w.more(); w.next()) {
      int split, m0, nt;
      w.coords(g, w.t, split, m0, nt);
      const int n0 = nt * NSTEP;
      if constexpr (XF != XF_NONE) {
        // Transform every A stage of this tile as it lands. Thread layout: two
        // threads per 128-byte smem row (four 16-byte chunks each); the chunk
        // order is rotated by the row so a warp's accesses spread over all banks.
        const int tid = threadIdx.x - 64;  // 0..255
        const int hrow = tid & 1;
        const int srow = tid >> 1;         // XF_ROWS: token row of the tile; XF_COLS: (box, token) pair
        const int kb0 = split * g.kb_per_split;
        int kb1 = kb0 + g.kb_per_split;
        if (kb1 > g.kb_total) kb1 = g.kb_total;
        // Per k block each thread needs, for its token: f = exp(m_b - lse) * scale
        // of the k block's vocabulary block b (block-major, so a warp's loads
        // are contiguous), the label and the label's gradient. The loads run
        // four k blocks ahead of their use.
        struct Coef {
          float f, gl;
          int64_t lab;
        };
        // XF_ROWS: the token, its label and label gradient are fixed for the tile
        float row_gl = 0.f;
        int64_t row_lab = -1;
        if constexpr (XF == XF_ROWS) {
          if (m0 + srow < g.tokens) {
            row_gl = __ldg(&g.rowc[m0 + srow].z);
            row_lab = __ldg(g.labels + m0 + srow);
          }
        }
        auto fetch = [&](int kb) {
          Coef c;
          const int token = XF == XF_ROWS ? m0 + srow : kb * kBK + (srow & 63);
          const int blk = XF == XF_ROWS ? (kb * kBK) >> 7 : m0 >> 7;
          if (kb < kb1 && token < g.tokens) {
            c.f = __ldg(g.fcoef + (int64_t)blk * g.fcoef_ld + token);
            if constexpr (XF == XF_ROWS) {
              c.gl = row_gl;
              c.lab = row_lab;
            } else {
              c.gl = __ldg(&g.rowc[token].z);
              c.lab = __ldg(g.labels + token);
            }
          } else {
            c.f = 0.f;
            c.gl = 0.f;
            c.lab = -1;
          }
          return c;
        };
        auto step = [&](int kb, const Coef& c) -> bool {
          const ChunkScale cs = chunk_scale<TIn>(c.f);
          bool sok = mbar_wait(full0 + 8 * xstage, xphase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
          sok = __all_sync(0xffffffffu, sok);
          if (!sok) return false;
          uint8_t* tile = sA + xstage * L::kA;
          if constexpr (XF == XF_ROWS) {
            uint8_t* rowp = tile + srow * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int pc = (hrow * 4 + q + srow) & 7;
              const int j = pc ^ (srow & 7);
              softmax_grad_chunk<TIn>(rowp + pc * 16, kb * kBK + j * 8, cs, c.lab, c.gl);
            }
          } else {
            const int box = srow >> 6, k = srow & 63;
            uint8_t* rowp = tile + box * 8192 + k * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int pc = (hrow * 4 + q + k) & 7;
              const int j = pc ^ (k & 7);
              softmax_grad_chunk<TIn>(rowp + pc * 16, m0 + box * 64 + j * 8, cs, c.lab, c.gl);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(xready0 + 8 * xstage);
          if (++xstage == STAGES) {
            xstage = 0;
            xphase ^= 1;
          }
          return true;
        };
        // four coefficient sets in flight, each reloaded right after its use
        // (no register copies that would wait on an outstanding load)
        Coef c0 = fetch(kb0), c1 = fetch(kb0 + 1), c2 = fetch(kb0 + 2), c3 = fetch(kb0 + 3);
        bool xok = true;
        for (int kb = kb0; kb < kb1 && xok; kb += 4) {
          xok = step(kb, c0);
          c0 = fetch(kb + 4);
          if (xok && kb + 1 < kb1) {
            xok = step(kb + 1, c1);
            c1 = fetch(kb + 5);
          }
          if (xok && kb + 2 < kb1) {
            xok = step(kb + 2, c2);
            c2 = fetch(kb + 6);
          }
          if (xok && kb + 3 < kb1) {
            xok = step(kb + 3, c3);
            c3 = fetch(kb + 7);
          }
        }
        if (!xok) break;
      }
      // SWIGLU_BWD: this warp's u rows (gate box and value box, 32 columns
      // each) of chunk ch of the tile at index tt go to chunk slot ch; issued
      // by lane 0.
      auto u_issue = [&](int tt, int ch) {
        if constexpr (EPI == EPI_SWIGLU_BWD) {
          int s2, m2, nt2;
          w.coords(g, tt, s2, m2, nt2);
          const int col = nt2 * NSTEP + half * 64 + ch * 32;
          if (col < g.ff) {
            const uint32_t box = smem_u32(sOut + (ew * 2 + ch) * 4096);
            const uint32_t ub = ubar0 + 8 * (ew * 2 + ch);
            mbar_arrive_expect_tx(ub, 4096);
            tma_load_2d(box, &tmD, ub, col, m2 + quarter * 32);
            tma_load_2d(box + 2048, &tmD, ub, g.ff + col, m2 + quarter * 32);
            upend |= 1u << ch;
          }
        }
      };
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        // The first tile's u is requested here; every later tile's chunk is
        // requested as soon as the previous tile's store has read that slot.
        if (lane == 0 && !uwarm) {
          u_issue(w.t, 0);
          u_issue(w.t, 1);
        }
        uwarm = true;
      }
      bool ok = mbar_wait(tfull0 + 8 * acc, acc_phase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        // du = swiglu_bwd(u, dh) with dh = round(accumulator): the operation
        // order of rk_swiglu_bwd on the rounded dgrad output, written in place
        // over the staged u boxes and TMA-stored (gate half, then value half).
        // Once a slot's store has read it, the slot is refilled with the next
        // tile's u, whose load then overlaps this tile's remaining work.
        static_assert(BN == 256 && sizeof(TOut) == 2 && EW == 16, "256-column tiles, 16-bit u, 16 warps");
        const int y = m0 + quarter * 32;
        const bool has_next = w.t + w.step < w.end;
        bool uok = true;
#pragma unroll 1
        for (int ch = 0; ch < 2; ++ch) {
          const int c = half * 64 + ch * 32;
          uint32_t r[32];
          tmem_ld_32cols_nowait(t_row + c, r);
          tmem_ld_wait();
          if (ch == 1) {  // TMEM is read: the MMA warp may reuse this accumulator
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
          }
          if (n0 + c < g.ff) {
            const uint32_t ub = ubar0 + 8 * (ew * 2 + ch);
            uok = mbar_wait(ub, (uphase >> ch) & 1u, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
            uok = __all_sync(0xffffffffu, uok);
            if (!uok) break;
            uphase ^= 1u << ch;
            upend &= ~(1u << ch);
            // boxes of 32 rows x 64 bytes, 64-byte swizzle: 16-byte chunk j of
            // row r at j ^ ((r / 2) % 4)
            uint8_t* gb = sOut + (ew * 2 + ch) * 4096;
            uint8_t* vb = gb + 2048;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int off = lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16);
              uint4 gw = *reinterpret_cast<const uint4*>(gb + off);
              uint4 vw = *reinterpret_cast<const uint4*>(vb + off);
              const uint32_t* q = r + j * 8;
              swiglu_bwd_word<TOut>(gw.x, vw.x, q[0], q[1]);
              swiglu_bwd_word<TOut>(gw.y, vw.y, q[2], q[3]);
              swiglu_bwd_word<TOut>(gw.z, vw.z, q[4], q[5]);
              swiglu_bwd_word<TOut>(gw.w, vw.w, q[6], q[7]);
              *reinterpret_cast<uint4*>(gb + off) = gw;
              *reinterpret_cast<uint4*>(vb + off) = vw;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, smem_u32(gb), n0 + c, y);
              tma_store_2d(&tmC, smem_u32(vb), g.ff + n0 + c, y);
              bulk_commit();
              if (has_next) bulk_wait_read<0>();  // the slot is free once the store has read it
            }
          }
          if (lane == 0 && has_next) u_issue(w.t + w.step, ch);
        }
        if (!uok) break;
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if constexpr (epi_is_swiglu(EPI)) {
        // h = round(silu(round(g))) * round(v) for this warp's 64 of the tile's
        // 128 columns; the same operation order as rk_swiglu_fwd on a bf16 u.
        static_assert(BN == 256, "the SwiGLU epilogue pairs 128 gate and 128 value columns");
        uint8_t* stage = sOut + ew * (EPI == EPI_SWIGLU_SAVE ? 8192 : 4096);
        const int y = m0 + quarter * 32;
        const int c = half * 64;
        uint8_t* hb = stage;
        uint8_t* gb = stage + 4096;
        if (lane == 0) bulk_wait_read<0>();  // this warp's boxes from the previous tile are free
        __syncwarp();
        uint32_t vkeep[EPI == EPI_SWIGLU_SAVE ? 32 : 1];  // packed value half, stored after h
        // two passes of 32 columns: gate and value chunks, then 4 of the 8
        // 16-byte chunks of each staged row. Conversions are packed (one per
        // two values); the arithmetic is per value as in rk_swiglu_fwd.
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t rg[32], rv[32];
          tmem_ld_32cols_nowait(t_row + c + q * 32, rg);
          tmem_ld_32cols_nowait(t_row + BN / 2 + c + q * 32, rv);
          tmem_ld_wait();
          if (q == 1) {  // TMEM is read: the MMA warp may reuse this accumulator
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t hw[4], gw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int i = j * 8 + 2 * k;
              gw[k] = pack2_rn<TOut>(__uint_as_float(rg[i]), __uint_as_float(rg[i + 1]));
              const uint32_t vw = pack2_rn<TOut>(__uint_as_float(rv[i]), __uint_as_float(rv[i + 1]));
              const float g0 = unpack_half<TOut>(gw[k], 0), g1 = unpack_half<TOut>(gw[k], 1);
              const uint32_t sw = pack2_rn<TOut>(silu_value(g0), silu_value(g1));
              hw[k] = pack2_rn<TOut>(__fmul_rn(unpack_half<TOut>(sw, 0), unpack_half<TOut>(vw, 0)),
                                     __fmul_rn(unpack_half<TOut>(sw, 1), unpack_half<TOut>(vw, 1)));
              if constexpr (EPI == EPI_SWIGLU_SAVE) vkeep[q * 16 + j * 4 + k] = vw;
            }
            const int off = lane * 128 + (((q * 4 + j) ^ (lane & 7)) * 16);
            *reinterpret_cast<uint4*>(hb + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            if constexpr (EPI == EPI_SWIGLU_SAVE)
              *reinterpret_cast<uint4*>(gb + off) = make_uint4(gw[0], gw[1], gw[2], gw[3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, smem_u32(hb), n0 + c, y);
          bulk_commit();
          if constexpr (EPI == EPI_SWIGLU_SAVE) {
            tma_store_2d(&tmD, smem_u32(gb), n0 + c, y);
            bulk_commit();
            bulk_wait_read<1>();  // the h box has been read: reuse it for the value half
          }
        }
        if constexpr (EPI == EPI_SWIGLU_SAVE) {
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(hb + lane * 128 + ((j ^ (lane & 7)) * 16)) =
                make_uint4(vkeep[4 * j], vkeep[4 * j + 1], vkeep[4 * j + 2], vkeep[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmD, smem_u32(hb), g.ff + n0 + c, y);
            bulk_commit();
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if constexpr (EPI == EPI_LSE) {
        // This warp's 64-column half h of 128-column block blk, for its 32 rows:
        // one TMEM read of 64 columns, rounded to the output type and packed in
        // pairs (the accumulator is released right after); the half's max
        // (packed 16-bit max: the values are already rounded) is exchanged with
        // the block's other warp through shared memory, e = exp(x - m_b) is
        // formed against the block max, each 32-column quarter staged in the
        // warp's 2 KB box (64-byte rows, 64-byte swizzle: 16-byte chunk j of
        // row r at j ^ ((r / 2) % 4)) and TMA-stored while the next one is
        // exponentiated, and the half-1 warp hands its partial sum to the
        // half-0 warp, which writes (m_b, s0 + s1). Per block pair and tile:
        // barrier A (both maxima written, two arrivals), B (half 0 has read
        // the max of half 1), C (the sum of half 1 written), D (half 0 has
        // read it); every wait bounded.
        static_assert(sizeof(TOut) == 2 && BN == 256 && EW == 16, "16-bit output, 256-column tiles, 16 warps");
        const int cg = ew >> 2;  // 64-column group of the tile: block cg / 2, half cg % 2
        const int blk = cg >> 1, hf = cg & 1;
        const int pr = quarter * 2 + blk;  // the block pair's slot
        const uint32_t barA = ubar0 + 8 * (4 * pr), barB = barA + 8, barC = barA + 16, barD = barA + 24;
        uint8_t* xch = sOut + EW * 2048 + pr * 128 + lane * 4;  // [pair][lane]: two 16-bit maxima or one fp32 sum
        const int row = m0 + quarter * 32 + lane;
        const int64_t lab = row < g.M ? g.labels[row] : -1;
        const int c0 = n0 + cg * 64;
        const int nvalid = g.vocab - c0;  // columns of this half below vocab (may be <= 0 or >= 64)
        uint32_t xp[32];                  // the half's 64 rounded logits, two per word
        {
          uint32_t r[64];
          tmem_ld_32cols_nowait(t_row + cg * 64, r);
          tmem_ld_32cols_nowait(t_row + cg * 64 + 32, r + 32);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) xp[k] = pack2_rn<TOut>(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
        }
        tc_fence_before();
        mbar_arrive(tempty0 + 8 * acc);  // TMEM read: the MMA warp may reuse the accumulator
        // columns at or past vocab become -inf
        constexpr uint32_t kNegInf = std::is_same_v<TOut, __nv_bfloat16> ? 0xff80u : 0xfc00u;
        if (nvalid < 64) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (2 * k >= nvalid) xp[k] = (xp[k] & 0xffff0000u) | kNegInf;
            if (2 * k + 1 >= nvalid) xp[k] = (xp[k] & 0x0000ffffu) | (kNegInf << 16);
          }
        }
        uint32_t m4[4] = {xp[0], xp[1], xp[2], xp[3]};
#pragma unroll
        for (int k = 4; k < 32; ++k) m4[k & 3] = max2_16<TOut>(m4[k & 3], xp[k]);
        uint32_t m2 = max2_16<TOut>(max2_16<TOut>(m4[0], m4[1]), max2_16<TOut>(m4[2], m4[3]));
        m2 = max2_16<TOut>(m2, __byte_perm(m2, 0, 0x1032));  // both halves: this half's max
        bool xok = true;
        // the half-1 warp reuses the slot (its sum overlapped both maxima) only
        // once half 0 has read the previous tile's sum
        if (hf == 1 && xtiles > 0) xok = mbar_wait(barD, (xtiles - 1) & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
        xok = __all_sync(0xffffffffu, xok);
        if (!xok) break;
        *reinterpret_cast<uint16_t*>(xch + 2 * hf) = (uint16_t)(m2 & 0xffffu);
        __syncwarp();
        if (lane == 0) mbar_arrive(barA);
        xok = mbar_wait(barA, xtiles & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
        xok = __all_sync(0xffffffffu, xok);
        if (!xok) break;
        const uint32_t other = *reinterpret_cast<const uint16_t*>(xch + 2 * (hf ^ 1));
        __syncwarp();
        if (hf == 0 && lane == 0) mbar_arrive(barB);  // half 1's max is read
        const uint32_t mb2 = max2_16<TOut>(m2, other | (other << 16));
        const float mx = unpack_half<TOut>(mb2, 0);  // the block max (-inf when no column is valid)
        const int64_t li = lab - c0;
        if (li >= 0 && li < 64 && li < nvalid) {  // this half holds the row's label: keep its logit
          float xl = 0.f;
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if ((int)(li >> 1) == k) xl = unpack_half<TOut>(xp[k], (int)(li & 1));
          g.xlabel[row] = xl;
        }
        const float nm = mx == -INFINITY ? 0.f : -mx * kLog2eF;
        const float2 l2 = make_float2(kLog2eF, kLog2eF), n2 = make_float2(nm, nm);
        float2 sm2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // packed fp32x2 partial sums
        uint8_t* buf = sOut + ew * 2048;
        const int y = m0 + quarter * 32;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
#pragma unroll
          for (int k = ch * 16; k < ch * 16 + 16; ++k) {  // a pair per step: one FFMA2, two ex2, one FADD2
            const float2 t = __ffma2_rn(make_float2(unpack_half<TOut>(xp[k], 0), unpack_half<TOut>(xp[k], 1)), l2, n2);
            const float e0 = ex2_fast(t.x), e1 = ex2_fast(t.y);
            sm2[k & 1] = __fadd2_rn(sm2[k & 1], make_float2(e0, e1));
            xp[k] = pack_unit2<TOut>(e0, e1);
          }
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) =
                make_uint4(xp[ch * 16 + 4 * j], xp[ch * 16 + 4 * j + 1], xp[ch * 16 + 4 * j + 2],
                           xp[ch * 16 + 4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, smem_u32(buf), c0 + ch * 32, y);
            bulk_commit();
          }
        }
        const float sm = (sm2[0].x + sm2[1].x) + (sm2[0].y + sm2[1].y);
        if (hf == 1) {
          xok = mbar_wait(barB, xtiles & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
          xok = __all_sync(0xffffffffu, xok);
          if (!xok) break;
          *reinterpret_cast<float*>(xch) = sm;
          __syncwarp();
          if (lane == 0) mbar_arrive(barC);
        } else {
          xok = mbar_wait(barC, xtiles & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
          xok = __all_sync(0xffffffffu, xok);
          if (!xok) break;
          const float s1 = *reinterpret_cast<const float*>(xch);
          __syncwarp();
          if (lane == 0) mbar_arrive(barD);  // the slot may be reused
          if (row < g.M) g.stats[(int64_t)row * g.stats_ld + 2 * nt + blk] = make_float2(mx, sm + s1);
        }
        ++xtiles;
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if constexpr (EPI == EPI_TMA || EPI == EPI_TMA_ADD || EPI == EPI_TMA_DSUM) {
        // Each warp stages its 32 rows, CW columns at a time, in a 128-byte
        // swizzled layout (16-byte chunk j of row r at j ^ (r % 8): conflict-free
        // stores) and writes them with one TMA store per chunk. DSUM: each
        // 64-column chunk is two 32-column heads or one 64-column head;
        // D = rowsum(round(acc) * o) per head in dsum_kernel's order (the two
        // column halves of a head summed separately, then added), o read
        // while the TMEM load is in flight.
        constexpr int CW = 128 / (int)sizeof(TOut);
        constexpr int HALF = BN / 2;
        static_assert(HALF % CW == 0, "column half must be whole staging boxes");
        uint8_t* buf = sOut + ew * 4096;
        const int y = split * g.split_rows + m0 + quarter * 32;
#pragma unroll 1
        for (int c = half * HALF; c < (half + 1) * HALF; c += CW) {
          uint32_t r[CW];
#pragma unroll
          for (int q = 0; q < CW / 32; ++q) tmem_ld_32cols_nowait(t_row + c + q * 32, r + q * 32);
          uint4 ov[EPI == EPI_TMA_DSUM ? 8 : 1];
          const int drow = m0 + quarter * 32 + lane;
          if constexpr (EPI == EPI_TMA_DSUM) {
            static_assert(sizeof(TOut) == 2 && CW == 64, "16-bit output, 64-column chunks");
            const uint4* op =
                reinterpret_cast<const uint4*>(static_cast<const TOut*>(g.dsum_o) + (int64_t)drow * g.dsum_ldo + n0 + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) ov[j] = drow < g.M ? __ldg(op + j) : make_uint4(0u, 0u, 0u, 0u);
          }
          tmem_ld_wait();
          if (c + CW == (half + 1) * HALF) {  // last TMEM read of this tile by this warp
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
          }
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          float dacc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // DSUM: [head][16-column half]
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 raw;
            if constexpr (sizeof(TOut) == 2) {  // packed conversions: one per two values
              const uint32_t* q = r + j * 8;
              raw = make_uint4(pack2_rn<TOut>(__uint_as_float(q[0]), __uint_as_float(q[1])),
                               pack2_rn<TOut>(__uint_as_float(q[2]), __uint_as_float(q[3])),
                               pack2_rn<TOut>(__uint_as_float(q[4]), __uint_as_float(q[5])),
                               pack2_rn<TOut>(__uint_as_float(q[6]), __uint_as_float(q[7])));
            } else {
              raw = make_uint4(r[j * 4], r[j * 4 + 1], r[j * 4 + 2], r[j * 4 + 3]);
            }
            if constexpr (EPI == EPI_TMA_DSUM) {
              // 32-column heads: head j / 4, half (j % 4) / 2; 64-column: half j / 4
              float& a = g.dsum_hw == 32 ? dacc[j >> 2][(j & 3) >> 1] : dacc[0][j >> 2];
              const uint32_t dw[4] = {raw.x, raw.y, raw.z, raw.w};
              const uint32_t owd[4] = {ov[j].x, ov[j].y, ov[j].z, ov[j].w};
#pragma unroll
              for (int e = 0; e < 8; ++e)
                a += unpack_half<TOut>(owd[e >> 1], e & 1) * unpack_half<TOut>(dw[e >> 1], e & 1);
            }
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) = raw;
          }
          if constexpr (EPI == EPI_TMA_DSUM) {
            if (drow < g.M) {
              const int b = drow / g.dsum_T, t = drow - b * g.dsum_T;
              if (g.dsum_hw == 32) {
                const int h0 = (n0 + c) >> 5;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
                  g.dsum[((int64_t)b * g.dsum_H + h0 + hh) * g.dsum_T + t] = dacc[hh][0] + dacc[hh][1];
              } else {
                g.dsum[((int64_t)b * g.dsum_H + ((n0 + c) >> 6)) * g.dsum_T + t] = dacc[0][0] + dacc[0][1];
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == EPI_TMA_ADD) tma_reduce_add_2d(&tmC, smem_u32(buf), n0 + c, y);
            else tma_store_2d(&tmC, smem_u32(buf), n0 + c, y);
            bulk_commit();
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if constexpr (EPI == EPI_RECON || EPI == EPI_RECON_NORM) {
        // Pass 1: the state update of this warp's 32 rows x BN/2 columns, four
        // 32-column chunks; with the fused RMSNorm (RECON_NORM: the tile spans
        // the whole row) each thread also forms, per 4-column group of its
        // half, the sum of squares chained in column order.
        constexpr bool norm = EPI == EPI_RECON_NORM;
        const int row = m0 + quarter * 32 + lane;
        const bool rv = row < g.M;
        const float* xrow = g.rc_state + (int64_t)row * g.rc_lds;
        const TOut* arow = g.rc_add ? static_cast<const TOut*>(g.rc_add) + (int64_t)row * g.rc_lda : nullptr;
        TOut* lrow = norm && g.rc_low ? static_cast<TOut*>(g.rc_low) + (int64_t)row * g.rc_ldl : nullptr;
        float* orow = g.rc_out + (int64_t)row * g.rc_ldo;
        float t[norm ? 16 : 1];  // fused norm: this half's 4-column-group sums of squares, first butterfly level applied
        static_assert(BN == 256, "four 32-column chunks per half");
#pragma unroll(norm ? 4 : 1)
        for (int cc = 0; cc < 4; ++cc) {
          const int c = half * (BN / 2) + cc * 32;
          uint32_t r[32];
          tmem_ld_32cols_nowait(t_row + c, r);
          const int col = n0 + c;
          const bool cv = rv && col < g.N;  // N is a multiple of 32 (host check)
          float4 xv[8];
          uint4 av[4];
          if (cv) {  // the state (and addend) chunk loads overlap the TMEM load
#pragma unroll
            for (int j = 0; j < 8; ++j) xv[j] = __ldg(reinterpret_cast<const float4*>(xrow + col) + j);
            if (arow) {
#pragma unroll
              for (int j = 0; j < 4; ++j) av[j] = __ldg(reinterpret_cast<const uint4*>(arow + col) + j);
            }
          }
          tmem_ld_wait();
          if (cc == 3) {  // last TMEM read of this tile by this warp
            tc_fence_before();
            mbar_arrive(tempty0 + 8 * acc);
          }
          if (cv) {
            const float* xs = reinterpret_cast<const float*>(xv);
            const uint32_t* aw = reinterpret_cast<const uint32_t*>(av);
            float o[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float mv = round_to<TOut>(__uint_as_float(r[e]));
              const float f = arow ? round_to<TOut>(__fadd_rn(mv, unpack_half<TOut>(aw[e >> 1], e & 1))) : mv;
              o[e] = __fsub_rn(xs[e], round_to<TOut>(__fmul_rn(g.rc_coeff, f)));
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<float4*>(orow + col)[j] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            if (norm && lrow) {  // the rounded sublayer output itself (what rk_gemm_fprop stores)
              uint32_t lo[16];
#pragma unroll
              for (int k = 0; k < 16; ++k) lo[k] = pack2_rn<TOut>(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(lrow + col)[j] = make_uint4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
            }
            if constexpr (norm) {  // group l = 8 cc + k; groups 16..31 are added onto l - 16 (the butterfly's first level)
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const float q = sumsq4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                if (cc < 2) t[cc * 8 + k] = q;
                else t[(cc - 2) * 8 + k] = __fadd_rn(t[(cc - 2) * 8 + k], q);
              }
            }
          }
        }
        if constexpr (norm) {
          // Row total in the standalone RMSNorm's order: the 32 group sums of
          // each half in xor-butterfly order, then half 0 + half 1. Half 0
          // hands its total to the half-1 warp of the same rows (barrier A),
          // which forms rstd and hands it back (barrier B); every wait bounded.
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) {
#pragma unroll
            for (int l = 0; l < o; ++l) t[l] = __fadd_rn(t[l], t[l + o]);
          }
          const uint32_t barA = ubar0 + 8 * (2 * quarter), barB = barA + 8;
          float* slot = reinterpret_cast<float*>(sOut) + quarter * 64 + lane;  // [rows][half-0 total | rstd]
          bool xok = true;
          float rs;
          if (half == 0) {
            slot[0] = t[0];
            __syncwarp();
            if (lane == 0) mbar_arrive(barA);
            xok = mbar_wait(barB, xtiles & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
            xok = __all_sync(0xffffffffu, xok);
            if (!xok) break;
            rs = slot[32];
          } else {
            xok = mbar_wait(barA, xtiles & 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
            xok = __all_sync(0xffffffffu, xok);
            if (!xok) break;
            rs = rms_rstd(__fadd_rn(slot[0], t[0]), g.N, g.rn_eps);
            slot[32] = rs;
            __syncwarp();
            if (lane == 0) mbar_arrive(barB);
            if (rv && g.rn_rstd) g.rn_rstd[row] = rs;
          }
          ++xtiles;
          // Pass 2: y = round((state' * rstd) * w) from this thread's own
          // stores of pass 1 (plain loads: written in this kernel).
          if (rv) {
            TOut* yrow = static_cast<TOut*>(g.rn_y) + (int64_t)row * g.rn_ldy;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const int col = n0 + half * (BN / 2) + cc * 32;
              float4 pv[8], wv[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                pv[j] = reinterpret_cast<const float4*>(orow + col)[j];
                wv[j] = __ldg(reinterpret_cast<const float4*>(g.rn_w + col) + j);
              }
              const float* ps = reinterpret_cast<const float*>(pv);
              const float* ws = reinterpret_cast<const float*>(wv);
              uint32_t yw[16];
#pragma unroll
              for (int k = 0; k < 16; ++k)
                yw[k] = pack2_rn<TOut>(__fmul_rn(__fmul_rn(ps[2 * k], rs), ws[2 * k]),
                                       __fmul_rn(__fmul_rn(ps[2 * k + 1], rs), ws[2 * k + 1]));
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(yrow + col)[j] = make_uint4(yw[4 * j], yw[4 * j + 1], yw[4 * j + 2], yw[4 * j + 3]);
            }
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      const int row = m0 + quarter * 32 + lane;
      TOut* out_row;
      int64_t ldo;
      if constexpr (EPI == EPI_PARTIAL) {
        ldo = g.N;
        out_row = reinterpret_cast<TOut*>(g.out) + (int64_t)split * g.split_rows * g.N + (int64_t)row * ldo;
      } else {
        ldo = g.ldo;
        out_row = reinterpret_cast<TOut*>(g.out) + (int64_t)row * ldo;
      }
      const bool vec_ok = ((ldo * (int64_t)sizeof(TOut)) % 16 == 0) &&
                          ((reinterpret_cast<uintptr_t>(out_row) & 15) == 0);
#pragma unroll 1
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
        float v[32];
        tmem_ld_32cols(t_row + c, v);
        const int col = n0 + c;
        if (row < g.M && col < g.N) {
          if constexpr (EPI == EPI_ACCUM) accum_row_chunk<TOut>(out_row + col, v, g.N - col, vec_ok);
          store_row_chunk<TOut>(out_row + col, v, g.N - col, vec_ok);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty0 + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if constexpr (EPI == EPI_SWIGLU_BWD) {
      // u loads issued for a tile that was abandoned land before the CTA exits
      if (lane == 0) {
        for (int ch = 0; ch < 2; ++ch)
          if (upend & (1u << ch))
            mbar_wait(ubar0 + 8 * (ew * 2 + ch), (uphase >> ch) & 1u, g.status, RK_DEV_GEMM_TIMEOUT, nullptr);
      }
    }
  }

  if constexpr (epi_stages_out(EPI)) {
    if (warp >= 2 && lane == 0) bulk_wait_all();
  }
  __syncthreads();
  if (*s_abort && threadIdx.x == 0) {
    // Wait (bounded) for the TMA loads this CTA issued that no MMA consumed.
    const int consumed = *s_consumed;
    for (int i = consumed; i < issued; ++i)
      mbar_wait(full0 + 8 * (i % STAGES), (uint32_t)((i / STAGES) & 1), g.status, RK_DEV_GEMM_TIMEOUT, nullptr);
    if (RES && b_issued > *s_b_consumed)  // the last resident B load was never waited on
      mbar_wait(bfull, (uint32_t)((b_issued - 1) & 1), g.status, RK_DEV_GEMM_TIMEOUT, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// dw[r, c] (+)= sum_s partial[s][r][c] (slices `slice_rows` rows apart), in
// slice order; 4 consecutive columns per thread when cols % 4 == 0. The loads
// of up to eight slices (and of dw when accumulating) are issued before their
// sums, which stay in slice order, so the result does not depend on the batch.
template <int V, typename TOut = float>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ partial, int splits, int64_t rows,
                                                           int64_t cols, int64_t slice_rows, TOut* __restrict__ dw,
                                                           int64_t lddw, int accumulate) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t n = rows * cols / V;
  const int64_t slice = slice_rows * cols;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t * V;
    const int64_t r = i / cols, c = i - r * cols;
    TOut* d = dw + r * lddw + c;
    float o[V];
    if constexpr (std::is_same_v<TOut, float>) {  // accumulation is fp32 only (host check)
      if (accumulate) load_vec<float, V>(d, o);
    }
    float s[V];
#pragma unroll
    for (int e = 0; e < V; ++e) s[e] = 0.f;
    constexpr int B = 8;
    for (int k = 0; k < splits; k += B) {
      float v[B][V];
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (k + b < splits) load_vec<float, V>(partial + (int64_t)(k + b) * slice + i, v[b]);
#pragma unroll
      for (int b = 0; b < B; ++b)
        if (k + b < splits) {
#pragma unroll
          for (int e = 0; e < V; ++e) s[e] += v[b][e];
        }
    }
    if constexpr (std::is_same_v<TOut, float>) {
      if (accumulate) {
#pragma unroll
        for (int e = 0; e < V; ++e) s[e] += o[e];
      }
    }
    store_vec<TOut, V>(d, s);
  }
}

// ---------------------------------------------------------------- fp32 CUDA-core GEMM
// C[m,n] (+)= sum_k A[m*sam + k*sak] * B[n*sbn + k*sbk]; 64x64 tile, 256 threads, 4x4 per thread.
template <typename TOut>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, int64_t sam, int64_t sak,
                                                       const float* __restrict__ B, int64_t sbn, int64_t sbk,
                                                       TOut* __restrict__ C, int64_t ldc, int M, int N, int K,
                                                       int accumulate) {
  pdl_wait();  // inputs are the previous kernel's outputs
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      int mm, kk;
      if (sak == 1) { mm = i / 16; kk = i % 16; } else { kk = i / 64; mm = i % 64; }
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? A[gm * sam + gk * sak] : 0.f;
      int nn, kk2;
      if (sbk == 1) { nn = i / 16; kk2 = i % 16; } else { kk2 = i / 64; nn = i % 64; }
      const int gn = n0 + nn, gk2 = k0 + kk2;
      Bs[kk2][nn] = (gn < N && gk2 < K) ? B[gn * sbn + gk2 * sbk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      TOut* c = C + (int64_t)gm * ldc + gn;
      float v = acc[i][j];
      if (accumulate) v += Dt<TOut>::to_f(*c);
      *c = Dt<TOut>::from_f(v);
    }
  }
}

}  // namespace rk

using namespace rk;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = c > 0 ? c : 148;
  }
  return counts[dev];
}

// 2-D tensor map over a row-major matrix with `rows` rows of `inner` 16-bit
// elements (row stride ld), box = box_inner x box_outer, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld, int dtype,
              uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Operand description for the tensor-core path.
struct Operand {
  const void* ptr;
  int64_t ld;
  bool mn_major;  // contiguous along M (or N) instead of K
};

// B-resident schedule on/off (REVK_GEMM_RES=0 in the environment turns it off; a tuning switch).
bool res_enabled() {
  static const bool on = [] {
    const char* e = getenv("REVK_GEMM_RES");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, typename TOut, bool RES = false, int XF = XF_NONE,
          typename TIn = __nv_bfloat16>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmArgs g, int dtype,
              cudaStream_t s, const CUtensorMap* td = nullptr) {
  using L = TcSmem<BN, STAGES, epi_out_bytes(EPI), RES>;
  static_assert(L::kTotal <= 232448, "shared memory over the per-block limit");
  auto kern = gemm_tc_kernel<BN, STAGES, A_MN, B_MN, EPI, TOut, RES, XF, TIn>;
  if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)L::kTotal)) return e_;
  const int total = g.tiles_m * g.tiles_n * g.splits;
  int grid = sm_count();
  if (total < grid) grid = total;
  const uint32_t idesc = idesc_f16(kBM, BN, dtype == RK_BF16 ? 1 : 0, A_MN ? 1 : 0, B_MN ? 1 : 0);
  rk_host::launch_k(kern, grid, gemm_threads(EPI), L::kTotal, s, ta, tb, tc, td ? *td : tc, g, idesc);
  return rk_host::launch_status();
}

template <int BN, int EPI, typename TOut>
int dispatch_major(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, bool a_mn, bool b_mn,
                   const GemmArgs& g, int dtype, cudaStream_t s) {
  constexpr int ST = BN == 256 ? 4 : 6;
  if (!a_mn && !b_mn) {
    // K <= 256 with one slice: keep the B block resident (fprop of the d_model-wide inputs)
    if constexpr (EPI == EPI_TMA || EPI == EPI_STORE) {
      if (g.kb_total <= kResKb && g.splits == 1 && res_enabled())
        return launch_tc<BN, 4, false, false, EPI, TOut, true>(ta, tb, tc, g, dtype, s);
    }
    return launch_tc<BN, ST, false, false, EPI, TOut>(ta, tb, tc, g, dtype, s);
  }
  if (!a_mn && b_mn) return launch_tc<BN, ST, false, true, EPI, TOut>(ta, tb, tc, g, dtype, s);
  if (a_mn && b_mn) return launch_tc<BN, ST, true, true, EPI, TOut>(ta, tb, tc, g, dtype, s);
  return RK_ERR_UNSUPPORTED;
}

// Output tensor map for the TMA-store epilogue: [M, N] row-major, box CW x 32 rows.
bool make_out_map(CUtensorMap* map, void* base, uint64_t N, uint64_t M, uint64_t ld, int out_dtype) {
  auto fn = encode_fn();
  if (!fn) return false;
  const uint32_t esz = out_dtype == RK_F32 ? 4 : 2;
  cuuint64_t dims[2] = {N, M};
  cuuint64_t strides[1] = {ld * esz};
  cuuint32_t box[2] = {128 / esz, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = out_dtype == RK_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : out_dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 16-bit [rows, inner] map with 32 x 32 boxes (64-byte rows, 64-byte swizzle):
// the staging boxes of the 16-warp epilogues (one warp's 32 rows x 32 columns).
bool make_box32_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld, int dtype) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output-tile width: 256 (fewer A-tile reads, measured faster than 128 on every
// shape of this model, including the narrow N=256 ones); 128 only for N <= 128.
// REVK_GEMM_BN=128|256 in the environment pins it (a tuning override).
int pick_bn(int M, int N) {
  (void)M;
  static int forced = [] {
    const char* e = getenv("REVK_GEMM_BN");
    return e ? atoi(e) : 0;
  }();
  if (forced == 128 || forced == 256) return forced;
  return N <= 128 ? 128 : 256;
}

// Tensor-core GEMM: C[M,N] = sum_k A(m,k) B(n,k).
int tc_gemm(Operand a, Operand b, int M, int N, int K, int dtype, void* out, int64_t ldo, int out_dtype, int splits,
            cudaStream_t s, bool accumulate = false, int split_rows = 0, int bn = 0, const void* dsum_o = nullptr,
            int64_t dsum_ldo = 0, float* dsum = nullptr, int dsum_T = 0, int dsum_H = 0) {
  const size_t esz = 2;
  if (!rk_host::aligned(a.ptr, 16) || !rk_host::aligned(b.ptr, 16)) return RK_ERR_ALIGN;
  if ((a.ld * esz) % 16 || (b.ld * esz) % 16) return RK_ERR_ALIGN;
  const int BN = bn ? bn : pick_bn(M, N);
  CUtensorMap ta, tb;
  bool ok;
  if (a.mn_major) ok = make_map(&ta, a.ptr, (uint64_t)M, (uint64_t)K, (uint64_t)a.ld, dtype, 64, 64);
  else ok = make_map(&ta, a.ptr, (uint64_t)K, (uint64_t)M, (uint64_t)a.ld, dtype, 64, kBM);
  if (!ok) return RK_ERR_LAUNCH;
  if (b.mn_major) ok = make_map(&tb, b.ptr, (uint64_t)N, (uint64_t)K, (uint64_t)b.ld, dtype, 64, 64);
  else ok = make_map(&tb, b.ptr, (uint64_t)K, (uint64_t)N, (uint64_t)b.ld, dtype, 64, (uint32_t)BN);
  if (!ok) return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.tiles_m = (M + kBM - 1) / kBM;
  g.tiles_n = (N + BN - 1) / BN;
  g.kb_total = (K + kBK - 1) / kBK;
  g.splits = splits < 1 ? 1 : splits;
  g.kb_per_split = (g.kb_total + g.splits - 1) / g.splits;
  g.out = out;
  g.ldo = ldo;
  g.out_dtype = out_dtype;
  g.status = rk_host::device_status_ptr();
  g.split_rows = 0;
  CUtensorMap tc = ta;  // placeholder unless a TMA epilogue is used
  const bool mn_a = a.mn_major, mn_b = b.mn_major;
  const size_t osz = out_dtype == RK_F32 ? 4 : 2;
  if (splits > 1) {
    if (split_rows < M) return RK_ERR_ARG;
    g.split_rows = split_rows;
    // slices are split_rows (>= tiles_m*128) rows apart, so a tile's rows past
    // M never reach the next slice and the whole tile can be TMA-stored
    if (split_rows >= g.tiles_m * kBM && rk_host::aligned(out, 16) && (N * 4) % 16 == 0 &&
        make_out_map(&tc, out, (uint64_t)N, (uint64_t)split_rows * g.splits, (uint64_t)N, RK_F32)) {
      if (BN == 256) return dispatch_major<256, EPI_TMA, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      return dispatch_major<128, EPI_TMA, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    }
    if (BN == 256) return dispatch_major<256, EPI_PARTIAL, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    return dispatch_major<128, EPI_PARTIAL, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
  }
  if (accumulate) {
    if (out_dtype != RK_F32) return RK_ERR_DTYPE;
    if (rk_host::aligned(out, 16) && (ldo * 4) % 16 == 0 &&
        make_out_map(&tc, out, (uint64_t)N, (uint64_t)M, (uint64_t)ldo, RK_F32)) {
      if (BN == 256) return dispatch_major<256, EPI_TMA_ADD, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      return dispatch_major<128, EPI_TMA_ADD, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    }
    if (BN == 256) return dispatch_major<256, EPI_ACCUM, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    return dispatch_major<128, EPI_ACCUM, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
  }
  const bool tma_out = rk_host::aligned(out, 16) && (ldo * (int64_t)osz) % 16 == 0 &&
                       make_out_map(&tc, out, (uint64_t)N, (uint64_t)M, (uint64_t)ldo, out_dtype);
  if (dsum) {  // output projection dgrad with D = rowsum(dO * O) per 32- or 64-column head
    if (!tma_out || BN != 256 || N % 64 || out_dtype != dtype || !dsum_o || dsum_T <= 0 || dsum_H <= 0 ||
        (dsum_H * 32 != N && dsum_H * 64 != N) ||
        M % dsum_T || !rk_host::aligned(dsum_o, 16) || (dsum_ldo * 2) % 16)
      return RK_ERR_UNSUPPORTED;
    g.dsum_o = dsum_o;
    g.dsum_ldo = dsum_ldo;
    g.dsum = dsum;
    g.dsum_T = dsum_T;
    g.dsum_H = dsum_H;
    g.dsum_hw = N / dsum_H;
    if (out_dtype == RK_BF16) return dispatch_major<256, EPI_TMA_DSUM, __nv_bfloat16>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    if (out_dtype == RK_F16) return dispatch_major<256, EPI_TMA_DSUM, __half>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    return RK_ERR_DTYPE;
  }
  switch (out_dtype) {
    case RK_F32:
      if (tma_out) {
        if (BN == 256) return dispatch_major<256, EPI_TMA, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
        return dispatch_major<128, EPI_TMA, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      }
      if (BN == 256) return dispatch_major<256, EPI_STORE, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      return dispatch_major<128, EPI_STORE, float>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    case RK_BF16:
      if (tma_out) {
        if (BN == 256) return dispatch_major<256, EPI_TMA, __nv_bfloat16>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
        return dispatch_major<128, EPI_TMA, __nv_bfloat16>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      }
      if (BN == 256) return dispatch_major<256, EPI_STORE, __nv_bfloat16>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      return dispatch_major<128, EPI_STORE, __nv_bfloat16>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    case RK_F16:
      if (tma_out) {
        if (BN == 256) return dispatch_major<256, EPI_TMA, __half>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
        return dispatch_major<128, EPI_TMA, __half>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      }
      if (BN == 256) return dispatch_major<256, EPI_STORE, __half>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
      return dispatch_major<128, EPI_STORE, __half>(ta, tb, tc, mn_a, mn_b, g, dtype, s);
    default:
      return RK_ERR_DTYPE;
  }
}

template <typename TOut>
int f32_gemm_typed(const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbn, int64_t sbk, void* C,
                   int64_t ldc, int M, int N, int K, int accumulate, cudaStream_t s) {
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  rk_host::launch_k(gemm_f32_kernel<TOut>, grid, 256, 0, s, A, sam, sak, B, sbn, sbk, static_cast<TOut*>(C), ldc, M, N, K, accumulate);
  return rk_host::launch_status();
}

int f32_gemm(const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbn, int64_t sbk, void* C, int64_t ldc,
             int out_dtype, int M, int N, int K, int accumulate, cudaStream_t s) {
  if ((M + 63) / 64 > 65535) return RK_ERR_UNSUPPORTED;
  switch (out_dtype) {
    case RK_F32: return f32_gemm_typed<float>(A, sam, sak, B, sbn, sbk, C, ldc, M, N, K, accumulate, s);
    case RK_BF16: return f32_gemm_typed<__nv_bfloat16>(A, sam, sak, B, sbn, sbk, C, ldc, M, N, K, accumulate, s);
    case RK_F16: return f32_gemm_typed<__half>(A, sam, sak, B, sbn, sbk, C, ldc, M, N, K, accumulate, s);
    default: return RK_ERR_DTYPE;
  }
}

bool dims_ok(int64_t M, int64_t N, int64_t K) {
  return M >= 0 && N > 0 && K >= 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31);
}

// Output-tile width of the split weight-gradient GEMM: 256 (each 64-token
// k-block brings 48 KB for 4.2 MFLOP instead of 32 KB for 2.1 MFLOP, and the
// operand loads from L2, not the MMA, bound the narrow tiles; the MLP
// backward GEMMs measured 86 us against 97 us with 128-wide tiles).
// REVK_WGRAD_BN=128 in the environment selects the narrow tiles (a tuning switch).
int wgrad_bn() {
  static const int bn = [] {
    const char* e = getenv("REVK_WGRAD_BN");
    return (e && atoi(e) == 128) ? 128 : 256;
  }();
  return bn;
}

// CTAs the split weight-gradient GEMM aims for: about half the SMs. The
// trainer runs these GEMMs on a side stream beside the reverse sweep, where
// fewer slices (less fp32 partial traffic, fewer SMs held) measured faster
// than filling the GPU (8.79 against 8.97 ms per cfg2 update).
// REVK_WGRAD_CTAS in the environment sets it (a tuning switch).
int wgrad_ctas() {
  static const int n = [] {
    const char* e = getenv("REVK_WGRAD_CTAS");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 74;
  }();
  return n;
}

int wgrad_splits(int64_t M, int64_t N, int64_t K) {
  // Output tiles of dW[N,K] (128 x wgrad_bn() when split); choose slices so
  // that tiles*slices fills ~wgrad_ctas() CTAs, with each slice at least 8
  // k-blocks (512 tokens) long. Fixed per shape.
  const int64_t tiles = ((N + 127) / 128) * ((K + wgrad_bn() - 1) / wgrad_bn());
  const int64_t kb = (M + 63) / 64;
  int64_t s = (wgrad_ctas() + tiles - 1) / tiles;
  if (s > kb / 8) s = kb / 8;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  // Every slice must own at least one k block: recompute the count from the
  // per-slice length the kernel will use.
  const int64_t per = (kb + s - 1) / s;
  return (int)((kb + per - 1) / per);
}

}  // namespace

extern "C" int rk_gemm_fprop(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int64_t M,
                             int64_t N, int64_t K, int dtype, int out_dtype, void* stream) {
  if (!x || !w || !y || !dims_ok(M, N, K) || ldx < K || ldw < K || ldy < N || K == 0) return RK_ERR_ARG;
  if (M == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_F32)
    return f32_gemm(static_cast<const float*>(x), ldx, 1, static_cast<const float*>(w), ldw, 1, y, ldy, out_dtype,
                    (int)M, (int)N, (int)K, 0, s);
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  return tc_gemm({x, ldx, false}, {w, ldw, false}, (int)M, (int)N, (int)K, dtype, y, ldy, out_dtype, 1, s);
}

extern "C" int rk_gemm_dgrad(const void* dy, int64_t lddy, const void* w, int64_t ldw, void* dx, int64_t lddx,
                             int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, void* stream) {
  // DX[M,K] = DY[M,N] . W[N,K]: output cols = K, reduction = N.
  if (!dy || !w || !dx || !dims_ok(M, K, N) || lddy < N || ldw < K || lddx < K || N == 0 || K == 0)
    return RK_ERR_ARG;
  if (M == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_F32)
    return f32_gemm(static_cast<const float*>(dy), lddy, 1, static_cast<const float*>(w), 1, ldw, dx, lddx, out_dtype,
                    (int)M, (int)K, (int)N, 0, s);
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  return tc_gemm({dy, lddy, false}, {w, ldw, true}, (int)M, (int)K, (int)N, dtype, dx, lddx, out_dtype, 1, s);
}

extern "C" int rk_gemm_dgrad_dsum(const void* dy, int64_t lddy, const void* w, int64_t ldw, void* dx, int64_t lddx,
                                  int64_t M, int64_t N, int64_t K, int dtype, const void* o, int64_t ldo, float* dsum,
                                  int64_t T, int64_t H, void* stream) {
  // DX[M,K] = DY[M,N] . W[N,K] as rk_gemm_dgrad (16-bit out), and D[b, h, t] =
  // sum over head h's columns of DX * O, O [M, K] with K = H * 32 or H * 64.
  if (!dy || !w || !dx || !o || !dsum || !dims_ok(M, K, N) || lddy < N || ldw < K || lddx < K || ldo < K || N == 0 ||
      K == 0 || T <= 0 || H <= 0 || (K != H * 32 && K != H * 64) || M % T)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (M == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return tc_gemm({dy, lddy, false}, {w, ldw, true}, (int)M, (int)K, (int)N, dtype, dx, lddx, dtype, 1, s, false, 0,
                 256, o, ldo, dsum, (int)T, (int)H);
}

extern "C" int64_t rk_gemm_wgrad_workspace(int64_t M, int64_t N, int64_t K) {
  const int s = wgrad_splits(M, N, K);
  const int64_t slice_rows = (N + kBM - 1) / kBM * kBM;
  return (int64_t)s * slice_rows * K * (int64_t)sizeof(float);
}

extern "C" int rk_gemm_wgrad(const void* dy, int64_t lddy, const void* x, int64_t ldx, float* dw, int64_t lddw,
                             int64_t M, int64_t N, int64_t K, int dtype, int accumulate, float* workspace,
                             int64_t workspace_bytes, void* stream) {
  // DW[N,K] (+)= DY[M,N]^T . X[M,K]: output rows = N, cols = K, reduction = M tokens.
  if (!dy || !x || !dw || !dims_ok(N, K, M) || lddy < N || ldx < K || lddw < K || N == 0 || K == 0)
    return RK_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0) {
    if (!accumulate)
      for (int64_t r = 0; r < N; ++r) cudaMemsetAsync(dw + r * lddw, 0, sizeof(float) * K, s);
    return rk_host::launch_status();
  }
  if (dtype == RK_F32)
    return f32_gemm(static_cast<const float*>(dy), 1, lddy, static_cast<const float*>(x), 1, ldx, dw, lddw, RK_F32,
                    (int)N, (int)K, (int)M, accumulate, s);
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  const int splits = wgrad_splits(M, N, K);
  if (splits == 1)  // enough output tiles: write (or accumulate into) dw directly, no workspace
    return tc_gemm({dy, lddy, true}, {x, ldx, true}, (int)N, (int)K, (int)M, dtype, dw, lddw, RK_F32, 1, s,
                   accumulate != 0);
  const int64_t slice_rows = (N + kBM - 1) / kBM * kBM;
  const int64_t need = (int64_t)splits * slice_rows * K * (int64_t)sizeof(float);
  if (!workspace || workspace_bytes < need) return RK_ERR_WORKSPACE;
  const int st = tc_gemm({dy, lddy, true}, {x, ldx, true}, (int)N, (int)K, (int)M, dtype, workspace, K, RK_F32,
                         splits, s, false, (int)slice_rows, wgrad_bn());
  if (st != RK_OK) return st;
  const bool vec = K % 4 == 0 && lddw % 4 == 0 && rk_host::aligned(dw, 16) && rk_host::aligned(workspace, 16);
  int64_t blocks = (N * K / (vec ? 4 : 1) + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (vec)
    rk_host::launch_k(split_reduce_kernel<4>, (unsigned)blocks, 256, 0, s, workspace, splits, N, K, slice_rows, dw, lddw, accumulate);
  else
    rk_host::launch_k(split_reduce_kernel<1>, (unsigned)blocks, 256, 0, s, workspace, splits, N, K, slice_rows, dw, lddw, accumulate);
  return rk_host::launch_status();
}

// ---------------------------------------------------------------- reversible state update
static int fprop_reconstruct(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* state, int64_t lds,
                             const void* addend, int64_t lda, float coeff, float* out, int64_t ldo, void* low,
                             int64_t ldl, const float* norm_w, float eps, void* y, int64_t ldy, float* rstd, int64_t M,
                             int64_t N, int64_t K, int dtype, void* stream) {
  if (!x || !w || !state || !out || !dims_ok(M, N, K) || K == 0 || ldx < K || ldw < K || lds < N || ldo < N ||
      (addend && lda < N) || (low && ldl < N) || (norm_w && (!y || ldy < N)))
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (N % 32 || (norm_w && N != 256)) return RK_ERR_UNSUPPORTED;
  if (M == 0) return RK_OK;
  if (!rk_host::aligned(x, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(state, 16) ||
      !rk_host::aligned(out, 16) || (addend && !rk_host::aligned(addend, 16)) || (ldx * 2) % 16 || (ldw * 2) % 16 ||
      lds % 4 || ldo % 4 || (addend && lda % 8) || (low && (!rk_host::aligned(low, 16) || ldl % 8)) ||
      (norm_w && (!rk_host::aligned(norm_w, 16) || !rk_host::aligned(y, 16) || ldy % 8)))
    return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb;
  if (!make_map(&ta, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, dtype, 64, kBM) ||
      !make_map(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, dtype, 64, 256))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)((N + 255) / 256);
  g.kb_total = (int)((K + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.status = rk_host::device_status_ptr();
  g.rc_state = state;
  g.rc_lds = lds;
  g.rc_add = addend;
  g.rc_lda = lda;
  g.rc_out = out;
  g.rc_ldo = ldo;
  g.rc_coeff = coeff;
  g.rc_low = low;
  g.rc_ldl = ldl;
  g.rn_w = norm_w;
  g.rn_y = y;
  g.rn_ldy = ldy;
  g.rn_rstd = rstd;
  g.rn_eps = eps;
  if (norm_w) {
    if (dtype == RK_BF16)
      return launch_tc<256, 4, false, false, EPI_RECON_NORM, __nv_bfloat16>(ta, tb, ta, g, dtype, s);
    return launch_tc<256, 4, false, false, EPI_RECON_NORM, __half>(ta, tb, ta, g, dtype, s);
  }
  if (dtype == RK_BF16) return launch_tc<256, 4, false, false, EPI_RECON, __nv_bfloat16>(ta, tb, ta, g, dtype, s);
  return launch_tc<256, 4, false, false, EPI_RECON, __half>(ta, tb, ta, g, dtype, s);
}

// out = state - round(coeff * round(round(x W^T) + addend)): the sublayer
// output projection (the MLP down projection, or the attention output
// projection for the Euler recurrence) with the reconstruction / forward state
// update of reversible.py:21-32 in its epilogue, so the sublayer output never
// reaches HBM. Bitwise equal to rk_gemm_fprop followed by
// rk_reconstruct_midpoint_sum (addend given) or rk_reconstruct_midpoint.
extern "C" int rk_gemm_fprop_reconstruct(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* state,
                                         int64_t lds, const void* addend, int64_t lda, float coeff, float* out,
                                         int64_t ldo, int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  return fprop_reconstruct(x, ldx, w, ldw, state, lds, addend, lda, coeff, out, ldo, nullptr, 0, nullptr, 0.f, nullptr,
                           0, nullptr, M, N, K, dtype, stream);
}

// The same state update followed, in the same pass, by the RMSNorm forward of
// the updated state (the next sublayer's input norm, model.py:62-64):
// y = round((out * rstd) * norm_w), rstd = rsqrt(mean(out^2) + eps), bitwise
// equal to rk_rmsnorm_fwd (fp32 x) or rk_add_rmsnorm_fwd on `out`. Optionally
// (low != NULL) also stores round(x W^T) itself, as rk_gemm_fprop would.
// N must be 256 (one output tile spans the row).
extern "C" int rk_gemm_fprop_reconstruct_norm(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                              const float* state, int64_t lds, const void* addend, int64_t lda,
                                              float coeff, float* out, int64_t ldo, void* low, int64_t ldl,
                                              const float* norm_w, float eps, void* y, int64_t ldy, float* rstd,
                                              int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  if (!norm_w) return RK_ERR_ARG;
  return fprop_reconstruct(x, ldx, w, ldw, state, lds, addend, lda, coeff, out, ldo, low, ldl, norm_w, eps, y, ldy,
                           rstd, M, N, K, dtype, stream);
}

// ---------------------------------------------------------------- fused SwiGLU up projection
extern "C" int rk_gemm_fprop_swiglu(const void* x, int64_t ldx, const void* w_up, int64_t ldw, void* h, int64_t ldh,
                                    void* u, int64_t ldu, int64_t M, int64_t ff, int64_t K, int dtype, void* stream) {
  if (!x || !w_up || !h || M < 0 || ff <= 0 || K <= 0 || ldx < K || ldw < K || ldh < ff || (u && ldu < 2 * ff))
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (ff % 128) return RK_ERR_UNSUPPORTED;
  if (M == 0) return RK_OK;
  if (!rk_host::aligned(x, 16) || !rk_host::aligned(w_up, 16) || !rk_host::aligned(h, 16) ||
      (u && !rk_host::aligned(u, 16)) || (ldx * 2) % 16 || (ldw * 2) % 16 || (ldh * 2) % 16 || (u && (ldu * 2) % 16))
    return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb, tc, td;
  if (!make_map(&ta, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, dtype, 64, kBM) ||
      !make_map(&tb, w_up, (uint64_t)K, (uint64_t)(2 * ff), (uint64_t)ldw, dtype, 64, 128) ||
      !make_out_map(&tc, h, (uint64_t)ff, (uint64_t)M, (uint64_t)ldh, dtype))
    return RK_ERR_LAUNCH;
  if (u && !make_out_map(&td, u, (uint64_t)(2 * ff), (uint64_t)M, (uint64_t)ldu, dtype)) return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)(2 * ff);
  g.K = (int)K;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)(ff / 128);
  g.kb_total = (int)((K + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.ff = (int)ff;
  g.out = h;
  g.ldo = ldh;
  g.out_dtype = dtype;
  g.status = rk_host::device_status_ptr();
  if (dtype == RK_BF16) {
    if (u) return launch_tc<256, 3, false, false, EPI_SWIGLU_SAVE, __nv_bfloat16>(ta, tb, tc, g, dtype, s, &td);
    if (g.kb_total <= kResKb && res_enabled())
      return launch_tc<256, 4, false, false, EPI_SWIGLU, __nv_bfloat16, true>(ta, tb, tc, g, dtype, s);
    return launch_tc<256, 4, false, false, EPI_SWIGLU, __nv_bfloat16>(ta, tb, tc, g, dtype, s);
  }
  if (u) return launch_tc<256, 3, false, false, EPI_SWIGLU_SAVE, __half>(ta, tb, tc, g, dtype, s, &td);
  return launch_tc<256, 4, false, false, EPI_SWIGLU, __half>(ta, tb, tc, g, dtype, s);
}

// ---------------------------------------------------------------- fused down-projection dgrad + SwiGLU backward
// du = swiglu_bwd(u, round(dy . w)): the down projection's dgrad (dy [M, N],
// w [N, ff], N = d_model) with rk_swiglu_bwd applied in the epilogue to the
// rounded result, reading u [M, 2ff] (gate columns first) and writing du of
// the same layout; dh never reaches global memory.
extern "C" int rk_gemm_dgrad_swiglu(const void* dy, int64_t lddy, const void* w, int64_t ldw, const void* u,
                                    int64_t ldu, void* du, int64_t lddu, int64_t M, int64_t ff, int64_t N, int dtype,
                                    void* stream) {
  if (!dy || !w || !u || !du || M < 0 || ff <= 0 || N <= 0 || lddy < N || ldw < ff || ldu < 2 * ff ||
      lddu < 2 * ff || M > INT32_MAX || ff > INT32_MAX / 2 || N > INT32_MAX)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (ff % 64) return RK_ERR_UNSUPPORTED;
  if (M == 0) return RK_OK;
  if (!rk_host::aligned(dy, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(u, 16) || !rk_host::aligned(du, 16) ||
      (lddy * 2) % 16 || (ldw * 2) % 16 || (ldu * 2) % 16 || (lddu * 2) % 16)
    return RK_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb, tc, td;
  if (!make_map(&ta, dy, (uint64_t)N, (uint64_t)M, (uint64_t)lddy, dtype, 64, kBM) ||
      !make_map(&tb, w, (uint64_t)ff, (uint64_t)N, (uint64_t)ldw, dtype, 64, 64) ||
      !make_box32_map(&tc, du, (uint64_t)(2 * ff), (uint64_t)M, (uint64_t)lddu, dtype) ||
      !make_box32_map(&td, u, (uint64_t)(2 * ff), (uint64_t)M, (uint64_t)ldu, dtype))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)ff;
  g.K = (int)N;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)((ff + 255) / 256);
  g.kb_total = (int)((N + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.ff = (int)ff;
  g.out = du;
  g.ldo = lddu;
  g.out_dtype = dtype;
  g.status = rk_host::device_status_ptr();
  if (dtype == RK_BF16)
    return launch_tc<256, 2, false, true, EPI_SWIGLU_BWD, __nv_bfloat16>(ta, tb, tc, g, dtype, s, &td);
  return launch_tc<256, 2, false, true, EPI_SWIGLU_BWD, __half>(ta, tb, tc, g, dtype, s, &td);
}

// ---------------------------------------------------------------- softmax head
// The vocabulary head and its cross-entropy without a pass of their own over
// the logits (the head GEMM and F.cross_entropy of model.py:104 and
// train_baseline.py:262, and their backward):
//   rk_head_fprop : e = exp(logit - m_b) (16-bit; m_b the max of the row's
//                   128-column block b of rounded logits), (m_b, sum e) per
//                   (row, b), and the logit at each row's label;
//   rk_head_loss  : lse = log-sum-exp over the blocks, loss = lse - logit[label],
//                   and per row (-lse*log2 e, scale, (exp(logit[label]-lse)-1)*scale);
//   rk_head_dgrad : dhidden = dlogits . W and
//   rk_head_wgrad : dW (+)= dlogits^T . hidden, each GEMM forming
//                   dlogit = e * exp(m_b - lse) * scale (label entry exact) in
//                   shared memory, so dlogits never exist in global memory.
namespace rk {

// 32 rows per CTA: warp w reduces rows w, w+8, .. of the CTA's 32 (lse, loss,
// rowc), then the CTA writes fcoef[b][row] = exp(m_b - lse) * scale for every
// block b with 32 consecutive rows per store (coalesced).
__global__ void __launch_bounds__(256, 4) head_loss_kernel(const float2* __restrict__ stats, int width,
                                                        const float* __restrict__ xlabel, int vocab,
                                                        const int64_t* __restrict__ labels, int rows, float scale,
                                                        const float* __restrict__ scale_dev,
                                                        float* __restrict__ loss_rows, float4* __restrict__ rowc,
                                                        float* __restrict__ fcoef, int64_t fcoef_ld,
                                                        int ignore_index, unsigned int* status) {
  pdl_wait();  // inputs are the previous kernel's outputs
  __shared__ float s_nl[32], s_sc[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * 32;
  if (scale_dev) scale *= *scale_dev;
  // Per row (the warp's rows warp, warp + 8, ..), up to 512 entries at a
  // time, 16 per lane loaded together (entries lane, lane + 32, ..): the
  // chunk's max over the warp (exact in any order) raises the running max M
  // (rescaling the lane's sum once when it rises), then each lane adds
  // s_b * 2^((m_b - M) log2 e) in entry order, and the lanes' sums add in a
  // fixed butterfly (every lane ends with the same sum).
  constexpr int kPer = 16;
#pragma unroll 1
  for (int r = 0; r < 4; ++r) {
    const int rr = warp + 8 * r;
    const int row = row0 + rr;
    float m = -INFINITY, s = 0.f;
    if (row < rows) {
      const float2* st = stats + (int64_t)row * width;
      for (int c0 = 0; c0 < width; c0 += 32 * kPer) {
        float2 p[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = c0 + lane + 32 * k;
          p[k] = i < width ? st[i] : make_float2(-INFINITY, 0.f);
        }
        float mc = p[0].x;
#pragma unroll
        for (int k = 1; k < kPer; ++k) mc = fmaxf(mc, p[k].x);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
        const float mn = fmaxf(m, mc);
        if (mn == -INFINITY) continue;  // warp-uniform: no block with a valid column yet
        if (mn > m && m != -INFINITY) s = __fmul_rn(s, ex2_fast(__fmul_rn(__fsub_rn(m, mn), kLog2eF)));
        m = mn;
#pragma unroll
        for (int k = 0; k < kPer; ++k)
          s = __fmaf_rn(p[k].y, ex2_fast(__fmul_rn(__fsub_rn(p[k].x, mn), kLog2eF)), s);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (row >= rows) {
      if (lane == 0) {
        s_nl[rr] = 0.f;
        s_sc[rr] = 0.f;
      }
      continue;
    }
    if (lane == 0) {
      const int64_t label = labels[row];
      const bool ignored = label == ignore_index;
      const bool bad = !ignored && (label < 0 || label >= vocab);
      if (bad) flag_error(status, RK_DEV_CE_LABEL);
      if (ignored || bad) {
        loss_rows[row] = 0.f;
        rowc[row] = make_float4(0.f, 0.f, 0.f, 0.f);
        s_nl[rr] = 0.f;
        s_sc[rr] = 0.f;
      } else {
        const float lse = m + logf(s);
        const float xl = xlabel[row];
        const float nl = -lse * kLog2eF;
        loss_rows[row] = lse - xl;
        rowc[row] = make_float4(nl, scale, (ex2_fast(fmaf(xl, kLog2eF, nl)) - 1.f) * scale, 0.f);
        s_nl[rr] = nl;
        s_sc[rr] = scale;
      }
    }
  }
  __syncthreads();
  // fcoef[b][row] for the CTA's rows: lane = row; each warp takes four
  // consecutive blocks at a time (the row's four (m_b, s) entries are one
  // 32-byte sector, read as two 16-byte loads) and stores each block's 32
  // rows contiguously
  const int nrow = min(32, rows - row0);
  const bool live = lane < nrow;
  const float nl = s_nl[lane], sc = s_sc[lane];
  const float2* srow = stats + (int64_t)(row0 + lane) * width;
  const bool vec = (reinterpret_cast<uintptr_t>(stats) & 15) == 0 && width % 2 == 0;
  for (int b0 = warp * 4; b0 < width; b0 += 32) {
    float mb[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (live) {
      if (vec && b0 + 3 < width) {
        const float4 lo = *reinterpret_cast<const float4*>(srow + b0);
        const float4 hi = *reinterpret_cast<const float4*>(srow + b0 + 2);
        mb[0] = lo.x;
        mb[1] = lo.z;
        mb[2] = hi.x;
        mb[3] = hi.z;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (b0 + k < width) mb[k] = srow[b0 + k].x;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (b0 + k < width)
          fcoef[(int64_t)(b0 + k) * fcoef_ld + row0 + lane] =
              (sc == 0.f || mb[k] == -INFINITY) ? 0.f : ex2_fast(fmaf(mb[k], kLog2eF, nl)) * sc;
    }
  }
}

}  // namespace rk

extern "C" int64_t rk_head_stats_width(int64_t vocab) { return vocab > 0 ? 2 * ((vocab + 255) / 256) : 0; }

extern "C" int rk_head_fprop(const void* hidden, int64_t ldh, const void* w, int64_t ldw, const int64_t* labels,
                             void* expo, int64_t lde, float* stats, float* xlabel, int64_t M, int64_t V, int64_t K,
                             int dtype, void* stream) {
  if (!hidden || !w || !labels || !expo || !stats || !xlabel || !dims_ok(M, V, K) || K == 0 || ldh < K ||
      ldw < K || lde < V)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (M == 0) return RK_OK;
  if (!rk_host::aligned(hidden, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(expo, 16) ||
      !rk_host::aligned(stats, 8) || (ldh * 2) % 16 || (ldw * 2) % 16 || (lde * 2) % 16)
    return RK_ERR_ALIGN;
  CUtensorMap ta, tb, tc;
  if (!make_map(&ta, hidden, (uint64_t)K, (uint64_t)M, (uint64_t)ldh, dtype, 64, kBM) ||
      !make_map(&tb, w, (uint64_t)K, (uint64_t)V, (uint64_t)ldw, dtype, 64, 256) ||
      !make_box32_map(&tc, expo, (uint64_t)V, (uint64_t)M, (uint64_t)lde, dtype))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)V;
  g.K = (int)K;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)((V + 255) / 256);
  g.kb_total = (int)((K + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.out = expo;
  g.ldo = lde;
  g.out_dtype = dtype;
  g.status = rk_host::device_status_ptr();
  g.stats = reinterpret_cast<float2*>(stats);
  g.stats_ld = 2 * g.tiles_n;
  g.labels = labels;
  g.xlabel = xlabel;
  g.vocab = (int)V;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool res = g.kb_total <= kResKb && res_enabled();
  if (dtype == RK_BF16) {
    if (res) return launch_tc<256, 4, false, false, EPI_LSE, __nv_bfloat16, true>(ta, tb, tc, g, dtype, s);
    return launch_tc<256, 4, false, false, EPI_LSE, __nv_bfloat16>(ta, tb, tc, g, dtype, s);
  }
  if (res) return launch_tc<256, 4, false, false, EPI_LSE, __half, true>(ta, tb, tc, g, dtype, s);
  return launch_tc<256, 4, false, false, EPI_LSE, __half>(ta, tb, tc, g, dtype, s);
}

extern "C" int rk_head_loss(const float* stats, int64_t width, const float* xlabel, const int64_t* labels,
                            int64_t rows, int64_t V, float grad_scale, const float* grad_scale_dev, float* loss_rows,
                            float* rowc, float* fcoef, int64_t fcoef_ld, int ignore_index, void* stream) {
  if (!stats || !xlabel || !labels || !loss_rows || !rowc || !fcoef || rows < 0 || V <= 0 || fcoef_ld < rows ||
      width < rk_head_stats_width(V) || rows >= (1ll << 31) || V >= (1ll << 31))
    return RK_ERR_ARG;
  if (!rk_host::aligned(stats, 8) || !rk_host::aligned(rowc, 16)) return RK_ERR_ALIGN;
  if (rows == 0) return RK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rk_host::launch_k(head_loss_kernel, (unsigned)((rows + 31) / 32), 256, 0, s, reinterpret_cast<const float2*>(stats),
                    (int)width, xlabel, (int)V, labels, (int)rows, grad_scale, grad_scale_dev, loss_rows,
                    reinterpret_cast<float4*>(rowc), fcoef, fcoef_ld, ignore_index, rk_host::device_status_ptr());
  return rk_host::launch_status();
}

namespace {
template <typename TIn>
int head_dgrad_typed(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                     int dtype, int out_dtype, cudaStream_t s) {
  switch (out_dtype) {
    case RK_F32: return launch_tc<256, 4, false, true, EPI_TMA, float, false, XF_ROWS, TIn>(ta, tb, tc, g, dtype, s);
    case RK_BF16:
      return launch_tc<256, 4, false, true, EPI_TMA, __nv_bfloat16, false, XF_ROWS, TIn>(ta, tb, tc, g, dtype, s);
    case RK_F16: return launch_tc<256, 4, false, true, EPI_TMA, __half, false, XF_ROWS, TIn>(ta, tb, tc, g, dtype, s);
    default: return RK_ERR_DTYPE;
  }
}
template <typename TIn>
int head_wgrad_typed(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                     int dtype, bool accumulate, cudaStream_t s) {
  if (accumulate) return launch_tc<256, 4, true, true, EPI_TMA_ADD, float, false, XF_COLS, TIn>(ta, tb, tc, g, dtype, s);
  return launch_tc<256, 4, true, true, EPI_TMA, float, false, XF_COLS, TIn>(ta, tb, tc, g, dtype, s);
}

bool head_bwd_args_ok(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                      const int64_t* labels, int64_t M, int64_t V) {
  return expo && fcoef && rowc && labels && lde >= V && fcoef_ld >= M;
}
}  // namespace

extern "C" int rk_head_dgrad(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                             const int64_t* labels, const void* w, int64_t ldw, void* dx, int64_t lddx, int64_t M,
                             int64_t V, int64_t K, int dtype, int out_dtype, void* stream) {
  // DX[M, K] = dlogits[M, V] . W[V, K]: output cols = K, reduction = V.
  if (!head_bwd_args_ok(expo, lde, fcoef, fcoef_ld, rowc, labels, M, V) || !w || !dx || !dims_ok(M, K, V) || V == 0 ||
      K == 0 || ldw < K || lddx < K)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (M == 0) return RK_OK;
  const int64_t osz = out_dtype == RK_F32 ? 4 : 2;
  if (!rk_host::aligned(expo, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(dx, 16) ||
      !rk_host::aligned(rowc, 16) || (lde * 2) % 16 || (ldw * 2) % 16 ||
      (lddx * osz) % 16)
    return RK_ERR_ALIGN;
  CUtensorMap ta, tb, tc;
  if (!make_map(&ta, expo, (uint64_t)V, (uint64_t)M, (uint64_t)lde, dtype, 64, kBM) ||
      !make_map(&tb, w, (uint64_t)K, (uint64_t)V, (uint64_t)ldw, dtype, 64, 64) ||
      !make_out_map(&tc, dx, (uint64_t)K, (uint64_t)M, (uint64_t)lddx, out_dtype))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)K;
  g.K = (int)V;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)((K + 255) / 256);
  g.kb_total = (int)((V + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.out = dx;
  g.ldo = lddx;
  g.out_dtype = out_dtype;
  g.status = rk_host::device_status_ptr();
  g.fcoef = fcoef;
  g.fcoef_ld = fcoef_ld;
  g.rowc = reinterpret_cast<const float4*>(rowc);
  g.labels = labels;
  g.vocab = (int)V;
  g.tokens = (int)M;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == RK_BF16) return head_dgrad_typed<__nv_bfloat16>(ta, tb, tc, g, dtype, out_dtype, s);
  return head_dgrad_typed<__half>(ta, tb, tc, g, dtype, out_dtype, s);
}

// Token-reduction split of the head dgrad. Its output has one 256-column tile
// per 128 tokens, fewer tiles than SMs at the training shapes (116 at cfg2), so
// the vocabulary reduction is cut into S slices, each an independent tile of
// fp32 partials, with S chosen to minimise the longest CTA's share
// ceil(tiles*S/SMs)/S (0.8 of a whole tile at cfg2 with S = 5); a
// fixed-order pass then sums the slices (deterministic). 1 = no split.
static int head_dgrad_splits(int64_t M, int64_t V, int64_t K) {
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((K + 255) / 256);
  const int64_t kb = (V + kBK - 1) / kBK;
  const int64_t sms = sm_count();
  if (tiles <= 0 || tiles >= sms) return 1;
  int best = 1;
  double best_t = 1.0;
  for (int S = 2; S <= 8 && S <= kb; ++S) {
    const double t = (double)((tiles * S + sms - 1) / sms) / S + 0.01 * S;  // + the slices' extra traffic
    if (t < best_t - 1e-9) {
      best_t = t;
      best = S;
    }
  }
  return best;
}

extern "C" int64_t rk_head_dgrad_workspace(int64_t M, int64_t V, int64_t K) {
  if (M <= 0 || V <= 0 || K <= 0) return 0;
  const int S = head_dgrad_splits(M, V, K);
  return S > 1 ? (int64_t)S * ((M + kBM - 1) / kBM) * kBM * K * 4 : 0;
}

extern "C" int rk_head_dgrad_ws(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld,
                                const float* rowc, const int64_t* labels, const void* w, int64_t ldw, void* dx,
                                int64_t lddx, int64_t M, int64_t V, int64_t K, int dtype, int out_dtype,
                                float* workspace, int64_t workspace_bytes, void* stream) {
  const int64_t need = rk_head_dgrad_workspace(M, V, K);
  const int S = head_dgrad_splits(M, V, K);
  if (need == 0 || S == 1 || !workspace || workspace_bytes < need || K % 4 || lddx % 4 ||
      !rk_host::aligned(workspace, 16))
    return rk_head_dgrad(expo, lde, fcoef, fcoef_ld, rowc, labels, w, ldw, dx, lddx, M, V, K, dtype, out_dtype,
                         stream);
  if (!head_bwd_args_ok(expo, lde, fcoef, fcoef_ld, rowc, labels, M, V) || !w || !dx || !dims_ok(M, K, V) ||
      ldw < K || lddx < K)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  if (out_dtype != RK_F32 && out_dtype != RK_BF16 && out_dtype != RK_F16) return RK_ERR_DTYPE;
  if (!rk_host::aligned(expo, 16) || !rk_host::aligned(w, 16) || !rk_host::aligned(dx, 16) ||
      !rk_host::aligned(rowc, 16) || (lde * 2) % 16 || (ldw * 2) % 16)
    return RK_ERR_ALIGN;
  const int64_t split_rows = ((M + kBM - 1) / kBM) * kBM;
  CUtensorMap ta, tb, tc;
  if (!make_map(&ta, expo, (uint64_t)V, (uint64_t)M, (uint64_t)lde, dtype, 64, kBM) ||
      !make_map(&tb, w, (uint64_t)K, (uint64_t)V, (uint64_t)ldw, dtype, 64, 64) ||
      !make_out_map(&tc, workspace, (uint64_t)K, (uint64_t)(split_rows * S), (uint64_t)K, RK_F32))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)K;
  g.K = (int)V;
  g.tiles_m = (int)((M + kBM - 1) / kBM);
  g.tiles_n = (int)((K + 255) / 256);
  g.kb_total = (int)((V + kBK - 1) / kBK);
  g.splits = S;
  g.kb_per_split = (g.kb_total + S - 1) / S;
  g.split_rows = (int)split_rows;
  g.out = workspace;
  g.ldo = K;
  g.out_dtype = RK_F32;
  g.status = rk_host::device_status_ptr();
  g.fcoef = fcoef;
  g.fcoef_ld = fcoef_ld;
  g.rowc = reinterpret_cast<const float4*>(rowc);
  g.labels = labels;
  g.vocab = (int)V;
  g.tokens = (int)M;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int st = dtype == RK_BF16
                     ? launch_tc<256, 4, false, true, EPI_TMA, float, false, XF_ROWS, __nv_bfloat16>(ta, tb, tc, g,
                                                                                                    dtype, s)
                     : launch_tc<256, 4, false, true, EPI_TMA, float, false, XF_ROWS, __half>(ta, tb, tc, g, dtype, s);
  if (st != RK_OK) return st;
  int64_t blocks = (M * K / 4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (out_dtype == RK_F32)
    rk_host::launch_k(split_reduce_kernel<4, float>, (unsigned)blocks, 256, 0, s, workspace, S, M, K, split_rows,
                      static_cast<float*>(dx), lddx, 0);
  else if (out_dtype == RK_BF16)
    rk_host::launch_k(split_reduce_kernel<4, __nv_bfloat16>, (unsigned)blocks, 256, 0, s, workspace, S, M, K,
                      split_rows, static_cast<__nv_bfloat16*>(dx), lddx, 0);
  else
    rk_host::launch_k(split_reduce_kernel<4, __half>, (unsigned)blocks, 256, 0, s, workspace, S, M, K, split_rows,
                      static_cast<__half*>(dx), lddx, 0);
  return rk_host::launch_status();
}

extern "C" int rk_head_wgrad(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                             const int64_t* labels, const void* x, int64_t ldx, float* dw, int64_t lddw, int64_t M,
                             int64_t V, int64_t K, int dtype, int accumulate, void* stream) {
  // DW[V, K] (+)= dlogits[M, V]^T . X[M, K]: output rows = V, cols = K, reduction = M tokens.
  if (!head_bwd_args_ok(expo, lde, fcoef, fcoef_ld, rowc, labels, M, V) || !x || !dw || !dims_ok(V, K, M) || V == 0 ||
      K == 0 || ldx < K || lddw < K)
    return RK_ERR_ARG;
  if (dtype != RK_BF16 && dtype != RK_F16) return RK_ERR_DTYPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0) {
    if (!accumulate)
      for (int64_t r = 0; r < V; ++r) cudaMemsetAsync(dw + r * lddw, 0, sizeof(float) * K, s);
    return rk_host::launch_status();
  }
  if (!rk_host::aligned(expo, 16) || !rk_host::aligned(x, 16) || !rk_host::aligned(dw, 16) ||
      !rk_host::aligned(rowc, 16) || (lde * 2) % 16 || (ldx * 2) % 16 ||
      (lddw * 4) % 16)
    return RK_ERR_ALIGN;
  CUtensorMap ta, tb, tc;
  if (!make_map(&ta, expo, (uint64_t)V, (uint64_t)M, (uint64_t)lde, dtype, 64, 64) ||
      !make_map(&tb, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, dtype, 64, 64) ||
      !make_out_map(&tc, dw, (uint64_t)K, (uint64_t)V, (uint64_t)lddw, RK_F32))
    return RK_ERR_LAUNCH;
  GemmArgs g{};
  g.M = (int)V;
  g.N = (int)K;
  g.K = (int)M;
  g.tiles_m = (int)((V + kBM - 1) / kBM);
  g.tiles_n = (int)((K + 255) / 256);
  g.kb_total = (int)((M + kBK - 1) / kBK);
  g.splits = 1;
  g.kb_per_split = g.kb_total;
  g.out = dw;
  g.ldo = lddw;
  g.out_dtype = RK_F32;
  g.status = rk_host::device_status_ptr();
  g.fcoef = fcoef;
  g.fcoef_ld = fcoef_ld;
  g.rowc = reinterpret_cast<const float4*>(rowc);
  g.labels = labels;
  g.vocab = (int)V;
  g.tokens = (int)M;
  if (dtype == RK_BF16) return head_wgrad_typed<__nv_bfloat16>(ta, tb, tc, g, dtype, accumulate != 0, s);
  return head_wgrad_typed<__half>(ta, tb, tc, g, dtype, accumulate != 0, s);
}
