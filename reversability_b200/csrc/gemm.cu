// Dense GEMMs for the Linear layers (replaces F.linear/cuBLAS at model.py:37,45,55-56
// and its autograd backward).
//
// bf16/f16 path: a persistent, warp-specialised tcgen05 kernel.
//   warp 0      : TMA producer (one elected thread) filling a STAGES-deep ring
//                 of 128x64 A tiles and BNx64 B tiles (128-byte swizzle).
//   warp 1      : allocates 2*BN tensor-memory columns (two accumulators) and
//                 issues tcgen05.mma (M=128, N=BN, K=16) from one thread;
//                 tcgen05.commit frees smem stages and publishes accumulators.
//   warps 2..5  : epilogue; warp w reads TMEM lanes 32*(w%4)..+31 (one output
//                 row per thread) with tcgen05.ld and stores to global memory.
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
enum { EPI_STORE = 0, EPI_PARTIAL = 1, EPI_ACCUM = 2, EPI_TMA = 3, EPI_TMA_ADD = 4, EPI_SWIGLU = 5, EPI_SWIGLU_SAVE = 6 };

__host__ __device__ constexpr bool epi_is_swiglu(int e) { return e == EPI_SWIGLU || e == EPI_SWIGLU_SAVE; }
__host__ __device__ constexpr bool epi_stages_out(int e) { return e == EPI_TMA || e == EPI_TMA_ADD || epi_is_swiglu(e); }
__host__ __device__ constexpr uint32_t epi_out_bytes(int e) {
  return e == EPI_SWIGLU_SAVE ? 4 * 3 * 4096 : (epi_stages_out(e) ? 4 * 2 * 4096 : 0);
}

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN, int STAGES, uint32_t OUT_BYTES = 0>
struct TcSmem {
  static constexpr uint32_t kA = kBM * kBK * 2;  // 16 KB
  static constexpr uint32_t kB = BN * kBK * 2;
  static constexpr uint32_t kStage = kA + kB;
  // output staging: 4 epilogue warps x 2 (or 3) buffers x (32 rows x 128 bytes)
  static constexpr uint32_t kOut = OUT_BYTES;
  static constexpr uint32_t kBarriers = (2 * STAGES + 5) * 8;
  static constexpr uint32_t kTotal = 1024 /*align slack*/ + STAGES * kStage + kOut + kBarriers + 16;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
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

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                   const GemmArgs g, const uint32_t idesc) {
  
  using L = TcSmem<BN, STAGES, epi_out_bytes(EPI)>;
  constexpr int NSTEP = epi_is_swiglu(EPI) ? BN / 2 : BN;  // output columns per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kA;
  uint8_t* sOut = smem + STAGES * L::kStage;  // EPI_TMA staging (1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStage + L::kOut);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + STAGES * 8;
  const uint32_t tfull0 = empty0 + STAGES * 8;
  const uint32_t tempty0 = tfull0 + 2 * 8;
  const uint32_t drain = tempty0 + 2 * 8;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(s_tmem + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    *s_abort = 0;
    *s_consumed = 0;
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

  const int tiles_mn = g.tiles_m * g.tiles_n;
  const int total = tiles_mn * g.splits;
  int issued = 0;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int split = t / tiles_mn;
      const int mn = t - split * tiles_mn;
      const int m0 = (mn / g.tiles_n) * kBM;
      const int n0 = (mn % g.tiles_n) * NSTEP;
      const int kb0 = split * g.kb_per_split;
      int kb1 = kb0 + g.kb_per_split;
      if (kb1 > g.kb_total) kb1 = g.kb_total;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        const uint32_t fb = full0 + 8 * stage;
        mbar_arrive_expect_tx(fb, L::kStage);
        const uint32_t a_dst = smem_u32(sA + stage * L::kA);
        const uint32_t b_dst = smem_u32(sB + stage * L::kB);
        const int k0 = kb * kBK;
        if constexpr (A_MN) {
          tma_load_2d(a_dst, &tmA, fb, m0, k0);
          tma_load_2d(a_dst + 8192, &tmA, fb, m0 + 64, k0);
        } else {
          tma_load_2d(a_dst, &tmA, fb, k0, m0);
        }
        if constexpr (epi_is_swiglu(EPI)) {  // gate rows, then the matching value rows
          tma_load_2d(b_dst, &tmB, fb, k0, n0);
          tma_load_2d(b_dst + (BN / 2) * 128, &tmB, fb, k0, g.ff + n0);
        } else if constexpr (B_MN) {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * 8192, &tmB, fb, n0 + 64 * c, k0);
        } else {
          tma_load_2d(b_dst, &tmB, fb, k0, n0);
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
    bool ok = true;
    bool pending = false;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int split = t / tiles_mn;
      const int kb0 = split * g.kb_per_split;
      int kb1 = kb0 + g.kb_per_split;
      if (kb1 > g.kb_total) kb1 = g.kb_total;
      if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(full0 + 8 * stage, phase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        ++consumed;
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + stage * L::kA);
        const uint32_t b_base = smem_u32(sB + stage * L::kB);
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
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    *s_consumed = consumed;
    if (!ok && pending) {
      // Let every MMA already issued finish before tensor memory is released.
      umma_commit(drain);
      mbar_wait(drain, 0, g.status, RK_DEV_GEMM_TIMEOUT, nullptr);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int split = t / tiles_mn;
      const int mn = t - split * tiles_mn;
      const int m0 = (mn / g.tiles_n) * kBM;
      const int n0 = (mn % g.tiles_n) * NSTEP;
      bool ok = mbar_wait(tfull0 + 8 * acc, acc_phase, g.status, RK_DEV_GEMM_TIMEOUT, s_abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if constexpr (epi_is_swiglu(EPI)) {
        // h = round(silu(round(g))) * round(v) for the tile's 128 columns, 64 at a
        // time; the same operation order as rk_swiglu_fwd on a bf16 u.
        uint8_t* stage = sOut + (warp - 2) * (EPI == EPI_SWIGLU_SAVE ? 12288 : 8192);
        const int y = m0 + quarter * 32;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 64) {
          float gv[64], vv[64];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            float part[32];
            tmem_ld_32cols(t_row + c + q * 32, part);
#pragma unroll
            for (int j = 0; j < 32; ++j) gv[q * 32 + j] = round_to<TOut>(part[j]);
            tmem_ld_32cols(t_row + BN / 2 + c + q * 32, part);
#pragma unroll
            for (int j = 0; j < 32; ++j) vv[q * 32 + j] = round_to<TOut>(part[j]);
          }
          if constexpr (EPI == EPI_SWIGLU_SAVE) {
            if (lane == 0) bulk_wait_read<0>();
          } else {
            if (lane == 0) bulk_wait_read<1>();
          }
          __syncwarp();
          uint8_t* hb = EPI == EPI_SWIGLU_SAVE ? stage : stage + ((c / 64) & 1) * 4096;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 raw;
            TOut* e = reinterpret_cast<TOut*>(&raw);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float gg = gv[j * 8 + k];
              const float silu = round_to<TOut>(silu_value(gg));
              e[k] = Dt<TOut>::from_f(__fmul_rn(silu, vv[j * 8 + k]));
            }
            *reinterpret_cast<uint4*>(hb + lane * 128 + ((j ^ (lane & 7)) * 16)) = raw;
          }
          if constexpr (EPI == EPI_SWIGLU_SAVE) {
            uint8_t* gb = stage + 4096;
            uint8_t* vb = stage + 8192;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint4 rg, rv;
              TOut* eg = reinterpret_cast<TOut*>(&rg);
              TOut* ev = reinterpret_cast<TOut*>(&rv);
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                eg[k] = Dt<TOut>::from_f(gv[j * 8 + k]);
                ev[k] = Dt<TOut>::from_f(vv[j * 8 + k]);
              }
              const int off = lane * 128 + ((j ^ (lane & 7)) * 16);
              *reinterpret_cast<uint4*>(gb + off) = rg;
              *reinterpret_cast<uint4*>(vb + off) = rv;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, smem_u32(hb), n0 + c, y);
            if constexpr (EPI == EPI_SWIGLU_SAVE) {
              tma_store_2d(&tmD, smem_u32(stage + 4096), n0 + c, y);
              tma_store_2d(&tmD, smem_u32(stage + 8192), g.ff + n0 + c, y);
            }
            bulk_commit();
          }
        }
        tc_fence_before();
        mbar_arrive(tempty0 + 8 * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if constexpr (EPI == EPI_TMA || EPI == EPI_TMA_ADD) {
        // Each warp stages its 32 rows, CW columns at a time, in a 128-byte
        // swizzled layout (16-byte chunk j of row r at j ^ (r % 8): conflict-free
        // stores) and writes them with one TMA store per chunk; two buffers per
        // warp let the next chunk be staged while the previous store drains.
        constexpr int CW = 128 / (int)sizeof(TOut);
        constexpr int PER16 = 16 / (int)sizeof(TOut);
        uint8_t* stage = sOut + (warp - 2) * 8192;
#pragma unroll 1
        for (int c = 0; c < BN; c += CW) {
          float v[CW];
#pragma unroll
          for (int q = 0; q < CW / 32; ++q) {
            float part[32];
            tmem_ld_32cols(t_row + c + q * 32, part);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[q * 32 + j] = part[j];
          }
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
          uint8_t* buf = stage + ((c / CW) & 1) * 4096;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 raw;
            TOut* e = reinterpret_cast<TOut*>(&raw);
#pragma unroll
            for (int k = 0; k < PER16; ++k) e[k] = Dt<TOut>::from_f(v[j * PER16 + k]);
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) = raw;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int y = split * g.split_rows + m0 + quarter * 32;
            if constexpr (EPI == EPI_TMA_ADD) tma_reduce_add_2d(&tmC, smem_u32(buf), n0 + c, y);
            else tma_store_2d(&tmC, smem_u32(buf), n0 + c, y);
            bulk_commit();
          }
        }
        tc_fence_before();
        mbar_arrive(tempty0 + 8 * acc);
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
      for (int c = 0; c < BN; c += 32) {
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
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// dw[r, c] (+)= sum_s partial[s][r][c] (slices `slice_rows` rows apart), in
// slice order; 4 consecutive columns per thread when cols % 4 == 0.
template <int V>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ partial, int splits, int64_t rows,
                                                           int64_t cols, int64_t slice_rows, float* __restrict__ dw,
                                                           int64_t lddw, int accumulate) {
  pdl_wait();  // inputs are the previous kernel's outputs
  const int64_t n = rows * cols / V;
  const int64_t slice = slice_rows * cols;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t * V;
    float s[V];
#pragma unroll
    for (int e = 0; e < V; ++e) s[e] = 0.f;
    for (int k = 0; k < splits; ++k) {
      float v[V];
      load_vec<float, V>(partial + (int64_t)k * slice + i, v);
#pragma unroll
      for (int e = 0; e < V; ++e) s[e] += v[e];
    }
    const int64_t r = i / cols, c = i - r * cols;
    float* d = dw + r * lddw + c;
    if (accumulate) {
      float o[V];
      load_vec<float, V>(d, o);
#pragma unroll
      for (int e = 0; e < V; ++e) s[e] += o[e];
    }
    store_vec<float, V>(d, s);
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

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, typename TOut>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmArgs g, int dtype,
              cudaStream_t s, const CUtensorMap* td = nullptr) {
  using L = TcSmem<BN, STAGES, epi_out_bytes(EPI)>;
  auto kern = gemm_tc_kernel<BN, STAGES, A_MN, B_MN, EPI, TOut>;
  rk_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)L::kTotal);
  const int total = g.tiles_m * g.tiles_n * g.splits;
  int grid = sm_count();
  if (total < grid) grid = total;
  const uint32_t idesc = idesc_f16(kBM, BN, dtype == RK_BF16 ? 1 : 0, A_MN ? 1 : 0, B_MN ? 1 : 0);
  rk_host::launch_k(kern, grid, kThreads, L::kTotal, s, ta, tb, tc, td ? *td : tc, g, idesc);
  return rk_host::launch_status();
}

template <int BN, int EPI, typename TOut>
int dispatch_major(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, bool a_mn, bool b_mn,
                   const GemmArgs& g, int dtype, cudaStream_t s) {
  constexpr int ST = BN == 256 ? 4 : 6;
  if (!a_mn && !b_mn) return launch_tc<BN, ST, false, false, EPI, TOut>(ta, tb, tc, g, dtype, s);
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
            cudaStream_t s, bool accumulate = false, int split_rows = 0, int bn = 0) {
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
  GemmArgs g;
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

int wgrad_splits(int64_t M, int64_t N, int64_t K) {
  // Output tiles of dW[N,K] (128x128 when split: the fp32 slice traffic is
  // slices x N x K, and narrower tiles halve the slice count for the same
  // SM fill); choose slices so that tiles*slices fills ~the SMs, with each
  // slice at least 8 k-blocks (512 tokens) long. Fixed per shape.
  const int64_t tiles = ((N + 127) / 128) * ((K + 127) / 128);
  const int64_t kb = (M + 63) / 64;
  int64_t s = (148 + tiles - 1) / tiles;
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
                         splits, s, false, (int)slice_rows, 128);
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
    return launch_tc<256, 4, false, false, EPI_SWIGLU, __nv_bfloat16>(ta, tb, tc, g, dtype, s);
  }
  if (u) return launch_tc<256, 3, false, false, EPI_SWIGLU_SAVE, __half>(ta, tb, tc, g, dtype, s, &td);
  return launch_tc<256, 4, false, false, EPI_SWIGLU, __half>(ta, tb, tc, g, dtype, s);
}
