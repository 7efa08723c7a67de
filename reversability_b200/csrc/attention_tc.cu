// Causal attention forward on the 5th-generation tensor cores for head_dim 32
// and 64 (replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) at
// model.py:42-44: the 20.3M model's 8 x 32 heads and the scaled model's
// 16 x 64 heads).
//
// One CTA per (128-query tile, batch*head), walking the key tiles 0..qt:
//   warp 0      TMA producer: Q once, then K_j and V_j (64 keys x HD) into a
//               ring (3-D tensor map over [B][T][ldq], so rows past T read as
//               zeros); rows of HD = 32 use the 64-byte swizzle, rows of
//               HD = 64 the 128-byte one.
//   warp 1      tcgen05.mma issuer: S_j = Q K_j^T (M=128, N=64, K=HD) into a
//               TMEM accumulator; O += P_j V_j (M=128, N=HD, K=64) into the
//               TMEM O accumulator.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): one
//               TMEM read of S_j (64 columns; the buffer is released at
//               once), the row max (no shuffles), P_j = exp2(s*c - m_ref)
//               (bf16/f16) into a 128-byte-swizzled shared tile for the PV
//               MMA and its row sum. m_ref moves only when the row max rises
//               by more than 2^8 (lazy rescale); O is then rescaled in TMEM.
// S is double-buffered in TMEM (the MMA warp issues S_{j+1} before waiting
// for P_j), two CTAs share an SM (256 TMEM columns each) and hide each other's
// latencies. lse is written in base 2 (m_ref + log2(sum)), the
// layout the backward kernels read.
//
// Every mbarrier wait is bounded (RK_DEV_ATTN_TIMEOUT); on expiry the CTA
// stops issuing, drains its own MMAs and TMA loads and frees its TMEM.
#include <cudaTypedefs.h>
#include <cstdlib>
#include <mutex>
#include <type_traits>
#include "common.cuh"

namespace rk {
namespace attn_tc {

constexpr int kTile = 128;  // query rows per tile
constexpr int kKT = 64;     // keys per key tile
constexpr int kThreads = 192;
// Score buffers in TMEM and resident CTAs per SM. One buffer and three CTAs
// (twelve softmax warps per SM, 128 TMEM columns each, two K/V stages) measured
// 46.5 us against 26.9 us for two buffers and two CTAs at cfg2 (the softmax
// warps then spill).
constexpr int kSBufs = 2;
constexpr int kCtasPerSm = 2;
constexpr uint32_t kPBytes = kTile * kKT * 2;     // 16 KB (one 64-key swizzle atom)
constexpr uint32_t kNumBars = 26;
constexpr uint32_t kOCol = kSBufs * kKT;          // S [0, 64 * kSBufs), O [kOCol, kOCol + HD)
constexpr uint32_t kTmemCols = 256;               // power of two >= kOCol + HD

// Per head-dim layout. Shared memory: Q0 Q1 | K ring | V ring | P buffers | barriers.
// The K/V ring must run ahead of the MMA warp: K/V tile j + kKVStages is
// loaded once PV_j has completed, at the end of the softmax of tile j, and S
// of that tile is issued at the end of the softmax of tile j + kKVStages - 2.
// HD = 64 holds three K/V stages and one P buffer (the softmax of tile j+1
// writes P after PV_j completes, which it has by then) so that two CTAs still
// share an SM; with two stages the softmax warps waited about 1,100 cycles
// per tile for S (44% of their time at the scaled model's shape).
template <int HD>
struct Fwd {
  static_assert(HD == 32 || HD == 64, "head_dim 32 or 64");
  static constexpr int kKVStages = HD == 32 ? 4 : 3;
  static constexpr int kPBufs = HD == 32 ? 2 : 1;
  static constexpr uint32_t kRow = HD * 2;              // bytes per row: the swizzle span
  static constexpr uint32_t kSwz = HD == 32 ? 4 : 2;    // descriptor layout: 64- / 128-byte swizzle
  static constexpr uint32_t kSbo = 8 * kRow;            // bytes between 8-row groups
  static constexpr uint32_t kVLbo = HD == 32 ? 4096 : 8192;  // V (MN-major): N-chunk stride (one chunk)
  static constexpr uint32_t kQBytes = kTile * HD * 2;   // 8 / 16 KB
  static constexpr uint32_t kKVBytes = kKT * HD * 2;    // 4 / 8 KB each for K and V
  static constexpr uint32_t kOffK = 2 * kQBytes;
  static constexpr uint32_t kOffV = kOffK + kKVStages * kKVBytes;
  static constexpr uint32_t kOffP = kOffV + kKVStages * kKVBytes;
  static constexpr uint32_t kOffBar = kOffP + kPBufs * kPBytes;
  static constexpr uint32_t kSmem = 1024 + kOffBar + kNumBars * 8 + 32;
  static_assert(kKVStages <= 4 && kOCol + HD <= kTmemCols, "barrier slots and TMEM columns");
  static_assert(2 * (kSmem + 1024) <= 233472, "two CTAs per SM");
};
// Lazy rescale: P is formed against a reference max that only moves when a
// row's max exceeds it by more than 2^8, so P <= 256 (exact in bf16's range)
// and the O accumulator in TMEM is rescaled rarely.
constexpr float kRescaleLog2 = 8.f;

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// UMMA shared-memory descriptor: address, LBO, SBO (bytes), layout type
// (2 = 128-byte swizzle, 4 = 64-byte swizzle), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t d;
  if constexpr (std::is_same_v<T, __nv_bfloat16>) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

struct Bars {
  uint32_t q_full0, q_empty0, kv_full0, kv_empty0, s_full0, s_empty0, p_full0, p_empty0, o_full0, o_empty0, drain;
};

// P rounded to 16 bits and packed two per word. bf16: round to nearest (ties
// away) by an integer add on the ALU (p is in [0, 1], so no overflow), leaving
// the exponential unit to ex2.
template <typename T>
__device__ __forceinline__ uint32_t pack_p(float p0, float p1) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    return __byte_perm(__float_as_uint(p0) + 0x8000u, __float_as_uint(p1) + 0x8000u, 0x7632);
  } else {
    return pack2<T>(p0, p1);
  }
}

// 32 lanes x 32 consecutive 32-bit columns, thread i -> lane (base + i).
__device__ __forceinline__ void tmem_st_32cols(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Persistent: grid = min(kCtasPerSm x SMs, items); item i (longest query tiles first)
// is (qt, bh) = (ntq - 1 - i / BH, i % BH); query tile qt meets key tiles
// 0 .. 2*qt+1 (64 keys each). All roles walk the same item sequence and keep
// running tile counters for the barrier phases: K/V tile g uses ring stage
// g % kKVStages; S tile t uses buffer t % kSBufs, P tile t buffer t % 2.
template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, T* __restrict__ out, float* __restrict__ lse, int H,
                  int BH, int ntq, int Tlen, int64_t ldo, float c_log2, unsigned int* status) {
  using C = Fwd<HD>;
  constexpr int kKVStages = C::kKVStages;
  constexpr uint32_t kQBytes = C::kQBytes, kKVBytes = C::kKVBytes;
  constexpr uint32_t kOffK = C::kOffK, kOffV = C::kOffV, kOffP = C::kOffP, kOffBar = C::kOffBar;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kOffBar;
  Bars bb;
  bb.q_full0 = bar0;          // 2
  bb.q_empty0 = bar0 + 16;    // 2
  bb.kv_full0 = bar0 + 32;    // kKVStages
  bb.kv_empty0 = bar0 + 64;   // kKVStages
  bb.s_full0 = bar0 + 96;     // 2
  bb.s_empty0 = bar0 + 112;   // 2
  bb.p_full0 = bar0 + 128;    // 2
  bb.p_empty0 = bar0 + 144;   // 2
  bb.o_full0 = bar0 + 160;    // 2
  bb.o_empty0 = bar0 + 176;   // 2
  bb.drain = bar0 + 192;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kOffBar + kNumBars * 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(s_tmem + 2);
  volatile int* s_qconsumed = reinterpret_cast<volatile int*>(s_tmem + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = H * HD;
  const int items = ntq * BH;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bb.q_full0 + 8 * i, 1);
      mbar_init(bb.q_empty0 + 8 * i, 1);
    }
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(bb.kv_full0 + 8 * i, 1);
      mbar_init(bb.kv_empty0 + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bb.s_full0 + 8 * i, 1);
      mbar_init(bb.s_empty0 + 8 * i, 4);
      mbar_init(bb.p_full0 + 8 * i, 4);
      mbar_init(bb.p_empty0 + 8 * i, 1);
      mbar_init(bb.o_full0 + 8 * i, 1);
      mbar_init(bb.o_empty0 + 8 * i, 4);
    }
    mbar_init(bb.drain, 1);
    fence_mbar_init();
    *s_abort = 0;
    *s_consumed = 0;
    *s_qconsumed = 0;
    tma_prefetch_desc(&tm);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  int issued = 0;   // producer: K/V tiles loaded
  int qissued = 0;  // producer: Q tiles loaded

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int g = 0;
      bool ok = true;
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int qt = ntq - 1 - it / BH, bh = it - (it / BH) * BH;
        const int b = bh / H, h = bh - (bh / H) * H;
        const int qb = n & 1;
        if (n >= 2 && !mbar_wait(bb.q_empty0 + 8 * qb, ((n - 2) >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort))
          break;
        const uint32_t qf = bb.q_full0 + 8 * qb;
        mbar_arrive_expect_tx(qf, kQBytes);
        tma_load_3d(sbase + qb * kQBytes, &tm, qf, h * HD, qt * kTile, b);
        tma_load_3d(sbase + qb * kQBytes + kQBytes / 2, &tm, qf, h * HD, qt * kTile + kKT, b);
        ++qissued;
        const int nk = 2 * qt + 2;
        for (int j = 0; j < nk; ++j, ++g) {
          const int st = g % kKVStages;
          if (g >= kKVStages &&
              !mbar_wait(bb.kv_empty0 + 8 * st, ((g / kKVStages) - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          const uint32_t fb = bb.kv_full0 + 8 * st;
          mbar_arrive_expect_tx(fb, 2 * kKVBytes);
          tma_load_3d(sbase + kOffK + st * kKVBytes, &tm, fb, D + h * HD, j * kKT, b);
          tma_load_3d(sbase + kOffV + st * kKVBytes, &tm, fb, 2 * D + h * HD, j * kKT, b);
          ++issued;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idS = idesc_f16(kTile, kKT, std::is_same_v<T, __nv_bfloat16> ? 1 : 0, 0, 0);
      constexpr uint32_t idPV = idesc_f16(kTile, HD, std::is_same_v<T, __nv_bfloat16> ? 1 : 0, 0, 1);
      bool ok = true, pending = false;
      int g = 0;   // K/V tiles consumed
      int gs = 0;  // S tiles issued
      int gp = 0;  // PV tiles issued
      int qc = 0;
      uint32_t qa = sbase;  // Q buffer of the current item
      auto issue_s = [&]() -> bool {
        const int st = g % kKVStages;
        if (!mbar_wait(bb.kv_full0 + 8 * st, (g / kKVStages) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) return false;
        ++g;
        const int sb = gs % kSBufs;
        if (gs >= kSBufs &&
            !mbar_wait(bb.s_empty0 + 8 * sb, ((gs - kSBufs) / kSBufs) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort))
          return false;
        tc_fence_after();
        const uint32_t ka = sbase + kOffK + st * kKVBytes;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + sb * kKT, smem_desc(qa + kk * 32, 16, C::kSbo, C::kSwz),
                   smem_desc(ka + kk * 32, 16, C::kSbo, C::kSwz), idS, kk > 0 ? 1u : 0u);
        umma_commit(bb.s_full0 + 8 * sb);
        ++gs;
        pending = true;
        return true;
      };
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int qt = ntq - 1 - it / BH;
        const int nk = 2 * qt + 2;
        const int qb = n & 1;
        if (!mbar_wait(bb.q_full0 + 8 * qb, (n >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        ++qc;
        qa = sbase + qb * kQBytes;
        int st_j = g % kKVStages;  // ring stage of key tile j
        if (!issue_s()) {
          ok = false;
          break;
        }
        for (int j = 0; j < nk; ++j) {
          const int st_next = g % kKVStages;
          if (j + 1 < nk) {
            if (!issue_s()) {
              ok = false;
              break;
            }
          } else {
            umma_commit(bb.q_empty0 + 8 * qb);  // every S of this item issued: its Q buffer may be refilled
          }
          const int pb = gp % C::kPBufs;
          if (!mbar_wait(bb.p_full0 + 8 * pb, (gp / C::kPBufs) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = sbase + kOffP + pb * kPBytes;
          const uint32_t va = sbase + kOffV + st_j * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kKT / 16; ++kk)
            umma_f16(tmem + kOCol, smem_desc(pa + kk * 32, 16, 1024, 2),
                     smem_desc(va + kk * 16 * C::kRow, C::kVLbo, C::kSbo, C::kSwz), idPV, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(bb.o_full0);
          umma_commit(bb.kv_empty0 + 8 * st_j);
          umma_commit(bb.p_empty0 + 8 * pb);
          ++gp;
          st_j = st_next;
        }
      }
      *s_consumed = g;
      *s_qconsumed = qc;
      if (!ok && pending) {
        umma_commit(bb.drain);
        mbar_wait(bb.drain, 0, status, RK_DEV_ATTN_TIMEOUT, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    int gs = 0, gp = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int qt = ntq - 1 - it / BH, bh = it - (it / BH) * BH;
      const int b = bh / H, h = bh - (bh / H) * H;
      const int grow = qt * kTile + row;
      const int nk = 2 * qt + 2;
      float m_ref = -INFINITY, l_run = 0.f;
      // wait until PV tile number `gidx` has completed (callers make sure no
      // earlier PV tile is still outstanding)
      auto wait_pv = [&](int gidx) -> bool {
        bool w = mbar_wait(bb.o_full0, gidx & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        w = __all_sync(0xffffffffu, w);
        if (w) tc_fence_after();
        return w;
      };
      for (int j = 0; j < nk; ++j) {
        const int sb = gs % kSBufs;
        bool w = mbar_wait(bb.s_full0 + 8 * sb, (gs / kSBufs) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        w = __all_sync(0xffffffffu, w);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int lim = grow - j * kKT;  // keys k of this tile with k <= lim are visible
        const bool diag = lim < kKT - 1;
        uint32_t ra[32], rb[32];
        tmem_ld_32cols_nowait(t_lane + sb * kKT, ra);
        tmem_ld_32cols_nowait(t_lane + sb * kKT + 32, rb);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bb.s_empty0 + 8 * sb);  // S is in registers: the buffer is free
        // diagonal tile: masked scores become -inf (their exp is 0)
        if (diag) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (k > lim) ra[k] = __float_as_uint(-INFINITY);
            if (32 + k > lim) rb[k] = __float_as_uint(-INFINITY);
          }
        }
        // tile row max: three-input max, four partial chains
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          mx4[(k >> 1) & 3] = fmax3(mx4[(k >> 1) & 3], __uint_as_float(ra[k]), __uint_as_float(ra[k + 1]));
          mx4[((k >> 1) + 2) & 3] = fmax3(mx4[((k >> 1) + 2) & 3], __uint_as_float(rb[k]), __uint_as_float(rb[k + 1]));
        }
        const float mt = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]) * c_log2;
        // P buffer free (PV tile gp - kPBufs done), and at most one PV (gp-1)
        // outstanding, so the o_full parity wait below is unambiguous. With two
        // buffers the S_gp just read implies it: the MMA warp committed S_gp
        // after issuing PV_{gp-2}, and a commit tracks every earlier MMA of
        // the issuing thread. One buffer needs PV_{gp-1}: wait for it.
        constexpr int kPB = C::kPBufs;
        const int pb = gp % kPB;
        if (kPB == 1 && gp >= 1) {
          w = mbar_wait(bb.p_empty0 + 8 * pb, ((gp - kPB) / kPB) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
          w = __all_sync(0xffffffffu, w);
          if (!w) {
            ok = false;
            break;
          }
        }
        // move the reference max (first tile, or a rise beyond the threshold);
        // the warp rescales O together because TMEM access is warp-wide
        const bool raise = m_ref == -INFINITY ? mt != -INFINITY : mt > m_ref + kRescaleLog2;
        if (__any_sync(0xffffffffu, raise)) {
          const float m_new = raise ? mt : m_ref;
          const float f = (m_ref == -INFINITY || !raise) ? 1.f : ex2f(m_ref - m_new);
          if (j > 0) {
            if (!wait_pv(gp - 1)) {
              ok = false;
              break;
            }
#pragma unroll
            for (int oc = 0; oc < HD; oc += 32) {
              uint32_t o[32];
              tmem_ld_32cols_nowait(t_lane + kOCol + oc, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
              tmem_st_32cols(t_lane + kOCol + oc, o);
            }
            tmem_st_wait();
          }
          l_run *= f;
          m_ref = m_new;
        }
        const float nm = m_ref == -INFINITY ? 0.f : -m_ref;
        // P = exp2(s*c - m_ref) into the swizzled P tile, and the row sum
        // (packed two-lane fp32 arithmetic for the scale and the sum)
        uint8_t* prow = smem + kOffP + pb * kPBytes + row * 128;
        const float2 c2 = make_float2(c_log2, c_log2), n2 = make_float2(nm, nm);
        float2 ls2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t* r = c ? rb : ra;
          uint32_t pw[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 t = __ffma2_rn(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), c2, n2);
            const float2 pp = make_float2(ex2f(t.x), ex2f(t.y));
            ls2[k & 1] = __fadd2_rn(ls2[k & 1], pp);
            pw[k] = pack_p<T>(pp.x, pp.y);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int lc = c * 4 + q;  // logical 16-byte chunk of the 128-byte row
            *reinterpret_cast<uint4*>(prow + ((lc ^ (row & 7)) * 16)) =
                make_uint4(pw[4 * q], pw[4 * q + 1], pw[4 * q + 2], pw[4 * q + 3]);
          }
        }
        l_run += (ls2[0].x + ls2[0].y) + (ls2[1].x + ls2[1].y);
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bb.p_full0 + 8 * pb);
        ++gs;
        ++gp;
      }
      // all of this item's PV tiles complete: with two P buffers first gp-2
      // through its P buffer barrier (at most one use outstanding there),
      // then gp-1 through o_full
      if (ok && C::kPBufs == 2 && gp >= 2) {
        bool w = mbar_wait(bb.p_empty0 + 8 * (gp & 1), ((gp - 2) >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        ok = __all_sync(0xffffffffu, w);
      }
      if (!ok || !wait_pv(gp - 1)) {
        ok = false;
        break;
      }
      {
        uint32_t o[HD];
#pragma unroll
        for (int oc = 0; oc < HD; oc += 32) tmem_ld_32cols_nowait(t_lane + kOCol + oc, o + oc);
        tmem_ld_wait();
        if (grow < Tlen) {
          const float inv = 1.f / l_run;
          T* orow = out + ((int64_t)b * Tlen + grow) * ldo + h * HD;
#pragma unroll
          for (int q = 0; q < HD / 8; ++q) {
            const float* oq = reinterpret_cast<const float*>(o + 8 * q);
            reinterpret_cast<uint4*>(orow)[q] =
                make_uint4(pack2<T>(oq[0] * inv, oq[1] * inv), pack2<T>(oq[2] * inv, oq[3] * inv),
                           pack2<T>(oq[4] * inv, oq[5] * inv), pack2<T>(oq[6] * inv, oq[7] * inv));
          }
          lse[(int64_t)bh * Tlen + grow] = m_ref + __log2f(l_run);
        }
      }
    }
  }

  __syncthreads();
  if (*s_abort && threadIdx.x == 0) {
    // wait (bounded) for the TMA loads of this CTA that no MMA consumed
    for (int i = *s_qconsumed; i < qissued; ++i)
      mbar_wait(bb.q_full0 + 8 * (i & 1), (i >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
    for (int i = *s_consumed; i < issued; ++i)
      mbar_wait(bb.kv_full0 + 8 * (i % kKVStages), (i / kKVStages) & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}


// ------------------------------------------------------------------ backward
// dQ and dK/dV of the causal attention on the tensor cores, deterministic (no
// atomics: dQ per query tile, dK/dV per key tile), with the conventions of the
// forward: P = exp2(s * c - lse) with the base-2 lse it wrote, D = rowsum(dO * O)
// precomputed, dS = P * (dP - D) rounded to 16 bits for the MMA, dQ and dK
// scaled by 1/sqrt(HD) in fp32 at the end.
//
// dQ kernel, one item per (128-query tile, batch*head), key tiles of 64:
//   warp 0      TMA: Q and dO once per item, K_j / V_j into a ring
//   warp 1      tcgen05.mma: S = Q K_j^T and dP = dO V_j^T (M=128, N=64,
//               K=HD) into TMEM; dQ += dS_j K_j (M=128, N=HD, K=64)
//   warps 2..5  one query row per thread: P, dS from the S / dP rows, dS
//               written to a 128-byte-swizzled shared tile; dQ read from TMEM
//               at the end of the item, scaled and stored
// dK/dV kernel, one item per (128-key tile, batch*head), query tiles of 64:
//   warp 0      TMA: K and V once per item, Q_t / dO_t into a ring
//   warp 1      tcgen05.mma: S^T = K Q_t^T and dP^T = V dO_t^T into TMEM;
//               dV += P^T dO_t and dK += dS^T Q_t (M=128, N=HD, K=64)
//   warps 2..5  one key row per thread: P^T and dS^T rows (lse and D of the
//               tile's 64 queries staged per warp in shared memory)
// S and dP are single-buffered in TMEM (two CTAs share an SM); the MMA warp
// issues tile j+1's S / dP as soon as the compute warps have read tile j's,
// before tile j's accumulating MMA, so both overlap the compute.
template <int HD>
struct Bwd {
  using F = Fwd<HD>;
  static constexpr uint32_t kRow = F::kRow, kSwz = F::kSwz, kSbo = F::kSbo, kVLbo = F::kVLbo;
  static constexpr uint32_t kTile128 = 128 * HD * 2;  // 128 rows x HD
  static constexpr uint32_t kTile64 = 64 * HD * 2;    // 64 rows x HD
  // dQ kernel smem: Q (kQBufs) | dO (kQBufs) | K ring | V ring | dS (kDSBufs) | barriers.
  // As in the forward, the K/V ring has to run a tile ahead of the MMA warp
  // (tile j + kKVStages loads once the dQ MMA of tile j completes): HD = 64
  // holds three stages and one dS buffer (the dS of tile j+1 is written
  // after the dQ MMA of tile j completes, which it has by then).
  static constexpr int kQBufs = HD == 32 ? 2 : 1;
  static constexpr int kKVStages = HD == 32 ? 4 : 3;
  static constexpr int kDSBufs = HD == 32 ? 2 : 1;
  static constexpr uint32_t kQ_OffDO = kQBufs * kTile128;
  static constexpr uint32_t kQ_OffK = 2 * kQBufs * kTile128;
  static constexpr uint32_t kQ_OffV = kQ_OffK + kKVStages * kTile64;
  static constexpr uint32_t kQ_OffS = kQ_OffV + kKVStages * kTile64;
  static constexpr uint32_t kQ_OffBar = kQ_OffS + kDSBufs * kPBytes;
  static constexpr uint32_t kQ_Smem = 1024 + kQ_OffBar + 32 * 8 + 32;
  // dK/dV kernel smem: K | V | Q ring | dO ring | P^T (kPBufs) | dS^T (kPBufs) |
  // per-warp lse/D (8 warps x 2 x 32 floats) | barriers
  static constexpr int kQStages = 2;
  static constexpr int kPBufs = HD == 32 ? 2 : 1;
  static constexpr uint32_t kK_OffV = kTile128;
  static constexpr uint32_t kK_OffQ = 2 * kTile128;
  static constexpr uint32_t kK_OffDO = kK_OffQ + kQStages * kTile64;
  static constexpr uint32_t kK_OffP = kK_OffDO + kQStages * kTile64;
  static constexpr uint32_t kK_OffDS = kK_OffP + kPBufs * kPBytes;
  static constexpr uint32_t kK_OffL = kK_OffDS + kPBufs * kPBytes;
  static constexpr uint32_t kK_OffBar = kK_OffL + 8 * 64 * 4;
  static constexpr uint32_t kK_Smem = 1024 + kK_OffBar + 32 * 8 + 32;
  // TMEM columns: S [0, 64), dP [64, 128), then dQ (HD) or dV, dK (HD each)
  static constexpr uint32_t kColS = 0, kColDP = 64, kColAcc = 128;
  static_assert(kColAcc + 2 * HD <= kTmemCols, "TMEM columns");
  static_assert(2 * (kQ_Smem + 1024) <= 233472 && 2 * (kK_Smem + 1024) <= 233472, "two CTAs per SM");
};

// P and dS for NC columns c0 .. c0+NC-1 of one row, two columns per step in
// packed fp32x2 arithmetic: p = exp2(s * c_log2 - lse), ds = p * (dp - D),
// with the negated lse / D of each column pair from `nl` / `nd` (COLS: shared
// memory, indexed by column) or the row's own values (nl_r, nd_r). MASK
// applies `valid(c)` (p = 0 where it fails); a warp whose columns are all
// visible skips it. Writes NC/2 packed P words (if pw) and NC/2 packed dS words.
template <typename T, int NC, bool COLS, bool MASK, typename Valid>
__device__ __forceinline__ void bwd_cols(const uint32_t* s, const uint32_t* dp, int c0, float c_log2,
                                         const float* nl, const float* nd, float nl_r, float nd_r, Valid valid,
                                         uint32_t* pw, uint32_t* dw) {
  const float2 c2 = make_float2(c_log2, c_log2);
#pragma unroll
  for (int k = 0; k < NC / 2; ++k) {
    const int c = c0 + 2 * k;
    const float2 l2 = COLS ? *reinterpret_cast<const float2*>(nl + c) : make_float2(nl_r, nl_r);
    const float2 d2 = COLS ? *reinterpret_cast<const float2*>(nd + c) : make_float2(nd_r, nd_r);
    const float2 t = __ffma2_rn(make_float2(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])), c2, l2);
    float2 pv = make_float2(ex2f(t.x), ex2f(t.y));
    if constexpr (MASK) {
      if (!valid(c)) pv.x = 0.f;
      if (!valid(c + 1)) pv.y = 0.f;
    }
    const float2 ds =
        __fmul2_rn(pv, __fadd2_rn(make_float2(__uint_as_float(dp[2 * k]), __uint_as_float(dp[2 * k + 1])), d2));
    if (pw) pw[k] = pack_p<T>(pv.x, pv.y);
    dw[k] = pack2<T>(ds.x, ds.y);
  }
}

// Backward kernels: producer warp, MMA warp and eight compute warps, two per
// TMEM lane quarter (warp w: quarter w % 4, column half (w - 2) / 4).
constexpr int kThreadsBwd = 64 + 8 * 32;

// 32 lanes x 16 consecutive 32-bit columns (no wait).
__device__ __forceinline__ void tmem_ld_16cols_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// `n` TMEM columns (16 or 32) of this thread's lane.
template <int n>
__device__ __forceinline__ void tmem_ld_cols_nowait(uint32_t taddr, uint32_t* r) {
  static_assert(n == 16 || n == 32, "16 or 32 columns");
  if constexpr (n == 16) tmem_ld_16cols_nowait(taddr, r);
  else tmem_ld_32cols_nowait(taddr, r);
}

// `nq` 16-byte chunks (8 columns each), starting at chunk q0, of a 64-column
// 16-bit row of a 128-byte-swizzled tile.
template <int nq>
__device__ __forceinline__ void store_chunks128(uint8_t* tile, int row, int q0, const uint32_t* w) {
  uint8_t* prow = tile + row * 128;
#pragma unroll
  for (int q = 0; q < nq; ++q)
    *reinterpret_cast<uint4*>(prow + (((q0 + q) ^ (row & 7)) * 16)) =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// HD fp32 TMEM columns of this thread's lane, scaled, stored as T to `dst`.
template <typename T, int HD>
__device__ __forceinline__ void store_acc_row(T* dst, const uint32_t* a, float scale) {
#pragma unroll
  for (int q = 0; q < HD / 8; ++q) {
    const float* v = reinterpret_cast<const float*>(a + 8 * q);
    reinterpret_cast<uint4*>(dst)[q] = make_uint4(pack2<T>(v[0] * scale, v[1] * scale), pack2<T>(v[2] * scale, v[3] * scale),
                                                  pack2<T>(v[4] * scale, v[5] * scale), pack2<T>(v[6] * scale, v[7] * scale));
  }
}

// dQ: items (qt, bh) longest first, as in the forward; key tiles 0 .. 2*qt+1.
template <typename T, int HD>
__global__ void __launch_bounds__(kThreadsBwd, kCtasPerSm)
    bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo,
                     const float* __restrict__ lse, const float* __restrict__ dsum, T* __restrict__ dqkv,
                     int64_t lddq, int H, int BH, int ntq, int Tlen, float c_log2, float scale,
                     unsigned int* status) {
  using C = Bwd<HD>;
  constexpr int kQB = C::kQBufs, kST = C::kKVStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::kQ_OffBar;
  const uint32_t q_full0 = bar0, q_empty0 = bar0 + 16;      // [kQB]
  const uint32_t kv_full0 = bar0 + 32, kv_empty0 = bar0 + 64;  // [kST]
  const uint32_t s_full = bar0 + 96, s_empty = bar0 + 104;
  const uint32_t p_full0 = bar0 + 112, p_empty0 = bar0 + 128;  // [2]
  const uint32_t acc_full = bar0 + 144, acc_empty = bar0 + 152, drain = bar0 + 160;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kQ_OffBar + 32 * 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(s_tmem + 2);
  volatile int* s_qconsumed = reinterpret_cast<volatile int*>(s_tmem + 3);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = H * HD;
  const int items = ntq * BH;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kQB; ++i) {
      mbar_init(q_full0 + 8 * i, 1);
      mbar_init(q_empty0 + 8 * i, 1);
    }
    for (int i = 0; i < kST; ++i) {
      mbar_init(kv_full0 + 8 * i, 1);
      mbar_init(kv_empty0 + 8 * i, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(p_full0 + 8 * i, 8);
      mbar_init(p_empty0 + 8 * i, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(drain, 1);
    fence_mbar_init();
    *s_abort = 0;
    *s_consumed = 0;
    *s_qconsumed = 0;
    tma_prefetch_desc(&tm);
    tma_prefetch_desc(&tmo);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  int issued = 0, qissued = 0;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int g = 0;
      bool ok = true;
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int qt = ntq - 1 - it / BH, bh = it - (it / BH) * BH;
        const int b = bh / H, h = bh - (bh / H) * H;
        const int qb = n % kQB;
        if (n >= kQB && !mbar_wait(q_empty0 + 8 * qb, ((n - kQB) / kQB) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort))
          break;
        const uint32_t qf = q_full0 + 8 * qb;
        mbar_arrive_expect_tx(qf, 2 * C::kTile128);
        const uint32_t qa = sbase + qb * C::kTile128, da = sbase + C::kQ_OffDO + qb * C::kTile128;
        tma_load_3d(qa, &tm, qf, h * HD, qt * kTile, b);
        tma_load_3d(qa + C::kTile64, &tm, qf, h * HD, qt * kTile + kKT, b);
        tma_load_3d(da, &tmo, qf, h * HD, qt * kTile, b);
        tma_load_3d(da + C::kTile64, &tmo, qf, h * HD, qt * kTile + kKT, b);
        ++qissued;
        const int nk = 2 * qt + 2;
        for (int j = 0; j < nk; ++j, ++g) {
          const int st = g % kST;
          if (g >= kST && !mbar_wait(kv_empty0 + 8 * st, ((g / kST) - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          const uint32_t fb = kv_full0 + 8 * st;
          mbar_arrive_expect_tx(fb, 2 * C::kTile64);
          tma_load_3d(sbase + C::kQ_OffK + st * C::kTile64, &tm, fb, D + h * HD, j * kKT, b);
          tma_load_3d(sbase + C::kQ_OffV + st * C::kTile64, &tm, fb, 2 * D + h * HD, j * kKT, b);
          ++issued;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr int fmt = std::is_same_v<T, __nv_bfloat16> ? 1 : 0;
      constexpr uint32_t idS = idesc_f16(kTile, kKT, fmt, 0, 0);
      constexpr uint32_t idA = idesc_f16(kTile, HD, fmt, 0, 1);
      bool ok = true, pending = false;
      int g = 0, gs = 0, gp = 0, qc = 0;
      uint32_t qa = sbase, da = sbase + C::kQ_OffDO;
      auto issue_s = [&]() -> bool {
        const int st = g % kST;
        if (!mbar_wait(kv_full0 + 8 * st, (g / kST) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) return false;
        ++g;
        if (gs >= 1 && !mbar_wait(s_empty, (gs - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) return false;
        tc_fence_after();
        const uint32_t ka = sbase + C::kQ_OffK + st * C::kTile64, va = sbase + C::kQ_OffV + st * C::kTile64;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + C::kColS, smem_desc(qa + kk * 32, 16, C::kSbo, C::kSwz),
                   smem_desc(ka + kk * 32, 16, C::kSbo, C::kSwz), idS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + C::kColDP, smem_desc(da + kk * 32, 16, C::kSbo, C::kSwz),
                   smem_desc(va + kk * 32, 16, C::kSbo, C::kSwz), idS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        ++gs;
        pending = true;
        return true;
      };
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int qt = ntq - 1 - it / BH;
        const int nk = 2 * qt + 2;
        const int qb = n % kQB;
        if (!mbar_wait(q_full0 + 8 * qb, (n / kQB) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        ++qc;
        qa = sbase + qb * C::kTile128;
        da = sbase + C::kQ_OffDO + qb * C::kTile128;
        int st_j = g % kST;
        if (!issue_s()) {
          ok = false;
          break;
        }
        for (int j = 0; j < nk; ++j) {
          const int st_next = g % kST;
          if (j + 1 < nk) {
            if (!issue_s()) {
              ok = false;
              break;
            }
          } else {
            umma_commit(q_empty0 + 8 * qb);  // every MMA reading Q / dO of this item issued
          }
          const int pb = gp % C::kDSBufs;
          if (!mbar_wait(p_full0 + 8 * pb, (gp / C::kDSBufs) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          if (j == 0 && n > 0 && !mbar_wait(acc_empty, (n - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;  // the previous item's dQ has been read out of TMEM
            break;
          }
          tc_fence_after();
          const uint32_t dsa = sbase + C::kQ_OffS + pb * kPBytes;
          const uint32_t ka = sbase + C::kQ_OffK + st_j * C::kTile64;
#pragma unroll
          for (int kk = 0; kk < kKT / 16; ++kk)
            umma_f16(tmem + C::kColAcc, smem_desc(dsa + kk * 32, 16, 1024, 2),
                     smem_desc(ka + kk * 16 * C::kRow, C::kVLbo, C::kSbo, C::kSwz), idA, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(kv_empty0 + 8 * st_j);
          umma_commit(p_empty0 + 8 * pb);
          ++gp;
          st_j = st_next;
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
      *s_consumed = g;
      *s_qconsumed = qc;
      if (!ok && pending) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, RK_DEV_ATTN_TIMEOUT, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ dS rows
    // warp w: lane quarter w % 4 (one query row per thread), column half
    // ch = (w - 2) / 4 of the key tile and of dQ's HD columns
    const int quarter = warp & 3, ch = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    int gs = 0, gp = 0;
    bool ok = true;
    for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
      const int qt = ntq - 1 - it / BH, bh = it - (it / BH) * BH;
      const int b = bh / H, h = bh - (bh / H) * H;
      const int grow = qt * kTile + row;
      const int nk = 2 * qt + 2;
      const bool vrow = grow < Tlen;
      const float lse_r = vrow ? lse[(int64_t)bh * Tlen + grow] : INFINITY;  // rows past T: P = 0
      const float d_r = vrow ? dsum[(int64_t)bh * Tlen + grow] : 0.f;
      for (int j = 0; j < nk; ++j) {
        bool w = mbar_wait(s_full, gs & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        w = __all_sync(0xffffffffu, w);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int lim = grow - j * kKT;  // keys c of this tile with c <= lim are visible
        auto valid = [lim](int c) { return c <= lim; };
        uint32_t dw[16];
        {
          uint32_t sv[32], dv[32];
          tmem_ld_32cols_nowait(t_lane + C::kColS + 32 * ch, sv);
          tmem_ld_32cols_nowait(t_lane + C::kColDP + 32 * ch, dv);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(s_empty);  // this warp's S and dP columns are in registers
          if (__all_sync(0xffffffffu, lim >= kKT - 1))  // every key of the tile visible to the warp's rows
            bwd_cols<T, 32, false, false>(sv, dv, 32 * ch, c_log2, nullptr, nullptr, -lse_r, -d_r, valid, nullptr, dw);
          else
            bwd_cols<T, 32, false, true>(sv, dv, 32 * ch, c_log2, nullptr, nullptr, -lse_r, -d_r, valid, nullptr, dw);
        }
        constexpr int kDS = C::kDSBufs;
        const int pb = gp % kDS;
        // the dQ MMA of tile gp - kDS has read this dS buffer: implied for two
        // buffers by S_gp (committed after the dQ MMA of tile gp - 2 was
        // issued), waited for with one
        if (kDS == 1 && gp >= 1) {
          w = mbar_wait(p_empty0 + 8 * pb, ((gp - kDS) / kDS) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
          w = __all_sync(0xffffffffu, w);
          if (!w) {
            ok = false;
            break;
          }
        }
        store_chunks128<4>(smem + C::kQ_OffS + pb * kPBytes, row, 4 * ch, dw);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full0 + 8 * pb);
        ++gs;
        ++gp;
      }
      if (!ok) break;
      bool w = mbar_wait(acc_full, n & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
      w = __all_sync(0xffffffffu, w);
      if (!w) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t acc[HD / 2];
      tmem_ld_cols_nowait<HD / 2>(t_lane + C::kColAcc + ch * (HD / 2), acc);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (vrow) store_acc_row<T, HD / 2>(dqkv + ((int64_t)b * Tlen + grow) * lddq + h * HD + ch * (HD / 2), acc, scale);
    }
  }

  __syncthreads();
  if (*s_abort && threadIdx.x == 0) {
    for (int i = *s_qconsumed; i < qissued; ++i)
      mbar_wait(q_full0 + 8 * (i % kQB), (i / kQB) & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
    for (int i = *s_consumed; i < issued; ++i)
      mbar_wait(kv_full0 + 8 * (i % kST), (i / kST) & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// dK/dV: items (kt, bh) with the small key tiles (most query tiles) first;
// query tiles of 64 from 2*kt to the last one.
template <typename T, int HD>
__global__ void __launch_bounds__(kThreadsBwd, kCtasPerSm)
    bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo,
                      const float* __restrict__ lse, const float* __restrict__ dsum, T* __restrict__ dqkv,
                      int64_t lddq, int H, int BH, int ntk, int nq, int Tlen, float c_log2, float scale,
                      unsigned int* status) {
  using C = Bwd<HD>;
  constexpr int kQS = C::kQStages, kPB = C::kPBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::kK_OffBar;
  const uint32_t kv_full = bar0, kv_empty = bar0 + 8;
  const uint32_t q_full0 = bar0 + 16, q_empty0 = bar0 + 32;  // [kQS]
  const uint32_t s_full = bar0 + 48, s_empty = bar0 + 56;
  const uint32_t p_full0 = bar0 + 64, p_empty0 = bar0 + 80;  // [kPB]
  const uint32_t acc_full = bar0 + 96, acc_empty = bar0 + 104, drain = bar0 + 112;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kK_OffBar + 32 * 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  volatile int* s_consumed = reinterpret_cast<volatile int*>(s_tmem + 2);   // Q/dO tiles consumed
  volatile int* s_kvconsumed = reinterpret_cast<volatile int*>(s_tmem + 3);  // K/V loads consumed
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = H * HD;
  const int items = ntk * BH;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < kQS; ++i) {
      mbar_init(q_full0 + 8 * i, 1);
      mbar_init(q_empty0 + 8 * i, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 8);
    for (int i = 0; i < kPB; ++i) {
      mbar_init(p_full0 + 8 * i, 8);
      mbar_init(p_empty0 + 8 * i, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(drain, 1);
    fence_mbar_init();
    *s_abort = 0;
    *s_consumed = 0;
    *s_kvconsumed = 0;
    tma_prefetch_desc(&tm);
    tma_prefetch_desc(&tmo);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  int issued = 0, kvissued = 0;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int g = 0;
      bool ok = true;
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int kt = it / BH, bh = it - (it / BH) * BH;
        const int b = bh / H, h = bh - (bh / H) * H;
        if (n >= 1 && !mbar_wait(kv_empty, (n - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) break;
        mbar_arrive_expect_tx(kv_full, 2 * C::kTile128);
        tma_load_3d(sbase, &tm, kv_full, D + h * HD, kt * kTile, b);
        tma_load_3d(sbase + C::kTile64, &tm, kv_full, D + h * HD, kt * kTile + kKT, b);
        tma_load_3d(sbase + C::kK_OffV, &tm, kv_full, 2 * D + h * HD, kt * kTile, b);
        tma_load_3d(sbase + C::kK_OffV + C::kTile64, &tm, kv_full, 2 * D + h * HD, kt * kTile + kKT, b);
        ++kvissued;
        for (int t = 2 * kt; t < nq; ++t, ++g) {
          const int st = g % kQS;
          if (g >= kQS && !mbar_wait(q_empty0 + 8 * st, ((g / kQS) - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          const uint32_t fb = q_full0 + 8 * st;
          mbar_arrive_expect_tx(fb, 2 * C::kTile64);
          tma_load_3d(sbase + C::kK_OffQ + st * C::kTile64, &tm, fb, h * HD, t * kKT, b);
          tma_load_3d(sbase + C::kK_OffDO + st * C::kTile64, &tmo, fb, h * HD, t * kKT, b);
          ++issued;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr int fmt = std::is_same_v<T, __nv_bfloat16> ? 1 : 0;
      constexpr uint32_t idS = idesc_f16(kTile, kKT, fmt, 0, 0);
      constexpr uint32_t idA = idesc_f16(kTile, HD, fmt, 0, 1);
      bool ok = true, pending = false;
      int g = 0, gs = 0, gp = 0, kvc = 0;
      const uint32_t ka = sbase, va = sbase + C::kK_OffV;
      auto issue_s = [&]() -> bool {
        const int st = g % kQS;
        if (!mbar_wait(q_full0 + 8 * st, (g / kQS) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) return false;
        ++g;
        if (gs >= 1 && !mbar_wait(s_empty, (gs - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) return false;
        tc_fence_after();
        const uint32_t qa = sbase + C::kK_OffQ + st * C::kTile64, da = sbase + C::kK_OffDO + st * C::kTile64;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + C::kColS, smem_desc(ka + kk * 32, 16, C::kSbo, C::kSwz),
                   smem_desc(qa + kk * 32, 16, C::kSbo, C::kSwz), idS, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + C::kColDP, smem_desc(va + kk * 32, 16, C::kSbo, C::kSwz),
                   smem_desc(da + kk * 32, 16, C::kSbo, C::kSwz), idS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        ++gs;
        pending = true;
        return true;
      };
      for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
        const int kt = it / BH;
        const int nqt = nq - 2 * kt;
        if (!mbar_wait(kv_full, n & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
          ok = false;
          break;
        }
        ++kvc;
        int st_t = g % kQS;
        if (!issue_s()) {
          ok = false;
          break;
        }
        for (int i = 0; i < nqt; ++i) {
          const int st_next = g % kQS;
          if (i + 1 < nqt) {
            if (!issue_s()) {
              ok = false;
              break;
            }
          } else {
            umma_commit(kv_empty);  // every MMA reading K / V of this item issued
          }
          const int pb = gp % kPB;
          if (!mbar_wait(p_full0 + 8 * pb, (gp / kPB) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          if (i == 0 && n > 0 && !mbar_wait(acc_empty, (n - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;  // the previous item's dK / dV have been read out of TMEM
            break;
          }
          tc_fence_after();
          const uint32_t pa = sbase + C::kK_OffP + pb * kPBytes, dsa = sbase + C::kK_OffDS + pb * kPBytes;
          const uint32_t qa = sbase + C::kK_OffQ + st_t * C::kTile64, da = sbase + C::kK_OffDO + st_t * C::kTile64;
#pragma unroll
          for (int kk = 0; kk < kKT / 16; ++kk)
            umma_f16(tmem + C::kColAcc, smem_desc(pa + kk * 32, 16, 1024, 2),
                     smem_desc(da + kk * 16 * C::kRow, C::kVLbo, C::kSbo, C::kSwz), idA, (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kKT / 16; ++kk)
            umma_f16(tmem + C::kColAcc + HD, smem_desc(dsa + kk * 32, 16, 1024, 2),
                     smem_desc(qa + kk * 16 * C::kRow, C::kVLbo, C::kSbo, C::kSwz), idA, (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(q_empty0 + 8 * st_t);
          umma_commit(p_empty0 + 8 * pb);
          ++gp;
          st_t = st_next;
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
      *s_consumed = g;
      *s_kvconsumed = kvc;
      if (!ok && pending) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, RK_DEV_ATTN_TIMEOUT, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ P^T, dS^T rows
    // warp w: lane quarter w % 4 (one key row per thread), column half
    // ch = (w - 2) / 4 of the query tile; at the end of an item the ch = 0
    // warps read out dV, the ch = 1 warps dK
    const int quarter = warp & 3, ch = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    // this warp's lse[32] and D[32] of the current query tile (queries past T:
    // lse = +inf, so P = 0); lane l prefetches query ch*32 + l of the next tile
    float* lw = reinterpret_cast<float*>(smem + C::kK_OffL) + (warp - 2) * 64;
    int gs = 0, gp = 0;
    bool ok = true;
    for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
      const int kt = it / BH, bh = it - (it / BH) * BH;
      const int b = bh / H, h = bh - (bh / H) * H;
      const int key = kt * kTile + row;
      const float* lb = lse + (int64_t)bh * Tlen;
      const float* db = dsum + (int64_t)bh * Tlen;
      auto fetch = [&](int t, float& l, float& d) {
        const int q = t * kKT + 32 * ch + lane;
        const bool qv = t < nq && q < Tlen;
        l = qv ? __ldg(lb + q) : INFINITY;
        d = qv ? __ldg(db + q) : 0.f;
      };
      float l_next, d_next;
      fetch(2 * kt, l_next, d_next);
      for (int t = 2 * kt; t < nq; ++t) {
        __syncwarp();  // every lane is done with the previous tile's values
        lw[lane] = -l_next;  // negated: p = exp2(s * c + nl), ds = p * (dp + nd)
        lw[32 + lane] = -d_next;
        __syncwarp();
        fetch(t + 1, l_next, d_next);  // lands while this tile is processed
        bool w = mbar_wait(s_full, gs & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        w = __all_sync(0xffffffffu, w);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int lim = key - t * kKT;  // queries c of this tile with c >= lim see this key
        auto valid = [lim](int c) { return c >= lim; };
        const float* lrow = lw - 32 * ch;  // indexed by the tile column c in [32 ch, 32 ch + 32)
        const bool full = __all_sync(0xffffffffu, lim <= 0);  // every query of the tile sees the warp's keys
        const int pb = gp % kPB;
        uint8_t* ptile = smem + C::kK_OffP + pb * kPBytes;
        uint8_t* dtile = smem + C::kK_OffDS + pb * kPBytes;
        // two 16-column pieces; the P / dS buffer is free once the MMAs of tile
        // gp - kPB completed
#pragma unroll
        for (int piece = 0; piece < 2; ++piece) {
          const int c0 = 32 * ch + 16 * piece;
          uint32_t sv[16], dv[16], pw[8], dw[8];
          tmem_ld_16cols_nowait(t_lane + C::kColS + c0, sv);
          tmem_ld_16cols_nowait(t_lane + C::kColDP + c0, dv);
          tmem_ld_wait();
          if (piece == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty);  // this warp's S^T and dP^T columns are in registers
          }
          if (full)
            bwd_cols<T, 16, true, false>(sv, dv, c0, c_log2, lrow, lrow + 32, 0.f, 0.f, valid, pw, dw);
          else
            bwd_cols<T, 16, true, true>(sv, dv, c0, c_log2, lrow, lrow + 32, 0.f, 0.f, valid, pw, dw);
          // the dV / dK MMAs of tile gp - kPB have read these buffers: implied
          // for two buffers by S^T_gp (committed after those MMAs of tile
          // gp - 2 were issued), waited for with one
          if (piece == 0 && kPB == 1 && gp >= 1) {
            w = mbar_wait(p_empty0 + 8 * pb, (gp - 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
            w = __all_sync(0xffffffffu, w);
            if (!w) {
              ok = false;
              break;
            }
          }
          store_chunks128<2>(ptile, row, c0 / 8, pw);
          store_chunks128<2>(dtile, row, c0 / 8, dw);
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full0 + 8 * pb);
        ++gs;
        ++gp;
      }
      if (!ok) break;
      bool w = mbar_wait(acc_full, n & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
      w = __all_sync(0xffffffffu, w);
      if (!w) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t acc[HD];  // ch 0: dV, ch 1: dK
#pragma unroll
      for (int c = 0; c < HD; c += 32) tmem_ld_32cols_nowait(t_lane + C::kColAcc + ch * HD + c, acc + c);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (key < Tlen)
        store_acc_row<T, HD>(dqkv + ((int64_t)b * Tlen + key) * lddq + (2 - ch) * D + h * HD, acc,
                             ch ? scale : 1.f);
    }
  }

  __syncthreads();
  if (*s_abort && threadIdx.x == 0) {
    for (int i = *s_kvconsumed; i < kvissued; ++i) mbar_wait(kv_full, i & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
    for (int i = *s_consumed; i < issued; ++i)
      mbar_wait(q_full0 + 8 * (i % kQS), (i / kQS) & 1, status, RK_DEV_ATTN_TIMEOUT, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}
}  // namespace attn_tc
}  // namespace rk

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode3d_fn() {
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

}  // namespace

namespace {
template <int HD>
int fwd_tc_launch(const CUtensorMap& tm, void* out, int64_t ldo, float* lse, int64_t B, int64_t H, int64_t T,
                  int dtype, cudaStream_t s) {
  using namespace rk::attn_tc;
  constexpr uint32_t kSmem = Fwd<HD>::kSmem;
  const int ntq = (int)((T + kTile - 1) / kTile);
  const int BH = (int)(B * H);
  const int64_t items = (int64_t)ntq * BH;
  int sms = 148;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const unsigned grid = (unsigned)(items < kCtasPerSm * sms ? items : kCtasPerSm * sms);
  const float c_log2 = 1.4426950408889634f / sqrtf((float)HD);
  unsigned int* st = rk_host::device_status_ptr();
  if (dtype == RK_BF16) {
    auto k = fwd_tc_kernel<__nv_bfloat16, HD>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)kSmem)) return e_;
    rk_host::launch_k(k, grid, kThreads, kSmem, s, tm, static_cast<__nv_bfloat16*>(out), lse, (int)H, BH, ntq, (int)T,
                      ldo, c_log2, st);
  } else {
    auto k = fwd_tc_kernel<__half, HD>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)kSmem)) return e_;
    rk_host::launch_k(k, grid, kThreads, kSmem, s, tm, static_cast<__half*>(out), lse, (int)H, BH, ntq, (int)T, ldo,
                      c_log2, st);
  }
  return rk_host::launch_status();
}
}  // namespace

// Tensor-core forward for head_dim 32 and 64 (bf16/f16); returns
// RK_ERR_UNSUPPORTED when the layout does not fit it, so the caller can use
// the mma.sync kernel.
int rk_attn_fwd_tc(const void* qkv, int64_t ldq, void* out, int64_t ldo, float* lse, int64_t B, int64_t H,
                   int64_t HD, int64_t T, int dtype, cudaStream_t s) {
  using namespace rk::attn_tc;
  if (HD != 32 && HD != 64) return RK_ERR_UNSUPPORTED;
  auto fn = encode3d_fn();
  if (!fn || !rk_host::aligned(qkv, 16) || !rk_host::aligned(out, 16) || ldq % 8 || ldo % 8 || T >= (1 << 24) ||
      B * H >= (1 << 24))
    return RK_ERR_UNSUPPORTED;
  CUtensorMap tm;
  cuuint64_t dims[3] = {(cuuint64_t)(3 * H * HD), (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ldq * 2, (cuuint64_t)ldq * 2 * (cuuint64_t)T};
  cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)kKT, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (fn(&tm, dt, 3, const_cast<void*>(qkv), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         HD == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return RK_ERR_UNSUPPORTED;
  return HD == 32 ? fwd_tc_launch<32>(tm, out, ldo, lse, B, H, T, dtype, s)
                  : fwd_tc_launch<64>(tm, out, ldo, lse, B, H, T, dtype, s);
}

namespace {

// 3-D map over [B][T][ld] 16-bit rows, HD x 64-row boxes, in the swizzle of the
// head dim (64-byte rows: 64-byte swizzle, 128-byte rows: 128-byte swizzle).
bool head_map(CUtensorMap* tm, const void* base, int64_t width, int64_t ld, int64_t T, int64_t B, int64_t HD,
              int dtype) {
  auto fn = encode3d_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * (cuuint64_t)T};
  cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)rk::attn_tc::kKT, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(tm, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            HD == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int HD>
int bwd_tc_launch(int piece, const CUtensorMap& tm, const CUtensorMap& tmo, const float* lse, const float* dsum,
                  void* dqkv, int64_t lddq, int64_t B, int64_t H, int64_t Tlen, cudaStream_t s) {
  using namespace rk::attn_tc;
  using C = Bwd<HD>;
  const int BH = (int)(B * H);
  int sms = 148;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const float scale = 1.f / sqrtf((float)HD);
  const float c_log2 = 1.4426950408889634f * scale;
  unsigned int* st = rk_host::device_status_ptr();
  if (piece == 1) {
    const int ntq = (int)((Tlen + kTile - 1) / kTile);
    const int64_t items = (int64_t)ntq * BH;
    const unsigned grid = (unsigned)(items < kCtasPerSm * sms ? items : kCtasPerSm * sms);
    auto k = bwd_dq_tc_kernel<T, HD>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)C::kQ_Smem)) return e_;
    rk_host::launch_k(k, grid, kThreadsBwd, C::kQ_Smem, s, tm, tmo, lse, dsum, static_cast<T*>(dqkv), lddq, (int)H, BH,
                      ntq, (int)Tlen, c_log2, scale, st);
  } else {
    const int ntk = (int)((Tlen + kTile - 1) / kTile);
    const int nq = (int)((Tlen + kKT - 1) / kKT);
    const int64_t items = (int64_t)ntk * BH;
    const unsigned grid = (unsigned)(items < kCtasPerSm * sms ? items : kCtasPerSm * sms);
    auto k = bwd_dkv_tc_kernel<T, HD>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)C::kK_Smem)) return e_;
    rk_host::launch_k(k, grid, kThreadsBwd, C::kK_Smem, s, tm, tmo, lse, dsum, static_cast<T*>(dqkv), lddq, (int)H, BH,
                      ntk, nq, (int)Tlen, c_log2, scale, st);
  }
  return rk_host::launch_status();
}

}  // namespace

// Tensor-core backward pieces for head_dim 32 and 64 (bf16/f16): piece 1 = dQ,
// piece 2 = dK and dV, both reading lse (base 2, from the forward) and
// D = rowsum(dO * O) (written beforehand). Returns RK_ERR_UNSUPPORTED when the
// layout does not fit, so the caller can use the mma.sync kernels.
int rk_attn_bwd_tc(int piece, const void* qkv, int64_t ldq, const void* dout, int64_t ldo, const float* lse,
                   const float* dsum, void* dqkv, int64_t lddq, int64_t B, int64_t H, int64_t HD, int64_t T, int dtype,
                   cudaStream_t s) {
  if ((HD != 32 && HD != 64) || (piece != 1 && piece != 2)) return RK_ERR_UNSUPPORTED;
  if (!rk_host::aligned(qkv, 16) || !rk_host::aligned(dout, 16) || !rk_host::aligned(dqkv, 16) || ldq % 8 ||
      ldo % 8 || lddq % 8 || T >= (1 << 24) || B * H >= (1 << 24))
    return RK_ERR_UNSUPPORTED;
  CUtensorMap tm, tmo;
  if (!head_map(&tm, qkv, 3 * H * HD, ldq, T, B, HD, dtype) || !head_map(&tmo, dout, H * HD, ldo, T, B, HD, dtype))
    return RK_ERR_UNSUPPORTED;
  if (dtype == RK_BF16)
    return HD == 32 ? bwd_tc_launch<__nv_bfloat16, 32>(piece, tm, tmo, lse, dsum, dqkv, lddq, B, H, T, s)
                    : bwd_tc_launch<__nv_bfloat16, 64>(piece, tm, tmo, lse, dsum, dqkv, lddq, B, H, T, s);
  return HD == 32 ? bwd_tc_launch<__half, 32>(piece, tm, tmo, lse, dsum, dqkv, lddq, B, H, T, s)
                  : bwd_tc_launch<__half, 64>(piece, tm, tmo, lse, dsum, dqkv, lddq, B, H, T, s);
}
