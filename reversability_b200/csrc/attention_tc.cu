// Causal attention forward on the 5th-generation tensor cores for head_dim 32
// (replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) at
// model.py:42-44 for the model's 8 x 32 heads).
//
// One CTA per (128-query tile, batch*head), walking the key tiles 0..qt:
//   warp 0      TMA producer: Q once, then K_j and V_j (128 keys x 32) into a
//               two-stage ring (3-D tensor map over [B][T][ldq], so rows past
//               T read as zeros).
//   warp 1      tcgen05.mma issuer: S_j = Q K_j^T (M=128, N=128, K=32) into a
//               TMEM accumulator; O_j = P_j V_j (M=128, N=32, K=128) into one
//               of two TMEM O buffers.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): pass 1
//               reads S_j for the row max (no shuffles), pass 2 re-reads it,
//               writes P_j = exp2(s*c - m) (bf16/f16) into a 128-byte-swizzled
//               shared tile for the PV MMA and sums it; the previous O_{j-1}
//               is merged into a register accumulator with the usual online
//               rescale while PV_j runs.
// S is single-buffered (the next S waits for pass 2), so two CTAs share an SM
// (256 TMEM columns and ~107 KB of shared memory each) and hide each other's
// latencies. lse is written in base 2 (max*c + log2(sum)), the layout the
// backward kernels read.
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
constexpr int kHD = 32;     // head dim
constexpr int kThreads = 192;
constexpr int kKVStages = 4;
// Score buffers in TMEM and resident CTAs per SM. One buffer and three CTAs
// (twelve softmax warps per SM, 128 TMEM columns each, two K/V stages) measured
// 46.5 us against 26.9 us for two buffers and two CTAs at cfg2 (the softmax
// warps then spill).
constexpr int kSBufs = 2;
constexpr int kCtasPerSm = 2;
constexpr uint32_t kQBytes = kTile * kHD * 2;     // 8 KB
constexpr uint32_t kKVBytes = kKT * kHD * 2;      // 4 KB each for K and V
constexpr uint32_t kPBytes = kTile * kKT * 2;     // 16 KB (one 64-key swizzle atom)
// layout: Q0 Q1 | K ring | V ring | P0 P1 | barriers
constexpr uint32_t kOffK = 2 * kQBytes;
constexpr uint32_t kOffV = kOffK + kKVStages * kKVBytes;
constexpr uint32_t kOffP = kOffV + kKVStages * kKVBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
constexpr uint32_t kNumBars = 26;
constexpr uint32_t kSmem = 1024 + kOffBar + kNumBars * 8 + 32;
constexpr uint32_t kOCol = kSBufs * kKT;                  // S [0, 64 * kSBufs), O [kOCol, kOCol + 32)
constexpr uint32_t kTmemCols = kSBufs == 1 ? 128 : 256;    // power of two >= kOCol + 32
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
template <typename T>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, T* __restrict__ out, float* __restrict__ lse, int H,
                  int BH, int ntq, int Tlen, int64_t ldo, float c_log2, unsigned int* status) {
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
  const int D = H * kHD;
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
        tma_load_3d(sbase + qb * kQBytes, &tm, qf, h * kHD, qt * kTile, b);
        tma_load_3d(sbase + qb * kQBytes + kQBytes / 2, &tm, qf, h * kHD, qt * kTile + kKT, b);
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
          tma_load_3d(sbase + kOffK + st * kKVBytes, &tm, fb, D + h * kHD, j * kKT, b);
          tma_load_3d(sbase + kOffV + st * kKVBytes, &tm, fb, 2 * D + h * kHD, j * kKT, b);
          ++issued;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idS = idesc_f16(kTile, kKT, std::is_same_v<T, __nv_bfloat16> ? 1 : 0, 0, 0);
      constexpr uint32_t idPV = idesc_f16(kTile, kHD, std::is_same_v<T, __nv_bfloat16> ? 1 : 0, 0, 1);
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
        for (int kk = 0; kk < kHD / 16; ++kk)
          umma_f16(tmem + sb * kKT, smem_desc(qa + kk * 32, 16, 512, 4), smem_desc(ka + kk * 32, 16, 512, 4), idS,
                   kk > 0 ? 1u : 0u);
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
          const int pb = gp & 1;
          if (!mbar_wait(bb.p_full0 + 8 * pb, (gp >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = sbase + kOffP + pb * kPBytes;
          const uint32_t va = sbase + kOffV + st_j * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kKT / 16; ++kk)
            umma_f16(tmem + kOCol, smem_desc(pa + kk * 32, 16, 1024, 2), smem_desc(va + kk * 1024, 4096, 512, 4),
                     idPV, (j > 0 || kk > 0) ? 1u : 0u);
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
        // P buffer free (PV tile gp-2 done): after this wait at most one PV
        // (gp-1) is outstanding, so the o_full parity wait below is unambiguous
        const int pb = gp & 1;
        if (gp >= 2) {
          w = mbar_wait(bb.p_empty0 + 8 * pb, ((gp - 2) >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
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
            uint32_t o[32];
            tmem_ld_32cols_nowait(t_lane + kOCol, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32cols(t_lane + kOCol, o);
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
      // all of this item's PV tiles complete: first gp-2 through its P buffer
      // barrier (at most one use outstanding there), then gp-1 through o_full
      if (ok && gp >= 2) {
        bool w = mbar_wait(bb.p_empty0 + 8 * (gp & 1), ((gp - 2) >> 1) & 1, status, RK_DEV_ATTN_TIMEOUT, s_abort);
        ok = __all_sync(0xffffffffu, w);
      }
      if (!ok || !wait_pv(gp - 1)) {
        ok = false;
        break;
      }
      {
        uint32_t o[32];
        tmem_ld_32cols_nowait(t_lane + kOCol, o);
        tmem_ld_wait();
        if (grow < Tlen) {
          const float inv = 1.f / l_run;
          T* orow = out + ((int64_t)b * Tlen + grow) * ldo + h * kHD;
#pragma unroll
          for (int q = 0; q < kHD / 8; ++q) {
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

// Tensor-core forward for head_dim 32 (bf16/f16); returns RK_ERR_UNSUPPORTED
// when the layout does not fit it, so the caller can use the mma.sync kernel.
int rk_attn_fwd_tc32(const void* qkv, int64_t ldq, void* out, int64_t ldo, float* lse, int64_t B, int64_t H,
                     int64_t T, int dtype, cudaStream_t s) {
  using namespace rk::attn_tc;
  auto fn = encode3d_fn();
  if (!fn || !rk_host::aligned(qkv, 16) || !rk_host::aligned(out, 16) || ldq % 8 || ldo % 8 || T >= (1 << 24) ||
      B * H >= (1 << 24))
    return RK_ERR_UNSUPPORTED;
  CUtensorMap tm;
  cuuint64_t dims[3] = {(cuuint64_t)(3 * H * kHD), (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ldq * 2, (cuuint64_t)ldq * 2 * (cuuint64_t)T};
  cuuint32_t box[3] = {(cuuint32_t)kHD, (cuuint32_t)kKT, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == RK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (fn(&tm, dt, 3, const_cast<void*>(qkv), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return RK_ERR_UNSUPPORTED;
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
  const float c_log2 = 1.4426950408889634f / sqrtf((float)kHD);
  unsigned int* st = rk_host::device_status_ptr();
  if (dtype == RK_BF16) {
    auto k = fwd_tc_kernel<__nv_bfloat16>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)kSmem)) return e_;
    rk_host::launch_k(k, grid, kThreads, kSmem, s, tm, static_cast<__nv_bfloat16*>(out), lse, (int)H, BH, ntq, (int)T,
                      ldo, c_log2, st);
  } else {
    auto k = fwd_tc_kernel<__half>;
    if (const int e_ = rk_host::ensure_smem_attr(reinterpret_cast<const void*>(k), (int)kSmem)) return e_;
    rk_host::launch_k(k, grid, kThreads, kSmem, s, tm, static_cast<__half*>(out), lse, (int)H, BH, ntq, (int)T, ldo,
                      c_log2, st);
  }
  return rk_host::launch_status();
}
