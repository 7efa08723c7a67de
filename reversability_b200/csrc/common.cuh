// Shared device helpers for librevk: dtype conversion, bounded mbarrier waits,
// TMA and tcgen05 (5th-generation tensor core) PTX wrappers for sm_100a.
//
// Every spin-wait in this library is bounded: after RK_WAIT_LIMIT_NS of
// wall-clock time (read from %globaltimer) the waiting thread records an error
// bit in `rk_device_status` and returns false, so the kernel can drain and
// exit instead of hanging the GPU. The host reads and clears the word with
// rk_device_status_read().
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "../../include/revk.h"

#define RK_WAIT_LIMIT_NS 2000000000ull  // 2 s: every healthy wait here ends in microseconds

namespace rk {

// Kernels with bounded waits receive a pointer to the library's device status
// word (bit flags, see revk.h) and OR their error bit into it.
__device__ __forceinline__ void flag_error(unsigned int* status, unsigned int bits) {
  if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------- dtypes
template <typename T> struct Dt;
template <> struct Dt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <typename T> __device__ __forceinline__ float ld_f(const T* p) { return Dt<T>::to_f(*p); }
template <typename T> __device__ __forceinline__ void st_f(T* p, float v) { *p = Dt<T>::from_f(v); }
// Round a float through storage type T (the reference's `.to(dtype).to(float32)`).
template <typename T> __device__ __forceinline__ float round_to(float v) { return Dt<T>::to_f(Dt<T>::from_f(v)); }

// Logistic pieces of SiLU with the hardware exponential and an approximate
// divide (ex2.approx + div.approx, a few ulp in fp32 — like the reference's
// Triton kernels, which compile exp and '/' to the same approximate
// instructions). Shared by the standalone SwiGLU kernels and the GEMM epilogue
// so both produce identical bits.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float exp_neg(float g) { return ex2_approx(-1.4426950408889634f * g); }
__device__ __forceinline__ float silu_value(float g) { return __fdividef(g, 1.f + exp_neg(g)); }
__device__ __forceinline__ float sigmoid_value(float g) { return __fdividef(1.f, 1.f + exp_neg(g)); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
// Bounded wait for phase `parity` of the barrier. Returns false (and ORs
// `err_bits` into *status) when the limit passes; also returns false once
// *abort has been set by another role of the same CTA.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* status,
                                          unsigned int err_bits, volatile int* abort) {
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (globaltimer() - t0 > RK_WAIT_LIMIT_NS) {
      flag_error(status, err_bits);
      if (abort) *abort = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Plain (non-multicast) 2-D tiled bulk tensor load into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 in, f32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32-bit, 32 consecutive columns: thread i of the warp receives
// lane (base_lane + i), columns [col, col + 32).
// tcgen05.ld of 32 consecutive columns without the wait: several loads may be
// in flight; tmem_ld_wait() makes all of them visible in their registers.
__device__ __forceinline__ void tmem_ld_32cols_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for tcgen05 (SWIZZLE_128B canonical layouts).
//   K-major : rows of 128 B (64 bf16 along K), 8-row groups 1024 B apart (SBO);
//             LBO is unused and set to 16 B.
//   MN-major: rows of 128 B (64 bf16 along M/N) indexed by K, 8-K-row groups
//             1024 B apart (SBO); consecutive 64-wide M/N chunks `lbo` apart (LBO).
// Bits: [0,14) addr>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
//       [49,52) base offset=0, [61,64) layout (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f32 accumulation.
// ab_fmt: 0 = f16, 1 = bf16. a_mn/b_mn: 1 when the operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_fmt, int a_mn, int b_mn) {
  return (1u << 4)                          // D format f32
         | ((uint32_t)ab_fmt << 7)          // A format
         | ((uint32_t)ab_fmt << 10)         // B format
         | ((uint32_t)a_mn << 15)           // A major
         | ((uint32_t)b_mn << 16)           // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (TMA stores, tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ int elect_lane0() { return (threadIdx.x & 31) == 0; }

// RMSNorm row statistics in one fixed order, shared by the standalone norm
// kernels and the norm fused into the GEMM epilogue so that both give the same
// bits: a lane's V consecutive squares are chained in column order, the 32
// lanes of a 32V-column group are added in xor-butterfly order, and the group
// totals are added in column order; rstd = rsqrt(sum / width + eps).
template <int V>
__device__ __forceinline__ float sumsq_chain(const float (&v)[V]) {
  float t = __fmul_rn(v[0], v[0]);
#pragma unroll
  for (int e = 1; e < V; ++e) t = __fmaf_rn(v[e], v[e], t);
  return t;
}
__device__ __forceinline__ float sumsq4(float a, float b, float c, float d) {
  return __fmaf_rn(d, d, __fmaf_rn(c, c, __fmaf_rn(b, b, __fmul_rn(a, a))));
}
__device__ __forceinline__ float rms_rstd(float ss, int width, float eps) {
  return rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)width), eps));
}

// Programmatic dependent launch: every librevk kernel is launched with
// programmatic stream serialization, so it may become resident while the
// previous kernel on the stream drains. pdl_wait() blocks until that kernel
// has completed and its writes are visible; a kernel calls it before its first
// read of inputs or write of outputs; it is a no-op when the launch had no PDL
// attribute. No kernel triggers its dependents explicitly: the next grid starts
// launching as this grid's blocks exit, so its prologue and launch latency
// overlap this grid's tail without taking SM slots from this grid's main loop
// (an explicit trigger at kernel entry measured slower).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace rk

// Host-side helpers shared by the translation units.
namespace rk_host {
// Counts every kernel launch the library makes (status.cu); read with rk_launch_count().
void count_launch();
// Programmatic dependent launch on/off (status.cu; REVK_PDL=0 in the environment disables it).
bool pdl_enabled();

// Launches `kernel` on stream `s` with programmatic stream serialization (see pdl_wait).
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
inline int launch_status() {
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RK_OK : RK_ERR_LAUNCH;
}
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t dtype_size(int dt) { return dt == RK_F32 ? 4 : 2; }
// Device address of the status word on the current device (status.cu).
unsigned int* device_status_ptr();
// Raises `kernel`'s dynamic shared-memory limit to at least `bytes` on the
// current device; the limit set is remembered per (kernel, device), so later
// calls (e.g. inside CUDA-graph capture) make no attribute calls at all.
// Returns RK_OK, or RK_ERR_LAUNCH when the attribute call fails (status.cu).
int ensure_smem_attr(const void* kernel, int bytes);
inline bool dtype_ok(int dt) { return dt == RK_F32 || dt == RK_BF16 || dt == RK_F16; }
}  // namespace rk_host
