// common.cuh - device helpers shared by the decode kernels (sm_100a only).
//
// * mbarrier + cp.async.bulk (TMA, non-tensor) producer/consumer ring helpers,
//   with bounded waits: a wait that does not complete within kSpinLimit polls
//   records an error code in dbk_device_error and returns false, so a kernel
//   can leave instead of hanging the GPU;
// * warp reductions and 16-bit <-> fp32 conversions for fp16 and bf16 payloads.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "decodebench_b200 kernels target sm_100a only"
#endif

namespace dbk {

// Error codes written to dbk_device_error by a kernel that gave up waiting.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,      // consumer waited too long for a stage to fill
  kDevTimeoutEmpty = 2,     // producer waited too long for a stage to drain
  kDevTimeoutMma = 3,       // waited too long for a tensor-core commit
  kDevTimeoutDrain = 4,     // waited too long for in-flight copies at exit
  kDevTimeoutPeer = 5,      // waited too long for another GPU's all-gather signal
  kDevTimeoutMerge = 6,     // waited too long for the other contributors of a tile
  kDevTimeoutGrid = 7,      // waited too long at a grid-wide barrier of a persistent kernel
};

extern __device__ int dbk_device_error;

// Default poll budget for every spin-wait: mbarrier.try_wait suspends for a
// hardware-chosen interval per poll, so 1<<24 polls is seconds, far beyond
// any legitimate wait in these kernels. The budget in force is dbk_spin_limit
// (per device, set by dbk_set_spin_limit; tests lower it to make a wait run out).
constexpr uint32_t kSpinLimit = 1u << 24;
// Constant memory: read through the constant cache, so a wait loop pays no
// global-memory latency for it.
extern __constant__ uint32_t dbk_spin_limit;

__device__ __forceinline__ uint32_t spin_limit() { return dbk_spin_limit; }

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&dbk_device_error, 0, code);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Adds 1 to *p with release semantics at GPU scope (prior writes visible first).
__device__ __forceinline__ void arrive_release_gpu(int* p) {
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p) : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- dev tracing
// Phase timestamps for development builds (-DDBK_TRACE) only; compiled out of
// the library. Slot k of CTA c is written to dbk_trace[c * 16 + k].
#ifdef DBK_TRACE
// Four launches are kept apart: every CTA takes a ticket at its start (the
// CTAs of launch n all start before those of launch n + 1 can), and launch
// (ticket / gridDim.x) % 4 picks the buffer.
extern __device__ unsigned long long dbk_trace[4 * 2048 * 16];
extern __device__ unsigned int dbk_trace_ticket;
__device__ __forceinline__ int& trace_launch() {
  __shared__ int s_launch;
  return s_launch;
}
#define DBK_TRACE_BEGIN()                                                          \
  do {                                                                             \
    if (threadIdx.x == 0)                                                          \
      dbk::trace_launch() = (int)((atomicAdd(&dbk::dbk_trace_ticket, 1u) / gridDim.x) & 3); \
  } while (0)
#define DBK_TRACE_SLOT(slot) \
  dbk::dbk_trace[((size_t)dbk::trace_launch() * 2048 + blockIdx.x) * 16 + (slot)]
#define DBK_MARK(cond, slot)                                              \
  do {                                                                    \
    if (cond) {                                                           \
      unsigned long long t_;                                              \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));              \
      DBK_TRACE_SLOT(slot) = t_;                                          \
    }                                                                     \
  } while (0)
// Adds the time spent in a wait to slot `slot` (cond threads only).
#define DBK_TIMED_WAIT(cond, slot, expr)                                  \
  ([&]() {                                                                \
    unsigned long long a_, b_;                                            \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(a_));                \
    const bool r_ = (expr);                                               \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(b_));                \
    if (cond) DBK_TRACE_SLOT(slot) += b_ - a_;                            \
    return r_;                                                            \
  }())
#else
#define DBK_TRACE_BEGIN() \
  do {                    \
  } while (0)
#define DBK_TIMED_WAIT(cond, slot, expr) (expr)
#define DBK_MARK(cond, slot) \
  do {                       \
  } while (0)
#endif

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err_code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint32_t lim = spin_limit();
  for (uint32_t i = 1; i < lim; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  record_error(err_code);
  return false;
}

// ---------------------------------------------------------------- bulk copies
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy completing on an mbarrier (no multicast).
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled 2-D TMA load (no multicast): box at coordinates (x = inner, y = row).
// x * sizeof(elem) must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled 3-D TMA load (no multicast) at coordinates (x, y, z).
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
      ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- warp MMA (m16n8k16)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

// Transpose an 8x8 matrix of 16-bit values held as one register per thread
// (thread t: row t/4, columns 2*(t%4) and 2*(t%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T> struct Mma;
template <> struct Mma<__half> {
  // d += a * b, a: 16x16 row-major fragment (4 regs), b: 16x8 col fragment (2 regs)
  __device__ __forceinline__ static void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
};
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
};

// ---------------------------------------------------------------- barriers
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------- 16-bit types
// Element traits: unpack a 32-bit word holding two 16-bit values into fp32s.
template <typename T> struct Elem;

template <> struct Elem<__half> {
  __device__ __forceinline__ static float2 unpack2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};

template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float2 unpack2(uint32_t w) {
    // bf16 is the upper half of an fp32: widening is a shift / mask.
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Unpack 8 packed 16-bit values (one 16-byte vector) into fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  float2 a = Elem<T>::unpack2(v.x), b = Elem<T>::unpack2(v.y);
  float2 c = Elem<T>::unpack2(v.z), d = Elem<T>::unpack2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Read-only 16-byte global load through the non-coherent path.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

}  // namespace dbk
