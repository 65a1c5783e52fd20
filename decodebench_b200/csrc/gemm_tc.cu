// gemm_tc.cu - batch 9..256 decode "thin GEMM" on tcgen05 tensor cores.
//
//   y[b, o] = sum_k W[o, k] * x'[b, k]       (W [d_out, d_in] row-major, x' [batch, d_in])
//
// with the same fused epilogues as the CUDA-core GEMV family (gemv.cu):
//   PLAIN  y = W x (+ residual)          NORM  y = inv_rms * W (x * gamma)
//   SWIGLU h = silu(Wg x') * (Wu x')      (x' = x, or RMSNorm(x) when gamma is given)
//
// At batch 16 the Llama-70B MLP does 16 flop per weight byte:
// still HBM-bound, but too much work for CUDA cores (~300 us of fp32 FMA vs
// ~210 us of HBM time), so the contraction runs on the 5th-generation tensor
// cores while the kernel stays a weight stream:
//   * D[128 weight rows x N] += A[128 x 64] * B[N x 64]^T per 64-column k-block:
//     A = a 128-row tile of W, B = the activations (N = batch rounded up to 16);
//     both K-major, staged by tiled TMA with the 128-byte swizzle, described to
//     tcgen05.mma by shared-memory descriptors; fp32 accumulators live in TMEM;
//   * persistent CTAs, one per SM, split the (m-tile, k-block) units evenly
//     ("stream-K"): CTA c owns units [c*U/G, (c+1)*U/G) in m-major order, so a
//     CTA's range cuts at most two m-tiles; an m-tile covered by one CTA is
//     finished in place, otherwise each contributor writes its fp32 partial to
//     the workspace and the last to arrive (self-resetting counter) sums the
//     partials in CTA order (deterministic) and applies the epilogue;
//   * warp roles: warp 0 streams tiles (TMA), warp 1 owns TMEM and issues the
//     MMAs (one elected thread; tcgen05.commit releases smem stages), warps 2-5
//     drain TMEM (tcgen05.ld) and run the epilogue;
//   * activations that are not exact in 16 bits (x * gamma) are written by a
//     small prep kernel as a high and a low bf16/fp16 part and both are
//     multiplied (two MMAs), so the products keep ~16-22 mantissa bits; the prep
//     kernel also computes inv_rms. Programmatic dependent launch lets the GEMM
//     start streaming weights while the prep kernel (or the previous op) runs.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

enum TcMode : int { TC_PLAIN = 0, TC_NORM = 1, TC_SWIGLU = 2 };

constexpr int kBM = 128;        // weight rows per m-tile
constexpr int kBK = 64;         // k-block (one 128-byte swizzle atom of 16-bit values)
constexpr int kTcThreads = 192; // producer, MMA, 4 epilogue warps
constexpr int kMaxN = 256;

struct TcArgs {
  CUtensorMap wmap0;   // W (or Wg) [d_out, d_in], box [128 rows x 64]
  CUtensorMap wmap1;   // Wu for SWIGLU
  CUtensorMap bmap;    // B operand rows [N, d_in] (x or the prep buffer's hi part), box [N x 64]
  CUtensorMap bmap_lo; // prep buffer's lo part (SPLIT only)
  const void* residual;   // [batch, d_out] or nullptr
  void* y;                // [batch, d_out]
  const float* inv_rms;   // [N] (NORM / SWIGLU with gamma) or nullptr
  float* part;            // [2 * grid][NACC][128][N] fp32 partials
  int* done;              // [m-tiles] arrival counters (zero between launches)
  int batch, n, d_in, d_out;
  int mtiles, kblocks;
  int nstages, stage_bytes;
  uint32_t tmem_cols;
};

__device__ __forceinline__ int owner(int64_t u, int64_t U, int64_t G) {
  return (int)(((u + 1) * G + U - 1) / U - 1);
}
__device__ __forceinline__ int range_start(int64_t c, int64_t U, int64_t G) {
  return (int)(c * U / G);
}

// ---------------------------------------------------------------- tcgen05 helpers
// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row core
// groups 1024 bytes apart (SBO); LBO unused for swizzled K-major layouts.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);           // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (unused)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, fp32 accumulate, A/B K-major, M = 128.
__device__ __forceinline__ uint32_t idesc_f16(bool bf16, int n) {
  uint32_t d = 0;
  d |= 1u << 4;                                      // D format f32
  d |= (bf16 ? 1u : 0u) << 7;                        // A format
  d |= (bf16 ? 1u : 0u) << 10;                       // B format
  d |= (uint32_t)(n >> 3) << 17;                     // N
  d |= (uint32_t)(kBM >> 4) << 24;                   // M
  return d;
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 16 columns of fp32 from TMEM (this warp's lane quarter).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- prep kernel
// B operand for non-exact activations: hi/lo parts of x * gamma (rows >= batch
// zero), and inv_rms[b] = rsqrt(mean(x^2) + eps). One CTA per batch row.
template <typename T>
__global__ void __launch_bounds__(256) tc_prep_kernel(const T* x, const T* gamma, T* b_hi, T* b_lo,
                                                      float* inv_rms, int batch, int d_in,
                                                      float eps) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < d_in; c += 256 * 8) {
    uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0, 0, 0, 0);
    if (b < batch) {
      float f[8], g[8];
      unpack8<T>(ldg_nc_v4(x + (size_t)b * d_in + c), f);
      if (gamma) unpack8<T>(ldg_nc_v4(gamma + c), g);
      uint32_t h[4], l[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float p0 = f[e], p1 = f[e + 1];
        ss = fmaf(p0, p0, fmaf(p1, p1, ss));
        if (gamma) { p0 *= g[e]; p1 *= g[e + 1]; }
        h[e / 2] = Mma<T>::pack(p0, p1);
        const float2 hf = Elem<T>::unpack2(h[e / 2]);
        l[e / 2] = Mma<T>::pack(p0 - hf.x, p1 - hf.y);
      }
      hv = make_uint4(h[0], h[1], h[2], h[3]);
      lv = make_uint4(l[0], l[1], l[2], l[3]);
    }
    *reinterpret_cast<uint4*>(b_hi + (size_t)b * d_in + c) = hv;
    *reinterpret_cast<uint4*>(b_lo + (size_t)b * d_in + c) = lv;
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    inv_rms[b] = (b < batch) ? rsqrtf(t / (float)d_in + eps) : 0.f;
  }
  asm volatile("griddepcontrol.launch_dependents;");
}

// ---------------------------------------------------------------- GEMM kernel
template <typename T, int MODE, bool SPLIT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcArgs a) {
  constexpr int NACC = (MODE == TC_SWIGLU) ? 2 : 1;   // accumulators (gate, up)
  constexpr int NB = SPLIT ? 2 : 1;                   // B parts (hi, lo)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.nstages * a.stage_bytes);
  uint64_t* empty = full + a.nstages;
  uint64_t* acc_full = empty + a.nstages;
  uint64_t* acc_empty = acc_full + 1;
  __shared__ uint32_t s_tmem;
  __shared__ int s_last[4];
  __shared__ volatile int s_bail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = a.n;
  const int a_bytes = kBM * kBK * 2;            // 16 KB per A tile
  const int b_bytes = N * kBK * 2;              // N x 128 B per B tile

  const int64_t U = (int64_t)a.mtiles * a.kblocks;
  const int G = (int)min((int64_t)gridDim.x, U);
  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    fence_barrier_init();
    s_bail = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&s_tmem)), "r"(a.tmem_cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  asm volatile("griddepcontrol.launch_dependents;");
  const uint32_t tmem = s_tmem;

  const bool active = blockIdx.x < G;
  const int u0 = active ? range_start(blockIdx.x, U, G) : 0;
  const int u1 = active ? range_start(blockIdx.x + 1, U, G) : 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && active) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // Weight tiles do not depend on the previous kernel: stream the first
      // stages' A tiles before waiting for it, their B tiles after.
      const int pre = min(a.nstages, u1 - u0);
      for (int j = 0; j < pre; ++j) {
        const int u = u0 + j, mt = u / a.kblocks, kb = u - mt * a.kblocks;
        uint8_t* st = smem + (size_t)j * a.stage_bytes;
        mbar_arrive_expect_tx(&full[j], (uint32_t)(NACC * a_bytes + NB * b_bytes));
        tma_load_2d(st, &a.wmap0, kb * kBK, mt * kBM, &full[j], pol_w);
        if constexpr (NACC == 2) tma_load_2d(st + a_bytes, &a.wmap1, kb * kBK, mt * kBM, &full[j], pol_w);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int j = 0; j < pre; ++j) {
        const int u = u0 + j, kb = u % a.kblocks;
        uint8_t* st = smem + (size_t)j * a.stage_bytes + NACC * a_bytes;
        tma_load_2d(st, &a.bmap, kb * kBK, 0, &full[j], pol_x);
        if constexpr (SPLIT) tma_load_2d(st + b_bytes, &a.bmap_lo, kb * kBK, 0, &full[j], pol_x);
      }
      for (int j = pre; j < u1 - u0; ++j) {
        const int s = j % a.nstages;
        if (!mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty)) { s_bail = 1; break; }
        const int u = u0 + j, mt = u / a.kblocks, kb = u - mt * a.kblocks;
        uint8_t* st = smem + (size_t)s * a.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(NACC * a_bytes + NB * b_bytes));
        tma_load_2d(st, &a.wmap0, kb * kBK, mt * kBM, &full[s], pol_w);
        if constexpr (NACC == 2) tma_load_2d(st + a_bytes, &a.wmap1, kb * kBK, mt * kBM, &full[s], pol_w);
        tma_load_2d(st + NACC * a_bytes, &a.bmap, kb * kBK, 0, &full[s], pol_x);
        if constexpr (SPLIT)
          tma_load_2d(st + NACC * a_bytes + b_bytes, &a.bmap_lo, kb * kBK, 0, &full[s], pol_x);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (active) {
      const uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value, N);
      int seg = 0;
      bool first = true;
      for (int j = 0; j < u1 - u0 && !s_bail; ++j) {
        const int u = u0 + j, mt = u / a.kblocks, kb = u - mt * a.kblocks;
        const int s = j % a.nstages;
        if (first && seg > 0) {
          // the epilogue must have drained the previous segment's accumulators
          if (!mbar_wait(acc_empty, (seg - 1) & 1, kDevTimeoutMma)) { s_bail = 1; break; }
          tc_fence_after();
        }
        if (!mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull)) { s_bail = 1; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + (size_t)s * a.stage_bytes);
#pragma unroll
          for (int acc = 0; acc < NACC; ++acc) {
#pragma unroll
            for (int part = 0; part < NB; ++part) {
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k) {
                const uint64_t da = sw128_desc(st + acc * a_bytes + k * 32);
                const uint64_t db = sw128_desc(st + NACC * a_bytes + part * b_bytes + k * 32);
                const uint32_t accumulate = (first && part == 0 && k == 0) ? 0u : 1u;
                umma(tmem + acc * N, da, db, idesc, accumulate);
              }
            }
          }
          umma_commit(&empty[s]);           // stage free once these MMAs have read it
        }
        __syncwarp();
        first = false;
        const bool seg_end = (kb == a.kblocks - 1) || (j == u1 - u0 - 1);
        if (seg_end) {
          if (lane == 0) umma_commit(acc_full);
          __syncwarp();
          ++seg;
          first = true;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
    const int row_local = quarter * 32 + lane;    // m-tile row of this thread
    const int etid = tid - 64;                    // 0..127
    T* y = static_cast<T*>(a.y);
    const T* res = static_cast<const T*>(a.residual);
    int seg = 0;
    for (int j0 = 0; active && j0 < u1 - u0 && !s_bail;) {
      const int u = u0 + j0, mt = u / a.kblocks, kb0 = u - mt * a.kblocks;
      const int len = min(a.kblocks - kb0, u1 - u);       // units of this segment
      if (!mbar_wait(acc_full, seg & 1, kDevTimeoutMma)) { s_bail = 1; break; }
      tc_fence_after();
      const int ngrp = N / 16;
      const bool whole = (kb0 == 0) && (len == a.kblocks);
      const int row = mt * kBM + row_local;
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      // Epilogue of 16 batch columns (gq) for this thread's output row.
      auto finish = [&](int gq, const float (&g0)[16], const float (&g1)[16]) {
        if (row >= a.d_out) return;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int b = gq * 16 + i;
          if (b >= a.batch) break;
          float val;
          if constexpr (MODE == TC_SWIGLU) {
            const float sc = a.inv_rms ? a.inv_rms[b] : 1.f;
            val = silu(g0[i] * sc) * (g1[i] * sc);
          } else if constexpr (MODE == TC_NORM) {
            val = g0[i] * a.inv_rms[b];
          } else {
            val = g0[i];
          }
          const size_t o = (size_t)b * a.d_out + row;
          if (res != nullptr) val += Elem<T>::to_f(res[o]);
          y[o] = Elem<T>::from_f(val);
        }
      };
      if (whole) {
        for (int gq = 0; gq < ngrp; ++gq) {
          float g0[16], g1[16];
          tmem_ld16(trow + gq * 16, g0);
          if constexpr (NACC == 2) tmem_ld16(trow + N + gq * 16, g1);
          finish(gq, g0, g1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);   // one arrival per epilogue warp
        j0 += len;
        ++seg;
        continue;
      }
      // Partial m-tile: publish this CTA's fp32 partial; the last contributor merges.
      const int slot = 2 * blockIdx.x + (u == u0 ? 0 : 1);
      float* dst = a.part + ((size_t)slot * NACC * kBM + row_local) * N;
      for (int gq = 0; gq < ngrp; ++gq) {
#pragma unroll
        for (int acc = 0; acc < NACC; ++acc) {
          float g0[16];
          tmem_ld16(trow + acc * N + gq * 16, g0);
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(dst + (size_t)acc * kBM * N + gq * 16 + i) =
                make_float4(g0[i], g0[i + 1], g0[i + 2], g0[i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      __threadfence();
      named_bar_sync(1, 128);
      const int first_u = mt * a.kblocks, last_u = first_u + a.kblocks - 1;
      const int c_first = owner(first_u, U, G), c_last = owner(last_u, U, G);
      if (etid == 0) {
        const int prev = atomicAdd(&a.done[mt], 1);
        s_last[0] = (prev == c_last - c_first);
      }
      named_bar_sync(1, 128);
      const bool last = s_last[0] != 0;
      named_bar_sync(1, 128);                   // s_last is rewritten by the next segment
      if (last) {
        __threadfence();
        for (int gq = 0; gq < ngrp; ++gq) {
          float g0[16], g1[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) g0[i] = g1[i] = 0.f;
          for (int c = c_first; c <= c_last; ++c) {
            const int sl = 2 * c + (range_start(c, U, G) >= first_u ? 0 : 1);
            const float* src = a.part + ((size_t)sl * NACC * kBM + row_local) * N + gq * 16;
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 p0 = __ldcg(reinterpret_cast<const float4*>(src + i));
              g0[i] += p0.x; g0[i + 1] += p0.y; g0[i + 2] += p0.z; g0[i + 3] += p0.w;
              if constexpr (NACC == 2) {
                const float4 p1 = __ldcg(reinterpret_cast<const float4*>(src + (size_t)kBM * N + i));
                g1[i] += p1.x; g1[i + 1] += p1.y; g1[i + 2] += p1.z; g1[i + 3] += p1.w;
              }
            }
          }
          finish(gq, g0, g1);
        }
        if (etid == 0) a.done[mt] = 0;        // ready for the next launch
      }
      j0 += len;
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(tmem), "r"(a.tmem_cols) : "memory");
  }
}

// ---------------------------------------------------------------- host side
struct TcPlan {
  int n, mtiles, kblocks, grid, nstages, stage_bytes;
  uint32_t tmem_cols;
  size_t smem, ws_b, ws_rms, ws_part, ws_done, ws_total;
};

TcPlan make_plan(int mode, bool split, int batch, int d_in, int d_out, int num_sms,
                 int smem_optin) {
  TcPlan p{};
  const int nacc = (mode == TC_SWIGLU) ? 2 : 1;
  p.n = ((batch + 15) / 16) * 16;
  p.mtiles = (d_out + kBM - 1) / kBM;
  p.kblocks = (d_in + kBK - 1) / kBK;
  const int64_t U = (int64_t)p.mtiles * p.kblocks;
  p.grid = (int)(U < num_sms ? U : num_sms);
  p.stage_bytes = nacc * kBM * kBK * 2 + (split ? 2 : 1) * p.n * kBK * 2;
  const size_t fixed = 1024 + 256;
  p.nstages = 8;
  while (p.nstages > 2 && fixed + (size_t)p.nstages * p.stage_bytes > (size_t)smem_optin - 1024)
    --p.nstages;
  p.smem = fixed + (size_t)p.nstages * p.stage_bytes;
  uint32_t cols = 32;
  while (cols < (uint32_t)(nacc * p.n)) cols <<= 1;
  p.tmem_cols = cols;
  p.ws_b = split ? (size_t)2 * p.n * d_in * 2 : 0;
  p.ws_rms = (size_t)p.n * sizeof(float);
  p.ws_part = (size_t)2 * num_sms * nacc * kBM * p.n * sizeof(float);
  p.ws_done = (size_t)p.mtiles * sizeof(int);
  p.ws_total = ((p.ws_b + 255) & ~(size_t)255) + ((p.ws_rms + 255) & ~(size_t)255) +
               ((p.ws_part + 255) & ~(size_t)255) + ((p.ws_done + 255) & ~(size_t)255);
  return p;
}

template <typename T, int MODE, bool SPLIT>
int launch_tc(TcArgs& a, const TcPlan& p, cudaStream_t st) {
  auto kern = tc_gemm_kernel<T, MODE, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return (int)e;
  return launch_pdl(reinterpret_cast<const void*>(kern), dim3(p.grid), dim3(kTcThreads), p.smem, st,
                    &a);
}

template <typename T>
int tc_run(int mode, const void* x, const void* gamma, const void* W0, const void* W1,
           const void* residual, void* y, int batch, int d_in, int d_out, float eps, int dtype,
           void* ws, size_t ws_bytes, void* stream) {
  if (batch > kMaxN) return DBK_ESHAPE;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const bool split = (gamma != nullptr);     // x alone is exact in 16 bits
  const TcPlan p = make_plan(mode, split, batch, d_in, d_out, dev.num_sms, dev.max_smem_optin);
  if (p.smem > (size_t)dev.max_smem_optin) return DBK_ESHAPE;
  if (!ws || ws_bytes < p.ws_total) return DBK_EWORKSPACE;
  if (!aligned16(ws)) return DBK_EALIGN;
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto take = [&](size_t n) { uint8_t* r = w; w += (n + 255) & ~(size_t)255; return r; };
  T* b_hi = reinterpret_cast<T*>(take(p.ws_b));
  T* b_lo = b_hi + (size_t)p.n * d_in;
  float* rms = reinterpret_cast<float*>(take(p.ws_rms));
  float* part = reinterpret_cast<float*>(take(p.ws_part));
  int* done = reinterpret_cast<int*>(take(p.ws_done));
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  TcArgs a{};
  a.residual = residual; a.y = y; a.part = part; a.done = done;
  a.inv_rms = split ? rms : nullptr;
  a.batch = batch; a.n = p.n; a.d_in = d_in; a.d_out = d_out;
  a.mtiles = p.mtiles; a.kblocks = p.kblocks; a.nstages = p.nstages; a.stage_bytes = p.stage_bytes;
  a.tmem_cols = p.tmem_cols;
  const uint64_t rs = (uint64_t)d_in * 2;
  if ((rc = encode_tmap_2d(&a.wmap0, W0, dtype, d_in, d_out, rs, kBK, kBM, true))) return rc;
  if (mode == TC_SWIGLU && (rc = encode_tmap_2d(&a.wmap1, W1, dtype, d_in, d_out, rs, kBK, kBM, true)))
    return rc;
  if (split) {
    if ((rc = encode_tmap_2d(&a.bmap, b_hi, dtype, d_in, p.n, rs, kBK, p.n, true))) return rc;
    if ((rc = encode_tmap_2d(&a.bmap_lo, b_lo, dtype, d_in, p.n, rs, kBK, p.n, true))) return rc;
    struct PrepArgs { const T* x; const T* g; T* hi; T* lo; float* rms; int batch, d_in; float eps; };
    // One CTA per B row (rows >= batch are written as zeros).
    void* args[8];
    const T* xx = static_cast<const T*>(x);
    const T* gg = static_cast<const T*>(gamma);
    int bb = batch, dd = d_in;
    float ee = eps;
    args[0] = &xx; args[1] = &gg; args[2] = &b_hi; args[3] = &b_lo; args[4] = &rms;
    args[5] = &bb; args[6] = &dd; args[7] = &ee;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.n);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(tc_prep_kernel<T>), args);
    if (e != cudaSuccess) return (int)e;
  } else {
    if ((rc = encode_tmap_2d(&a.bmap, x, dtype, d_in, batch, rs, kBK, p.n, true))) return rc;
  }
  switch (mode) {
    case TC_PLAIN:
      return split ? launch_tc<T, TC_PLAIN, true>(a, p, st) : launch_tc<T, TC_PLAIN, false>(a, p, st);
    case TC_NORM:
      return launch_tc<T, TC_NORM, true>(a, p, st);
    default:
      return split ? launch_tc<T, TC_SWIGLU, true>(a, p, st) : launch_tc<T, TC_SWIGLU, false>(a, p, st);
  }
}

int tc_dispatch(int mode, const void* x, const void* gamma, const void* W0, const void* W1,
                const void* residual, void* y, int batch, int d_in, int d_out, float eps, int dtype,
                void* ws, size_t ws_bytes, void* stream) {
  if (dtype == DBK_F16)
    return tc_run<__half>(mode, x, gamma, W0, W1, residual, y, batch, d_in, d_out, eps, dtype, ws,
                          ws_bytes, stream);
  if (dtype == DBK_BF16)
    return tc_run<__nv_bfloat16>(mode, x, gamma, W0, W1, residual, y, batch, d_in, d_out, eps,
                                 dtype, ws, ws_bytes, stream);
  return DBK_EDTYPE;
}

}  // namespace
}  // namespace dbk

using namespace dbk;

int dbk_tc_rmsnorm_gemv(const void* x, const void* gamma, const void* W, void* y, int batch,
                        int d_in, int d_out, float eps, int dtype, void* ws, size_t ws_bytes,
                        void* stream) {
  return tc_dispatch(TC_NORM, x, gamma, W, nullptr, nullptr, y, batch, d_in, d_out, eps, dtype, ws,
                     ws_bytes, stream);
}

int dbk_tc_gateup_swiglu(const void* x, const void* gamma, const void* Wg, const void* Wu,
                         void* h, int batch, int d_in, int d_ff, float eps, int dtype, void* ws,
                         size_t ws_bytes, void* stream) {
  return tc_dispatch(TC_SWIGLU, x, gamma, Wg, Wu, nullptr, h, batch, d_in, d_ff, eps, dtype, ws,
                     ws_bytes, stream);
}

int dbk_tc_gemv(const void* x, const void* W, const void* residual, void* y, int batch, int d_in,
                int d_out, int dtype, void* ws, size_t ws_bytes, void* stream) {
  return tc_dispatch(TC_PLAIN, x, nullptr, W, nullptr, residual, y, batch, d_in, d_out, 0.f, dtype,
                     ws, ws_bytes, stream);
}

size_t dbk_tc_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out) {
  if (batch < 1 || batch > kMaxN || d_in < 8 || d_out < 1) return 0;
  DeviceInfo dev;
  int nsm = 148, optin = 232448;
  if (current_device_info(&dev) == DBK_OK) { nsm = dev.num_sms; optin = dev.max_smem_optin; }
  const int mode = op == DBK_OP_GATEUP_SWIGLU ? TC_SWIGLU : op == DBK_OP_RMSNORM_GEMV ? TC_NORM : TC_PLAIN;
  // Sized for the split (gamma) case, which needs the most.
  return make_plan(mode, mode != TC_PLAIN, (int)batch, (int)d_in, (int)d_out, nsm, optin).ws_total;
}

extern "C" size_t dbk_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out) {
  if (batch <= dbk::kSimtMaxBatch) return 0;
  return dbk_tc_workspace_bytes(op, batch, d_in, d_out);
}
