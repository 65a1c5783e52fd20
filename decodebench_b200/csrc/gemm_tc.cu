// gemm_tc.cu - batch 9..256 decode "thin GEMM" on tcgen05 tensor cores.
//
//   y[b, o] = sum_k W[o, k] * x'[b, k]       (W [d_out, d_in] row-major, x' [batch, d_in])
//
// with the same fused epilogues as the CUDA-core GEMV family (gemv.cu):
//   PLAIN  y = W x (+ residual)          NORM  y = inv_rms * W (x * gamma)
//   SWIGLU h = silu(Wg x') * (Wu x')      (x' = x, or RMSNorm(x) when gamma is given)
//
// At batch 16 the Llama-70B MLP (config C4) does 16 flop per weight byte:
// still HBM-bound, but too much work for CUDA cores (~300 us of fp32 FMA vs
// ~210 us of HBM time), so the contraction runs on the 5th-generation tensor
// cores while the kernel stays a weight stream:
//   * D[activation rows x 256 weight rows] += A[128 x 16] * B[256 x 16]^T per
//     16-column k-step: B = a 256-row tile of W, A = the activation rows (R <= 128
//     real rows; the MMA's 128-row A read runs on into the weight tile that
//     follows A in shared memory, and those output lanes are never read). A
//     tcgen05.mma costs ~156 cycles to issue whatever its N (measured), so the
//     weights take the N = 256 side: 8 KB of weights per instruction keeps the
//     single issuing thread ahead of HBM, where a 128-row A-side weight tile
//     (4 KB per instruction) could not keep up. Both operands are K-major,
//     staged by tiled TMA with the 128-byte swizzle and described to
//     tcgen05.mma by shared-memory descriptors; fp32 accumulators live in TMEM
//     (one 256-column accumulator, two for gate and up);
//   * persistent CTAs, one per SM, split the (n-tile, k-block) units evenly
//     ("stream-K"): CTA c owns units [c*U/G, (c+1)*U/G) in tile-major order, so
//     a CTA's range cuts at most two tiles; a tile covered by one CTA is
//     finished in place, otherwise each contributor writes its fp32 partial to
//     the workspace and the last to arrive (self-resetting counter) sums the
//     partials in CTA order (deterministic) and applies the epilogue;
//   * warp roles: warp 0 streams tiles (TMA), warp 1 owns TMEM and issues the
//     MMAs (one elected thread; tcgen05.commit releases smem stages), warps 2-5
//     drain TMEM (tcgen05.ld) and run the epilogue;
//   * activations that are not exact in 16 bits (x * gamma) are written by a
//     small prep kernel as a high and a low bf16/fp16 part, stacked as A rows
//     (hi rows 0..NB-1, lo rows NB..2NB-1) and summed in the epilogue, so the
//     products keep ~16-22 mantissa bits at no extra MMA; the prep kernel also
//     computes inv_rms. Programmatic dependent launch lets the GEMM start
//     streaming weights while the prep kernel (or the previous op) runs.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

enum TcMode : int { TC_PLAIN = 0, TC_NORM = 1, TC_SWIGLU = 2 };

constexpr int kBN = 256;        // weight rows per tile (the MMA N)
constexpr int kBK = 64;         // k-block (one 128-byte swizzle atom of 16-bit values)
constexpr int kTcThreads = 192; // producer, MMA, 4 epilogue warps
constexpr int kMaxRows = 128;   // A rows per pass (hi + lo rows when split)
// Tiles with at most this many contributing CTAs are merged at once by the last
// to arrive; tiles with more are merged by all contributors together at the end.
constexpr int kLocalMerge = 4;

struct TcArgs {
  CUtensorMap wmap0;   // W (or Wg) [d_out, d_in], box [256 rows x 64]
  CUtensorMap wmap1;   // Wu for SWIGLU
  CUtensorMap amap;    // activation rows: x [batch, d_in] or the prep buffer [2 NB, d_in], box [R x 64]
  const void* residual;   // [batch, d_out] or nullptr
  void* y;                // [batch, d_out]
  const float* inv_rms;   // [NB] (NORM / SWIGLU with gamma) or nullptr
  float* part;            // [2 * grid][NACC][batch][256] fp32 partials
  int* done;              // [2][n-tiles] arrival / departure counters (zero between launches)
  int batch, nb, rows;    // batch, its padding to 8 (lo rows start at nb), A rows loaded
  int d_in, d_out;
  int ntiles, kblocks;
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

// Instruction descriptor: kind::f16, fp32 accumulate, A/B K-major, M = 128, N = 256.
__device__ __forceinline__ uint32_t idesc_f16(bool bf16) {
  uint32_t d = 0;
  d |= 1u << 4;                                      // D format f32
  d |= (bf16 ? 1u : 0u) << 7;                        // A format
  d |= (bf16 ? 1u : 0u) << 10;                       // B format
  d |= (uint32_t)(kBN >> 3) << 17;                   // N
  d |= (uint32_t)(128 >> 4) << 24;                   // M
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
// Two 16-column loads (e.g. gate and up accumulators) with one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float (&va)[16],
                                            float (&vb)[16]) {
  uint32_t r[16], q[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(ta));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]), "=r"(q[6]),
        "=r"(q[7]), "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]),
        "=r"(q[14]), "=r"(q[15])
      : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) { va[i] = __uint_as_float(r[i]); vb[i] = __uint_as_float(q[i]); }
}

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
  // b_hi: rows 0..N-1 of the B buffer; b_lo = b_hi + N * d_in (rows N..2N-1).
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
  constexpr int NACC = (MODE == TC_SWIGLU) ? 2 : 1;   // output accumulators (gate, up)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.nstages * a.stage_bytes);
  uint64_t* empty = full + a.nstages;
  uint64_t* acc_full = empty + a.nstages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* teardown = acc_empty + 1;
  uint64_t* mrg_bar = teardown + 1;            // merge copies (the ring is idle by then)
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_bail;
  __shared__ int s_last;
  __shared__ float xbuf[kMaxRows / 2][17];    // lo-row exchange (split)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  DBK_TRACE_BEGIN();
  DBK_MARK(tid == 0, 0);
  const int a_bytes = a.rows * 128;            // A rows of one k-block
  const int w_bytes = kBN * 128;               // 32 KB weight tile of one k-block

  const int64_t U = (int64_t)a.ntiles * a.kblocks;
  const int G = (int)min((int64_t)gridDim.x, U);
  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(teardown, kTcThreads / 32);
    mbar_init(mrg_bar, 1);
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
  DBK_MARK(tid == 0, 13);
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
      // stages' weights before waiting for it, their activation rows after.
      const int pre = min(a.nstages, u1 - u0);
      for (int j = 0; j < pre; ++j) {
        const int u = u0 + j, nt = u / a.kblocks, kb = u - nt * a.kblocks;
        uint8_t* st = smem + (size_t)j * a.stage_bytes;
        mbar_arrive_expect_tx(&full[j], (uint32_t)(a_bytes + NACC * w_bytes));
        tma_load_2d(st + a_bytes, &a.wmap0, kb * kBK, nt * kBN, &full[j], pol_w);
        if constexpr (NACC == 2)
          tma_load_2d(st + a_bytes + w_bytes, &a.wmap1, kb * kBK, nt * kBN, &full[j], pol_w);
      }
      DBK_MARK(true, 1);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      DBK_MARK(true, 2);
      for (int j = 0; j < pre; ++j) {
        const int kb = (u0 + j) % a.kblocks;
        tma_load_2d(smem + (size_t)j * a.stage_bytes, &a.amap, kb * kBK, 0, &full[j], pol_x);
      }
      for (int j = pre; j < u1 - u0; ++j) {
        const int s = j % a.nstages;
        if (!mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty)) { s_bail = 1; break; }
        const int u = u0 + j, nt = u / a.kblocks, kb = u - nt * a.kblocks;
        uint8_t* st = smem + (size_t)s * a.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(a_bytes + NACC * w_bytes));
        tma_load_2d(st, &a.amap, kb * kBK, 0, &full[s], pol_x);
        tma_load_2d(st + a_bytes, &a.wmap0, kb * kBK, nt * kBN, &full[s], pol_w);
        if constexpr (NACC == 2)
          tma_load_2d(st + a_bytes + w_bytes, &a.wmap1, kb * kBK, nt * kBN, &full[s], pol_w);
      }
      DBK_MARK(true, 3);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (active) {
      const uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value);
      int seg = 0;
      bool first = true;
      for (int j = 0; j < u1 - u0 && !s_bail; ++j) {
        const int u = u0 + j, kb = u % a.kblocks;
        const int s = j % a.nstages;
        if (first && seg > 0) {
          // the epilogue must have drained the previous segment's accumulators
          if (!mbar_wait(acc_empty, (seg - 1) & 1, kDevTimeoutMma)) { s_bail = 1; break; }
          tc_fence_after();
        }
        if (!mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull)) { s_bail = 1; break; }
        tc_fence_after();
        DBK_MARK(lane == 0 && j == 0, 4);
        DBK_MARK(lane == 0 && j == 32, 9);
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + (size_t)s * a.stage_bytes);
          const uint64_t da0 = sw128_desc(st);
          const uint64_t dw0 = sw128_desc(st + a_bytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
#pragma unroll
            for (int acc = 0; acc < NACC; ++acc)
              umma(tmem + acc * kBN, da0 + (uint64_t)(k * 2),
                   dw0 + (uint64_t)((acc * w_bytes + k * 32) >> 4), idesc,
                   (first && k == 0) ? 0u : 1u);
          }
          umma_commit(&empty[s]);           // stage free once these MMAs have read it
        }
        __syncwarp();
        first = false;
        const bool seg_end = (kb == a.kblocks - 1) || (j == u1 - u0 - 1);
        if (seg_end) {
          DBK_MARK(lane == 0, seg == 0 ? 5 : 10);
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
    const int r = quarter * 32 + lane;            // A row = activation row of this thread
    const int etid = tid - 64;                    // 0..127
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    T* y = static_cast<T*>(a.y);
    const T* res = static_cast<const T*>(a.residual);
    const bool owner_row = r < a.batch;           // holds (the hi part of) batch row r
    // D columns gq*16 .. +15 of accumulator acc, hi + lo summed on the owner rows.
    auto gather = [&](int acc, int gq, float (&v)[16]) {
      tmem_ld16(trow + acc * kBN + gq * 16, v);
      if constexpr (SPLIT) {
        if (a.nb <= 16) {
          // hi row r and lo row r + nb are lanes of the same warp (TMEM lanes 0..31)
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += __shfl_down_sync(0xffffffffu, v[i], a.nb);
          return;
        }
        if (r >= a.nb && r < a.nb + a.batch)
#pragma unroll
          for (int i = 0; i < 16; ++i) xbuf[r - a.nb][i] = v[i];
        named_bar_sync(1, 128);
        if (owner_row)
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += xbuf[r][i];
        named_bar_sync(1, 128);
      }
    };
    // Both accumulators of columns gq*16 .. +15 (one TMEM wait), hi + lo summed.
    auto gather2 = [&](int gq, float (&v0)[16], float (&v1)[16]) {
      if (SPLIT && a.nb > 16) {
        gather(0, gq, v0);
        gather(1, gq, v1);
        return;
      }
      tmem_ld16x2(trow + gq * 16, trow + kBN + gq * 16, v0, v1);
      if constexpr (SPLIT) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v0[i] += __shfl_down_sync(0xffffffffu, v0[i], a.nb);
          v1[i] += __shfl_down_sync(0xffffffffu, v1[i], a.nb);
        }
      }
    };
    // Epilogue of batch row b, weight rows col0 + gq*16 .. +15.
    auto finish_row = [&](int col0, int b, int gq, const float (&g0)[16], const float (&g1)[16]) {
      const float scb = a.inv_rms ? a.inv_rms[b] : 1.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = col0 + gq * 16 + i;
        if (c >= a.d_out) break;
        float val;
        if constexpr (MODE == TC_SWIGLU) val = silu(g0[i] * scb) * (g1[i] * scb);
        else if constexpr (MODE == TC_NORM) val = g0[i] * scb;
        else val = g0[i];
        const size_t o = (size_t)b * a.d_out + c;
        if (res != nullptr) val += Elem<T>::to_f(res[o]);
        y[o] = Elem<T>::from_f(val);
      }
    };
    int pend[2];                                  // partial tiles of this CTA (<= 2)
    int npend = 0;
    uint32_t mphase = 0;                          // parity of mrg_bar
    int seg = 0;
    for (int j0 = 0; active && j0 < u1 - u0 && !s_bail;) {
      const int u = u0 + j0, nt = u / a.kblocks, kb0 = u - nt * a.kblocks;
      const int len = min(a.kblocks - kb0, u1 - u);       // units of this segment
      if (!mbar_wait(acc_full, seg & 1, kDevTimeoutMma)) { s_bail = 1; break; }
      tc_fence_after();
      DBK_MARK(etid == 0, seg == 0 ? 6 : 11);
      const bool whole = (kb0 == 0) && (len == a.kblocks);
      const int col0 = nt * kBN;
      auto finish = [&](int gq, const float (&g0)[16], const float (&g1)[16]) {
        if (owner_row) finish_row(col0, r, gq, g0, g1);
      };

      if (whole) {
        for (int gq = 0; gq < kBN / 16; ++gq) {
          float g0[16], g1[16];
          if constexpr (NACC == 2) gather2(gq, g0, g1);
          else gather(0, gq, g0);
          finish(gq, g0, g1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);   // one arrival per epilogue warp
        j0 += len;
        ++seg;
        continue;
      }
      // Partial tile: publish this CTA's fp32 partial; the last contributor merges.
      const int slot = 2 * blockIdx.x + (u == u0 ? 0 : 1);
      for (int gq = 0; gq < kBN / 16; ++gq) {
        float gv[NACC][16];
        if constexpr (NACC == 2) gather2(gq, gv[0], gv[1]);
        else gather(0, gq, gv[0]);
        if (owner_row) {
#pragma unroll
          for (int acc = 0; acc < NACC; ++acc) {
            float* dst = a.part + (((size_t)slot * NACC + acc) * a.batch + r) * kBN + gq * 16;
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(dst + i) =
                  make_float4(gv[acc][i], gv[acc][i + 1], gv[acc][i + 2], gv[acc][i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      __threadfence();
      named_bar_sync(1, 128);
      const int first_u = nt * a.kblocks, last_u = first_u + a.kblocks - 1;
      const int c_first = owner(first_u, U, G), c_last = owner(last_u, U, G);
      if (c_last - c_first + 1 > kLocalMerge) {
        // Arrive at once; the merge runs after the last segment (an arrival never
        // waits on a merge, so no CTA waits on a chain of its neighbours).
        if (etid == 0) atomicAdd(&a.done[nt], 1);
        if (npend < 2) pend[npend++] = nt;
        j0 += len;
        ++seg;
        continue;
      }
      // Few contributors: the last to arrive merges the whole tile now.
      if (etid == 0) s_last = (atomicAdd(&a.done[nt], 1) == c_last - c_first);
      named_bar_sync(1, 128);
      const bool last = s_last != 0;
      named_bar_sync(1, 128);                   // s_last is rewritten by the next segment
      if (last) {
        __threadfence();
        for (int it = etid; it < a.batch * (kBN / 16); it += 128) {
          const int b = it / (kBN / 16), gq = it - b * (kBN / 16);
          float g0[16], g1[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) g0[i] = g1[i] = 0.f;
          for (int c = c_first; c <= c_last; ++c) {
            const int sl = 2 * c + (range_start(c, U, G) >= first_u ? 0 : 1);
#pragma unroll
            for (int acc = 0; acc < NACC; ++acc) {
              const float4* src = reinterpret_cast<const float4*>(
                  a.part + (((size_t)sl * NACC + acc) * a.batch + b) * kBN + gq * 16);
              float4 p4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) p4[i] = __ldcg(src + i);
              float* g = acc ? g1 : g0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                g[4 * i] += p4[i].x; g[4 * i + 1] += p4[i].y;
                g[4 * i + 2] += p4[i].z; g[4 * i + 3] += p4[i].w;
              }
            }
          }
          finish_row(col0, b, gq, g0, g1);
        }
        if (etid == 0) a.done[nt] = 0;        // ready for the next launch
      }
      j0 += len;
      ++seg;
    }
    // Merges of the partial tiles: every contributor waits (bounded) until all
    // contributors have arrived, then merges its own slice of the tile's outputs,
    // so the merge's reads are spread over all contributing SMs instead of one.
    // Arrivals happen above, before any wait, so every wait ends once the
    // contributors' MMAs are done.
    for (int pi = 0; pi < npend && !s_bail; ++pi) {
      const int nt = pend[pi];
      const int first_u = nt * a.kblocks, last_u = first_u + a.kblocks - 1;
      const int c_first = owner(first_u, U, G), c_last = owner(last_u, U, G);
      const int ncon = c_last - c_first + 1, me = (int)blockIdx.x - c_first;
      if (etid == 0) {
        uint32_t n = 0;
        while (ld_acquire_gpu(&a.done[nt]) < ncon) {
          if (++n >= spin_limit()) { record_error(kDevTimeoutMerge); break; }
          __nanosleep(64);
        }
      }
      named_bar_sync(1, 128);
      DBK_MARK(etid == 0 && pi == 0, 14);
      const int total = a.batch * (kBN / 16);                    // items (batch row, 16 cols)
      const int i0 = (int)((int64_t)me * total / ncon), i1 = (int)((int64_t)(me + 1) * total / ncon);
      const int col0 = nt * kBN;
      // This CTA's items are contiguous in every contributor's partial, so one bulk
      // copy per (contributor, accumulator) brings them into the idle ring: all
      // copies are in flight at once. Rounds bound the ring bytes used.
      const size_t ring = (size_t)a.nstages * a.stage_bytes;
      const int per_item = 64 * NACC * (ncon + 1);               // copies + sums
      const int R = max(1, min(i1 - i0, (int)(ring / per_item)));
      for (int ib = i0; ib < i1; ib += R) {
        const int ni = min(R, i1 - ib);
        const uint32_t piece = (uint32_t)ni * 64;                // bytes per copy
        float* cp = reinterpret_cast<float*>(smem);              // [ncon][NACC][ni][16]
        float* sm = cp + (size_t)ncon * NACC * ni * 16;          // [ni][NACC][16]
        if (etid < 32) {
          if (etid == 0) mbar_arrive_expect_tx(mrg_bar, piece * (uint32_t)(ncon * NACC));
          __syncwarp();
          asm volatile("fence.proxy.async.global;" ::: "memory");   // peers' generic stores
          const uint64_t pol = policy_evict_first();
          for (int w = etid; w < ncon * NACC; w += 32) {
            const int c = c_first + w / NACC, acc = w % NACC;
            const int sl = 2 * c + (range_start(c, U, G) >= first_u ? 0 : 1);
            bulk_g2s(cp + (size_t)w * ni * 16,
                     a.part + ((size_t)sl * NACC + acc) * a.batch * kBN + (size_t)ib * 16,
                     piece, mrg_bar, pol);
          }
        }
        if (!mbar_wait(mrg_bar, mphase, kDevTimeoutMerge)) { s_bail = 1; break; }
        mphase ^= 1;
        // sums in contributor order (deterministic)
        for (int w = etid; w < ni * NACC * 16; w += 128) {
          const int it = w / (NACC * 16), acc = (w / 16) % NACC, f = w & 15;
          float t = 0.f;
          for (int c = 0; c < ncon; ++c) t += cp[((size_t)(c * NACC + acc) * ni + it) * 16 + f];
          sm[(it * NACC + acc) * 16 + f] = t;
        }
        named_bar_sync(1, 128);
        DBK_MARK(etid == 0 && pi == 0 && ib == i0, 15);
        for (int it = etid; it < ni; it += 128) {
          const int item = ib + it, b = item / (kBN / 16), gq = item - b * (kBN / 16);
          float g0[16], g1[16];
#pragma unroll
          for (int f = 0; f < 16; ++f) {
            g0[f] = sm[(it * NACC + 0) * 16 + f];
            g1[f] = (NACC == 2) ? sm[(it * NACC + (NACC - 1)) * 16 + f] : 0.f;
          }
          finish_row(col0, b, gq, g0, g1);
        }
        named_bar_sync(1, 128);                   // the ring is rewritten by the next batch of items
      }
      // Departure: the last contributor to leave resets both counters for the next
      // launch (which touches them only after its griddepcontrol.wait).
      if (etid == 0) {
        __threadfence();
        if (atomicAdd(&a.done[a.ntiles + nt], 1) == ncon - 1) {
          a.done[nt] = 0;
          a.done[a.ntiles + nt] = 0;
        }
      }
    }
  }
  DBK_MARK(tid == 64, 7);
  // Teardown: each warp arrives once, converged, on an mbarrier; warp 1 waits
  // for all six and then frees TMEM. (A CTA-wide bar.sync after this
  // warp-specialised, divergent code let warps pass before the epilogue had
  // finished, and the TMEM release then stalled.)
  __syncwarp();
  tc_fence_before();
  if (lane == 0) mbar_arrive(teardown);
  if (warp == 1) {
    mbar_wait(teardown, 0, kDevTimeoutDrain);
    tc_fence_after();
    DBK_MARK(lane == 0, 8);
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(tmem), "r"(a.tmem_cols) : "memory");
    DBK_MARK(lane == 0, 12);
  }
}

// ---------------------------------------------------------------- host side
struct TcPlan {
  int nb, rows, ntiles, kblocks, grid, nstages, stage_bytes;
  uint32_t tmem_cols;
  size_t smem, ws_b, ws_rms, ws_part, ws_done, ws_total;
};

// One pass handles up to kMaxRows A rows: batch <= 128, or <= 64 with a hi/lo split.
int pass_batch(bool split) { return split ? kMaxRows / 2 : kMaxRows; }

TcPlan make_plan(int mode, bool split, int batch, int d_in, int d_out, int num_sms,
                 int smem_optin) {
  TcPlan p{};
  const int nacc = (mode == TC_SWIGLU) ? 2 : 1;
  p.nb = ((batch + 7) / 8) * 8;
  p.rows = split ? 2 * p.nb : p.nb;
  p.ntiles = (d_out + kBN - 1) / kBN;
  p.kblocks = (d_in + kBK - 1) / kBK;
  const int64_t U = (int64_t)p.ntiles * p.kblocks;
  p.grid = (int)(U < num_sms ? U : num_sms);
  p.stage_bytes = p.rows * 128 + nacc * kBN * 128;
  static const int env_st = [] { const char* v = std::getenv("DBK_TC_STAGES"); return v ? std::atoi(v) : 12; }();
  const size_t fixed = 1024 + 512;
  p.nstages = env_st < 2 ? 2 : (env_st > 12 ? 12 : env_st);
  while (p.nstages > 2 && fixed + (size_t)p.nstages * p.stage_bytes > (size_t)smem_optin - 6144)
    --p.nstages;
  p.smem = fixed + (size_t)p.nstages * p.stage_bytes;
  p.tmem_cols = (uint32_t)(nacc * kBN);
  p.ws_b = split ? (size_t)2 * p.nb * d_in * 2 : 0;
  p.ws_rms = (size_t)p.nb * sizeof(float);
  p.ws_part = (size_t)2 * num_sms * nacc * batch * kBN * sizeof(float);
  p.ws_done = (size_t)2 * p.ntiles * sizeof(int);
  p.ws_total = ((p.ws_b + 255) & ~(size_t)255) + ((p.ws_rms + 255) & ~(size_t)255) +
               ((p.ws_part + 255) & ~(size_t)255) + ((p.ws_done + 255) & ~(size_t)255);
  return p;
}

template <typename T, int MODE, bool SPLIT>
int launch_tc(TcArgs& a, const TcPlan& p, cudaStream_t st, const DeviceInfo& dev) {
  auto kern = tc_gemm_kernel<T, MODE, SPLIT>;
  if (int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kern), dev, p.smem)) return rc;
  return launch_pdl(reinterpret_cast<const void*>(kern), dim3(p.grid), dim3(kTcThreads), p.smem, st,
                    &a);
}

// One pass: batch <= pass_batch(split).
template <typename T>
int tc_pass(int mode, const void* x, const void* gamma, const void* W0, const void* W1,
            const void* residual, void* y, int batch, int d_in, int d_out, float eps, int dtype,
            void* ws, size_t ws_bytes, cudaStream_t st, const DeviceInfo& dev) {
  const bool split = (gamma != nullptr);     // x alone is exact in 16 bits
  const TcPlan p = make_plan(mode, split, batch, d_in, d_out, dev.num_sms, dev.max_smem_optin);
  if (p.smem > (size_t)dev.max_smem_optin) return DBK_ESHAPE;
  if (!ws || ws_bytes < p.ws_total) return DBK_EWORKSPACE;
  if (!aligned16(ws)) return DBK_EALIGN;
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto take = [&](size_t n) { uint8_t* r = w; w += (n + 255) & ~(size_t)255; return r; };
  T* b_hi = reinterpret_cast<T*>(take(p.ws_b));
  T* b_lo = b_hi + (size_t)p.nb * d_in;
  float* rms = reinterpret_cast<float*>(take(p.ws_rms));
  float* part = reinterpret_cast<float*>(take(p.ws_part));
  int* done = reinterpret_cast<int*>(take(p.ws_done));

  TcArgs a{};
  a.residual = residual; a.y = y; a.part = part; a.done = done;
  a.inv_rms = split ? rms : nullptr;
  a.batch = batch; a.nb = p.nb; a.rows = p.rows; a.d_in = d_in; a.d_out = d_out;
  a.ntiles = p.ntiles; a.kblocks = p.kblocks; a.nstages = p.nstages; a.stage_bytes = p.stage_bytes;
  a.tmem_cols = p.tmem_cols;
  const uint64_t rs = (uint64_t)d_in * 2;
  int rc;
  if ((rc = encode_tmap_2d(&a.wmap0, W0, dtype, d_in, d_out, rs, kBK, kBN, true))) return rc;
  if (mode == TC_SWIGLU && (rc = encode_tmap_2d(&a.wmap1, W1, dtype, d_in, d_out, rs, kBK, kBN, true)))
    return rc;
  if (split) {
    if ((rc = encode_tmap_2d(&a.amap, b_hi, dtype, d_in, p.rows, rs, kBK, p.rows, true))) return rc;
    void* args[8];
    const T* xx = static_cast<const T*>(x);
    const T* gg = static_cast<const T*>(gamma);
    int bb = batch, dd = d_in;
    float ee = eps;
    args[0] = &xx; args[1] = &gg; args[2] = &b_hi; args[3] = &b_lo; args[4] = &rms;
    args[5] = &bb; args[6] = &dd; args[7] = &ee;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p.nb);                 // one CTA per hi row (rows >= batch: zeros)
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
    if ((rc = encode_tmap_2d(&a.amap, x, dtype, d_in, batch, rs, kBK, p.rows, true))) return rc;
  }
  switch (mode) {
    case TC_PLAIN:
      return split ? launch_tc<T, TC_PLAIN, true>(a, p, st, dev) : launch_tc<T, TC_PLAIN, false>(a, p, st, dev);
    case TC_NORM:
      return launch_tc<T, TC_NORM, true>(a, p, st, dev);
    default:
      return split ? launch_tc<T, TC_SWIGLU, true>(a, p, st, dev) : launch_tc<T, TC_SWIGLU, false>(a, p, st, dev);
  }
}

// Batches beyond one pass run as consecutive passes over row slices of x / y.
template <typename T>
int tc_run(int mode, const void* x, const void* gamma, const void* W0, const void* W1,
           const void* residual, void* y, int batch, int d_in, int d_out, float eps, int dtype,
           void* ws, size_t ws_bytes, void* stream) {
  if (batch > 256) return DBK_ESHAPE;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const int pb = pass_batch(gamma != nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < batch; b0 += pb) {
    const int nb = batch - b0 < pb ? batch - b0 : pb;
    const T* xs = static_cast<const T*>(x) + (size_t)b0 * d_in;
    const T* rsd = residual ? static_cast<const T*>(residual) + (size_t)b0 * d_out : nullptr;
    T* ys = static_cast<T*>(y) + (size_t)b0 * d_out;
    rc = tc_pass<T>(mode, xs, gamma, W0, W1, rsd, ys, nb, d_in, d_out, eps, dtype, ws, ws_bytes, st,
                    dev);
    if (rc) return rc;
  }
  return DBK_OK;
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
  if (batch < 1 || batch > 256 || d_in < 8 || d_out < 1) return 0;
  DeviceInfo dev;
  int nsm = 148, optin = 232448;
  if (current_device_info(&dev) == DBK_OK) { nsm = dev.num_sms; optin = dev.max_smem_optin; }
  const int mode = op == DBK_OP_GATEUP_SWIGLU ? TC_SWIGLU : op == DBK_OP_RMSNORM_GEMV ? TC_NORM : TC_PLAIN;
  // Sized for one pass of the split (gamma) case, which needs the most.
  const bool split = mode != TC_PLAIN;
  const int pb = (int)(batch < pass_batch(split) ? batch : pass_batch(split));
  const size_t a = make_plan(mode, split, pb, (int)d_in, (int)d_out, nsm, optin).ws_total;
  const size_t b = make_plan(mode, false, (int)(batch < pass_batch(false) ? batch : pass_batch(false)),
                             (int)d_in, (int)d_out, nsm, optin).ws_total;
  return a > b ? a : b;
}

extern "C" size_t dbk_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out) {
  if (batch <= dbk::kSimtMaxBatch) return 0;
  return dbk_tc_workspace_bytes(op, batch, d_in, d_out);
}
