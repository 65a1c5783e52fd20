// gemv.cu - batch-1..8 decode GEMV family on CUDA cores, weights streamed by TMA.
//
// One kernel template serves three fused operations:
//   MODE_PLAIN    y = W x (+ residual)                       (down projection)
//   MODE_NORM     y = inv_rms * W (x * gamma)                 (F1: RMSNorm -> GEMV)
//   MODE_SWIGLU   h = silu(Wg x') * (Wu x'), x' = x or the    (F2: gate+up -> SwiGLU)
//                 RMSNorm of x when gamma is given
//   MODE_QKV      qkv = Wqkv x' with RoPE on q and k; q to     (QKV + RoPE + paged-KV append;
//                 q_out, k and v into the paged cache          tensor-core variant only)
//
// Design (B200): the op is a pure HBM stream of W (2 bytes per weight, 1..8 FMAs
// per weight), so the kernel is built to keep ~190 KB of weight bytes in flight
// per SM from the first cycle:
//   * one persistent CTA per SM owns a contiguous block of output rows;
//   * a producer warp walks the CTA's weight rows in K-chunks and issues one
//     cp.async.bulk (TMA, non-tensor) per (row, chunk) segment into a ring of
//     32 KB shared-memory stages tracked by mbarriers (L2 evict-first policy);
//   * eight consumer warps each own the weight rows i = w (mod 8) of the CTA, so
//     per-row accumulation order is fixed (deterministic results); a lane keeps
//     the activation chunk it needs in registers (x*gamma in fp32), reads 16-byte
//     vectors of W from shared memory, and a warp reduction adds each segment's
//     partial dot to the row's fp32 accumulator in shared memory;
//   * RMSNorm is not a separate pass: inv_rms is a per-batch-row scalar, so
//     W (x * gamma * inv_rms) = inv_rms * W (x * gamma); the consumers compute
//     sum(x^2) while the producer's first copies are in flight and apply
//     inv_rms in the epilogue, where SwiGLU and the residual add are fused too.
//   * programmatic dependent launch: the weight stream starts before
//     griddepcontrol.wait; activations are read and outputs written after it.
//
// Reference semantics: fused f1_kernel / f2_kernel
// (validation/src/kernels/fused/f1.cu:18-84, f2.cu:17-76) and the Python stages
// (src/decodebench/demos/llama_decode.py:36-43, :77-87): fp32 accumulation,
// silu(g) = g / (1 + exp(-g)) (f2.cu:73), output rounded once to fp16/bf16.
#include <cstdlib>
#include <type_traits>

#include "comm.cuh"
#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

enum GemvMode : int { MODE_PLAIN = 0, MODE_NORM = 1, MODE_SWIGLU = 2, MODE_QKV = 3 };

// MODE_QKV operands (rows of Wqkv: the q heads, then the k heads, then the v
// heads, head_dim rows each; inside a q or k head, row 2i holds dim i and row
// 2i + 1 holds dim i + head_dim/2, so a RoPE pair is two adjacent rows).
struct QkvArgs {
  const int* pos;          // [batch] position of the new token (= cache slot)
  const float* inv_freq;   // [head_dim / 2] rotary frequencies
  void* q_out;             // [batch, hq, head_dim]
  void* k_cache;           // [pages, hkv, page_size, head_dim] (or [batch, hkv, max_len, head_dim])
  void* v_cache;
  const int* page_table;   // [batch, max_pages] or nullptr (contiguous cache)
  int hq, hkv, head_dim, page_size, max_pages;
};

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;   // + one producer warp
constexpr int kStageBytes = 32 * 1024;
constexpr int kMaxStages = 6;

struct GemvArgs {
  const void* x;         // [batch, d_in]
  const void* gamma;     // [d_in] or nullptr
  const void* w0;        // [d_out, d_in]   (W, or Wg)
  const void* w1;        // [d_out, d_in]   (Wu) for MODE_SWIGLU
  const void* residual;  // [batch, d_out] or nullptr
  void* y;               // [batch, d_out]
  int batch, d_in, d_out;
  float eps;
  int kc;                // columns per (row, chunk) segment
  int nchunks;           // ceil(d_in / kc)
  int slots;             // segments per stage (multiple of 8)
  int nstages;           // ring depth
  int max_rows;          // max output rows of any CTA
  int pcols;             // tensor-core variant: B columns in use (batch, or 2 * batch packed)
  long long y_ld;        // row stride of y and residual (elements)
  long long y_col0;      // column of y (and residual) where this op's rows start
  PeerSet ps;            // ps.world > 1: all-gather the output over the peers (fused)
  QkvArgs qkv;           // MODE_QKV
  const float* wscale0;  // fp8 weights: per-row scale of w0 (and of w1); nullptr for 16-bit W
  const float* wscale1;
};

// Shared-memory carve-up (dynamic): ring | full[] | empty[] | acc | inv_rms
struct Smem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  float* acc;      // [max_rows * nmat][NB]
  float* inv_rms;  // [NB]
};

__device__ __forceinline__ Smem carve(uint8_t* base, const GemvArgs& a, int nmat, int nb) {
  Smem s;
  s.ring = base;
  s.full = reinterpret_cast<uint64_t*>(base + (size_t)a.nstages * kStageBytes);
  s.empty = s.full + a.nstages;
  s.acc = reinterpret_cast<float*>(s.empty + a.nstages);
  s.inv_rms = s.acc + (size_t)a.max_rows * nmat * nb;
  return s;
}

template <typename T, int NB, int MODE, int KCG>
__global__ void __launch_bounds__(kThreads, 1) gemv_stream_kernel(const GemvArgs a) {
  constexpr int NMAT = (MODE == MODE_SWIGLU) ? 2 : 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem sm = carve(smem_raw, a, NMAT, NB);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int row0 = (int)(((int64_t)blockIdx.x * a.d_out) / G);
  const int row1 = (int)(((int64_t)(blockIdx.x + 1) * a.d_out) / G);
  const int nrows = row1 - row0;
  const int nwr = nrows * NMAT;                       // weight rows of this CTA
  const int spc = (nwr + a.slots - 1) / a.slots;      // stages per chunk
  const int total = spc * a.nchunks;
  const int slot_bytes = a.kc * (int)sizeof(T);

  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Let the next kernel in the stream start its own weight stream early.
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const T* W[2] = {static_cast<const T*>(a.w0), static_cast<const T*>(a.w1)};
      for (int j = 0; j < total; ++j) {
        const int s = j % a.nstages;
        if (j >= a.nstages &&
            !mbar_wait(&sm.empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty))
          return;
        const int k = j / spc;
        const int i0 = (j % spc) * a.slots;
        const int n = min(a.slots, nwr - i0);
        const int col0 = k * a.kc;
        const int seg = min(a.kc, a.d_in - col0);
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(n * seg * sizeof(T)));
        uint8_t* dst = sm.ring + (size_t)s * kStageBytes;
        for (int q = 0; q < n; ++q) {
          const int i = i0 + q;
          const int r = row0 + i / NMAT;
          const T* src = W[i % NMAT] + (size_t)r * a.d_in + col0;
          bulk_g2s(dst + q * slot_bytes, src, (uint32_t)(seg * sizeof(T)), &sm.full[s], pol);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Activations may be produced by the previous kernel in the stream.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const T* x = static_cast<const T*>(a.x);
  const T* gam = static_cast<const T*>(a.gamma);

  for (int idx = tid; idx < a.max_rows * NMAT * NB; idx += kConsumers) sm.acc[idx] = 0.f;
  if constexpr (MODE != MODE_PLAIN) {
    if (gam != nullptr) {
      // sum(x^2) per batch row: every CTA recomputes it (x is a few KB, L2-resident).
      __shared__ float red[kConsumerWarps][NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float ss = 0.f;
        if (b < a.batch) {
          for (int c = tid * 8; c < a.d_in; c += kConsumers * 8) {
            float f[8];
            unpack8<T>(ldg_nc_v4(x + (size_t)b * a.d_in + c), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp][b] = ss;
      }
      named_bar_sync(1, kConsumers);
      if (tid < NB) {
        float ss = 0.f;
        for (int w = 0; w < kConsumerWarps; ++w) ss += red[w][tid];
        sm.inv_rms[tid] = rsqrtf(ss / (float)a.d_in + a.eps);
      }
    } else if (tid < NB) {
      sm.inv_rms[tid] = 1.f;
    }
  }
  named_bar_sync(1, kConsumers);

  float xr[NB][KCG][8];
  int cur_k = -1;
  for (int j = 0; j < total; ++j) {
    const int s = j % a.nstages;
    const int k = j / spc;
    const int i0 = (j % spc) * a.slots;
    const int n = min(a.slots, nwr - i0);
    const int col0 = k * a.kc;
    const int seg = min(a.kc, a.d_in - col0);
    if (k != cur_k) {   // new K-chunk: load x (* gamma) for this lane's columns
      cur_k = k;
#pragma unroll
      for (int g = 0; g < KCG; ++g) {
        const int c = (lane + 32 * g) * 8;
        float gm[8];
        if (gam != nullptr && c < seg) unpack8<T>(ldg_nc_v4(gam + col0 + c), gm);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < a.batch && c < seg) {
            unpack8<T>(ldg_nc_v4(x + (size_t)b * a.d_in + col0 + c), xr[b][g]);
            if (gam != nullptr) {
#pragma unroll
              for (int e = 0; e < 8; ++e) xr[b][g][e] *= gm[e];
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) xr[b][g][e] = 0.f;
          }
        }
      }
    }
    if (!mbar_wait(&sm.full[s], (j / a.nstages) & 1, kDevTimeoutFull)) return;
    const uint32_t stage = smem_u32(sm.ring + (size_t)s * kStageBytes);
    for (int q = warp; q < n; q += kConsumerWarps) {
      float part[NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) part[b] = 0.f;
#pragma unroll
      for (int g = 0; g < KCG; ++g) {
        const int c = (lane + 32 * g) * 8;
        if (c < seg) {
          float wf[8];
          unpack8<T>(ld_shared_v4(stage + q * slot_bytes + c * (int)sizeof(T)), wf);
#pragma unroll
          for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int e = 0; e < 8; ++e) part[b] = fmaf(wf[e], xr[b][g][e], part[b]);
        }
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) part[b] = warp_sum(part[b]);
      if (lane == 0) {
        float* acc = sm.acc + (size_t)(i0 + q) * NB;
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] += part[b];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }

  named_bar_sync(1, kConsumers);
  T* y = static_cast<T*>(a.y);
  const T* res = static_cast<const T*>(a.residual);
  for (int idx = tid; idx < nrows * NB; idx += kConsumers) {
    const int b = idx / nrows, r = idx - b * nrows;
    if (b >= a.batch) break;
    float v;
    if constexpr (MODE == MODE_SWIGLU) {
      const float sc = (gam != nullptr) ? sm.inv_rms[b] : 1.f;
      const float gt = sm.acc[(size_t)(2 * r) * NB + b] * sc;
      const float up = sm.acc[(size_t)(2 * r + 1) * NB + b] * sc;
      v = silu(gt) * up;
    } else if constexpr (MODE == MODE_NORM) {
      v = sm.acc[(size_t)r * NB + b] * sm.inv_rms[b];
    } else {
      v = sm.acc[(size_t)r * NB + b];
    }
    const size_t o = (size_t)b * a.y_ld + a.y_col0 + row0 + r;
    if (res != nullptr) v += Elem<T>::to_f(res[o]);
    y[o] = Elem<T>::from_f(v);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core variant (d_in % 16 == 0, activations fit in shared memory).
//
// On CUDA cores the stream above is issue-bound on 16-bit -> fp32 conversions
// (16K per 32 KB stage at quarter rate). Here the weights go from shared memory
// straight into mma.m16n8k16 (fp32 accumulation) through ldmatrix, so no
// per-weight conversion or FMA is issued:
//   * a stage is one m-tile of 16 weight rows x KC = 2048 columns; each row
//     segment (4 KB) is one cp.async.bulk into a slot padded to 4112 bytes, so
//     the 8 rows of an ldmatrix 8x8 block fall in 8 different bank groups.
//     Segments of 4 KB or more keep DRAM near its streaming rate when they come
//     from different rows; 2 KB segments measured ~30% slower;
//   * warp w owns columns [256 w, 256 w + 256) of every stage (16 k-steps); its
//     fp32 partial of the m-tile stays in the mma accumulator across the K
//     chunks and is written once per m-tile to a per-warp buffer; the epilogue
//     sums the 8 warp partials in a fixed order (deterministic);
//   * the activation is the B operand (N = 8 columns = the batch, up to 8):
//     x * gamma is staged in shared memory as a high and a low 16-bit part and
//     both are multiplied, so x * gamma keeps ~22 (fp16) / ~16 (bf16) bits.
//     For batch <= 4 the two parts sit in different B columns of the same mma
//     (columns b and batch + b), so the split costs no extra tensor-core work;
//     the epilogue adds the two columns. For batch 5..8 a second mma multiplies
//     the low parts;
//   * SwiGLU: an m-tile holds 8 gate rows (rows 0..7) and the 8 up rows of the
//     same outputs (rows 8..15), so the epilogue reads gate and up of an output
//     from neighbouring partial rows.
// Two e4m3 bytes (the low or the high half of a 32-bit register) -> f16x2; every
// e4m3 value is exact in fp16.
__device__ __forceinline__ uint32_t e4m3x2_lo(uint32_t r) {
  uint32_t d;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; cvt.rn.f16x2.e4m3x2 %0, l; }" : "=r"(d) : "r"(r));
  return d;
}
__device__ __forceinline__ uint32_t e4m3x2_hi(uint32_t r) {
  uint32_t d;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; cvt.rn.f16x2.e4m3x2 %0, h; }" : "=r"(d) : "r"(r));
  return d;
}

constexpr int kMmaKC = 2048;
constexpr int kMmaKC8 = 4096;                 // fp8 weights: same 4 KB row segments
constexpr int kMmaSlot = kMmaKC * 2 + 16;     // padded row slot (bytes)
constexpr int kMmaStage = 16 * kMmaSlot;      // 65,792 bytes
constexpr int kMmaStages = 3;

// W8: weights are e4m3 bytes with a per-row fp32 scale. A stage then holds 4096
// columns; ldmatrix on the bytes gives each lane 4 consecutive k of a row, which
// are widened to f16 and used as the mma's k slots (2q, 2q+1, 2q+8, 2q+9) -- the
// activation fragment is loaded with the same k order, so the dot product is
// unchanged. The activation is staged in fp16 (hi + lo) whatever T is.
template <typename T, int MODE, bool SPLIT, bool W8 = false>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const GemvArgs a) {
  using MT = typename std::conditional<W8, __half, T>::type;   // mma / staging type
  constexpr int KC = W8 ? kMmaKC8 : kMmaKC;
  constexpr int WB = W8 ? 1 : (int)sizeof(T);                 // bytes per weight
  constexpr int NMAT = (MODE == MODE_SWIGLU) ? 2 : 1;
  constexpr int RPT = 16 / NMAT;                  // output rows per m-tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = smem_raw;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)a.nstages * kMmaStage);
  uint64_t* empty = full + a.nstages;
  const int nmt_max = (a.max_rows + RPT - 1) / RPT;
  float* part = reinterpret_cast<float*>(empty + a.nstages);   // [8 warps][nmt_max*16][pcols]
  const int pc = a.pcols;
  uint16_t* xs_hi = reinterpret_cast<uint16_t*>(part + (size_t)kConsumerWarps * nmt_max * 16 * pc);
  uint16_t* xs_lo = xs_hi + (size_t)a.batch * a.d_in;
  __shared__ float red[kConsumerWarps][8];
  __shared__ float inv_rms[8];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  // MODE_QKV: CTA row ranges start on even rows, so a RoPE pair never straddles CTAs
  const int row0 = MODE == MODE_QKV ? 2 * (int)(((int64_t)blockIdx.x * (a.d_out / 2)) / G)
                                    : (int)(((int64_t)blockIdx.x * a.d_out) / G);
  const int row1 = MODE == MODE_QKV ? 2 * (int)(((int64_t)(blockIdx.x + 1) * (a.d_out / 2)) / G)
                                    : (int)(((int64_t)(blockIdx.x + 1) * a.d_out) / G);
  const int nrows = row1 - row0;
  const int nmt = (nrows + RPT - 1) / RPT;
  const int total = nmt * a.nchunks;
  DBK_TRACE_BEGIN();
  DBK_MARK(tid == 0, 0);

  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t* W0 = static_cast<const uint8_t*>(a.w0);
      const uint8_t* W1 = static_cast<const uint8_t*>(a.w1);
      for (int j = 0; j < total; ++j) {
        const int s = j % a.nstages;
        if (j >= a.nstages &&
            !DBK_TIMED_WAIT(true, 10, mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty)))
          return;
        const int mt = j / a.nchunks, c = j - mt * a.nchunks;
        const int col0 = c * KC;
        const int seg = min(KC, a.d_in - col0);
        const int r_first = row0 + mt * RPT;
        const int valid = min(RPT, row1 - r_first);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(valid * NMAT * seg * WB));
        uint8_t* dst = ring + (size_t)s * kMmaStage;
        for (int q = 0; q < valid; ++q) {
          const size_t off = ((size_t)(r_first + q) * a.d_in + col0) * WB;
          bulk_g2s(dst + q * kMmaSlot, W0 + off, (uint32_t)(seg * WB), &full[s], pol);
          if constexpr (NMAT == 2)
            bulk_g2s(dst + (8 + q) * kMmaSlot, W1 + off, (uint32_t)(seg * WB), &full[s], pol);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int ag_world = a.ps.world;
  const unsigned long long ag_e =
      ag_world > 1 ? *reinterpret_cast<volatile unsigned long long*>(a.ps.peer[a.ps.rank]) : 0ull;
  const int ag_parity = (int)(ag_e & 1);
  const T* x = static_cast<const T*>(a.x);
  const T* gam = static_cast<const T*>(a.gamma);
  {
    // Stage x (* gamma) as high + low 16-bit parts; sum(x^2) in the same pass.
    float ss[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) ss[b] = 0.f;
    const int per_row = a.d_in / 8;
    for (int v = tid; v < a.batch * per_row; v += kConsumers) {
      const int b = v / per_row, c = (v - b * per_row) * 8;
      float f[8], g[8];
      unpack8<T>(ldg_nc_v4(x + (size_t)b * a.d_in + c), f);
      if (gam != nullptr) unpack8<T>(ldg_nc_v4(gam + c), g);
      uint32_t hi[4], lo[4];
      float sq = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float p0 = f[e], p1 = f[e + 1];
        sq = fmaf(p0, p0, fmaf(p1, p1, sq));
        if (gam != nullptr) { p0 *= g[e]; p1 *= g[e + 1]; }
        hi[e / 2] = Mma<MT>::pack(p0, p1);
        const float2 h = Elem<MT>::unpack2(hi[e / 2]);
        lo[e / 2] = Mma<MT>::pack(p0 - h.x, p1 - h.y);
      }
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) ss[bb] += (bb == b) ? sq : 0.f;
      *reinterpret_cast<uint4*>(xs_hi + (size_t)b * a.d_in + c) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(xs_lo + (size_t)b * a.d_in + c) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const float t = warp_sum(ss[b]);
      if (lane == 0) red[warp][b] = t;
    }
  }
  named_bar_sync(1, kConsumers);
  DBK_MARK(tid == 0, 1);
  if (tid < 8) {
    float v = 1.f;
    if (MODE != MODE_PLAIN && gam != nullptr && tid < a.batch) {
      float t = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) t += red[w][tid];
      v = rsqrtf(t / (float)a.d_in + a.eps);
    }
    inv_rms[tid] = v;
  }

  // ldmatrix.x4 addressing: lane supplies row (lane&7) + 8*((lane>>3)&1) and
  // column offset 8*(lane>>4) within a 16-column k-step.
  const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const uint32_t a_lane_off = (uint32_t)(a_row * kMmaSlot + (8 * (lane >> 4)) * 2);
  const int bn = lane >> 2;                  // B column held by this lane
  const bool packed = SPLIT && pc > a.batch;  // columns [batch, 2 batch) hold the low parts
  const bool b_ok = bn < pc;
  const int kq = (W8 ? 4 : 2) * (lane & 3);   // this lane's first k in a 16- (32-) k step
  const uint16_t* xh =
      (packed && bn >= a.batch ? xs_lo + (size_t)(bn - a.batch) * a.d_in
                               : xs_hi + (size_t)(b_ok ? bn : 0) * a.d_in) + kq;
  const uint16_t* xl = xs_lo + (size_t)(b_ok && bn < a.batch ? bn : 0) * a.d_in + kq;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float acc2[4] = {0.f, 0.f, 0.f, 0.f};
  // d_in <= 2 * KC with one B operand per k-step (no separate low-part MMA): a
  // warp always multiplies the same 16 k-steps of each chunk, so its activation
  // fragments are loaded from shared memory once instead of once per m-tile.
  // (Not for the QKV epilogue, whose registers would then spill.)
  const bool cache_b = !W8 && a.nchunks <= 2 && !(SPLIT && !packed);
  uint32_t bfrag[2][16][2];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      const int col = c * KC + warp * 256 + kk * 16;
      const bool ok = cache_b && b_ok && c < a.nchunks && col < a.d_in;
      bfrag[c][kk][0] = ok ? *reinterpret_cast<const uint32_t*>(xh + col) : 0u;
      bfrag[c][kk][1] = ok ? *reinterpret_cast<const uint32_t*>(xh + col + 8) : 0u;
    }
  for (int j = 0; j < total; ++j) {
    const int s = j % a.nstages;
    const int mt = j / a.nchunks, c = j - mt * a.nchunks;
    const int col0 = c * KC;
    const int seg = min(KC, a.d_in - col0);
    if (!DBK_TIMED_WAIT(tid == 0, 11, mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull))) return;
    DBK_MARK(tid == 0 && j == 0, 2);
    const uint32_t stage = smem_u32(ring + (size_t)s * kMmaStage) + a_lane_off;
    if constexpr (W8) {
#pragma unroll 4
      for (int kk = 0; kk < 16; ++kk) {
        const int k = warp * 512 + kk * 32;     // 32 fp8 columns = 32 bytes per row
        if (k < seg) {
          uint32_t af[4];
          ldsm_x4(stage + k, af);               // rows g / g+8, bytes k+4q..+3 and k+16+4q..+3
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t ra = af[2 * h], rb = af[2 * h + 1];
            const int kx = col0 + k + 16 * h;
            uint32_t b0 = 0u, b1 = 0u;
            if (b_ok) {
              b0 = *reinterpret_cast<const uint32_t*>(xh + kx);
              b1 = *reinterpret_cast<const uint32_t*>(xh + kx + 2);
            }
            Mma<__half>::run(acc, e4m3x2_lo(ra), e4m3x2_lo(rb), e4m3x2_hi(ra), e4m3x2_hi(rb), b0, b1);
            if (SPLIT && !packed) {
              uint32_t l0 = 0u, l1 = 0u;
              if (b_ok) {
                l0 = *reinterpret_cast<const uint32_t*>(xl + kx);
                l1 = *reinterpret_cast<const uint32_t*>(xl + kx + 2);
              }
              Mma<__half>::run(acc, e4m3x2_lo(ra), e4m3x2_lo(rb), e4m3x2_hi(ra), e4m3x2_hi(rb), l0, l1);
            }
          }
        }
      }
    } else if (cache_b) {
      // The activation fragments of this warp's k-steps were loaded once (before
      // the loop); the weight loads of 8 k-steps are issued back to back before
      // their MMAs, which alternate between two accumulator chains.
      // weight loads in batches of KB k-steps (4 for the QKV epilogue's registers)
      constexpr int KB = MODE == MODE_QKV ? 4 : 8;
      auto run_stage = [&](const uint32_t (&bb)[16][2]) {
#pragma unroll
        for (int k8 = 0; k8 < 16; k8 += KB) {
          uint32_t af[KB][4];
#pragma unroll
          for (int kk = 0; kk < KB; ++kk) {
            const int k = warp * 256 + (k8 + kk) * 16;
            if (k < seg) ldsm_x4(stage + k * 2, af[kk]);
          }
#pragma unroll
          for (int kk = 0; kk < KB; ++kk) {
            const int k = warp * 256 + (k8 + kk) * 16;
            if (k < seg)
              Mma<T>::run((kk & 1) ? acc2 : acc, af[kk][0], af[kk][1], af[kk][2], af[kk][3],
                          bb[k8 + kk][0], bb[k8 + kk][1]);
          }
        }
      };
      if (c == 0) run_stage(bfrag[0]);
      else run_stage(bfrag[1]);
    } else {
#pragma unroll 4
      for (int kk = 0; kk < 16; ++kk) {
        const int k = warp * 256 + kk * 16;
        if (k < seg) {
          uint32_t af[4];
          ldsm_x4(stage + k * 2, af);
          uint32_t b0 = 0u, b1 = 0u;
          if (b_ok) {
            b0 = *reinterpret_cast<const uint32_t*>(xh + col0 + k);
            b1 = *reinterpret_cast<const uint32_t*>(xh + col0 + k + 8);
          }
          Mma<T>::run(acc, af[0], af[1], af[2], af[3], b0, b1);
          if (SPLIT && !packed) {
            uint32_t l0 = 0u, l1 = 0u;
            if (b_ok) {
              l0 = *reinterpret_cast<const uint32_t*>(xl + col0 + k);
              l1 = *reinterpret_cast<const uint32_t*>(xl + col0 + k + 8);
            }
            Mma<T>::run(acc, af[0], af[1], af[2], af[3], l0, l1);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (c == a.nchunks - 1) {
      // m-tile done: accumulator rows (lane>>2) and (lane>>2)+8, columns 2*(lane&3) + {0,1}
#pragma unroll
      for (int e = 0; e < 4; ++e) { acc[e] += acc2[e]; acc2[e] = 0.f; }
      const int r = mt * 16 + (lane >> 2), n0 = 2 * (lane & 3);
      float* pw = part + (size_t)warp * nmt_max * 16 * pc;
      if (n0 < pc) {
        pw[(size_t)r * pc + n0] = acc[0];
        pw[(size_t)(r + 8) * pc + n0] = acc[2];
      }
      if (n0 + 1 < pc) {
        pw[(size_t)r * pc + n0 + 1] = acc[1];
        pw[(size_t)(r + 8) * pc + n0 + 1] = acc[3];
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
  }
  named_bar_sync(1, kConsumers);
  DBK_MARK(tid == 0, 3);

  if constexpr (MODE == MODE_QKV) {
    // pairs of adjacent rows: RoPE on q and k, then q out and k, v into the cache
    const QkvArgs& Q = a.qkv;
    const int D = Q.head_dim, np = nrows / 2;
    for (int idx = tid; idx < np * a.batch; idx += kConsumers) {
      const int b = idx / np, r = 2 * (idx - b * np);
      float v2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int mt = (r + e) / RPT, slot = (r + e) - mt * RPT;
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* pr = part + ((size_t)w * nmt_max * 16 + mt * 16 + slot) * pc;
          t += packed ? pr[b] + pr[a.batch + b] : pr[b];
        }
        v2[e] = t * inv_rms[b];
      }
      const int grow = row0 + r, head = grow / D, j = grow - head * D;   // j even
      const int pos = Q.pos[b];
      if (head < Q.hq + Q.hkv) {
        const int i = j >> 1;
        float sn, cs;
        sincosf((float)pos * Q.inv_freq[i], &sn, &cs);
        const float x0 = v2[0], x1 = v2[1];      // dims i and i + D/2
        v2[0] = x0 * cs - x1 * sn;
        v2[1] = x1 * cs + x0 * sn;
      }
      if (head < Q.hq) {
        T* qo = static_cast<T*>(Q.q_out) + ((size_t)b * Q.hq + head) * D;
        qo[j >> 1] = Elem<T>::from_f(v2[0]);
        qo[(j >> 1) + D / 2] = Elem<T>::from_f(v2[1]);
        continue;
      }
      const bool is_k = head < Q.hq + Q.hkv;
      const int hk = head - Q.hq - (is_k ? 0 : Q.hkv);
      if (pos < 0 || pos >= Q.page_size * Q.max_pages) continue;   // no slot: nothing cached
      const int base = Q.page_table ? Q.page_table[(size_t)b * Q.max_pages + pos / Q.page_size] : b;
      const int off = Q.page_table ? pos % Q.page_size : pos;
      T* c = static_cast<T*>(is_k ? Q.k_cache : Q.v_cache) +
             (((size_t)base * Q.hkv + hk) * Q.page_size + off) * D;
      if (is_k) {
        c[j >> 1] = Elem<T>::from_f(v2[0]);
        c[(j >> 1) + D / 2] = Elem<T>::from_f(v2[1]);
      } else {                                    // v rows are in natural order
        c[j] = Elem<T>::from_f(v2[0]);
        c[j + 1] = Elem<T>::from_f(v2[1]);
      }
    }
    return;
  }
  T* y = static_cast<T*>(a.y);
  const T* res = static_cast<const T*>(a.residual);
  for (int idx = tid; idx < nrows * a.batch; idx += kConsumers) {
    const int b = idx / nrows, r = idx - b * nrows;
    const int mt = r / RPT, q = r - mt * RPT;
    auto sum_row = [&](int slot) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float* pr = part + ((size_t)w * nmt_max * 16 + mt * 16 + slot) * pc;
        t += packed ? pr[b] + pr[a.batch + b] : pr[b];
      }
      return t;
    };
    float v;
    const float s0 = W8 ? a.wscale0[row0 + r] : 1.f;
    if constexpr (MODE == MODE_SWIGLU) {
      const float sc = inv_rms[b];
      const float s1 = W8 ? a.wscale1[row0 + r] : 1.f;
      v = silu(sum_row(q) * sc * s0) * (sum_row(8 + q) * sc * s1);
    } else if constexpr (MODE == MODE_NORM) {
      v = sum_row(q) * inv_rms[b] * s0;
    } else {
      v = sum_row(q) * s0;
    }
    const size_t o = (size_t)b * a.y_ld + a.y_col0 + row0 + r;
    if (res != nullptr) v += Elem<T>::to_f(res[o]);
    const T out = Elem<T>::from_f(v);
    y[o] = out;
    // fused all-gather: the same value into every peer's staging block of this rank
    for (int p = 0; p < ag_world; ++p)
      if (p != a.ps.rank)
        reinterpret_cast<T*>(staging(a.ps.peer[p], a.ps, ag_parity, a.ps.rank))
            [(size_t)b * a.d_out + row0 + r] = out;
  }
  DBK_MARK(tid == 0, 4);
  if (ag_world > 1) {
    // Rows [row0, row1) of every rank's block come from the CTA with this index on
    // that rank (same shape, same grid), so the CTA pairs up with its namesakes only.
    char* local = a.ps.peer[a.ps.rank];
    named_bar_sync(1, kConsumers);        // this CTA's stores precede the release below
    if (tid < ag_world && tid != a.ps.rank) {
      st_release_sys(flag_slot(a.ps.peer[tid], a.ps.rank, blockIdx.x), ag_e + 1);
      wait_flag(flag_slot(local, tid, blockIdx.x), ag_e + 1);
    }
    named_bar_sync(1, kConsumers);
    for (int idx = tid; idx < (ag_world - 1) * nrows * a.batch; idx += kConsumers) {
      const int q = idx / (nrows * a.batch), rem = idx - q * nrows * a.batch;
      const int p = q + (q >= a.ps.rank ? 1 : 0);
      const int b = rem / nrows, r = rem - b * nrows;
      const T* st = reinterpret_cast<const T*>(staging(local, a.ps, ag_parity, p));
      const unsigned short u =
          __ldcg(reinterpret_cast<const unsigned short*>(st) + (size_t)b * a.d_out + row0 + r);
      reinterpret_cast<unsigned short*>(y)[(size_t)b * a.y_ld + (size_t)p * a.d_out + row0 + r] = u;
    }
    named_bar_sync(1, kConsumers);
    if (tid == 0) finish_exchange(local, ag_e);
  }
}

// Shared-memory bytes of the tensor-core variant for a stage count (0 if it
// cannot run: d_in % 16 != 0 or batch > 8).
size_t mma_smem_bytes(const GemvArgs& a, int rpt, int nst) {
  if (a.d_in % 16 != 0 || a.batch > 8) return 0;
  const int nmt_max = (a.max_rows + rpt - 1) / rpt;
  return (size_t)nst * (kMmaStage + 16) + (size_t)kConsumerWarps * nmt_max * 16 * a.pcols * 4 +
         (size_t)a.batch * a.d_in * 4 + 256;
}

template <typename T, int MODE>
int launch_mma(GemvArgs a, cudaStream_t st, const DeviceInfo& dev, size_t smem) {
  const bool w8 = a.wscale0 != nullptr;
  a.kc = w8 ? kMmaKC8 : kMmaKC;
  a.nchunks = (a.d_in + a.kc - 1) / a.kc;
  // x alone is exact in 16 bits: no low part (except for fp8 weights with bf16 x,
  // whose activation is restaged in fp16)
  const bool split = a.gamma != nullptr || (w8 && std::is_same<T, __nv_bfloat16>::value);
  const void* kern;
  if constexpr (MODE == MODE_QKV) {
    kern = split ? reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, true>)
                 : reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, false>);
  } else {
    kern = w8 ? (split ? reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, true, true>)
                       : reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, false, true>))
              : (split ? reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, true>)
                       : reinterpret_cast<const void*>(gemv_mma_kernel<T, MODE, false>));
  }
  if (int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kern), dev, smem)) return rc;
  return launch_pdl(kern, dim3(a.d_out < dev.num_sms ? a.d_out : dev.num_sms), dim3(kThreads),
                    smem, st, &a);
}

template <typename T, int NB, int MODE>
int launch_nb(GemvArgs a, cudaStream_t st, const DeviceInfo& dev) {
  constexpr int KCG = (NB >= 8) ? 1 : 8 / NB;    // x registers: NB * KCG * 8 = 64
  constexpr int NMAT = (MODE == MODE_SWIGLU) ? 2 : 1;
  a.kc = 256 * KCG;
  a.nchunks = (a.d_in + a.kc - 1) / a.kc;
  const int seg_max = a.kc < a.d_in ? a.kc : a.d_in;
  const int slot_bytes = a.kc * (int)sizeof(T);
  a.slots = kStageBytes / slot_bytes;            // 8 .. 64, multiple of 8
  (void)seg_max;
  const int grid = a.d_out < dev.num_sms ? a.d_out : dev.num_sms;
  a.max_rows = (a.d_out + grid - 1) / grid;
  size_t fixed = (size_t)a.max_rows * NMAT * NB * sizeof(float) + NB * sizeof(float) + 64;
  int nst = kMaxStages;
  while (nst > 2 && (size_t)nst * (kStageBytes + 16) + fixed > (size_t)dev.max_smem_optin) --nst;
  a.nstages = nst;
  const size_t smem = (size_t)nst * (kStageBytes + 16) + fixed;
  if (smem > (size_t)dev.max_smem_optin) return DBK_ESHAPE;

  auto kern = gemv_stream_kernel<T, NB, MODE, KCG>;
  if (int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kern), dev, smem)) return rc;
  return launch_pdl(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), smem, st, &a);
}

template <typename T, int MODE>
int launch_t(const GemvArgs& a0, cudaStream_t st, const DeviceInfo& dev) {
  static const bool simt_only = [] {
    const char* v = std::getenv("DBK_GEMV_SIMT");
    return v && v[0] == '1';
  }();
  GemvArgs a = a0;
  {
    const int grid = a.d_out < dev.num_sms ? a.d_out : dev.num_sms;
    a.max_rows = (MODE == MODE_QKV) ? 2 * ((a.d_out / 2 + grid - 1) / grid)
                                    : (a.d_out + grid - 1) / grid;
    const int rpt = (MODE == MODE_SWIGLU) ? 8 : 16;
    // x * gamma needs its low part; with batch <= 4 it rides in spare B columns
    const bool split = a.gamma != nullptr ||
                       (a.wscale0 != nullptr && std::is_same<T, __nv_bfloat16>::value);
    a.pcols = (split && 2 * a.batch <= 8) ? 2 * a.batch : a.batch;
    for (int nst = kMmaStages; nst >= 2 && !simt_only; --nst) {
      const size_t smem = mma_smem_bytes(a, rpt, nst);
      if (smem != 0 && smem <= (size_t)dev.max_smem_optin - 1024) {
        a.nstages = nst;
        return launch_mma<T, MODE>(a, st, dev, smem);
      }
    }
  }
  if (a.ps.world > 1 || a.wscale0 != nullptr)
    return DBK_ESHAPE;   // the fused all-gather and fp8 weights need the tensor-core variant
  if constexpr (MODE == MODE_QKV) {
    return DBK_ESHAPE;                      // no CUDA-core variant of the QKV epilogue
  } else {
    if (a.batch <= 1) return launch_nb<T, 1, MODE>(a, st, dev);
    if (a.batch <= 2) return launch_nb<T, 2, MODE>(a, st, dev);
    if (a.batch <= 4) return launch_nb<T, 4, MODE>(a, st, dev);
    return launch_nb<T, 8, MODE>(a, st, dev);
  }
}

int gemv_dispatch(int mode, GemvArgs a, int dtype, cudaStream_t st) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  if (a.y_ld == 0) a.y_ld = a.d_out;
  if (dtype == DBK_F16) {
    switch (mode) {
      case MODE_PLAIN: return launch_t<__half, MODE_PLAIN>(a, st, dev);
      case MODE_NORM: return launch_t<__half, MODE_NORM>(a, st, dev);
      case MODE_QKV: return launch_t<__half, MODE_QKV>(a, st, dev);
      default: return launch_t<__half, MODE_SWIGLU>(a, st, dev);
    }
  }
  switch (mode) {
    case MODE_PLAIN: return launch_t<__nv_bfloat16, MODE_PLAIN>(a, st, dev);
    case MODE_NORM: return launch_t<__nv_bfloat16, MODE_NORM>(a, st, dev);
    case MODE_QKV: return launch_t<__nv_bfloat16, MODE_QKV>(a, st, dev);
    default: return launch_t<__nv_bfloat16, MODE_SWIGLU>(a, st, dev);
  }
}

int check_common(const void* x, const void* w, const void* y, int batch, int d_in, int d_out,
                 int dtype) {
  if (!x || !w || !y) return DBK_ENULL;
  if (dtype != DBK_F16 && dtype != DBK_BF16) return DBK_EDTYPE;
  if (batch < 1 || d_in < 8 || d_out < 1 || (d_in % 8) != 0) return DBK_ESHAPE;
  if (!aligned16(x) || !aligned16(w)) return DBK_EALIGN;
  return DBK_OK;
}

}  // namespace
}  // namespace dbk

using namespace dbk;

extern "C" int dbk_rmsnorm_gemv(const void* x, const void* gamma, const void* W, void* y,
                                int batch, int d_in, int d_out, float eps, int dtype,
                                void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(x, W, y, batch, d_in, d_out, dtype);
  if (rc) return rc;
  if (!gamma) return DBK_ENULL;
  if (!aligned16(gamma)) return DBK_EALIGN;
  if (batch > kSimtMaxBatch)
    return dbk_tc_rmsnorm_gemv(x, gamma, W, y, batch, d_in, d_out, eps, dtype, workspace,
                               workspace_bytes, stream);
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = W; a.y = y;
  a.batch = batch; a.d_in = d_in; a.d_out = d_out; a.eps = eps;
  return gemv_dispatch(MODE_NORM, a, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int dbk_gateup_swiglu(const void* x, const void* gamma, const void* Wg,
                                 const void* Wu, void* h, int batch, int d_in, int d_ff,
                                 float eps, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  int rc = check_common(x, Wg, h, batch, d_in, d_ff, dtype);
  if (rc) return rc;
  if (!Wu) return DBK_ENULL;
  if (!aligned16(Wu) || (gamma && !aligned16(gamma))) return DBK_EALIGN;
  if (batch > kSimtMaxBatch)
    return dbk_tc_gateup_swiglu(x, gamma, Wg, Wu, h, batch, d_in, d_ff, eps, dtype, workspace,
                                workspace_bytes, stream);
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = Wg; a.w1 = Wu; a.y = h;
  a.batch = batch; a.d_in = d_in; a.d_out = d_ff; a.eps = eps;
  return gemv_dispatch(MODE_SWIGLU, a, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int dbk_gemv(const void* x, const void* W, const void* residual, void* y, int batch,
                        int d_in, int d_out, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_common(x, W, y, batch, d_in, d_out, dtype);
  if (rc) return rc;
  if (batch > kSimtMaxBatch)
    return dbk_tc_gemv(x, W, residual, y, batch, d_in, d_out, dtype, workspace,
                       workspace_bytes, stream);
  GemvArgs a{};
  a.x = x; a.w0 = W; a.residual = residual; a.y = y;
  a.batch = batch; a.d_in = d_in; a.d_out = d_out;
  return gemv_dispatch(MODE_PLAIN, a, dtype, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Sharded GEMV with the shard-boundary all-gather fused into the epilogue
// (batch 1..8). Each rank computes d_local output columns; every CTA stores its
// rows into the peers' staging blocks as it produces them, publishes a release
// flag, waits (bounded) for the same-index CTA of each peer and copies their
// rows into y_full [batch][world * d_local] (rank p's columns start at
// p * d_local). No separate collective launch.
namespace {

int gemv_ag(int mode, dbk_comm* comm, GemvArgs a, int dtype, void* stream) {
  if (!comm) return DBK_ENULL;
  if (a.batch > kSimtMaxBatch) return DBK_ESHAPE;
  PeerSet ps;
  if (int rc = comm_peerset(comm, &ps)) return rc;
  if ((long long)a.batch * a.d_out * 2 > ps.capacity) return DBK_EWORKSPACE;
  a.ps = ps;
  a.y_ld = (long long)ps.world * a.d_out;
  a.y_col0 = (long long)ps.rank * a.d_out;
  if (ps.world == 1) a.ps.world = 0;   // nothing to exchange
  return gemv_dispatch(mode, a, dtype, static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" int dbk_rmsnorm_gemv_allgather(dbk_comm* comm, const void* x, const void* gamma,
                                          const void* W, void* y_full, int batch, int d_in,
                                          int d_local, float eps, int dtype, void* stream) {
  int rc = check_common(x, W, y_full, batch, d_in, d_local, dtype);
  if (rc) return rc;
  if (!gamma) return DBK_ENULL;
  if (!aligned16(gamma)) return DBK_EALIGN;
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = W; a.y = y_full;
  a.batch = batch; a.d_in = d_in; a.d_out = d_local; a.eps = eps;
  return gemv_ag(MODE_NORM, comm, a, dtype, stream);
}

extern "C" int dbk_gateup_swiglu_allgather(dbk_comm* comm, const void* x, const void* gamma,
                                           const void* Wg, const void* Wu, void* h_full,
                                           int batch, int d_in, int d_local, float eps,
                                           int dtype, void* stream) {
  int rc = check_common(x, Wg, h_full, batch, d_in, d_local, dtype);
  if (rc) return rc;
  if (!Wu) return DBK_ENULL;
  if (!aligned16(Wu) || (gamma && !aligned16(gamma))) return DBK_EALIGN;
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = Wg; a.w1 = Wu; a.y = h_full;
  a.batch = batch; a.d_in = d_in; a.d_out = d_local; a.eps = eps;
  return gemv_ag(MODE_SWIGLU, comm, a, dtype, stream);
}

extern "C" int dbk_gemv_allgather(dbk_comm* comm, const void* x, const void* W,
                                  const void* residual_full, void* y_full, int batch, int d_in,
                                  int d_local, int dtype, void* stream) {
  int rc = check_common(x, W, y_full, batch, d_in, d_local, dtype);
  if (rc) return rc;
  GemvArgs a{};
  a.x = x; a.w0 = W; a.residual = residual_full; a.y = y_full;
  a.batch = batch; a.d_in = d_in; a.d_out = d_local;
  return gemv_ag(MODE_PLAIN, comm, a, dtype, stream);
}

// ---------------------------------------------------------------------------
// QKV projection + RoPE + KV-cache append (batch 1..8).
extern "C" int dbk_qkv_rope_append(const void* x, const void* gamma, const void* Wqkv,
                                   const int32_t* positions, const float* inv_freq, void* q_out,
                                   void* k_cache, void* v_cache, const int32_t* page_table,
                                   int batch, int d_in, int n_q_heads, int n_kv_heads,
                                   int head_dim, int page_size, int max_pages_per_seq,
                                   float eps, int dtype, void* stream) {
  const int d_out = (n_q_heads + 2 * n_kv_heads) * head_dim;
  int rc = check_common(x, Wqkv, q_out, batch, d_in, d_out > 0 ? d_out : 1, dtype);
  if (rc) return rc;
  if (!positions || !inv_freq || !k_cache || !v_cache) return DBK_ENULL;
  if (gamma && !aligned16(gamma)) return DBK_EALIGN;
  if (n_q_heads < 1 || n_kv_heads < 1 || head_dim < 2 || head_dim % 2 || page_size < 1 ||
      max_pages_per_seq < 1 || batch > kSimtMaxBatch)
    return DBK_ESHAPE;
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = Wqkv; a.y = q_out;
  a.batch = batch; a.d_in = d_in; a.d_out = d_out; a.eps = eps;
  a.qkv.pos = positions; a.qkv.inv_freq = inv_freq; a.qkv.q_out = q_out;
  a.qkv.k_cache = k_cache; a.qkv.v_cache = v_cache; a.qkv.page_table = page_table;
  a.qkv.hq = n_q_heads; a.qkv.hkv = n_kv_heads; a.qkv.head_dim = head_dim;
  a.qkv.page_size = page_size; a.qkv.max_pages = page_table ? max_pages_per_seq : 1;
  return gemv_dispatch(MODE_QKV, a, dtype, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// fp8 (e4m3) weights with a per-row fp32 scale, batch 1..8: half the weight bytes
// of the 16-bit entry points. y[b, r] = scale[r] * sum_k W8[r, k] x'[b, k].
namespace {
int check_fp8(const void* x, const void* w, const float* sc, const void* y, int batch, int d_in,
              int d_out, int dtype) {
  if (int rc = check_common(x, w, y, batch, d_in, d_out, dtype)) return rc;
  if (!sc) return DBK_ENULL;
  if (batch > kSimtMaxBatch || d_in % 32 != 0) return DBK_ESHAPE;
  return DBK_OK;
}
}  // namespace

extern "C" int dbk_gemv_fp8(const void* x, const void* W8, const float* w_scale,
                            const void* residual, void* y, int batch, int d_in, int d_out,
                            int dtype, void* stream) {
  if (int rc = check_fp8(x, W8, w_scale, y, batch, d_in, d_out, dtype)) return rc;
  GemvArgs a{};
  a.x = x; a.w0 = W8; a.wscale0 = w_scale; a.residual = residual; a.y = y;
  a.batch = batch; a.d_in = d_in; a.d_out = d_out;
  return gemv_dispatch(MODE_PLAIN, a, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int dbk_rmsnorm_gemv_fp8(const void* x, const void* gamma, const void* W8,
                                    const float* w_scale, void* y, int batch, int d_in,
                                    int d_out, float eps, int dtype, void* stream) {
  if (int rc = check_fp8(x, W8, w_scale, y, batch, d_in, d_out, dtype)) return rc;
  if (!gamma) return DBK_ENULL;
  if (!aligned16(gamma)) return DBK_EALIGN;
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = W8; a.wscale0 = w_scale; a.y = y;
  a.batch = batch; a.d_in = d_in; a.d_out = d_out; a.eps = eps;
  return gemv_dispatch(MODE_NORM, a, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int dbk_gateup_swiglu_fp8(const void* x, const void* gamma, const void* Wg8,
                                     const float* g_scale, const void* Wu8,
                                     const float* u_scale, void* h, int batch, int d_in,
                                     int d_ff, float eps, int dtype, void* stream) {
  if (int rc = check_fp8(x, Wg8, g_scale, h, batch, d_in, d_ff, dtype)) return rc;
  if (!Wu8 || !u_scale) return DBK_ENULL;
  if (!aligned16(Wu8) || (gamma && !aligned16(gamma))) return DBK_EALIGN;
  GemvArgs a{};
  a.x = x; a.gamma = gamma; a.w0 = Wg8; a.w1 = Wu8; a.wscale0 = g_scale; a.wscale1 = u_scale;
  a.y = h; a.batch = batch; a.d_in = d_in; a.d_out = d_ff; a.eps = eps;
  return gemv_dispatch(MODE_SWIGLU, a, dtype, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Persistent MLP block (batch 1..4): h = silu(Wg x') * (Wu x') with x' = x, or the
// RMSNorm of x when gamma is given, then y = Wd h (+ residual), in ONE launch:
//   * one CTA per SM with gemv_mma_kernel's producer / consumer split and ring;
//     the producer walks the CTA's gate/up rows and then, without a pause, its
//     down rows, so the ring already holds Wd when phase 2 may start;
//   * phase 1 writes h to global memory, then every CTA meets the others at a
//     grid-wide barrier (two counters in the workspace, bounded wait, left at
//     zero by the last CTA through) -- the only synchronisation between the
//     GEMVs, instead of a kernel boundary and a second pipeline fill;
//   * phase 2 stages all of h (exact in 16 bits: no low part) over the shared
//     bytes that phase 1 used for its activation stage and partial sums.
// Per output the arithmetic is that of dbk_gateup_swiglu followed by dbk_gemv
// (the same k-step order per warp, the same fixed warp order in the epilogue,
// fp32 accumulation), so the two agree bit for bit.
// Reference semantics: fused f2_kernel (validation/src/kernels/fused/f2.cu:17-76)
// and the down projection of the decode MLP (src/decodebench/demos/llama_decode.py:77-87).
namespace dbk {
namespace {

struct MlpArgs {
  GemvArgs o;        // optional phase 0: MODE_PLAIN, y = h_attn = Wo o + residual
  GemvArgs g;        // phase 1: MODE_SWIGLU, y = h
  GemvArgs d;        // phase 2: MODE_PLAIN, x = h, with residual
  int* sync;         // [2 per barrier]: arrivals, departures (zero before and after a launch)
  int nstages;
  int region_bytes;  // shared bytes after the ring shared by the two phases
};

// CTA rows [row0, row1) of a d_out-row operand over G CTAs.
__device__ __forceinline__ int2 cta_rows(int d_out, int G) {
  return make_int2((int)(((int64_t)blockIdx.x * d_out) / G),
                   (int)(((int64_t)(blockIdx.x + 1) * d_out) / G));
}

// Producer: one phase's (m-tile, K chunk) stages into the ring, continuing the
// ring position j. NMAT = 2 puts the gate rows in slots 0..7 and the up rows in
// slots 8..15 of a stage. False when a bounded wait gave up.
template <int NMAT>
__device__ __forceinline__ bool mlp_produce(const GemvArgs& a, int2 rows, uint8_t* ring,
                                            uint64_t* full, uint64_t* empty, int nst, int& j,
                                            uint64_t pol) {
  constexpr int RPT = 16 / NMAT;
  const int nmt = (rows.y - rows.x + RPT - 1) / RPT;
  const uint8_t* W0 = static_cast<const uint8_t*>(a.w0);
  const uint8_t* W1 = static_cast<const uint8_t*>(a.w1);
  for (int t = 0; t < nmt * a.nchunks; ++t, ++j) {
    const int s = j % nst;
    if (j >= nst && !mbar_wait(&empty[s], ((j / nst) & 1) ^ 1, kDevTimeoutEmpty)) return false;
    const int mt = t / a.nchunks, c = t - mt * a.nchunks;
    const int col0 = c * kMmaKC;
    const int seg = min(kMmaKC, a.d_in - col0);
    const int r_first = rows.x + mt * RPT;
    const int valid = min(RPT, rows.y - r_first);
    mbar_arrive_expect_tx(&full[s], (uint32_t)(valid * NMAT * seg * 2));
    uint8_t* dst = ring + (size_t)s * kMmaStage;
    for (int q = 0; q < valid; ++q) {
      const size_t off = ((size_t)(r_first + q) * a.d_in + col0) * 2;
      bulk_g2s(dst + q * kMmaSlot, W0 + off, (uint32_t)(seg * 2), &full[s], pol);
      if constexpr (NMAT == 2)
        bulk_g2s(dst + (8 + q) * kMmaSlot, W1 + off, (uint32_t)(seg * 2), &full[s], pol);
    }
  }
  return true;
}

// Grid-wide barrier, called by one thread per CTA after the CTA's stores.
// Arrivals count up to the grid size; the CTA that departs last puts both
// counters back to zero (no CTA reads them again in this launch).
__device__ __forceinline__ bool grid_barrier(int* sync, int nblocks) {
  __threadfence();
  arrive_release_gpu(&sync[0]);
  uint32_t n = 0;
  const uint32_t lim = spin_limit();
  bool ok = true;
  while (ld_acquire_gpu(&sync[0]) < nblocks) {
    if (++n >= lim) { record_error(kDevTimeoutGrid); ok = false; break; }
    __nanosleep(32);
  }
  if (atomicAdd(&sync[1], 1) == nblocks - 1) {
    sync[0] = 0;
    sync[1] = 0;
  }
  return ok;
}

// Consumers: one phase's MMA loop over the ring, writing each m-tile's per-warp
// partials to `part`. The activation fragments are read from shared memory per
// k-step. TWO_CHAINS alternates the k-steps between two accumulators and adds
// them at the end of the m-tile -- the order of gemv_mma_kernel's register-cached
// variant (d_in <= 2 chunks); without it one chain, the order of its per-k-step
// variant. With skip, stages are waited for and released without computing
// (drains the ring after a failed barrier). False when a bounded wait gave up.
template <typename T, int NMAT, bool TWO_CHAINS, bool CACHED = false>
__device__ __forceinline__ bool mlp_consume(const GemvArgs& a, int2 rows, const uint8_t* ring,
                                            uint64_t* full, uint64_t* empty, int nst, int& j,
                                            float* part, int pc, const uint16_t* xs, bool packed,
                                            bool skip) {
  constexpr int RPT = 16 / NMAT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nmt = (rows.y - rows.x + RPT - 1) / RPT;
  const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const uint32_t a_lane_off = (uint32_t)(a_row * kMmaSlot + (8 * (lane >> 4)) * 2);
  const int bn = lane >> 2;
  const bool b_ok = bn < pc;
  const int kq = 2 * (lane & 3);
  // packed: columns [batch, 2 batch) hold the low parts of the activation
  const uint16_t* xh = (packed && bn >= a.batch ? xs + (size_t)a.batch * a.d_in +
                                                      (size_t)(bn - a.batch) * a.d_in
                                                : xs + (size_t)(b_ok ? bn : 0) * a.d_in) + kq;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float acc2[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t bfrag[CACHED ? 2 : 1][16][2];
  if constexpr (CACHED) {
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const int col = c * kMmaKC + warp * 256 + kk * 16;
        const bool ok = !skip && b_ok && c < a.nchunks && col < a.d_in;
        bfrag[c][kk][0] = ok ? *reinterpret_cast<const uint32_t*>(xh + col) : 0u;
        bfrag[c][kk][1] = ok ? *reinterpret_cast<const uint32_t*>(xh + col + 8) : 0u;
      }
  }
  for (int t = 0; t < nmt * a.nchunks; ++t, ++j) {
    const int s = j % nst;
    const int mt = t / a.nchunks, c = t - mt * a.nchunks;
    const int col0 = c * kMmaKC;
    const int seg = min(kMmaKC, a.d_in - col0);
    if (!mbar_wait(&full[s], (j / nst) & 1, kDevTimeoutFull)) return false;
    const uint32_t stage = smem_u32(ring + (size_t)s * kMmaStage) + a_lane_off;
    if (skip) {
    } else if constexpr (CACHED) {
      auto run_stage = [&](const uint32_t (&bb)[16][2]) {
#pragma unroll
        for (int k4 = 0; k4 < 16; k4 += 4) {
          uint32_t af[4][4];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int k = warp * 256 + (k4 + kk) * 16;
            if (k < seg) ldsm_x4(stage + k * 2, af[kk]);
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int k = warp * 256 + (k4 + kk) * 16;
            if (k < seg)
              Mma<T>::run((kk & 1) ? acc2 : acc, af[kk][0], af[kk][1], af[kk][2], af[kk][3],
                          bb[k4 + kk][0], bb[k4 + kk][1]);
          }
        }
      };
      if (c == 0) run_stage(bfrag[0]);
      else run_stage(bfrag[1]);
    } else {
#pragma unroll 4
      for (int kk = 0; kk < 16; ++kk) {
        const int k = warp * 256 + kk * 16;
        if (k < seg) {
          uint32_t af[4];
          ldsm_x4(stage + k * 2, af);
          uint32_t b0 = 0u, b1 = 0u;
          if (b_ok) {
            b0 = *reinterpret_cast<const uint32_t*>(xh + col0 + k);
            b1 = *reinterpret_cast<const uint32_t*>(xh + col0 + k + 8);
          }
          Mma<T>::run((TWO_CHAINS && (kk & 1)) ? acc2 : acc, af[0], af[1], af[2], af[3], b0, b1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (c == a.nchunks - 1 && !skip) {
#pragma unroll
      for (int e = 0; e < 4; ++e) { acc[e] += acc2[e]; acc2[e] = 0.f; }
      const int r = mt * 16 + (lane >> 2), n0 = 2 * (lane & 3);
      float* pw = part + (size_t)warp * nmt * 16 * pc;
      if (n0 < pc) {
        pw[(size_t)r * pc + n0] = acc[0];
        pw[(size_t)(r + 8) * pc + n0] = acc[2];
      }
      if (n0 + 1 < pc) {
        pw[(size_t)r * pc + n0 + 1] = acc[1];
        pw[(size_t)(r + 8) * pc + n0 + 1] = acc[3];
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
  }
  return true;
}

// Sum of the 8 warp partials of CTA row r (slot within its m-tile), column b.
__device__ __forceinline__ float mlp_row_sum(const float* part, int nmt, int pc, int mt, int slot,
                                             int b, int batch, bool packed) {
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const float* pr = part + ((size_t)w * nmt * 16 + mt * 16 + slot) * pc;
    t += packed ? pr[b] + pr[batch + b] : pr[b];
  }
  return t;
}

// A phase y = W x (+ residual) of the persistent kernel (MODE_PLAIN): stages x
// (written by this launch when in_kernel: read through L2, not the non-coherent
// path), runs the ring, adds the 8 warp partials and the residual, stores y.
// The k-step order is gemv_mma_kernel's for the same d_in. False when a bounded
// wait gave up; with skip it only drains its stages.
template <typename T>
__device__ __forceinline__ bool mlp_plain_phase(const GemvArgs& P, uint8_t* region,
                                                const uint8_t* ring, uint64_t* full,
                                                uint64_t* empty, int nst, int& j, bool in_kernel,
                                                bool skip) {
  const int tid = threadIdx.x;
  const int2 rows = cta_rows(P.d_out, gridDim.x);
  const int nmt = (rows.y - rows.x + 15) / 16;
  const int pc = P.batch;
  float* part = reinterpret_cast<float*>(region);
  uint16_t* xs = reinterpret_cast<uint16_t*>(part + (size_t)kConsumerWarps * nmt * 16 * pc);
  if (!skip) {
    const uint4* src = static_cast<const uint4*>(P.x);
    for (int v = tid; v < P.batch * P.d_in / 8; v += kConsumers)
      reinterpret_cast<uint4*>(xs)[v] = in_kernel ? __ldcg(src + v) : ldg_nc_v4(src + v);
  }
  named_bar_sync(1, kConsumers);
  const bool ok =
      P.nchunks <= 2
          ? mlp_consume<T, 1, true>(P, rows, ring, full, empty, nst, j, part, pc, xs, false, skip)
          : mlp_consume<T, 1, false>(P, rows, ring, full, empty, nst, j, part, pc, xs, false, skip);
  if (!ok) return false;
  if (skip) return true;
  named_bar_sync(1, kConsumers);
  T* y = static_cast<T*>(P.y);
  const unsigned short* res = static_cast<const unsigned short*>(P.residual);
  const int nrows = rows.y - rows.x;
  for (int idx = tid; idx < nrows * P.batch; idx += kConsumers) {
    const int b = idx / nrows, r = idx - b * nrows;
    const int mt = r / 16, q = r - mt * 16;
    float v = mlp_row_sum(part, nmt, pc, mt, q, b, P.batch, false);
    const size_t o = (size_t)b * P.d_out + rows.x + r;
    if (res != nullptr) {
      const unsigned short u = __ldcg(res + o);      // may have been written by this launch
      v += Elem<T>::to_f(*reinterpret_cast<const T*>(&u));
    }
    y[o] = Elem<T>::from_f(v);
  }
  named_bar_sync(1, kConsumers);      // the partials are read before the region is reused
  return true;
}

// PRE: a phase 0 first, h_attn = Wo o + residual (the attention output
// projection), whose output is phase 1's x and phase 2's residual.
template <typename T, bool SPLIT, bool PRE>
__global__ void __launch_bounds__(kThreads, 1) mlp_block_kernel(const MlpArgs m) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int nst = m.nstages;
  uint8_t* ring = smem_raw;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)nst * kMmaStage);
  uint64_t* empty = full + nst;
  uint8_t* region = reinterpret_cast<uint8_t*>(empty + nst);
  __shared__ float red[kConsumerWarps][8];
  __shared__ float inv_rms[8];
  __shared__ int s_ok;

  const GemvArgs& A = m.g;
  const GemvArgs& D = m.d;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int j = 0;
      if ((!PRE || mlp_produce<1>(m.o, cta_rows(m.o.d_out, G), ring, full, empty, nst, j, pol)) &&
          mlp_produce<2>(A, cta_rows(A.d_out, G), ring, full, empty, nst, j, pol))
        mlp_produce<1>(D, cta_rows(D.d_out, G), ring, full, empty, nst, j, pol);
    }
    return;
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");
  int j = 0;
  int barrier = 0;
  // Every output store of this CTA precedes its arrival at the grid-wide barrier.
  auto meet = [&]() {
    named_bar_sync(1, kConsumers);
    if (tid == 0) s_ok = grid_barrier(m.sync + 2 * barrier, G) ? 1 : 0;
    ++barrier;
    named_bar_sync(1, kConsumers);
    return s_ok != 0;
  };
  bool skip = false;
  // ------------------------------------------- phase 0: o_proj (+ residual)
  if constexpr (PRE) {
    if (!mlp_plain_phase<T>(m.o, region, ring, full, empty, nst, j, false, false)) return;
    skip = !meet();
  }

  // -------------------------------------------------- phase 1: gate/up + SwiGLU
  const int2 rows_a = cta_rows(A.d_out, G);
  const int nmt_a = (rows_a.y - rows_a.x + 7) / 8;
  const int pc_a = A.pcols;
  const bool packed_a = SPLIT && pc_a > A.batch;
  float* part = reinterpret_cast<float*>(region);
  uint16_t* xs = reinterpret_cast<uint16_t*>(part + (size_t)kConsumerWarps * nmt_a * 16 * pc_a);
  if (!skip) {
    const T* x = static_cast<const T*>(A.x);
    const T* gam = static_cast<const T*>(A.gamma);
    uint16_t* xs_lo = xs + (size_t)A.batch * A.d_in;
    float ss[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) ss[b] = 0.f;
    const int per_row = A.d_in / 8;
    for (int v = tid; v < A.batch * per_row; v += kConsumers) {
      const int b = v / per_row, c = (v - b * per_row) * 8;
      const uint4* xv = reinterpret_cast<const uint4*>(x + (size_t)b * A.d_in + c);
      float f[8], g[8];
      unpack8<T>(PRE ? __ldcg(xv) : ldg_nc_v4(xv), f);      // phase 0 wrote x when PRE
      if (gam != nullptr) unpack8<T>(ldg_nc_v4(gam + c), g);
      uint32_t hi[4], lo[4];
      float sq = 0.f;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float p0 = f[e], p1 = f[e + 1];
        sq = fmaf(p0, p0, fmaf(p1, p1, sq));
        if (gam != nullptr) { p0 *= g[e]; p1 *= g[e + 1]; }
        hi[e / 2] = Mma<T>::pack(p0, p1);
        const float2 h = Elem<T>::unpack2(hi[e / 2]);
        lo[e / 2] = Mma<T>::pack(p0 - h.x, p1 - h.y);
      }
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) ss[bb] += (bb == b) ? sq : 0.f;
      *reinterpret_cast<uint4*>(xs + (size_t)b * A.d_in + c) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      if (SPLIT)
        *reinterpret_cast<uint4*>(xs_lo + (size_t)b * A.d_in + c) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const float t = warp_sum(ss[b]);
      if (lane == 0) red[warp][b] = t;
    }
  }
  named_bar_sync(1, kConsumers);
  if (tid < 8) {
    float v = 1.f;
    if (!skip && A.gamma != nullptr && tid < A.batch) {
      float t = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) t += red[w][tid];
      v = rsqrtf(t / (float)A.d_in + A.eps);
    }
    inv_rms[tid] = v;
  }
  if (!mlp_consume<T, 2, true, true>(A, rows_a, ring, full, empty, nst, j, part, pc_a, xs,
                                     packed_a, skip))
    return;
  named_bar_sync(1, kConsumers);
  if (!skip) {
    T* h = static_cast<T*>(A.y);
    const int nrows = rows_a.y - rows_a.x;
    for (int idx = tid; idx < nrows * A.batch; idx += kConsumers) {
      const int b = idx / nrows, r = idx - b * nrows;
      const int mt = r / 8, q = r - mt * 8;
      const float sc = inv_rms[b];
      const float v = silu(mlp_row_sum(part, nmt_a, pc_a, mt, q, b, A.batch, packed_a) * sc) *
                      (mlp_row_sum(part, nmt_a, pc_a, mt, 8 + q, b, A.batch, packed_a) * sc);
      h[(size_t)b * A.d_out + rows_a.x + r] = Elem<T>::from_f(v);
    }
    skip = !meet();
  }

  // -------------------------------------------------- phase 2: down (+ residual)
  // (d_ff > 2 chunks: gemv_mma_kernel's per-k-step variant, so the sums run in the same order)
  mlp_plain_phase<T>(D, region, ring, full, empty, nst, j, true, skip);
}

// Shared bytes after the ring: the largest phase's partials + activation stage.
int mlp_region_bytes(int batch, int d_attn, int d_model, int d_ff, int G, bool split) {
  auto plain = [&](int d_in, int d_out) {
    return (size_t)kConsumerWarps * (((d_out + G - 1) / G + 15) / 16) * 16 * batch * 4 +
           (size_t)batch * d_in * 2;
  };
  const int pc_a = split ? 2 * batch : batch;
  const size_t ra = (size_t)kConsumerWarps * (((d_ff + G - 1) / G + 7) / 8) * 16 * pc_a * 4 +
                    (size_t)batch * d_model * 2 * (split ? 2 : 1);
  size_t r = ra > plain(d_ff, d_model) ? ra : plain(d_ff, d_model);
  if (d_attn > 0 && plain(d_attn, d_model) > r) r = plain(d_attn, d_model);
  return (int)((r + 15) & ~(size_t)15);
}

template <typename T, bool PRE>
int launch_mlp(MlpArgs m, cudaStream_t st, const DeviceInfo& dev) {
  const bool split = m.g.gamma != nullptr;
  const void* kern = split ? reinterpret_cast<const void*>(mlp_block_kernel<T, true, PRE>)
                           : reinterpret_cast<const void*>(mlp_block_kernel<T, false, PRE>);
  const size_t smem = (size_t)m.nstages * (kMmaStage + 16) + m.region_bytes;
  if (int rc = allow_dynamic_smem(kern, dev, smem)) return rc;
  return launch_pdl(kern, dim3(dev.num_sms), dim3(kThreads), smem, st, &m);
}

// Shared checks and set-up of both entry points; d_attn = 0 without phase 0.
int mlp_launch(MlpArgs& m, int batch, int d_attn, int d_model, int d_ff, int dtype,
               void* workspace, size_t workspace_bytes, void* stream);

}  // namespace
}  // namespace dbk

extern "C" size_t dbk_mlp_block_workspace_bytes(void) { return 256; }

namespace dbk {
namespace {
int mlp_launch(MlpArgs& m, int batch, int d_attn, int d_model, int d_ff, int dtype,
               void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < dbk_mlp_block_workspace_bytes()) return DBK_EWORKSPACE;
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  // one CTA per SM owns rows of every GEMV (d_model, d_ff >= the SM count); gate/up
  // caches nothing in registers but keeps the two-chain k-step order of
  // gemv_mma_kernel's variant for d_in <= 2 chunks
  if (batch > 4 || d_model % 16 != 0 || d_ff % 16 != 0 || d_attn % 16 != 0 ||
      d_model > 2 * kMmaKC || d_model < dev.num_sms || d_ff < dev.num_sms)
    return DBK_ESHAPE;
  auto chunks = [](int d_in) { return (d_in + kMmaKC - 1) / kMmaKC; };
  m.g.batch = batch; m.g.d_in = d_model; m.g.d_out = d_ff;
  m.g.nchunks = chunks(d_model);
  m.g.pcols = m.g.gamma ? 2 * batch : batch;
  m.d.x = m.g.y;
  m.d.batch = batch; m.d.d_in = d_ff; m.d.d_out = d_model;
  m.d.nchunks = chunks(d_ff);
  m.d.pcols = batch;
  if (d_attn > 0) {
    m.o.batch = batch; m.o.d_in = d_attn; m.o.d_out = d_model;
    m.o.nchunks = chunks(d_attn);
    m.o.pcols = batch;
  }
  m.sync = static_cast<int*>(workspace);
  m.region_bytes = mlp_region_bytes(batch, d_attn, d_model, d_ff, dev.num_sms,
                                    m.g.gamma != nullptr);
  m.nstages = 0;
  for (int nst = kMmaStages; nst >= 2; --nst)
    if ((size_t)nst * (kMmaStage + 16) + m.region_bytes <= (size_t)dev.max_smem_optin - 1024) {
      m.nstages = nst;
      break;
    }
  if (m.nstages == 0) return DBK_ESHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d_attn > 0)
    return dtype == DBK_F16 ? launch_mlp<__half, true>(m, st, dev)
                            : launch_mlp<__nv_bfloat16, true>(m, st, dev);
  return dtype == DBK_F16 ? launch_mlp<__half, false>(m, st, dev)
                          : launch_mlp<__nv_bfloat16, false>(m, st, dev);
}
}  // namespace
}  // namespace dbk

extern "C" int dbk_mlp_block(const void* x, const void* gamma, const void* Wg, const void* Wu,
                             const void* Wd, const void* residual, void* h, void* y, int batch,
                             int d_model, int d_ff, float eps, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (int rc = check_common(x, Wg, h, batch, d_model, d_ff, dtype)) return rc;
  if (!Wu || !Wd || !y) return DBK_ENULL;
  if (!aligned16(Wu) || !aligned16(Wd) || !aligned16(h) || (gamma && !aligned16(gamma)))
    return DBK_EALIGN;
  MlpArgs m{};
  m.g.x = x; m.g.gamma = gamma; m.g.w0 = Wg; m.g.w1 = Wu; m.g.y = h; m.g.eps = eps;
  m.d.w0 = Wd; m.d.residual = residual; m.d.y = y;
  return mlp_launch(m, batch, 0, d_model, d_ff, dtype, workspace, workspace_bytes, stream);
}

extern "C" int dbk_oproj_mlp_block(const void* attn, const void* Wo, const void* x,
                                   const void* gamma, const void* Wg, const void* Wu,
                                   const void* Wd, void* h_attn, void* h, void* y, int batch,
                                   int d_attn, int d_model, int d_ff, float eps, int dtype,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_common(attn, Wo, h_attn, batch, d_attn, d_model, dtype)) return rc;
  if (int rc = check_common(h_attn, Wg, h, batch, d_model, d_ff, dtype)) return rc;
  if (!x || !Wu || !Wd || !y) return DBK_ENULL;
  if (!aligned16(Wu) || !aligned16(Wd) || !aligned16(h) || !aligned16(h_attn) ||
      (gamma && !aligned16(gamma)))
    return DBK_EALIGN;
  MlpArgs m{};
  m.o.x = attn; m.o.w0 = Wo; m.o.residual = x; m.o.y = h_attn;
  m.g.x = h_attn; m.g.gamma = gamma; m.g.w0 = Wg; m.g.w1 = Wu; m.g.y = h; m.g.eps = eps;
  m.d.w0 = Wd; m.d.residual = h_attn; m.d.y = y;
  return mlp_launch(m, batch, d_attn, d_model, d_ff, dtype, workspace, workspace_bytes, stream);
}
