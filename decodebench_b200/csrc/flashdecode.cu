// flashdecode.cu - split-KV FlashDecode for one query token per sequence.
//
// Semantics (per sequence b, query head h, kv head hk = h / G, G = Hq / Hkv):
//   s_t = scale * q[b,h,:] . K[b,hk,t,:],  p = softmax(s over t < len_b),
//   out[b,h,:] = sum_t p_t V[b,hk,t,:]
// following the reference's fused f4_partial_kernel + f4_reduce_kernel
// (validation/src/kernels/fused/f4.cu:173-319): per split an unnormalised
// (m, l, o) partial from an online softmax, then a log-sum-exp merge
// m* = max m_s, o = sum e^(m_s-m*) o_s / sum e^(m_s-m*) l_s  (f4.cu:294-319).
//
// Design (B200):
//   * Schedule: the (b, kv head) rows of 64-token tiles are laid end to end and
//     CTA c (one per SM, persistent) takes tiles [c*T/grid, (c+1)*T/grid): every
//     SM gets the same number of tiles (within one) whatever the sequence
//     lengths, and a CTA's range cuts at most two rows, so it emits at most two
//     partials. A row covered by one CTA is written directly; otherwise the last
//     CTA to finish a row (self-resetting atomic counter) merges its partials.
//   * A producer warp streams K and V tiles into a ring of 32 KB stages tracked
//     by mbarriers, gathering a paged cache ([page, kv_head, page_size, 128],
//     per-head page blocks contiguous) through the int32 page table.
//   * Tensor-core path (any G, whenever 16-token boxes stay inside pages): the
//     G query heads of a kv head form the first G of the M=16 rows of
//     mma.m16n8k16 tiles. K/V arrive by tiled TMA (cp.async.bulk.tensor over a
//     3-D view [2][rows][64], so each box reads 16 whole rows = 4 KB)
//     with a 128-byte swizzle so ldmatrix reads are conflict free; two groups of four
//     warps take alternate stages, each warp 16 tokens: S = Q K^T (fp32
//     accumulate), online softmax in registers, O += P V with P split into a
//     high and a low 16-bit part so the probabilities keep fp32-like accuracy.
//     (On CUDA cores the 16-bit -> fp32 conversions of K and V alone cap the
//     rate near half of HBM bandwidth; the tensor cores take them for free.)
//   * CUDA-core path (G <= 2 with page sizes that are not multiples of 16):
//     cp.async.bulk page runs; eight consumer warps each take 8 tokens of a tile
//     with their own online-softmax state.
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

constexpr int kD = 128;                 // head_dim
constexpr int kTile = 64;               // tokens per stage
constexpr int kWarps = 8;
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kMaxStages = 6;
constexpr int kMinBoxRows = 16;         // smallest TMA box height (tokens) on the tensor-core path
constexpr int kMaxBatchSmem = 1024;     // sequences whose tile offsets live in shared memory
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMrg = kD + 4;            // merge-row stride: o[128], m, l, pad (16-byte rows)

struct FdArgs {
  CUtensorMap kmap;       // tensor-core path: 2-D view [rows, 128] of the K cache
  CUtensorMap vmap;
  const void* q;          // [batch, Hq, 128]
  const void* k;          // contiguous [batch, Hkv, max_len, 128] | paged [pages, Hkv, ps, 128]
  const void* v;
  const int32_t* pages;   // [batch, max_pages] or nullptr
  const int32_t* lens;    // [batch] or nullptr
  void* out;              // [batch, Hq, 128]
  float* part_o;          // [2 * grid, G, 128]
  float2* part_ml;        // [2 * grid, G]
  int* done;              // [batch * Hkv] arrival counters (zero between launches)
  int batch, hq, hkv, max_len, page_size, max_pages;
  float qscale;           // scale * log2(e)
  int nstages;
  int box_shift;          // tensor-core path: log2 of the TMA box height (16, 32 or 64 tokens)
};

// Shared-memory line (128 bytes) holding dims [64 h, 64 h + 64) of token `tok` of
// a stage on the tensor-core path: boxes of 2^sh tokens land one after another,
// each as [half][row] lines. The 128-byte swizzle phase of a line is its index
// mod 8 = tok mod 8, so the 8 rows of an ldmatrix block never share banks.
__device__ __forceinline__ int kv_line(int tok, int h, int sh) {
  return ((tok >> sh) << (sh + 1)) + (h << sh) + (tok & ((1 << sh) - 1));
}

__device__ __forceinline__ int seq_len(const FdArgs& a, int b) {
  return a.lens ? min(max(a.lens[b], 0), a.max_len) : a.max_len;
}

// Tile offsets: tile0[b] = first global tile of (b, kv head 0); row (b, hk)
// starts at tile0[b] + hk * ntiles(b). Computed by warp 0 with a warp scan.
__device__ void build_tile_offsets(const FdArgs& a, int* tile0, int lane) {
  int carry = 0;
  for (int base = 0; base < a.batch; base += 32) {
    const int b = base + lane;
    const int nt = (b < a.batch) ? ((seq_len(a, b) + kTile - 1) / kTile) * a.hkv : 0;
    int incl = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (b < a.batch) tile0[b] = carry + incl - nt;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) tile0[a.batch] = carry;
}

// Walks the global tile sequence: current (b, hk, tile within row).
struct TileWalker {
  const FdArgs& a;
  const int* tile0;
  int b, hk, tt, ntb, len;   // ntb = tiles per row of sequence b
  __device__ TileWalker(const FdArgs& args, const int* t0, int u) : a(args), tile0(t0) {
    int lo = 0, hi = a.batch - 1;             // last b with tile0[b] <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tile0[mid] <= u) lo = mid; else hi = mid - 1;
    }
    b = lo;
    len = seq_len(a, b);
    ntb = (len + kTile - 1) / kTile;
    while (ntb == 0) { ++b; len = seq_len(a, b); ntb = (len + kTile - 1) / kTile; }
    const int off = u - tile0[b];
    hk = off / ntb;
    tt = off - hk * ntb;
  }
  __device__ void next() {
    if (++tt < ntb) return;
    tt = 0;
    if (++hk < a.hkv) return;
    hk = 0;
    do { ++b; if (b >= a.batch) return; len = seq_len(a, b); ntb = (len + kTile - 1) / kTile; }
    while (ntb == 0);
  }
  __device__ int row() const { return b * a.hkv + hk; }
  __device__ int row_start() const { return tile0[b] + hk * ntb; }
  __device__ int ntok() const { return min(kTile, len - tt * kTile); }
};

// Row index (into the 2-D cache view) of token t of (b, hk), and tokens left
// in its page run.
__device__ __forceinline__ int64_t kv_rowidx(const FdArgs& a, int b, int hk, int t, int* run) {
  if (a.pages == nullptr) {
    *run = 1 << 30;
    return ((int64_t)b * a.hkv + hk) * a.max_len + t;
  }
  const int pg = a.pages[(size_t)b * a.max_pages + t / a.page_size];
  const int off = t % a.page_size;
  *run = a.page_size - off;
  return ((int64_t)pg * a.hkv + hk) * a.page_size + off;
}

// CTA whose tile range contains global tile u (ranges [c*T/grid, (c+1)*T/grid)).
__device__ __forceinline__ int owner(int64_t u, int64_t T, int64_t grid) {
  return (int)(((u + 1) * grid + T - 1) / T - 1);
}
__device__ __forceinline__ int range_start(int64_t c, int64_t T, int64_t grid) {
  return (int)(c * T / grid);
}

// Arrival at a row's counter: releases this CTA's partial (the caller's
// barrier orders every consumer thread's partial stores before it). Nothing
// comes back, so the CTA does not wait on the round trip.
__device__ __forceinline__ void arrive_release(int* p) {
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p) : "memory");
}

// Bounded wait (acquire) until *p == v; records kDevTimeoutMerge and gives up.
__device__ __forceinline__ bool wait_count(const int* p, int v) {
  uint32_t n = 0;
  const uint32_t lim = spin_limit();
  while (ld_acquire_gpu(p) != v) {
    if (++n >= lim) {
      record_error(kDevTimeoutMerge);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Log-sum-exp merge of row (b, hk)'s partials (reference f4_reduce_kernel,
// validation/src/kernels/fused/f4.cu:294-319), by the consumer threads of the
// CTA that holds the row's last tile, once the others have arrived:
// M = max_c m_c, out = sum_c 2^(m_c - M) o_c / sum_c 2^(m_c - M) l_c (m in log2
// units), contributors in CTA order (results do not depend on timing). The
// contributors' workspace slots are worked out once into shared memory (`slots`,
// np ints); then every thread issues all of its loads -- (m, l) and o of every
// contributor for its outputs -- before using any of them, so a merge costs
// about one L2 round trip whatever the number of contributors.
template <typename T, int G>
__device__ void merge_row(const FdArgs& a, int b, int hk, int rs, int ntb, int64_t Ttot,
                          int grid, int tid, int* slots) {
  T* out = static_cast<T*>(a.out);
  const int c_first = owner(rs, Ttot, grid), c_last = owner(rs + ntb - 1, Ttot, grid);
  const int np = c_last - c_first + 1;
  for (int i = tid; i < np; i += kConsumers) {
    const int c = c_first + i;
    slots[i] = 2 * c + (range_start(c, Ttot, grid) >= rs ? 0 : 1);
  }
  named_bar_sync(1, kConsumers);
  for (int idx = tid; idx < G * kD; idx += kConsumers) {
    const int g = idx / kD, d = idx - g * kD;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int c0 = 0; c0 < np; c0 += 16) {
      float mc[16], lc[16], oc[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        mc[k] = -INFINITY; lc[k] = 0.f; oc[k] = 0.f;
        if (c0 + k < np) {
          const int sl = slots[c0 + k];
          const float2 ml = __ldcg(&a.part_ml[(size_t)sl * G + g]);
          mc[k] = ml.x; lc[k] = ml.y;
          oc[k] = __ldcg(&a.part_o[((size_t)sl * G + g) * kD + d]);
        }
      }
      float Mn = M;
#pragma unroll
      for (int k = 0; k < 16; ++k) Mn = fmaxf(Mn, mc[k]);
      const float sc = (M == -INFINITY) ? 0.f : exp2f(M - Mn);
      L *= sc;
      O *= sc;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float f = (lc[k] > 0.f) ? exp2f(mc[k] - Mn) : 0.f;
        L = fmaf(f, lc[k], L);
        O = fmaf(f, oc[k], O);
      }
      M = Mn;
    }
    out[((size_t)b * a.hq + (size_t)hk * G + g) * kD + d] = Elem<T>::from_f(O / L);
  }
}

// The same merge with the row's partials first staged in shared memory: the
// consumer threads copy every contributor's (m, l) and o into `buf` (the ring,
// idle once the CTA's tiles are consumed) with independent 16-byte loads -- about
// one L2 round trip for the whole row -- then the weights and sums come from
// shared memory. `buf` must hold np * G * (kD + 2) floats (merge_staged_fits).
__host__ __device__ inline bool merge_staged_fits(int np, int G, size_t buf_bytes) {
  return (size_t)np * G * (kD + 2) * sizeof(float) + (size_t)G * sizeof(float) <= buf_bytes;
}

template <typename T, int G>
__device__ void merge_row_staged(const FdArgs& a, int b, int hk, int rs, int ntb, int64_t Ttot,
                                 int grid, int tid, int* slots, float* buf) {
  T* out = static_cast<T*>(a.out);
  const int c_first = owner(rs, Ttot, grid), c_last = owner(rs + ntb - 1, Ttot, grid);
  const int np = c_last - c_first + 1;
  float* o_s = buf;                                   // [np][G][kD]
  float* w_s = o_s + (size_t)np * G * kD;             // [np][G]: m, then the weight
  float* l_s = w_s + np * G;                          // [np][G]
  float* inv_l = l_s + np * G;                        // [G]
  for (int i = tid; i < np; i += kConsumers) {
    const int c = c_first + i;
    slots[i] = 2 * c + (range_start(c, Ttot, grid) >= rs ? 0 : 1);
  }
  named_bar_sync(1, kConsumers);
  constexpr int kV = G * kD / 4;                      // float4 per contributor
  const int nv = np * kV, nml = np * G;
  // Every (m, l) pair and every float4 of o in flight at once: the loads of up to
  // 16 float4 per thread go to registers before any shared-memory store (a store
  // through the generic pointer could alias a later load, so loads and stores
  // interleaved would run one round trip each).
  float2 ml0 = make_float2(0.f, 0.f);
  if (tid < nml) ml0 = __ldcg(&a.part_ml[(size_t)slots[tid / G] * G + (tid % G)]);
  for (int base = tid; base < nv; base += 16 * kConsumers) {
    float4 r[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int v = base + k * kConsumers;
      if (v < nv) {
        const int c = v / kV, rr = v - c * kV;
        r[k] = __ldcg(reinterpret_cast<const float4*>(a.part_o + (size_t)slots[c] * G * kD) + rr);
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int v = base + k * kConsumers;
      if (v < nv) reinterpret_cast<float4*>(o_s)[v] = r[k];
    }
  }
  if (tid < nml) {
    w_s[tid] = ml0.x;
    l_s[tid] = ml0.y;
  }
  for (int i = kConsumers + tid; i < nml; i += kConsumers) {
    const float2 ml = __ldcg(&a.part_ml[(size_t)slots[i / G] * G + (i % G)]);
    w_s[i] = ml.x;
    l_s[i] = ml.y;
  }
  named_bar_sync(1, kConsumers);
  DBK_MARK(tid == 0, 13);
  // Weights: warp g handles head g, its lanes the contributors.
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += kConsumers / 32) {
      float M = -INFINITY;
      for (int c = lane; c < np; c += 32) M = fmaxf(M, w_s[c * G + g]);
      M = warp_max(M);
      float L = 0.f;
      for (int c = lane; c < np; c += 32) {
        const float lc = l_s[c * G + g];
        const float f = (lc > 0.f) ? exp2f(w_s[c * G + g] - M) : 0.f;
        w_s[c * G + g] = f;
        L = fmaf(f, lc, L);
      }
      L = warp_sum(L);
      if (lane == 0) inv_l[g] = 1.f / L;
    }
  }
  named_bar_sync(1, kConsumers);
  DBK_MARK(tid == 0, 14);
  for (int idx = tid; idx < G * kD; idx += kConsumers) {
    const int g = idx / kD;
    float O = 0.f;
    for (int c = 0; c < np; ++c) O = fmaf(w_s[c * G + g], o_s[(size_t)c * G * kD + idx], O);
    out[((size_t)b * a.hq + (size_t)hk * G) * kD + idx] = Elem<T>::from_f(O * inv_l[g]);
  }
}

// ------------------------------------------------------------------ kernel
template <typename T, int G, bool kMma>
__global__ void __launch_bounds__(kThreads, 1) flashdecode_kernel(const __grid_constant__ FdArgs a) {
  constexpr int kStage = 2 * kTile * kD * (int)sizeof(T);   // K tile | V tile (32 KB)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.nstages * kStage);
  uint64_t* empty = full + a.nstages;
  // Segment-end combine buffer: one slot per warp on the CUDA-core path; on the
  // tensor-core path warps 4-7 first fold their state into warps 0-3, so 4 slots.
  constexpr int kMrgSlots = kMma ? kWarps / 2 : kWarps;
  float* mrg = reinterpret_cast<float*>(empty + a.nstages);              // [kMrgSlots][G][kMrg]
  int* tile0 = reinterpret_cast<int*>(mrg + kMrgSlots * G * kMrg);        // [batch + 1]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  DBK_TRACE_BEGIN();
  DBK_MARK(tid == 0, 0);
  if (tid == 0) {
    // A stage is released by every consumer warp (CUDA-core path) or by the
    // four warps of the group that consumed it (tensor-core path).
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMma ? 4 : kWarps);
    }
    fence_barrier_init();
  }
  if (warp == 0) build_tile_offsets(a, tile0, lane);
  __syncthreads();
  DBK_MARK(tid == 0, 1);
  asm volatile("griddepcontrol.launch_dependents;");

  // Sequences of length 0 have no tiles: their output is defined as zeros.
  if (blockIdx.x == 0 && a.lens != nullptr && warp < kWarps) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    T* out = static_cast<T*>(a.out);
    for (int b = 0; b < a.batch; ++b)
      if (seq_len(a, b) == 0)
        for (int i = tid; i < a.hq * kD; i += kConsumers)
          out[(size_t)b * a.hq * kD + i] = Elem<T>::from_f(0.f);
  }

  // Effective grid: never more CTAs than tiles, so every range is non-empty and
  // the CTAs covering a row are exactly owner(first tile) .. owner(last tile).
  const int64_t Ttot = tile0[a.batch];
  if (Ttot == 0 || blockIdx.x >= Ttot) return;
  const int grid = (int)min((int64_t)gridDim.x, Ttot);
  const int u0 = range_start(blockIdx.x, Ttot, grid);
  const int u1 = range_start(blockIdx.x + 1, Ttot, grid);
  __shared__ int s_last;

  if (warp == kWarps) {
    // ------------------------------------------------------------ producer
    // The whole warp gathers: for each group of 32 tiles, lane l looks up the
    // cache rows of tile (group + l) in parallel (one page-table latency per
    // 32 tiles instead of one per box); lane 0 then issues the copies in order.
    const uint64_t pol = policy_evict_first();
    if constexpr (kMma) {
      if (lane == 0) { prefetch_tmap(&a.kmap); prefetch_tmap(&a.vmap); }
    }
    const T* K = static_cast<const T*>(a.k);
    const T* V = static_cast<const T*>(a.v);
    const bool boxed = (a.pages == nullptr) || (a.page_size % kMinBoxRows == 0);
    const int br = 1 << a.box_shift;          // tokens per TMA box (tensor-core path)
    if (!boxed) {
      // page_size not a multiple of 16 (CUDA-core path only): page runs one by one
      if (lane != 0) return;
      TileWalker w(a, tile0, u0);
      for (int u = u0, j = 0; u < u1; ++u, ++j, w.next()) {
        const int s = j % a.nstages;
        if (j >= a.nstages && !DBK_TIMED_WAIT(lane == 0, 10, mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty)))
          return;
        const int n = w.ntok();
        uint8_t* dk = smem + (size_t)s * kStage;
        uint8_t* dv = dk + kStage / 2;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * n * kD * sizeof(T)));
        for (int t = 0; t < n;) {
          int run;
          const int64_t r = kv_rowidx(a, w.b, w.hk, w.tt * kTile + t, &run);
          const int m = min(run, n - t);
          const uint32_t bytes = (uint32_t)(m * kD * sizeof(T));
          bulk_g2s(dk + (size_t)t * kD * sizeof(T), K + r * kD, bytes, &full[s], pol);
          bulk_g2s(dv + (size_t)t * kD * sizeof(T), V + r * kD, bytes, &full[s], pol);
          t += m;
        }
      }
      return;
    }
    TileWalker w(a, tile0, min(u0 + lane, u1 - 1));
    for (int g0 = u0; g0 < u1; g0 += 32) {
      // this lane's tile: g0 + lane
      int n_l = 0;
      int64_t r_l[4] = {0, 0, 0, 0};
      if (g0 + lane < u1) {
        n_l = w.ntok();
#pragma unroll
        for (int bx = 0; bx < 4; ++bx) {
          int run;
          if (bx * br < n_l) r_l[bx] = kv_rowidx(a, w.b, w.hk, w.tt * kTile + bx * br, &run);
        }
      }
      const int cnt = min(32, u1 - g0);
      bool gave_up = false;
      for (int i = 0; i < cnt; ++i) {
        const int n = __shfl_sync(0xffffffffu, n_l, i);
        int64_t r[4];
#pragma unroll
        for (int bx = 0; bx < 4; ++bx) r[bx] = __shfl_sync(0xffffffffu, r_l[bx], i);
        if (lane == 0 && !gave_up) {
          const int j = g0 - u0 + i;
          const int s = j % a.nstages;
          if (j >= a.nstages &&
              !DBK_TIMED_WAIT(lane == 0, 10, mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty)))
            gave_up = true;   // the error is recorded; leave after this group
          else {
            uint8_t* dk = smem + (size_t)s * kStage;
            uint8_t* dv = dk + kStage / 2;
            if constexpr (kMma) {
              // boxes of br tokens x both dim halves, for K and for V (one 16 KB copy
              // each when a box covers the whole 64-token tile)
              const int boxes = (n + br - 1) / br;
              mbar_arrive_expect_tx(&full[s], (uint32_t)(boxes * br * 512));
#pragma unroll
              for (int bx = 0; bx < 4; ++bx) {
                if (bx >= boxes) break;
                tma_load_3d(dk + bx * br * 256, &a.kmap, 0, (int)r[bx], 0, &full[s], pol);
                tma_load_3d(dv + bx * br * 256, &a.vmap, 0, (int)r[bx], 0, &full[s], pol);
              }
            } else {
              const int boxes = (n + kMinBoxRows - 1) / kMinBoxRows;
              mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * n * kD * sizeof(T)));
#pragma unroll
              for (int bx = 0; bx < 4; ++bx) {
                if (bx >= boxes) break;
                const int m = min(kMinBoxRows, n - bx * kMinBoxRows);
                const uint32_t bytes = (uint32_t)(m * kD * sizeof(T));
                const size_t so = (size_t)bx * kMinBoxRows * kD * sizeof(T);
                bulk_g2s(dk + so, K + r[bx] * kD, bytes, &full[s], pol);
                bulk_g2s(dv + so, V + r[bx] * kD, bytes, &full[s], pol);
              }
            }
          }
        }
      }
      if (__shfl_sync(0xffffffffu, gave_up ? 1 : 0, 0)) return;
      for (int k = 0; k < 32; ++k) w.next();
      DBK_MARK(lane == 0 && g0 == u0, 8);
    }
    DBK_MARK(lane == 0, 9);
    return;
  }

  // -------------------------------------------------------------- consumers
  asm volatile("griddepcontrol.wait;" ::: "memory");
  DBK_MARK(tid == 0, 2);
  const T* q = static_cast<const T*>(a.q);
  T* out = static_cast<T*>(a.out);

  // Per-warp online-softmax state. CUDA-core path: lane owns dims 4l..4l+3 of
  // each of the G heads. Tensor-core path: lane owns heads 2*(lane%4) + {0,1}
  // and dims 16*mt + lane/4 (+8) for mt < 8 (the O^T accumulator fragment).
  constexpr int kO = kMma ? 32 : 4 * G;
  constexpr int kS = kMma ? 2 : G;
  float o[kO], m[kS], l[kS];
  float qr[kMma ? 1 : G][4];
  uint32_t qa[kMma ? 8 : 1][2];     // B fragments of Q^T (columns = heads), 8 k-steps
  const int grp = warp >> 2, wi = warp & 3;
  const int r_head = lane >> 2;     // tensor-core path: the head whose Q this lane loads

  TileWalker w(a, tile0, u0);
  int seg_first = u0;
  // The split row whose last tile this CTA holds (at most one: a range's first
  // segment). This CTA merges it after its own tiles, so the merge never stalls
  // the stream; the row's other contributors only announce their partials.
  int pend_b = -1, pend_hk = 0, pend_rs = 0, pend_ntb = 0, pend_np = 0;
  for (int u = u0, j = 0; u < u1; ++u, ++j, w.next()) {
    const int s = j % a.nstages;
    const bool seg_begin = (u == u0) || (w.tt == 0);
    const bool seg_end = (u == u1 - 1) || (w.tt == w.ntb - 1);
    if (seg_begin) {
      seg_first = u;
      const T* qb = q + ((size_t)w.b * a.hq + (size_t)w.hk * G) * kD;
      if constexpr (kMma) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if (r_head < G) {
            const T* qp = qb + (size_t)r_head * kD + kk * 16 + 2 * (lane & 3);
            qa[kk][0] = *reinterpret_cast<const uint32_t*>(qp);
            qa[kk][1] = *reinterpret_cast<const uint32_t*>(qp + 8);
          } else {
            qa[kk][0] = qa[kk][1] = 0u;
          }
        }
        m[0] = m[1] = -INFINITY; l[0] = l[1] = 0.f;
#pragma unroll
        for (int e = 0; e < kO; ++e) o[e] = 0.f;
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const uint2 raw = *reinterpret_cast<const uint2*>(qb + (size_t)g * kD + 4 * lane);
          const float2 lo = Elem<T>::unpack2(raw.x), hi = Elem<T>::unpack2(raw.y);
          qr[g][0] = lo.x * a.qscale; qr[g][1] = lo.y * a.qscale;
          qr[g][2] = hi.x * a.qscale; qr[g][3] = hi.y * a.qscale;
          m[g] = -INFINITY; l[g] = 0.f;
          o[4 * g] = o[4 * g + 1] = o[4 * g + 2] = o[4 * g + 3] = 0.f;
        }
      }
    }

    const int n = w.ntok();
    const uint32_t kst = smem_u32(smem + (size_t)s * kStage);
    const uint32_t vst = kst + kStage / 2;
    if constexpr (kMma) {
      if ((j & 1) == grp) {
        if (!DBK_TIMED_WAIT(tid == 0, 11, mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull))) return;
        DBK_MARK(lane == 0 && warp == 0 && j == 0, 3);
        DBK_MARK(lane == 0 && warp == 0 && j == 16, 4);
        const int t0 = wi * 16;                 // this warp's 16 tokens
        if (t0 < n) {
          if (n < kTile && t0 + 16 > n) {
            // ragged tail: zero this warp's V rows >= n (their probabilities are 0,
            // but the rows may hold stale or out-of-sequence data)
            for (int r = max(n, t0); r < t0 + 16; ++r) {
              uint8_t* p0 = smem + (size_t)s * kStage + kStage / 2 +
                            kv_line(r, lane >> 4, a.box_shift) * 128;
              reinterpret_cast<uint4*>(p0)[lane & 7] = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();   // order these writes before the next TMA refill
            __syncwarp();
          }
          if (w.tt == w.ntb - 1 && n - 1 >= t0 && n - 1 < t0 + 16) {
            // The newest token's K/V may come from the kernel just before this one
            // (e.g. dbk_qkv_rope_append): the producer streamed this tile before
            // that kernel had finished, so re-read that one row pair now, after
            // griddepcontrol.wait. Lane l < 16: 16 bytes of K; l >= 16: of V.
            const int tok = n - 1, cc = lane & 15;
            int run;
            const int64_t rr = kv_rowidx(a, w.b, w.hk, w.tt * kTile + tok, &run);
            const T* src = static_cast<const T*>(lane < 16 ? a.k : a.v) + rr * kD + cc * 8;
            const int line = kv_line(tok, cc >> 3, a.box_shift);
            uint8_t* dst = smem + (size_t)s * kStage + (lane < 16 ? 0 : kStage / 2) + line * 128 +
                           (((cc & 7) ^ (line & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = __ldcg(reinterpret_cast<const uint4*>(src));
            fence_proxy_async_smem();
            __syncwarp();
          }
          // S^T[16 tokens x 8 heads] = K Q^T: tokens are the M rows (no padding);
          // heads 0..G-1 are the N columns. Two accumulators halve the MMA chain.
          // The K loads are issued back to back before the MMAs, and the V loads
          // right after them (they do not depend on the softmax), so their
          // shared-memory latencies overlap with each other and with the softmax.
          float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t va[8][4];
          {
            uint32_t ka[8][4];
            const int tok = t0 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const int chunk = 2 * kk + (lane >> 4);     // 16-byte chunk of the 256-byte row
              const int h = chunk >> 3, c = chunk & 7;
              const int line = kv_line(tok, h, a.box_shift);
              ldsm_x4(kst + line * 128 + ((c ^ (line & 7)) << 4), ka[kk]);
            }
            const int vtok = t0 + (lane & 7) + 8 * (lane >> 4);
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {        // 16-dim m-tiles of V^T
              const int chunk = 2 * mt + ((lane >> 3) & 1);
              const int h = chunk >> 3, c = chunk & 7;
              const int line = kv_line(vtok, h, a.box_shift);
              ldsm_x4_t(vst + line * 128 + ((c ^ (line & 7)) << 4), va[mt]);
            }
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              Mma<T>::run((kk & 1) ? sb : sa, ka[kk][0], ka[kk][1], ka[kk][2], ka[kk][3],
                          qa[kk][0], qa[kk][1]);
          }
          // fragment: sc[0..1] = tokens t0+g, heads 2q, 2q+1; sc[2..3] = tokens t0+g+8
          const int g = lane >> 2;
          float sc[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = t0 + g + (e >> 1) * 8;
            sc[e] = (tok < n) ? (sa[e] + sb[e]) * a.qscale : -INFINITY;
          }
          // online softmax per head (column): reduce over the 8 lanes sharing qd
          float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
          for (int o2 = 4; o2 < 32; o2 <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o2));
          }
          mx0 = fmaxf(mx0, m[0]);
          mx1 = fmaxf(mx1, m[1]);
          const float al0 = exp2f(m[0] - mx0), al1 = exp2f(m[1] - mx1);
          m[0] = mx0; m[1] = mx1;
          sc[0] = exp2f(sc[0] - mx0); sc[2] = exp2f(sc[2] - mx0);
          sc[1] = exp2f(sc[1] - mx1); sc[3] = exp2f(sc[3] - mx1);
          l[0] = l[0] * al0 + sc[0] + sc[2];      // lane-partial column sums
          l[1] = l[1] * al1 + sc[1] + sc[3];
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[4 * mt] *= al0; o[4 * mt + 2] *= al0;
            o[4 * mt + 1] *= al1; o[4 * mt + 3] *= al1;
          }
          // P^T as the B operand of O^T += V^T P^T: transpose the 8x8 blocks of
          // the S^T fragment in registers (tokens 0..7 -> b0, 8..15 -> b1), with a
          // high and a low 16-bit part for bf16.
          const uint32_t ph0 = movmatrix_trans(Mma<T>::pack(sc[0], sc[1]));
          const uint32_t ph1 = movmatrix_trans(Mma<T>::pack(sc[2], sc[3]));
          uint32_t pl0 = 0u, pl1 = 0u;
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            const float2 h0 = Elem<T>::unpack2(Mma<T>::pack(sc[0], sc[1]));
            const float2 h1 = Elem<T>::unpack2(Mma<T>::pack(sc[2], sc[3]));
            pl0 = movmatrix_trans(Mma<T>::pack(sc[0] - h0.x, sc[1] - h0.y));
            pl1 = movmatrix_trans(Mma<T>::pack(sc[2] - h1.x, sc[3] - h1.y));
          }
          // O^T[128 dims x 8 heads] += V^T[dims x 16 tokens] P^T[16 tokens x 8 heads]
          {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {        // 16-dim m-tiles
              float* d = &o[4 * mt];
              float acc4[4] = {d[0], d[1], d[2], d[3]};
              Mma<T>::run(acc4, va[mt][0], va[mt][1], va[mt][2], va[mt][3], ph0, ph1);
              d[0] = acc4[0]; d[1] = acc4[1]; d[2] = acc4[2]; d[3] = acc4[3];
            }
            if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
              for (int mt = 0; mt < 8; ++mt) {
                float* d = &o[4 * mt];
                float acc4[4] = {d[0], d[1], d[2], d[3]};
                Mma<T>::run(acc4, va[mt][0], va[mt][1], va[mt][2], va[mt][3], pl0, pl1);
                d[0] = acc4[0]; d[1] = acc4[1]; d[2] = acc4[2]; d[3] = acc4[3];
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    } else {
      if (!DBK_TIMED_WAIT(tid == 0, 11, mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull))) return;
      const int mine = min(8, n - warp * 8);           // tokens of this warp
      if (w.tt == w.ntb - 1 && n - 1 >= warp * 8 && n - 1 < warp * 8 + 8) {
        // newest token re-read after griddepcontrol.wait (see the tensor-core path)
        const int tok = n - 1, cc = lane & 15;
        int run;
        const int64_t rr = kv_rowidx(a, w.b, w.hk, w.tt * kTile + tok, &run);
        const T* src = static_cast<const T*>(lane < 16 ? a.k : a.v) + rr * kD + cc * 8;
        uint8_t* dst = smem + (size_t)s * kStage + (lane < 16 ? 0 : kStage / 2) +
                       (size_t)tok * kD * sizeof(T) + cc * 16;
        *reinterpret_cast<uint4*>(dst) = __ldcg(reinterpret_cast<const uint4*>(src));
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (mine > 0) {
        const uint32_t kbase = kst + (uint32_t)((warp * 8) * kD + 4 * lane) * sizeof(T);
        const uint32_t vbase = kbase + kStage / 2;
        float sc[8][G];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < mine) {
            uint2 kv;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                         : "=r"(kv.x), "=r"(kv.y) : "r"(kbase + t * kD * (int)sizeof(T)));
            const float2 k01 = Elem<T>::unpack2(kv.x), k23 = Elem<T>::unpack2(kv.y);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              float d = qr[g][0] * k01.x;
              d = fmaf(qr[g][1], k01.y, d);
              d = fmaf(qr[g][2], k23.x, d);
              d = fmaf(qr[g][3], k23.y, d);
              sc[t][g] = warp_sum(d);
            }
          } else {
#pragma unroll
            for (int g = 0; g < G; ++g) sc[t][g] = -INFINITY;
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float mx = m[g];
#pragma unroll
          for (int t = 0; t < 8; ++t) mx = fmaxf(mx, sc[t][g]);
          const float alpha = exp2f(m[g] - mx);
          m[g] = mx;
          l[g] *= alpha;
#pragma unroll
          for (int e = 0; e < 4; ++e) o[4 * g + e] *= alpha;
#pragma unroll
          for (int t = 0; t < 8; ++t) sc[t][g] = exp2f(sc[t][g] - mx);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < mine) {
            uint2 vv;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                         : "=r"(vv.x), "=r"(vv.y) : "r"(vbase + t * kD * (int)sizeof(T)));
            const float2 v01 = Elem<T>::unpack2(vv.x), v23 = Elem<T>::unpack2(vv.y);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float p = sc[t][g];
              l[g] += p;
              o[4 * g] = fmaf(p, v01.x, o[4 * g]);
              o[4 * g + 1] = fmaf(p, v01.y, o[4 * g + 1]);
              o[4 * g + 2] = fmaf(p, v23.x, o[4 * g + 2]);
              o[4 * g + 3] = fmaf(p, v23.y, o[4 * g + 3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!seg_end) continue;
    DBK_MARK(tid == 0, 5);

    // ---- segment done: merge the 8 warps' states in shared memory
    named_bar_sync(1, kConsumers);     // readers of the previous segment's mrg are done
    if constexpr (kMma) {
      // Round 1: warps 4-7 store their (o, m, l); warps 0-3 fold their partner's state
      // (warp w + 4, same fragment layout) into their own and store the result.
      const int g8 = lane >> 2, qd = lane & 3;
      float lsum[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        lsum[e] = l[e];
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) lsum[e] += __shfl_xor_sync(0xffffffffu, lsum[e], o2);
      }
      if (warp >= kWarps / 2) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int head = 2 * qd + e;
          if (head < G) {
            float* dst = mrg + ((warp - kWarps / 2) * G + head) * kMrg;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              dst[16 * mt + g8] = o[4 * mt + e];
              dst[16 * mt + g8 + 8] = o[4 * mt + 2 + e];
            }
            if (g8 == 0) { dst[kD] = m[e]; dst[kD + 1] = lsum[e]; }
          }
        }
      }
      named_bar_sync(1, kConsumers);
      if (warp < kWarps / 2) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int head = 2 * qd + e;
          float* dst = mrg + (warp * G + (head < G ? head : 0)) * kMrg;
          const float mp = dst[kD], lp = dst[kD + 1];
          const float M = fmaxf(m[e], mp);
          const float fa = (lsum[e] > 0.f) ? exp2f(m[e] - M) : 0.f;
          const float fb = (lp > 0.f) ? exp2f(mp - M) : 0.f;
          float ov[16];
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            ov[2 * mt] = fmaf(fa, o[4 * mt + e], fb * dst[16 * mt + g8]);
            ov[2 * mt + 1] = fmaf(fa, o[4 * mt + 2 + e], fb * dst[16 * mt + g8 + 8]);
          }
          __syncwarp();                  // every lane has read the partner's m, l and o
          if (head < G) {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              dst[16 * mt + g8] = ov[2 * mt];
              dst[16 * mt + g8 + 8] = ov[2 * mt + 1];
            }
            if (g8 == 0) { dst[kD] = M; dst[kD + 1] = fmaf(fa, lsum[e], fb * lp); }
          }
          __syncwarp();
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float* dst = mrg + (warp * G + g) * kMrg;
        *reinterpret_cast<float4*>(dst + 4 * lane) =
            make_float4(o[4 * g], o[4 * g + 1], o[4 * g + 2], o[4 * g + 3]);
        if (lane == 0) { dst[kD] = m[g]; dst[kD + 1] = l[g]; }
      }
    }
    named_bar_sync(1, kConsumers);
    const int rs = w.row_start();
    const bool whole = (seg_first == rs) && (w.tt == w.ntb - 1);
    const int slot = 2 * blockIdx.x + (seg_first == u0 ? 0 : 1);
    for (int idx = tid; idx < G * kD; idx += kConsumers) {
      const int g = idx / kD, d = idx - g * kD;
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < kMrgSlots; ++ww) M = fmaxf(M, mrg[(ww * G + g) * kMrg + kD]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int ww = 0; ww < kMrgSlots; ++ww) {
        const float* src = mrg + (ww * G + g) * kMrg;
        const float f = (src[kD + 1] > 0.f) ? exp2f(src[kD] - M) : 0.f;
        L = fmaf(f, src[kD + 1], L);
        O = fmaf(f, src[d], O);
      }
      if (whole) {
        out[((size_t)w.b * a.hq + (size_t)w.hk * G + g) * kD + d] = Elem<T>::from_f(O / L);
      } else {
        a.part_o[((size_t)slot * G + g) * kD + d] = O;
        if (d == 0) a.part_ml[(size_t)slot * G + g] = make_float2(M, L);
      }
    }
    if (whole) continue;

    // ---- publish the partial: the barrier orders every thread's partial stores
    // before thread 0's release. The CTA with the row's last tile merges it.
    named_bar_sync(1, kConsumers);
    if (w.tt == w.ntb - 1) {
      pend_b = w.b; pend_hk = w.hk; pend_rs = rs; pend_ntb = w.ntb;
      pend_np = owner(rs + w.ntb - 1, Ttot, grid) - owner(rs, Ttot, grid) + 1;
    } else if (tid == 0) {
      arrive_release(&a.done[w.row()]);
    }
  }
  if (pend_b >= 0) {
    // Every other contributor announces exactly once; all CTAs of the grid are
    // resident together (one per SM, grid <= SM count), so the wait ends.
    int* cnt = &a.done[pend_b * a.hkv + pend_hk];
    if (tid == 0) s_last = wait_count(cnt, pend_np - 1) ? 1 : 0;
    DBK_MARK(tid == 0, 12);
    named_bar_sync(1, kConsumers);
    // mrg and the ring are free once every consumer has passed the barrier above
    // (every stage the producer filled has been consumed).
    if (s_last) {
      if (merge_staged_fits(pend_np, G, (size_t)a.nstages * kStage))
        merge_row_staged<T, G>(a, pend_b, pend_hk, pend_rs, pend_ntb, Ttot, grid, tid,
                               reinterpret_cast<int*>(mrg), reinterpret_cast<float*>(smem));
      else
        merge_row<T, G>(a, pend_b, pend_hk, pend_rs, pend_ntb, Ttot, grid, tid,
                        reinterpret_cast<int*>(mrg));
    }
    if (tid == 0) *cnt = 0;                   // ready for the next launch
    DBK_MARK(tid == 0, 7);
  }
  DBK_MARK(tid == 0, 6);
}

size_t ws_bytes_for(int grid, int batch, int hq, int hkv) {
  const int G = hq / hkv;
  size_t b = (size_t)2 * grid * G * kD * sizeof(float);   // part_o
  b += (size_t)2 * grid * G * sizeof(float2);             // part_ml
  b += (size_t)batch * hkv * sizeof(int);                 // arrival counters
  return (b + 255) & ~(size_t)255;
}

template <typename T, int G>
int launch_g(FdArgs a, cudaStream_t st, const DeviceInfo& dev, int grid, bool mma) {
  constexpr int kStage = 2 * kTile * kD * (int)sizeof(T);
  const size_t fixed = 1024 + (size_t)(mma ? kWarps / 2 : kWarps) * G * kMrg * 4 +
                       (size_t)(a.batch + 1) * 4 + 64;
  static const int max_st = [] {   // DBK_FD_STAGES caps the ring depth (tuning knob)
    const char* v = std::getenv("DBK_FD_STAGES");
    const int n = v ? std::atoi(v) : kMaxStages;
    return n < 2 ? 2 : (n > kMaxStages ? kMaxStages : n);
  }();
  int nst = max_st;
  while (nst > 2 && (size_t)nst * (kStage + 16) + fixed > (size_t)dev.max_smem_optin - 1024) --nst;
  a.nstages = nst;
  const size_t smem = (size_t)nst * (kStage + 16) + fixed;
  if (smem > (size_t)dev.max_smem_optin) return DBK_ESHAPE;
  auto kern = mma ? flashdecode_kernel<T, G, true> : flashdecode_kernel<T, G, false>;
  if (int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kern), dev, smem)) return rc;
  return launch_pdl(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), smem, st, &a);
}

template <typename T>
int launch_t(const FdArgs& a, int G, cudaStream_t st, const DeviceInfo& dev, int grid, bool mma) {
  switch (G) {
    case 1: return launch_g<T, 1>(a, st, dev, grid, mma);
    case 2: return launch_g<T, 2>(a, st, dev, grid, mma);
    case 4: return launch_g<T, 4>(a, st, dev, grid, mma);
    case 8: return launch_g<T, 8>(a, st, dev, grid, mma);
    default: return DBK_ESHAPE;
  }
}

}  // namespace
}  // namespace dbk

using namespace dbk;

extern "C" size_t dbk_flashdecode_workspace_bytes(int batch, int n_q_heads, int n_kv_heads,
                                                  int max_len, int split_tokens) {
  (void)max_len;
  (void)split_tokens;
  if (batch < 1 || n_kv_heads < 1 || n_q_heads < n_kv_heads || max_len < 1) return 0;
  DeviceInfo dev;
  int nsm = 148;
  if (current_device_info(&dev) == DBK_OK) nsm = dev.num_sms;
  return ws_bytes_for(nsm, batch, n_q_heads, n_kv_heads);
}

extern "C" int dbk_flashdecode(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* page_table, const int32_t* seq_lens, void* out,
                               int batch, int n_q_heads, int n_kv_heads, int head_dim,
                               int max_len, int page_size, int max_pages_per_seq, float scale,
                               int split_tokens, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return DBK_ENULL;
  if (dtype != DBK_F16 && dtype != DBK_BF16) return DBK_EDTYPE;
  if (head_dim != kD || batch < 1 || batch > kMaxBatchSmem || n_kv_heads < 1 ||
      n_q_heads < n_kv_heads || n_q_heads % n_kv_heads != 0 || max_len < 1)
    return DBK_ESHAPE;
  const int G = n_q_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return DBK_ESHAPE;
  if (split_tokens < 0) return DBK_ESHAPE;
  if (page_table) {
    if (page_size < 1 || max_pages_per_seq < 1 ||
        (int64_t)page_size * max_pages_per_seq < max_len)
      return DBK_ESHAPE;
    if (G >= 4 && page_size % kMinBoxRows != 0) return DBK_ESHAPE;
  }
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return DBK_EALIGN;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  // Grid: one CTA per SM, or fewer when there are fewer tiles than SMs
  // (an upper bound on tiles: every sequence at max_len).
  const int64_t max_tiles = (int64_t)batch * n_kv_heads * ((max_len + kTile - 1) / kTile);
  static const int min_tiles = [] {   // DBK_FD_MIN_TILES: fewest tiles per CTA (experiments)
    const char* v = std::getenv("DBK_FD_MIN_TILES");
    const int n = v ? std::atoi(v) : 1;
    return n < 1 ? 1 : n;
  }();
  const int64_t want = (max_tiles + min_tiles - 1) / min_tiles;
  const int grid = (int)(want < dev.num_sms ? want : dev.num_sms);
  const size_t need = ws_bytes_for(dev.num_sms, batch, n_q_heads, n_kv_heads);
  if (!workspace || workspace_bytes < need) return DBK_EWORKSPACE;
  if (!aligned16(workspace)) return DBK_EALIGN;

  FdArgs a{};
  a.q = q; a.k = k_cache; a.v = v_cache; a.pages = page_table; a.lens = seq_lens; a.out = out;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.part_o = reinterpret_cast<float*>(ws);
  ws += (size_t)2 * dev.num_sms * G * kD * sizeof(float);
  a.part_ml = reinterpret_cast<float2*>(ws);
  ws += (size_t)2 * dev.num_sms * G * sizeof(float2);
  a.done = reinterpret_cast<int*>(ws);
  a.batch = batch; a.hq = n_q_heads; a.hkv = n_kv_heads; a.max_len = max_len;
  a.page_size = page_table ? page_size : max_len;
  a.max_pages = page_table ? max_pages_per_seq : 1;
  a.qscale = scale * kLog2e;
  // Tensor-core path whenever 16-token TMA boxes stay inside pages; CUDA cores
  // otherwise (page sizes that are not multiples of 16, G <= 2 only).
  const bool mma = (page_table == nullptr) || (page_size % kMinBoxRows == 0);
  // TMA box height: a whole 64-token tile per copy (16 KB of K, 16 KB of V) for
  // contiguous caches, where copies of 16 KB stream near the HBM rate and 4 KB
  // copies do not; 16 tokens (4 KB) for paged caches.
  a.box_shift = (mma && page_table == nullptr) ? 6 : 4;
  if (mma) {
    // 2-D views [rows, 128] of the caches for the tensor-core path's TMA boxes.
    // Contiguous caches: exact extent, so a box overhanging the end of the cache
    // reads zeros. Paged caches: the page count is not an argument; every box
    // (box_rows dividing page_size, box-aligned within its page) stays inside
    // one page of the table, so the view's extent only needs to cover them.
    const uint64_t prow = page_table ? (((uint64_t)1 << 31) - 1)
                                     : (uint64_t)batch * n_kv_heads * max_len;
    rc = encode_tmap_kv3d(&a.kmap, k_cache, dtype, prow, 1u << a.box_shift);
    if (rc) return rc;
    rc = encode_tmap_kv3d(&a.vmap, v_cache, dtype, prow, 1u << a.box_shift);
    if (rc) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == DBK_F16 ? launch_t<__half>(a, G, st, dev, grid, mma)
                          : launch_t<__nv_bfloat16>(a, G, st, dev, grid, mma);
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at all: plugins loaded into a
// host process whose allocator owns the whole device (no cudaMalloc allowed,
// no torch allocator available), or code running where an allocation would
// break a fixed memory budget. dbk_flashdecode needs a scratch workspace; this
// variant takes it from a fixed array compiled into the library instead.
//
// The array lives in every GPU that loads the library, until the process
// exits. Its address is looked up (cudaGetSymbolAddress) on the first call
// made in each CUDA context, so that first call should come before any stream
// capture. All calls share the one array: calls that
// overlap on the GPU (different streams, different threads) race and give
// wrong results. Each call clears the arrival counters it uses before the
// kernel runs.
namespace {
constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;   // 2 MiB
static __device__ __align__(256) uint8_t g_fd_scratch[kNoAllocScratchBytes];

// The array's device address differs per CUDA context: a device's primary
// context and any context the host creates on it each load their own copy of
// the module, and a context re-created after cudaDeviceReset loads it anew.
// The cache is therefore keyed by the context's process-unique id
// (cuCtxGetId; ids are never reused), not by the device ordinal.
constexpr int kMaxContextsNoAlloc = 64;
struct ScratchEntry {
  unsigned long long ctx_id;
  void* ptr;
};
ScratchEntry g_fd_scratch_cache[kMaxContextsNoAlloc];
int g_fd_scratch_n = 0;
std::mutex g_fd_scratch_mu;

// Driver entry points resolved through the runtime (the library does not link
// libcuda directly, so it still loads on machines without a driver).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

int scratch_address(void** out) {
  static const CtxGetCurrentFn cu_ctx_get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn cu_ctx_get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (!cu_ctx_get_current || !cu_ctx_get_id) return DBK_EDEVICE;
  CUcontext ctx = nullptr;
  if (cu_ctx_get_current(&ctx) != CUDA_SUCCESS) return DBK_EDEVICE;
  void* p = nullptr;
  cudaError_t e;
  if (ctx == nullptr) {
    // No context current yet: the runtime call makes the device's primary
    // context current (and gives its address of the array).
    e = cudaGetSymbolAddress(&p, g_fd_scratch);
    if (e != cudaSuccess) return (int)e;
    if (cu_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return DBK_EDEVICE;
  }
  unsigned long long id = 0;
  if (cu_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return DBK_EDEVICE;
  std::lock_guard<std::mutex> lk(g_fd_scratch_mu);
  for (int i = 0; i < g_fd_scratch_n; ++i)
    if (g_fd_scratch_cache[i].ctx_id == id) {
      *out = g_fd_scratch_cache[i].ptr;
      return DBK_OK;
    }
  e = cudaGetSymbolAddress(&p, g_fd_scratch);
  if (e != cudaSuccess) return (int)e;
  // A full table (many short-lived contexts) drops the oldest entry.
  if (g_fd_scratch_n == kMaxContextsNoAlloc) {
    for (int i = 1; i < kMaxContextsNoAlloc; ++i) g_fd_scratch_cache[i - 1] = g_fd_scratch_cache[i];
    --g_fd_scratch_n;
  }
  g_fd_scratch_cache[g_fd_scratch_n++] = {id, p};
  *out = p;
  return DBK_OK;
}
}  // namespace

extern "C" int dbk_flashdecode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* page_table, const int32_t* seq_lens,
                                       void* out, int batch, int n_q_heads, int n_kv_heads,
                                       int head_dim, int max_len, int page_size,
                                       int max_pages_per_seq, float scale, int dtype,
                                       void* stream) {
  if (batch < 1 || n_kv_heads < 1 || n_q_heads < n_kv_heads || max_len < 1) return DBK_ESHAPE;
  const size_t need = dbk_flashdecode_workspace_bytes(batch, n_q_heads, n_kv_heads, max_len, 0);
  if (need == 0 || need > kNoAllocScratchBytes) return DBK_EWORKSPACE;
  void* ws = nullptr;
  int rc = scratch_address(&ws);
  if (rc) return rc;
  // The arrival counters sit after the partials; the array may hold another
  // shape's partials there from an earlier call, so start them at zero.
  const size_t counters = (size_t)batch * n_kv_heads * sizeof(int);
  const size_t G = (size_t)(n_q_heads / n_kv_heads);
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const size_t off = (size_t)2 * dev.num_sms * G * kD * sizeof(float) +
                     (size_t)2 * dev.num_sms * G * sizeof(float2);
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(ws) + off, 0, counters,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return (int)e;
  return dbk_flashdecode(q, k_cache, v_cache, page_table, seq_lens, out, batch, n_q_heads,
                         n_kv_heads, head_dim, max_len, page_size, max_pages_per_seq, scale, 0,
                         dtype, ws, kNoAllocScratchBytes, stream);
}
