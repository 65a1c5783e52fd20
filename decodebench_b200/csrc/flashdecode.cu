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
//   * work items are (b, hk, split) with split_tokens tokens each; CTAs (one per
//     SM, persistent) take items round-robin, so a ragged batch still spreads
//     over all 148 SMs;
//   * a producer warp streams each item's K and V in 64-token tiles with
//     cp.async.bulk into a ring of 32 KB stages (K tile | V tile); a paged cache
//     ([page, kv_head, page_size, 128], the per-head page block contiguous) is
//     gathered page-run by page-run through the int32 page table;
//   * eight consumer warps each take 8 tokens of a tile and keep their own
//     online-softmax state (m, l, o) for the G query heads: no block barrier per
//     tile; lane l owns head dims 4l..4l+3 of q and o;
//   * at the end of an item the warps' states are merged in shared memory; a
//     single-split sequence writes its output directly, otherwise the partial
//     goes to the workspace and the last CTA to finish a (b, hk) (atomic
//     counter, self-resetting) performs the LSE merge: no second launch.
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
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMrg = kD + 4;             // merge-row stride: o[128], m, l, pad (16-byte rows)

struct FdArgs {
  const void* q;          // [batch, Hq, 128]
  const void* k;          // contiguous [batch, Hkv, max_len, 128] | paged [pages, Hkv, ps, 128]
  const void* v;
  const int32_t* pages;   // [batch, max_pages] or nullptr
  const int32_t* lens;    // [batch] or nullptr
  void* out;              // [batch, Hq, 128]
  float* part_o;          // [items_cap, G, 128]
  float2* part_ml;        // [items_cap, G]
  int* done;              // [batch * Hkv] arrival counters (zero between launches)
  int batch, hq, hkv, max_len, page_size, max_pages;
  int split_tokens;       // multiple of kTile
  int items_per_seqhead;  // ceil(max_len / split_tokens): item-id stride
  float qscale;           // scale * log2(e)
  int nstages;
};

struct Item {
  int b, hk, s, t0, ntok, nsplit;
};

__device__ __forceinline__ int seq_len(const FdArgs& a, int b) {
  return a.lens ? min(max(a.lens[b], 0), a.max_len) : a.max_len;
}

// Item enumeration: id -> (b, hk, split), skipping splits past len_b.
// Items are numbered densely over (b, hk, s < nsplit_b) in that order; every CTA
// walks the same enumeration, so producer and consumers agree without messages.
struct ItemWalker {
  const FdArgs& a;
  int b = 0, hk = 0, s = 0, nsplit = 0;
  __device__ explicit ItemWalker(const FdArgs& args) : a(args) { reset_seq(); }
  __device__ void reset_seq() {
    while (b < a.batch) {
      const int L = seq_len(a, b);
      nsplit = (L + a.split_tokens - 1) / a.split_tokens;
      if (nsplit > 0) return;
      ++b;
    }
  }
  __device__ bool valid() const { return b < a.batch; }
  __device__ void advance(int n) {  // move forward n items
    while (n > 0 && valid()) {
      const int left = nsplit - s;
      if (n < left) { s += n; return; }
      n -= left;
      s = 0;
      if (++hk == a.hkv) { hk = 0; ++b; reset_seq(); }
    }
  }
  __device__ Item get() const {
    Item it;
    it.b = b; it.hk = hk; it.s = s; it.nsplit = nsplit;
    it.t0 = s * a.split_tokens;
    it.ntok = min(a.split_tokens, seq_len(a, b) - it.t0);
    return it;
  }
};

// Address of K/V row (token t of (b, hk)); paged caches go through the table.
template <typename T>
__device__ __forceinline__ const T* kv_row(const FdArgs& a, const void* base, int b, int hk,
                                           int t, int* run) {
  const T* p = static_cast<const T*>(base);
  if (a.pages == nullptr) {
    *run = 1 << 30;
    return p + (((size_t)b * a.hkv + hk) * a.max_len + t) * kD;
  }
  const int pg = a.pages[(size_t)b * a.max_pages + t / a.page_size];
  const int off = t % a.page_size;
  *run = a.page_size - off;   // tokens left in this page
  return p + (((size_t)pg * a.hkv + hk) * a.page_size + off) * kD;
}

template <typename T, int G>
__global__ void __launch_bounds__(kThreads, 1) flashdecode_kernel(const FdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int kStage = 2 * kTile * kD * (int)sizeof(T);       // K tile | V tile
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.nstages * kStage);
  uint64_t* empty = full + a.nstages;
  float* mrg = reinterpret_cast<float*>(empty + a.nstages);     // [kWarps][G][kMrg] (o, m, l)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == kWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    ItemWalker w(a);
    w.advance(blockIdx.x);
    int j = 0;
    for (; w.valid(); w.advance(gridDim.x)) {
      const Item it = w.get();
      for (int t0 = 0; t0 < it.ntok; t0 += kTile, ++j) {
        const int s = j % a.nstages;
        if (j >= a.nstages && !mbar_wait(&empty[s], ((j / a.nstages) & 1) ^ 1, kDevTimeoutEmpty))
          return;
        const int n = min(kTile, it.ntok - t0);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * n * kD * sizeof(T)));
        uint8_t* dk = smem + (size_t)s * kStage;
        uint8_t* dv = dk + kTile * kD * sizeof(T);
        for (int t = 0; t < n;) {
          int run;
          const T* ks = kv_row<T>(a, a.k, it.b, it.hk, it.t0 + t0 + t, &run);
          const T* vs = kv_row<T>(a, a.v, it.b, it.hk, it.t0 + t0 + t, &run);
          const int m = min(run, n - t);
          const uint32_t bytes = (uint32_t)(m * kD * sizeof(T));
          bulk_g2s(dk + (size_t)t * kD * sizeof(T), ks, bytes, &full[s], pol);
          bulk_g2s(dv + (size_t)t * kD * sizeof(T), vs, bytes, &full[s], pol);
          t += m;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const T* q = static_cast<const T*>(a.q);
  T* out = static_cast<T*>(a.out);

  // Sequences of length 0 have no items: their output is defined as zeros.
  if (blockIdx.x == 0 && a.lens != nullptr) {
    for (int b = 0; b < a.batch; ++b)
      if (seq_len(a, b) == 0)
        for (int i = tid; i < a.hq * kD; i += kConsumers)
          out[(size_t)b * a.hq * kD + i] = Elem<T>::from_f(0.f);
  }

  ItemWalker w(a);
  w.advance(blockIdx.x);
  int j = 0;
  for (; w.valid(); w.advance(gridDim.x)) {
    const Item it = w.get();
    // q for the G heads sharing this kv head, dims 4*lane..4*lane+3, pre-scaled.
    float qr[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const T* qp = q + ((size_t)it.b * a.hq + it.hk * G + g) * kD + 4 * lane;
      const uint2 raw = *reinterpret_cast<const uint2*>(qp);
      const float2 lo = Elem<T>::unpack2(raw.x), hi = Elem<T>::unpack2(raw.y);
      qr[g][0] = lo.x * a.qscale; qr[g][1] = lo.y * a.qscale;
      qr[g][2] = hi.x * a.qscale; qr[g][3] = hi.y * a.qscale;
    }
    float m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY; l[g] = 0.f;
      o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }

    for (int t0 = 0; t0 < it.ntok; t0 += kTile, ++j) {
      const int s = j % a.nstages;
      if (!mbar_wait(&full[s], (j / a.nstages) & 1, kDevTimeoutFull)) return;
      const int n = min(kTile, it.ntok - t0);
      const int mine = min(8, n - warp * 8);           // tokens of this warp
      if (mine > 0) {
        const uint32_t kbase = smem_u32(smem + (size_t)s * kStage) +
                               (uint32_t)((warp * 8) * kD + 4 * lane) * sizeof(T);
        const uint32_t vbase = kbase + kTile * kD * sizeof(T);
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
          const float alpha = exp2f(m[g] - mx);   // 0 on the first tile (m = -inf)
          m[g] = mx;
          l[g] *= alpha;
#pragma unroll
          for (int e = 0; e < 4; ++e) o[g][e] *= alpha;
#pragma unroll
          for (int t = 0; t < 8; ++t) sc[t][g] = exp2f(sc[t][g] - mx);   // -inf -> 0
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
              o[g][0] = fmaf(p, v01.x, o[g][0]);
              o[g][1] = fmaf(p, v01.y, o[g][1]);
              o[g][2] = fmaf(p, v23.x, o[g][2]);
              o[g][3] = fmaf(p, v23.y, o[g][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the 8 warps' states for this item
    named_bar_sync(1, kConsumers);   // previous item's readers of mrg are done
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float* dst = mrg + (warp * G + g) * kMrg;
      *reinterpret_cast<float4*>(dst + 4 * lane) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
      if (lane == 0) { dst[kD] = m[g]; dst[kD + 1] = l[g]; }
    }
    named_bar_sync(1, kConsumers);
    const bool single = (it.nsplit == 1);
    const int item_id = ((it.b * a.hkv + it.hk) * a.items_per_seqhead) + it.s;
    for (int idx = tid; idx < G * kD; idx += kConsumers) {
      const int g = idx / kD, d = idx - g * kD;
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, mrg[(ww * G + g) * kMrg + kD]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int ww = 0; ww < kWarps; ++ww) {
        const float* src = mrg + (ww * G + g) * kMrg;
        const float f = exp2f(src[kD] - M);   // warps without tokens: m = -inf -> 0
        L = fmaf(f, src[kD + 1], L);
        O = fmaf(f, src[d], O);
      }
      if (single) {
        out[((size_t)it.b * a.hq + it.hk * G + g) * kD + d] = Elem<T>::from_f(O / L);
      } else {
        a.part_o[((size_t)item_id * G + g) * kD + d] = O;
        if (d == 0) a.part_ml[(size_t)item_id * G + g] = make_float2(M, L);
      }
    }
    if (single) continue;

    // ---- publish the partial; the last split of (b, hk) to arrive merges all
    __threadfence();
    named_bar_sync(1, kConsumers);
    __shared__ int last;
    if (tid == 0) {
      const int prev = atomicAdd(&a.done[it.b * a.hkv + it.hk], 1);
      last = (prev == it.nsplit - 1);
    }
    named_bar_sync(1, kConsumers);
    if (!last) continue;
    __threadfence();
    const int base = (it.b * a.hkv + it.hk) * a.items_per_seqhead;
    for (int idx = tid; idx < G * kD; idx += kConsumers) {
      const int g = idx / kD, d = idx - g * kD;
      float M = -INFINITY;
      for (int sp = 0; sp < it.nsplit; ++sp)
        M = fmaxf(M, __ldcg(&a.part_ml[(size_t)(base + sp) * G + g].x));
      float L = 0.f, O = 0.f;
      for (int sp = 0; sp < it.nsplit; ++sp) {
        const float2 ml = __ldcg(&a.part_ml[(size_t)(base + sp) * G + g]);
        const float f = exp2f(ml.x - M);
        L = fmaf(f, ml.y, L);
        O = fmaf(f, __ldcg(&a.part_o[((size_t)(base + sp) * G + g) * kD + d]), O);
      }
      out[((size_t)it.b * a.hq + it.hk * G + g) * kD + d] = Elem<T>::from_f(O / L);
    }
    if (tid == 0) a.done[it.b * a.hkv + it.hk] = 0;   // ready for the next launch
  }
}

struct FdPlan {
  int split_tokens, items_per_seqhead;
  size_t items_cap;
};

FdPlan plan(int batch, int hkv, int max_len, int split_tokens, int num_sms) {
  FdPlan p{};
  int st = split_tokens;
  if (st <= 0) {
    // ~16 items per SM if every sequence had max_len tokens.
    const int64_t total = (int64_t)batch * hkv * max_len;
    const int64_t per = (total + (int64_t)num_sms * 16 - 1) / ((int64_t)num_sms * 16);
    st = (int)((per + kTile - 1) / kTile) * kTile;
    if (st < kTile) st = kTile;
  }
  p.split_tokens = st;
  p.items_per_seqhead = (max_len + st - 1) / st;
  p.items_cap = (size_t)batch * hkv * p.items_per_seqhead;
  return p;
}

size_t ws_bytes_for(const FdPlan& p, int batch, int hq, int hkv) {
  const int G = hq / hkv;
  size_t b = 0;
  b += p.items_cap * G * kD * sizeof(float);      // part_o
  b += p.items_cap * G * sizeof(float2);          // part_ml
  b += (size_t)batch * hkv * sizeof(int);         // done counters
  return (b + 255) & ~(size_t)255;
}

template <typename T, int G>
int launch_g(FdArgs a, cudaStream_t st, const DeviceInfo& dev, int grid) {
  constexpr int kStage = 2 * kTile * kD * (int)sizeof(T);
  const size_t fixed = (size_t)kWarps * G * kMrg * 4 + G * 8 + 64;
  int nst = kMaxStages;
  while (nst > 2 && (size_t)nst * (kStage + 16) + fixed > (size_t)dev.max_smem_optin - 1024) --nst;
  a.nstages = nst;
  const size_t smem = (size_t)nst * (kStage + 16) + fixed;
  auto kern = flashdecode_kernel<T, G>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  return launch_pdl(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), smem, st, &a);
}

template <typename T>
int launch_t(const FdArgs& a, int G, cudaStream_t st, const DeviceInfo& dev, int grid) {
  switch (G) {
    case 1: return launch_g<T, 1>(a, st, dev, grid);
    case 2: return launch_g<T, 2>(a, st, dev, grid);
    case 4: return launch_g<T, 4>(a, st, dev, grid);
    case 8: return launch_g<T, 8>(a, st, dev, grid);
    default: return DBK_ESHAPE;
  }
}

}  // namespace
}  // namespace dbk

using namespace dbk;

extern "C" size_t dbk_flashdecode_workspace_bytes(int batch, int n_q_heads, int n_kv_heads,
                                                  int max_len, int split_tokens) {
  if (batch < 1 || n_kv_heads < 1 || n_q_heads < n_kv_heads || max_len < 1) return 0;
  DeviceInfo dev;
  int nsm = 148;
  if (current_device_info(&dev) == DBK_OK) nsm = dev.num_sms;
  const FdPlan p = plan(batch, n_kv_heads, max_len, split_tokens, nsm);
  return ws_bytes_for(p, batch, n_q_heads, n_kv_heads);
}

extern "C" int dbk_flashdecode(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* page_table, const int32_t* seq_lens, void* out,
                               int batch, int n_q_heads, int n_kv_heads, int head_dim,
                               int max_len, int page_size, int max_pages_per_seq, float scale,
                               int split_tokens, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return DBK_ENULL;
  if (dtype != DBK_F16 && dtype != DBK_BF16) return DBK_EDTYPE;
  if (head_dim != kD || batch < 1 || n_kv_heads < 1 || n_q_heads < n_kv_heads ||
      n_q_heads % n_kv_heads != 0 || max_len < 1)
    return DBK_ESHAPE;
  const int G = n_q_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return DBK_ESHAPE;
  if (split_tokens < 0 || split_tokens % kTile != 0) return DBK_ESHAPE;
  if (page_table) {
    if (page_size < 1 || max_pages_per_seq < 1 ||
        (int64_t)page_size * max_pages_per_seq < max_len)
      return DBK_ESHAPE;
  }
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return DBK_EALIGN;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc) return rc;
  const FdPlan p = plan(batch, n_kv_heads, max_len, split_tokens, dev.num_sms);
  const size_t need = ws_bytes_for(p, batch, n_q_heads, n_kv_heads);
  if (!workspace || workspace_bytes < need) return DBK_EWORKSPACE;
  if (!aligned16(workspace)) return DBK_EALIGN;

  FdArgs a{};
  a.q = q; a.k = k_cache; a.v = v_cache; a.pages = page_table; a.lens = seq_lens; a.out = out;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.part_o = reinterpret_cast<float*>(ws);
  ws += p.items_cap * G * kD * sizeof(float);
  a.part_ml = reinterpret_cast<float2*>(ws);
  ws += p.items_cap * G * sizeof(float2);
  a.done = reinterpret_cast<int*>(ws);
  a.batch = batch; a.hq = n_q_heads; a.hkv = n_kv_heads; a.max_len = max_len;
  a.page_size = page_table ? page_size : max_len;
  a.max_pages = page_table ? max_pages_per_seq : 1;
  a.split_tokens = p.split_tokens;
  a.items_per_seqhead = p.items_per_seqhead;
  a.qscale = scale * kLog2e;
  const int grid = (int)((p.items_cap < (size_t)dev.num_sms) ? p.items_cap : dev.num_sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == DBK_F16 ? launch_t<__half>(a, G, st, dev, grid)
                          : launch_t<__nv_bfloat16>(a, G, st, dev, grid);
}
