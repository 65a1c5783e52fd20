/* dbk_oracle.c - CPU restatement of the reference's decode hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the sm_100a
 * kernels: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load it. The product path never calls it (and has no CPU fallback).
 *
 * Sources restated (paths inside animeshsri14/Decodebench):
 *   - fp32 primitives: validation/src/reference/cpu_reference.cpp:7-111
 *     (rmsnorm_ref, gemv_ref, silu_ref, swiglu_ref, softmax_ref, attention_ref);
 *   - fp16 harness oracles: validation/src/bench/bench_variant.cu:127-217
 *     (cpu_rmsnorm with eps 1e-5 and one rounding of x*gamma*inv_rms, cpu_gemv,
 *     cpu_swiglu, cpu_f1, cpu_f2, cpu_f4 with scale 1/sqrt(D));
 *   - PyTorch stage semantics: src/decodebench/demos/llama_decode.py:36-43
 *     (rmsnorm: (x * rsqrt(mean x^2 + eps)).half() * g, two roundings),
 *     :77-87 (gate/up rounded to the dtype, silu(gate) rounded, product rounded),
 *     :120-134 (scores rounded to the dtype then fp32, softmax fp32, p rounded);
 *   - the split-KV algorithm: validation/src/kernels/fused/f4.cu:173-319
 *     (online softmax per split -> (m, l, o) partials -> log-sum-exp merge).
 *
 * Rounding conventions are a parameter (`round_mode`):
 *   ORC_ROUND_FUSED  (0): fp32 everywhere, one rounding of the output
 *                         (what a fused kernel computes);
 *   ORC_ROUND_HARNESS(1): bench_variant.cu's cpu_f1/cpu_f2 roundings;
 *   ORC_ROUND_STAGES (2): the PyTorch stage chain's roundings.
 * 16-bit values travel as raw uint16 bit patterns; dtype 0 = fp16, 1 = bf16.
 * Accumulation is sequential fp32, as in cpu_reference.cpp.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_F16 0
#define ORC_BF16 1
#define ORC_ROUND_FUSED 0
#define ORC_ROUND_HARNESS 1
#define ORC_ROUND_STAGES 2

/* ------------------------------------------------------------------ 16-bit types */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));        /* inf / nan */
  if (exp == 0) {                                                          /* zero / subnormal */
    float v = (float)man * 5.9604644775390625e-08f;                        /* man * 2^-24 */
    return (sign ? -v : v);
  }
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t orc_f32_to_f16(float f) {
  uint32_t u = f2u(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);                 /* nan */
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);                 /* >= 65520: inf */
  if (a < 0x38800000u) {                                                   /* below 2^-14: subnormal */
    /* value = a as float; subnormal step is 2^-24: round |f| / 2^-24 to nearest even */
    float v = u2f(a) * 16777216.0f;                                         /* exact (power of 2) */
    uint32_t q = (uint32_t)v;
    float rem = v - (float)q;
    if (rem > 0.5f || (rem == 0.5f && (q & 1u))) q++;
    return (uint16_t)(sign | q);                                            /* q == 0x400 -> min normal */
  }
  /* normal: keep 10 mantissa bits, round to nearest even on the 13 dropped bits */
  uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
  return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
}

float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  /* quiet nan */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float ld16(const uint16_t* p, size_t i, int dt) {
  return dt == ORC_BF16 ? orc_bf16_to_f32(p[i]) : orc_f16_to_f32(p[i]);
}
static inline uint16_t st16(float v, int dt) {
  return dt == ORC_BF16 ? orc_f32_to_bf16(v) : orc_f32_to_f16(v);
}
static inline float rnd(float v, int dt) { return ld16(&(uint16_t){st16(v, dt)}, 0, dt); }

/* ------------------------------------------------------------------ fp32 primitives
 * Same contracts as cpu_reference.h:8-30 (restated). */
void orc_rmsnorm_f32(const float* x, const float* gamma, float* out, int d, float eps) {
  float ss = 0.f;
  for (int i = 0; i < d; ++i) ss += x[i] * x[i];
  float rms = sqrtf(ss / (float)d + eps);
  for (int i = 0; i < d; ++i) out[i] = x[i] / rms * gamma[i];
}

void orc_gemv_f32(const float* W, const float* x, float* out, int d_out, int d_in) {
  for (int r = 0; r < d_out; ++r) {
    float acc = 0.f;
    const float* w = W + (size_t)r * d_in;
    for (int c = 0; c < d_in; ++c) acc += w[c] * x[c];
    out[r] = acc;
  }
}

float orc_silu(float g) { return g / (1.f + expf(-g)); }

void orc_swiglu_f32(const float* g, const float* u, float* out, int n) {
  for (int i = 0; i < n; ++i) out[i] = orc_silu(g[i]) * u[i];
}

void orc_softmax_f32(const float* s, float* p, int rows, int n) {
  for (int r = 0; r < rows; ++r) {
    const float* a = s + (size_t)r * n;
    float* o = p + (size_t)r * n;
    float mx = a[0];
    for (int i = 1; i < n; ++i) mx = a[i] > mx ? a[i] : mx;
    float sum = 0.f;
    for (int i = 0; i < n; ++i) { o[i] = expf(a[i] - mx); sum += o[i]; }
    for (int i = 0; i < n; ++i) o[i] /= sum;
  }
}

/* Unscaled single-query attention per head, as attention_ref (cpu_reference.cpp:64-111). */
void orc_attention_f32(const float* q, const float* K, const float* V, float* out, int heads,
                       int len, int d) {
  float* s = (float*)malloc(sizeof(float) * (size_t)len);
  float* p = (float*)malloc(sizeof(float) * (size_t)len);
  for (int h = 0; h < heads; ++h) {
    const float* qh = q + (size_t)h * d;
    const float* Kh = K + (size_t)h * len * d;
    const float* Vh = V + (size_t)h * len * d;
    for (int t = 0; t < len; ++t) {
      float dot = 0.f;
      for (int i = 0; i < d; ++i) dot += qh[i] * Kh[(size_t)t * d + i];
      s[t] = dot;
    }
    orc_softmax_f32(s, p, 1, len);
    for (int i = 0; i < d; ++i) {
      float acc = 0.f;
      for (int t = 0; t < len; ++t) acc += p[t] * Vh[(size_t)t * d + i];
      out[(size_t)h * d + i] = acc;
    }
  }
  free(s);
  free(p);
}

/* ------------------------------------------------------------------ 16-bit fused ops */

/* F1. round_mode: FUSED xn = x*g*r (fp32); HARNESS xn = rnd(x*g*r);
 * STAGES xn = rnd(rnd(x*r)*g). */
void orc_rmsnorm_gemv(const uint16_t* x, const uint16_t* gamma, const uint16_t* W, uint16_t* y,
                      int batch, int d_in, int d_out, float eps, int dt, int round_mode) {
  float* xn = (float*)malloc(sizeof(float) * (size_t)d_in);
  for (int b = 0; b < batch; ++b) {
    const uint16_t* xb = x + (size_t)b * d_in;
    float ss = 0.f;
    for (int i = 0; i < d_in; ++i) { float v = ld16(xb, i, dt); ss += v * v; }
    const float r = 1.f / sqrtf(ss / (float)d_in + eps);
    for (int i = 0; i < d_in; ++i) {
      const float v = ld16(xb, i, dt), g = ld16(gamma, i, dt);
      if (round_mode == ORC_ROUND_STAGES) xn[i] = rnd(rnd(v * r, dt) * g, dt);
      else if (round_mode == ORC_ROUND_HARNESS) xn[i] = rnd(v * g * r, dt);
      else xn[i] = v * g * r;
    }
    for (int o = 0; o < d_out; ++o) {
      float acc = 0.f;
      const uint16_t* w = W + (size_t)o * d_in;
      for (int i = 0; i < d_in; ++i) acc += ld16(w, i, dt) * xn[i];
      y[(size_t)b * d_out + o] = st16(acc, dt);
    }
  }
  free(xn);
}

/* F2 (optionally with an RMSNorm prologue when gamma != NULL; normalised x is
 * kept in fp32 for FUSED and rounded once otherwise). */
void orc_gateup_swiglu(const uint16_t* x, const uint16_t* gamma, const uint16_t* Wg,
                       const uint16_t* Wu, uint16_t* h, int batch, int d_in, int d_ff,
                       float eps, int dt, int round_mode) {
  float* xn = (float*)malloc(sizeof(float) * (size_t)d_in);
  for (int b = 0; b < batch; ++b) {
    const uint16_t* xb = x + (size_t)b * d_in;
    float r = 1.f;
    if (gamma) {
      float ss = 0.f;
      for (int i = 0; i < d_in; ++i) { float v = ld16(xb, i, dt); ss += v * v; }
      r = 1.f / sqrtf(ss / (float)d_in + eps);
    }
    for (int i = 0; i < d_in; ++i) {
      float v = ld16(xb, i, dt);
      if (gamma) {
        const float g = ld16(gamma, i, dt);
        if (round_mode == ORC_ROUND_STAGES) v = rnd(rnd(v * r, dt) * g, dt);
        else if (round_mode == ORC_ROUND_HARNESS) v = rnd(v * g * r, dt);
        else v = v * g * r;
      }
      xn[i] = v;
    }
    for (int o = 0; o < d_ff; ++o) {
      float ga = 0.f, ua = 0.f;
      const uint16_t* wg = Wg + (size_t)o * d_in;
      const uint16_t* wu = Wu + (size_t)o * d_in;
      for (int i = 0; i < d_in; ++i) {
        ga += ld16(wg, i, dt) * xn[i];
        ua += ld16(wu, i, dt) * xn[i];
      }
      float val;
      if (round_mode == ORC_ROUND_STAGES) val = rnd(orc_silu(rnd(ga, dt)), dt) * rnd(ua, dt);
      else if (round_mode == ORC_ROUND_HARNESS) val = orc_silu(rnd(ga, dt)) * rnd(ua, dt);
      else val = orc_silu(ga) * ua;
      h[(size_t)b * d_ff + o] = st16(val, dt);
    }
  }
  free(xn);
}

/* y = W x (+ residual), fp32 accumulation, one rounding (residual added in fp32). */
void orc_gemv(const uint16_t* x, const uint16_t* W, const uint16_t* residual, uint16_t* y,
              int batch, int d_in, int d_out, int dt) {
  for (int b = 0; b < batch; ++b)
    for (int o = 0; o < d_out; ++o) {
      float acc = 0.f;
      const uint16_t* w = W + (size_t)o * d_in;
      for (int i = 0; i < d_in; ++i) acc += ld16(w, i, dt) * ld16(x, (size_t)b * d_in + i, dt);
      if (residual) acc += ld16(residual, (size_t)b * d_out + o, dt);
      y[(size_t)b * d_out + o] = st16(acc, dt);
    }
}

/* Row pointer of token t of (b, hk): contiguous [batch, hkv, max_len, D] or
 * paged [pages, hkv, page_size, D] through page_table [batch, max_pages]. */
static const uint16_t* kv_row(const uint16_t* base, const int32_t* pt, int b, int hk, int t,
                              int hkv, int max_len, int page_size, int max_pages, int d) {
  if (!pt) return base + (((size_t)b * hkv + hk) * max_len + t) * d;
  int pg = pt[(size_t)b * max_pages + t / page_size];
  return base + (((size_t)pg * hkv + hk) * page_size + t % page_size) * d;
}

/* F4 attention for one query per sequence. FUSED: fp32 throughout;
 * STAGES: scores rounded to dt, softmax fp32, p rounded to dt. */
void orc_attention(const uint16_t* q, const uint16_t* K, const uint16_t* V,
                   const int32_t* page_table, const int32_t* seq_lens, uint16_t* out, int batch,
                   int hq, int hkv, int d, int max_len, int page_size, int max_pages, float scale,
                   int dt, int round_mode) {
  const int G = hq / hkv;
  float* s = (float*)malloc(sizeof(float) * (size_t)(max_len > 0 ? max_len : 1));
  float* acc = (float*)malloc(sizeof(float) * (size_t)d);
  for (int b = 0; b < batch; ++b) {
    int L = seq_lens ? seq_lens[b] : max_len;
    if (L > max_len) L = max_len;
    for (int h = 0; h < hq; ++h) {
      const int hk = h / G;
      const uint16_t* qh = q + ((size_t)b * hq + h) * d;
      uint16_t* oh = out + ((size_t)b * hq + h) * d;
      if (L <= 0) { for (int i = 0; i < d; ++i) oh[i] = st16(0.f, dt); continue; }
      float mx = -INFINITY;
      for (int t = 0; t < L; ++t) {
        const uint16_t* kr = kv_row(K, page_table, b, hk, t, hkv, max_len, page_size, max_pages, d);
        float dot = 0.f;
        for (int i = 0; i < d; ++i) dot += ld16(qh, i, dt) * ld16(kr, i, dt);
        if (round_mode == ORC_ROUND_STAGES) dot = rnd(dot, dt);
        s[t] = dot * scale;
        if (s[t] > mx) mx = s[t];
      }
      float sum = 0.f;
      for (int t = 0; t < L; ++t) { s[t] = expf(s[t] - mx); sum += s[t]; }
      for (int i = 0; i < d; ++i) acc[i] = 0.f;
      for (int t = 0; t < L; ++t) {
        float p = s[t] / sum;
        if (round_mode == ORC_ROUND_STAGES) p = rnd(p, dt);
        const uint16_t* vr = kv_row(V, page_table, b, hk, t, hkv, max_len, page_size, max_pages, d);
        for (int i = 0; i < d; ++i) acc[i] += p * ld16(vr, i, dt);
      }
      for (int i = 0; i < d; ++i) oh[i] = st16(acc[i], dt);
    }
  }
  free(s);
  free(acc);
}

/* Split-KV restatement of f4.cu:173-319 for one head: the L tokens are cut into
 * `splits` contiguous ranges; each produces an unnormalised partial (m, l, o[d])
 * by an online softmax over tiles of `tile` tokens; the partials are merged by
 * log-sum-exp. q, K, V fp32; K/V rows [L, d]. Returns the normalised output. */
void orc_splitkv_head(const float* q, const float* K, const float* V, float* out, int L, int d,
                      float scale, int splits, int tile) {
  float* pm = (float*)malloc(sizeof(float) * (size_t)splits);
  float* pl = (float*)malloc(sizeof(float) * (size_t)splits);
  float* po = (float*)calloc((size_t)splits * d, sizeof(float));
  float* st = (float*)malloc(sizeof(float) * (size_t)tile);
  const int per = (L + splits - 1) / splits;
  for (int sp = 0; sp < splits; ++sp) {
    const int t0 = sp * per, t1 = (t0 + per < L) ? t0 + per : L;
    float m = -INFINITY, l = 0.f;
    float* o = po + (size_t)sp * d;
    for (int a = t0; a < t1; a += tile) {
      const int n = (a + tile < t1) ? tile : t1 - a;
      float mt = -INFINITY;
      for (int j = 0; j < n; ++j) {
        float dot = 0.f;
        for (int i = 0; i < d; ++i) dot += q[i] * K[(size_t)(a + j) * d + i];
        st[j] = dot * scale;
        if (st[j] > mt) mt = st[j];
      }
      const float mn = m > mt ? m : mt;
      const float cp = expf(m - mn);
      l *= cp;
      for (int i = 0; i < d; ++i) o[i] *= cp;
      for (int j = 0; j < n; ++j) {
        const float p = expf(st[j] - mn);
        l += p;
        for (int i = 0; i < d; ++i) o[i] += p * V[(size_t)(a + j) * d + i];
      }
      m = mn;
    }
    pm[sp] = m;   /* -inf with l = 0 for an empty split: drops out of the merge */
    pl[sp] = l;
  }
  float M = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) if (pm[sp] > M) M = pm[sp];
  float Lsum = 0.f;
  for (int i = 0; i < d; ++i) out[i] = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    if (pl[sp] == 0.f) continue;
    const float w = expf(pm[sp] - M);
    Lsum += w * pl[sp];
    for (int i = 0; i < d; ++i) out[i] += w * po[(size_t)sp * d + i];
  }
  for (int i = 0; i < d; ++i) out[i] /= Lsum;
  free(pm); free(pl); free(po); free(st);
}

/* Batched conversions, for tests (bit-exact against numpy/torch RNE). */
void orc_to16(const float* src, uint16_t* dst, size_t n, int dt) {
  for (size_t i = 0; i < n; ++i) dst[i] = st16(src[i], dt);
}
void orc_from16(const uint16_t* src, float* dst, size_t n, int dt) {
  for (size_t i = 0; i < n; ++i) dst[i] = ld16(src, i, dt);
}
