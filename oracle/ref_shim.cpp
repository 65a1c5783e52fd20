// ref_shim.cpp - C entry points over the reference's own CPU oracle.
//
// TEST INFRASTRUCTURE ONLY (parity pinning and the timed CPU baseline). It is
// compiled together with the reference's validation/src/reference/cpu_reference.cpp,
// read in place from the reference checkout by oracle/Makefile, into
// oracle/_ref/libdbref.so. Nothing here re-implements the reference: every entry
// calls one of its functions (cpu_reference.h:8-30), and the threaded helpers
// only split rows of a GEMV across threads.
#include <pthread.h>

#include <vector>

#include "cpu_reference.h"

extern "C" {

void ref_rmsnorm(const float* x, const float* gamma, float* out, int d, float eps) {
  rmsnorm_ref(x, gamma, out, d, eps);
}
void ref_gemv(const float* W, const float* x, float* out, int d_out, int d_in) {
  gemv_ref(W, x, out, d_out, d_in);
}
float ref_silu(float x) { return silu_ref(x); }
void ref_swiglu(const float* g, const float* u, float* out, int n) { swiglu_ref(g, u, out, n); }
void ref_softmax(const float* s, float* p, int heads, int len) { softmax_ref(s, p, heads, len); }
void ref_attention(const float* q, const float* K, const float* V, float* out, int heads, int len,
                   int d) {
  attention_ref(q, K, V, out, heads, len, d);
}

struct GemvJob {
  const float* W;
  const float* x;
  float* out;
  int rows, d_in;
};

static void* gemv_job(void* p) {
  GemvJob* j = static_cast<GemvJob*>(p);
  gemv_ref(j->W, j->x, j->out, j->rows, j->d_in);
  return nullptr;
}

// gemv_ref over d_out rows split into `threads` contiguous row blocks.
void ref_gemv_threaded(const float* W, const float* x, float* out, int d_out, int d_in,
                       int threads) {
  if (threads < 1) threads = 1;
  if (threads > d_out) threads = d_out;
  std::vector<pthread_t> tid(threads);
  std::vector<GemvJob> jobs(threads);
  for (int t = 0; t < threads; ++t) {
    const int r0 = (int)((long long)d_out * t / threads);
    const int r1 = (int)((long long)d_out * (t + 1) / threads);
    jobs[t] = GemvJob{W + (size_t)r0 * d_in, x, out + r0, r1 - r0, d_in};
    pthread_create(&tid[t], nullptr, gemv_job, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], nullptr);
}

}  // extern "C"
