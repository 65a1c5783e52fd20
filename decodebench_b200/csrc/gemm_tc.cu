// gemm_tc.cu - batch > 8 decode GEMMs on tcgen05 tensor cores (placeholder:
// rejects the shape until the tensor-core kernels land).
#include "common.cuh"
#include "dbk_internal.h"

int dbk_tc_rmsnorm_gemv(const void*, const void*, const void*, void*, int, int, int, float, int,
                        void*, size_t, void*) {
  return DBK_ESHAPE;
}
int dbk_tc_gateup_swiglu(const void*, const void*, const void*, const void*, void*, int, int, int,
                         float, int, void*, size_t, void*) {
  return DBK_ESHAPE;
}
int dbk_tc_gemv(const void*, const void*, const void*, void*, int, int, int, int, void*, size_t,
                void*) {
  return DBK_ESHAPE;
}
size_t dbk_tc_workspace_bytes(int, int64_t, int64_t, int64_t) { return 0; }

extern "C" size_t dbk_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out) {
  if (batch <= dbk::kSimtMaxBatch) return 0;
  return dbk_tc_workspace_bytes(op, batch, d_in, d_out);
}
