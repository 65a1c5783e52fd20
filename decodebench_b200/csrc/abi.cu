// abi.cu - C-ABI utilities: versions, status strings, device info, PDL launch,
// the device error flag written by kernels that gave up a bounded wait.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "comm.cuh"
#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {

__device__ int dbk_device_error = 0;
__constant__ uint32_t dbk_spin_limit = kSpinLimit;
#ifdef DBK_TRACE
__device__ unsigned long long dbk_trace[4 * 2048 * 16];
__device__ unsigned int dbk_trace_ticket;
}  // namespace dbk
// Development builds only: copies the phase timestamps to the host / clears them.
extern "C" int dbk_trace_read(void* host, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(host, dbk::dbk_trace, bytes);
}
extern "C" int dbk_trace_clear(void) {
  static unsigned long long zeros[4 * 2048 * 16];
  unsigned int z = 0;
  cudaError_t e = cudaMemcpyToSymbol(dbk::dbk_trace, zeros, sizeof(zeros));
  if (e != cudaSuccess) return (int)e;
  return (int)cudaMemcpyToSymbol(dbk::dbk_trace_ticket, &z, sizeof(z));
}
namespace dbk {
#endif

namespace {
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
bool g_have[kMaxDevices];
std::mutex g_mu;

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DBK_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}
}  // namespace

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return DBK_EDEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_have[dev]) {
    DeviceInfo d{};
    d.device = dev;
    if ((e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev))) return (int)e;
    if ((e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)))
      return (int)e;
    if ((e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev))) return (int)e;
    g_info[dev] = d;
    g_have[dev] = true;
  }
  if (g_info[dev].cc_major != 10) return DBK_EDEVICE;
  *out = g_info[dev];
  return DBK_OK;
}

namespace {
std::mutex g_attr_mu;
struct AttrDone {
  const void* kern;
  int device;
  int most;      // dynamic shared memory limit that was set
};
std::vector<AttrDone> g_attr_done;
}  // namespace

int allow_dynamic_smem(const void* kern, const DeviceInfo& dev, size_t smem) {
  if (smem > (size_t)dev.max_smem_optin) return DBK_ESHAPE;
  if (smem <= 48 * 1024) return DBK_OK;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  for (const auto& kd : g_attr_done)
    if (kd.kern == kern && kd.device == dev.device)
      return (long long)smem > kd.most ? DBK_ESHAPE : DBK_OK;
  // Raise the limit to the most the kernel can have (the opt-in maximum less its
  // static shared memory) once; launches then pass their own size.
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return (int)e;
  const int most = dev.max_smem_optin - (int)fa.sharedSizeBytes;
  if ((long long)smem > most) return DBK_ESHAPE;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
  if (e != cudaSuccess) return (int)e;
  g_attr_done.push_back(AttrDone{kern, dev.device, most});
  return DBK_OK;
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

int encode_tmap_2d(CUtensorMap* out, const void* base, int dtype, uint64_t inner, uint64_t rows,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                   bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return (int)cudaErrorNotSupported;
  if (!aligned16(base) || (row_stride_bytes % 16) != 0 || (box_inner * 2) % 16 != 0)
    return DBK_EALIGN;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dtype == DBK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DBK_OK : DBK_ESHAPE;
}

int encode_tmap_kv3d(CUtensorMap* out, const void* base, int dtype, uint64_t rows,
                     uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return (int)cudaErrorNotSupported;
  if (!aligned16(base)) return DBK_EALIGN;
  const cuuint64_t dims[3] = {64, rows, 2};
  const cuuint64_t strides[2] = {256, 128};
  if (box_rows < 8 || box_rows > 256) return DBK_ESHAPE;
  const cuuint32_t box[3] = {64, box_rows, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(out, dtype == DBK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DBK_OK : DBK_ESHAPE;
}

int launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               void* args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  void* params[1] = {args};
  cudaError_t e = cudaLaunchKernelExC(&cfg, func, params);
  return e == cudaSuccess ? DBK_OK : (int)e;
}

}  // namespace dbk

extern "C" int dbk_abi_version(void) { return DBK_ABI_VERSION; }

extern "C" const char* dbk_status_string(int s) {
  switch (s) {
    case DBK_OK: return "ok";
    case DBK_ENULL: return "a required pointer is NULL";
    case DBK_ESHAPE: return "a size is outside the supported range";
    case DBK_EALIGN: return "a pointer or row stride is not 16-byte aligned";
    case DBK_EWORKSPACE: return "workspace missing or too small";
    case DBK_EDTYPE: return "unknown dtype";
    case DBK_EDEVICE: return "current device is not an sm_100 (B200) GPU";
    default: break;
  }
  if (s > 0) return cudaGetErrorString(static_cast<cudaError_t>(s));
  return "unknown status";
}

extern "C" int dbk_take_device_error(void) {
  int v = 0, zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return (int)e;
  e = cudaMemcpyFromSymbol(&v, dbk::dbk_device_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  e = cudaMemcpyToSymbol(dbk::dbk_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  return v;
}

extern "C" int dbk_set_spin_limit(uint32_t polls) {
  const uint32_t v = polls == 0 ? dbk::kSpinLimit : polls;
  return (int)cudaMemcpyToSymbol(dbk::dbk_spin_limit, &v, sizeof(v));
}

// ---------------------------------------------------------------------------
// Test hook: one CTA runs the library's own bounded waits on events that never
// happen, so that a test can watch a wait give up, record its code and return.
namespace dbk {
namespace {
__device__ unsigned long long g_never_set_flag = 0;

__global__ void bounded_wait_probe_kernel(int which) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  if (which == 0) {
    // An mbarrier expecting one arrival that nobody makes.
    mbar_init(&bar, 1);
    fence_barrier_init();
    (void)mbar_wait(&bar, 0, kDevTimeoutFull);
  } else {
    // A peer flag that no peer ever raises.
    (void)wait_flag(&g_never_set_flag, 1ull);
  }
}
}  // namespace
}  // namespace dbk

extern "C" int dbk_test_bounded_wait(int which, void* stream) {
  if (which != 0 && which != 1) return DBK_ESHAPE;
  dbk::bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(which);
  return (int)cudaGetLastError();
}
