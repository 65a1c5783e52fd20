// stage.cu - stream-ordered copies of a decode step's small inputs and outputs
// between pinned host memory and the GPU, done by a kernel.
//
// A decode step moves a few KB in (the token's activation or query) and a few KB
// out (the result) around a 10-300 us kernel. A copy-engine transfer of that size
// costs several microseconds of fixed latency on each side and breaks the chain
// of programmatic dependent launches. Here a small kernel reads (or writes) the
// pinned host buffer directly through its unified-address mapping:
//   * it releases its dependents at once, so the next kernel (a GEMV) starts
//     streaming its weights while the input is still arriving; the dependent's
//     griddepcontrol.wait still orders its reads of the input after this copy;
//   * a copy out waits for the producing kernel (griddepcontrol.wait) and writes
//     the result into host memory with ordinary stores; the stream's completion
//     (event, synchronize) makes it visible to the host.
// Not in the reference, whose harness copies with cudaMemcpy.
#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

constexpr int kCopyThreads = 256;

struct CopyArgs {
  char* dst;
  const char* src;
  long long n16;     // 16-byte units
  long long tail;    // bytes after the units
};

__global__ void __launch_bounds__(kCopyThreads) stage_copy_kernel(const CopyArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (long long i = i0; i < a.n16; i += stride)
    reinterpret_cast<uint4*>(a.dst)[i] = __ldcv(reinterpret_cast<const uint4*>(a.src) + i);
  if (i0 < a.tail) a.dst[a.n16 * 16 + i0] = a.src[a.n16 * 16 + i0];
}

// Device-usable address of p: device memory as is, pinned (mapped) host memory
// through its device pointer; nullptr for pageable host memory.
const void* device_view(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return p;
  if (at.type == cudaMemoryTypeHost) return at.devicePointer;
  return nullptr;
}

}  // namespace
}  // namespace dbk

extern "C" int dbk_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src) return DBK_ENULL;
  if (bytes == 0) return DBK_OK;
  const void* s = dbk::device_view(src);
  void* d = const_cast<void*>(dbk::device_view(dst));
  if (!s || !d) return DBK_EDEVICE;   // pageable host memory: not reachable by a kernel
  if ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) return DBK_EALIGN;
  dbk::CopyArgs a;
  a.dst = static_cast<char*>(d);
  a.src = static_cast<const char*>(s);
  a.n16 = (long long)(bytes / 16);
  a.tail = (long long)(bytes % 16);
  long long grid = (a.n16 + 2 * dbk::kCopyThreads - 1) / (2 * dbk::kCopyThreads);
  if (grid < 1) grid = 1;
  if (grid > 64) grid = 64;
  return dbk::launch_pdl(reinterpret_cast<const void*>(dbk::stage_copy_kernel), dim3((unsigned)grid),
                         dim3(dbk::kCopyThreads), 0, static_cast<cudaStream_t>(stream), &a);
}
