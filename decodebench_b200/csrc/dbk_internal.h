// dbk_internal.h - host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "dbk.h"

namespace dbk {

// Largest batch served by the CUDA-core GEMV path; larger batches use tcgen05.
constexpr int kSimtMaxBatch = 8;

struct DeviceInfo {
  int device;
  int num_sms;
  int max_smem_optin;
  int cc_major;
};

// Cached per-device properties of the current device; DBK_EDEVICE if not sm_100.
int current_device_info(DeviceInfo* out);
// Lets `kern` launch with up to the device's opt-in shared memory (once per kernel and
// device; later calls only check `smem` against the limit).
int allow_dynamic_smem(const void* kern, const DeviceInfo& dev, size_t smem);

struct PeerSet;   // comm.cuh
// The peers of an open communicator, for kernels that fuse the all-gather
// (DBK_EDEVICE unless the current device is the communicator's).
int comm_peerset(const dbk_comm* c, PeerSet* ps);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Encode a 2-D tiled TMA descriptor over a row-major [rows, inner] matrix of
// 16-bit elements (dtype DBK_F16 / DBK_BF16), box [box_rows, box_inner], with
// 128-byte swizzle when swizzle128 (box_inner * 2 must then be 128), zero
// fill out of bounds. Returns DBK_OK or a DBK_E* / cudaError_t code.
int encode_tmap_2d(CUtensorMap* out, const void* base, int dtype, uint64_t inner, uint64_t rows,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                   bool swizzle128);

// 3-D tiled TMA descriptor viewing a row-major [rows, 128] matrix of 16-bit
// elements as [2 halves][rows][64] (strides 128 B and 256 B): one box (box_rows
// rows x both halves) reads box_rows whole 256-byte rows (box_rows * 256 bytes in
// one copy) and lands as 2 * box_rows swizzled 128-byte lines,
// line = box_rows * half + row, so 8 consecutive rows of one half occupy 8
// different swizzle phases (conflict-free ldmatrix).
int encode_tmap_kv3d(CUtensorMap* out, const void* base, int dtype, uint64_t rows,
                     uint32_t box_rows);

// Launch `func(*args)` (one by-value struct parameter) with programmatic
// dependent launch enabled unless DBK_PDL=0 is set in the environment.
int launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               void* args);

}  // namespace dbk

// Tensor-core (tcgen05) paths for batch > kSimtMaxBatch, defined in gemm_tc.cu.
int dbk_tc_rmsnorm_gemv(const void* x, const void* gamma, const void* W, void* y, int batch,
                        int d_in, int d_out, float eps, int dtype, void* ws, size_t ws_bytes,
                        void* stream);
int dbk_tc_gateup_swiglu(const void* x, const void* gamma, const void* Wg, const void* Wu,
                         void* h, int batch, int d_in, int d_ff, float eps, int dtype, void* ws,
                         size_t ws_bytes, void* stream);
int dbk_tc_gemv(const void* x, const void* W, const void* residual, void* y, int batch,
                int d_in, int d_out, int dtype, void* ws, size_t ws_bytes, void* stream);
size_t dbk_tc_workspace_bytes(int op, int64_t batch, int64_t d_in, int64_t d_out);
