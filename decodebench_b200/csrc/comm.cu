// comm.cu - the shard-boundary all-gather over NVLink peer memory.
//
// The multi-GPU decode path (weight rows or kv heads split over the GPUs of one
// node) ends every sharded op with an all-gather of its small output (8 KB to
// 1 MB). This kernel does the exchange with plain stores into the peers' memory
// (CUDA IPC mappings, through NVSwitch) and one counter per peer:
//
//   1. every CTA stores its share of this rank's block into each peer's staging
//      area (and straight into the local output), then one thread writes the
//      exchange's sequence number into the CTA's flag slot in each peer with a
//      system-scope release store (which orders the CTA's data stores before it);
//   2. every CTA waits (bounded, acquire loads) until every flag slot of every
//      peer holds this exchange's sequence number, i.e. all CTAs of all peers
//      have delivered (every rank runs the same exchanges in the same order with
//      the same grid size, so sequence numbers and slots agree);
//   3. the CTAs copy the peers' blocks from local staging to the output layout;
//   4. the last CTA to finish advances the local sequence number.
//
// Staging is double-buffered by epoch parity. A peer can write step e + 2 into
// the half this rank reads at step e only after its own step e + 1 exchange has
// finished, which needs this rank's step e + 1 signal, which comes after this
// rank's step e kernel has completed (stream order): the halves never race.
//
// The comm buffer layout is in comm.cuh.
//
// No TMA and no multicast: only ordinary loads and stores, which is the only
// kind of access to another GPU's memory this library makes.
//
// There is no counterpart in the reference, which is single-GPU; the collective
// it replaces in this build is ncclAllGather at the shard boundary.
#include <cstring>
#include <new>

#include "comm.cuh"
#include "common.cuh"
#include "dbk_internal.h"

namespace dbk {
namespace {

constexpr int kAgThreads = 256;

struct AgArgs {
  char* peer[kMaxWorld];      // comm buffer of every rank (peer[rank] is local)
  const char* src;            // this rank's block: rows x row_bytes, rows src_ld apart
  char* out;                  // rank p's row i lands at out + p * out_block + i * out_ld
  long long src_ld, out_ld, out_block, capacity;
  int rank, world, rows, row_units;   // row_units = row_bytes / 16
};


__global__ void __launch_bounds__(kAgThreads) allgather_kernel(const AgArgs a) {
  DBK_MARK(threadIdx.x == 0, 6);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // src comes from the previous kernel
  char* local = a.peer[a.rank];
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(local);
  const int parity = (int)(e & 1);
  DBK_MARK(threadIdx.x == 0, 0);
  const long long units = (long long)a.rows * a.row_units;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;

  // 1. push this rank's block to every peer's staging, and to the local output
  for (long long u = first; u < units; u += stride) {
    const int i = (int)(u / a.row_units), c = (int)(u % a.row_units);
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.src + i * a.src_ld) + c);
    reinterpret_cast<uint4*>(a.out + a.rank * a.out_block + i * a.out_ld)[c] = v;
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      char* st = a.peer[p] + kHeader + ((long long)parity * a.world + a.rank) * a.capacity;
      reinterpret_cast<uint4*>(st + (long long)i * a.row_units * 16)[c] = v;
    }
  }
  DBK_MARK(threadIdx.x == 0, 1);
  __syncthreads();              // the CTA's stores happen before thread 0's release
  DBK_MARK(threadIdx.x == 0, 2);
  if ((int)threadIdx.x < a.world && (int)threadIdx.x != a.rank)   // release: cumulative over
    st_release_sys(flag_slot(a.peer[threadIdx.x], a.rank, blockIdx.x), e + 1);  // the CTA's stores

  DBK_MARK(threadIdx.x == 0, 3);
  // 2. wait until every CTA slot of every peer holds this exchange's number
  const int nslots = a.world * (int)gridDim.x;
  for (int t = threadIdx.x; t < nslots; t += blockDim.x) {
    const int p = t / (int)gridDim.x, c = t % (int)gridDim.x;
    if (p == a.rank) continue;
    wait_flag(flag_slot(local, p, c), e + 1);
  }
  __syncthreads();
  DBK_MARK(threadIdx.x == 0, 4);

  // 3. peers' blocks: local staging -> output layout
  const long long all = units * (a.world - 1);
  for (long long u = first; u < all; u += stride) {
    const int q = (int)(u / units);
    const long long w = u % units;
    const int p = q + (q >= a.rank ? 1 : 0);
    const int i = (int)(w / a.row_units), c = (int)(w % a.row_units);
    const char* st = local + kHeader + ((long long)parity * a.world + p) * a.capacity;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(st + (long long)i * a.row_units * 16) + c);
    reinterpret_cast<uint4*>(a.out + p * a.out_block + i * a.out_ld)[c] = v;
  }

  // 4. the last CTA advances the sequence number (read by the next exchange
  //    after its griddepcontrol.wait, i.e. after this grid has completed)
  __syncthreads();
  if (threadIdx.x == 0) finish_exchange(local, e);
  DBK_MARK(threadIdx.x == 0, 5);
  asm volatile("griddepcontrol.launch_dependents;");
}

// What one rank publishes to the others (dbk_comm_alloc -> dbk_comm_open).
struct PeerRecord {
  cudaIpcMemHandle_t handle;   // 64 bytes
  unsigned char uuid[16];      // GPU identity: no two ranks may share a GPU
  unsigned long long capacity; // staging bytes per rank
  int world;
  int device;
  unsigned char pad[128 - 64 - 16 - 8 - 4 - 4];
};
static_assert(sizeof(PeerRecord) == DBK_COMM_RECORD_BYTES, "peer record size");

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace
}  // namespace dbk

struct dbk_comm {
  char* peer[dbk::kMaxWorld];
  bool opened[dbk::kMaxWorld];
  int rank, world, device, nsms;
  size_t capacity;
};

using dbk::PeerRecord;

int dbk::comm_peerset(const dbk_comm* c, dbk::PeerSet* ps) {
  if (!c || !ps) return DBK_ENULL;
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return (int)e;
  if (cur != c->device) return DBK_EDEVICE;
  for (int p = 0; p < dbk::kMaxWorld; ++p) ps->peer[p] = p < c->world ? c->peer[p] : nullptr;
  ps->capacity = (long long)c->capacity;
  ps->rank = c->rank;
  ps->world = c->world;
  return DBK_OK;
}

extern "C" size_t dbk_comm_buffer_bytes(size_t capacity_per_rank, int world) {
  if (world < 1 || world > dbk::kMaxWorld) return 0;
  return dbk::kHeader + 2 * (size_t)world * dbk::round_up(capacity_per_rank, 256);
}

extern "C" int dbk_comm_alloc(size_t capacity_per_rank, int world, void** buf_out,
                              void* record_out) {
  if (!buf_out || !record_out) return DBK_ENULL;
  if (world < 1 || world > dbk::kMaxWorld || capacity_per_rank == 0) return DBK_ESHAPE;
  dbk::DeviceInfo dev;
  if (int rc = dbk::current_device_info(&dev)) return rc;
  const size_t cap = dbk::round_up(capacity_per_rank, 256);
  const size_t bytes = dbk_comm_buffer_bytes(cap, world);
  void* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, bytes);
  if (e != cudaSuccess) return (int)e;
  PeerRecord rec;
  std::memset(&rec, 0, sizeof(rec));
  cudaDeviceProp prop;
  if ((e = cudaMemset(buf, 0, bytes)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(&rec.handle, buf)) != cudaSuccess ||
      (e = cudaGetDeviceProperties(&prop, dev.device)) != cudaSuccess) {
    cudaFree(buf);
    return (int)e;
  }
  std::memcpy(rec.uuid, &prop.uuid, 16);
  rec.capacity = cap;
  rec.world = world;
  rec.device = dev.device;
  std::memcpy(record_out, &rec, sizeof(rec));
  *buf_out = buf;
  return DBK_OK;
}

extern "C" int dbk_comm_open(int rank, int world, void* local_buf, const void* records,
                             dbk_comm** out) {
  if (!local_buf || !records || !out) return DBK_ENULL;
  if (world < 1 || world > dbk::kMaxWorld || rank < 0 || rank >= world) return DBK_ESHAPE;
  dbk::DeviceInfo dev;
  if (int rc = dbk::current_device_info(&dev)) return rc;
  const auto* rec = static_cast<const PeerRecord*>(records);
  for (int p = 0; p < world; ++p) {
    if (rec[p].world != world || rec[p].capacity != rec[0].capacity) return DBK_ESHAPE;
    // Ranks whose exchanges wait on one another must run on different GPUs.
    for (int q = 0; q < p; ++q)
      if (std::memcmp(rec[p].uuid, rec[q].uuid, 16) == 0) return DBK_EDEVICE;
  }
  // One flag slot per CTA: the exchanging grids (at most one CTA per SM) must fit.
  if (dev.num_sms > dbk::kMaxCtas) return DBK_EDEVICE;
  auto* c = new (std::nothrow) dbk_comm();
  if (!c) return DBK_ESHAPE;
  c->rank = rank;
  c->world = world;
  c->device = dev.device;
  c->nsms = dev.num_sms;
  c->capacity = rec[0].capacity;
  for (int p = 0; p < world; ++p) {
    if (p == rank) {
      c->peer[p] = static_cast<char*>(local_buf);
      continue;
    }
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, rec[p].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (c->opened[q]) cudaIpcCloseMemHandle(c->peer[q]);
      delete c;
      return (int)e;
    }
    c->peer[p] = static_cast<char*>(ptr);
    c->opened[p] = true;
  }
  *out = c;
  return DBK_OK;
}

extern "C" int dbk_comm_close(dbk_comm* c) {
  if (!c) return DBK_ENULL;
  int rc = DBK_OK;
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) {
      cudaError_t e = cudaIpcCloseMemHandle(c->peer[p]);
      if (e != cudaSuccess && rc == DBK_OK) rc = (int)e;
    }
  delete c;
  return rc;
}

extern "C" int dbk_comm_free(void* buf) {
  if (!buf) return DBK_ENULL;
  cudaError_t e = cudaFree(buf);
  return e == cudaSuccess ? DBK_OK : (int)e;
}

extern "C" int dbk_allgather(dbk_comm* c, const void* src, void* out, int rows, size_t row_bytes,
                             size_t src_ld, size_t out_ld, size_t out_block, void* stream) {
  if (!c || !src || !out) return DBK_ENULL;
  if (rows < 1 || row_bytes == 0) return DBK_ESHAPE;
  if (row_bytes % 16 || src_ld % 16 || out_ld % 16 || out_block % 16 || src_ld < row_bytes ||
      (rows > 1 && out_ld < row_bytes))
    return DBK_EALIGN;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15) return DBK_EALIGN;
  if ((size_t)rows * row_bytes > c->capacity) return DBK_EWORKSPACE;
  dbk::AgArgs a{};
  for (int p = 0; p < c->world; ++p) a.peer[p] = c->peer[p];
  a.src = static_cast<const char*>(src);
  a.out = static_cast<char*>(out);
  a.src_ld = (long long)src_ld;
  a.out_ld = (long long)out_ld;
  a.out_block = (long long)out_block;
  a.capacity = (long long)c->capacity;
  a.rank = c->rank;
  a.world = c->world;
  a.rows = rows;
  a.row_units = (int)(row_bytes / 16);
  // The grid size is a function of the shape and the SM count only, so that every
  // rank (same shape, same GPU model) counts the same number of CTAs per peer.
  const long long units = (long long)rows * a.row_units;
  long long grid = (units + 2 * dbk::kAgThreads - 1) / (2 * dbk::kAgThreads);
  if (grid < 1) grid = 1;
  if (grid > c->nsms) grid = c->nsms;
  if (grid > dbk::kMaxCtas) grid = dbk::kMaxCtas;
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return (int)e;
  if (cur != c->device) return DBK_EDEVICE;
  return dbk::launch_pdl(reinterpret_cast<const void*>(dbk::allgather_kernel), dim3((unsigned)grid),
                         dim3(dbk::kAgThreads), 0, static_cast<cudaStream_t>(stream), &a);
}
