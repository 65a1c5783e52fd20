// comm.cuh - layout of the peer-exchange comm buffer and the device helpers
// shared by the all-gather kernel (comm.cu) and the kernels that fuse the
// all-gather into their epilogue (gemv.cu).
//
// Comm buffer of each rank (allocated by dbk_comm_alloc, zero-filled):
//   [0, 8)         uint64 epoch   exchanges completed by this rank
//   [8, 12)        uint32 arrive  CTAs of the running exchange that finished
//   [256, +10 KB)  uint64 flag[8][160]  flag[p][c]: last exchange CTA c of rank p delivered
//   [kHeader, ...) staging[2][world][capacity]
// Every exchange (standalone or fused) advances the epoch by one on every rank,
// so the sequence numbers written into the flag slots agree across ranks.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace dbk {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 160;          // >= SMs per GPU: one flag slot per CTA
constexpr size_t kFlags = 256;
constexpr size_t kHeader = kFlags + (size_t)kMaxWorld * kMaxCtas * 8;   // 10496, 256-aligned

// What a kernel needs to take part in an exchange (passed by value).
struct PeerSet {
  char* peer[kMaxWorld];   // comm buffer of every rank (peer[rank] is local)
  long long capacity;      // staging bytes per rank block
  int rank, world;         // world <= 1: no exchange
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long* flag_slot(char* buf, int src_rank, int cta) {
  return reinterpret_cast<unsigned long long*>(buf + kFlags) + src_rank * kMaxCtas + cta;
}

// Staging block of rank `src` in the buffer `buf`, for sequence parity `parity`.
__device__ __forceinline__ char* staging(char* buf, const PeerSet& ps, int parity, int src) {
  return buf + kHeader + ((long long)parity * ps.world + src) * ps.capacity;
}

// Bounded wait until *f >= v (acquire); records kDevTimeoutPeer and gives up.
__device__ __forceinline__ bool wait_flag(const unsigned long long* f, unsigned long long v) {
  uint32_t n = 0;
  const uint32_t lim = spin_limit();
  while (ld_acquire_sys(f) < v) {
    if (++n >= lim) {
      record_error(kDevTimeoutPeer);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

// Called by thread 0 of every CTA at the end of an exchange: the last CTA to get
// here advances the local epoch (read by the next exchange after its
// griddepcontrol.wait, i.e. after this grid has completed).
__device__ __forceinline__ void finish_exchange(char* local, unsigned long long e) {
  __threadfence();
  auto* arrive = reinterpret_cast<unsigned int*>(local + 8);
  if (atomicAdd(arrive, 1u) == gridDim.x - 1) {
    *arrive = 0;
    *reinterpret_cast<volatile unsigned long long*>(local) = e + 1;
  }
}

}  // namespace dbk
