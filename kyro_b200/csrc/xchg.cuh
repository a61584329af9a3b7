// xchg.cuh -- the layout of a rank's peer-exchange region and the device
// helpers of one exchange round, shared by the exchange kernel
// (peer_exchange.cu) and the tensor-parallel sampler kernels that store
// their round-1 payload straight into the peers' regions (sampler.cu).
//
// Region of one rank (mapped by every peer through CUDA IPC):
//   [0, 64 * 2 * 8)    flag[p][s]: the last round of parity s whose payload
//                      peer p has completed in this region (64 bytes apart)
//   [2048, 2056)       this rank's round counter
//   [2112, 2116)       finished-CTA count of a round pushed by a producer
//                      kernel (back at zero when the round's flags are up)
//   [4096, 4096+2H)    two halves (round parity) of world slots, slot p
//                      holding peer p's payload of the current round
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace kyro {
namespace xchg {

constexpr size_t kCtlBytes = 4096;
constexpr size_t kFlagStride = 64;
constexpr size_t kSeqOffset = 2048;
constexpr size_t kDoneOffset = 2112;
constexpr size_t kHalfBytes = size_t(4) << 20;  // one parity half: world slots of one round
static_assert(2 * KYRO_MAX_TP_WORLD * kFlagStride <= kSeqOffset, "flags overlap the counter");
static_assert(kDoneOffset + 4 <= kCtlBytes, "the count overlaps the slots");

struct Peers {
  uint8_t* p[KYRO_MAX_TP_WORLD];  // every rank's region, mapped here (own: local)
};

// the bytes between two senders' slots for a payload of `bytes`
__host__ __device__ __forceinline__ size_t slot_stride(size_t bytes) {
  return (bytes + 15) & ~size_t(15);
}

// flag[p][s] of a region
__device__ __forceinline__ unsigned long long* flag_of(uint8_t* region, int p,
                                                       unsigned long long seq) {
  return reinterpret_cast<unsigned long long*>(region + ((size_t)p * 2 + (size_t)(seq & 1ull)) *
                                                             kFlagStride);
}

// slot of sender `from` for round seq
__device__ __forceinline__ uint8_t* slot_of(uint8_t* region, unsigned long long seq, int from,
                                            size_t stride) {
  return region + kCtlBytes + (size_t)(seq & 1ull) * kHalfBytes + (size_t)from * stride;
}

__device__ __forceinline__ unsigned long long* round_counter(uint8_t* region) {
  return reinterpret_cast<unsigned long long*>(region + kSeqOffset);
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One thread waits until sender p's flag of round seq's parity reads seq,
// giving up after wait_ns; returns false on timeout.
__device__ __forceinline__ bool wait_flag(uint8_t* own, int p, unsigned long long seq,
                                          unsigned long long wait_ns) {
  const unsigned long long* flag = flag_of(own, p, seq);
  if (ld_acquire_sys(flag) >= seq) return true;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(flag) < seq) {
    if (globaltimer() - t0 > wait_ns) return false;
    __nanosleep(64);
  }
  return true;
}

}  // namespace xchg
}  // namespace kyro
