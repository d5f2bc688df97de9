// Layout and flag protocol of the NVLink peer buffers shared by the peer-memory all-reduce
// (peer_allreduce.cu) and the kernels that fuse their own reduction into it (lut_grad.cu).
//
// Buffer: [flags kPeerMaxSlices x kPeerMaxRanks u32][call counter kPeerMaxSlices u32] (header),
//         then 2 (call parity) x kPeerMaxRanks (sender) x capacity f32 receive areas.
// Slot (slice) b of a call: the sending rank stores its data into the receivers' areas
// (parity = call & 1, sender = its rank), then flag [b][sender] = call in every rank's
// header; a receiver waits until every sender's flag for b reached the call (signed compare:
// the flags are monotone call counters), then reads its own areas. The per-slot call counter
// lives in the rank's own header, so CUDA-graph replays advance it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tropnn_b200.h"

namespace tropnn_b200 {
namespace peer {

constexpr int kPeerMaxRanks = TROPNN_B200_PEER_MAX_RANKS;
constexpr int kPeerMaxSlices = 512;
constexpr unsigned long long kPeerWaitLimitNs = 2000ull * 1000ull * 1000ull;
constexpr size_t kPeerFlagWords = size_t(kPeerMaxSlices) * kPeerMaxRanks + kPeerMaxSlices;
constexpr size_t kPeerHeaderBytes = (kPeerFlagWords * 4 + 255) / 256 * 256;

__device__ __forceinline__ uint32_t *flags(unsigned char *b) { return reinterpret_cast<uint32_t *>(b); }
__device__ __forceinline__ uint32_t *counters(unsigned char *b) {
  return reinterpret_cast<uint32_t *>(b) + kPeerMaxSlices * kPeerMaxRanks;
}
__device__ __forceinline__ float *recv(unsigned char *b, int64_t capacity, uint32_t parity, int sender) {
  return reinterpret_cast<float *>(b + kPeerHeaderBytes) + (int64_t(parity) * kPeerMaxRanks + sender) * capacity;
}

__device__ __forceinline__ void store_volatile(uint32_t *p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_volatile(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t peer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One thread: publishes this rank's arrival at slot b of `call` in every rank's header (after
// a system fence, so the stores before it are visible first), then waits (bounded) until every
// rank arrived. Returns false after kPeerWaitLimitNs, raising *error_word.
__device__ inline bool slot_barrier(unsigned char *const *bufs, int world, int rank, int b, uint32_t call,
                                    int *error_word) {
  __threadfence_system();
  for (int p = 0; p < world; ++p) store_volatile(flags(bufs[p]) + b * kPeerMaxRanks + rank, call);
  const uint32_t *mine = flags(bufs[rank]) + b * kPeerMaxRanks;
  const uint64_t start = peer_ns();
  for (int p = 0; p < world; ++p) {
    while (static_cast<int32_t>(load_volatile(mine + p) - call) < 0) {
      if (peer_ns() - start > kPeerWaitLimitNs) {
        atomicExch(error_word, 1);
        __threadfence_system();
        return false;
      }
    }
  }
  __threadfence_system();
  return true;
}

}  // namespace peer
}  // namespace tropnn_b200
