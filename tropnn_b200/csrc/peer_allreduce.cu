// Gradient all-reduce over NVLink peer memory (one process per GPU, one node). Buffer layout
// and flag protocol: peer.cuh.
//
// The reference is single-device; the b200 layers scale by batch-row sharding and
// average their parameter gradients across ranks after the backward. NCCL takes ~22 us
// for the 2 MiB LUT gradient of config 2 on two B200s (a latency-bound protocol), a
// fifth of the 0.1 ms step. This is a push-based one-shot all-reduce for that size range:
// every rank exposes one "peer buffer" (cudaMalloc + CUDA IPC handle, opened by the other
// ranks) holding a receive area per sending rank, and one kernel per rank
//   phase 0  stores its gradient tensors straight into every rank's receive area over
//            NVLink (posted stores: no round trip per access),
//   barrier  after a system fence, a flag stored into every rank's buffer; spin on its own
//            flags (each rank's flag is a call counter, so a rank that already moved on to
//            the next call still counts as arrived),
//   phase 1  sums the W received copies from its own memory in rank order (bit-identical
//            results on every rank) and writes them (times 1/W when averaging) back.
// Receive areas are double-buffered by call parity: a rank can only start call k+2, which
// reuses call k's area, after every rank arrived at the barrier of call k+1, i.e. after
// every rank finished reading call k's copies. CTA b of every rank owns slice b, so the
// barrier is per CTA, and the per-CTA call counter lives on the device, so CUDA-graph
// replays advance it too. Each wait is bounded (kWaitLimitNs): a rank that does not
// arrive makes the others give up, set the library's error word and return.
// More than two ranks use a two-shot variant (reduce-scatter by pushes, then all-gather by
// pushes; below). Loads and stores only: no TMA, no multicast, no NVLink multicast objects.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "peer.cuh"
#include "tropnn_b200.h"

namespace tropnn_b200 {

namespace {

using namespace peer;

constexpr int kMaxRanks = kPeerMaxRanks;
constexpr int kMaxSegments = TROPNN_B200_PEER_MAX_SEGMENTS;
constexpr int kMaxSlices = kPeerMaxSlices;  // CTAs per call
constexpr int kThreads = 512;
constexpr unsigned long long kWaitLimitNs = kPeerWaitLimitNs;
constexpr size_t kHeaderBytes = kPeerHeaderBytes;

__device__ int g_peer_error = 0;

struct PeerArgs {
  unsigned char *buf[kMaxRanks];        // every rank's peer buffer, mapped into this process
  float *seg[kMaxSegments];             // caller's tensors (this rank)
  int64_t seg_begin[kMaxSegments + 1];  // prefix sums of the segment lengths
  int nseg;
  int world;
  int rank;
  int64_t count;     // total floats
  int64_t slice;     // floats per CTA slice (a multiple of 4)
  int64_t capacity;  // floats per receive area
  float scale;       // 1/world when averaging, else 1
};

__device__ __forceinline__ uint64_t global_ns() { return peer_ns(); }

// Element i of the caller's concatenated segments.
__device__ __forceinline__ float *seg_ptr(const PeerArgs &a, int64_t i) {
  int s = 0;
  while (s + 1 < a.nseg && i >= a.seg_begin[s + 1]) ++s;
  return a.seg[s] + (i - a.seg_begin[s]);
}

// Address of elements i..i+3 when they lie in one segment, 16-byte aligned; else null.
__device__ __forceinline__ float *seg_ptr4(const PeerArgs &a, int64_t i) {
  int s = 0;
  while (s + 1 < a.nseg && i >= a.seg_begin[s + 1]) ++s;
  float *p = a.seg[s] + (i - a.seg_begin[s]);
  return (i + 4 <= a.seg_begin[s + 1] && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) ? p : nullptr;
}

__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const PeerArgs a) {
  __shared__ int ok_s;
  __shared__ uint32_t call_s;
  const int b = blockIdx.x;
  const int64_t lo = int64_t(b) * a.slice;
  const int64_t hi = min(a.count, lo + a.slice);
  unsigned char *mine = a.buf[a.rank];
  if (threadIdx.x == 0) call_s = counters(mine)[b] + 1;
  __syncthreads();
  const uint32_t call = call_s;
  const uint32_t parity = call & 1u;

  // Phase 0: push this rank's slice into every rank's receive area for this sender.
  for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * blockDim.x) {
    float4 v;
    const float *p4 = seg_ptr4(a, i);
    if (p4 != nullptr) {
      v = *reinterpret_cast<const float4 *>(p4);
    } else {
      v.x = *seg_ptr(a, i);
      v.y = i + 1 < hi ? *seg_ptr(a, i + 1) : 0.f;
      v.z = i + 2 < hi ? *seg_ptr(a, i + 2) : 0.f;
      v.w = i + 3 < hi ? *seg_ptr(a, i + 3) : 0.f;
    }
    for (int p = 0; p < a.world; ++p)
      *reinterpret_cast<float4 *>(recv(a.buf[p], a.capacity, parity, a.rank) + i) = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Every push of this CTA is visible system-wide before the flags are.
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) store_volatile(flags(a.buf[p]) + b * kMaxRanks + a.rank, call);
    const uint32_t *mine_flags = flags(mine) + b * kMaxRanks;
    const uint64_t start = global_ns();
    int ok = 1;
    for (int p = 0; p < a.world && ok; ++p) {
      while (static_cast<int32_t>(load_volatile(mine_flags + p) - call) < 0) {
        if (global_ns() - start > kWaitLimitNs) {
          atomicExch(&g_peer_error, 1);
          ok = 0;
          break;
        }
      }
    }
    __threadfence_system();
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;

  // Phase 1: sum the received copies (this GPU's memory) in rank order.
  for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * blockDim.x) {
    float4 acc = __ldcg(reinterpret_cast<const float4 *>(recv(mine, a.capacity, parity, 0) + i));
    for (int p = 1; p < a.world; ++p) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(recv(mine, a.capacity, parity, p) + i));
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    const float4 r = make_float4(__fmul_rn(acc.x, a.scale), __fmul_rn(acc.y, a.scale), __fmul_rn(acc.z, a.scale),
                                 __fmul_rn(acc.w, a.scale));
    float *p4 = seg_ptr4(a, i);
    if (p4 != nullptr && i + 4 <= hi) {
      *reinterpret_cast<float4 *>(p4) = r;
    } else {
      *seg_ptr(a, i) = r.x;
      if (i + 1 < hi) *seg_ptr(a, i + 1) = r.y;
      if (i + 2 < hi) *seg_ptr(a, i + 2) = r.z;
      if (i + 3 < hi) *seg_ptr(a, i + 3) = r.w;
    }
  }
  if (threadIdx.x == 0) counters(mine)[b] = call;
}

// Bounded wait of one thread until every rank's flag for CTA b reached `target` (signed
// compare: flags are monotone counters). Returns false after kWaitLimitNs.
__device__ bool wait_flags(const uint32_t *mine_flags, int world, uint32_t target) {
  const uint64_t start = global_ns();
  for (int p = 0; p < world; ++p) {
    while (static_cast<int32_t>(load_volatile(mine_flags + p) - target) < 0) {
      if (global_ns() - start > kWaitLimitNs) {
        atomicExch(&g_peer_error, 1);
        return false;
      }
    }
  }
  return true;
}

// Two-shot variant for more than two ranks (the one-shot push sends (W-1) copies of the
// whole gradient per rank; this sends 2 (W-1)/W of it). CTA b's slice is cut into W chunks;
// chunk q belongs to rank q.
//   phase 0  push chunk q of this rank's slice into rank q's receive area (sender = this rank)
//   barrier  flag 2 call - 1
//   phase 1  sum chunk `rank` over the W received copies in rank order, scale, write it to
//            the caller's tensor and push it into every other rank's receive area at the same
//            place (sender = this rank: that chunk of that area is unused in phase 0)
//   barrier  flag 2 call
//   phase 2  copy the other ranks' reduced chunks from this rank's own memory to the tensor.
// Double-buffered by call parity as the one-shot kernel; every rank's result is bit-identical.
__global__ void __launch_bounds__(kThreads) peer_allreduce_2shot_kernel(const PeerArgs a) {
  __shared__ int ok_s;
  __shared__ uint32_t call_s;
  const int b = blockIdx.x;
  const int64_t lo = int64_t(b) * a.slice;
  const int64_t hi = min(a.count, lo + a.slice);
  // Chunk length: a multiple of 4 floats.
  const int64_t chunk = ((a.slice + a.world - 1) / a.world + 3) / 4 * 4;
  unsigned char *mine = a.buf[a.rank];
  if (threadIdx.x == 0) call_s = counters(mine)[b] + 1;
  __syncthreads();
  const uint32_t call = call_s;
  const uint32_t parity = call & 1u;
  uint32_t *mine_flags = flags(mine) + b * kMaxRanks;

  // Phase 0.
  for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * blockDim.x) {
    float4 v;
    const float *p4 = seg_ptr4(a, i);
    if (p4 != nullptr) {
      v = *reinterpret_cast<const float4 *>(p4);
    } else {
      v.x = *seg_ptr(a, i);
      v.y = i + 1 < hi ? *seg_ptr(a, i + 1) : 0.f;
      v.z = i + 2 < hi ? *seg_ptr(a, i + 2) : 0.f;
      v.w = i + 3 < hi ? *seg_ptr(a, i + 3) : 0.f;
    }
    const int q = static_cast<int>((i - lo) / chunk);
    *reinterpret_cast<float4 *>(recv(a.buf[q], a.capacity, parity, a.rank) + i) = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) store_volatile(flags(a.buf[p]) + b * kMaxRanks + a.rank, 2 * call - 1);
    ok_s = wait_flags(mine_flags, a.world, 2 * call - 1) ? 1 : 0;
    __threadfence_system();
  }
  __syncthreads();
  if (!ok_s) return;

  // Phase 1: this rank's chunk.
  const int64_t c_lo = lo + a.rank * chunk;
  const int64_t c_hi = min(hi, c_lo + chunk);
  for (int64_t i = c_lo + 4 * threadIdx.x; i < c_hi; i += 4 * blockDim.x) {
    float4 acc = __ldcg(reinterpret_cast<const float4 *>(recv(mine, a.capacity, parity, 0) + i));
    for (int p = 1; p < a.world; ++p) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(recv(mine, a.capacity, parity, p) + i));
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    const float4 r = make_float4(__fmul_rn(acc.x, a.scale), __fmul_rn(acc.y, a.scale), __fmul_rn(acc.z, a.scale),
                                 __fmul_rn(acc.w, a.scale));
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank) *reinterpret_cast<float4 *>(recv(a.buf[p], a.capacity, parity, a.rank) + i) = r;
    float *p4 = seg_ptr4(a, i);
    if (p4 != nullptr && i + 4 <= c_hi) {
      *reinterpret_cast<float4 *>(p4) = r;
    } else {
      *seg_ptr(a, i) = r.x;
      if (i + 1 < c_hi) *seg_ptr(a, i + 1) = r.y;
      if (i + 2 < c_hi) *seg_ptr(a, i + 2) = r.z;
      if (i + 3 < c_hi) *seg_ptr(a, i + 3) = r.w;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) store_volatile(flags(a.buf[p]) + b * kMaxRanks + a.rank, 2 * call);
    ok_s = wait_flags(mine_flags, a.world, 2 * call) ? 1 : 0;
    __threadfence_system();
  }
  __syncthreads();
  if (!ok_s) return;

  // Phase 2: the other ranks' reduced chunks, from this rank's memory.
  for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * blockDim.x) {
    const int q = static_cast<int>((i - lo) / chunk);
    if (q == a.rank) continue;
    const int64_t q_hi = min(hi, lo + (q + 1) * chunk);
    const float4 r = __ldcg(reinterpret_cast<const float4 *>(recv(mine, a.capacity, parity, q) + i));
    float *p4 = seg_ptr4(a, i);
    if (p4 != nullptr && i + 4 <= q_hi) {
      *reinterpret_cast<float4 *>(p4) = r;
    } else {
      *seg_ptr(a, i) = r.x;
      if (i + 1 < q_hi) *seg_ptr(a, i + 1) = r.y;
      if (i + 2 < q_hi) *seg_ptr(a, i + 2) = r.z;
      if (i + 3 < q_hi) *seg_ptr(a, i + 3) = r.w;
    }
  }
  if (threadIdx.x == 0) counters(mine)[b] = call;
}

}  // namespace

size_t peer_buffer_bytes(int64_t capacity) { return kHeaderBytes + size_t(2) * kMaxRanks * capacity * 4; }

}  // namespace tropnn_b200

using namespace tropnn_b200;

extern "C" {

int tropnn_b200_peer_buffer_create(int64_t capacity_floats, void **local, unsigned char *handle) {
  TB_CHECK(check_current_device());
  TB_REQUIRE(local && handle, TROPNN_B200_ERR_INVALID, "peer_buffer_create: null pointer");
  TB_REQUIRE(capacity_floats > 0 && capacity_floats % 64 == 0 && capacity_floats <= (int64_t(1) << 34),
             TROPNN_B200_ERR_INVALID, "peer_buffer_create: capacity %lld floats (a positive multiple of 64)",
             (long long)capacity_floats);
  void *p = nullptr;
  const size_t bytes = peer_buffer_bytes(capacity_floats);
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return set_error(TROPNN_B200_ERR_DEVICE, "peer_buffer_create: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(err));
  err = cudaMemset(p, 0, kHeaderBytes);
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    cudaFree(p);
    return set_error(TROPNN_B200_ERR_DEVICE, "peer_buffer_create: %s", cudaGetErrorString(err));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == TROPNN_B200_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *local = p;
  return clear_error();
}

int tropnn_b200_peer_buffer_open(const unsigned char *handle, void **peer) {
  TB_CHECK(check_current_device());
  TB_REQUIRE(handle && peer, TROPNN_B200_ERR_INVALID, "peer_buffer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return set_error(TROPNN_B200_ERR_DEVICE, "peer_buffer_open: %s", cudaGetErrorString(err));
  *peer = p;
  return clear_error();
}

int tropnn_b200_peer_buffer_close(void *peer) {
  TB_CHECK(check_current_device());
  cudaError_t err = cudaIpcCloseMemHandle(peer);
  if (err != cudaSuccess) return set_error(TROPNN_B200_ERR_DEVICE, "peer_buffer_close: %s", cudaGetErrorString(err));
  return clear_error();
}

int tropnn_b200_peer_buffer_destroy(void *local) {
  TB_CHECK(check_current_device());
  cudaError_t err = cudaFree(local);
  if (err != cudaSuccess) return set_error(TROPNN_B200_ERR_DEVICE, "peer_buffer_destroy: %s", cudaGetErrorString(err));
  return clear_error();
}

int tropnn_b200_peer_allreduce_f32(void *const *buffers, int world, int rank, int64_t capacity_floats,
                                   float *const *segments, const int64_t *counts, int nseg, int average,
                                   void *stream) {
  TB_CHECK(check_current_device());
  TB_REQUIRE(buffers && segments && counts, TROPNN_B200_ERR_INVALID, "peer_allreduce: null pointer");
  TB_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, TROPNN_B200_ERR_INVALID,
             "peer_allreduce: rank %d of world %d (at most %d ranks)", rank, world, kMaxRanks);
  TB_REQUIRE(nseg >= 1 && nseg <= kMaxSegments, TROPNN_B200_ERR_INVALID, "peer_allreduce: %d segments (1..%d)", nseg,
             kMaxSegments);
  TB_REQUIRE(capacity_floats > 0 && capacity_floats % 64 == 0, TROPNN_B200_ERR_INVALID,
             "peer_allreduce: capacity %lld floats (a positive multiple of 64)", (long long)capacity_floats);
  PeerArgs a{};
  a.world = world;
  a.rank = rank;
  a.nseg = nseg;
  a.capacity = capacity_floats;
  a.scale = average ? 1.f / float(world) : 1.f;
  int64_t total = 0;
  for (int s = 0; s < nseg; ++s) {
    TB_REQUIRE(counts[s] >= 0 && segments[s] != nullptr, TROPNN_B200_ERR_INVALID, "peer_allreduce: bad segment %d", s);
    a.seg[s] = segments[s];
    a.seg_begin[s] = total;
    total += counts[s];
  }
  a.seg_begin[nseg] = total;
  TB_REQUIRE(total <= capacity_floats, TROPNN_B200_ERR_INVALID,
             "peer_allreduce: %lld floats exceed the peer buffers' %lld", (long long)total, (long long)capacity_floats);
  if (total == 0 || world == 1) return clear_error();  // one rank: the average is the input
  for (int p = 0; p < world; ++p) {
    TB_REQUIRE(buffers[p] != nullptr, TROPNN_B200_ERR_INVALID, "peer_allreduce: buffer of rank %d is null", p);
    a.buf[p] = static_cast<unsigned char *>(buffers[p]);
  }
  // Slices of >= 2048 floats (a multiple of 4), at most kMaxSlices of them. The slice length
  // depends on the buffers' capacity only, so CTA b covers the same floats in every call and
  // its call counter orders every reuse of them (the parity double-buffering relies on it).
  int64_t slice = std::max<int64_t>(2048, ceil_div(capacity_floats, int64_t(kMaxSlices)));
  slice = ceil_div(slice, int64_t(4)) * 4;
  const int slices = static_cast<int>(ceil_div(total, slice));
  a.slice = slice;
  a.count = total;
  if (world > 2)
    peer_allreduce_2shot_kernel<<<slices, kThreads, 0, as_stream(stream)>>>(a);
  else
    peer_allreduce_kernel<<<slices, kThreads, 0, as_stream(stream)>>>(a);
  TB_CHECK(check_launch("peer_allreduce"));
  return clear_error();
}

}  // extern "C"

namespace tropnn_b200 {

int read_peer_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200
