// sm_100a building blocks shared by the tensor-core kernels: mbarriers with bounded
// waits, TMA tile loads, tcgen05 MMA / TMEM access and the tensor-map encoder.
//
// Every wait here is bounded by %globaltimer (kWaitLimitNs): a wait that gives up raises
// the caller's CTA abort flag and its library error word, so a protocol error ends the
// kernel instead of hanging the GPU. Every TMA load is a plain per-CTA load (no cluster
// delivery), so the kernels stay safe in multi-GPU processes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace tropnn_b200 {
namespace sm100 {

constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`. Returns false (raising *abort and
// *error_word) after kWaitLimitNs, or false at once once another role has aborted.
__device__ inline bool mbar_wait(uint64_t *bar, uint32_t parity, int *abort, int *error_word) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  volatile int *ab = abort;
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (*ab) return false;
      if (global_ns() - start > kWaitLimitNs) {
        *ab = 1;
        atomicExch(error_word, 1);
        return false;
      }
    }
  }
}

// Bounded wait as mbar_wait, polling with the mbarrier suspend-time hint `hint_ns`: the thread
// sleeps between polls until the phase completes (or the hint expires), so that whole warps
// can wait without taking issue slots from the TMA and MMA threads.
__device__ inline bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, int *abort, int *error_word, uint32_t hint_ns) {
  const uint64_t start = global_ns();
  volatile int *ab = abort;
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    if (ok) return true;
    if (*ab) return false;
    if (global_ns() - start > kWaitLimitNs) {
      *ab = 1;
      atomicExch(error_word, 1);
      return false;
    }
  }
}

// Drain-only wait used on exit paths: bounded, raises nothing.
__device__ inline void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > kWaitLimitNs) return;
  }
}

// 1-D bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// memory into this CTA's shared memory, completion counted on `bar` (no cluster delivery).
__device__ __forceinline__ void bulk_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2-D tiled TMA store from this CTA's shared memory (bulk-group completion); the rows and
// columns of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared-memory sources of all committed bulk stores have been read.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle layout: rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1, swizzle mode 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t(1) << 16;          // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;  // stride byte offset
  d |= uint64_t(1) << 46;          // descriptor version (sm_100)
  d |= uint64_t(2) << 61;          // SWIZZLE_128B
  return d;
}

// UMMA shared-memory descriptor of an MN-major tf32 operand: strips of 32 MN elements, each a
// run of 128-byte K rows in the 128-byte swizzle with 32-byte atoms (the 32-byte chunk index
// XOR (row & 3); 4-row groups 512 bytes apart, SBO), strips `strip_bytes` apart (LBO). (The
// 16-byte-atom swizzle is K-major only for tf32: MN-major tf32 MMAs on it produce nothing.)
__device__ __forceinline__ uint64_t umma_desc_mn_tf32(uint32_t saddr, uint32_t strip_bytes) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((strip_bytes >> 4) & 0x3FFFu) << 16;  // leading byte offset: MN strip stride
  d |= uint64_t(512 >> 4) << 32;                      // stride byte offset: 4-row K groups
  d |= uint64_t(1) << 46;
  d |= uint64_t(1) << 61;                             // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor of kind::tf32: f32 accumulator, A/B tf32, each K-major (false) or
// MN-major (true).
__host__ __device__ constexpr uint32_t umma_idesc_tf32(bool a_mn, bool b_mn, int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one M x N x 8 tf32 step.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// x rounded to tf32 (nearest, ties away; the low 13 mantissa bits zero), as an f32.
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Instruction descriptor of kind::f16: f32 accumulator, A/B f16 (0) or bf16 (1), both
// K-major, N and M in their encoded fields.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int ab_format, int m, int n) {
  return (1u << 4) | (uint32_t(ab_format) << 7) | (uint32_t(ab_format) << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one M x N x 16 step.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A's M rows in TMEM lanes, K packed two 16-bit
// elements per 32-bit column (8 columns per K=16 step).
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-collective TMEM allocation of `cols` columns (address written to *slot), and its
// release; both must run converged in one warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive 32-bit columns written to this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Ties registers written by tcgen05.ld to the preceding tcgen05.wait::ld, so that no use
// of them is scheduled above the wait.
__device__ __forceinline__ void reg_fence(float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+f"(v[i]));
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `threads` threads.
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------------------ host

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda), resolved
// once per process.
inline int encode_fn(EncodeTiledFn *out) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (fn == nullptr)
    return set_error(TROPNN_B200_ERR_DEVICE, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(err));
  *out = fn;
  return TROPNN_B200_OK;
}

// 2-D K-major tensor map over a row-major [outer, inner] 16-bit matrix, boxes of
// 64 x box_rows elements with the 128-byte swizzle; out-of-range elements read as zero.
inline int make_map_k64(CUtensorMap *map, const void *ptr, CUtensorMapDataType dt, int64_t inner, int64_t outer,
                        int box_rows) {
  EncodeTiledFn fn = nullptr;
  TB_CHECK(encode_fn(&fn));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
  const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TROPNN_B200_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return TROPNN_B200_OK;
}

// 2-D tensor map over a row-major f32 [outer, inner] matrix for 32 x 32 TMA stores
// staged in shared memory with the 128-byte swizzle (one 128-byte row per box row).
inline int make_map_f32_store32(CUtensorMap *map, void *ptr, int64_t inner, int64_t outer) {
  EncodeTiledFn fn = nullptr;
  TB_CHECK(encode_fn(&fn));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 4};
  const cuuint32_t box[2] = {32u, 32u};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TROPNN_B200_ERR_LAUNCH, "cuTensorMapEncodeTiled (store) failed (%d)", int(r));
  return TROPNN_B200_OK;
}

// 2-D K-major tensor map over a row-major f32 [outer, inner] matrix: boxes of 32 x box_rows
// elements (one 128-byte row each) with the 128-byte swizzle; out-of-range elements read as zero.
inline int make_map_f32_k32(CUtensorMap *map, const void *ptr, int64_t inner, int64_t outer, int box_rows) {
  EncodeTiledFn fn = nullptr;
  TB_CHECK(encode_fn(&fn));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 4};
  const cuuint32_t box[2] = {32u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TROPNN_B200_ERR_LAUNCH, "cuTensorMapEncodeTiled (f32 K) failed (%d)", int(r));
  return TROPNN_B200_OK;
}

// 3-D MN-major view of a row-major f32 [k_rows, cols] matrix (cols a multiple of 32): element
// (x, k, s) = m[k, 32 s + x]. A box {32, box_k, box_strips} lands as box_strips strips of
// box_k 128-byte rows (strip stride box_k * 128 bytes) in the 128-byte swizzle with 32-byte
// atoms, the MN-major tf32 UMMA operand layout (umma_desc_mn_tf32); out-of-range elements read
// as zero.
inline int make_map_f32_mn(CUtensorMap *map, const void *ptr, int64_t cols, int64_t k_rows, int box_k, int box_strips) {
  EncodeTiledFn fn = nullptr;
  TB_CHECK(encode_fn(&fn));
  const cuuint64_t dims[3] = {32u, static_cast<cuuint64_t>(k_rows), static_cast<cuuint64_t>(cols / 32)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 4, 128u};
  const cuuint32_t box[3] = {32u, static_cast<cuuint32_t>(box_k), static_cast<cuuint32_t>(box_strips)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TROPNN_B200_ERR_LAUNCH, "cuTensorMapEncodeTiled (f32 MN) failed (%d)", int(r));
  return TROPNN_B200_OK;
}

inline int sm_count(int *out) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    return set_error(TROPNN_B200_ERR_DEVICE, "cannot read the SM count");
  *out = sms;
  return TROPNN_B200_OK;
}

}  // namespace sm100
}  // namespace tropnn_b200
