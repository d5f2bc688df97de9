// TropLinear route scores on the sm_100a tensor cores: tcgen05.mma (kind::f16, f32
// accumulation in TMEM) fed by TMA, with the per-head top-2 fused into the epilogue, so
// the [rows, heads*cells] score matrix never reaches HBM.
//
// Reference behaviour (paths inside the tropnn package): scores = einsum(z, W) + b
// (backend.py:45-46), top-2 and margin (routing.py:7-10), packed route indices
// (routing.py:18-31). This is the path for half-precision parameters, where z and W are
// exactly representable in the MMA's f16/bf16 operands (z is rounded to the parameter
// dtype by the projection, tropical.py:99) and each product is exact in f32.
//
// Work unit = (128-row block of z, 256-column score tile of 256/cells heads). N=256 MMAs
// keep the tensor pipe at its rate with the weight tiles streaming in by TMA (N=128 MMAs
// fed the same way ran at ~60% of it). The grid is persistent, one CTA per SM, each CTA
// running a contiguous range of the row-major unit sequence, so the load is balanced to
// within one unit and consecutive units share their z block. CTA = 2 + 16 warps:
//   warp 0      TMA producer: the z block (resident, K-major, 128B swizzle; reloaded
//               when the unit sequence enters the next row block, once the MMAs on the
//               old block are done), then the router-weight tile of every (unit,
//               64-wide k block) through a 3-8 stage ring of 32 KB stages.
//   warp 1      allocates all 512 TMEM columns (two 256-column f32 accumulators); lane
//               0 issues the MMAs (M=128, N=256, K=16 each) and commits them to mbarriers.
//   warps 2-17  epilogue: each thread owns one accumulator row (TMEM lane) and 64 of the
//               unit's columns; per 32-column chunk it reads them with one tcgen05.ld,
//               adds the bias, takes the top-2 of every head, and at the end of the unit
//               writes winner (u8) and, when asked, runner (u8), margin (f32) and the
//               int64 winner.
// Every mbarrier wait gives up after ~1 s (clock64-independent %globaltimer), sets the
// library's device error word, lets the other roles exit, drains the copies and MMAs it
// issued (bounded again) and frees TMEM, so a protocol error cannot hang the GPU.
// Every TMA load is a plain per-CTA load of this GPU's own memory (no cluster-wide
// delivery, no peer memory), so the kernel is safe in multi-GPU processes.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;               // rows per unit (MMA M, TMEM lanes)
constexpr int kBN = 256;               // score columns per unit (MMA N)
constexpr int kBK = 64;                // k-block width: 64 f16 = one 128-byte swizzle row
constexpr int kMaxStages = 8;          // router-weight ring depth (as shared memory allows)
constexpr int kMinStages = 3;
constexpr int kTileBytesA = kBM * 128;  // one k block of the z block
constexpr int kTileBytesB = kBN * 128;  // one k block of a weight tile
constexpr int kBoxRows = 128;           // weight rows per TMA copy (two per stage)
#ifndef TROPNN_B200_SCORE_EPILOGUE_WARPS
#define TROPNN_B200_SCORE_EPILOGUE_WARPS 16
#endif
constexpr int kEpiWarps = TROPNN_B200_SCORE_EPILOGUE_WARPS;  // 8 or 16
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kEpiCols = kBN * 4 / kEpiWarps;  // accumulator columns per epilogue warp
constexpr int kTmemCols = 2 * kBN;             // double-buffered accumulator: all 512 columns
constexpr int kMaxKBlocks = 8;                 // code_dim <= 512
constexpr size_t kSmemLimit = 227 * 1024;
constexpr uint32_t kSleepHintNs = 1000000u;  // mbarrier suspend-time hint of whole-warp waits

// Library-wide device error word: nonzero after a bounded wait gave up.
__device__ int g_score_error = 0;

struct Barriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t a_full;
  uint64_t a_empty;
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int epi_go[2];
};

// Bounded mbarrier wait bound to this CTA's abort flag and the kernel's error word.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, Barriers *bs) {
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_score_error);
}

// Named barrier 1 over the epilogue warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void epilogue_sync() { named_sync(1, kEpiWarps * 32); }

__host__ __device__ constexpr int score_store_heads(int K) { return kEpiCols / K <= 4 ? kEpiCols / K : 32 / K; }

// Score with its kIdxBits lowest bits replaced by a cell code.
template <uint32_t kMask>
__device__ __forceinline__ float packed_key(float score, uint32_t code) {
  return __uint_as_float((__float_as_uint(score) & ~kMask) | code);
}

// Three-input max.f32 (PTX ISA 8.8, sm_100): one instruction instead of two.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 32 bias values from `c` on (f32, so the epilogue converts nothing; every lane reads the
// same addresses), zero past `hk`.
__device__ __forceinline__ void load_bias32(const float *__restrict__ bias, int64_t c, int64_t hk, float (&bv)[32]) {
  const float *bp = bias + c;
  if (c + 32 <= hk) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(bp + i));
      bv[i] = q.x;
      bv[i + 1] = q.y;
      bv[i + 2] = q.z;
      bv[i + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) bv[i] = (c + i < hk) ? __ldg(bp + i) : 0.f;
  }
}

constexpr int kWriteRunner = 1;
constexpr int kWriteMargins = 2;

// N consecutive route bytes / margins of one row, as 4-byte / 16-byte stores when N allows
// (the caller guarantees the destination is N-element aligned).
template <int N>
__device__ __forceinline__ void store_run(uint8_t *dst, const uint8_t (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      *reinterpret_cast<uint32_t *>(dst + i) =
          uint32_t(v[i]) | (uint32_t(v[i + 1]) << 8) | (uint32_t(v[i + 2]) << 16) | (uint32_t(v[i + 3]) << 24);
  } else if constexpr (N == 2) {
    *reinterpret_cast<uint16_t *>(dst) = static_cast<uint16_t>(uint32_t(v[0]) | (uint32_t(v[1]) << 8));
  } else {
    dst[0] = v[0];
  }
}

template <int N>
__device__ __forceinline__ void store_run(float *dst, const float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else if constexpr (N == 2) {
    *reinterpret_cast<float2 *>(dst) = make_float2(v[0], v[1]);
  } else {
    dst[0] = v[0];
  }
}

// The epilogue adds the f32 bias to each score (its 32 values per chunk loaded while the
// TMEM read is in flight). Folding the bias into the MMA as one more k step against a
// "ones" block measured 7 % slower at 65536 rows and no faster at 16384: that step streams
// one more 32 KB ring stage per unit beside the four weight k blocks.
template <typename PT, int K>
__global__ void __launch_bounds__(kThreads, 1) trop_score_top2_kernel(
    const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_w,
    const float *__restrict__ bias, int64_t rows, int H, int kblocks,
    int stages, int tiles_total, int64_t units, int flags, bool vec_stores, int64_t *__restrict__ winner_i64,
    uint8_t *__restrict__ winner, uint8_t *__restrict__ runner, float *__restrict__ margins) {
  static_assert(32 % K == 0 && K >= 2, "cells must divide 32");
  static_assert(kEpiCols % 32 == 0, "an epilogue warp reads whole 32-column chunks");
  constexpr int kHeadsPerGroup = kEpiCols / K;  // heads in one epilogue warp's columns
  constexpr int kHeadsPerChunk = 32 / K;
  // Heads whose routes are kept in registers before one store: the warp's whole group
  // for 16 and 32 cells, one chunk's for fewer cells (whose groups hold many heads).
  constexpr int kStoreHeads = score_store_heads(K);
  constexpr int kHeadsPerTile = kBN / K;
  constexpr int kIdxBits = K <= 2 ? 1 : K <= 4 ? 2 : K <= 8 ? 3 : K <= 16 ? 4 : 5;
  constexpr uint32_t kIdxMask = (1u << kIdxBits) - 1u;
  constexpr uint32_t kIdesc = umma_idesc_f16(sizeof(PT) == 2 && !std::is_same<PT, __half>::value ? 1 : 0, kBM, kBN);

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *a_smem = smem;                               // kblocks x [128 rows x 128 B]
  uint8_t *b_smem = a_smem + kblocks * kTileBytesA;     // stages x [256 rows x 128 B]
  Barriers *bs = reinterpret_cast<Barriers *>(b_smem + stages * kTileBytesB);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // This CTA's contiguous range of the unit sequence u = row_block * tiles_total + tile.
  const int64_t u_begin = units * blockIdx.x / gridDim.x;
  const int64_t u_end = units * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bs->full[s], 1);
      mbar_init(&bs->empty[s], 1);
    }
    mbar_init(&bs->a_full, 1);
    mbar_init(&bs->a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bs->tmem_full[b], 1);
      mbar_init(&bs->tmem_empty[b], kEpiWarps);
    }
    mbar_init(&bs->mma_done, 1);
    bs->abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(&bs->tmem_base, kTmemCols);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = bs->tmem_base;
  const int ksteps = kblocks;  // ring stages per unit

  if (warp == 0) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- TMA producer ----------------
      prefetch_map(&map_z);
      prefetch_map(&map_w);
      uint32_t issued[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) issued[s] = 0;
      bool ok = true;
      int it = 0, a_loads = 0;
      int64_t cur_rb = -1;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        const int64_t rb = u / tiles_total;
        const int tile = static_cast<int>(u - rb * tiles_total);
        if (rb != cur_rb) {
          // z block of the next row block, once the MMAs have released the previous one.
          if (a_loads > 0 && !mbar_wait(&bs->a_empty, uint32_t(a_loads - 1) & 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->a_full, uint32_t(kblocks) * kTileBytesA);
          for (int kb = 0; kb < kblocks; ++kb)
            tma_load_2d(a_smem + kb * kTileBytesA, &map_z, &bs->a_full, kb * kBK, static_cast<int>(rb * kBM));
          ++a_loads;
          cur_rb = rb;
        }
        for (int kb = 0; kb < ksteps; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t phase = uint32_t(it / stages) & 1u;
          if (!mbar_wait(&bs->empty[s], phase ^ 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->full[s], kTileBytesB);
          for (int q = 0; q < kBN / kBoxRows; ++q)
            tma_load_2d(b_smem + s * kTileBytesB + q * kBoxRows * 128, &map_w, &bs->full[s], kb * kBK,
                        tile * kBN + q * kBoxRows);
          issued[s] = uint32_t(it / stages) + 1;
        }
      }
      // Every copy this thread issued must land before the CTA may exit. A z load is only
      // issued after the MMAs consumed the previous one, so only the last can be pending.
      if (a_loads > 0) mbar_drain(&bs->a_full, uint32_t(a_loads - 1) & 1u);
      for (int s = 0; s < stages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- MMA issuer ----------------
      bool ok = true;
      int it = 0, a_uses = 0;
      int64_t cur_rb = -1;
      uint32_t t = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u, ++t) {
        const int64_t rb = u / tiles_total;
        if (rb != cur_rb) {
          // The previous z block is free once every MMA issued so far has completed.
          if (a_uses > 0) umma_commit(&bs->a_empty);
          if (!mbar_wait(&bs->a_full, uint32_t(a_uses) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          ++a_uses;
          cur_rb = rb;
        }
        const int b = t & 1;
        const uint32_t use = t >> 1;
        if (!mbar_wait(&bs->tmem_empty[b], (use & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * kBN);
        for (int kb = 0; kb < ksteps; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t phase = uint32_t(it / stages) & 1u;
          if (!mbar_wait(&bs->full[s], phase, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t b_base = smem_addr(b_smem + s * kTileBytesB);
          const uint32_t a_base = smem_addr(a_smem + kb * kTileBytesA);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d_tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), kIdesc,
                     (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&bs->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bs->tmem_full[b]);
      }
      // All MMAs issued by this thread must finish before TMEM is freed.
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int group = (warp - 2) >> 2;  // which kEpiCols columns of the tile
    const int r = quarter * 32 + lane;  // accumulator row
    const int64_t hk = int64_t(H) * K;
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      const int64_t rb = u / tiles_total;
      const int tile = static_cast<int>(u - rb * tiles_total);
      const int b = t & 1;
      const uint32_t use = t >> 1;
      const int h0 = tile * kHeadsPerTile + group * kHeadsPerGroup;
      const int64_t c0 = int64_t(tile) * kBN + group * kEpiCols;
      const int64_t row = rb * kBM + r;
      // Lane 0 of every epilogue warp waits for the accumulator with the mbarrier suspend
      // hint (sleeping between polls, so that 16 waiting warps take no issue slots from the
      // TMA and MMA threads) and the warp follows its verdict, converged, so the .sync.aligned
      // TMEM loads below run converged; warps start as soon as the accumulator is ready.
      int go = 1;
      if (lane == 0) go = mbar_wait_sleep(&bs->tmem_full[b], use & 1u, &bs->abort, &g_score_error, kSleepHintNs) ? 1 : 0;
      __syncwarp();
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) break;
      tmem_fence_after();
      uint8_t wv[kStoreHeads], rv[kStoreHeads];
      float mv[kStoreHeads];
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * kBN + group * kEpiCols);
#pragma unroll
      for (int c = 0; c < kEpiCols; c += 32) {
        float v[32], bv[32];
        tmem_ld32(taddr + uint32_t(c), v);
        load_bias32(bias, c0 + c, hk, bv);  // in flight together with the TMEM read
        tmem_wait_ld();
        reg_fence(v);
        if (c + 32 == kEpiCols) {
          // All of this warp's columns are in registers: the accumulator may be reused.
          // One arrive per warp (512 per-thread arrives on one mbarrier per unit slowed
          // the whole pipeline).
          tmem_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
        }
        // Top-2 per head on index-packed keys: the cell index K-1-k replaces the kIdxBits
        // lowest mantissa bits of each score, which makes the K keys of a head distinct and
        // keeps their order wherever the scores differ by more than 2^kIdxBits ulp (~2^-19
        // relative for 16 cells, far inside the 1e-4 relative parity gate). Scores equal
        // after packing go to the lower cell when positive, the higher when negative. The
        // best two are found with K + 3 (K/2 - 1) min/max for K keys, three-input max.f32
        // (sm_100) included. The margin is the difference of the two packed keys.
#pragma unroll
        for (int hh = 0; hh < kHeadsPerChunk; ++hh) {
          // (max, min) of every key pair, then a merge tree of best-two pairs: ILP of
          // K/2 at the leaves, 1 + log2(K/2) dependent levels.
          float hi[K / 2], lo[K / 2];
#pragma unroll
          for (int p = 0; p < K / 2; ++p) {
            const int k = 2 * p;
            const float sx = __fadd_rn(v[hh * K + k], bv[hh * K + k]);
            const float sy = __fadd_rn(v[hh * K + k + 1], bv[hh * K + k + 1]);
            const float x = packed_key<kIdxMask>(sx, uint32_t(K - 1 - k));
            const float y = packed_key<kIdxMask>(sy, uint32_t(K - 2 - k));
            hi[p] = fmaxf(x, y);
            lo[p] = fminf(x, y);
          }
#pragma unroll
          for (int w = 1; w < K / 2; w *= 2) {
#pragma unroll
            for (int p = 0; p + w < K / 2; p += 2 * w) {
              const float a1 = hi[p], b1 = hi[p + w];
              lo[p] = fmax3(fminf(a1, b1), lo[p], lo[p + w]);
              hi[p] = fmaxf(a1, b1);
            }
          }
          const float k1 = hi[0], k2 = lo[0];
          const uint32_t l1 = __float_as_uint(k1) & kIdxMask, l2 = __float_as_uint(k2) & kIdxMask;
          const int g = (c / K + hh) % kStoreHeads;
          wv[g] = static_cast<uint8_t>(K - 1 - l1);
          rv[g] = static_cast<uint8_t>(K - 1 - l2);
          mv[g] = __fsub_rn(k1, k2);
        }
        if ((c / K + kHeadsPerChunk) % kStoreHeads == 0 && row < rows) {
          // kStoreHeads consecutive heads of one row: vector stores where aligned.
          const int hs = h0 + c / K + kHeadsPerChunk - kStoreHeads;
          const int64_t o = row * H + hs;
          if (vec_stores && hs + kStoreHeads <= H) {
            store_run<kStoreHeads>(winner + o, wv);
            if (flags & kWriteRunner) store_run<kStoreHeads>(runner + o, rv);
            if (flags & kWriteMargins) store_run<kStoreHeads>(margins + o, mv);
          } else {
#pragma unroll
            for (int hh = 0; hh < kStoreHeads; ++hh) {
              if (hs + hh < H) {
                winner[o + hh] = wv[hh];
                if (flags & kWriteRunner) runner[o + hh] = rv[hh];
                if (flags & kWriteMargins) margins[o + hh] = mv[hh];
              }
            }
          }
          if (winner_i64 != nullptr) {
#pragma unroll
            for (int hh = 0; hh < kStoreHeads; ++hh)
              if (hs + hh < H) winner_i64[o + hh] = wv[hh];
          }
        }
      }
    }
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// --------------------------------------------------------------------------- host side

size_t score_smem_bytes(int kblocks, int stages) {
  return 1024 + size_t(kblocks) * kTileBytesA + size_t(stages) * kTileBytesB + sizeof(Barriers);
}

// Weight-ring depth: the shared memory left after the resident z block, up to kMaxStages; 0
// when fewer than kMinStages fit.
int score_stages(int kblocks) {
  const size_t fixed = score_smem_bytes(kblocks, 0);
  if (fixed >= kSmemLimit) return 0;
  const int stages = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / kTileBytesB));
  return stages >= kMinStages ? stages : 0;
}

template <typename PT, int K>
int launch_score(const void *z, int64_t rows, int D, const void *W, const void *bias, int H, int64_t *w64,
                 uint8_t *win, uint8_t *run, float *m, cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int kblocks = (D + kBK - 1) / kBK;
  const int64_t hk = int64_t(H) * K;
  const int stages = score_stages(kblocks);
  TB_REQUIRE(stages > 0, TROPNN_B200_ERR_INVALID, "trop_score_sm100: code_dim=%d does not fit shared memory", D);
  const size_t smem = score_smem_bytes(kblocks, stages);
  CUtensorMap map_z, map_w;
  TB_CHECK(make_map_k64(&map_z, z, dt, D, rows, kBM));
  TB_CHECK(make_map_k64(&map_w, W, dt, D, hk, kBoxRows));
  const int tiles_total = static_cast<int>(ceil_div(hk, kBN));
  const int64_t units = ceil_div(rows, int64_t(kBM)) * tiles_total;
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const int flags = (run != nullptr ? kWriteRunner : 0) | (m != nullptr ? kWriteMargins : 0);
  // Vector stores need every row's run of heads to start on a multiple of its length.
  constexpr int kRun = score_store_heads(K);
  auto al16 = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool vec_stores = (H % kRun == 0) && al16(win) && al16(run) && al16(m);
  auto kernel = trop_score_top2_kernel<PT, K>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_score_sm100"));
  // Persistent grid: one CTA per SM (shared memory and TMEM admit no second), units
  // split evenly.
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(units, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_z, map_w, static_cast<const float *>(bias), rows, H, kblocks, stages,
                                           tiles_total, units, flags, vec_stores, w64, win, run, m);
  return check_launch("trop_score_sm100");
}

template <typename PT>
int dispatch_cells(int K, const void *z, int64_t rows, int D, const void *W, const void *bias, int H, int64_t *w64,
                   uint8_t *win, uint8_t *run, float *m, cudaStream_t stream) {
  switch (K) {
    case 2: return launch_score<PT, 2>(z, rows, D, W, bias, H, w64, win, run, m, stream);
    case 4: return launch_score<PT, 4>(z, rows, D, W, bias, H, w64, win, run, m, stream);
    case 8: return launch_score<PT, 8>(z, rows, D, W, bias, H, w64, win, run, m, stream);
    case 16: return launch_score<PT, 16>(z, rows, D, W, bias, H, w64, win, run, m, stream);
    default: return launch_score<PT, 32>(z, rows, D, W, bias, H, w64, win, run, m, stream);
  }
}

// ---------------------------------------------------------------------------------------
// f32 parameters: the same route on kind::tf32 with split operands (3xTF32).
//
// The reference's f32 scores (backend.py:45-46) have no f32 MMA to run on; with x = big +
// small (big = tf32(x), small = tf32(x - big)) the products big*big' + big*small' +
// small*big' keep about 2^-22 relative accuracy per product (3xTF32), far inside the 1e-4
// relative margin gate that decides which routes are pinned. big*big' accumulates in one TMEM
// accumulator and the cross terms in another (the accumulator's per-addition truncation then
// stays at the level of the dominant sum), added in the epilogue before the top-2. z and the
// router weights arrive split (tf32_split into the caller's workspace): the z block (big and
// small, K-major f32, code_dim <= 128) is resident, the weight tiles stream through a ring of
// 32 KB stages (big and small 128 x 32 f32 each). Unit = 128 rows x 128 score columns; two
// units in flight use all 512 TMEM columns. Roles as the f16 kernel: warp 0 TMA, warp 1
// TMEM + MMA (3 MMAs per 8-wide k step), warps 2-17 epilogue (32 columns each: one
// tcgen05.ld of each accumulator, bias, top-2 per head).
constexpr int kBNt = 128;                  // score columns per tf32 unit
constexpr int kBKt = 32;                   // f32 per 128-byte swizzled row
constexpr int kTileT = kBM * 128;          // one 128 x 32 f32 tile (16 KB)
constexpr int kStageBytesT = 2 * kTileT;   // big + small weight tile
constexpr int kMaxKBlocksT = 4;            // code_dim <= 128
constexpr int kEpiColsT = kBNt * 4 / kEpiWarps;

static_assert(kEpiColsT == 32, "the tf32 epilogue reads one 32-column chunk per warp");

template <int K>
__global__ void __launch_bounds__(kThreads, 1) trop_score_tf32_kernel(
    const __grid_constant__ CUtensorMap map_zb, const __grid_constant__ CUtensorMap map_zs,
    const __grid_constant__ CUtensorMap map_wb, const __grid_constant__ CUtensorMap map_ws,
    const float *__restrict__ bias, int64_t rows, int H, int kblocks, int stages, int tiles_total, int64_t units,
    int flags, bool vec_stores, int64_t *__restrict__ winner_i64, uint8_t *__restrict__ winner,
    uint8_t *__restrict__ runner, float *__restrict__ margins) {
  static_assert(32 % K == 0 && K >= 2, "cells must divide 32");
  constexpr int kHeadsPerChunk = 32 / K;
  constexpr int kHeadsPerTile = kBNt / K;
  constexpr int kIdxBits = K <= 2 ? 1 : K <= 4 ? 2 : K <= 8 ? 3 : K <= 16 ? 4 : 5;
  constexpr uint32_t kIdxMask = (1u << kIdxBits) - 1u;
  constexpr uint32_t kIdesc = umma_idesc_tf32(false, false, kBM, kBNt);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *a_smem = smem;                                // kblocks x [z big | z small] (32 KB each)
  uint8_t *b_smem = a_smem + kblocks * 2 * kTileT;       // stages x [w big | w small]
  Barriers *bs = reinterpret_cast<Barriers *>(b_smem + stages * kStageBytesT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t u_begin = units * blockIdx.x / gridDim.x;
  const int64_t u_end = units * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bs->full[s], 1);
      mbar_init(&bs->empty[s], 1);
    }
    mbar_init(&bs->a_full, 1);
    mbar_init(&bs->a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bs->tmem_full[b], 1);
      mbar_init(&bs->tmem_empty[b], kEpiWarps);
    }
    mbar_init(&bs->mma_done, 1);
    bs->abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(&bs->tmem_base, kTmemCols);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = bs->tmem_base;

  if (warp == 0) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- TMA producer ----------------
      prefetch_map(&map_zb);
      prefetch_map(&map_zs);
      prefetch_map(&map_wb);
      prefetch_map(&map_ws);
      uint32_t issued[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) issued[s] = 0;
      bool ok = true;
      int it = 0, a_loads = 0;
      int64_t cur_rb = -1;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        const int64_t rb = u / tiles_total;
        const int tile = static_cast<int>(u - rb * tiles_total);
        if (rb != cur_rb) {
          if (a_loads > 0 && !mbar_wait(&bs->a_empty, uint32_t(a_loads - 1) & 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->a_full, uint32_t(kblocks) * 2 * kTileT);
          for (int kb = 0; kb < kblocks; ++kb) {
            tma_load_2d(a_smem + kb * 2 * kTileT, &map_zb, &bs->a_full, kb * kBKt, static_cast<int>(rb * kBM));
            tma_load_2d(a_smem + kb * 2 * kTileT + kTileT, &map_zs, &bs->a_full, kb * kBKt, static_cast<int>(rb * kBM));
          }
          ++a_loads;
          cur_rb = rb;
        }
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          if (!mbar_wait(&bs->empty[s], (uint32_t(it / stages) & 1u) ^ 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->full[s], kStageBytesT);
          tma_load_2d(b_smem + s * kStageBytesT, &map_wb, &bs->full[s], kb * kBKt, tile * kBNt);
          tma_load_2d(b_smem + s * kStageBytesT + kTileT, &map_ws, &bs->full[s], kb * kBKt, tile * kBNt);
          issued[s] = uint32_t(it / stages) + 1;
        }
      }
      if (a_loads > 0) mbar_drain(&bs->a_full, uint32_t(a_loads - 1) & 1u);
      for (int s = 0; s < stages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- MMA issuer ----------------
      bool ok = true;
      int it = 0, a_uses = 0;
      int64_t cur_rb = -1;
      uint32_t t = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u, ++t) {
        const int64_t rb = u / tiles_total;
        if (rb != cur_rb) {
          if (a_uses > 0) umma_commit(&bs->a_empty);
          if (!mbar_wait(&bs->a_full, uint32_t(a_uses) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          ++a_uses;
          cur_rb = rb;
        }
        const int b = t & 1;
        if (!mbar_wait(&bs->tmem_empty[b], ((t >> 1) & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_big = tmem_base + uint32_t(b * 2 * kBNt);
        const uint32_t d_cross = d_big + kBNt;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          if (!mbar_wait(&bs->full[s], uint32_t(it / stages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t za = smem_addr(a_smem + kb * 2 * kTileT), zs = za + kTileT;
          const uint32_t wa = smem_addr(b_smem + s * kStageBytesT), ws = wa + kTileT;
#pragma unroll
          for (int kk = 0; kk < kBKt / 8; ++kk) {
            const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
            const uint64_t dz = umma_desc_sw128(za + kk * 32), dw = umma_desc_sw128(wa + kk * 32);
            umma_tf32(d_big, dz, dw, kIdesc, acc);
            umma_tf32(d_cross, dz, umma_desc_sw128(ws + kk * 32), kIdesc, acc);
            umma_tf32(d_cross, umma_desc_sw128(zs + kk * 32), dw, kIdesc, 1u);
          }
          umma_commit(&bs->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bs->tmem_full[b]);
      }
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const int group = (warp - 2) >> 2;  // which 32 columns of the unit
    const int r = quarter * 32 + lane;
    const int64_t hk = int64_t(H) * K;
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      const int64_t rb = u / tiles_total;
      const int tile = static_cast<int>(u - rb * tiles_total);
      const int b = t & 1;
      const int64_t row = rb * kBM + r;
      const int64_t c0 = int64_t(tile) * kBNt + group * kEpiColsT;
      int go = 1;
      if (lane == 0) go = mbar_wait_sleep(&bs->tmem_full[b], (t >> 1) & 1u, &bs->abort, &g_score_error, kSleepHintNs) ? 1 : 0;
      __syncwarp();
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) break;
      tmem_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * 2 * kBNt + group * kEpiColsT);
      float v[32];
      {
        float x[32];
        tmem_ld32(taddr, v);
        tmem_ld32(taddr + kBNt, x);
        tmem_wait_ld();
        reg_fence(v);
        reg_fence(x);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], x[j]);  // big products + cross terms
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
      {
        float bv[32];
        load_bias32(bias, c0, hk, bv);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bv[j]);
      }
      uint8_t wv[kHeadsPerChunk], rv[kHeadsPerChunk];
      float mv[kHeadsPerChunk];
#pragma unroll
      for (int hh = 0; hh < kHeadsPerChunk; ++hh) {
        // Top-2 on index-packed keys, as the f16 kernel (the cell index K-1-k in the lowest
        // kIdxBits mantissa bits).
        float hi[K / 2], lo[K / 2];
#pragma unroll
        for (int p = 0; p < K / 2; ++p) {
          const int k = 2 * p;
          const float a = packed_key<kIdxMask>(v[hh * K + k], uint32_t(K - 1 - k));
          const float c = packed_key<kIdxMask>(v[hh * K + k + 1], uint32_t(K - 2 - k));
          hi[p] = fmaxf(a, c);
          lo[p] = fminf(a, c);
        }
#pragma unroll
        for (int w = 1; w < K / 2; w *= 2) {
#pragma unroll
          for (int p = 0; p + w < K / 2; p += 2 * w) {
            const float a1 = hi[p], b1 = hi[p + w];
            lo[p] = fmax3(fminf(a1, b1), lo[p], lo[p + w]);
            hi[p] = fmaxf(a1, b1);
          }
        }
        const float k1 = hi[0], k2 = lo[0];
        wv[hh] = static_cast<uint8_t>(K - 1 - (__float_as_uint(k1) & kIdxMask));
        rv[hh] = static_cast<uint8_t>(K - 1 - (__float_as_uint(k2) & kIdxMask));
        mv[hh] = __fsub_rn(k1, k2);
      }
      if (row < rows) {
        const int hs = tile * kHeadsPerTile + group * kHeadsPerChunk;
        const int64_t o = row * H + hs;
        if (vec_stores && hs + kHeadsPerChunk <= H) {
          store_run<kHeadsPerChunk>(winner + o, wv);
          if (flags & kWriteRunner) store_run<kHeadsPerChunk>(runner + o, rv);
          if (flags & kWriteMargins) store_run<kHeadsPerChunk>(margins + o, mv);
        } else {
#pragma unroll
          for (int hh = 0; hh < kHeadsPerChunk; ++hh) {
            if (hs + hh < H) {
              winner[o + hh] = wv[hh];
              if (flags & kWriteRunner) runner[o + hh] = rv[hh];
              if (flags & kWriteMargins) margins[o + hh] = mv[hh];
            }
          }
        }
        if (winner_i64 != nullptr) {
#pragma unroll
          for (int hh = 0; hh < kHeadsPerChunk; ++hh)
            if (hs + hh < H) winner_i64[o + hh] = wv[hh];
        }
      }
    }
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

size_t score_tf32_smem_bytes(int kblocks, int stages) {
  return 1024 + size_t(kblocks) * 2 * kTileT + size_t(stages) * kStageBytesT + sizeof(Barriers);
}

int score_tf32_stages(int kblocks) {
  const size_t fixed = score_tf32_smem_bytes(kblocks, 0);
  if (fixed >= kSmemLimit) return 0;
  const int stages = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / kStageBytesT));
  return stages >= kMinStages ? stages : 0;
}

template <int K>
int launch_score_tf32(const float *zb, const float *zs, int64_t rows, int D, const float *wb, const float *wsm,
                      const float *bias, int H, int64_t *w64, uint8_t *win, uint8_t *run, float *m,
                      cudaStream_t stream) {
  const int kblocks = static_cast<int>(ceil_div(D, kBKt));
  const int stages = score_tf32_stages(kblocks);
  TB_REQUIRE(stages > 0, TROPNN_B200_ERR_INVALID, "trop_score_tf32: code_dim=%d does not fit shared memory", D);
  CUtensorMap map_zb, map_zs, map_wb, map_ws;
  TB_CHECK(make_map_f32_k32(&map_zb, zb, D, rows, kBM));
  TB_CHECK(make_map_f32_k32(&map_zs, zs, D, rows, kBM));
  TB_CHECK(make_map_f32_k32(&map_wb, wb, D, int64_t(H) * K, kBNt));
  TB_CHECK(make_map_f32_k32(&map_ws, wsm, D, int64_t(H) * K, kBNt));
  const int tiles_total = static_cast<int>(ceil_div(int64_t(H) * K, kBNt));
  const int64_t units = ceil_div(rows, int64_t(kBM)) * tiles_total;
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const int flags = (run != nullptr ? kWriteRunner : 0) | (m != nullptr ? kWriteMargins : 0);
  constexpr int kRun = 32 / K;
  auto al16 = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool vec_stores = (H % kRun == 0) && al16(win) && al16(run) && al16(m);
  const size_t smem = score_tf32_smem_bytes(kblocks, stages);
  auto kernel = trop_score_tf32_kernel<K>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_score_tf32"));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(units, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_zb, map_zs, map_wb, map_ws, bias, rows, H, kblocks, stages, tiles_total,
                                           units, flags, vec_stores, w64, win, run, m);
  return check_launch("trop_score_tf32");
}

}  // namespace

bool score_sm100_supported(int64_t D, int64_t K, int pt, int bias_dtype, const void *z, const void *W,
                           const void *bias) {
  const bool cells_ok = K == 2 || K == 4 || K == 8 || K == 16 || K == 32;
  const int64_t kblocks = (D + kBK - 1) / kBK;
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return (pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16) && bias_dtype == TROPNN_B200_F32 && cells_ok &&
         D % 8 == 0 && kblocks <= kMaxKBlocks && score_stages(static_cast<int>(kblocks)) > 0 && al16(z) &&
         al16(W) && al16(bias);
}

int trop_score_sm100_impl(const void *z, int64_t items, int64_t D, const void *W, const void *bias, int pt, int64_t H,
                          int64_t K, int64_t *w64, uint8_t *win, uint8_t *run, float *m, cudaStream_t stream) {
  TB_REQUIRE(score_sm100_supported(D, K, pt, TROPNN_B200_F32, z, W, bias), TROPNN_B200_ERR_INVALID,
             "trop_score_sm100: unsupported shape or alignment code_dim=%lld cells=%lld dtype=%s", (long long)D,
             (long long)K, dtype_name(pt));
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(z && W && bias && win, TROPNN_B200_ERR_INVALID, "trop_score_sm100: null pointer");
  // TMA row coordinates are 32-bit.
  TB_REQUIRE(items <= (int64_t(1) << 31) - 1024 && H * K <= (int64_t(1) << 31) - 1024, TROPNN_B200_ERR_INVALID,
             "trop_score_sm100: %lld rows x %lld score columns exceed the 32-bit tile coordinates",
             (long long)items, (long long)(H * K));
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H), Ki = static_cast<int>(K);
  if (pt == TROPNN_B200_F16) return dispatch_cells<__half>(Ki, z, items, Di, W, bias, Hi, w64, win, run, m, stream);
  return dispatch_cells<__nv_bfloat16>(Ki, z, items, Di, W, bias, Hi, w64, win, run, m, stream);
}


int tf32_split_impl(const float *x, int64_t count, float *big, float *small, cudaStream_t stream);

bool score_tf32_supported(int64_t D, int64_t K, int pt, int bias_dtype, const void *z, const void *W,
                          const void *bias) {
  const bool cells_ok = K == 2 || K == 4 || K == 8 || K == 16 || K == 32;
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return pt == TROPNN_B200_F32 && bias_dtype == TROPNN_B200_F32 && cells_ok && D % 4 == 0 && D >= 4 &&
         D <= kMaxKBlocksT * kBKt && score_tf32_stages(static_cast<int>(ceil_div(D, kBKt))) > 0 && al16(z) && al16(W) &&
         al16(bias);
}

size_t score_tf32_workspace(int64_t items, int64_t D, int64_t H, int64_t K) {
  return 2 * WorkspaceCarver::align(size_t(items) * D * sizeof(float)) +
         2 * WorkspaceCarver::align(size_t(H) * K * D * sizeof(float));
}

int trop_score_tf32_impl(const float *z, int64_t items, int64_t D, const float *W, const float *bias, int64_t H,
                         int64_t K, int64_t *w64, uint8_t *win, uint8_t *run, float *m, void *ws, size_t ws_bytes,
                         cudaStream_t stream) {
  TB_REQUIRE(score_tf32_supported(D, K, TROPNN_B200_F32, TROPNN_B200_F32, z, W, bias), TROPNN_B200_ERR_INVALID,
             "trop_score_tf32: unsupported shape or alignment code_dim=%lld cells=%lld", (long long)D, (long long)K);
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(items <= (int64_t(1) << 31) - 1024 && H * K <= (int64_t(1) << 31) - 1024, TROPNN_B200_ERR_INVALID,
             "trop_score_tf32: sizes exceed the 32-bit tile coordinates");
  WorkspaceCarver c(ws, ws_bytes);
  float *zb = c.take<float>(size_t(items) * D), *zs = c.take<float>(size_t(items) * D);
  float *wb = c.take<float>(size_t(H) * K * D), *wsm = c.take<float>(size_t(H) * K * D);
  TB_REQUIRE(zb && zs && wb && wsm, TROPNN_B200_ERR_WORKSPACE,
             "trop_score_tf32: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes,
             score_tf32_workspace(items, D, H, K));
  TB_CHECK(tf32_split_impl(z, items * D, zb, zs, stream));
  TB_CHECK(tf32_split_impl(W, H * K * D, wb, wsm, stream));
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H);
  switch (K) {
    case 2: return launch_score_tf32<2>(zb, zs, items, Di, wb, wsm, bias, Hi, w64, win, run, m, stream);
    case 4: return launch_score_tf32<4>(zb, zs, items, Di, wb, wsm, bias, Hi, w64, win, run, m, stream);
    case 8: return launch_score_tf32<8>(zb, zs, items, Di, wb, wsm, bias, Hi, w64, win, run, m, stream);
    case 16: return launch_score_tf32<16>(zb, zs, items, Di, wb, wsm, bias, Hi, w64, win, run, m, stream);
    default: return launch_score_tf32<32>(zb, zs, items, Di, wb, wsm, bias, Hi, w64, win, run, m, stream);
  }
}

int read_score_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_score_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_score_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200
