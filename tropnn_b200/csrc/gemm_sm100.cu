// Dense f32-output linear map on the sm_100a tensor cores:
//   out[m, n] = sum_s sum_k a[m, s*K + k] * w[n, k] + bias[n]      (f32 accumulation)
// with a and w in f16/bf16 and `slices` copies of the K-wide left operand side by side.
// With slices = 2 and a = [hi | lo], hi = half(x), lo = half(x - hi) (split_half), this
// is an f32 x half-precision-weight product accurate to ~2^-22 relative for f16: the
// output map of TropLinear (layers/tropical.py:140-146), whose reference computes an
// f32 GEMM with the half-precision weight upcast, runs on tcgen05 instead of f32 FMA.
//
// Work unit = (128-row block, 256-column output tile); persistent grid, one CTA per SM,
// each CTA running a contiguous range of the row-major unit sequence (consecutive units
// share their left block). CTA = 2 + 8 warps:
//   warp 0      TMA producer: the left block (all slices, resident, K-major, 128B swizzle;
//               reloaded when the unit sequence enters the next row block, once the MMAs
//               on the old one are done), then the weight k blocks (256 x 64) through a
//               ring; each weight k block serves every slice.
//   warp 1      allocates all 512 TMEM columns (two 256-column f32 accumulators); lane 0
//               issues the MMAs (M=128, N=256, K=16) and commits them to mbarriers.
//   warps 2-9   epilogue: each thread owns one accumulator row and 128 columns: adds the
//               bias; the warp stages 32 x 32 f32 tiles in shared memory and writes each
//               with one TMA store.
// Waits are bounded (sm100.cuh); one epilogue thread polls the accumulator barrier and
// the other epilogue warps wait on a named barrier.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tropnn_b200.h"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kMaxStages = 8;
constexpr int kMinStages = 2;
constexpr int kTileBytesA = kBM * 128;
constexpr int kTileBytesB = kBN * 128;
constexpr int kBoxRows = 128;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kEpiCols = kBN * 4 / kEpiWarps;  // 128
constexpr int kStageOutBytes = 32 * 128;       // one warp's 32 x 32 f32 store tile
// Shared memory of the epilogue's store staging: the f32 output map (K = 0) only; the
// route-margin gradient (K > 0) gives it to the weight ring (3 stages instead of 2 with a
// 128 KiB left block).
__host__ __device__ constexpr size_t out_stage_bytes(int K) { return K == 0 ? size_t(kEpiWarps) * kStageOutBytes : 0; }
constexpr int kTmemCols = 2 * kBN;
constexpr int kMaxABlocks = 8;                 // slices * K <= 512
constexpr size_t kSmemLimit = 227 * 1024;

__device__ int g_gemm_error = 0;

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

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Barriers *bs) {
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_gemm_error);
}

// Epilogue of the min-face backward's route-margin gradient (kernel mode GM): the GEMM
// computes <g_n, c_{h,k}> for every cell, the epilogue keeps the winner's and the
// runner-up's and forms gm[n,h] = code_scale (<g,c_r> - <g,c_w>) U'(m),
// U'(m) = -0.5 sign(m) / (1+|m|)^2 (layers/tropical_exact.py:204-237).
struct GmArgs {
  const uint8_t *winner;
  const uint8_t *runner;
  const float *margins;
  float *gm;
  int64_t rows;
  int heads;
  float code_scale;
  const uint32_t *absmax;  // the g split was scaled by pow2_grad_scale(*absmax) (NULL: not scaled)
  int vec;                 // routes / margins / gm rows allow the per-thread vector accesses below
};

// code_scale * U'(m), U'(m) = -0.5 sign(m) / (1+|m|)^2 (layers/tropical_exact.py:204-237).
__device__ __forceinline__ float margin_factor(float code_scale, float m) {
  const float den = __fadd_rn(1.f, fabsf(m));
  const float sgn = (m > 0.f) ? 1.f : ((m < 0.f) ? -1.f : 0.f);
  return __fmul_rn(code_scale, __fdiv_rn(__fmul_rn(-0.5f, sgn), __fmul_rn(den, den)));
}

// The kN consecutive bytes / floats of one row starting at `o` (a multiple of kN), by vector
// loads when `vec`, else element by element (entries at or past `valid` read as 0xFF / 0).
template <int kN>
__device__ __forceinline__ void load_bytes(const uint8_t *p, int64_t o, bool vec, int valid, uint8_t (&out)[kN]) {
  if (vec && valid >= kN) {
    if constexpr (kN == 16) {
      *reinterpret_cast<uint4 *>(out) = __ldg(reinterpret_cast<const uint4 *>(p + o));
    } else if constexpr (kN == 8) {
      *reinterpret_cast<uint2 *>(out) = __ldg(reinterpret_cast<const uint2 *>(p + o));
    } else {
      *reinterpret_cast<uint32_t *>(out) = __ldg(reinterpret_cast<const uint32_t *>(p + o));
    }
  } else {
#pragma unroll
    for (int i = 0; i < kN; ++i) out[i] = i < valid ? __ldg(p + o + i) : uint8_t(0xFF);
  }
}
template <int kN>
__device__ __forceinline__ void load_floats(const float *p, int64_t o, bool vec, int valid, float (&out)[kN]) {
#pragma unroll
  for (int i = 0; i < kN; i += 4) {
    if (vec && valid >= kN) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(p + o + i));
      out[i] = q.x, out[i + 1] = q.y, out[i + 2] = q.z, out[i + 3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) out[i + j] = i + j < valid ? __ldg(p + o + i + j) : 0.f;
    }
  }
}

template <typename PT, int K>  // K = 0: f32 output map; K = cells: route-margin gradient
__global__ void __launch_bounds__(kThreads, 1) linear_f32out_kernel(
    const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
    const __grid_constant__ CUtensorMap map_out, const float *__restrict__ bias, int out_features, int slices,
    int b_kblocks, int stages, int tiles_total, int64_t units, const GmArgs gmx) {
  constexpr uint32_t kIdesc =
      umma_idesc_f16(std::is_same<PT, __half>::value ? 0 : 1, kBM, kBN);
  const int a_blocks = slices * b_kblocks;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *a_smem = smem;                               // a_blocks x [128 rows x 128 B]
  uint8_t *b_smem = a_smem + a_blocks * kTileBytesA;    // stages x [256 rows x 128 B]
  uint8_t *o_smem = b_smem + stages * kTileBytesB;      // kEpiWarps x [32 rows x 128 B] (f32 output only)
  Barriers *bs = reinterpret_cast<Barriers *>(o_smem + out_stage_bytes(K));

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
      prefetch_map(&map_a);
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
          if (a_loads > 0 && !wait_bar(&bs->a_empty, uint32_t(a_loads - 1) & 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->a_full, uint32_t(a_blocks) * kTileBytesA);
          for (int kb = 0; kb < a_blocks; ++kb)
            tma_load_2d(a_smem + kb * kTileBytesA, &map_a, &bs->a_full, kb * kBK, static_cast<int>(rb * kBM));
          ++a_loads;
          cur_rb = rb;
        }
        for (int kb = 0; kb < b_kblocks; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t phase = uint32_t(it / stages) & 1u;
          if (!wait_bar(&bs->empty[s], phase ^ 1u, bs)) {
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
          if (!wait_bar(&bs->a_full, uint32_t(a_uses) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          ++a_uses;
          cur_rb = rb;
        }
        const int b = t & 1;
        const uint32_t use = t >> 1;
        if (!wait_bar(&bs->tmem_empty[b], (use & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * kBN);
        for (int kb = 0; kb < b_kblocks; ++kb, ++it) {
          const int s = it % stages;
          if (!wait_bar(&bs->full[s], uint32_t(it / stages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t b_base = smem_addr(b_smem + s * kTileBytesB);
          for (int sl = 0; sl < slices; ++sl) {
            const uint32_t a_base = smem_addr(a_smem + (sl * b_kblocks + kb) * kTileBytesA);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16(d_tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), kIdesc,
                       (kb | sl | kk) != 0 ? 1u : 0u);
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
    // Each warp owns 32 accumulator rows x 128 columns of a unit and writes them as four
    // 32 x 32 f32 tiles: registers -> its 4 KB shared tile (128-byte swizzle, so the 32
    // lanes' row writes hit distinct banks) -> one TMA store, which writes whole lines
    // (row-per-lane global stores ran at a third of HBM bandwidth).
    const int quarter = warp & 3;
    const int group = (warp - 2) >> 2;
    uint8_t *stage = o_smem + (warp - 2) * kStageOutBytes;
    // Route-margin gradient: undo the power-of-two scale of the g split (exact).
    const float gm_unscale = K > 0 ? pow2_inverse(grad_scale_of(gmx.absmax)) : 1.f;
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      const int64_t rb = u / tiles_total;
      const int tile = static_cast<int>(u - rb * tiles_total);
      const int b = t & 1;
      const uint32_t use = t >> 1;
      const int col0 = tile * kBN + group * kEpiCols;
      if constexpr (K >= 8) {
        // Route-margin gradient, kEpiCols / K heads of this thread's row per unit: their routes
        // and margin factors are loaded (vector loads) and computed before the accumulator is
        // ready, so the loads overlap the MMAs; gm leaves in one vector store per 4 heads.
        constexpr int kHpt = kEpiCols / K;
        const int64_t row = rb * kBM + quarter * 32 + lane;
        const int hb = col0 / K;
        const int valid = row < gmx.rows ? max(0, min(kHpt, gmx.heads - hb)) : 0;
        const int64_t o = row * gmx.heads + hb;
        uint8_t wq[kHpt], rq[kHpt];
        float fq[kHpt];
        load_bytes<kHpt>(gmx.winner, o, gmx.vec != 0, valid, wq);
        load_bytes<kHpt>(gmx.runner, o, gmx.vec != 0, valid, rq);
        load_floats<kHpt>(gmx.margins, o, gmx.vec != 0, valid, fq);
#pragma unroll
        for (int i = 0; i < kHpt; ++i) fq[i] = __fmul_rn(margin_factor(gmx.code_scale, fq[i]), gm_unscale);
        if (warp == 2 && lane == 0) bs->epi_go[b] = wait_bar(&bs->tmem_full[b], use & 1u, bs) ? 1 : 0;
        named_sync(1, kEpiWarps * 32);
        if (*reinterpret_cast<volatile int *>(&bs->epi_go[b]) == 0) break;
        __syncwarp();
        tmem_fence_after();
        const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * kBN + group * kEpiCols);
        float gq[kHpt];
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 32) {
          float v[32];
          tmem_ld32(taddr + uint32_t(c), v);
          tmem_wait_ld();
          reg_fence(v);
          if (c + 32 == kEpiCols) {
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
          }
#pragma unroll
          for (int hh = 0; hh < 32 / K; ++hh) {
            const int i = c / K + hh;
            // Bitwise pick (one cell matches): masks, not selects, so that the accumulator
            // values stay in registers.
            uint32_t bw = 0u, br = 0u;
#pragma unroll
            for (int k = 0; k < K; ++k) {
              const uint32_t x = __float_as_uint(v[hh * K + k]);
              bw |= x & (0u - uint32_t(wq[i] == uint32_t(k)));
              br |= x & (0u - uint32_t(rq[i] == uint32_t(k)));
            }
            gq[i] = __fmul_rn(__fsub_rn(__uint_as_float(br), __uint_as_float(bw)), fq[i]);
          }
        }
        if (valid == kHpt && gmx.vec != 0) {
#pragma unroll
          for (int i = 0; i < kHpt; i += 4)
            *reinterpret_cast<float4 *>(gmx.gm + o + i) = make_float4(gq[i], gq[i + 1], gq[i + 2], gq[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < kHpt; ++i)
            if (i < valid) gmx.gm[o + i] = gq[i];
        }
        continue;
      }
      // One thread polls; the verdict travels through a two-slot flag (slot t&1 is
      // rewritten two units later, after every epilogue warp has read it).
      if (warp == 2 && lane == 0) bs->epi_go[b] = wait_bar(&bs->tmem_full[b], use & 1u, bs) ? 1 : 0;
      named_sync(1, kEpiWarps * 32);
      if (*reinterpret_cast<volatile int *>(&bs->epi_go[b]) == 0) break;
      __syncwarp();
      tmem_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * kBN + group * kEpiCols);
#pragma unroll 1
      for (int c = 0; c < kEpiCols; c += 32) {
        float v[32];
        tmem_ld32(taddr + uint32_t(c), v);
        const int cc = col0 + c;
        if constexpr (K > 0) {
          // Route-margin gradient: 32 / K heads of this row in the chunk.
          constexpr int kHeads = 32 / K;
          const int64_t row = rb * kBM + quarter * 32 + lane;
          const int h0 = cc / K;
          // Routes and the margin factor code_scale * U'(m) of each head, computed while the
          // TMEM read is in flight (and before the 32 accumulator values are live, so that
          // the division does not force them out of registers).
          uint32_t wv[kHeads], rv[kHeads];
          float fv[kHeads];
#pragma unroll
          for (int hh = 0; hh < kHeads; ++hh) {
            wv[hh] = rv[hh] = 0u;
            fv[hh] = 0.f;
            if (row < gmx.rows && h0 + hh < gmx.heads) {
              const int64_t o = row * gmx.heads + h0 + hh;
              wv[hh] = __ldg(gmx.winner + o);
              rv[hh] = __ldg(gmx.runner + o);
              const float m = __ldg(gmx.margins + o);
              const float den = __fadd_rn(1.f, fabsf(m));
              const float sgn = (m > 0.f) ? 1.f : ((m < 0.f) ? -1.f : 0.f);
              fv[hh] = __fmul_rn(gmx.code_scale, __fdiv_rn(__fmul_rn(-0.5f, sgn), __fmul_rn(den, den)));
            }
          }
          tmem_wait_ld();
          reg_fence(v);
          if (c + 32 == kEpiCols) {
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
          }
#pragma unroll
          for (int hh = 0; hh < kHeads; ++hh) {
            // Bitwise pick (one cell matches): written as masks, not selects, so that the
            // compiler keeps the accumulator values in registers instead of turning the chain
            // into an indexed load from a local-memory copy.
            uint32_t bw = 0u, br = 0u;
#pragma unroll
            for (int k = 0; k < K; ++k) {
              const uint32_t x = __float_as_uint(v[hh * K + k]);
              bw |= x & (0u - uint32_t(wv[hh] == uint32_t(k)));
              br |= x & (0u - uint32_t(rv[hh] == uint32_t(k)));
            }
            const float dw = __uint_as_float(bw), dr = __uint_as_float(br);
            const float gm = __fmul_rn(__fmul_rn(__fsub_rn(dr, dw), fv[hh]), gm_unscale);
            if (row < gmx.rows && h0 + hh < gmx.heads) gmx.gm[row * gmx.heads + h0 + hh] = gm;
          }
          continue;
        }
        float bv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) bv[i] = 0.f;
        if (bias != nullptr) {
          if (cc + 32 <= out_features) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 q = __ldg(reinterpret_cast<const float4 *>(bias + cc + i));
              bv[i] = q.x;
              bv[i + 1] = q.y;
              bv[i + 2] = q.z;
              bv[i + 3] = q.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (cc + i < out_features) bv[i] = __ldg(bias + cc + i);
          }
        }
        tmem_wait_ld();
        reg_fence(v);
        if (c + 32 == kEpiCols) {
          tmem_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
        }
        // The previous tile's TMA store must have read the staging buffer.
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        uint8_t *my_row = stage + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = make_float4(__fadd_rn(v[4 * j], bv[4 * j]), __fadd_rn(v[4 * j + 1], bv[4 * j + 1]),
                                       __fadd_rn(v[4 * j + 2], bv[4 * j + 2]), __fadd_rn(v[4 * j + 3], bv[4 * j + 3]));
          *reinterpret_cast<float4 *>(my_row + ((j ^ (lane & 7)) << 4)) = q;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_out, stage, cc, static_cast<int>(rb * kBM + quarter * 32));
          bulk_commit();
        }
      }
    }
    // Every store must be complete before the CTA exits.
    if constexpr (K == 0) {
      if (lane == 0) bulk_wait_all();
      __syncwarp();
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

// [hi | lo] halves of each f32 row: hi = half(x s), lo = half(x s - hi), s = the power-of-two
// gradient scale of *absmax (1 without it).
template <typename PT>
__global__ void __launch_bounds__(256) split_half_kernel(const float *__restrict__ x, int64_t rows, int cols,
                                                          const uint32_t *__restrict__ absmax, PT *__restrict__ out) {
  const float s = grad_scale_of(absmax);
  const int64_t total = rows * cols / 4;
  for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < total; q += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = q * 4;
    const int64_t row = i / cols;
    const int col = static_cast<int>(i - row * cols);
    const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + q);
    const float xs[4] = {__fmul_rn(v.x, s), __fmul_rn(v.y, s), __fmul_rn(v.z, s), __fmul_rn(v.w, s)};
    PT hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hi[e] = from_f32<PT>(xs[e]);
      lo[e] = from_f32<PT>(__fsub_rn(xs[e], to_f32(hi[e])));
    }
    PT *o = out + row * (2 * int64_t(cols)) + col;
    *reinterpret_cast<uint2 *>(o) = *reinterpret_cast<const uint2 *>(hi);
    *reinterpret_cast<uint2 *>(o + cols) = *reinterpret_cast<const uint2 *>(lo);
  }
}

template <typename PT>
__device__ __forceinline__ uint32_t pack_pair(PT a, PT b) {
  return uint32_t(*reinterpret_cast<const unsigned short *>(&a)) |
         (uint32_t(*reinterpret_cast<const unsigned short *>(&b)) << 16);
}

// split_half and its transpose in one pass over x: out_split [rows, 2 cols] = [hi | lo] of
// x s (split_half_kernel's arithmetic) and out_t [cols, rows] = hi^T (what transpose_to_half
// writes for the same x and scale). 64 x 64 tiles of 256 threads; each warp takes pairs of
// rows, so the shared tile holds (row 2p, row 2p + 1) pairs per 4-byte word and every
// transposed store is a 128-byte warp store. Even rows and cols (the host checks).
template <typename PT>
__global__ void __launch_bounds__(256) split_transpose_half_kernel(const float *__restrict__ x, int64_t rows,
                                                                   int cols, const uint32_t *__restrict__ absmax,
                                                                   PT *__restrict__ out_split,
                                                                   PT *__restrict__ out_t) {
  __shared__ uint32_t pair_t[64][33];  // [tile column][row pair]
  const float s = grad_scale_of(absmax);
  const int64_t r0 = int64_t(blockIdx.x) * 64;
  const int c0 = blockIdx.y * 64;
  const int tx = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = c0 + 2 * tx;
  const bool col_ok = c < cols;
  float2 v[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 2 * (w + 8 * i);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      v[i][h] = make_float2(0.f, 0.f);
      if (col_ok && r + h < rows) v[i][h] = __ldg(reinterpret_cast<const float2 *>(x + (r + h) * cols + c));
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = w + 8 * i;
    const int64_t r = r0 + 2 * p;
    PT hi[2][2];  // [row of the pair][column of the pair]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float xs0 = __fmul_rn(v[i][h].x, s), xs1 = __fmul_rn(v[i][h].y, s);
      hi[h][0] = from_f32<PT>(xs0);
      hi[h][1] = from_f32<PT>(xs1);
      const PT lo0 = from_f32<PT>(__fsub_rn(xs0, to_f32(hi[h][0])));
      const PT lo1 = from_f32<PT>(__fsub_rn(xs1, to_f32(hi[h][1])));
      if (col_ok && r + h < rows) {
        PT *o = out_split + (r + h) * (2 * int64_t(cols)) + c;
        *reinterpret_cast<uint32_t *>(o) = pack_pair(hi[h][0], hi[h][1]);
        *reinterpret_cast<uint32_t *>(o + cols) = pack_pair(lo0, lo1);
      }
    }
    pair_t[2 * tx][p] = pack_pair(hi[0][0], hi[1][0]);
    pair_t[2 * tx + 1][p] = pack_pair(hi[0][1], hi[1][1]);
  }
  __syncthreads();
  const int64_t rr = r0 + 2 * tx;  // first of this thread's pair of output columns
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int cc = w + 8 * i;
    if (c0 + cc < cols && rr < rows)
      *reinterpret_cast<uint32_t *>(out_t + int64_t(c0 + cc) * rows + rr) = pair_t[cc][tx];
  }
}

// *bits = max(*bits, f32 bits of max |x|): non-negative floats order as their bit patterns,
// so the integer maximum is order-independent (deterministic). The caller zeroes *bits first.
__global__ void __launch_bounds__(256) absmax_kernel(const float *__restrict__ x, int64_t n,
                                                     uint32_t *__restrict__ bits) {
  uint32_t m = 0u;
  const int64_t quads = n / 4;
  for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < quads; q += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + q);
    m = max(m, max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                   max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w)))));
  }
  for (int64_t i = quads * 4 + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    m = max(m, __float_as_uint(fabsf(__ldg(x + i))));
  m = __reduce_max_sync(0xffffffffu, m);
  __shared__ uint32_t wmax[8];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t b = wmax[0];
    for (int w = 1; w < 8; ++w) b = max(b, wmax[w]);
    atomicMax(bits, b);
  }
}

size_t linear_fixed_smem(int a_blocks, int K) {
  return 1024 + size_t(a_blocks) * kTileBytesA + out_stage_bytes(K) + sizeof(Barriers);
}

int linear_stages(int a_blocks, int K) {
  const size_t fixed = linear_fixed_smem(a_blocks, K);
  if (fixed >= kSmemLimit) return 0;
  const int s = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / kTileBytesB));
  return s >= kMinStages ? s : 0;
}

template <typename PT, int K>
int launch_linear(const void *a, int64_t rows, int slices, const void *w, int out_features, int in_features,
                  const float *bias, float *out, const GmArgs &gmx, cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int b_kblocks = in_features / kBK;
  const int a_blocks = slices * b_kblocks;
  const int stages = linear_stages(a_blocks, K);
  const size_t smem = linear_fixed_smem(a_blocks, K) + size_t(stages) * kTileBytesB;
  CUtensorMap map_a, map_w, map_out;
  TB_CHECK(make_map_k64(&map_a, a, dt, int64_t(slices) * in_features, rows, kBM));
  TB_CHECK(make_map_k64(&map_w, w, dt, in_features, out_features, kBoxRows));
  if constexpr (K == 0) {
    TB_CHECK(make_map_f32_store32(&map_out, out, out_features, rows));
  } else {
    map_out = map_a;  // unused by the route-margin epilogue
  }
  const int tiles_total = static_cast<int>(ceil_div(int64_t(out_features), int64_t(kBN)));
  const int64_t units = ceil_div(rows, int64_t(kBM)) * tiles_total;
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  auto kernel = linear_f32out_kernel<PT, K>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "linear_f32out"));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(units, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_a, map_w, map_out, bias, out_features, slices, b_kblocks, stages,
                                           tiles_total, units, gmx);
  return check_launch(K == 0 ? "linear_f32out" : "trop_gm_sm100");
}

}  // namespace

bool linear_f32out_supported(int64_t rows, int64_t slices, int64_t out_features, int64_t in_features, int dtype) {
  return (dtype == TROPNN_B200_F16 || dtype == TROPNN_B200_BF16) && (slices == 1 || slices == 2) && rows >= 1 &&
         rows <= (int64_t(1) << 31) - 1024 && in_features % kBK == 0 && in_features >= kBK &&
         slices * (in_features / kBK) <= kMaxABlocks && linear_stages(static_cast<int>(slices * in_features / kBK), 0) > 0 &&
         out_features >= 1 && out_features % 4 == 0 && out_features <= (int64_t(1) << 30);
}

int linear_f32out_impl(const void *a, int64_t rows, int64_t slices, const void *w, int64_t out_features,
                       int64_t in_features, int dtype, const float *bias, float *out, cudaStream_t stream) {
  TB_REQUIRE(linear_f32out_supported(rows, slices, out_features, in_features, dtype), TROPNN_B200_ERR_INVALID,
             "linear_f32out: unsupported shape rows=%lld slices=%lld out=%lld in=%lld dtype=%s", (long long)rows,
             (long long)slices, (long long)out_features, (long long)in_features, dtype_name(dtype));
  TB_REQUIRE(a && w && out, TROPNN_B200_ERR_INVALID, "linear_f32out: null pointer");
  auto al16 = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  TB_REQUIRE(al16(a) && al16(w) && al16(bias) && al16(out), TROPNN_B200_ERR_INVALID,
             "linear_f32out: operands must be 16-byte aligned");
  const int s = static_cast<int>(slices), n = static_cast<int>(out_features), k = static_cast<int>(in_features);
  const GmArgs none{};
  if (dtype == TROPNN_B200_F16) return launch_linear<__half, 0>(a, rows, s, w, n, k, bias, out, none, stream);
  return launch_linear<__nv_bfloat16, 0>(a, rows, s, w, n, k, bias, out, none, stream);
}

// gm[n,h] of the min-face backward from g split into [hi | lo] ([rows, 2*code_dim]) and
// the code table [heads*cells, code_dim] (the B operand as stored).
int trop_gm_sm100_impl(const void *g_split, int64_t rows, int64_t code_dim, const void *code, int dtype, int64_t heads,
                       int64_t cells, const uint8_t *winner, const uint8_t *runner, const float *margins,
                       float code_scale, float *gm, const uint32_t *absmax, cudaStream_t stream) {
  const int64_t hk = heads * cells;
  TB_REQUIRE(linear_f32out_supported(rows, 2, hk, code_dim, dtype) &&
                 (cells == 2 || cells == 4 || cells == 8 || cells == 16 || cells == 32),
             TROPNN_B200_ERR_INVALID, "trop_gm_sm100: unsupported shape rows=%lld code_dim=%lld heads=%lld cells=%lld",
             (long long)rows, (long long)code_dim, (long long)heads, (long long)cells);
  TB_REQUIRE(g_split && code && winner && runner && margins && gm, TROPNN_B200_ERR_INVALID, "trop_gm_sm100: null pointer");
  // Per-thread vector accesses of kEpiCols / cells consecutive heads (cells >= 8): whole
  // vectors inside each row and 16-byte aligned bases.
  const int64_t hpt = 128 / cells;
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int vec = (cells >= 8 && heads % hpt == 0 && al16(winner) && al16(runner) && al16(margins) && al16(gm)) ? 1 : 0;
  const GmArgs gmx{winner, runner, margins, gm, rows, static_cast<int>(heads), code_scale, absmax, vec};
  const int n = static_cast<int>(hk), k = static_cast<int>(code_dim);
  auto go = [&](auto pt_tag) -> int {
    using T = decltype(pt_tag);
    switch (cells) {
      case 2: return launch_linear<T, 2>(g_split, rows, 2, code, n, k, nullptr, nullptr, gmx, stream);
      case 4: return launch_linear<T, 4>(g_split, rows, 2, code, n, k, nullptr, nullptr, gmx, stream);
      case 8: return launch_linear<T, 8>(g_split, rows, 2, code, n, k, nullptr, nullptr, gmx, stream);
      case 16: return launch_linear<T, 16>(g_split, rows, 2, code, n, k, nullptr, nullptr, gmx, stream);
      default: return launch_linear<T, 32>(g_split, rows, 2, code, n, k, nullptr, nullptr, gmx, stream);
    }
  };
  if (dtype == TROPNN_B200_F16) return go(__half());
  return go(__nv_bfloat16());
}

int split_half_impl(const float *x, int64_t rows, int64_t cols, int dtype, const uint32_t *absmax, void *out,
                    cudaStream_t stream) {
  TB_REQUIRE(dtype == TROPNN_B200_F16 || dtype == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "split_half: dtype %s unsupported (f16/bf16 only)", dtype_name(dtype));
  TB_REQUIRE(rows >= 0 && cols > 0 && cols % 4 == 0 && cols <= (1 << 30), TROPNN_B200_ERR_INVALID,
             "split_half: cols=%lld must be a positive multiple of 4", (long long)cols);
  if (rows == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && out, TROPNN_B200_ERR_INVALID, "split_half: null pointer");
  TB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 8 == 0,
             TROPNN_B200_ERR_INVALID, "split_half: misaligned operands");
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const int64_t quads = rows * cols / 4;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(quads, int64_t(256)), int64_t(sms) * 8));
  if (dtype == TROPNN_B200_F16)
    split_half_kernel<__half><<<grid, 256, 0, stream>>>(x, rows, static_cast<int>(cols), absmax,
                                                        static_cast<__half *>(out));
  else
    split_half_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(x, rows, static_cast<int>(cols), absmax,
                                                               static_cast<__nv_bfloat16 *>(out));
  return check_launch("split_half");
}

int split_transpose_half_impl(const float *x, int64_t rows, int64_t cols, int dtype, const uint32_t *absmax,
                              void *out_split, void *out_t, cudaStream_t stream) {
  TB_REQUIRE(dtype == TROPNN_B200_F16 || dtype == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "split_transpose_half: dtype %s unsupported (f16/bf16 only)", dtype_name(dtype));
  TB_REQUIRE(rows >= 0 && rows % 2 == 0 && cols > 0 && cols % 4 == 0 && cols <= (1 << 20), TROPNN_B200_ERR_INVALID,
             "split_transpose_half: rows=%lld must be even and cols=%lld a positive multiple of 4", (long long)rows,
             (long long)cols);
  if (rows == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && out_split && out_t, TROPNN_B200_ERR_INVALID, "split_transpose_half: null pointer");
  TB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out_split) % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(out_t) % 4 == 0,
             TROPNN_B200_ERR_INVALID, "split_transpose_half: misaligned operands");
  const int64_t row_tiles = ceil_div(rows, int64_t(64)), col_tiles = ceil_div(cols, int64_t(64));
  TB_REQUIRE(row_tiles < (int64_t(1) << 31) && col_tiles < 65536, TROPNN_B200_ERR_INVALID,
             "split_transpose_half: rows=%lld too large", (long long)rows);
  const dim3 grid(static_cast<unsigned>(row_tiles), static_cast<unsigned>(col_tiles));
  if (dtype == TROPNN_B200_F16)
    split_transpose_half_kernel<__half><<<grid, 256, 0, stream>>>(x, rows, static_cast<int>(cols), absmax,
                                                                  static_cast<__half *>(out_split),
                                                                  static_cast<__half *>(out_t));
  else
    split_transpose_half_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(x, rows, static_cast<int>(cols), absmax,
                                                                         static_cast<__nv_bfloat16 *>(out_split),
                                                                         static_cast<__nv_bfloat16 *>(out_t));
  return check_launch("split_transpose_half");
}

int absmax_impl(const float *x, int64_t n, uint32_t *bits, cudaStream_t stream) {
  TB_REQUIRE(n >= 0 && bits != nullptr && (n == 0 || x != nullptr), TROPNN_B200_ERR_INVALID, "absmax: bad arguments");
  TB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0, TROPNN_B200_ERR_INVALID, "absmax: x must be 16-byte aligned");
  if (n == 0) return TROPNN_B200_OK;
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(n, int64_t(1024)), int64_t(sms) * 4));
  absmax_kernel<<<grid, 256, 0, stream>>>(x, n, bits);
  return check_launch("absmax");
}

int read_gemm_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

int tropnn_b200_split_half(const float *x, int64_t rows, int64_t cols, int dtype, const void *grad_absmax, void *out,
                           void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::split_half_impl(x, rows, cols, dtype, static_cast<const uint32_t *>(grad_absmax), out,
                                        tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_split_transpose_half(const float *x, int64_t rows, int64_t cols, int dtype, const void *grad_absmax,
                                     void *out_split, void *out_t, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::split_transpose_half_impl(x, rows, cols, dtype, static_cast<const uint32_t *>(grad_absmax),
                                                  out_split, out_t, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_absmax_f32(const float *x, int64_t n, void *bits, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::absmax_impl(x, n, static_cast<uint32_t *>(bits), tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_linear_f32out(const void *a, int64_t rows, int64_t slices, const void *weight, int64_t out_features,
                              int64_t in_features, int dtype, const float *bias, float *out, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  if (rows == 0) return tropnn_b200::clear_error();
  TB_CHECK(tropnn_b200::linear_f32out_impl(a, rows, slices, weight, out_features, in_features, dtype, bias, out,
                                           tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
