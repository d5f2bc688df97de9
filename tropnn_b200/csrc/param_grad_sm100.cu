// TropLinear parameter gradients on the sm_100a tensor cores (half-precision parameters):
//   grad_code[h,k,:]   = sum_n (vw[n,h] [w[n,h]==k] + vr[n,h] [r[n,h]==k]) g[n,:]
//        vw = code_scale (1 - U(m)), vr = code_scale U(m) in training; vw = code_scale,
//        vr = 0 in eval                          (layers/tropical_exact.py:204-237)
//   grad_router[h,k,:] = sum_n (gm[n,h] [w[n,h]==k] - gm[n,h] [r[n,h]==k]) z[n,:]
// i.e. P^T X with P the (weighted) one-hot route matrix [rows, H*K] and X = g or z. The
// reference's coefficient einsums (and this library's per-bucket row sums) read a D-wide
// row of X per (row, head); as a GEMM with M = H*K, N = code_dim, K = rows, X streams
// through the tensor cores once per 128 (head, cell) entries.
//
// Operands: B = X^T [code_dim, rows] (K-major, f16/bf16; g is rounded once to the
// parameter dtype, within the 2e-2 tolerance of half-precision layers), loaded by TMA in
// 64-row k blocks; A = P^T built in registers and written into TMEM with tcgen05.st (MMA
// reads A from TMEM): TMEM lane L of a tile is entry (h0 + L / K, L % K). For each k
// block the builders first stage the tile's routes and weights ([64 rows x 128/K heads],
// 8 bytes each) in shared memory, then every lane assembles its 32 packed pairs.
//
// CTA = 14 warps, persistent over 128-entry tiles:
//   warp 0      TMA producer of the X^T k blocks.
//   warp 1      TMEM (accumulator [0, D), one-hot ring [256, 512)); lane 0 issues the
//               MMAs (M=128, N=code_dim, K=16, A from TMEM).
//   warps 2-9   builders: warps 2-5 take the even k blocks, 6-9 the odd ones (each warp
//               its TMEM lane quarter); each set stages its k block cooperatively.
//   warps 10-13 epilogue: the accumulator rows, rounded to the parameter dtype, to
//               out[(h,k), :].
// All waits are bounded (sm100.cuh); whole-warp waits use mbarrier suspend hints.
#include <cuda.h>

#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;         // (head, cell) entries per tile = TMEM lanes
constexpr int kBK = 64;          // sample rows per k block
constexpr int kMaxD = 256;
constexpr int kMaxBStages = 6;
constexpr int kMinBStages = 3;
constexpr int kAStages = 8;
constexpr int kBuildWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kBuildWarps + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAColBase = 256;
constexpr size_t kSmemLimit = 227 * 1024;
constexpr uint32_t kSleepHintNs = 1000000u;
constexpr int kPRowHalves = kBK + 8;                           // 64 samples + 16 bytes of padding
constexpr int kStageBytes = kBM * kPRowHalves * 2;             // one parity's one-hot block

enum Mode { kCodeEval = 0, kCodeTrain = 1, kRouter = 2 };

__device__ int g_param_grad_error = 0;

struct Barriers {
  int verdict[2][2];
  uint64_t b_full[kMaxBStages];
  uint64_t b_empty[kMaxBStages];
  uint64_t a_full[kAStages];
  uint64_t a_empty[kAStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Barriers *bs) {
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_param_grad_error);
}

__device__ __forceinline__ bool wait_bar_sleep(uint64_t *bar, uint32_t parity, Barriers *bs) {
  const uint64_t start = global_ns();
  volatile int *abort = &bs->abort;
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSleepHintNs)
        : "memory");
    if (ok) return true;
    if (*abort) return false;
    if (global_ns() - start > kWaitLimitNs) {
      *abort = 1;
      atomicExch(&g_param_grad_error, 1);
      return false;
    }
  }
}

__device__ __forceinline__ bool warp_wait_sleep(uint64_t *bar, uint32_t parity, Barriers *bs, int lane) {
  int ok = 1;
  if (lane == 0) ok = wait_bar_sleep(bar, parity, bs) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

template <typename PT>
__device__ __forceinline__ uint32_t half_bits(float x) {
  if constexpr (std::is_same<PT, __half>::value)
    return __half_as_ushort(__float2half_rn(x));
  else
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

template <typename PT, int K, int MODE>
__global__ void __launch_bounds__(kThreads, 1) trop_param_grad_kernel(
    const __grid_constant__ CUtensorMap map_xt, const uint8_t *__restrict__ winner, const uint8_t *__restrict__ runner,
    const float *__restrict__ mvals, float code_scale, int64_t rows, int H, int D, int kblocks, int bstages, int tiles,
    const uint32_t *__restrict__ absmax, PT *__restrict__ out) {
  static_assert(K >= 2 && K <= 32 && (K & (K - 1)) == 0, "cells must be a power of two in [2, 32]");
  constexpr int kHeadsPerTile = kBM / K;
  const uint32_t idesc = umma_idesc_f16(std::is_same<PT, __half>::value ? 0 : 1, kBM, D);
  const int b_stage_bytes = D * 128;
  // Gradient scale (power of two) of g_t (modes 0, 1: applied by its transpose) or of the gm
  // weights (mode 2: applied by the builders), undone by the epilogue.
  const float gscale = grad_scale_of(absmax);
  const float out_scale = __fmul_rn(MODE == kRouter ? 1.f : code_scale, pow2_inverse(gscale));

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *b_smem = smem;                                       // bstages x [D rows x 128 B]
  uint8_t *stage = b_smem + bstages * b_stage_bytes;  // 2 parities x [kBM][kPRowHalves] 16-bit weights
  Barriers *bs = reinterpret_cast<Barriers *>(stage + 2 * kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int (*verdict)[2] = bs->verdict;

  if (threadIdx.x == 0) {
    for (int s = 0; s < bstages; ++s) {
      mbar_init(&bs->b_full[s], 1);
      mbar_init(&bs->b_empty[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&bs->a_full[s], kBuildWarps / 2);
      mbar_init(&bs->a_empty[s], 1);
    }
    mbar_init(&bs->acc_full, 1);
    mbar_init(&bs->acc_empty, kEpiWarps);
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
    if (lane == 0) {
      // ---------------- TMA producer: X^T k blocks ----------------
      prefetch_map(&map_xt);
      uint32_t issued[kMaxBStages];
      for (int s = 0; s < kMaxBStages; ++s) issued[s] = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % bstages;
          if (!wait_bar(&bs->b_empty[s], (uint32_t(it / bstages) & 1u) ^ 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->b_full[s], uint32_t(b_stage_bytes));
          tma_load_2d(b_smem + s * b_stage_bytes, &map_xt, &bs->b_full[s], kb * kBK, 0);
          issued[s] = uint32_t(it / bstages) + 1;
        }
      }
      for (int s = 0; s < bstages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->b_full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = true;
      int bit = 0, ait = 0;
      uint32_t i = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++i) {
        if (!wait_bar(&bs->acc_empty, (i & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        for (int kb = 0; kb < kblocks; ++kb, ++bit, ++ait) {
          const int sa = ait % kAStages, sb = bit % bstages;
          if (!wait_bar(&bs->a_full[sa], uint32_t(ait / kAStages) & 1u, bs) ||
              !wait_bar(&bs->b_full[sb], uint32_t(bit / bstages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t b_base = smem_addr(b_smem + sb * b_stage_bytes);
          const uint32_t a_col = tmem_base + kAColBase + uint32_t(sa * 32);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16_tmem_a(tmem_base, a_col + uint32_t(kk * 8), umma_desc_sw128(b_base + kk * 32), idesc,
                            (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&bs->a_empty[sa]);
          umma_commit(&bs->b_empty[sb]);
        }
        if (!ok) break;
        umma_commit(&bs->acc_full);
      }
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else if (warp < 2 + kBuildWarps) {
    // ---------------- builders ----------------
    const int quarter = warp & 3;
    const int parity = (warp - 2) >> 2;
    const int tid = (warp - 2 - 4 * parity) * 32 + lane;  // 0..127 within this parity's set
    const int L = quarter * 32 + lane;                     // TMEM lane = tile entry
    const uint32_t lane_base = tmem_base + (uint32_t(quarter * 32) << 16) + kAColBase;
    // Entries of a staged k block per builder thread; with few of them (cells >= 8) the
    // raw route bytes and weights of the set's next k block are loaded into registers while
    // the current one is built, so their latency leaves the critical path.
    constexpr int kPer = kBK * kHeadsPerTile / 128;
    constexpr bool kPrefetch = kPer <= 8;
    constexpr int kPerRegs = kPrefetch ? kPer : 1;
    uint32_t pw[kPerRegs], pr[kPerRegs];
    float pm[kPerRegs];
    auto fetch = [&](int a) {
      const int i = a / kblocks;
      const int kb = a - i * kblocks;
      const int tile = blockIdx.x + i * gridDim.x;
      const int h0 = tile * kHeadsPerTile;
      const int64_t n0 = int64_t(kb) * kBK;
#pragma unroll
      for (int q = 0; q < kPerRegs; ++q) {
        const int e = tid + q * 128;
        const int rr = e / kHeadsPerTile;
        const int h = h0 + (e - rr * kHeadsPerTile);
        const int64_t n = n0 + rr;
        pw[q] = pr[q] = 0xFFu;
        pm[q] = 0.f;
        if (tile < tiles && n < rows && h < H) {
          const int64_t o = n * H + h;
          pw[q] = __ldg(winner + o);
          if constexpr (MODE != kCodeEval) {
            pr[q] = __ldg(runner + o);
            pm[q] = __ldg(mvals + o);
          }
        }
      }
    };
    auto encode = [&](uint32_t w, uint32_t r, float mv) -> uint2 {
      uint32_t vw = 0u, vr = 0u;
      if (w != 0xFFu) {
        if constexpr (MODE == kCodeEval) {
          vw = half_bits<PT>(1.f);  // code_scale is applied in f32 by the epilogue
        } else if constexpr (MODE == kCodeTrain) {
          const float alpha = __fdiv_rn(0.5f, __fadd_rn(1.f, fabsf(mv)));
          vw = half_bits<PT>(__fsub_rn(1.f, alpha));
          vr = half_bits<PT>(alpha);
        } else {
          vw = half_bits<PT>(__fmul_rn(mv, gscale));
          vr = half_bits<PT>(-__fmul_rn(mv, gscale));
        }
      }
      return make_uint2(w | (r << 8), vw | (vr << 16));
    };
    // One-hot block of the item, [128 entries][64 samples] 16-bit weights in shared memory
    // (rows kPRowHalves apart: the padding spreads the row-per-lane 16-byte reads over the
    // banks): the staging threads scatter each (sample, head)'s winner / runner-up weight into
    // its entry's row, then every builder thread reads its own entry's row (the TMEM column
    // layout: 32-bit word j = samples 2j, 2j+1) and clears it for the next item.
    uint16_t *pm_rows = reinterpret_cast<uint16_t *>(stage) + parity * (kBM * kPRowHalves);
    auto scatter = [&](int e, uint32_t w, uint32_t r, float mv) {
      const uint2 v = encode(w, r, mv);
      const int rr = e / kHeadsPerTile;
      const int hl = e - rr * kHeadsPerTile;
      if (w < uint32_t(K)) pm_rows[(hl * K + int(w)) * kPRowHalves + rr] = uint16_t(v.y & 0xFFFFu);
      if constexpr (MODE != kCodeEval)
        if (r < uint32_t(K) && r != w) pm_rows[(hl * K + int(r)) * kPRowHalves + rr] = uint16_t(v.y >> 16);
    };
    {
      // This thread's row starts clear (the first named barrier below orders it before any
      // scatter into it).
      uint4 *my_row = reinterpret_cast<uint4 *>(pm_rows + L * kPRowHalves);
#pragma unroll
      for (int c = 0; c < 8; ++c) my_row[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    if constexpr (kPrefetch) fetch(parity);
    for (int ait = parity;; ait += 2) {
      const int i = ait / kblocks;
      const int kb = ait - i * kblocks;
      const int tile = blockIdx.x + i * gridDim.x;
      if (tile >= tiles) break;
      const int h0 = tile * kHeadsPerTile;
      const int64_t n0 = int64_t(kb) * kBK;
      // One thread of the set waits for the TMEM slot; the verdict passes through a
      // two-slot flag behind the named barrier, so all 128 builders of the set take the same
      // branch (a warp leaving alone would strand the others at the next named barrier).
      // Slot (ait/2)&1 is rewritten two items later, after every builder of the set has
      // passed this item's later named barriers and so has read it. The barrier also orders
      // the previous item's row clears before this item's scatter.
      if (tid == 0)
        verdict[parity][(ait >> 1) & 1] =
            wait_bar_sleep(&bs->a_empty[ait % kAStages], (uint32_t(ait / kAStages) & 1u) ^ 1u, bs) ? 1 : 0;
      named_sync(2 + parity, 128);
      if (*reinterpret_cast<volatile int *>(&verdict[parity][(ait >> 1) & 1]) == 0) break;
      if constexpr (kPrefetch) {
#pragma unroll
        for (int q = 0; q < kPer; ++q) scatter(tid + q * 128, pw[q], pr[q], pm[q]);
        fetch(ait + 2);
      } else {
        for (int e = tid; e < kBK * kHeadsPerTile; e += 128) {
          const int rr = e / kHeadsPerTile;
          const int h = h0 + (e - rr * kHeadsPerTile);
          const int64_t n = n0 + rr;
          uint32_t w = 0xFFu, r = 0xFFu;
          float mv = 0.f;
          if (n < rows && h < H) {
            const int64_t o = n * H + h;
            w = __ldg(winner + o);
            if constexpr (MODE != kCodeEval) {
              r = __ldg(runner + o);
              mv = __ldg(mvals + o);
            }
          }
          scatter(e, w, r, mv);
        }
      }
      named_sync(2 + parity, 128);  // the block is complete
      tmem_fence_after();
      uint32_t reg[32];
      uint4 *my_row = reinterpret_cast<uint4 *>(pm_rows + L * kPRowHalves);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 q = my_row[c];
        reg[4 * c] = q.x, reg[4 * c + 1] = q.y, reg[4 * c + 2] = q.z, reg[4 * c + 3] = q.w;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) my_row[c] = make_uint4(0u, 0u, 0u, 0u);
      tmem_st32(lane_base + uint32_t((ait % kAStages) * 32), reg);
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bs->a_full[ait % kAStages]);
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem_base + (uint32_t(quarter * 32) << 16);
    uint32_t i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      const int L = quarter * 32 + lane;
      const int64_t entry = int64_t(tile) * kBM + L;  // h * K + k
      if (!warp_wait_sleep(&bs->acc_full, i & 1u, bs, lane)) break;
      tmem_fence_after();
      for (int c = 0; c < D; c += 32) {
        float acc[32];
        tmem_ld32(lane_base + uint32_t(c), acc);
        tmem_wait_ld();
        reg_fence(acc);
        if (c + 32 >= D) {
          tmem_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bs->acc_empty);
        }
        if (entry < int64_t(H) * K) {
          PT *o = out + entry * D + c;
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 q;
            q.x = half_bits<PT>(__fmul_rn(acc[e], out_scale)) | (half_bits<PT>(__fmul_rn(acc[e + 1], out_scale)) << 16);
            q.y = half_bits<PT>(__fmul_rn(acc[e + 2], out_scale)) | (half_bits<PT>(__fmul_rn(acc[e + 3], out_scale)) << 16);
            q.z = half_bits<PT>(__fmul_rn(acc[e + 4], out_scale)) | (half_bits<PT>(__fmul_rn(acc[e + 5], out_scale)) << 16);
            q.w = half_bits<PT>(__fmul_rn(acc[e + 6], out_scale)) | (half_bits<PT>(__fmul_rn(acc[e + 7], out_scale)) << 16);
            *reinterpret_cast<uint4 *>(o + e) = q;
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

// Router-bias gradient: grad_b[h,k] = sum_n gm[n,h] ([w==k] - [r==k]). A cluster of
// kBiasSlices CTAs owns 32 heads (one per lane, so every warp load reads 32 consecutive heads of
// a row); CTA y of the cluster takes row slice y, its 16 warps take interleaved rows. Warp
// partials are combined in warp order, then slice partials in slice order through distributed
// shared memory, so the result is deterministic.
constexpr int kBiasSlices = 8, kBiasWarps = 16;

template <int K>
constexpr size_t bias_smem_bytes() {
  return sizeof(float) * (size_t(kBiasWarps) * 32 * (K + 1) + 32 * K);
}

template <typename PT, int K>
__global__ void __cluster_dims__(1, kBiasSlices, 1) __launch_bounds__(kBiasWarps * 32, K >= 32 ? 1 : 2)
    router_bias_grad_kernel(const uint8_t *__restrict__ winner, const uint8_t *__restrict__ runner,
                            const float *__restrict__ gm, int64_t rows, int H, PT *__restrict__ grad_b) {
  extern __shared__ float bias_smem[];
  float *part = bias_smem;                                    // [kBiasWarps][32][K + 1]
  float *red = bias_smem + size_t(kBiasWarps) * 32 * (K + 1);  // [32 * K]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.x * 32 + lane;
  const int64_t per = (rows + kBiasSlices - 1) / kBiasSlices;
  const int64_t n_begin = per * blockIdx.y, n_end = n_begin + per < rows ? n_begin + per : rows;
  // This thread's K partial sums live in its own shared-memory row (stride K + 1: no bank
  // conflicts): each row adds gm to the winner's cell and subtracts it from the runner-up's,
  // two read-modify-writes instead of K selects (the same sums, bit for bit: the other cells
  // would only add 0).
  float *mine = part + (warp * 32 + lane) * (K + 1);
#pragma unroll
  for (int k = 0; k < K; ++k) mine[k] = 0.f;
  if (h < H) {
    constexpr int kUnroll = 8;
    for (int64_t n = n_begin + warp; n < n_end; n += kUnroll * kBiasWarps) {
      uint32_t w[kUnroll], r[kUnroll];
      float v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t nu = n + int64_t(u) * kBiasWarps;
        const bool ok = nu < n_end;
        const int64_t o = (ok ? nu : n) * H + h;
        // Routes come from this library's route kernel; clamped anyway so that a corrupt one
        // cannot address outside the thread's row.
        w[u] = min(uint32_t(__ldg(winner + o)), uint32_t(K - 1));
        r[u] = min(uint32_t(__ldg(runner + o)), uint32_t(K - 1));
        v[u] = ok ? __ldg(gm + o) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        mine[w[u]] = __fadd_rn(mine[w[u]], __fsub_rn(v[u], 0.f));
        mine[r[u]] = __fadd_rn(mine[r[u]], __fsub_rn(0.f, v[u]));
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * K; e += kBiasWarps * 32) {
    const int hl = e / K, k = e - hl * K;
    float sum = 0.f;
    for (int wi = 0; wi < kBiasWarps; ++wi) sum = __fadd_rn(sum, part[(wi * 32 + hl) * (K + 1) + k]);
    red[e] = sum;
  }
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  constexpr int kShare = 32 * K / kBiasSlices;
  const int slice = static_cast<int>(cluster.block_rank());
  for (int i = threadIdx.x; i < kShare; i += kBiasWarps * 32) {
    const int e = slice * kShare + i;
    float sum = 0.f;
    for (int y = 0; y < kBiasSlices; ++y) sum = __fadd_rn(sum, cluster.map_shared_rank(red, y)[e]);
    const int hl = e / K, k = e - hl * K;
    if (blockIdx.x * 32 + hl < H) grad_b[int64_t(blockIdx.x * 32 + hl) * K + k] = from_f32<PT>(sum);
  }
  cluster.sync();
}

template <typename PT, int K>
int launch_bias_grad(const uint8_t *w, const uint8_t *r, const float *gm, int64_t rows, int H, PT *grad_b,
                     cudaStream_t stream) {
  constexpr size_t smem = bias_smem_bytes<K>();
  if (smem > 48 * 1024)
    TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(router_bias_grad_kernel<PT, K>), smem,
                                 "router_bias_grad"));
  const dim3 grid(static_cast<unsigned>(ceil_div(int64_t(H), int64_t(32))), kBiasSlices);
  router_bias_grad_kernel<PT, K><<<grid, kBiasWarps * 32, smem, stream>>>(w, r, gm, rows, H, grad_b);
  return check_launch("router_bias_grad");
}

// x [rows_in, cols] (f32 or half) times the power-of-two gradient scale of *absmax (1 without it)
// -> out [cols, rows_in] in PT, 32 x 32 tiles.
template <typename IT, typename PT>
__global__ void __launch_bounds__(256) transpose_to_half_kernel(const IT *__restrict__ in, PT *__restrict__ out,
                                                                int64_t rows_in, int cols,
                                                                const uint32_t *__restrict__ absmax) {
  __shared__ float tile[32][33];
  const float s = grad_scale_of(absmax);
  const int64_t r0 = int64_t(blockIdx.x) * 32;
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int j = ty; j < 32; j += 8)
    if (r0 + j < rows_in && c0 + tx < cols) tile[j][tx] = __fmul_rn(to_f32(in[(r0 + j) * cols + c0 + tx]), s);
  __syncthreads();
  for (int j = ty; j < 32; j += 8)
    if (c0 + j < cols && r0 + tx < rows_in) out[int64_t(c0 + j) * rows_in + r0 + tx] = from_f32<PT>(tile[tx][j]);
}

// The same for an even row count: 64 input rows per tile, and each thread writes two
// consecutive rows of one output row as one 4-byte store (128-byte coalesced warp stores).
template <typename IT, typename PT>
__global__ void __launch_bounds__(256) transpose_to_half_pairs_kernel(const IT *__restrict__ in, PT *__restrict__ out,
                                                                      int64_t rows_in, int cols,
                                                                      const uint32_t *__restrict__ absmax) {
  __shared__ float tile[64][33];
  const float s = grad_scale_of(absmax);
  const int64_t r0 = int64_t(blockIdx.x) * 64;
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int j = ty; j < 64; j += 8)
    if (r0 + j < rows_in && c0 + tx < cols) tile[j][tx] = __fmul_rn(to_f32(in[(r0 + j) * cols + c0 + tx]), s);
  __syncthreads();
  for (int j = ty; j < 32; j += 8) {
    const int64_t r = r0 + 2 * tx;
    if (c0 + j < cols && r < rows_in) {
      *reinterpret_cast<uint32_t *>(out + int64_t(c0 + j) * rows_in + r) =
          half_bits<PT>(tile[2 * tx][j]) | (half_bits<PT>(tile[2 * tx + 1][j]) << 16);
    }
  }
}

int b_stages(int D) {
  const size_t stage = size_t(D) * 128;
  const size_t room = kSmemLimit - 1024 - 2 * size_t(kStageBytes) - sizeof(Barriers);
  const int s = static_cast<int>(std::min<size_t>(kMaxBStages, room / stage));
  return s >= kMinBStages ? s : 0;
}

template <typename PT, int K, int MODE>
int launch_param_grad(const void *xt, int64_t rows, int D, int H, const uint8_t *win, const uint8_t *run,
                      const float *mvals, float code_scale, const uint32_t *absmax, void *out, cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap map_xt;
  TB_CHECK(make_map_k64(&map_xt, xt, dt, rows, D, D));
  const int kblocks = static_cast<int>(ceil_div(rows, int64_t(kBK)));
  const int bst = b_stages(D);
  const size_t smem = std::max<size_t>(1024 + size_t(bst) * D * 128 + 2 * size_t(kStageBytes) + sizeof(Barriers),
                                       120 * 1024);
  const int tiles = static_cast<int>(ceil_div(int64_t(H) * K, int64_t(kBM)));
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  auto kernel = trop_param_grad_kernel<PT, K, MODE>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_param_grad"));
  const unsigned grid = static_cast<unsigned>(std::min(tiles, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_xt, win, run, mvals, code_scale, rows, H, D, kblocks, bst, tiles,
                                           absmax, static_cast<PT *>(out));
  return check_launch("trop_param_grad");
}

template <typename PT, int MODE>
int dispatch_param_grad(int K, const void *xt, int64_t rows, int D, int H, const uint8_t *win, const uint8_t *run,
                        const float *mvals, float code_scale, const uint32_t *absmax, void *out, cudaStream_t stream) {
  switch (K) {
    case 2: return launch_param_grad<PT, 2, MODE>(xt, rows, D, H, win, run, mvals, code_scale, absmax, out, stream);
    case 4: return launch_param_grad<PT, 4, MODE>(xt, rows, D, H, win, run, mvals, code_scale, absmax, out, stream);
    case 8: return launch_param_grad<PT, 8, MODE>(xt, rows, D, H, win, run, mvals, code_scale, absmax, out, stream);
    case 16: return launch_param_grad<PT, 16, MODE>(xt, rows, D, H, win, run, mvals, code_scale, absmax, out, stream);
    default: return launch_param_grad<PT, 32, MODE>(xt, rows, D, H, win, run, mvals, code_scale, absmax, out, stream);
  }
}

}  // namespace

bool param_grad_sm100_supported(int64_t rows, int64_t D, int64_t H, int64_t K, int pt) {
  const bool cells_ok = K == 2 || K == 4 || K == 8 || K == 16 || K == 32;
  return (pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16) && cells_ok && D % 64 == 0 && D >= 64 && D <= kMaxD &&
         rows >= kBK && rows % 8 == 0 && rows <= (int64_t(1) << 31) - 1024 && b_stages(static_cast<int>(D)) > 0;
}

// mode: 0 code grad eval, 1 code grad training (mvals = margins), 2 router grad (mvals = gm;
// then grad_b (param dtype [H, K]) may be given).
int trop_param_grad_sm100_impl(int mode, const void *xt, int64_t rows, int64_t D, int pt, int64_t H, int64_t K,
                               const void *win, const void *run, const float *mvals, float code_scale, void *out,
                               void *grad_b, const uint32_t *absmax, cudaStream_t stream) {
  TB_REQUIRE(param_grad_sm100_supported(rows, D, H, K, pt), TROPNN_B200_ERR_INVALID,
             "trop_param_grad_sm100: unsupported shape rows=%lld code_dim=%lld cells=%lld dtype=%s", (long long)rows,
             (long long)D, (long long)K, dtype_name(pt));
  TB_REQUIRE(mode >= 0 && mode <= 2, TROPNN_B200_ERR_INVALID, "trop_param_grad_sm100: bad mode %d", mode);
  TB_REQUIRE(xt && win && out && (mode == 0 || (run && mvals)), TROPNN_B200_ERR_INVALID,
             "trop_param_grad_sm100: null pointer");
  const auto *w = static_cast<const uint8_t *>(win);
  const auto *r = static_cast<const uint8_t *>(run);
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H), Ki = static_cast<int>(K);
  int status;
  if (pt == TROPNN_B200_F16) {
    status = mode == 0   ? dispatch_param_grad<__half, kCodeEval>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale, absmax, out, stream)
             : mode == 1 ? dispatch_param_grad<__half, kCodeTrain>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale, absmax, out, stream)
                         : dispatch_param_grad<__half, kRouter>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale, absmax, out, stream);
  } else {
    status = mode == 0 ? dispatch_param_grad<__nv_bfloat16, kCodeEval>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale, absmax, out,
                                                                        stream)
             : mode == 1 ? dispatch_param_grad<__nv_bfloat16, kCodeTrain>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale,
                                                                          absmax, out, stream)
                         : dispatch_param_grad<__nv_bfloat16, kRouter>(Ki, xt, rows, Di, Hi, w, r, mvals, code_scale,
                                                                       absmax, out, stream);
  }
  TB_CHECK(status);
  if (mode == 2 && grad_b != nullptr) {
    auto launch_bias = [&](auto pt_tag) -> int {
      using T = decltype(pt_tag);
      T *gb = static_cast<T *>(grad_b);
      switch (Ki) {
        case 2: return launch_bias_grad<T, 2>(w, r, mvals, rows, Hi, gb, stream);
        case 4: return launch_bias_grad<T, 4>(w, r, mvals, rows, Hi, gb, stream);
        case 8: return launch_bias_grad<T, 8>(w, r, mvals, rows, Hi, gb, stream);
        case 16: return launch_bias_grad<T, 16>(w, r, mvals, rows, Hi, gb, stream);
        default: return launch_bias_grad<T, 32>(w, r, mvals, rows, Hi, gb, stream);
      }
    };
    if (pt == TROPNN_B200_F16) return launch_bias(__half());
    return launch_bias(__nv_bfloat16());
  }
  return TROPNN_B200_OK;
}

int trop_code_transpose_impl(const void *code, int pt, int64_t H, int64_t K, int64_t D, void *code_t,
                             cudaStream_t stream);

int transpose_to_half_impl(const void *x, int xt_dtype, int64_t rows, int64_t cols, int pt, void *out,
                           const uint32_t *absmax, cudaStream_t stream) {
  TB_REQUIRE(pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "transpose_to_half: dtype %s unsupported", dtype_name(pt));
  TB_REQUIRE(xt_dtype == TROPNN_B200_F32 || xt_dtype == pt, TROPNN_B200_ERR_DTYPE,
             "transpose_to_half: input dtype %s must be f32 or %s", dtype_name(xt_dtype), dtype_name(pt));
  TB_REQUIRE(rows >= 0 && cols > 0 && cols <= (1 << 20), TROPNN_B200_ERR_INVALID, "transpose_to_half: bad shape");
  if (rows == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && out, TROPNN_B200_ERR_INVALID, "transpose_to_half: null pointer");
  // Half in, half out, no scale: a plain transpose of 2-byte values, which the parameter
  // transpose does with 4-byte moves on both sides (the kernels below load 2 bytes a thread).
  if (xt_dtype == pt && absmax == nullptr) return trop_code_transpose_impl(x, pt, rows, 1, cols, out, stream);
  const int c = static_cast<int>(cols);
  if (rows % 2 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0) {
    // 64-row tiles, pairs of output elements per 4-byte store.
    const dim3 grid2(static_cast<unsigned>(ceil_div(rows, int64_t(64))), static_cast<unsigned>(ceil_div(cols, int64_t(32))));
    TB_REQUIRE(grid2.y < 65536, TROPNN_B200_ERR_INVALID, "transpose_to_half: too many columns");
    if (pt == TROPNN_B200_F16) {
      if (xt_dtype == TROPNN_B200_F32)
        transpose_to_half_pairs_kernel<float, __half><<<grid2, 256, 0, stream>>>(
            static_cast<const float *>(x), static_cast<__half *>(out), rows, c, absmax);
      else
        transpose_to_half_pairs_kernel<__half, __half><<<grid2, 256, 0, stream>>>(
            static_cast<const __half *>(x), static_cast<__half *>(out), rows, c, absmax);
    } else {
      if (xt_dtype == TROPNN_B200_F32)
        transpose_to_half_pairs_kernel<float, __nv_bfloat16><<<grid2, 256, 0, stream>>>(
            static_cast<const float *>(x), static_cast<__nv_bfloat16 *>(out), rows, c, absmax);
      else
        transpose_to_half_pairs_kernel<__nv_bfloat16, __nv_bfloat16><<<grid2, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16 *>(x), static_cast<__nv_bfloat16 *>(out), rows, c, absmax);
    }
    return check_launch("transpose_to_half");
  }
  const dim3 grid(static_cast<unsigned>(ceil_div(rows, int64_t(32))), static_cast<unsigned>(ceil_div(cols, int64_t(32))));
  if (pt == TROPNN_B200_F16) {
    if (xt_dtype == TROPNN_B200_F32)
      transpose_to_half_kernel<float, __half><<<grid, 256, 0, stream>>>(static_cast<const float *>(x),
                                                                      static_cast<__half *>(out), rows, c, absmax);
    else
      transpose_to_half_kernel<__half, __half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(x),
                                                                       static_cast<__half *>(out), rows, c, absmax);
  } else {
    if (xt_dtype == TROPNN_B200_F32)
      transpose_to_half_kernel<float, __nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const float *>(x), static_cast<__nv_bfloat16 *>(out), rows, c, absmax);
    else
      transpose_to_half_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16 *>(x), static_cast<__nv_bfloat16 *>(out), rows, c, absmax);
  }
  return check_launch("transpose_to_half");
}

int read_param_grad_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_param_grad_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_param_grad_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200
