// TropLinear selected-code sum on the sm_100a tensor cores. With half-precision codes the
// gather-sum of layers/tropical.py:131-138 is a GEMM with a one-hot left operand:
//   hidden[n,:] = latent[n,:] + code_scale * sum_{h,k} P[n,(h,k)] * code[h,k,:]
//   P[n,(h,k)] = 1 at the winner cell (eval), or 1-U(m) at the winner and U(m) at the
//   runner-up (training, the min-face mix of routing.py:13-15, U(m) = 0.5/(1+|m|)).
// A 128-row block of items then streams the code table once through the tensor cores
// (tcgen05, f32 accumulation in TMEM) instead of gathering heads x code_dim values per
// item: the gather's L2 traffic shrinks by a factor of 128 / cells-per-k-block.
//
// Eval is exact up to f32 summation order: P is 0/1 and every product is a code value.
// In training the two mixing weights are rounded to the parameter dtype (relative error
// 2^-11 for f16, 2^-8 for bf16), far inside the 2e-2 tolerance of half-precision layers.
//
// Operands: B = code^T [code_dim, heads*cells] (K-major, built by trop_code_transpose),
// loaded by TMA in 64-wide k blocks; A = the one-hot block, built in registers from the
// u8 routes and written straight into TMEM (tcgen05.st), so it never touches shared
// memory: the MMA reads A from TMEM and B from shared memory.
//
// CTA = 14 warps, persistent over row blocks rb = blockIdx.x + i * gridDim.x; each CTA
// walks the k blocks from its own starting point (rotated), so that the CTAs spread
// their code-table reads over L2:
//   warp 0      TMA producer of the code^T k blocks (3-8 stage ring, D x 128 B each).
//   warp 1      allocates all 512 TMEM columns (accumulator [0, D), one-hot ring
//               [256, 512): 8 slots of 32 columns); lane 0 issues the MMAs (M=128,
//               N=code_dim, K=16, A from TMEM) and commits them to mbarriers.
//   warps 2-9   build the one-hot k blocks: one thread per row, 32 packed f16/bf16 pairs
//               per k block, stored with tcgen05.st into the thread's TMEM lane; two
//               warps per lane quarter take alternate k blocks.
//   warps 10-13 epilogue: hidden = latent + code_scale * acc for the thread's row.
// All waits are bounded (sm100.cuh); waits by whole warps of builders and epilogue use
// mbarrier suspend hints instead of spinning, which kept the TMA/MMA pipeline at rate.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;                 // rows per row block (MMA M, TMEM lanes)
constexpr int kBK = 64;                  // (head, cell) entries per k block
constexpr int kMaxD = 256;               // MMA N = code_dim
constexpr int kMaxBStages = 8;
constexpr int kMinBStages = 3;
constexpr int kAStages = 8;              // one-hot ring slots in TMEM
constexpr int kBuildWarps = 8;           // two per TMEM lane quarter (even / odd k items)
constexpr int kEpiWarps = 4;             // one per TMEM lane quarter
constexpr int kThreads = 32 * (2 + kBuildWarps + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAColBase = 256;      // one-hot ring after the (<= 256-column) accumulator
constexpr size_t kSmemLimit = 227 * 1024;
constexpr uint32_t kSleepHintNs = 1000000u;

// Library-wide device error word of this kernel: nonzero after a bounded wait gave up.
// What the one-hot left operand holds per (row, head): 1 at the winner (eval); 1-U(m) at
// the winner and U(m) at the runner-up (training, min-face mix); +gm at the winner and -gm
// at the runner-up (backward router term of grad_latent, gm read from `margins`).
enum OneHotMode { kOneHotEval = 0, kOneHotMinFace = 1, kOneHotSigned = 2 };

__device__ int g_hidden_error = 0;

struct Barriers {
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
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_hidden_error);
}

// Bounded wait that suspends the thread between polls (mbarrier suspend-time hint).
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
      atomicExch(&g_hidden_error, 1);
      return false;
    }
  }
}

// Warp-collective form: lane 0 waits, the warp follows its verdict (converged after).
__device__ __forceinline__ bool warp_wait_sleep(uint64_t *bar, uint32_t parity, Barriers *bs, int lane) {
  int ok = 1;
  if (lane == 0) ok = wait_bar_sleep(bar, parity, bs) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

template <typename PT>
struct HalfBits;
template <>
struct HalfBits<__half> {
  static constexpr uint32_t kOne = 0x3C00u;
  static constexpr int kFormat = 0;
  __device__ static uint32_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};
template <>
struct HalfBits<__nv_bfloat16> {
  static constexpr uint32_t kOne = 0x3F80u;
  static constexpr int kFormat = 1;
  __device__ static uint32_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};

// The f32 value of half-precision bits.
template <typename PT>
__device__ __forceinline__ float half_value(uint32_t bits) {
  if constexpr (std::is_same<PT, __half>::value)
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
  else
    return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(bits)));
}

// 32 latent values of one row as f32.
template <typename LT>
__device__ __forceinline__ void load_row32(const LT *__restrict__ p, float (&out)[32]) {
  if constexpr (std::is_same<LT, float>::value) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(p + i));
      out[i] = q.x;
      out[i + 1] = q.y;
      out[i + 2] = q.z;
      out[i + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      float t[8];
      VecLoad<LT, 8>::load(p + i, t);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[i + e] = t[e];
    }
  }
}

// N consecutive route bytes / margins by vector loads (N a power of two; p aligned to N
// bytes / N floats, at most 16 bytes per load).
template <int N>
__device__ __forceinline__ void load_vec(const uint8_t *p, uint8_t (&o)[N]) {
  if constexpr (N >= 16) {
#pragma unroll
    for (int i = 0; i < N / 16; ++i) *reinterpret_cast<uint4 *>(o + 16 * i) = __ldg(reinterpret_cast<const uint4 *>(p) + i);
  } else if constexpr (N == 8) {
    *reinterpret_cast<uint2 *>(o) = __ldg(reinterpret_cast<const uint2 *>(p));
  } else if constexpr (N == 4) {
    *reinterpret_cast<uint32_t *>(o) = __ldg(reinterpret_cast<const uint32_t *>(p));
  } else {
    *reinterpret_cast<uint16_t *>(o) = __ldg(reinterpret_cast<const unsigned short *>(p));
  }
}
template <int N>
__device__ __forceinline__ void load_vec(const float *p, float (&o)[N]) {
  if constexpr (N >= 4) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 q = __ldg(reinterpret_cast<const float4 *>(p) + i);
      o[4 * i] = q.x, o[4 * i + 1] = q.y, o[4 * i + 2] = q.z, o[4 * i + 3] = q.w;
    }
  } else {
    const float2 q = __ldg(reinterpret_cast<const float2 *>(p));
    o[0] = q.x, o[1] = q.y;
  }
}

template <typename PT, typename LT, int K, int MODE>
__global__ void __launch_bounds__(kThreads, 1) trop_hidden_onehot_kernel(
    const __grid_constant__ CUtensorMap map_ct, const LT *__restrict__ latent, const uint8_t *__restrict__ winner,
    const uint8_t *__restrict__ runner, const float *__restrict__ margins, float code_scale, int64_t rows, int H,
    int D, int kblocks, int bstages, int64_t row_blocks, const uint32_t *__restrict__ absmax, int vec_routes,
    float *__restrict__ hidden, PT *__restrict__ hidden_split, int splits, float4 *__restrict__ partial) {
  static_assert(K >= 2 && K <= kBK && K % 2 == 0, "cells must be even and at most 64");
  constexpr int kHeadsPerBlock = kBK / K;
  // Signed mode (router term of grad_z): the gm weights are scaled by the power-of-two gradient
  // scale of *absmax before their conversion to PT, the product scaled back in the epilogue.
  const float gscale = MODE == kOneHotSigned ? grad_scale_of(absmax) : 1.f;
  const float out_scale = __fmul_rn(code_scale, pow2_inverse(gscale));
  constexpr uint32_t kOne = HalfBits<PT>::kOne;
  const uint32_t idesc = umma_idesc_f16(HalfBits<PT>::kFormat, kBM, D);
  const int b_stage_bytes = D * 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *b_smem = smem;  // bstages x [D rows x 128 B], K-major, 128-byte swizzle
  Barriers *bs = reinterpret_cast<Barriers *>(b_smem + bstages * b_stage_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Every CTA walks the code table from its own starting k block (all CTAs reading the
  // same k block at once made its L2 lines the bottleneck); position kb of the walk is
  // k block kb + rot (mod kblocks).
  // With the contraction split into `splits` slices of kps k blocks, unit u = (row block
  // u / splits, slice u % splits) walks its slice from a rotated start the same way.
  const int kps = kblocks / splits;
  const int64_t units = row_blocks * splits;
  const int rot = static_cast<int>(int64_t(blockIdx.x) * kps / gridDim.x);
  auto kblock_at = [&](int64_t u, int kb) {
    const int ks = static_cast<int>(u % splits);
    return ks * kps + (kb + rot < kps ? kb + rot : kb + rot - kps);
  };

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
      // ---------------- TMA producer: code^T k blocks ----------------
      prefetch_map(&map_ct);
      uint32_t issued[kMaxBStages];
      for (int s = 0; s < kMaxBStages; ++s) issued[s] = 0;
      bool ok = true;
      int it = 0;
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
        for (int kb = 0; kb < kps; ++kb, ++it) {
          const int s = it % bstages;
          const uint32_t phase = uint32_t(it / bstages) & 1u;
          if (!wait_bar(&bs->b_empty[s], phase ^ 1u, bs)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bs->b_full[s], uint32_t(b_stage_bytes));
          tma_load_2d(b_smem + s * b_stage_bytes, &map_ct, &bs->b_full[s], kblock_at(u, kb) * kBK, 0);
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
      for (int64_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
        if (!wait_bar(&bs->acc_empty, (i & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        for (int kb = 0; kb < kps; ++kb, ++bit, ++ait) {
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
      // All MMAs issued by this thread must finish before TMEM is freed.
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else if (warp < 2 + kBuildWarps) {
    // ---------------- one-hot builders ----------------
    // Warps 2-5 build the even k items of the CTA's sequence (ait = i * kps + kb over its
    // units i), warps 6-9 the odd ones; each warp its TMEM lane quarter.
    const int quarter = warp & 3;
    const int parity = (warp - 2) >> 2;
    const uint32_t lane_base = tmem_base + (uint32_t(quarter * 32) << 16) + kAColBase;
    bool ok = true;
    // The route bytes (and margins) of the thread's row for one k item: the next item's are
    // fetched while this one is built, with vector loads of the item's consecutive heads.
    struct Raw {
      uint8_t w[kHeadsPerBlock];
      uint8_t r[kHeadsPerBlock];
      float m[kHeadsPerBlock];
    };
    auto fetch = [&](int a, Raw &raw) {
      const int64_t ii = a / kps;
      const int kb = static_cast<int>(a - ii * kps);
      const int64_t u = blockIdx.x + ii * gridDim.x;
      if (u >= units) return;
      const int64_t row = (u / splits) * kBM + quarter * 32 + lane;
      const int h0 = kblock_at(u, kb) * kHeadsPerBlock;
      const int valid = row < rows ? max(0, min(kHeadsPerBlock, H - h0)) : 0;
      const int64_t o = (row < rows ? row : 0) * H + h0;
      if (vec_routes && valid == kHeadsPerBlock) {
        load_vec<kHeadsPerBlock>(winner + o, raw.w);
        if constexpr (MODE != kOneHotEval) {
          load_vec<kHeadsPerBlock>(runner + o, raw.r);
          load_vec<kHeadsPerBlock>(margins + o, raw.m);
        }
      } else {
#pragma unroll
        for (int hh = 0; hh < kHeadsPerBlock; ++hh) {
          raw.w[hh] = hh < valid ? __ldg(winner + o + hh) : uint8_t(0xFF);
          if constexpr (MODE != kOneHotEval) {
            raw.r[hh] = hh < valid ? __ldg(runner + o + hh) : uint8_t(0xFF);
            raw.m[hh] = hh < valid ? __ldg(margins + o + hh) : 0.f;
          }
        }
      }
    };
    // Prefetch only while both items fit the registers (up to 8 heads per item: cells >= 8).
    constexpr bool kPrefetch = kHeadsPerBlock <= 8;
    Raw nxt;
    if constexpr (kPrefetch) fetch(parity, nxt);
    for (int ait = parity;; ait += 2) {
      const int64_t i = ait / kps;
      const int64_t u = blockIdx.x + i * gridDim.x;
      if (u >= units || !ok) break;
      Raw cur;
      if constexpr (kPrefetch) {
        cur = nxt;
        fetch(ait + 2, nxt);
      } else {
        fetch(ait, cur);
      }
      {
        const int sa = ait % kAStages;
        uint32_t wc[kHeadsPerBlock], rc[kHeadsPerBlock], vw[kHeadsPerBlock], vr[kHeadsPerBlock];
#pragma unroll
        for (int hh = 0; hh < kHeadsPerBlock; ++hh) {
          wc[hh] = cur.w[hh];
          rc[hh] = 0xFFu;
          vw[hh] = kOne;
          vr[hh] = 0u;
          if (wc[hh] != 0xFFu) {
            if constexpr (MODE == kOneHotMinFace) {
              rc[hh] = cur.r[hh];
              const float alpha = __fdiv_rn(0.5f, __fadd_rn(1.f, fabsf(cur.m[hh])));
              vw[hh] = HalfBits<PT>::bits(__fsub_rn(1.f, alpha));
              vr[hh] = HalfBits<PT>::bits(alpha);
            } else if constexpr (MODE == kOneHotSigned) {
              rc[hh] = cur.r[hh];
              const float gm = __fmul_rn(cur.m[hh], gscale);
              vw[hh] = HalfBits<PT>::bits(gm);
              vr[hh] = HalfBits<PT>::bits(-gm);
            }
          }
        }
        if (!warp_wait_sleep(&bs->a_empty[sa], (uint32_t(ait / kAStages) & 1u) ^ 1u, bs, lane)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        // Column j of the k block holds entries 2j (low half) and 2j+1 (high half), entry
        // hh * K + k being head hh's cell k. Head hh's routed cells land in words
        // hh * K/2 + (cell >> 1), in the half given by cell & 1: each word is a compare and a
        // select against the (at most two) routed word indices, all in registers.
        uint32_t reg[32];
#pragma unroll
        for (int hh = 0; hh < kHeadsPerBlock; ++hh) {
          const uint32_t qa = wc[hh] >> 1;
          const uint32_t a = vw[hh] << ((wc[hh] & 1u) << 4);
#pragma unroll
          for (int p = 0; p < K / 2; ++p) {
            uint32_t v = qa == uint32_t(p) ? a : 0u;
            if constexpr (MODE != kOneHotEval) {
              const uint32_t qb = rc[hh] != wc[hh] ? rc[hh] >> 1 : 0xFFu;
              const uint32_t b = vr[hh] << ((rc[hh] & 1u) << 4);
              v |= qb == uint32_t(p) ? b : 0u;
            }
            reg[hh * (K / 2) + p] = v;
          }
        }
        tmem_st32(lane_base + uint32_t(sa * 32), reg);
        tmem_wait_st();
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bs->a_full[sa]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem_base + (uint32_t(quarter * 32) << 16);
    uint32_t i = 0;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x, ++i) {
      const int64_t row = (u / splits) * kBM + quarter * 32 + lane;
      if (!warp_wait_sleep(&bs->acc_full, i & 1u, bs, lane)) break;
      tmem_fence_after();
      for (int c = 0; c < D; c += 32) {
        float acc[32];
        tmem_ld32(lane_base + uint32_t(c), acc);
        float lat[32];
        if (splits == 1 && row < rows) load_row32<LT>(latent + row * D + c, lat);
        tmem_wait_ld();
        reg_fence(acc);
        if (c + 32 >= D) {
          // The accumulator is in registers: the next unit may start.
          tmem_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bs->acc_empty);
        }
        if (splits > 1) {
          // Slice partial for slice_reduce: [unit][column / 4][row], row index fastest, with the
          // signed mode's power-of-two gradient scale undone (exact; slice_reduce applies
          // code_scale and adds the latent).
          const float unscale = pow2_inverse(gscale);
          float4 *p = partial + (size_t(u) * (D / 4) + c / 4) * kBM + quarter * 32 + lane;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            p[size_t(e) * kBM] = make_float4(__fmul_rn(acc[4 * e], unscale), __fmul_rn(acc[4 * e + 1], unscale),
                                             __fmul_rn(acc[4 * e + 2], unscale), __fmul_rn(acc[4 * e + 3], unscale));
        } else if (row < rows) {
          float h[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) h[e] = __fadd_rn(lat[e], __fmul_rn(acc[e], out_scale));
          float *out = hidden + row * D + c;
#pragma unroll
          for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4 *>(out + e) = make_float4(h[e], h[e + 1], h[e + 2], h[e + 3]);
          if (hidden_split != nullptr) {
            // The output map's operand [hi | lo] of the row (hi = half(h), lo = half(h - hi)),
            // written here instead of by a separate split pass over hidden.
            PT *hi_row = hidden_split + row * (2 * int64_t(D)) + c;
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint32_t hb[4], lb[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t h0 = HalfBits<PT>::bits(h[e + 2 * k]), h1 = HalfBits<PT>::bits(h[e + 2 * k + 1]);
                hb[k] = h0 | (h1 << 16);
                lb[k] = HalfBits<PT>::bits(__fsub_rn(h[e + 2 * k], half_value<PT>(h0))) |
                        (HalfBits<PT>::bits(__fsub_rn(h[e + 2 * k + 1], half_value<PT>(h1))) << 16);
              }
              *reinterpret_cast<uint4 *>(hi_row + e) = make_uint4(hb[0], hb[1], hb[2], hb[3]);
              *reinterpret_cast<uint4 *>(hi_row + D + e) = make_uint4(lb[0], lb[1], lb[2], lb[3]);
            }
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

// code [rows_in, cols_in] -> code_t [cols_in, rows_in] (32 x 32 tiles through shared memory).
template <typename PT>
__global__ void __launch_bounds__(256) transpose_kernel(const PT *__restrict__ in, PT *__restrict__ out,
                                                        int64_t rows_in, int cols_in) {
  __shared__ PT tile[32][33];
  const int64_t r0 = int64_t(blockIdx.x) * 32;
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int j = ty; j < 32; j += 8)
    if (r0 + j < rows_in && c0 + tx < cols_in) tile[j][tx] = in[(r0 + j) * cols_in + c0 + tx];
  __syncthreads();
  for (int j = ty; j < 32; j += 8)
    if (c0 + j < cols_in && r0 + tx < rows_in) out[int64_t(c0 + j) * rows_in + r0 + tx] = tile[tx][j];
}

// The same transpose for even sizes, 64 x 64 tiles moved as 32-bit pairs: a thread reads two
// consecutive input rows' pair (r, c..c+1), (r+1, c..c+1), regroups them into the pairs
// (c, r..r+1) and (c+1, r..r+1) with byte permutes, and the two 32 x 33-word shared tiles give
// 128-byte coalesced reads and writes without bank conflicts.
__global__ void __launch_bounds__(256) transpose_pairs_kernel(const uint32_t *__restrict__ in, uint32_t *__restrict__ out,
                                                              int64_t rows_in, int cols_in) {
  __shared__ uint32_t lo_t[32][33], hi_t[32][33];
  const int64_t r0 = int64_t(blockIdx.x) * 64;  // input rows (output columns)
  const int c0 = blockIdx.y * 64;              // input columns (output rows)
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t in_words = cols_in / 2, out_words = rows_in / 2;
  for (int rr = ty; rr < 32; rr += 8) {
    const int64_t r = r0 + 2 * rr;
    const int c = c0 + 2 * tx;
    uint32_t a = 0u, b = 0u;
    if (c < cols_in) {
      if (r < rows_in) a = in[r * in_words + c / 2];
      if (r + 1 < rows_in) b = in[(r + 1) * in_words + c / 2];
    }
    lo_t[rr][tx] = __byte_perm(a, b, 0x5410);  // (a.lo, b.lo): column c, rows r, r + 1
    hi_t[rr][tx] = __byte_perm(a, b, 0x7632);  // (a.hi, b.hi): column c + 1
  }
  __syncthreads();
  for (int cc = ty; cc < 32; cc += 8) {
    const int c = c0 + 2 * cc;
    const int64_t r = r0 + 2 * tx;
    if (r < rows_in) {
      if (c < cols_in) out[int64_t(c) * out_words + r / 2] = lo_t[tx][cc];
      if (c + 1 < cols_in) out[int64_t(c + 1) * out_words + r / 2] = hi_t[tx][cc];
    }
  }
}

int b_stages(int D) {
  const size_t stage = size_t(D) * 128;
  const size_t room = kSmemLimit - 1024 - sizeof(Barriers);
  const int s = static_cast<int>(std::min<size_t>(kMaxBStages, room / stage));
  return s >= kMinBStages ? s : 0;
}

constexpr int kTargetUnits = 148;  // B200 SMs
constexpr int kMaxSplits = 16;
constexpr int kMinKBlocksPerSplit = 8;

// Slices of the (head, cell) contraction: 1 with enough row blocks for the SMs, else the
// largest divisor of the k-block count up to the SMs' share of the row blocks (>= 8 k blocks
// a slice).
int onehot_splits(int64_t rows, int64_t hk) {
  const int64_t row_blocks = ceil_div(rows, int64_t(kBM));
  const int kblocks = static_cast<int>(ceil_div(hk, int64_t(kBK)));
  if (row_blocks * 4 >= int64_t(kTargetUnits) * 3) return 1;
  const int want = static_cast<int>(std::min<int64_t>(kMaxSplits, ceil_div(kTargetUnits, row_blocks)));
  for (int s = want; s > 1; --s)
    if (kblocks % s == 0 && kblocks / s >= kMinKBlocksPerSplit) return s;
  return 1;
}

size_t onehot_workspace(int64_t rows, int64_t D, int64_t hk) {
  const int splits = onehot_splits(rows, hk);
  if (splits == 1) return 0;
  return WorkspaceCarver::align(size_t(ceil_div(rows, int64_t(kBM))) * splits * size_t(D) * kBM * sizeof(float));
}

template <typename PT, typename LT, int K>
int launch_onehot(const void *latent, int64_t rows, int D, const void *code_t, int H, const uint8_t *win,
                  const uint8_t *run, const float *m, float code_scale, int mode, const uint32_t *absmax, float *hidden,
                  void *hidden_split, void *ws, size_t ws_bytes, cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int64_t hk = int64_t(H) * K;
  CUtensorMap map_ct;
  TB_CHECK(make_map_k64(&map_ct, code_t, dt, hk, D, D));
  const int kblocks = static_cast<int>(ceil_div(hk, int64_t(kBK)));
  const int bst = b_stages(D);
  // At least half of the SM's shared memory, so that no second CTA shares the SM: each
  // CTA allocates all 512 TMEM columns.
  const size_t smem = std::max<size_t>(1024 + size_t(bst) * D * 128 + sizeof(Barriers), 120 * 1024);
  const int64_t row_blocks = ceil_div(rows, int64_t(kBM));
  // Few row blocks: split the contraction when the caller gave room for the slice partials.
  int splits = onehot_splits(rows, hk);
  float4 *partial = nullptr;
  if (splits > 1) {
    WorkspaceCarver wc(ws, ws_bytes);
    partial = wc.take<float4>(size_t(row_blocks) * splits * size_t(D / 4) * kBM);
    if (partial == nullptr) splits = 1;
  }
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(row_blocks * splits, sms));
  // Vector loads of an item's 64 / K consecutive heads: whole vectors inside each row and
  // 16-byte aligned route / margin arrays.
  auto al16 = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int vec_routes = (H % (kBK / K) == 0 && al16(win) && al16(run) && al16(m)) ? 1 : 0;
  auto kernel = mode == kOneHotSigned   ? trop_hidden_onehot_kernel<PT, LT, K, kOneHotSigned>
                : mode == kOneHotMinFace ? trop_hidden_onehot_kernel<PT, LT, K, kOneHotMinFace>
                                         : trop_hidden_onehot_kernel<PT, LT, K, kOneHotEval>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_hidden_sm100"));
  kernel<<<grid, kThreads, smem, stream>>>(map_ct, static_cast<const LT *>(latent), win, run, m, code_scale, rows, H, D,
                                           kblocks, bst, row_blocks, absmax, vec_routes, hidden,
                                           static_cast<PT *>(hidden_split), splits, partial);
  TB_CHECK(check_launch("trop_hidden_sm100"));
  if (splits == 1) return TROPNN_B200_OK;
  // hidden = latent + code_scale * (slices summed in slice order), and its [hi | lo] split.
  return slice_reduce_impl(kReduceHidden, partial, splits, 1, D, rows, D, hidden, TROPNN_B200_F32, D, nullptr, latent,
                           std::is_same<LT, float>::value ? TROPNN_B200_F32
                           : std::is_same<LT, __half>::value ? TROPNN_B200_F16 : TROPNN_B200_BF16,
                           code_scale, stream, hidden_split,
                           std::is_same<PT, __half>::value ? TROPNN_B200_F16 : TROPNN_B200_BF16);
}

template <typename PT, typename LT>
int dispatch_onehot(int K, const void *latent, int64_t rows, int D, const void *code_t, int H, const uint8_t *win,
                    const uint8_t *run, const float *m, float code_scale, int mode, const uint32_t *absmax, float *hidden,
                    void *hs, void *ws, size_t wsb, cudaStream_t stream) {
  switch (K) {
    case 2: return launch_onehot<PT, LT, 2>(latent, rows, D, code_t, H, win, run, m, code_scale, mode, absmax, hidden, hs,
                                        ws, wsb, stream);
    case 4: return launch_onehot<PT, LT, 4>(latent, rows, D, code_t, H, win, run, m, code_scale, mode, absmax, hidden, hs,
                                        ws, wsb, stream);
    case 8: return launch_onehot<PT, LT, 8>(latent, rows, D, code_t, H, win, run, m, code_scale, mode, absmax, hidden, hs,
                                        ws, wsb, stream);
    case 16:
      return launch_onehot<PT, LT, 16>(latent, rows, D, code_t, H, win, run, m, code_scale, mode, absmax, hidden, hs,
                                        ws, wsb, stream);
    default:
      return launch_onehot<PT, LT, 32>(latent, rows, D, code_t, H, win, run, m, code_scale, mode, absmax, hidden, hs,
                                        ws, wsb, stream);
  }
}

}  // namespace

bool hidden_sm100_supported(int64_t items, int64_t D, int64_t H, int64_t K, int pt, int zt, int it, const void *latent,
                            const void *code_t, const void *hidden) {
  const bool cells_ok = K == 2 || K == 4 || K == 8 || K == 16 || K == 32;
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return code_t != nullptr && (pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16) && (zt == pt || zt == TROPNN_B200_F32) &&
         it == TROPNN_B200_U8 && cells_ok && D % 64 == 0 && D >= 64 && D <= kMaxD && (H * K) % 8 == 0 &&
         items >= kBM && b_stages(static_cast<int>(D)) > 0 && al16(latent) && al16(code_t) && al16(hidden);
}

size_t trop_hidden_sm100_workspace(int64_t items, int64_t D, int64_t H, int64_t K) {
  if (items < 0 || D < 1 || H < 1 || K < 1) return 0;
  return onehot_workspace(items, D, H * K);
}

int trop_hidden_sm100_impl(const void *latent, int zt, int64_t items, int64_t D, const void *code_t, int pt,
                           int64_t H, int64_t K, const void *win, const void *run, const float *m, float code_scale,
                           int mode, const uint32_t *absmax, float *hidden, void *hidden_split, void *ws, size_t wsb,
                           cudaStream_t stream) {
  TB_REQUIRE(hidden_split == nullptr || reinterpret_cast<uintptr_t>(hidden_split) % 16 == 0, TROPNN_B200_ERR_INVALID,
             "trop_hidden_sm100: hidden_split must be 16-byte aligned");
  TB_REQUIRE(hidden_sm100_supported(items, D, H, K, pt, zt, TROPNN_B200_U8, latent, code_t, hidden),
             TROPNN_B200_ERR_INVALID, "trop_hidden_sm100: unsupported shape, dtype or alignment");
  TB_REQUIRE(mode >= kOneHotEval && mode <= kOneHotSigned, TROPNN_B200_ERR_INVALID, "trop_hidden_sm100: bad mode");
  TB_REQUIRE(win && (mode == kOneHotEval || (run && m)), TROPNN_B200_ERR_INVALID, "trop_hidden_sm100: null pointer");
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H), Ki = static_cast<int>(K);
  const auto *w = static_cast<const uint8_t *>(win);
  const auto *r = static_cast<const uint8_t *>(run);
  if (pt == TROPNN_B200_F16) {
    if (zt == TROPNN_B200_F32)
      return dispatch_onehot<__half, float>(Ki, latent, items, Di, code_t, Hi, w, r, m, code_scale, mode, absmax, hidden,
                                            hidden_split, ws, wsb, stream);
    return dispatch_onehot<__half, __half>(Ki, latent, items, Di, code_t, Hi, w, r, m, code_scale, mode, absmax, hidden,
                                           hidden_split, ws, wsb, stream);
  }
  if (zt == TROPNN_B200_F32)
    return dispatch_onehot<__nv_bfloat16, float>(Ki, latent, items, Di, code_t, Hi, w, r, m, code_scale, mode, absmax,
                                                 hidden, hidden_split, ws, wsb, stream);
  return dispatch_onehot<__nv_bfloat16, __nv_bfloat16>(Ki, latent, items, Di, code_t, Hi, w, r, m, code_scale, mode,
                                                       absmax, hidden, hidden_split, ws, wsb, stream);
}

int trop_code_transpose_impl(const void *code, int pt, int64_t H, int64_t K, int64_t D, void *code_t,
                             cudaStream_t stream) {
  TB_REQUIRE(pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "trop_code_transpose: param dtype %s unsupported (f16/bf16 only)", dtype_name(pt));
  TB_REQUIRE(H > 0 && K > 0 && D > 0 && D <= (1 << 20) && H * K < (int64_t(1) << 36), TROPNN_B200_ERR_INVALID,
             "trop_code_transpose: bad shape heads=%lld cells=%lld code_dim=%lld", (long long)H, (long long)K,
             (long long)D);
  TB_REQUIRE(code && code_t, TROPNN_B200_ERR_INVALID, "trop_code_transpose: null pointer");
  const int64_t rows_in = H * K;
  const bool pairs = rows_in % 2 == 0 && D % 2 == 0 && reinterpret_cast<uintptr_t>(code) % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(code_t) % 4 == 0;
  if (pairs) {
    const dim3 grid2(static_cast<unsigned>(ceil_div(rows_in, int64_t(64))), static_cast<unsigned>(ceil_div(D, int64_t(64))));
    TB_REQUIRE(grid2.y < 65536, TROPNN_B200_ERR_INVALID, "trop_code_transpose: code_dim too large");
    transpose_pairs_kernel<<<grid2, 256, 0, stream>>>(static_cast<const uint32_t *>(code),
                                                      static_cast<uint32_t *>(code_t), rows_in, static_cast<int>(D));
    return check_launch("trop_code_transpose");
  }
  const dim3 grid(static_cast<unsigned>(ceil_div(rows_in, int64_t(32))), static_cast<unsigned>(ceil_div(D, int64_t(32))));
  if (pt == TROPNN_B200_F16)
    transpose_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(code), static_cast<__half *>(code_t),
                                                       rows_in, static_cast<int>(D));
  else
    transpose_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(code),
                                                              static_cast<__nv_bfloat16 *>(code_t), rows_in,
                                                              static_cast<int>(D));
  return check_launch("trop_code_transpose");
}

int read_hidden_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_hidden_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_hidden_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200
