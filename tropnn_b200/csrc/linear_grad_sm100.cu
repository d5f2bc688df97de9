// Gradients of TropLinear's f32 output map out = hidden W^T + b (layers/tropical.py:140-146:
// the reference upcasts the half-precision weight and bias and runs F.linear in f32, so its
// backward is three f32 products) on the sm_100a tensor cores:
//   grad_hidden[n, i] = sum_o g[n, o] W[o, i]            (DGRAD)
//   grad_W[o, i]      = sum_n g[n, o] hidden[n, i]       (WGRAD, rounded to W's dtype)
//   grad_b[o]         = sum_n g[n, o]                    (WGRAD's converter warps, f32)
//
// Precision: tcgen05 kind::tf32 multiplies 11-bit-significand operands with f32 accumulation.
// Every f32 operand x is split as x = big + small, big = tf32(x), small = tf32(x - big), and
// the products are formed as big*big' + small*big' + big*small' (the small*small' term is below
// f32 rounding), which keeps f32 range and products exact to ~2^-22. W (f16/bf16) is exact in
// tf32, so DGRAD needs two products per k step; WGRAD needs three. The tensor-core accumulator
// loses about half an ulp per addition (the error grows linearly with the contraction length),
// so big*big' and the cross terms accumulate in separate TMEM accumulators, summed in the
// epilogue: about 1e-5 of the largest output at a 4096-long contraction (an f32 FMA GEMM:
// 2.4e-6), far inside the half-precision layer tolerance.
//
// g, the largest operand ([rows, out] f32), is read once per kernel by TMA and split in shared
// memory by 4 converter warps (big written in place, small to a second buffer, elementwise).
// hidden is split ahead of WGRAD (tf32_split); W is widened to f32 ahead of DGRAD.
//
// DGRAD: one CTA per 128-row block; A = g (K-major, 128 x 32 per stage), B = W as f32 viewed
// MN-major (32 x in_features per stage, 32-byte-atom swizzle); the accumulator (128 x in_features f32) leaves TMEM
// through 32 x 32 swizzled shared tiles and TMA stores.
// WGRAD: one cluster of kSlices CTAs per 128-row block of W; CTA y of the cluster contracts row
// slice y (A = g^T MN-major 128 x 16 per stage, B = hidden^T MN-major big and small), leaves
// its partial tile in shared memory, and the cluster sums the kSlices partials in slice order
// through distributed shared memory (each CTA finishing 128 / kSlices rows of W).
//
// CTA = 6 warps: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer (one thread), warps 2-5
// converters, then epilogue (warp w reads TMEM lanes 32 (w % 4) ...). All waits are bounded.
#include <cuda.h>

#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kMaxN = 256;
constexpr int kConvWarps = 4;
constexpr int kThreads = 32 * (2 + kConvWarps);
constexpr int kMaxStages = 8;
constexpr int kMinStages = 2;
constexpr int kSlices = 4;
constexpr size_t kSmemLimit = 227 * 1024;

enum GradKind { kDgrad = 0, kWgrad = 1 };

// Contraction rows per pipeline stage: one 128-byte K row (DGRAD, K-major A) or 16 rows of
// the MN-major strips (WGRAD).
constexpr int stage_k(int kind) { return kind == kDgrad ? 32 : 16; }

__device__ int g_linear_grad_error = 0;

struct Barriers {
  uint64_t full[kMaxStages];
  uint64_t conv[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full;
  uint32_t tmem_base;
  int abort;
  int epi_go;
};

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Barriers *bs) {
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_linear_grad_error);
}

constexpr uint32_t a_tile_bytes(int kind) { return uint32_t(kBM) * stage_k(kind) * 4; }
inline uint32_t b_tile_bytes(int kind, int n) { return uint32_t(n) * stage_k(kind) * 4; }
inline uint32_t stage_bytes(int kind, int n) {
  return 2 * a_tile_bytes(kind) + (kind == kWgrad ? 2 : 1) * b_tile_bytes(kind, n);
}
// Shared memory after the stage ring: WGRAD's column-sum partials [kConvWarps][kBM] and the
// CTA's per-row bias partial [kBM], then the barriers.
constexpr size_t kTailBytes = sizeof(float) * (kConvWarps + 1) * kBM;

int grad_stages(int kind, int n) {
  const size_t fixed = 1024 + kTailBytes + sizeof(Barriers);
  const size_t per = stage_bytes(kind, n);
  int s = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / per));
  // WGRAD's partial tile (128 x n f32) reuses the ring.
  if (kind == kWgrad && size_t(s) * per < size_t(kBM) * n * 4) return 0;
  return s >= kMinStages ? s : 0;
}

// Dynamic shared memory of a launch; at least kOneCtaSmem, so that one CTA (and its 256 TMEM
// columns) occupies an SM: CTAs of different clusters never wait on each other's TMEM.
constexpr size_t kOneCtaSmem = 120 * 1024;
size_t grad_smem(int kind, int n, int stages) {
  return std::max(kOneCtaSmem, 1024 + size_t(stages) * stage_bytes(kind, n) + kTailBytes + sizeof(Barriers));
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    linear_grad_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_b2, const __grid_constant__ CUtensorMap map_out, int n,
                       int kblocks, int stages, int m_extent, void *__restrict__ grad_w, int pt,
                       float *__restrict__ grad_b, int dgrad_splits, float4 *__restrict__ dgrad_partial) {
  constexpr int KS = stage_k(KIND);
  constexpr uint32_t kABytes = a_tile_bytes(KIND);
  const uint32_t b_bytes = uint32_t(n) * KS * 4;
  const uint32_t st_bytes = 2 * kABytes + (KIND == kWgrad ? 2u : 1u) * b_bytes;
  const uint32_t idesc = umma_idesc_tf32(KIND == kWgrad, true, kBM, n);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;
  float *colsum = reinterpret_cast<float *>(ring + size_t(stages) * st_bytes);  // [kConvWarps][kBM]
  float *bias_part = colsum + kConvWarps * kBM;                                 // [kBM]
  Barriers *bs = reinterpret_cast<Barriers *>(bias_part + kBM);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  int kb_begin = 0, kb_end = kblocks;
  if constexpr (KIND == kWgrad) {
    kb_begin = static_cast<int>(int64_t(kblocks) * blockIdx.y / kSlices);
    kb_end = static_cast<int>(int64_t(kblocks) * (blockIdx.y + 1) / kSlices);
  } else {
    // DGRAD with few row blocks: CTA (x, y) contracts slice y of dgrad_splits (blockIdx.y).
    kb_begin = static_cast<int>(int64_t(kblocks) * blockIdx.y / dgrad_splits);
    kb_end = static_cast<int>(int64_t(kblocks) * (blockIdx.y + 1) / dgrad_splits);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bs->full[s], 1);
      mbar_init(&bs->conv[s], kConvWarps);
      mbar_init(&bs->empty[s], 1);
    }
    mbar_init(&bs->tmem_full, 1);
    bs->abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(&bs->tmem_base, 2 * kMaxN);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = bs->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      prefetch_map(&map_a);
      prefetch_map(&map_b);
      uint32_t issued[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) issued[s] = 0;
      int it = 0;
      for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
        const int s = it % stages;
        if (!wait_bar(&bs->empty[s], (uint32_t(it / stages) & 1u) ^ 1u, bs)) break;
        uint8_t *st = ring + size_t(s) * st_bytes;
        mbar_expect_tx(&bs->full[s], kABytes + (KIND == kWgrad ? 2u : 1u) * b_bytes);
        if constexpr (KIND == kDgrad) {
          tma_load_2d(st, &map_a, &bs->full[s], kb * KS, m0);
        } else {
          tma_load_3d(st, &map_a, &bs->full[s], 0, kb * KS, m0 / 32);
          tma_load_3d(st + 2 * kABytes + b_bytes, &map_b2, &bs->full[s], 0, kb * KS, 0);
        }
        tma_load_3d(st + 2 * kABytes, &map_b, &bs->full[s], 0, kb * KS, 0);
        issued[s] = uint32_t(it / stages) + 1;
      }
      for (int s = 0; s < stages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // big x big products accumulate in columns [0, 256), the cross terms (about 2^-11 of
      // them) in [256, 512): the tensor-core accumulation error grows with the number of
      // additions into one accumulator, so the dominant sum gets one addition per k step.
      const uint32_t tmem_big = tmem_base, tmem_cross = tmem_base + kMaxN;
      int it = 0;
      for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
        const int s = it % stages;
        const uint32_t ph = uint32_t(it / stages) & 1u;
        if (!wait_bar(&bs->full[s], ph, bs) || !wait_bar(&bs->conv[s], ph, bs)) break;
        tmem_fence_after();
        const uint32_t a = smem_addr(ring + size_t(s) * st_bytes);
        const uint32_t a_small = a + kABytes;
        const uint32_t b = a + 2 * kABytes;
#pragma unroll
        for (int kk = 0; kk < KS / 8; ++kk) {
          const uint32_t acc = (it | kk) != 0 ? 1u : 0u;
          const uint64_t db = umma_desc_mn_tf32(b + kk * 1024, KS * 128);
          if constexpr (KIND == kDgrad) {
            umma_tf32(tmem_big, umma_desc_sw128(a + kk * 32), db, idesc, acc);
            umma_tf32(tmem_cross, umma_desc_sw128(a_small + kk * 32), db, idesc, acc);
          } else {
            const uint64_t da = umma_desc_mn_tf32(a + kk * 1024, KS * 128);
            const uint64_t da_small = umma_desc_mn_tf32(a_small + kk * 1024, KS * 128);
            const uint64_t db_small = umma_desc_mn_tf32(b + b_bytes + kk * 1024, KS * 128);
            umma_tf32(tmem_big, da, db, idesc, acc);
            umma_tf32(tmem_cross, da_small, db, idesc, acc);
            umma_tf32(tmem_cross, da, db_small, idesc, 1u);
          }
        }
        umma_commit(&bs->empty[s]);
      }
      umma_commit(&bs->tmem_full);
    }
  } else {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - 64;
    float csum[4] = {0.f, 0.f, 0.f, 0.f};
    int it = 0;
    for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
      const int s = it % stages;
      int ok = 1;
      if (lane == 0) ok = wait_bar(&bs->full[s], uint32_t(it / stages) & 1u, bs) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      uint8_t *a = ring + size_t(s) * st_bytes;
      uint8_t *a_small = a + kABytes;
      if constexpr (KIND == kDgrad) {
        // Elementwise over the whole 16 KB tile.
#pragma unroll
        for (int i = 0; i < int(kABytes / 16) / (32 * kConvWarps); ++i) {
          const uint32_t off = uint32_t(ct + i * 32 * kConvWarps) * 16;
          float4 x = *reinterpret_cast<float4 *>(a + off);
          float4 hi, lo;
          hi.x = round_tf32(x.x), lo.x = round_tf32(__fsub_rn(x.x, hi.x));
          hi.y = round_tf32(x.y), lo.y = round_tf32(__fsub_rn(x.y, hi.y));
          hi.z = round_tf32(x.z), lo.z = round_tf32(__fsub_rn(x.z, hi.z));
          hi.w = round_tf32(x.w), lo.w = round_tf32(__fsub_rn(x.w, hi.w));
          *reinterpret_cast<float4 *>(a + off) = hi;
          *reinterpret_cast<float4 *>(a_small + off) = lo;
        }
      } else {
        // Thread = 4 consecutive W rows (o) of one strip x 4 contraction rows; the column sums
        // of g (grad_b) accumulate per thread in row order. In a 128-byte row the 32-byte chunk
        // c sits at c ^ (row & 3).
        const int pair = ct & 31, strip = pair >> 3, chunk = pair & 7;
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int r = (ct >> 5) * 4 + rr;
          const uint32_t off =
              uint32_t(strip * KS * 128 + r * 128 + ((((chunk >> 1) ^ (r & 3)) << 5) | ((chunk & 1) << 4)));
          float4 x = *reinterpret_cast<float4 *>(a + off);
          csum[0] = __fadd_rn(csum[0], x.x);
          csum[1] = __fadd_rn(csum[1], x.y);
          csum[2] = __fadd_rn(csum[2], x.z);
          csum[3] = __fadd_rn(csum[3], x.w);
          float4 hi, lo;
          hi.x = round_tf32(x.x), lo.x = round_tf32(__fsub_rn(x.x, hi.x));
          hi.y = round_tf32(x.y), lo.y = round_tf32(__fsub_rn(x.y, hi.y));
          hi.z = round_tf32(x.z), lo.z = round_tf32(__fsub_rn(x.z, hi.z));
          hi.w = round_tf32(x.w), lo.w = round_tf32(__fsub_rn(x.w, hi.w));
          *reinterpret_cast<float4 *>(a + off) = hi;
          *reinterpret_cast<float4 *>(a_small + off) = lo;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bs->conv[s]);
    }

    // ---------------- epilogue ----------------
    if (warp == 2 && lane == 0) bs->epi_go = wait_bar(&bs->tmem_full, 0, bs) ? 1 : 0;
    named_sync(1, 32 * kConvWarps);
    const bool go = *reinterpret_cast<volatile int *>(&bs->epi_go) != 0;
    __syncwarp();
    tmem_fence_after();
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16);
    // 32 columns of this lane: big-product sum + cross-term sum.
    auto load_sum = [&](uint32_t addr, float (&v)[32]) {
      float w[32];
      tmem_ld32(addr, v);
      tmem_ld32(addr + kMaxN, w);
      tmem_wait_ld();
      reg_fence(v);
      reg_fence(w);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], w[j]);
    };
    const bool have = go && kb_end > kb_begin;
    if constexpr (KIND == kDgrad) {
      // 32 x 32 f32 tiles: registers -> this warp's 4 KB swizzled shared tile -> TMA store.
      uint8_t *stage = ring + (warp - 2) * 4096;
      if (go && dgrad_partial != nullptr) {
        // Slice partial for slice_reduce: [row block * splits + slice][column / 4][row].
        float4 *p = dgrad_partial + (size_t(blockIdx.x) * dgrad_splits + blockIdx.y) * size_t(n / 4) * kBM + row;
        for (int c = 0; c < n; c += 32) {
          float v[32];
          if (kb_end > kb_begin) {
            load_sum(taddr + uint32_t(c), v);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            p[size_t(c / 4 + j) * kBM] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      } else if (go) {
        for (int c = 0; c < n; c += 32) {
          float v[32];
          load_sum(taddr + uint32_t(c), v);
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          uint8_t *my_row = stage + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4 *>(my_row + ((j ^ (lane & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_out, stage, c, m0 + quarter * 32);
            bulk_commit();
          }
        }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    } else {
      // Partial tile -> shared [128][n] f32 (16-byte chunks XOR-swizzled by row & 7 so that
      // the 32 row-per-lane writes spread over the banks); rows of an empty slice are zero.
      float *part = reinterpret_cast<float *>(ring);
      for (int c = 0; c < n; c += 32) {
        float v[32];
        if (have) {
          load_sum(taddr + uint32_t(c), v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        float *my_row = part + size_t(row) * n;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4 *>(my_row + 4 * (((c >> 2) + j) ^ (row & 7))) =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      // Column sums: [contraction-row group][o] then summed in group order.
      const int pair = (threadIdx.x - 64) & 31, rg = (threadIdx.x - 64) >> 5;
#pragma unroll
      for (int e = 0; e < 4; ++e) colsum[rg * kBM + pair * 4 + e] = csum[e];
      named_sync(1, 32 * kConvWarps);
      const int o = threadIdx.x - 64;
      float t = 0.f;
      for (int g = 0; g < kConvWarps; ++g) t = __fadd_rn(t, colsum[g * kBM + o]);
      bias_part[o] = t;
    }
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem_base, 2 * kMaxN);
  }

  if constexpr (KIND == kWgrad) {
    // Cluster reduction: CTA y finishes W rows [y * 32, y * 32 + 32) of the block, adding the
    // kSlices partials in slice order.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    constexpr int kRows = kBM / kSlices;
    const int y = static_cast<int>(cluster.block_rank());
    const int c4n = n / 4;
    const float *parts[kSlices];
    const float *bparts[kSlices];
    float *part = reinterpret_cast<float *>(ring);
#pragma unroll
    for (int q = 0; q < kSlices; ++q) {
      parts[q] = cluster.map_shared_rank(part, q);
      bparts[q] = cluster.map_shared_rank(bias_part, q);
    }
    for (int e = threadIdx.x; e < kRows * c4n; e += kThreads) {
      const int r = y * kRows + e / c4n, c4 = e % c4n;
      const int o = m0 + r;
      const size_t off = size_t(r) * n + 4 * (c4 ^ (r & 7));
      float4 acc = *reinterpret_cast<const float4 *>(parts[0] + off);
#pragma unroll
      for (int q = 1; q < kSlices; ++q) {
        const float4 p = *reinterpret_cast<const float4 *>(parts[q] + off);
        acc.x = __fadd_rn(acc.x, p.x);
        acc.y = __fadd_rn(acc.y, p.y);
        acc.z = __fadd_rn(acc.z, p.z);
        acc.w = __fadd_rn(acc.w, p.w);
      }
      if (o < m_extent) {
        const size_t dst = size_t(o) * n + 4 * c4;
        if (pt == TROPNN_B200_F16) {
          __half h[4] = {__float2half_rn(acc.x), __float2half_rn(acc.y), __float2half_rn(acc.z), __float2half_rn(acc.w)};
          *reinterpret_cast<uint2 *>(static_cast<__half *>(grad_w) + dst) = *reinterpret_cast<const uint2 *>(h);
        } else {
          __nv_bfloat16 h[4] = {__float2bfloat16_rn(acc.x), __float2bfloat16_rn(acc.y), __float2bfloat16_rn(acc.z),
                                __float2bfloat16_rn(acc.w)};
          *reinterpret_cast<uint2 *>(static_cast<__nv_bfloat16 *>(grad_w) + dst) = *reinterpret_cast<const uint2 *>(h);
        }
      }
    }
    if (grad_b != nullptr && threadIdx.x < kRows) {
      const int r = y * kRows + threadIdx.x;
      float t = bparts[0][r];
#pragma unroll
      for (int q = 1; q < kSlices; ++q) t = __fadd_rn(t, bparts[q][r]);
      if (m0 + r < m_extent) grad_b[m0 + r] = t;
    }
    cluster.sync();
  }
}

// x = big + small with big, small tf32-representable (the split the WGRAD B operand reads).
__global__ void __launch_bounds__(256) tf32_split_kernel(const float4 *__restrict__ x, int64_t quads,
                                                          float4 *__restrict__ big, float4 *__restrict__ small) {
  for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < quads; q += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = __ldg(x + q);
    float4 hi, lo;
    hi.x = round_tf32(v.x), lo.x = round_tf32(__fsub_rn(v.x, hi.x));
    hi.y = round_tf32(v.y), lo.y = round_tf32(__fsub_rn(v.y, hi.y));
    hi.z = round_tf32(v.z), lo.z = round_tf32(__fsub_rn(v.z, hi.z));
    hi.w = round_tf32(v.w), lo.w = round_tf32(__fsub_rn(v.w, hi.w));
    big[q] = hi;
    small[q] = lo;
  }
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

bool linear_grad_supported(int64_t rows, int64_t out_features, int64_t in_features) {
  return rows >= 1 && rows <= (int64_t(1) << 31) - 1024 && out_features >= 32 && out_features % 32 == 0 &&
         out_features <= (int64_t(1) << 30) && in_features >= 32 && in_features <= kMaxN && in_features % 32 == 0 &&
         grad_stages(kDgrad, static_cast<int>(in_features)) > 0 && grad_stages(kWgrad, static_cast<int>(in_features)) > 0;
}

// DGRAD's contraction (out_features) in slices when the row blocks leave most SMs idle.
constexpr int kDgradTargetCtas = 148;
int dgrad_splits(int64_t rows, int64_t out_features, int64_t in_features) {
  // CTA (row block, slice): slices of at least 8 k blocks (~0.53 us each: big and small g
  // against the 32-deep f32 weight slab), filling the SMs in whole rounds; each slice adds a
  // [rows, in] f32 partial to the ordered reduction (~5 TB/s).
  const int64_t row_blocks = ceil_div(rows, int64_t(kBM));
  const int64_t kblocks = ceil_div(out_features, int64_t(stage_k(kDgrad)));
  return balanced_splits(row_blocks, kblocks, kDgradTargetCtas, 16, 8, 0.53,
                         double(rows) * double(in_features) * 4.0 / 5e6);
}

size_t dgrad_workspace(int64_t rows, int64_t out_features, int64_t in_features) {
  const int s = dgrad_splits(rows, out_features, in_features);
  if (s == 1) return 0;
  return WorkspaceCarver::align(size_t(ceil_div(rows, int64_t(kBM))) * s * size_t(in_features) * kBM * sizeof(float));
}

int linear_dgrad_impl(const float *g, int64_t rows, int64_t out_features, const float *weight32, int64_t in_features,
                      float *grad_hidden, void *ws, size_t ws_bytes, cudaStream_t stream) {
  TB_REQUIRE(linear_grad_supported(rows, out_features, in_features), TROPNN_B200_ERR_INVALID,
             "linear_dgrad: unsupported shape rows=%lld out=%lld in=%lld", (long long)rows, (long long)out_features,
             (long long)in_features);
  TB_REQUIRE(g && weight32 && grad_hidden, TROPNN_B200_ERR_INVALID, "linear_dgrad: null pointer");
  TB_REQUIRE(aligned16(g) && aligned16(weight32) && aligned16(grad_hidden), TROPNN_B200_ERR_INVALID,
             "linear_dgrad: operands must be 16-byte aligned");
  const int n = static_cast<int>(in_features);
  const int stages = grad_stages(kDgrad, n);
  CUtensorMap map_a, map_b, map_out;
  TB_CHECK(make_map_f32_k32(&map_a, g, out_features, rows, kBM));
  TB_CHECK(make_map_f32_mn(&map_b, weight32, in_features, out_features, stage_k(kDgrad), n / 32));
  TB_CHECK(make_map_f32_store32(&map_out, grad_hidden, in_features, rows));
  const size_t smem = grad_smem(kDgrad, n, stages);
  auto kernel = linear_grad_kernel<kDgrad>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "linear_dgrad"));
  const int kblocks = static_cast<int>(ceil_div(out_features, int64_t(stage_k(kDgrad))));
  const int64_t row_blocks = ceil_div(rows, int64_t(kBM));
  // Few row blocks: split the contraction when the caller gave room for the slice partials.
  int splits = dgrad_splits(rows, out_features, in_features);
  float4 *partial = nullptr;
  if (splits > 1) {
    WorkspaceCarver wc(ws, ws_bytes);
    partial = wc.take<float4>(size_t(row_blocks) * splits * size_t(n / 4) * kBM);
    if (partial == nullptr) splits = 1;
  }
  const dim3 grid(static_cast<unsigned>(row_blocks), static_cast<unsigned>(splits));
  kernel<<<grid, kThreads, smem, stream>>>(map_a, map_b, map_b, map_out, n, kblocks, stages, static_cast<int>(rows),
                                           nullptr, 0, nullptr, splits, partial);
  TB_CHECK(check_launch("linear_dgrad"));
  if (splits == 1) return TROPNN_B200_OK;
  return slice_reduce_impl(kReduceF32, partial, splits, 1, n, rows, in_features, grad_hidden, TROPNN_B200_F32,
                           in_features, nullptr, nullptr, TROPNN_B200_F32, 1.f, stream);
}

int linear_wgrad_impl(const float *g, int64_t rows, int64_t out_features, const float *hidden_big,
                      const float *hidden_small, int64_t in_features, int dtype, void *grad_weight, float *grad_bias,
                      cudaStream_t stream) {
  TB_REQUIRE(dtype == TROPNN_B200_F16 || dtype == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "linear_wgrad: dtype %s unsupported (f16/bf16 only)", dtype_name(dtype));
  TB_REQUIRE(linear_grad_supported(rows, out_features, in_features), TROPNN_B200_ERR_INVALID,
             "linear_wgrad: unsupported shape rows=%lld out=%lld in=%lld", (long long)rows, (long long)out_features,
             (long long)in_features);
  TB_REQUIRE(g && hidden_big && hidden_small && grad_weight, TROPNN_B200_ERR_INVALID, "linear_wgrad: null pointer");
  TB_REQUIRE(aligned16(g) && aligned16(hidden_big) && aligned16(hidden_small) && reinterpret_cast<uintptr_t>(grad_weight) % 8 == 0,
             TROPNN_B200_ERR_INVALID, "linear_wgrad: misaligned operands");
  const int n = static_cast<int>(in_features);
  const int stages = grad_stages(kWgrad, n);
  CUtensorMap map_a, map_b, map_b2;
  TB_CHECK(make_map_f32_mn(&map_a, g, out_features, rows, stage_k(kWgrad), kBM / 32));
  TB_CHECK(make_map_f32_mn(&map_b, hidden_big, in_features, rows, stage_k(kWgrad), n / 32));
  TB_CHECK(make_map_f32_mn(&map_b2, hidden_small, in_features, rows, stage_k(kWgrad), n / 32));
  const size_t smem = grad_smem(kWgrad, n, stages);
  auto kernel = linear_grad_kernel<kWgrad>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "linear_wgrad"));
  const int kblocks = static_cast<int>(ceil_div(rows, int64_t(stage_k(kWgrad))));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(out_features, int64_t(kBM))), kSlices, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = kSlices;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, map_b2, map_a, n, kblocks, stages,
                                             static_cast<int>(out_features), grad_weight, dtype, grad_bias, 1,
                                             static_cast<float4 *>(nullptr));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "linear_wgrad launch failed: %s", cudaGetErrorString(err));
  return check_launch("linear_wgrad");
}

int tf32_split_impl(const float *x, int64_t count, float *big, float *small, cudaStream_t stream) {
  TB_REQUIRE(count >= 0 && count % 4 == 0, TROPNN_B200_ERR_INVALID, "tf32_split: count %lld must be a multiple of 4",
             (long long)count);
  if (count == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && big && small, TROPNN_B200_ERR_INVALID, "tf32_split: null pointer");
  TB_REQUIRE(aligned16(x) && aligned16(big) && aligned16(small), TROPNN_B200_ERR_INVALID,
             "tf32_split: operands must be 16-byte aligned");
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const int64_t quads = count / 4;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(quads, int64_t(256)), int64_t(sms) * 8));
  tf32_split_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float4 *>(x), quads, reinterpret_cast<float4 *>(big),
                                               reinterpret_cast<float4 *>(small));
  return check_launch("tf32_split");
}

int read_linear_grad_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_linear_grad_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_linear_grad_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

size_t tropnn_b200_linear_dgrad_workspace_size(int64_t rows, int64_t out_features, int64_t in_features) {
  if (rows < 1 || out_features < 1 || in_features < 1) return 0;
  return tropnn_b200::dgrad_workspace(rows, out_features, in_features);
}

int tropnn_b200_linear_dgrad(const float *g, int64_t rows, int64_t out_features, const float *weight32,
                             int64_t in_features, float *grad_hidden, void *workspace, size_t workspace_bytes,
                             void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  if (rows == 0) return tropnn_b200::clear_error();
  TB_CHECK(tropnn_b200::linear_dgrad_impl(g, rows, out_features, weight32, in_features, grad_hidden, workspace,
                                          workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_linear_wgrad(const float *g, int64_t rows, int64_t out_features, const float *hidden_big,
                             const float *hidden_small, int64_t in_features, int dtype, void *grad_weight,
                             float *grad_bias, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  if (rows == 0) {
    // Empty contraction: zero gradients.
    TB_REQUIRE(dtype == TROPNN_B200_F16 || dtype == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
               "linear_wgrad: dtype unsupported (f16/bf16 only)");
    TB_REQUIRE(out_features >= 0 && in_features >= 0 && grad_weight, TROPNN_B200_ERR_INVALID,
               "linear_wgrad: bad arguments");
    cudaStream_t s = tropnn_b200::as_stream(stream);
    if (cudaMemsetAsync(grad_weight, 0, size_t(out_features) * size_t(in_features) * 2, s) != cudaSuccess ||
        (grad_bias && cudaMemsetAsync(grad_bias, 0, size_t(out_features) * 4, s) != cudaSuccess))
      return tropnn_b200::set_error(TROPNN_B200_ERR_LAUNCH, "linear_wgrad: memset failed");
    return tropnn_b200::clear_error();
  }
  TB_CHECK(tropnn_b200::linear_wgrad_impl(g, rows, out_features, hidden_big, hidden_small, in_features, dtype,
                                          grad_weight, grad_bias, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_tf32_split(const float *x, int64_t count, float *big, float *small, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::tf32_split_impl(x, count, big, small, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
