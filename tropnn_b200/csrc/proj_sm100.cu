// TropLinear input projection on the sm_100a tensor cores: z = half(half(x) P^T).
//
// Reference behaviour (layers/tropical.py:96-99): `z = proj(x.to(P.dtype))` with P the
// half-precision projection weight [code_dim, in]: x is rounded to P's dtype, the product
// is accumulated in f32 and rounded to P's dtype (cuBLAS's f16 GEMM output), and the route
// then reads z upcast to f32. Here the f32 input is read once from HBM and rounded in
// shared memory, so neither a separate cast pass over x nor a library GEMM is needed;
// products of the rounded operands are exact in f32 and only the summation order differs
// from the reference's.
//
// Work unit = (128-row block of x, k slice of in/64 k blocks). With enough row blocks every
// unit covers all of `in` (one slice); with few (small batches, or one GPU's shard of a
// strong-scaled batch) the contraction is cut into up to 16 slices so that every SM has a
// unit: each slice's f32 partial goes to the caller's workspace in a TMEM-native layout
// (row index fastest: coalesced stores), and slice_reduce (launched next, stream-ordered)
// sums the slices in slice order and rounds them, so results are deterministic.
// Persistent grid, one CTA per SM, contiguous unit ranges. CTA = 14 warps:
//   warp 0      TMA producer: per k block two 128 x 32 f32 boxes of x (128-byte swizzle)
//               and the code_dim x 64 tile of P, into a 3-4 stage ring.
//   warp 1      allocates 2 x code_dim TMEM columns (double-buffered f32 accumulator);
//               lane 0 issues the MMAs (kind::f16, M=128, N=code_dim, K=16).
//   warps 2-5   converters: one thread per x row rounds its 64 f32 of the k block to the
//               parameter dtype and writes the 128-byte row in place, in the K-major
//               128-byte-swizzle layout the MMA reads as its A operand.
//   warps 6-13  epilogue: 64-column chunks of the accumulator, rounded to the parameter
//               dtype, staged in shared memory and written with TMA stores (or written as
//               f32 slice partials for slice_reduce).
// Every wait is bounded (sm100.cuh): a wait that gives up sets the library's device error
// word, the other roles leave, copies and MMAs in flight are drained and TMEM is freed.
// Every TMA load is a plain per-CTA load of this GPU's own memory.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kXBox = kBM * 128;        // one 128-row x 32-float box of x (16 KB)
constexpr int kXBytes = 2 * kXBox;      // the f32 k block of x (32 KB); its first half holds the rounded tile
constexpr int kPBoxRows = 64;
constexpr int kConvWarps = 4;
constexpr int kEpiWarps = 8;
constexpr int kFirstConv = 2;
constexpr int kFirstEpi = kFirstConv + kConvWarps;
constexpr int kThreads = 32 * (kFirstEpi + kEpiWarps);
constexpr int kMaxStages = 4;
constexpr int kMinStages = 2;
constexpr int kStageOutBytes = 32 * 128;  // one warp's 32 rows x 64 half-precision columns
constexpr int kMaxSplits = 16;
constexpr int kMinKBlocksPerSplit = 4;
constexpr int kTargetUnits = 148;  // B200 SMs: fill them when the row blocks alone do not
constexpr size_t kSmemLimit = 227 * 1024;

__device__ int g_proj_error = 0;

struct Barriers {
  uint64_t full[kMaxStages];
  uint64_t conv[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int epi_go[2];
};

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Barriers *bs) {
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_proj_error);
}

__device__ __forceinline__ void epilogue_sync() { named_sync(1, kEpiWarps * 32); }

template <typename PT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<PT, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
}

struct ProjGeom {
  int64_t rows;
  int D;            // code_dim (MMA N, a multiple of 64, <= 256)
  int kblocks;      // ceil(in / 64)
  int splits;       // k slices per row block
  int kb_per_split;
  int stages;
  int64_t units;    // row blocks x splits
};

// Unit u = (row block u / splits, slice u % splits); the slice's k-block range.
__device__ __forceinline__ void unit_range(const ProjGeom &g, int64_t u, int64_t *rb, int *ks, int *kb0, int *kb1) {
  *rb = u / g.splits;
  *ks = static_cast<int>(u - *rb * g.splits);
  *kb0 = *ks * g.kb_per_split;
  *kb1 = min(g.kblocks, *kb0 + g.kb_per_split);
}

// The 64 accumulator columns [c, c + 64) of this thread's row, rounded to PT, written to the
// warp's staging tile (128-byte swizzle) and stored by one TMA store.
template <typename PT>
__device__ __forceinline__ void store_chunk(const float (&v)[64], uint8_t *stage, int lane, const CUtensorMap *map_z,
                                            int col, int row0) {
  if (lane == 0) bulk_wait_read_all();  // the previous store has read the staging tile
  __syncwarp();
  uint8_t *my_row = stage + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 q;
    q.x = pack2<PT>(v[8 * j], v[8 * j + 1]);
    q.y = pack2<PT>(v[8 * j + 2], v[8 * j + 3]);
    q.z = pack2<PT>(v[8 * j + 4], v[8 * j + 5]);
    q.w = pack2<PT>(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4 *>(my_row + ((j ^ (lane & 7)) << 4)) = q;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map_z, stage, col, row0);
    bulk_commit();
  }
}

template <typename PT>
__global__ void __launch_bounds__(kThreads, 1) trop_proj_kernel(const __grid_constant__ CUtensorMap map_x,
                                                                const __grid_constant__ CUtensorMap map_p,
                                                                const __grid_constant__ CUtensorMap map_z,
                                                                const ProjGeom g, float4 *__restrict__ partial) {
  constexpr int kFmt = std::is_same<PT, __half>::value ? 0 : 1;
  const uint32_t idesc = umma_idesc_f16(kFmt, kBM, g.D);
  const int stage_bytes = kXBytes + g.D * 128;
  const int chunks = g.D / 64;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;                                    // stages x [x k block | P tile]
  uint8_t *o_smem = ring + g.stages * stage_bytes;         // kEpiWarps x 4 KB store staging
  Barriers *bs = reinterpret_cast<Barriers *>(o_smem + kEpiWarps * kStageOutBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t u_begin = g.units * blockIdx.x / gridDim.x;
  const int64_t u_end = g.units * (blockIdx.x + 1) / gridDim.x;
  const uint32_t tmem_cols = g.D <= 64 ? 128u : (g.D <= 128 ? 256u : 512u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&bs->full[s], 1);
      mbar_init(&bs->conv[s], kConvWarps);
      mbar_init(&bs->empty[s], 1);
    }
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
    tmem_alloc(&bs->tmem_base, tmem_cols);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = bs->tmem_base;

  if (warp == 0) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- TMA producer ----------------
      prefetch_map(&map_x);
      prefetch_map(&map_p);
      uint32_t issued[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) issued[s] = 0;
      const uint32_t tx = uint32_t(kXBytes + g.D * 128);
      bool ok = true;
      int it = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        int64_t rb;
        int ks, kb0, kb1;
        unit_range(g, u, &rb, &ks, &kb0, &kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->empty[s], (uint32_t(it / g.stages) & 1u) ^ 1u, bs)) {
            ok = false;
            break;
          }
          uint8_t *st = ring + s * stage_bytes;
          mbar_expect_tx(&bs->full[s], tx);
          tma_load_2d(st, &map_x, &bs->full[s], kb * kBK, static_cast<int>(rb * kBM));
          tma_load_2d(st + kXBox, &map_x, &bs->full[s], kb * kBK + 32, static_cast<int>(rb * kBM));
          for (int q = 0; q < g.D / kPBoxRows; ++q)
            tma_load_2d(st + kXBytes + q * kPBoxRows * 128, &map_p, &bs->full[s], kb * kBK, q * kPBoxRows);
          issued[s] = uint32_t(it / g.stages) + 1;
        }
      }
      for (int s = 0; s < g.stages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- MMA issuer ----------------
      bool ok = true;
      int it = 0;
      uint32_t t = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u, ++t) {
        int64_t rb;
        int ks, kb0, kb1;
        unit_range(g, u, &rb, &ks, &kb0, &kb1);
        const int b = t & 1;
        if (!wait_bar(&bs->tmem_empty[b], ((t >> 1) & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * g.D);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->conv[s], uint32_t(it / g.stages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t a_base = smem_addr(ring + s * stage_bytes);
          const uint32_t b_base = a_base + kXBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d_tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), idesc,
                     (kb != kb0 || kk != 0) ? 1u : 0u);
          umma_commit(&bs->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bs->tmem_full[b]);
      }
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else if (warp < kFirstEpi) {
    // ---------------- converters ----------------
    // Thread r rounds row r of the k block: its 32 + 32 floats from the two f32 boxes (row
    // r's 16-byte chunk j sits at r * 128 + ((j ^ (r & 7)) * 16)) become eight 16-byte
    // chunks of 8 half-precision values written to the same places of the first box.
    const int r = (warp - kFirstConv) * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int64_t u = u_begin; u < u_end && ok; ++u) {
      int64_t rb;
      int ks, kb0, kb1;
      unit_range(g, u, &rb, &ks, &kb0, &kb1);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % g.stages;
        int go = 1;
        if (lane == 0) go = wait_bar(&bs->full[s], uint32_t(it / g.stages) & 1u, bs) ? 1 : 0;
        __syncwarp();  // orders lane 0's completed wait before the other lanes' reads
        go = __shfl_sync(0xffffffffu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        uint8_t *row = ring + s * stage_bytes + r * 128;
        float4 f[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          f[j] = *reinterpret_cast<const float4 *>(row + ((j ^ (r & 7)) << 4));
          f[8 + j] = *reinterpret_cast<const float4 *>(row + kXBox + ((j ^ (r & 7)) << 4));
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          uint4 q;
          q.x = pack2<PT>(f[2 * m].x, f[2 * m].y);
          q.y = pack2<PT>(f[2 * m].z, f[2 * m].w);
          q.z = pack2<PT>(f[2 * m + 1].x, f[2 * m + 1].y);
          q.w = pack2<PT>(f[2 * m + 1].z, f[2 * m + 1].w);
          *reinterpret_cast<uint4 *>(row + ((m ^ (r & 7)) << 4)) = q;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bs->conv[s]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - kFirstEpi;
    const int quarter = warp & 3;       // TMEM lane quarter this warp may read
    const int group = ew >> 2;          // chunks group, group + 2, ...
    const int r = quarter * 32 + lane;  // accumulator row
    uint8_t *stage = o_smem + ew * kStageOutBytes;
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      int64_t rb;
      int ks, kb0, kb1;
      unit_range(g, u, &rb, &ks, &kb0, &kb1);
      const int b = t & 1;
      if (ew == 0 && lane == 0) bs->epi_go[b] = wait_bar(&bs->tmem_full[b], (t >> 1) & 1u, bs) ? 1 : 0;
      epilogue_sync();
      if (*reinterpret_cast<volatile int *>(&bs->epi_go[b]) == 0) break;
      __syncwarp();
      tmem_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * g.D);
      const int row0 = static_cast<int>(rb * kBM + quarter * 32);
      for (int ch = group; ch < chunks; ch += 2) {
        float lo[32], hi[32], v[64];
        tmem_ld32(taddr + uint32_t(ch * 64), lo);
        tmem_ld32(taddr + uint32_t(ch * 64 + 32), hi);
        tmem_wait_ld();
        reg_fence(lo);
        reg_fence(hi);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = lo[i];
          v[32 + i] = hi[i];
        }
        if (g.splits == 1) {
          store_chunk<PT>(v, stage, lane, &map_z, ch * 64, row0);
        } else {
          float4 *p = partial + (size_t(u) * (g.D / 4) + ch * 16) * kBM + r;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            p[size_t(j) * kBM] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      // Every TMEM read of this unit is complete (tcgen05.wait::ld above).
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Weight gradient of the projection: grad_P[d, i] = sum_n g[n, d] half(x[n, i]), the
// reference's half-precision F.linear backward (f16 operands, f32 accumulation, one rounding).
// Computed as its transpose C[i, d] = sum_n half(x)^T[i, n] g^T[d, n]: unit = (128 input
// features, slice of the samples). The f32 x tile [64 samples x 128 features] arrives by TMA
// as four 64 x 32-float boxes; the converter warps transpose and round it into the K-major A
// tile [128 features x 64 samples] (one thread per feature: eight samples per 16-byte chunk);
// B is the g^T k block [code_dim x 64 samples] by TMA. x is read from HBM once, in f32.
// The epilogue writes grad_P directly (each store of a warp covers 32 consecutive features of
// one row of grad_P), or f32 slice partials that slice_reduce sums in slice order and writes
// transposed.
constexpr int kWBK = 64;                    // samples per k block
constexpr int kWXBox = kWBK * 128;          // one 64-sample x 32-feature f32 box (8 KB)
constexpr int kWXBytes = 4 * kWXBox;        // 64 samples x 128 features f32 (32 KB)
constexpr int kWABytes = kBM * 128;         // the transposed, rounded A tile (16 KB)
constexpr int kWMaxStages = 3;

struct WgradGeom {
  int64_t rows;     // samples (the contraction)
  int64_t in;       // input features (rows of C)
  int D;            // code_dim (MMA N)
  int kblocks;      // ceil(rows / 64)
  int splits;
  int kb_per_split;
  int stages;
  int64_t units;    // feature tiles x splits
};

__device__ __forceinline__ void wgrad_unit(const WgradGeom &g, int64_t u, int64_t *tile, int *kb0, int *kb1) {
  *tile = u / g.splits;
  const int ks = static_cast<int>(u - *tile * g.splits);
  *kb0 = ks * g.kb_per_split;
  *kb1 = min(g.kblocks, *kb0 + g.kb_per_split);
}

template <typename PT>
__global__ void __launch_bounds__(kThreads, 1) trop_proj_wgrad_kernel(const __grid_constant__ CUtensorMap map_x,
                                                                      const __grid_constant__ CUtensorMap map_g,
                                                                      const WgradGeom g, PT *__restrict__ grad_w,
                                                                      float4 *__restrict__ partial) {
  constexpr int kFmt = std::is_same<PT, __half>::value ? 0 : 1;
  const uint32_t idesc = umma_idesc_f16(kFmt, kBM, g.D);
  const int stage_bytes = kWXBytes + kWABytes + g.D * 128;
  const int chunks = g.D / 64;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;  // stages x [x tile f32 | A tile | g^T tile]
  Barriers *bs = reinterpret_cast<Barriers *>(ring + g.stages * stage_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t u_begin = g.units * blockIdx.x / gridDim.x;
  const int64_t u_end = g.units * (blockIdx.x + 1) / gridDim.x;
  const uint32_t tmem_cols = g.D <= 64 ? 128u : (g.D <= 128 ? 256u : 512u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&bs->full[s], 1);
      mbar_init(&bs->conv[s], kConvWarps);
      mbar_init(&bs->empty[s], 1);
    }
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
    tmem_alloc(&bs->tmem_base, tmem_cols);
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = bs->tmem_base;

  if (warp == 0) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- TMA producer ----------------
      prefetch_map(&map_x);
      prefetch_map(&map_g);
      uint32_t issued[kWMaxStages];
      for (int s = 0; s < kWMaxStages; ++s) issued[s] = 0;
      const uint32_t tx = uint32_t(kWXBytes + g.D * 128);
      bool ok = true;
      int it = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        int64_t tile;
        int kb0, kb1;
        wgrad_unit(g, u, &tile, &kb0, &kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->empty[s], (uint32_t(it / g.stages) & 1u) ^ 1u, bs)) {
            ok = false;
            break;
          }
          uint8_t *st = ring + s * stage_bytes;
          mbar_expect_tx(&bs->full[s], tx);
          for (int q = 0; q < 4; ++q)
            tma_load_2d(st + q * kWXBox, &map_x, &bs->full[s], static_cast<int>(tile * kBM + q * 32), kb * kWBK);
          for (int q = 0; q < g.D / kPBoxRows; ++q)
            tma_load_2d(st + kWXBytes + kWABytes + q * kPBoxRows * 128, &map_g, &bs->full[s], kb * kWBK,
                        q * kPBoxRows);
          issued[s] = uint32_t(it / g.stages) + 1;
        }
      }
      for (int s = 0; s < g.stages; ++s)
        if (issued[s] > 0) mbar_drain(&bs->full[s], (issued[s] - 1) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0 && u_begin < u_end) {
      // ---------------- MMA issuer ----------------
      bool ok = true;
      int it = 0;
      uint32_t t = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u, ++t) {
        int64_t tile;
        int kb0, kb1;
        wgrad_unit(g, u, &tile, &kb0, &kb1);
        const int b = t & 1;
        if (!wait_bar(&bs->tmem_empty[b], ((t >> 1) & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * g.D);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->conv[s], uint32_t(it / g.stages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t a_base = smem_addr(ring + s * stage_bytes + kWXBytes);
          const uint32_t b_base = a_base + kWABytes;
#pragma unroll
          for (int kk = 0; kk < kWBK / 16; ++kk)
            umma_f16(d_tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), idesc,
                     (kb != kb0 || kk != 0) ? 1u : 0u);
          umma_commit(&bs->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bs->tmem_full[b]);
      }
      umma_commit(&bs->mma_done);
      mbar_drain(&bs->mma_done, 0);
    }
  } else if (warp < kFirstEpi) {
    // ---------------- converters ----------------
    // Thread f writes feature f's row of A: chunk j holds samples 8j..8j+7, read from row
    // 8j + e of box f / 32 (float f % 32 of that 128-byte row sits in chunk (f % 32) / 4
    // XOR (row & 7)). A warp reads one whole box row per load (no bank conflicts) and writes
    // 32 rows' chunk j (swizzled: eight distinct 16-byte slots per eight rows).
    const int f = (warp - kFirstConv) * 32 + lane;
    const int box = f >> 5, fl = f & 31;
    int it = 0;
    bool ok = true;
    for (int64_t u = u_begin; u < u_end && ok; ++u) {
      int64_t tile;
      int kb0, kb1;
      wgrad_unit(g, u, &tile, &kb0, &kb1);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % g.stages;
        int go = 1;
        if (lane == 0) go = wait_bar(&bs->full[s], uint32_t(it / g.stages) & 1u, bs) ? 1 : 0;
        __syncwarp();
        go = __shfl_sync(0xffffffffu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        const uint8_t *xb = ring + s * stage_bytes + box * kWXBox;
        uint8_t *arow = ring + s * stage_bytes + kWXBytes + f * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int k = 8 * j + e;
            v[e] = *reinterpret_cast<const float *>(xb + k * 128 + ((((fl >> 2) ^ (k & 7))) << 4) + ((fl & 3) << 2));
          }
          uint4 q;
          q.x = pack2<PT>(v[0], v[1]);
          q.y = pack2<PT>(v[2], v[3]);
          q.z = pack2<PT>(v[4], v[5]);
          q.w = pack2<PT>(v[6], v[7]);
          *reinterpret_cast<uint4 *>(arow + ((j ^ (f & 7)) << 4)) = q;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bs->conv[s]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - kFirstEpi;
    const int quarter = warp & 3;
    const int group = ew >> 2;
    const int r = quarter * 32 + lane;  // accumulator row = feature within the tile
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      int64_t tile;
      int kb0, kb1;
      wgrad_unit(g, u, &tile, &kb0, &kb1);
      const int b = t & 1;
      if (ew == 0 && lane == 0) bs->epi_go[b] = wait_bar(&bs->tmem_full[b], (t >> 1) & 1u, bs) ? 1 : 0;
      epilogue_sync();
      if (*reinterpret_cast<volatile int *>(&bs->epi_go[b]) == 0) break;
      __syncwarp();
      tmem_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * g.D);
      const int64_t feat = tile * kBM + r;
      for (int ch = group; ch < chunks; ch += 2) {
        float lo[32], hi[32];
        tmem_ld32(taddr + uint32_t(ch * 64), lo);
        tmem_ld32(taddr + uint32_t(ch * 64 + 32), hi);
        tmem_wait_ld();
        reg_fence(lo);
        reg_fence(hi);
        if (g.splits == 1) {
          if (feat < g.in) {
            PT *col = grad_w + int64_t(ch * 64) * g.in + feat;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              col[int64_t(c) * g.in] = from_f32<PT>(lo[c]);
              col[int64_t(32 + c) * g.in] = from_f32<PT>(hi[c]);
            }
          }
        } else {
          float4 *p = partial + (size_t(u) * (g.D / 4) + ch * 16) * kBM + r;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            p[size_t(j) * kBM] = make_float4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
            p[size_t(8 + j) * kBM] = make_float4(hi[4 * j], hi[4 * j + 1], hi[4 * j + 2], hi[4 * j + 3]);
          }
        }
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bs->tmem_empty[b]);
    }
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// --------------------------------------------------------------------------- host side

size_t proj_stage_bytes(int64_t D) { return size_t(kXBytes) + size_t(D) * 128; }

size_t proj_smem_bytes(int64_t D, int stages) {
  return 1024 + size_t(stages) * proj_stage_bytes(D) + size_t(kEpiWarps) * kStageOutBytes + sizeof(Barriers);
}

int proj_stages(int64_t D) {
  const size_t fixed = proj_smem_bytes(D, 0);
  const int stages = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / proj_stage_bytes(D)));
  return stages >= kMinStages ? stages : 0;
}

ProjGeom proj_geometry(int64_t rows, int64_t in, int64_t D) {
  ProjGeom g{};
  g.rows = rows;
  g.D = static_cast<int>(D);
  g.kblocks = static_cast<int>(ceil_div(in, kBK));
  const int64_t row_blocks = ceil_div(rows, int64_t(kBM));
  // Few row blocks: cut the contraction so that the units fill the SMs in whole rounds. A k
  // block streams 32 KB of x per CTA (~0.75 us at the HBM rate per SM); each slice adds a
  // [rows, D] f32 partial to the ordered reduction (~5 TB/s).
  const int splits = balanced_splits(row_blocks, g.kblocks, kTargetUnits, kMaxSplits, kMinKBlocksPerSplit, 0.75,
                                     double(rows) * double(D) * 4.0 / 5e6);
  g.kb_per_split = static_cast<int>(ceil_div(g.kblocks, splits));
  g.splits = static_cast<int>(ceil_div(g.kblocks, g.kb_per_split));
  g.stages = proj_stages(D);
  g.units = row_blocks * g.splits;
  return g;
}

size_t proj_workspace_bytes(const ProjGeom &g) {
  if (g.splits == 1) return 0;
  return WorkspaceCarver::align(size_t(g.units) * size_t(g.D) * kBM * sizeof(float));
}

template <typename PT>
int launch_proj(const float *x, const void *P, void *z, const ProjGeom &g, int64_t in, void *ws, size_t ws_bytes,
                cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap map_x, map_p, map_z;
  TB_CHECK(make_map_f32_k32(&map_x, x, in, g.rows, kBM));
  TB_CHECK(make_map_k64(&map_p, P, dt, in, g.D, kPBoxRows));
  TB_CHECK(make_map_k64(&map_z, z, dt, g.D, g.rows, 32));
  float4 *partial = nullptr;
  if (g.splits > 1) {
    WorkspaceCarver c(ws, ws_bytes);
    partial = c.take<float4>(size_t(g.units) * size_t(g.D / 4) * kBM);
    TB_REQUIRE(partial != nullptr, TROPNN_B200_ERR_WORKSPACE,
               "trop_proj: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes,
               proj_workspace_bytes(g));
  }
  const size_t smem = proj_smem_bytes(g.D, g.stages);
  auto kernel = trop_proj_kernel<PT>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_proj"));
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(g.units, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_x, map_p, map_z, g, partial);
  TB_CHECK(check_launch("trop_proj"));
  if (g.splits == 1) return TROPNN_B200_OK;
  // The slices summed in slice order and rounded to the parameter dtype.
  return slice_reduce_impl(kReduceHalf, partial, g.splits, 1, g.D, g.rows, g.D, z,
                           std::is_same<PT, __half>::value ? TROPNN_B200_F16 : TROPNN_B200_BF16, g.D, nullptr, nullptr,
                           TROPNN_B200_F32, 1.f, stream);
}

size_t wgrad_stage_bytes(int64_t D) { return size_t(kWXBytes) + kWABytes + size_t(D) * 128; }

size_t wgrad_smem_bytes(int64_t D, int stages) {
  return 1024 + size_t(stages) * wgrad_stage_bytes(D) + sizeof(Barriers);
}

int wgrad_stages(int64_t D) {
  const size_t fixed = wgrad_smem_bytes(D, 0);
  const int stages = static_cast<int>(std::min<size_t>(kWMaxStages, (kSmemLimit - fixed) / wgrad_stage_bytes(D)));
  return stages >= 2 ? stages : 0;
}

WgradGeom wgrad_geometry(int64_t rows, int64_t in, int64_t D) {
  WgradGeom g{};
  g.rows = rows;
  g.in = in;
  g.D = static_cast<int>(D);
  g.kblocks = static_cast<int>(ceil_div(rows, kWBK));
  const int64_t tiles = ceil_div(in, int64_t(kBM));
  // Slices of the sample range: as many as keep all units in one wave of the SMs (the kernel
  // streams x from HBM, which ~7/8 of the SMs already saturate), at least 4 k blocks each.
  int splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxSplits, kTargetUnits / tiles)));
  splits = std::max(1, std::min(splits, g.kblocks / kMinKBlocksPerSplit));
  g.kb_per_split = static_cast<int>(ceil_div(g.kblocks, splits));
  g.splits = static_cast<int>(ceil_div(g.kblocks, g.kb_per_split));
  g.stages = wgrad_stages(D);
  g.units = tiles * g.splits;
  return g;
}

size_t wgrad_workspace_bytes(const WgradGeom &g) {
  if (g.splits == 1) return 0;
  return WorkspaceCarver::align(size_t(g.units) * size_t(g.D) * kBM * sizeof(float));
}

template <typename PT>
int launch_wgrad(const float *x, const void *gt, void *grad_w, const WgradGeom &g, void *ws, size_t ws_bytes,
                 cudaStream_t stream) {
  const CUtensorMapDataType dt =
      std::is_same<PT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap map_x, map_g;
  TB_CHECK(make_map_f32_k32(&map_x, x, g.in, g.rows, kWBK));
  TB_CHECK(make_map_k64(&map_g, gt, dt, g.rows, g.D, kPBoxRows));
  float4 *partial = nullptr;
  if (g.splits > 1) {
    WorkspaceCarver c(ws, ws_bytes);
    partial = c.take<float4>(size_t(g.units) * size_t(g.D / 4) * kBM);
    TB_REQUIRE(partial != nullptr, TROPNN_B200_ERR_WORKSPACE,
               "trop_proj_wgrad: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes,
               wgrad_workspace_bytes(g));
  }
  const size_t smem = wgrad_smem_bytes(g.D, g.stages);
  auto kernel = trop_proj_wgrad_kernel<PT>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_proj_wgrad"));
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(g.units, sms));
  kernel<<<grid, kThreads, smem, stream>>>(map_x, map_g, g, static_cast<PT *>(grad_w), partial);
  TB_CHECK(check_launch("trop_proj_wgrad"));
  if (g.splits == 1) return TROPNN_B200_OK;
  // The slices summed in slice order, rounded, written as grad_P [code_dim, in].
  return slice_reduce_impl(kReduceHalfT, partial, g.splits, 1, g.D, g.in, g.D, grad_w,
                           std::is_same<PT, __half>::value ? TROPNN_B200_F16 : TROPNN_B200_BF16, g.in, nullptr,
                           nullptr, TROPNN_B200_F32, 1.f, stream);
}

}  // namespace

size_t trop_proj_wgrad_workspace(int64_t rows, int64_t in, int64_t D) {
  if (rows < 1 || in < 1 || D < 64 || D > 256 || D % 64 != 0) return 0;
  return wgrad_workspace_bytes(wgrad_geometry(rows, in, D));
}

int trop_proj_wgrad_impl(const float *x, int64_t rows, int64_t in, const void *gt, int pt, int64_t D, void *grad_w,
                         void *ws, size_t ws_bytes, cudaStream_t stream) {
  TB_REQUIRE((pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16) && D >= 64 && D <= 256 && D % 64 == 0 && in >= 1 &&
                 in % 8 == 0 && rows % 8 == 0 && wgrad_stages(D) > 0,
             TROPNN_B200_ERR_INVALID,
             "trop_proj_wgrad: unsupported shape items=%lld in_features=%lld code_dim=%lld dtype=%s (needs f16/bf16, "
             "code_dim in {64, 128, 192, 256}, items and in_features multiples of 8)",
             (long long)rows, (long long)in, (long long)D, dtype_name(pt));
  TB_REQUIRE(rows >= 0 && rows <= (int64_t(1) << 31) - 1024 && in <= (int64_t(1) << 31) - 1024,
             TROPNN_B200_ERR_INVALID, "trop_proj_wgrad: sizes exceed the 32-bit tile coordinates");
  TB_REQUIRE(x && gt && grad_w, TROPNN_B200_ERR_INVALID, "trop_proj_wgrad: null pointer");
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  TB_REQUIRE(al16(x) && al16(gt), TROPNN_B200_ERR_INVALID, "trop_proj_wgrad: x and grad_z_t must be 16-byte aligned");
  if (rows == 0) {
    TB_CHECK(cudaMemsetAsync(grad_w, 0, size_t(D) * size_t(in) * 2, stream) == cudaSuccess
                 ? TROPNN_B200_OK
                 : set_error(TROPNN_B200_ERR_LAUNCH, "trop_proj_wgrad: zero fill failed"));
    return TROPNN_B200_OK;
  }
  const WgradGeom g = wgrad_geometry(rows, in, D);
  if (pt == TROPNN_B200_F16) return launch_wgrad<__half>(x, gt, grad_w, g, ws, ws_bytes, stream);
  return launch_wgrad<__nv_bfloat16>(x, gt, grad_w, g, ws, ws_bytes, stream);
}

bool proj_sm100_supported(int64_t in, int64_t D, int pt) {
  return (pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16) && D >= 64 && D <= 256 && D % 64 == 0 && in >= 1 &&
         in % 8 == 0 && proj_stages(D) > 0;
}

size_t trop_proj_workspace(int64_t rows, int64_t in, int64_t D) {
  if (rows < 0 || in < 1 || D < 64 || D > 256 || D % 64 != 0) return 0;
  return proj_workspace_bytes(proj_geometry(rows, in, D));
}

int trop_proj_impl(const float *x, int64_t rows, int64_t in, const void *P, int pt, int64_t D, void *z, void *ws,
                   size_t ws_bytes, cudaStream_t stream) {
  TB_REQUIRE(proj_sm100_supported(in, D, pt), TROPNN_B200_ERR_INVALID,
             "trop_proj: unsupported shape in_features=%lld code_dim=%lld dtype=%s (needs f16/bf16, code_dim in "
             "{64, 128, 192, 256}, in_features a multiple of 8)",
             (long long)in, (long long)D, dtype_name(pt));
  TB_REQUIRE(rows >= 0 && rows <= (int64_t(1) << 31) - 1024, TROPNN_B200_ERR_INVALID, "trop_proj: rows=%lld",
             (long long)rows);
  if (rows == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && P && z, TROPNN_B200_ERR_INVALID, "trop_proj: null pointer");
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  TB_REQUIRE(al16(x) && al16(P) && al16(z), TROPNN_B200_ERR_INVALID, "trop_proj: pointers must be 16-byte aligned");
  const ProjGeom g = proj_geometry(rows, in, D);
  if (pt == TROPNN_B200_F16) return launch_proj<__half>(x, P, z, g, in, ws, ws_bytes, stream);
  return launch_proj<__nv_bfloat16>(x, P, z, g, in, ws, ws_bytes, stream);
}

int read_proj_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_proj_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_proj_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

size_t tropnn_b200_trop_proj_workspace_size(int64_t items, int64_t in_features, int64_t code_dim) {
  return tropnn_b200::trop_proj_workspace(items, in_features, code_dim);
}

size_t tropnn_b200_trop_proj_wgrad_workspace_size(int64_t items, int64_t in_features, int64_t code_dim) {
  return tropnn_b200::trop_proj_wgrad_workspace(items, in_features, code_dim);
}

int tropnn_b200_trop_proj_wgrad(const float *x, int64_t items, int64_t in_features, const void *grad_z_t,
                                int param_dtype, int64_t code_dim, void *grad_weight, void *workspace,
                                size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_proj_wgrad_impl(x, items, in_features, grad_z_t, param_dtype, code_dim, grad_weight,
                                             workspace, workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_proj(const float *x, int64_t items, int64_t in_features, const void *proj_weight,
                          int param_dtype, int64_t code_dim, void *z, void *workspace, size_t workspace_bytes,
                          void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_proj_impl(x, items, in_features, proj_weight, param_dtype, code_dim, z, workspace,
                                       workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
