// f32 matrix product on the sm_100a tensor cores: C[m, n] = sum_k A[m, k] B[n, k] (+ bias[n]),
// A, B and C f32 row-major (A and B K-major), for TropLinear's f32 parameters: the input
// projection z = x P^T (layers/tropical.py:96-99), the output map y = hidden Wout^T + b
// (tropical.py:140-146), their backward products, and the effective weights and base output
// of the exact eval path (layers/tropical_exact.py:257-358). The reference computes these as
// f32 GEMMs (cuBLAS / MKL); there is no f32 tensor-core MMA, so every operand is split as
// x = big + small, big = tf32(x), small = tf32(x - big), and the product is formed as
// big*big' + big*small' + small*big' (3xTF32, Ootomo & Yokota 2022; small*small' is below f32
// rounding), which keeps f32 range and about 2^-22 relative accuracy per product. The
// tensor-core accumulator loses about half an ulp per addition, so big*big' accumulates in its
// own TMEM accumulator and the two cross terms in a second one, summed in the epilogue.
//
// Work unit = (128-row block of C, 128-column block of C, k slice); persistent grid, one CTA
// per SM, contiguous unit ranges. With fewer output tiles than ~3/4 of the SMs (the small
// products of configs 1 and 3) the contraction is cut into up to 16 slices: each slice's f32
// partial goes to the caller's workspace (row index fastest) and slice_reduce, launched next,
// sums them in slice order (deterministic) and adds the bias. CTA = 10 warps:
//   warp 0      TMA producer: per 32-wide k block the 128 x 32 f32 tiles of A and B
//               (128-byte swizzle) into a 3-stage ring.
//   warp 1      allocates 512 TMEM columns (two units in flight, each a big and a cross
//               accumulator of 128 columns); lane 0 issues 3 MMAs per 8-wide k step
//               (kind::tf32, M=128, N=128).
//   warps 2-5   converters: split both tiles in place (big) and into a second buffer
//               (small), elementwise.
//   warps 6-9   epilogue: per 32-column chunk, big + cross + bias, staged in shared memory
//               and written by TMA stores (plain stores when C's row stride is not a multiple
//               of 16 bytes).
// Waits are bounded (sm100.cuh); every TMA load is a plain per-CTA load of this GPU's memory.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kBK = 32;                      // f32 per 128-byte swizzled row
constexpr int kTile = kBM * 128;             // one 128 x 32 f32 tile (16 KB)
constexpr int kStageBytes = 4 * kTile;       // A, A small, B, B small
constexpr int kConvWarps = 4;
constexpr int kEpiWarps = 4;
constexpr int kFirstEpi = 2 + kConvWarps;
constexpr int kThreads = 32 * (kFirstEpi + kEpiWarps);
constexpr int kMaxStages = 4;
constexpr int kStageOutBytes = 32 * 128;
constexpr uint32_t kTmemCols = 512;
constexpr size_t kSmemLimit = 227 * 1024;
constexpr int kTargetUnits = 148;  // B200 SMs
constexpr int kMaxSplits = 16;
constexpr int kMinKBlocksPerSplit = 3;

__device__ int g_gemm_tf32_error = 0;

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
  return sm100::mbar_wait(bar, parity, &bs->abort, &g_gemm_tf32_error);
}

struct GemmGeom {
  int64_t m, n;
  int kblocks;
  int n_tiles;
  int splits;        // k slices per output tile
  int kb_per_split;
  int64_t units;     // output tiles x splits
  int stages;
  int64_t ldc;
  int tma_store;  // C's rows start on 16-byte boundaries: TMA stores, else plain stores
};

// Unit u = (output tile u / splits = (row block, column block), k slice u % splits).
struct GemmUnit {
  int64_t tile, mt;
  int nt, ks, kb0, kb1;
};
__device__ __forceinline__ GemmUnit decode(const GemmGeom &g, int64_t u) {
  GemmUnit w;
  w.tile = u / g.splits;
  w.ks = static_cast<int>(u - w.tile * g.splits);
  w.mt = w.tile / g.n_tiles;
  w.nt = static_cast<int>(w.tile - w.mt * g.n_tiles);
  w.kb0 = w.ks * g.kb_per_split;
  w.kb1 = min(g.kblocks, w.kb0 + g.kb_per_split);
  return w;
}

__device__ __forceinline__ float4 split_big(float4 x, float4 *small) {
  float4 hi;
  hi.x = round_tf32(x.x), small->x = round_tf32(__fsub_rn(x.x, hi.x));
  hi.y = round_tf32(x.y), small->y = round_tf32(__fsub_rn(x.y, hi.y));
  hi.z = round_tf32(x.z), small->z = round_tf32(__fsub_rn(x.z, hi.z));
  hi.w = round_tf32(x.w), small->w = round_tf32(__fsub_rn(x.w, hi.w));
  return hi;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                       const __grid_constant__ CUtensorMap map_c, const GemmGeom g, const float *__restrict__ bias,
                       float *__restrict__ c_ptr, float4 *__restrict__ partial) {
  const uint32_t idesc = umma_idesc_tf32(false, false, kBM, kBN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;
  uint8_t *o_smem = ring + g.stages * kStageBytes;
  Barriers *bs = reinterpret_cast<Barriers *>(o_smem + kEpiWarps * kStageOutBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t u_begin = g.units * blockIdx.x / gridDim.x;
  const int64_t u_end = g.units * (blockIdx.x + 1) / gridDim.x;

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
      prefetch_map(&map_b);
      uint32_t issued[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) issued[s] = 0;
      bool ok = true;
      int it = 0;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        const GemmUnit w = decode(g, u);
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->empty[s], (uint32_t(it / g.stages) & 1u) ^ 1u, bs)) {
            ok = false;
            break;
          }
          uint8_t *st = ring + s * kStageBytes;
          mbar_expect_tx(&bs->full[s], 2 * kTile);
          tma_load_2d(st, &map_a, &bs->full[s], kb * kBK, static_cast<int>(w.mt * kBM));
          tma_load_2d(st + 2 * kTile, &map_b, &bs->full[s], kb * kBK, w.nt * kBN);
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
        const GemmUnit w = decode(g, u);
        const int b = t & 1;
        if (!wait_bar(&bs->tmem_empty[b], ((t >> 1) & 1u) ^ 1u, bs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t d_big = tmem_base + uint32_t(b * 2 * kBN);
        const uint32_t d_cross = d_big + kBN;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % g.stages;
          if (!wait_bar(&bs->conv[s], uint32_t(it / g.stages) & 1u, bs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t a = smem_addr(ring + s * kStageBytes);
          const uint32_t a_small = a + kTile, bb = a + 2 * kTile, b_small = a + 3 * kTile;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint32_t acc = (kb != w.kb0 || kk != 0) ? 1u : 0u;
            const uint64_t da = umma_desc_sw128(a + kk * 32), db = umma_desc_sw128(bb + kk * 32);
            umma_tf32(d_big, da, db, idesc, acc);
            umma_tf32(d_cross, da, umma_desc_sw128(b_small + kk * 32), idesc, acc);
            umma_tf32(d_cross, umma_desc_sw128(a_small + kk * 32), db, idesc, 1u);
          }
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
    const int ct = threadIdx.x - 64;
    int it = 0;
    bool ok = true;
    for (int64_t u = u_begin; u < u_end && ok; ++u) {
      const GemmUnit w = decode(g, u);
      for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
        const int s = it % g.stages;
        int go = 1;
        if (lane == 0) go = wait_bar(&bs->full[s], uint32_t(it / g.stages) & 1u, bs) ? 1 : 0;
        __syncwarp();
        go = __shfl_sync(0xffffffffu, go, 0);
        if (!go) {
          ok = false;
          break;
        }
        uint8_t *st = ring + s * kStageBytes;
#pragma unroll
        for (int op = 0; op < 2; ++op) {  // A, then B
          uint8_t *t = st + op * 2 * kTile;
#pragma unroll 8
          for (int i = 0; i < kTile / 16 / (32 * kConvWarps); ++i) {
            const uint32_t off = uint32_t(ct + i * 32 * kConvWarps) * 16;
            float4 small;
            const float4 big = split_big(*reinterpret_cast<const float4 *>(t + off), &small);
            *reinterpret_cast<float4 *>(t + off) = big;
            *reinterpret_cast<float4 *>(t + kTile + off) = small;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bs->conv[s]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const int ew = warp - kFirstEpi;
    const int r = quarter * 32 + lane;  // accumulator row
    uint8_t *stage = o_smem + ew * kStageOutBytes;
    // 32 columns of C at `col` for this thread's row: staged + TMA store, or plain stores.
    auto store32 = [&](float (&v)[32], int64_t mt, int64_t col) {
      if (g.tma_store) {
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
          tma_store_2d(&map_c, stage, static_cast<int>(col), static_cast<int>(mt * kBM + quarter * 32));
          bulk_commit();
        }
      } else {
        const int64_t row = mt * kBM + r;
        if (row < g.m) {
          float *out = c_ptr + row * g.ldc + col;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j < g.n) out[j] = v[j];
        }
      }
    };
    auto add_bias = [&](float (&v)[32], int64_t col) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float bj = (bias != nullptr && col + j < g.n) ? __ldg(bias + col + j) : 0.f;
        v[j] = __fadd_rn(v[j], bj);
      }
    };
    uint32_t t = 0;
    for (int64_t u = u_begin; u < u_end; ++u, ++t) {
      const GemmUnit w = decode(g, u);
      const int b = t & 1;
      if (ew == 0 && lane == 0) bs->epi_go[b] = wait_bar(&bs->tmem_full[b], (t >> 1) & 1u, bs) ? 1 : 0;
      named_sync(1, kEpiWarps * 32);
      if (*reinterpret_cast<volatile int *>(&bs->epi_go[b]) == 0) break;
      __syncwarp();
      tmem_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(b * 2 * kBN);
      for (int c = 0; c < kBN; c += 32) {
        float v[32], x[32];
        tmem_ld32(taddr + uint32_t(c), v);
        tmem_ld32(taddr + uint32_t(kBN + c), x);
        tmem_wait_ld();
        reg_fence(v);
        reg_fence(x);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], x[j]);
        if (g.splits == 1) {
          const int64_t col = int64_t(w.nt) * kBN + c;
          add_bias(v, col);
          store32(v, w.mt, col);
        } else {
          // Slice partial, row index fastest (coalesced): [unit][column / 4][row].
          float4 *p = partial + (size_t(u) * (kBN / 4) + c / 4) * kBM + r;
#pragma unroll
          for (int j = 0; j < 8; ++j) p[size_t(j) * kBM] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
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
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// out[c * ldo + r] = x[r * ldx + c] for r < rows, c < cols (32 x 32 shared tiles); the
// padding columns r in [rows, ldo) of every output row are zero-filled.
__global__ void transpose_f32_kernel(const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                     float *__restrict__ out, int64_t ldo) {
  __shared__ float tile[32][33];
  const int64_t r0 = int64_t(blockIdx.y) * 32, c0 = int64_t(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? x[r * ldx + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < ldo) out[c * ldo + r] = tile[threadIdx.x][i];
  }
}

// out[c] = sum_r x[r * ldx + c]: block = 32 columns x 32 warps; warp w sums rows w, w + 32, ...
// in order, then the 32 warp partials are added in warp order (deterministic).
__global__ void colsum_f32_kernel(const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                  float *__restrict__ out) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = int64_t(blockIdx.x) * 32 + lane;
  float acc = 0.f;
  if (c < cols)
    for (int64_t r = w; r < rows; r += 32) acc = __fadd_rn(acc, __ldg(x + r * ldx + c));
  part[w][lane] = acc;
  __syncthreads();
  if (w == 0 && c < cols) {
    float s = 0.f;
    for (int i = 0; i < 32; ++i) s = __fadd_rn(s, part[i][lane]);
    out[c] = s;
  }
}

// Products with at most kSmallRows rows of C (config 1's 8-row batch): an M=128 MMA tile
// would be mostly padding and the TMA / TMEM pipeline set-up its whole cost, so they run as
// f32 FMA: one warp per column of C, lanes over k (coalesced rows of A and B), up to 8 rows
// of C per pass, partial sums added across the warp by a fixed butterfly (deterministic).
constexpr int kSmallRows = 32;
constexpr int kSmallWarps = 8;

__global__ void __launch_bounds__(kSmallWarps * 32) gemm_f32_rows_kernel(
    const float *__restrict__ a, int64_t lda, const float *__restrict__ b, int64_t ldb, int m, int64_t n, int64_t k,
    const float *__restrict__ bias, float *__restrict__ c, int64_t ldc) {
  const int lane = threadIdx.x & 31;
  const int64_t col = int64_t(blockIdx.x) * kSmallWarps + (threadIdx.x >> 5);
  if (col >= n) return;
  const float *brow = b + col * ldb;
  const float bcol = bias != nullptr ? __ldg(bias + col) : 0.f;
  for (int r0 = 0; r0 < m; r0 += 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int64_t kk = lane; kk < k; kk += 32) {
      const float bv = __ldg(brow + kk);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (r0 + i < m) acc[i] = fmaf(__ldg(a + int64_t(r0 + i) * lda + kk), bv, acc[i]);
    }
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = warp_sum(acc[i]);
      if (lane == i) mine = v;
    }
    if (lane < 8 && r0 + lane < m) c[int64_t(r0 + lane) * ldc + col] = __fadd_rn(mine, bcol);
  }
}

// --------------------------------------------------------------------------- host side

size_t gemm_smem_bytes(int stages) {
  return 1024 + size_t(stages) * kStageBytes + size_t(kEpiWarps) * kStageOutBytes + sizeof(Barriers);
}

int gemm_stages() {
  const size_t fixed = gemm_smem_bytes(0);
  return static_cast<int>(std::min<size_t>(kMaxStages, (kSmemLimit - fixed) / kStageBytes));
}

// 2-D K-major f32 map with an explicit row stride (elements).
int make_map_f32_ld(CUtensorMap *map, const void *ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                    int box_rows, bool swizzle) {
  EncodeTiledFn fn = nullptr;
  TB_CHECK(encode_fn(&fn));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TROPNN_B200_ERR_LAUNCH, "cuTensorMapEncodeTiled (f32) failed (%d)", int(r));
  return TROPNN_B200_OK;
}

GemmGeom gemm_geometry(int64_t m, int64_t n, int64_t k) {
  GemmGeom g{};
  g.m = m;
  g.n = n;
  g.kblocks = static_cast<int>(ceil_div(k, kBK));
  g.n_tiles = static_cast<int>(ceil_div(n, kBN));
  const int64_t tiles = ceil_div(m, int64_t(kBM)) * g.n_tiles;
  int splits = 1;
  if (tiles * 4 < int64_t(kTargetUnits) * 3 && g.kblocks >= 2 * kMinKBlocksPerSplit) {
    // Too few output tiles to fill the SMs: cut the contraction, at least 3 k blocks a slice so
    // that the slices' reduction pays for itself.
    splits = static_cast<int>(std::min<int64_t>(
        {int64_t(kMaxSplits), ceil_div(kTargetUnits, tiles), int64_t(g.kblocks / kMinKBlocksPerSplit)}));
  }
  g.kb_per_split = static_cast<int>(ceil_div(g.kblocks, splits));
  g.splits = static_cast<int>(ceil_div(g.kblocks, g.kb_per_split));
  g.units = tiles * g.splits;
  g.stages = gemm_stages();
  return g;
}

size_t gemm_workspace_bytes(const GemmGeom &g) {
  if (g.splits == 1) return 0;
  return WorkspaceCarver::align(size_t(g.units) * kBM * kBN * sizeof(float));
}

}  // namespace

size_t gemm_tf32x3_workspace(int64_t m, int64_t n, int64_t k) {
  if (m <= kSmallRows || n < 1 || k < 1) return 0;
  return gemm_workspace_bytes(gemm_geometry(m, n, k));
}

int gemm_tf32x3_impl(const float *a, int64_t lda, const float *b, int64_t ldb, int64_t m, int64_t n, int64_t k,
                     const float *bias, float *c, int64_t ldc, void *ws, size_t ws_bytes, cudaStream_t stream) {
  TB_REQUIRE(m >= 0 && n >= 1 && k >= 1 && lda >= k && ldb >= k && ldc >= n, TROPNN_B200_ERR_INVALID,
             "gemm_tf32x3: bad sizes m=%lld n=%lld k=%lld lda=%lld ldb=%lld ldc=%lld", (long long)m, (long long)n,
             (long long)k, (long long)lda, (long long)ldb, (long long)ldc);
  TB_REQUIRE(lda % 4 == 0 && ldb % 4 == 0, TROPNN_B200_ERR_INVALID,
             "gemm_tf32x3: lda=%lld / ldb=%lld must be multiples of 4 (16-byte TMA rows)", (long long)lda,
             (long long)ldb);
  TB_REQUIRE(m <= (int64_t(1) << 31) - 1024 && n <= (int64_t(1) << 31) - 1024, TROPNN_B200_ERR_INVALID,
             "gemm_tf32x3: sizes exceed the 32-bit tile coordinates");
  if (m == 0) return TROPNN_B200_OK;
  TB_REQUIRE(a && b && c, TROPNN_B200_ERR_INVALID, "gemm_tf32x3: null pointer");
  auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  TB_REQUIRE(al16(a) && al16(b), TROPNN_B200_ERR_INVALID, "gemm_tf32x3: A and B must be 16-byte aligned");
  if (m <= kSmallRows) {
    TB_REQUIRE(ceil_div(n, int64_t(kSmallWarps)) < (int64_t(1) << 31), TROPNN_B200_ERR_INVALID,
               "gemm_tf32x3: n=%lld exceeds the grid", (long long)n);
    gemm_f32_rows_kernel<<<static_cast<unsigned>(ceil_div(n, int64_t(kSmallWarps))), kSmallWarps * 32, 0, stream>>>(
        a, lda, b, ldb, static_cast<int>(m), n, k, bias, c, ldc);
    return check_launch("gemm_tf32x3");
  }
  GemmGeom g = gemm_geometry(m, n, k);
  g.ldc = ldc;
  g.tma_store = (ldc % 4 == 0 && al16(c)) ? 1 : 0;
  float4 *partial = nullptr;
  if (g.splits > 1) {
    WorkspaceCarver wc(ws, ws_bytes);
    partial = wc.take<float4>(size_t(g.units) * kBM * (kBN / 4));
    TB_REQUIRE(partial != nullptr, TROPNN_B200_ERR_WORKSPACE,
               "gemm_tf32x3: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes,
               gemm_workspace_bytes(g));
  }
  CUtensorMap map_a, map_b, map_c;
  TB_CHECK(make_map_f32_ld(&map_a, a, k, m, lda, kBK, kBM, true));
  TB_CHECK(make_map_f32_ld(&map_b, b, k, n, ldb, kBK, kBN, true));
  if (g.tma_store) {
    // Extent n with row stride ldc: the stores leave columns n..ldc-1 of a padded C alone.
    TB_CHECK(make_map_f32_ld(&map_c, c, n, m, ldc, 32, 32, true));
  } else {
    map_c = map_a;  // unused
  }
  const size_t smem = gemm_smem_bytes(g.stages);
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(gemm_tf32x3_kernel), smem, "gemm_tf32x3"));
  int sms = 0;
  TB_CHECK(sm_count(&sms));
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(g.units, sms));
  gemm_tf32x3_kernel<<<grid, kThreads, smem, stream>>>(map_a, map_b, map_c, g, bias, c, partial);
  TB_CHECK(check_launch("gemm_tf32x3"));
  if (g.splits == 1) return TROPNN_B200_OK;
  // The slices summed in slice order, plus the bias.
  return slice_reduce_impl(kReduceF32, partial, g.splits, g.n_tiles, kBN, m, n, c, TROPNN_B200_F32, ldc, bias,
                           nullptr, TROPNN_B200_F32, 1.f, stream);
}

int transpose_f32_impl(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out, int64_t ldo,
                       cudaStream_t stream) {
  TB_REQUIRE(rows >= 0 && cols >= 0 && ldx >= cols && ldo >= rows, TROPNN_B200_ERR_INVALID,
             "transpose_f32: bad sizes rows=%lld cols=%lld ldx=%lld ldo=%lld", (long long)rows, (long long)cols,
             (long long)ldx, (long long)ldo);
  if (cols == 0 || ldo == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x && out, TROPNN_B200_ERR_INVALID, "transpose_f32: null pointer");
  TB_REQUIRE(ceil_div(ldo, 32) < 65536, TROPNN_B200_ERR_INVALID, "transpose_f32: %lld rows exceed the grid",
             (long long)rows);
  const dim3 grid(static_cast<unsigned>(ceil_div(cols, 32)), static_cast<unsigned>(ceil_div(ldo, 32)));
  transpose_f32_kernel<<<grid, dim3(32, 8), 0, stream>>>(x, rows, cols, ldx, out, ldo);
  return check_launch("transpose_f32");
}

int colsum_f32_impl(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out, cudaStream_t stream) {
  TB_REQUIRE(rows >= 0 && cols >= 0 && ldx >= cols, TROPNN_B200_ERR_INVALID, "colsum_f32: bad sizes");
  if (cols == 0) return TROPNN_B200_OK;
  TB_REQUIRE(x != nullptr || rows == 0, TROPNN_B200_ERR_INVALID, "colsum_f32: null pointer");
  TB_REQUIRE(out != nullptr, TROPNN_B200_ERR_INVALID, "colsum_f32: null pointer");
  colsum_f32_kernel<<<static_cast<unsigned>(ceil_div(cols, 32)), 1024, 0, stream>>>(x, rows, cols, ldx, out);
  return check_launch("colsum_f32");
}

int read_gemm_tf32_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_gemm_tf32_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_tf32_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

size_t tropnn_b200_gemm_tf32x3_workspace_size(int64_t m, int64_t n, int64_t k) {
  return tropnn_b200::gemm_tf32x3_workspace(m, n, k);
}

int tropnn_b200_gemm_tf32x3(const float *a, int64_t lda, const float *b, int64_t ldb, int64_t m, int64_t n, int64_t k,
                            const float *bias, float *c, int64_t ldc, void *workspace, size_t workspace_bytes,
                            void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::gemm_tf32x3_impl(a, lda, b, ldb, m, n, k, bias, c, ldc, workspace, workspace_bytes,
                                         tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_transpose_f32(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out, int64_t ldo,
                              void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::transpose_f32_impl(x, rows, cols, ldx, out, ldo, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_colsum_f32(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::colsum_f32_impl(x, rows, cols, ldx, out, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
