// PairwiseLinear on sm_100a: comparator routing fused with the LUT gather-sum, and the
// straight-through-estimator backward.
//
// Reference behaviour (paths inside the tropnn package):
//   forward   layers/pairwise.py:127-135 (_compute_indices), :99-122 (_lookup_chunked),
//             layers/base.py:76-77 (output_scale); TileLang kernels
//             backends/pairwise_tilelang.py:17-115.
//   backward  autograd of layers/pairwise.py:137-200 (_min_margin_ste / _full_ste) with
//             the surrogates of layers/surrogate.py:9-38; TileLang kernels
//             backends/pairwise_tilelang.py:159-410.
//
// Layout: latent f32 [N, in] row-major; anchors int64 [T, C, 2]; thresholds [T, C];
// lut [T, 2^C, out] (f32/f16/bf16) row-major so a selected LUT row is one contiguous
// `out`-wide vector; indices int64 [N, T]; margins f32 [N, T, C].
#include <cooperative_groups.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace tropnn_b200 {

int bucket_sort_impl(const void *keys, int key_dtype, int64_t rows, int64_t groups, int64_t stride,
                     int64_t buckets, int32_t *perm, int32_t *seg, cudaStream_t stream);
int segment_rowsum_impl(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                        int64_t buckets, const int32_t *perm0, const int32_t *seg0, const float *coef0,
                        float coef_sign0, const int32_t *perm1, const int32_t *seg1, const float *coef1,
                        float coef_sign1, float scale, void *out, int out_dtype, void *bucket_sum,
                        cudaStream_t stream);

namespace {

constexpr int kMaxComparisons = 12;
constexpr int kFwdWarps = 4;
constexpr int kFwdRows = 4;  // rows per CTA in the forward (one per warp)

__device__ __forceinline__ int64_t clamp_feature(int64_t a, int64_t in) { return a < 0 ? 0 : (a >= in ? in - 1 : a); }

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// CTA = 4 warps, kFwdRows rows, one column tile of 32*VEC*NV outputs.
// Phase 1: all threads compute the T route indices of the CTA's rows (and, in the
//          first column tile, write indices + margins).
// Phase 2: each warp sums the selected LUT rows of its rows over the column tile,
//          lanes holding VEC consecutive columns (16-byte loads when aligned).
template <typename LutT, typename ThrT, int VEC, int NV>
__global__ void __launch_bounds__(kFwdWarps * 32) pairwise_forward_kernel(
    const float *__restrict__ x, int64_t rows, int64_t in, const int64_t *__restrict__ anchors,
    const ThrT *__restrict__ thr, int T, int C, const LutT *__restrict__ lut, int64_t out, float out_scale,
    float *__restrict__ y, int64_t *__restrict__ idx_out, float *__restrict__ u_out) {
  extern __shared__ int idx_s[];  // [kFwdRows][T]
  const int64_t row0 = int64_t(blockIdx.x) * kFwdRows;
  const int rows_here = static_cast<int>(min64(kFwdRows, rows - row0));
  const bool write_routes = blockIdx.y == 0;
  const int64_t table_size = int64_t(1) << C;

  for (int task = threadIdx.x; task < rows_here * T; task += kFwdWarps * 32) {
    const int r = task / T;
    const int t = task - r * T;
    const int64_t n = row0 + r;
    const float *xrow = x + n * in;
    int bits = 0;
    // Fully unrolled over the comparison slots so the 2C anchor and latent loads of a
    // table are independent and in flight together.
#pragma unroll
    for (int c = 0; c < kMaxComparisons; ++c) {
      if (c < C) {
        const int64_t e = (int64_t(t) * C + c) * 2;
        const int64_t a = clamp_feature(__ldg(anchors + e), in);
        const int64_t b = clamp_feature(__ldg(anchors + e + 1), in);
        const float u = __fsub_rn(__fsub_rn(__ldg(xrow + a), __ldg(xrow + b)), ldg_f32(thr + int64_t(t) * C + c));
        if (write_routes) u_out[(n * T + t) * C + c] = u;
        bits |= (u > 0.f ? 1 : 0) << c;
      }
    }
    idx_s[r * T + t] = bits;
    if (write_routes) idx_out[n * T + t] = bits;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t col0 = int64_t(blockIdx.y) * (32 * VEC * NV);
  for (int r = warp; r < rows_here; r += kFwdWarps) {
    float acc[NV][VEC];
#pragma unroll
    for (int s = 0; s < NV; ++s)
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[s][e] = 0.f;
    const int *my_idx = idx_s + r * T;
#pragma unroll 4
    for (int t = 0; t < T; ++t) {
      const LutT *lrow = lut + (int64_t(t) * table_size + my_idx[t]) * out;
#pragma unroll
      for (int s = 0; s < NV; ++s) {
        const int64_t col = col0 + int64_t(s) * 32 * VEC + int64_t(lane) * VEC;
        if (col < out) {
          float v[VEC];
          VecLoad<LutT, VEC>::load(lrow + col, v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[s][e] = __fadd_rn(acc[s][e], v[e]);
        }
      }
    }
    float *yrow = y + (row0 + r) * out;
#pragma unroll
    for (int s = 0; s < NV; ++s) {
      const int64_t col = col0 + int64_t(s) * 32 * VEC + int64_t(lane) * VEC;
      if (col < out) {
        if constexpr (VEC % 4 == 0) {
#pragma unroll
          for (int e = 0; e < VEC; e += 4) {
            *reinterpret_cast<float4 *>(yrow + col + e) =
                make_float4(__fmul_rn(acc[s][e], out_scale), __fmul_rn(acc[s][e + 1], out_scale),
                            __fmul_rn(acc[s][e + 2], out_scale), __fmul_rn(acc[s][e + 3], out_scale));
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) yrow[col + e] = __fmul_rn(acc[s][e], out_scale);
        }
      }
    }
  }
}

template <typename LutT, typename ThrT, int VEC, int NV>
int launch_forward(const float *x, int64_t rows, int64_t in, const int64_t *anchors, const void *thr, int T, int C,
                   const void *lut, int64_t out, float out_scale, float *y, int64_t *idx, float *u,
                   cudaStream_t stream) {
  const int64_t col_tiles = ceil_div(out, 32 * VEC * NV);
  const int64_t row_blocks = ceil_div(rows, kFwdRows);
  TB_REQUIRE(row_blocks < (int64_t(1) << 31) && col_tiles < 65536, TROPNN_B200_ERR_INVALID,
             "pairwise_forward: grid too large (items=%lld out=%lld)", (long long)rows, (long long)out);
  const size_t smem = sizeof(int) * kFwdRows * T;
  auto kernel = pairwise_forward_kernel<LutT, ThrT, VEC, NV>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_forward"));
  dim3 grid(static_cast<unsigned>(row_blocks), static_cast<unsigned>(col_tiles));
  kernel<<<grid, kFwdWarps * 32, smem, stream>>>(x, rows, in, anchors, static_cast<const ThrT *>(thr), T, C,
                                                 static_cast<const LutT *>(lut), out, out_scale, y, idx, u);
  return check_launch("pairwise_forward");
}

// Forward for LUTs larger than L2 (config 5: 1024 tables x 256 entries x 4096 f16 columns =
// 2 GiB): pairwise_forward_staged_kernel. A selected LUT row is only reused from L2 while the
// rows that select it pass its table at about the same time, so the CTAs must walk the tables
// in step: a CTA takes a unit of kStageRows rows x one 8 KB column chunk of the LUT rows, and
// the units run in waves of one unit per SM (one launch per wave), whose CTAs start together,
// do the same work per table and so read the LUT from DRAM about once per wave.
//
// A CTA first computes its rows' routes (their latent rows staged in the still idle stage
// ring, a thread per table: anchors and thresholds read once for all the rows), keeps them in
// shared memory and, in the first column chunk, writes them out with the margins. Then one
// producer thread streams, table after table, the unit's selected row slices (kStageRows bulk
// copies of 8 KB, one per producer lane) into a ring of shared-memory slots of kSlotRows row
// slices, each slot with its own full and empty barrier, about 200 KB in flight per SM
// whatever the registers, and 16 consumer warps add 16 bytes of every row slice per thread
// into f32 accumulators (kStageRows x 16 bytes of columns each), in the order of the copies. Per output element
// the tables are summed in table order from 0, as in pairwise_forward_kernel: both kernels
// give identical y, indices and margins. Every wait is bounded (an expired wait raises the
// CTA's abort flag and g_pairwise_error); the producer lets its copies in flight land before
// the CTA exits.
__device__ int g_pairwise_error = 0;

// 16 bytes of LUT values in shared memory as VEC f32.
template <typename LutT, int VEC>
__device__ __forceinline__ void smem_vec16(const uint8_t *p, float (&v)[VEC]) {
  const uint4 q = *reinterpret_cast<const uint4 *>(p);
  if constexpr (std::is_same<LutT, float>::value) {
    v[0] = __uint_as_float(q.x);
    v[1] = __uint_as_float(q.y);
    v[2] = __uint_as_float(q.z);
    v[3] = __uint_as_float(q.w);
  } else {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if constexpr (std::is_same<LutT, __half>::value)
        f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

constexpr int kStageRows = 8;
constexpr int kStageConsumers = 512;                    // 16 warps, 16 bytes of a row slice per thread
constexpr int kStageSliceBytes = kStageConsumers * 16;  // 8 KB of each selected LUT row per unit
constexpr int kSlotRows = 8;                                  // row slices per ring slot
constexpr int kSlotsPerTable = kStageRows / kSlotRows;
constexpr int kSlotBytes = kSlotRows * kStageSliceBytes;
constexpr int kSlotMax = 32;
constexpr int kStageSmemLimit = 227 * 1024;  // dynamic shared memory of one CTA

struct StageBarriers {
  uint64_t full[kSlotMax];
  uint64_t empty[kSlotMax];
  int abort;
};

template <typename LutT, typename ThrT>
__global__ void __launch_bounds__(kStageConsumers + 32, 1) pairwise_forward_staged_kernel(
    const float *__restrict__ x, int64_t rows, int64_t in, const int64_t *__restrict__ anchors,
    const ThrT *__restrict__ thr, int T, int C, const LutT *__restrict__ lut, int64_t out, float out_scale,
    float *__restrict__ y, int64_t *__restrict__ idx_out, float *__restrict__ u_out, int64_t unit0, int64_t groups,
    int slots) {
  constexpr int VEC = 16 / sizeof(LutT);
  constexpr int64_t kSliceCols = kStageSliceBytes / sizeof(LutT);
  extern __shared__ __align__(128) uint8_t stage_smem[];
  uint8_t *ring = stage_smem;  // [slots][kSlotRows][kStageSliceBytes]
  auto *bars = reinterpret_cast<StageBarriers *>(stage_smem + size_t(slots) * kSlotBytes);
  auto *widx = reinterpret_cast<uint16_t *>(bars + 1);  // [kStageRows][T]

  const int64_t unit = unit0 + blockIdx.x;
  const int64_t chunk = unit / groups;  // the units of one column chunk are consecutive
  const int64_t row0 = (unit - chunk * groups) * kStageRows;
  const int rows_here = static_cast<int>(min64(kStageRows, rows - row0));
  const int64_t col0 = chunk * kSliceCols;
  const int64_t slice_cols = min64(kSliceCols, out - col0);
  const uint32_t slice_bytes = static_cast<uint32_t>(slice_cols * sizeof(LutT));
  const int64_t table_size = int64_t(1) << C;
  const bool write_routes = chunk == 0;

  // Routes: as many latent rows as the ring holds at a time, a thread per table.
  float *xs = reinterpret_cast<float *>(ring);
  const int ring_rows = static_cast<int>(min64(rows_here, int64_t(slots) * kSlotBytes / (in * 4)));
  for (int r0 = 0; r0 < rows_here; r0 += ring_rows) {
    const int rn = min(ring_rows, rows_here - r0);
    const float *xb = x + (row0 + r0) * in;
    const int64_t n = rn * in;
    if ((in & 3) == 0 && (reinterpret_cast<uintptr_t>(xb) & 15) == 0) {
      // Four 16-byte loads in flight per thread per pass.
      const float4 *src = reinterpret_cast<const float4 *>(xb);
      float4 *dst = reinterpret_cast<float4 *>(xs);
      const int64_t n4 = n / 4, step = blockDim.x;
      for (int64_t i = threadIdx.x; i < n4; i += 4 * step) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (i + k * step < n4) v[k] = __ldg(src + i + k * step);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (i + k * step < n4) dst[i + k * step] = v[k];
      }
    } else {
      for (int64_t i = threadIdx.x; i < n; i += blockDim.x) xs[i] = __ldg(xb + i);
    }
    __syncthreads();
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      int a[kMaxComparisons], b[kMaxComparisons];
      float th[kMaxComparisons];
#pragma unroll
      for (int c = 0; c < kMaxComparisons; ++c) {
        if (c < C) {
          const int64_t e = (int64_t(t) * C + c) * 2;
          a[c] = static_cast<int>(clamp_feature(__ldg(anchors + e), in));
          b[c] = static_cast<int>(clamp_feature(__ldg(anchors + e + 1), in));
          th[c] = ldg_f32(thr + int64_t(t) * C + c);
        }
      }
      for (int r = 0; r < rn; ++r) {
        const float *xr = xs + int64_t(r) * in;
        const int64_t nt = (row0 + r0 + r) * T + t;
        int bits = 0;
#pragma unroll
        for (int c = 0; c < kMaxComparisons; ++c) {
          if (c < C) {
            const float u = __fsub_rn(__fsub_rn(xr[a[c]], xr[b[c]]), th[c]);
            if (write_routes) u_out[nt * C + c] = u;
            bits |= (u > 0.f ? 1 : 0) << c;
          }
        }
        widx[(r0 + r) * T + t] = static_cast<uint16_t>(bits);
        if (write_routes) idx_out[nt] = bits;
      }
    }
    __syncthreads();
  }
  // The ring's generic reads above come before the bulk copies that write it.
  sm100::fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      sm100::mbar_init(&bars->full[s], 1);
      sm100::mbar_init(&bars->empty[s], kStageConsumers / 32);
    }
    bars->abort = 0;
    sm100::mbar_init_fence();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == kStageConsumers / 32) {
    // Producer warp, one table per pass: lane j < kSlotsPerTable claims the table's slot j
    // (waits for it to be free, posts its byte count), then lane r copies row r.
    int64_t issued = 0;  // slots issued
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      const int64_t q = int64_t(t) * kSlotsPerTable + lane;
      bool lane_ok = true;
      if (lane < kSlotsPerTable) {
        const int slot = static_cast<int>(q % slots);
        if (q >= slots)
          lane_ok = sm100::mbar_wait(&bars->empty[slot], static_cast<uint32_t>(((q / slots) - 1) & 1), &bars->abort,
                                     &g_pairwise_error);
        const int rows_in = max(0, min(kSlotRows, rows_here - lane * kSlotRows));
        if (lane_ok) sm100::mbar_expect_tx(&bars->full[slot], slice_bytes * rows_in);
      }
      if (!__all_sync(0xffffffffu, lane_ok)) {
        ok = false;
        break;
      }
      if (lane < rows_here) {
        const int slot = static_cast<int>((int64_t(t) * kSlotsPerTable + lane / kSlotRows) % slots);
        sm100::bulk_load_1d(ring + size_t(slot) * kSlotBytes + (lane % kSlotRows) * kStageSliceBytes,
                            lut + (int64_t(t) * table_size + widx[lane * T + t]) * out + col0, slice_bytes,
                            &bars->full[slot]);
      }
      issued += kSlotsPerTable;
      __syncwarp();
    }
    if (!ok && lane == 0) {
      // Aborted: the copies already issued land before the CTA's shared memory is released.
      for (int64_t u = issued > slots ? issued - slots : 0; u < issued; ++u)
        sm100::mbar_drain(&bars->full[u % slots], static_cast<uint32_t>((u / slots) & 1));
    }
    return;
  }

  // Consumers: thread i owns columns [i * VEC, i * VEC + VEC) of the slice for every row.
  const int64_t c = int64_t(threadIdx.x) * VEC;
  float acc[kStageRows][VEC];
#pragma unroll
  for (int r = 0; r < kStageRows; ++r)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
  int slot = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int t = 0; t < T && ok; ++t) {
#pragma unroll
    for (int j = 0; j < kSlotsPerTable; ++j) {
      if (ok) {
        if (!sm100::mbar_wait(&bars->full[slot], phase, &bars->abort, &g_pairwise_error)) {
          ok = false;
        } else {
          const uint8_t *src = ring + size_t(slot) * kSlotBytes + threadIdx.x * 16;
#pragma unroll
          for (int rr = 0; rr < kSlotRows; ++rr) {
            const int r = j * kSlotRows + rr;
            if (r < rows_here) {
              float v[VEC];
              smem_vec16<LutT, VEC>(src + rr * kStageSliceBytes, v);
#pragma unroll
              for (int e = 0; e < VEC; ++e) acc[r][e] = __fadd_rn(acc[r][e], v[e]);
            }
          }
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&bars->empty[slot]);
          if (++slot == slots) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
    }
  }
  if (c >= slice_cols) return;
#pragma unroll
  for (int r = 0; r < kStageRows; ++r) {
    if (r < rows_here) {
      float *yrow = y + (row0 + r) * out + col0 + c;
#pragma unroll
      for (int e = 0; e < VEC; e += 4)
        *reinterpret_cast<float4 *>(yrow + e) =
            make_float4(__fmul_rn(acc[r][e], out_scale), __fmul_rn(acc[r][e + 1], out_scale),
                        __fmul_rn(acc[r][e + 2], out_scale), __fmul_rn(acc[r][e + 3], out_scale));
    }
  }
}

// LUT bytes above which the forward runs staged in waves: a LUT within a quarter of L2 stays
// resident there under any schedule, and pairwise_forward_kernel fills the GPU with smaller CTAs.
constexpr int64_t kStagedLutBytes = int64_t(32) << 20;

size_t staged_smem(int slots, int T) {
  return size_t(slots) * kSlotBytes + sizeof(StageBarriers) + sizeof(uint16_t) * kStageRows * T;
}

// Ring slots that fit next to the unit's routes (0 when fewer than two tables' rows fit).
int staged_slots(int T) {
  for (int s = kSlotMax; s >= 2 * kSlotsPerTable; --s)
    if (staged_smem(s, T) <= size_t(kStageSmemLimit)) return s;
  return 0;
}

template <typename LutT, typename ThrT>
int launch_forward_staged(const float *x, int64_t rows, int64_t in, const int64_t *anchors, const void *thr, int T,
                          int C, const void *lut, int64_t out, float out_scale, float *y, int64_t *idx, float *u,
                          cudaStream_t stream) {
  int dev = 0, sms = 0;
  TB_REQUIRE(cudaGetDevice(&dev) == cudaSuccess &&
                 cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0,
             TROPNN_B200_ERR_LAUNCH, "pairwise_forward: device query failed");
  constexpr int64_t kSliceCols = kStageSliceBytes / sizeof(LutT);
  const int slots = staged_slots(T);
  const size_t smem = staged_smem(slots, T);
  const int64_t groups = ceil_div(rows, int64_t(kStageRows));
  const int64_t units = groups * ceil_div(out, kSliceCols);
  auto kernel = pairwise_forward_staged_kernel<LutT, ThrT>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_forward_staged"));
  for (int64_t unit0 = 0; unit0 < units; unit0 += sms) {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(sms, units - unit0));
    kernel<<<grid, kStageConsumers + 32, smem, stream>>>(x, rows, in, anchors, static_cast<const ThrT *>(thr), T, C,
                                                         static_cast<const LutT *>(lut), out, out_scale, y, idx, u,
                                                         unit0, groups, slots);
    TB_CHECK(check_launch("pairwise_forward_staged"));
  }
  return TROPNN_B200_OK;
}

// Forward for a few rows (latency-bound batches): a CTA per row, its threads over the columns,
// eight tables' LUT loads in flight per thread. Each output element is still summed in table
// order from 0, so y, indices and margins are bit-identical to pairwise_forward_kernel's.
constexpr int kFwdRowThreads = 128;
constexpr int64_t kFwdRowCtaRows = 64;

template <typename LutT, typename ThrT, int VEC>
__global__ void __launch_bounds__(kFwdRowThreads) pairwise_forward_rowcta_kernel(
    const float *__restrict__ x, int64_t rows, int64_t in, const int64_t *__restrict__ anchors,
    const ThrT *__restrict__ thr, int T, int C, const LutT *__restrict__ lut, int64_t out, float out_scale,
    float *__restrict__ y, int64_t *__restrict__ idx_out, float *__restrict__ u_out) {
  extern __shared__ int row_idx[];  // [T]
  const int64_t n = blockIdx.x;
  const int64_t table_size = int64_t(1) << C;
  const float *xrow = x + n * in;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    int bits = 0;
#pragma unroll
    for (int c = 0; c < kMaxComparisons; ++c) {
      if (c < C) {
        const int64_t e = (int64_t(t) * C + c) * 2;
        const int64_t a = clamp_feature(__ldg(anchors + e), in);
        const int64_t b = clamp_feature(__ldg(anchors + e + 1), in);
        const float uv = __fsub_rn(__fsub_rn(__ldg(xrow + a), __ldg(xrow + b)), ldg_f32(thr + int64_t(t) * C + c));
        u_out[(n * T + t) * C + c] = uv;
        bits |= (uv > 0.f ? 1 : 0) << c;
      }
    }
    row_idx[t] = bits;
    idx_out[n * T + t] = bits;
  }
  __syncthreads();
  for (int64_t col = int64_t(threadIdx.x) * VEC; col < out; col += int64_t(blockDim.x) * VEC) {
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
#pragma unroll 8
    for (int t = 0; t < T; ++t) {
      float v[VEC];
      VecLoad<LutT, VEC>::load(lut + (int64_t(t) * table_size + row_idx[t]) * out + col, v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = __fadd_rn(acc[e], v[e]);
    }
    float *yrow = y + n * out + col;
#pragma unroll
    for (int e = 0; e < VEC; ++e) yrow[e] = __fmul_rn(acc[e], out_scale);
  }
}

template <typename LutT, typename ThrT, int VEC>
int launch_forward_rowcta(const float *x, int64_t rows, int64_t in, const int64_t *anchors, const void *thr, int T,
                          int C, const void *lut, int64_t out, float out_scale, float *y, int64_t *idx, float *u,
                          cudaStream_t stream) {
  const size_t smem = sizeof(int) * T;
  auto kernel = pairwise_forward_rowcta_kernel<LutT, ThrT, VEC>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_forward_rowcta"));
  kernel<<<static_cast<unsigned>(rows), kFwdRowThreads, smem, stream>>>(
      x, rows, in, anchors, static_cast<const ThrT *>(thr), T, C, static_cast<const LutT *>(lut), out, out_scale, y,
      idx, u);
  return check_launch("pairwise_forward");
}

template <typename LutT, typename ThrT>
int forward_by_width(const float *x, int64_t rows, int64_t in, const int64_t *anchors, const void *thr, int T, int C,
                     const void *lut, int64_t out, float out_scale, float *y, int64_t *idx, float *u,
                     cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(LutT);
  const bool vec_ok = (out % kVec == 0) && (reinterpret_cast<uintptr_t>(lut) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(y) % 16 == 0);
  if (vec_ok) {
    // LUTs far larger than L2 with wide rows: the staged kernel in waves.
    const int64_t lut_bytes = int64_t(T) * (int64_t(1) << C) * out * int64_t(sizeof(LutT));
    if (lut_bytes > kStagedLutBytes && out * int64_t(sizeof(LutT)) >= kStageSliceBytes / 2 && staged_slots(T) > 0 &&
        in * 4 <= int64_t(staged_slots(T)) * kSlotBytes)
      return launch_forward_staged<LutT, ThrT>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                               stream);
    // A few rows: a CTA per row.
    if (rows <= kFwdRowCtaRows)
      return launch_forward_rowcta<LutT, ThrT, kVec>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                                     stream);
    // Column tile of 512 outputs (f32) or 1024 (16-bit) when the rows alone fill the GPU,
    // narrower tiles otherwise.
    if (out > 32 * kVec * 2 || ceil_div(rows, kFwdRows) >= 4 * 148)
      return launch_forward<LutT, ThrT, kVec, 4>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                                 stream);
    return launch_forward<LutT, ThrT, kVec, 1>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                               stream);
  }
  if (rows <= kFwdRowCtaRows)
    return launch_forward_rowcta<LutT, ThrT, 1>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                                stream);
  if (out > 64)
    return launch_forward<LutT, ThrT, 1, 4>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u, stream);
  return launch_forward<LutT, ThrT, 1, 1>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u, stream);
}

template <typename LutT>
int forward_by_thr(int thr_dtype, const float *x, int64_t rows, int64_t in, const int64_t *anchors, const void *thr,
                   int T, int C, const void *lut, int64_t out, float out_scale, float *y, int64_t *idx, float *u,
                   cudaStream_t stream) {
  switch (thr_dtype) {
    case TROPNN_B200_F32:
      return forward_by_width<LutT, float>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u, stream);
    case TROPNN_B200_F16:
      return forward_by_width<LutT, __half>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u, stream);
    default:
      return forward_by_width<LutT, __nv_bfloat16>(x, rows, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                                   stream);
  }
}

// ---------------------------------------------------------------------------
// STE backward
// ---------------------------------------------------------------------------
// One warp per row. For every table the warp reduces sum_o g[o] (lut[nb,o] - lut[cur,o])
// across its lanes, applies the surrogate, and keeps gu (and r*) in shared memory.
// grad_latent is then gathered per input feature through the inverse anchor map, so
// each element is written once in a fixed order (no atomics, no zero fill).
constexpr int kSteMaxWarps = 4;

template <typename LutT, int VEC, bool MIN>
__global__ void __launch_bounds__(kSteMaxWarps * 32) pairwise_ste_kernel(
    const float *__restrict__ g, int64_t rows, int64_t out, float out_scale, const int64_t *__restrict__ idx,
    const float *__restrict__ u, int T, int C, int64_t in, const LutT *__restrict__ lut, int surrogate,
    const int32_t *__restrict__ feat_start, const int32_t *__restrict__ feat_entries, float *__restrict__ grad_x,
    float *__restrict__ gu_out, uint8_t *__restrict__ rstar_out) {
  extern __shared__ float ste_smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = int64_t(blockIdx.x) * warps + warp;
  if (n >= rows) return;
  const int per_row = MIN ? T : T * C;
  float *gu_s = ste_smem + warp * per_row;
  uint8_t *rs_s = reinterpret_cast<uint8_t *>(ste_smem + warps * per_row) + warp * T;
  uint16_t *cur_s = reinterpret_cast<uint16_t *>(ste_smem + warps * per_row + (warps * T + 3) / 4) + warp * T;
  const int64_t table_size = int64_t(1) << C;
  const float *grow = g + n * out;

  if (MIN) {
    // Prologue, lanes over tables: r* = argmin |u| (first on ties), the current bucket,
    // and u at r* (parked in gu_s until lane 0 turns it into gu).
    for (int t = lane; t < T; t += 32) {
      const float *urow = u + (n * T + t) * C;
      int rmin = 0;
      float ustar = __ldg(urow);
      float best = fabsf(ustar);
      for (int c = 1; c < C; ++c) {
        const float v = __ldg(urow + c);
        if (fabsf(v) < best) { best = fabsf(v); rmin = c; ustar = v; }
      }
      rs_s[t] = static_cast<uint8_t>(rmin);
      cur_s[t] = static_cast<uint16_t>(__ldg(idx + n * T + t));
      gu_s[t] = ustar;
    }
    __syncwarp();
    // Four tables per pass: one read of g, eight LUT rows in flight, four reductions.
    constexpr int TB = 4;
    for (int t0 = 0; t0 < T; t0 += TB) {
      const LutT *lcur[TB];
      const LutT *lnb[TB];
      float dot[TB];
#pragma unroll
      for (int k = 0; k < TB; ++k) {
        const int t = min(t0 + k, T - 1);
        const int cur = cur_s[t];
        lcur[k] = lut + (int64_t(t) * table_size + cur) * out;
        lnb[k] = lut + (int64_t(t) * table_size + (cur ^ (1 << rs_s[t]))) * out;
        dot[k] = 0.f;
      }
      for (int64_t col = int64_t(lane) * VEC; col < out; col += 32 * VEC) {
        float gv[VEC];
        VecLoad<float, VEC>::load(grow + col, gv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) gv[e] = __fmul_rn(gv[e], out_scale);
#pragma unroll
        for (int k = 0; k < TB; ++k) {
          float vc[VEC], vn[VEC];
          VecLoad<LutT, VEC>::load(lcur[k] + col, vc);
          VecLoad<LutT, VEC>::load(lnb[k] + col, vn);
#pragma unroll
          for (int e = 0; e < VEC; ++e) dot[k] = fmaf(gv[e], __fsub_rn(vn[e], vc[e]), dot[k]);
        }
      }
#pragma unroll
      for (int k = 0; k < TB; ++k) dot[k] = warp_sum(dot[k]);
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < TB; ++k) {
          const int t = t0 + k;
          if (t < T) {
            const float gu = __fmul_rn(dot[k], surrogate_grad(gu_s[t], surrogate));
            gu_s[t] = gu;
            gu_out[n * T + t] = gu;
            rstar_out[n * T + t] = rs_s[t];
          }
        }
      }
    }
  }

  for (int t = 0; t < (MIN ? 0 : T); ++t) {
    const float *urow = u + (n * T + t) * C;
    const int cur = static_cast<int>(__ldg(idx + n * T + t));
    const LutT *lcur = lut + (int64_t(t) * table_size + cur) * out;
    {
      float dot[kMaxComparisons];
#pragma unroll
      for (int c = 0; c < kMaxComparisons; ++c) dot[c] = 0.f;
      for (int64_t col = int64_t(lane) * VEC; col < out; col += 32 * VEC) {
        float vc[VEC], gv[VEC];
        VecLoad<LutT, VEC>::load(lcur + col, vc);
        VecLoad<float, VEC>::load(grow + col, gv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) gv[e] = __fmul_rn(gv[e], out_scale);
#pragma unroll
        for (int c = 0; c < kMaxComparisons; ++c) {
          if (c < C) {
            const LutT *lnb = lut + (int64_t(t) * table_size + (cur ^ (1 << c))) * out;
            float vn[VEC];
            VecLoad<LutT, VEC>::load(lnb + col, vn);
#pragma unroll
            for (int e = 0; e < VEC; ++e) dot[c] = fmaf(gv[e], __fsub_rn(vn[e], vc[e]), dot[c]);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kMaxComparisons; ++c) {
        if (c < C) {
          const float d = warp_sum(dot[c]);
          if (lane == 0) {
            const float gu = __fmul_rn(d, surrogate_grad(__ldg(urow + c), surrogate));
            gu_s[t * C + c] = gu;
            gu_out[(n * T + t) * C + c] = gu;
          }
        }
      }
    }
  }
  __syncwarp();

  float *gxrow = grad_x + n * in;
  for (int64_t i = lane; i < in; i += 32) {
    const int lo = __ldg(feat_start + i);
    const int hi = __ldg(feat_start + i + 1);
    float acc = 0.f;
    for (int j = lo; j < hi; ++j) {
      const int e = __ldg(feat_entries + j);
      const int tc = e >> 1;
      const int t = tc / C;
      const int c = tc - t * C;
      float v;
      if (MIN) {
        v = (rs_s[t] == c) ? gu_s[t] : 0.f;
      } else {
        v = gu_s[tc];
      }
      acc = (e & 1) ? __fsub_rn(acc, v) : __fadd_rn(acc, v);
    }
    gxrow[i] = acc;
  }
}

// Min-margin STE backward for a few rows (latency-bound batches: the per-row kernel above gives
// each row one warp, which walks all its tables in series): a CTA per row, its warps taking the
// tables in parallel. Every table's dot is formed exactly as above (lane l sums columns l*VEC +
// k*32*VEC in order, then the warp butterfly), and grad_latent is the same per-feature gather,
// so gu, r* and grad_latent are bit-identical to pairwise_ste_kernel's.
constexpr int kSteRowWarps = 8;

template <typename LutT, int VEC>
__global__ void __launch_bounds__(kSteRowWarps * 32) pairwise_ste_rowcta_kernel(
    const float *__restrict__ g, int64_t rows, int64_t out, float out_scale, const int64_t *__restrict__ idx,
    const float *__restrict__ u, int T, int C, int64_t in, const LutT *__restrict__ lut, int surrogate,
    const int32_t *__restrict__ feat_start, const int32_t *__restrict__ feat_entries, float *__restrict__ grad_x,
    float *__restrict__ gu_out, uint8_t *__restrict__ rstar_out) {
  extern __shared__ float row_smem[];
  float *gu_s = row_smem;                                        // [T]
  uint8_t *rs_s = reinterpret_cast<uint8_t *>(gu_s + T);         // [T]
  uint16_t *cur_s = reinterpret_cast<uint16_t *>(rs_s + ((T + 1) & ~1));  // [T]
  const int64_t n = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t table_size = int64_t(1) << C;
  // r* = argmin |u| (first on ties), the current bucket and u at r* per table.
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const float *urow = u + (n * T + t) * C;
    int rmin = 0;
    float ustar = __ldg(urow);
    float best = fabsf(ustar);
    for (int c = 1; c < C; ++c) {
      const float v = __ldg(urow + c);
      if (fabsf(v) < best) {
        best = fabsf(v);
        rmin = c;
        ustar = v;
      }
    }
    rs_s[t] = static_cast<uint8_t>(rmin);
    cur_s[t] = static_cast<uint16_t>(__ldg(idx + n * T + t));
    gu_s[t] = ustar;
  }
  __syncthreads();
  const float *grow = g + n * out;
  for (int t = warp; t < T; t += kSteRowWarps) {
    const int cur = cur_s[t];
    const LutT *lcur = lut + (int64_t(t) * table_size + cur) * out;
    const LutT *lnb = lut + (int64_t(t) * table_size + (cur ^ (1 << rs_s[t]))) * out;
    float dot = 0.f;
    for (int64_t col = int64_t(lane) * VEC; col < out; col += 32 * VEC) {
      float gv[VEC], vc[VEC], vn[VEC];
      VecLoad<float, VEC>::load(grow + col, gv);
      VecLoad<LutT, VEC>::load(lcur + col, vc);
      VecLoad<LutT, VEC>::load(lnb + col, vn);
#pragma unroll
      for (int e = 0; e < VEC; ++e) dot = fmaf(__fmul_rn(gv[e], out_scale), __fsub_rn(vn[e], vc[e]), dot);
    }
    dot = warp_sum(dot);
    if (lane == 0) {
      const float gu = __fmul_rn(dot, surrogate_grad(gu_s[t], surrogate));
      gu_s[t] = gu;
      gu_out[n * T + t] = gu;
      rstar_out[n * T + t] = rs_s[t];
    }
  }
  __syncthreads();
  float *gxrow = grad_x + n * in;
  for (int64_t i = threadIdx.x; i < in; i += blockDim.x) {
    const int lo = __ldg(feat_start + i);
    const int hi = __ldg(feat_start + i + 1);
    float acc = 0.f;
    for (int j = lo; j < hi; ++j) {
      const int e = __ldg(feat_entries + j);
      const int tc = e >> 1;
      const int t = tc / C;
      const int c = tc - t * C;
      const float v = (rs_s[t] == c) ? gu_s[t] : 0.f;
      acc = (e & 1) ? __fsub_rn(acc, v) : __fadd_rn(acc, v);
    }
    gxrow[i] = acc;
  }
}

// Rows below which the min-margin STE takes a CTA per row: fewer rows than about two waves of the
// per-row kernel's 4-warp CTAs.
constexpr int64_t kSteRowCtaRows = 256;

template <typename LutT, int VEC>
int launch_ste(bool use_min, const float *g, int64_t rows, int64_t out, float out_scale, const int64_t *idx,
               const float *u, int T, int C, int64_t in, const void *lut, int surrogate, const int32_t *fs,
               const int32_t *fe, float *gx, float *gu, uint8_t *rs, cudaStream_t stream) {
  if (use_min && rows <= kSteRowCtaRows && rows > 0) {
    const size_t row_smem = sizeof(float) * T + size_t((T + 1) & ~1) + sizeof(uint16_t) * T;
    auto kernel = pairwise_ste_rowcta_kernel<LutT, VEC>;
    TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), row_smem, "pairwise_ste_rowcta"));
    kernel<<<static_cast<unsigned>(rows), kSteRowWarps * 32, row_smem, stream>>>(
        g, rows, out, out_scale, idx, u, T, C, in, static_cast<const LutT *>(lut), surrogate, fs, fe, gx, gu, rs);
    return check_launch("pairwise_ste_backward");
  }
  // gu (f32, one per table or per comparison) + r* (u8) + current bucket (u16) per row.
  const size_t per_warp = sizeof(float) * (use_min ? T : T * C) + 3 * size_t(T);
  int warps = kSteMaxWarps;
  while (warps > 1 && per_warp * warps > 96 * 1024) --warps;
  const size_t smem = per_warp * warps + 16;
  TB_REQUIRE(smem <= 200 * 1024, TROPNN_B200_ERR_INVALID,
             "pairwise_ste_backward: tables*comparisons=%d too large for the per-row shared buffer", T * C);
  const int64_t blocks = ceil_div(rows, warps);
  TB_REQUIRE(blocks < (int64_t(1) << 31), TROPNN_B200_ERR_INVALID, "pairwise_ste_backward: too many rows");
  auto kernel = use_min ? pairwise_ste_kernel<LutT, VEC, true> : pairwise_ste_kernel<LutT, VEC, false>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_ste_backward"));
  kernel<<<static_cast<unsigned>(blocks), warps * 32, smem, stream>>>(
      g, rows, out, out_scale, idx, u, T, C, in, static_cast<const LutT *>(lut), surrogate, fs, fe, gx, gu, rs);
  return check_launch("pairwise_ste_backward");
}

// Min-margin STE backward for LUTs larger than L2 (config 5): pairwise_ste_staged_kernel, staged
// like pairwise_forward_staged_kernel. A unit is kSteRows rows (all `out` columns in one 8 KB
// LUT row slice); units run in waves of one per SM, so that the rows of a wave gather the same
// tables at about the same time and the LUT comes from DRAM about once per wave. Per table, the
// producer warp copies the current bucket's and the min-margin neighbour's row slices of every
// row (2 x kSteRows bulk copies, one per lane) into one slot of a three-table ring. Consumer
// thread i keeps g[row, i*VEC .. i*VEC+VEC) * out_scale of the unit's rows in registers and
// forms its partial of dot = g . (lut[nb] - lut[cur]) per row; a warp reduces its rows'
// partials with a transposed butterfly, and every kSteBatch tables the 16 warps' sums are added
// in warp order, times the surrogate slope at u*, into gu. grad_x is then gathered per input
// feature through the inverse anchor map, as in pairwise_ste_kernel. Four rows per unit keep a
// table's slot at 64 KB (three tables in flight, like the forward) and g in 32 registers.
// Every wait is bounded; after an expired wait the consumers keep taking the same named
// barriers (skipping the work), so none is left waiting.
constexpr int kSteRows = 4;
constexpr int kSteSlotBytes = kSteRows * 2 * kStageSliceBytes;  // [rows][cur, nb][slice]
constexpr int kSteSlotMax = 8;
constexpr int kSteBatch = 16;
constexpr int kSteWarps = kStageConsumers / 32;

struct SteBarriers {
  uint64_t full[kSteSlotMax];
  uint64_t empty[kSteSlotMax];
  int abort;
};

size_t ste_staged_smem(int slots, int T) {
  return size_t(slots) * kSteSlotBytes + sizeof(SteBarriers) + sizeof(float) * kSteBatch * kSteWarps * kSteRows +
         sizeof(uint16_t) * kSteRows * T;
}

// Ring slots (one table each) that fit next to the routes and the batch sums, at least two.
int ste_staged_slots(int T) {
  for (int s = kSteSlotMax; s >= 2; --s)
    if (ste_staged_smem(s, T) <= size_t(kStageSmemLimit)) return s;
  return 0;
}

// Sum over the warp of p[r] for each of 4 rows; lane l ends with row ((l >> 4) & 1) * 2 +
// ((l >> 3) & 1) (a fixed order: deterministic).
__device__ __forceinline__ float warp_sum_rows4(const float (&p)[4], int lane) {
  const bool hi16 = lane & 16, hi8 = lane & 8;
  float q[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = hi16 ? p[k] : p[k + 2];
    const float keep = hi16 ? p[k + 2] : p[k];
    q[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float x = (hi8 ? q[1] : q[0]) + __shfl_xor_sync(0xffffffffu, hi8 ? q[0] : q[1], 8);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x;
}

template <typename LutT>
__global__ void __launch_bounds__(kStageConsumers + 32, 1) pairwise_ste_staged_kernel(
    const float *__restrict__ g, int64_t rows, int64_t out, float out_scale, const int64_t *__restrict__ idx,
    const float *__restrict__ u, int T, int C, int64_t in, const LutT *__restrict__ lut, int surrogate,
    const int32_t *__restrict__ feat_start, const int32_t *__restrict__ feat_entries, float *__restrict__ grad_x,
    float *__restrict__ gu_out, uint8_t *__restrict__ rstar_out, int64_t unit0, int slots) {
  constexpr int VEC = 16 / sizeof(LutT);
  extern __shared__ __align__(128) uint8_t ste_stage_smem[];
  uint8_t *ring = ste_stage_smem;  // [slots][kSteRows][2][kStageSliceBytes]
  auto *bars = reinterpret_cast<SteBarriers *>(ste_stage_smem + size_t(slots) * kSteSlotBytes);
  auto *red = reinterpret_cast<float *>(bars + 1);                                 // [kSteBatch][kSteWarps][kSteRows]
  auto *info = reinterpret_cast<uint16_t *>(red + kSteBatch * kSteWarps * kSteRows);  // cur | r* << 12

  const int64_t row0 = (unit0 + blockIdx.x) * kSteRows;
  const int rows_here = static_cast<int>(min64(kSteRows, rows - row0));
  const uint32_t slice_bytes = static_cast<uint32_t>(out * sizeof(LutT));
  const int64_t table_size = int64_t(1) << C;

  // r* = argmin_c |u| (first on ties) and the current bucket of every (row, table).
  for (int i = threadIdx.x; i < rows_here * T; i += blockDim.x) {
    const int r = i / T;
    const int t = i - r * T;
    const int64_t nt = (row0 + r) * T + t;
    const float *urow = u + nt * C;
    int rmin = 0;
    float best = fabsf(__ldg(urow));
    for (int c = 1; c < C; ++c) {
      const float v = fabsf(__ldg(urow + c));
      if (v < best) {
        best = v;
        rmin = c;
      }
    }
    info[i] = static_cast<uint16_t>(__ldg(idx + nt) | (rmin << 12));
    rstar_out[nt] = static_cast<uint8_t>(rmin);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      sm100::mbar_init(&bars->full[s], 1);
      sm100::mbar_init(&bars->empty[s], kSteWarps);
    }
    bars->abort = 0;
    sm100::mbar_init_fence();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp == kSteWarps) {
    // Producer warp, one table per pass: lane 0 claims the table's slot, then lane l < 2 kSteRows
    // copies row l % kSteRows's current (l < kSteRows) or neighbour row slice.
    bool ok = true;
    int t = 0;
    for (; t < T; ++t) {
      const int slot = t % slots;
      bool lane_ok = true;
      if (lane == 0) {
        if (t >= slots)
          lane_ok = sm100::mbar_wait(&bars->empty[slot], static_cast<uint32_t>(((t / slots) - 1) & 1), &bars->abort,
                                     &g_pairwise_error);
        if (lane_ok) sm100::mbar_expect_tx(&bars->full[slot], 2 * slice_bytes * rows_here);
      }
      if (!__all_sync(0xffffffffu, lane_ok)) {
        ok = false;
        break;
      }
      const int r = lane % kSteRows;
      if (lane < 2 * kSteRows && r < rows_here) {
        const int which = lane / kSteRows;  // 0: current bucket, 1: min-margin neighbour
        const int v = info[r * T + t];
        const int cur = v & 0xfff;
        const int entry = which ? (cur ^ (1 << (v >> 12))) : cur;
        sm100::bulk_load_1d(ring + size_t(slot) * kSteSlotBytes + (r * 2 + which) * kStageSliceBytes,
                            lut + (int64_t(t) * table_size + entry) * out, slice_bytes, &bars->full[slot]);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      for (int q = t > slots ? t - slots : 0; q < t; ++q)
        sm100::mbar_drain(&bars->full[q % slots], static_cast<uint32_t>((q / slots) & 1));
    }
    return;
  }

  // Consumers.
  const int64_t c = int64_t(threadIdx.x) * VEC;
  const bool has_cols = c < out;
  float gv[kSteRows][VEC];
#pragma unroll
  for (int r = 0; r < kSteRows; ++r) {
    if (r < rows_here && has_cols) {
      VecLoad<float, VEC>::load(g + (row0 + r) * out + c, gv[r]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) gv[r][e] = __fmul_rn(gv[r][e], out_scale);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) gv[r][e] = 0.f;
    }
  }
  const int my_row = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
  bool ok = true;
  for (int t = 0; t < T; ++t) {
    const int slot = t % slots;
    float part[kSteRows];
#pragma unroll
    for (int r = 0; r < kSteRows; ++r) part[r] = 0.f;
    if (ok) {
      ok = __all_sync(0xffffffffu, sm100::mbar_wait(&bars->full[slot], static_cast<uint32_t>((t / slots) & 1),
                                                    &bars->abort, &g_pairwise_error));
      if (ok) {
        const uint8_t *src = ring + size_t(slot) * kSteSlotBytes + threadIdx.x * 16;
#pragma unroll
        for (int r = 0; r < kSteRows; ++r) {
          // Columns past `out` and rows past the unit's were not copied: never read them.
          if (has_cols && r < rows_here) {
            float vc[VEC], vn[VEC];
            smem_vec16<LutT, VEC>(src + (r * 2) * kStageSliceBytes, vc);
            smem_vec16<LutT, VEC>(src + (r * 2 + 1) * kStageSliceBytes, vn);
#pragma unroll
            for (int e = 0; e < VEC; ++e) part[r] = fmaf(gv[r][e], __fsub_rn(vn[e], vc[e]), part[r]);
          }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&bars->empty[slot]);
      }
    }
    const int tb = t % kSteBatch;
    const float sum = warp_sum_rows4(part, lane);
    if ((lane & 7) == 0) red[(tb * kSteWarps + warp) * kSteRows + my_row] = sum;
    if (tb == kSteBatch - 1 || t == T - 1) {
      // The batch's dots: the warps' sums in warp order, times the surrogate slope at u*.
      sm100::named_sync(1, kStageConsumers);
      const int t0 = t - tb;
      for (int k = threadIdx.x; k < (tb + 1) * kSteRows; k += kStageConsumers) {
        const int b = k / kSteRows, r = k - b * kSteRows;
        if (r < rows_here) {
          float dot = 0.f;
          for (int w = 0; w < kSteWarps; ++w) dot = __fadd_rn(dot, red[(b * kSteWarps + w) * kSteRows + r]);
          const int64_t nt = (row0 + r) * T + t0 + b;
          const float ustar = __ldg(u + nt * C + (info[r * T + t0 + b] >> 12));
          gu_out[nt] = __fmul_rn(dot, surrogate_grad(ustar, surrogate));
        }
      }
      sm100::named_sync(1, kStageConsumers);
    }
  }

  // grad_x[n, i] = sum over the (table, comparison) entries that read feature i (sign by side)
  // of gu where the comparison is the row's r*, in entry order.
  for (int64_t k = threadIdx.x; k < int64_t(rows_here) * in; k += kStageConsumers) {
    const int r = static_cast<int>(k / in);
    const int64_t i = k - int64_t(r) * in;
    const int64_t n = row0 + r;
    const int lo = __ldg(feat_start + i);
    const int hi = __ldg(feat_start + i + 1);
    float acc = 0.f;
    for (int j = lo; j < hi; ++j) {
      const int e = __ldg(feat_entries + j);
      const int tc = e >> 1;
      const int t = tc / C;
      const int cc = tc - t * C;
      const float v = (info[r * T + t] >> 12) == cc ? gu_out[n * T + t] : 0.f;
      acc = (e & 1) ? __fsub_rn(acc, v) : __fadd_rn(acc, v);
    }
    grad_x[n * in + i] = acc;
  }
}

template <typename LutT>
int launch_ste_staged(const float *g, int64_t rows, int64_t out, float out_scale, const int64_t *idx, const float *u,
                      int T, int C, int64_t in, const void *lut, int surrogate, const int32_t *fs, const int32_t *fe,
                      float *gx, float *gu, uint8_t *rs, cudaStream_t stream) {
  int dev = 0, sms = 0;
  TB_REQUIRE(cudaGetDevice(&dev) == cudaSuccess &&
                 cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0,
             TROPNN_B200_ERR_LAUNCH, "pairwise_ste_backward: device query failed");
  const int slots = ste_staged_slots(T);
  const size_t smem = ste_staged_smem(slots, T);
  auto kernel = pairwise_ste_staged_kernel<LutT>;
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_ste_staged"));
  const int64_t units = ceil_div(rows, int64_t(kSteRows));
  for (int64_t unit0 = 0; unit0 < units; unit0 += sms) {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(sms, units - unit0));
    kernel<<<grid, kStageConsumers + 32, smem, stream>>>(g, rows, out, out_scale, idx, u, T, C, in,
                                                         static_cast<const LutT *>(lut), surrogate, fs, fe, gx, gu,
                                                         rs, unit0, slots);
    TB_CHECK(check_launch("pairwise_ste_staged"));
  }
  return TROPNN_B200_OK;
}

template <typename LutT>
int ste_by_width(bool use_min, const float *g, int64_t rows, int64_t out, float out_scale, const int64_t *idx,
                 const float *u, int T, int C, int64_t in, const void *lut, int surrogate, const int32_t *fs,
                 const int32_t *fe, float *gx, float *gu, uint8_t *rs, cudaStream_t stream) {
  constexpr int kVec = 16 / sizeof(LutT);
  // 16-byte LUT loads need kVec | out; g is f32 so with kVec = 8 two float4 loads.
  const bool vec_ok = (out % kVec == 0) && (reinterpret_cast<uintptr_t>(lut) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(g) % 16 == 0);
  // Min-margin STE over a LUT far larger than L2 whose rows fit one 8 KB slice: staged in waves.
  const int64_t lut_bytes = int64_t(T) * (int64_t(1) << C) * out * int64_t(sizeof(LutT));
  const int64_t row_bytes = out * int64_t(sizeof(LutT));
  if (use_min && vec_ok && lut_bytes > kStagedLutBytes && row_bytes <= kStageSliceBytes &&
      row_bytes >= kStageSliceBytes / 2 && ste_staged_slots(T) > 0 && C <= 12)
    return launch_ste_staged<LutT>(g, rows, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx, gu, rs,
                                   stream);
  if (vec_ok)
    return launch_ste<LutT, kVec>(use_min, g, rows, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx, gu,
                                  rs, stream);
  return launch_ste<LutT, 1>(use_min, g, rows, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx, gu, rs,
                             stream);
}

// ---------------------------------------------------------------------------
// threshold gradient: fixed-order reduction over rows, one launch
// ---------------------------------------------------------------------------
// grad_thresholds[t,c] = -sum_n gu (min mode: rows whose r* == c; full mode: gu[n,t,c]). A
// cluster of kThrSlices CTAs owns 32 tables (one per lane, so every warp load reads 32
// consecutive (row, table) entries); CTA y of the cluster takes row slice y and its warps take
// interleaved rows. Each thread keeps its C sums in its own shared-memory row (stride
// kMaxComparisons + 1: no bank conflicts; min mode adds gu to cell r* only, the same sums as
// adding 0 to the others). Warp partials are combined in warp order, slice partials in slice
// order through distributed shared memory, so the result is deterministic, and nothing goes
// through global memory between the two stages.
constexpr int kThrSlices = 8, kThrWarps = 16, kThrStride = kMaxComparisons + 1;

template <bool MIN, typename OutT>
__global__ void __cluster_dims__(1, kThrSlices, 1) __launch_bounds__(kThrWarps * 32, 1)
    threshold_grad_kernel(const float *__restrict__ gu, const uint8_t *__restrict__ rstar, int64_t rows, int T,
                          int C, OutT *__restrict__ grad) {
  __shared__ float part[kThrWarps * 32 * kThrStride];
  __shared__ float red[32 * kMaxComparisons];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 32 + lane;
  const int64_t per = (rows + kThrSlices - 1) / kThrSlices;
  const int64_t n_begin = per * blockIdx.y, n_end = n_begin + per < rows ? n_begin + per : rows;
  float *mine = part + (warp * 32 + lane) * kThrStride;
#pragma unroll
  for (int c = 0; c < kMaxComparisons; ++c) mine[c] = 0.f;
  if (t < T) {
    constexpr int kUnroll = 16;  // row loads in flight per warp
    for (int64_t n = n_begin + warp; n < n_end; n += kUnroll * kThrWarps) {
      if constexpr (MIN) {
        float v[kUnroll];
        uint32_t r[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t nu = n + int64_t(u) * kThrWarps;
          const bool ok = nu < n_end;
          const int64_t o = (ok ? nu : n) * T + t;
          // r* comes from this library's STE kernel; clamped anyway so that a corrupt one
          // cannot address outside the thread's row.
          r[u] = min(uint32_t(__ldg(rstar + o)), uint32_t(C - 1));
          v[u] = ok ? __ldg(gu + o) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) mine[r[u]] = __fadd_rn(mine[r[u]], v[u]);
      } else {
#pragma unroll 4
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t nu = n + int64_t(u) * kThrWarps;
          if (nu < n_end) {
            const float *row = gu + (nu * T + t) * C;
            for (int c = 0; c < C; ++c) mine[c] = __fadd_rn(mine[c], __ldg(row + c));
          }
        }
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * C; e += kThrWarps * 32) {
    const int l = e / C, c = e - l * C;
    float sum = 0.f;
    for (int w = 0; w < kThrWarps; ++w) sum = __fadd_rn(sum, part[(w * 32 + l) * kThrStride + c]);
    red[e] = sum;
  }
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int share = (32 * C + kThrSlices - 1) / kThrSlices;
  const int slice = static_cast<int>(cluster.block_rank());
  for (int i = threadIdx.x; i < share; i += kThrWarps * 32) {
    const int e = slice * share + i;
    if (e >= 32 * C) break;
    float sum = 0.f;
    for (int y = 0; y < kThrSlices; ++y) sum = __fadd_rn(sum, cluster.map_shared_rank(red, y)[e]);
    const int l = e / C, c = e - l * C;
    const int tt = blockIdx.x * 32 + l;
    if (tt < T) grad[int64_t(tt) * C + c] = from_f32<OutT>(-sum);
  }
  cluster.sync();  // the other CTAs' shared memory stays live until every read is done
}

// ---------------------------------------------------------------------------
// inverse anchor map (one CTA; built once per anchors buffer)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) anchor_index_kernel(const int64_t *__restrict__ anchors, int E, int64_t in,
                                                            int32_t *start, int32_t *__restrict__ entries) {
  __shared__ int tmp[1024];
  const int tid = threadIdx.x;
  for (int64_t i = tid; i <= in; i += 1024) start[i] = 0;
  __syncthreads();
  for (int e = tid; e < E; e += 1024) atomicAdd(start + clamp_feature(anchors[e], in) + 1, 1);
  __syncthreads();
  // In-place exclusive scan of start[1..in]: afterwards start[f+1] = first slot of feature f.
  const int64_t per = (in + 1023) / 1024;
  const int64_t lo = min64(in, tid * per);
  const int64_t hi = min64(in, lo + per);
  int local = 0;
  for (int64_t i = lo; i < hi; ++i) local += start[i + 1];
  tmp[tid] = local;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    int v = tid >= off ? tmp[tid - off] : 0;
    __syncthreads();
    tmp[tid] += v;
    __syncthreads();
  }
  int run = tmp[tid] - local;
  for (int64_t i = lo; i < hi; ++i) {
    int v = start[i + 1];
    start[i + 1] = run;
    run += v;
  }
  __syncthreads();
  // Stable fill in entry order by one warp; start[f+1] is the cursor of feature f and
  // ends as the first slot of feature f+1.
  if (tid < 32) {
    volatile int32_t *cursor = start;
    const unsigned lt_mask = (1u << tid) - 1u;
    for (int base = 0; base < E; base += 32) {
      const int e = base + tid;
      const bool valid = e < E;
      const unsigned active = __ballot_sync(0xffffffffu, valid);
      int64_t f = 0;
      unsigned peers = 0;
      if (valid) {
        f = clamp_feature(anchors[e], in);
        peers = __match_any_sync(active, static_cast<unsigned long long>(f));
        entries[cursor[f + 1] + __popc(peers & lt_mask)] = e;
      }
      __syncwarp();
      if (valid && tid == __ffs(peers) - 1) cursor[f + 1] = cursor[f + 1] + __popc(peers);
      __syncwarp();
    }
  }
}

int validate_pairwise(int64_t items, int64_t in, int64_t tables, int64_t comparisons, int64_t out) {
  TB_REQUIRE(items >= 0 && in >= 1 && tables >= 1 && out >= 1, TROPNN_B200_ERR_INVALID,
             "pairwise: bad sizes items=%lld in=%lld tables=%lld out=%lld", (long long)items, (long long)in,
             (long long)tables, (long long)out);
  TB_REQUIRE(comparisons >= 1 && comparisons <= kMaxComparisons, TROPNN_B200_ERR_INVALID,
             "pairwise: comparisons=%lld outside the supported range [1, %d]", (long long)comparisons,
             kMaxComparisons);
  TB_REQUIRE(tables * comparisons * 2 < (int64_t(1) << 31) && tables < (int64_t(1) << 24), TROPNN_B200_ERR_INVALID,
             "pairwise: tables=%lld too large", (long long)tables);
  TB_REQUIRE(items < (int64_t(1) << 31), TROPNN_B200_ERR_INVALID, "pairwise: items=%lld exceeds int32",
             (long long)items);
  return TROPNN_B200_OK;
}

}  // namespace

int pairwise_forward_impl(const float *latent, int64_t items, int64_t in, const int64_t *anchors, const void *thr,
                          int thr_dtype, int64_t tables, int64_t comparisons, const void *lut, int lut_dtype,
                          int64_t out, float out_scale, float *y, int64_t *idx, float *u, cudaStream_t stream) {
  TB_CHECK(validate_pairwise(items, in, tables, comparisons, out));
  TB_REQUIRE(is_float_dtype(thr_dtype) && is_float_dtype(lut_dtype), TROPNN_B200_ERR_DTYPE,
             "pairwise_forward: thresholds dtype %s / lut dtype %s unsupported", dtype_name(thr_dtype),
             dtype_name(lut_dtype));
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(latent && anchors && thr && lut && y && idx && u, TROPNN_B200_ERR_INVALID,
             "pairwise_forward: null pointer");
  const int T = static_cast<int>(tables), C = static_cast<int>(comparisons);
  switch (lut_dtype) {
    case TROPNN_B200_F32:
      return forward_by_thr<float>(thr_dtype, latent, items, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                   stream);
    case TROPNN_B200_F16:
      return forward_by_thr<__half>(thr_dtype, latent, items, in, anchors, thr, T, C, lut, out, out_scale, y, idx, u,
                                    stream);
    default:
      return forward_by_thr<__nv_bfloat16>(thr_dtype, latent, items, in, anchors, thr, T, C, lut, out, out_scale, y,
                                           idx, u, stream);
  }
}

int read_pairwise_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_pairwise_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_pairwise_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

int pairwise_anchor_index_impl(const int64_t *anchors, int64_t tables, int64_t comparisons, int64_t in,
                               int32_t *fs, int32_t *fe, cudaStream_t stream) {
  TB_CHECK(validate_pairwise(0, in, tables, comparisons, 1));
  TB_REQUIRE(anchors && fs && fe, TROPNN_B200_ERR_INVALID, "pairwise_anchor_index: null pointer");
  anchor_index_kernel<<<1, 1024, 0, stream>>>(anchors, static_cast<int>(tables * comparisons * 2), in, fs, fe);
  return check_launch("pairwise_anchor_index");
}

int pairwise_ste_impl(const float *g, int64_t items, int64_t out, float out_scale, const int64_t *idx, const float *u,
                      const int64_t *anchors, int64_t tables, int64_t comparisons, int64_t in, const void *lut,
                      int lut_dtype, int use_min, int surrogate, const int32_t *fs, const int32_t *fe, float *gx,
                      float *gu, uint8_t *rs, cudaStream_t stream) {
  (void)anchors;
  TB_CHECK(validate_pairwise(items, in, tables, comparisons, out));
  TB_REQUIRE(is_float_dtype(lut_dtype), TROPNN_B200_ERR_DTYPE, "pairwise_ste_backward: lut dtype %s unsupported",
             dtype_name(lut_dtype));
  TB_REQUIRE(surrogate == TROPNN_B200_SURROGATE_FAST_SIGMOID_ODD || surrogate == TROPNN_B200_SURROGATE_IZHIKEVICH,
             TROPNN_B200_ERR_INVALID, "pairwise_ste_backward: unknown surrogate %d", surrogate);
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(g && idx && u && lut && fs && fe && gx && gu && (rs || !use_min), TROPNN_B200_ERR_INVALID,
             "pairwise_ste_backward: null pointer");
  const int T = static_cast<int>(tables), C = static_cast<int>(comparisons);
  const bool m = use_min != 0;
  switch (lut_dtype) {
    case TROPNN_B200_F32:
      return ste_by_width<float>(m, g, items, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx, gu, rs,
                                 stream);
    case TROPNN_B200_F16:
      return ste_by_width<__half>(m, g, items, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx, gu, rs,
                                  stream);
    default:
      return ste_by_width<__nv_bfloat16>(m, g, items, out, out_scale, idx, u, T, C, in, lut, surrogate, fs, fe, gx,
                                         gu, rs, stream);
  }
}

size_t threshold_grad_workspace(int64_t items, int64_t tables, int64_t comparisons) {
  (void)items, (void)tables, (void)comparisons;
  return 0;  // one cluster launch; its stages meet in shared memory
}

int pairwise_threshold_grad_impl(const float *gu, const uint8_t *rs, int64_t items, int64_t tables,
                                 int64_t comparisons, int use_min, void *grad, int grad_dtype, void *ws,
                                 size_t ws_bytes, cudaStream_t stream) {
  TB_CHECK(validate_pairwise(items, 1, tables, comparisons, 1));
  TB_REQUIRE(is_float_dtype(grad_dtype), TROPNN_B200_ERR_DTYPE, "pairwise_threshold_grad: dtype %s unsupported",
             dtype_name(grad_dtype));
  TB_REQUIRE(grad && (items == 0 || (gu && (rs || !use_min))), TROPNN_B200_ERR_INVALID,
             "pairwise_threshold_grad: null pointer");
  (void)ws, (void)ws_bytes;  // needs none (threshold_grad_workspace is 0); kept for the ABI
  const int T = static_cast<int>(tables), C = static_cast<int>(comparisons);
  const dim3 grid(static_cast<unsigned>(ceil_div(tables, int64_t(32))), kThrSlices);
  auto go = [&](auto *out) {
    using OutT = std::remove_pointer_t<decltype(out)>;
    if (use_min)
      threshold_grad_kernel<true, OutT><<<grid, kThrWarps * 32, 0, stream>>>(gu, rs, items, T, C, out);
    else
      threshold_grad_kernel<false, OutT><<<grid, kThrWarps * 32, 0, stream>>>(gu, rs, items, T, C, out);
  };
  switch (grad_dtype) {
    case TROPNN_B200_F32: go(static_cast<float *>(grad)); break;
    case TROPNN_B200_F16: go(static_cast<__half *>(grad)); break;
    default: go(static_cast<__nv_bfloat16 *>(grad)); break;
  }
  return check_launch("pairwise_threshold_grad");
}

struct PairwiseBackwardLayout {
  int32_t *perm, *seg, *fs, *fe;
  float *gu;
  uint8_t *rs;
  void *thr;
  size_t thr_bytes;
};

static size_t pairwise_backward_layout(void *ws, size_t bytes, int64_t items, int64_t tables, int64_t comparisons,
                                       int64_t in, int use_min, PairwiseBackwardLayout *L) {
  WorkspaceCarver c(ws, bytes);
  const int64_t buckets = int64_t(1) << comparisons;
  L->perm = c.take<int32_t>(size_t(items) * tables);
  L->seg = c.take<int32_t>(size_t(tables) * (buckets + 1));
  L->fs = c.take<int32_t>(size_t(in) + 1);
  L->fe = c.take<int32_t>(size_t(tables) * comparisons * 2);
  L->gu = c.take<float>(size_t(items) * tables * (use_min ? 1 : comparisons));
  L->rs = c.take<uint8_t>(size_t(items) * tables);
  L->thr_bytes = threshold_grad_workspace(items, tables, comparisons);
  L->thr = c.take<char>(L->thr_bytes);
  return WorkspaceCarver::align(c.used);
}

bool lut_grad_supported(int64_t tables, int64_t comparisons, int64_t out_features);
struct LutPeer;
int lut_grad_impl(const float *g, int64_t rows, int64_t out_features, const int64_t *indices, int64_t tables,
                  int64_t comparisons, float scale, void *grad_lut, int lut_dtype, const LutPeer *peer,
                  cudaStream_t stream);

int pairwise_backward_impl(const float *g, int64_t items, int64_t out, float out_scale, const int64_t *idx,
                           const float *u, const int64_t *anchors, int64_t tables, int64_t comparisons, int64_t in,
                           const void *lut, int lut_dtype, int use_min, int surrogate, float *gx, void *gthr,
                           int gthr_dtype, void *glut, void *ws, size_t ws_bytes, cudaStream_t stream) {
  TB_CHECK(validate_pairwise(items, in, tables, comparisons, out));
  TB_REQUIRE(gthr == nullptr || gx != nullptr, TROPNN_B200_ERR_INVALID,
             "pairwise_backward: grad_thresholds needs grad_latent (both come from the STE pass)");
  PairwiseBackwardLayout L{};
  const size_t need = pairwise_backward_layout(ws, ws_bytes, items, tables, comparisons, in, use_min, &L);
  TB_REQUIRE(ws != nullptr && need <= ws_bytes, TROPNN_B200_ERR_WORKSPACE,
             "pairwise_backward: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes, need);
  // The one-kernel LUT gradient re-sorts a table's rows per 64-column block: taken up to
  // 1024 columns, the sort + segmented-sum pair above that.
  if (glut != nullptr && lut_grad_supported(tables, comparisons, out) && out <= 1024) {
    TB_CHECK(lut_grad_impl(g, items, out, idx, tables, comparisons, out_scale, glut, lut_dtype, nullptr, stream));
  } else if (glut != nullptr) {
    TB_CHECK(bucket_sort_impl(idx, TROPNN_B200_I64, items, tables, tables, int64_t(1) << comparisons, L.perm, L.seg,
                              stream));
    TB_CHECK(segment_rowsum_impl(g, items, out, out, tables, int64_t(1) << comparisons, L.perm, L.seg, nullptr,
                                 out_scale, nullptr, nullptr, nullptr, 0.f, 1.f, glut, lut_dtype, nullptr, stream));
  }
  if (gx != nullptr) {
    TB_CHECK(pairwise_anchor_index_impl(anchors, tables, comparisons, in, L.fs, L.fe, stream));
    TB_CHECK(pairwise_ste_impl(g, items, out, out_scale, idx, u, anchors, tables, comparisons, in, lut, lut_dtype,
                               use_min, surrogate, L.fs, L.fe, gx, L.gu, L.rs, stream));
    if (gthr != nullptr)
      TB_CHECK(pairwise_threshold_grad_impl(L.gu, L.rs, items, tables, comparisons, use_min, gthr, gthr_dtype, L.thr,
                                            L.thr_bytes, stream));
  }
  return TROPNN_B200_OK;
}

size_t pairwise_backward_workspace(int64_t items, int64_t tables, int64_t comparisons, int64_t in, int use_min) {
  if (items < 0 || tables < 1 || comparisons < 1 || comparisons > kMaxComparisons || in < 1) return 0;
  PairwiseBackwardLayout L{};
  return pairwise_backward_layout(nullptr, 0, items, tables, comparisons, in, use_min, &L);
}

}  // namespace tropnn_b200

extern "C" {

int tropnn_b200_pairwise_forward(const float *latent, int64_t items, int64_t in_features, const int64_t *anchors,
                                 const void *thresholds, int thresholds_dtype, int64_t tables, int64_t comparisons,
                                 const void *lut, int lut_dtype, int64_t out_features, float output_scale,
                                 float *out, int64_t *indices, float *margins, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::pairwise_forward_impl(latent, items, in_features, anchors, thresholds, thresholds_dtype,
                                              tables, comparisons, lut, lut_dtype, out_features, output_scale, out,
                                              indices, margins, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_pairwise_anchor_index(const int64_t *anchors, int64_t tables, int64_t comparisons,
                                      int64_t in_features, int32_t *feat_start, int32_t *feat_entries, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::pairwise_anchor_index_impl(anchors, tables, comparisons, in_features, feat_start,
                                                   feat_entries, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_pairwise_ste_backward(const float *grad_out, int64_t items, int64_t out_features, float output_scale,
                                      const int64_t *indices, const float *margins, const int64_t *anchors,
                                      int64_t tables, int64_t comparisons, int64_t in_features, const void *lut,
                                      int lut_dtype, int use_min_margin_ste, int surrogate, const int32_t *feat_start,
                                      const int32_t *feat_entries, float *grad_latent, float *gu, uint8_t *rstar,
                                      void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::pairwise_ste_impl(grad_out, items, out_features, output_scale, indices, margins, anchors,
                                          tables, comparisons, in_features, lut, lut_dtype, use_min_margin_ste,
                                          surrogate, feat_start, feat_entries, grad_latent, gu, rstar,
                                          tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

size_t tropnn_b200_pairwise_threshold_grad_workspace_size(int64_t items, int64_t tables, int64_t comparisons) {
  if (items < 0 || tables < 1 || comparisons < 1) return 0;
  return tropnn_b200::threshold_grad_workspace(items, tables, comparisons);
}

int tropnn_b200_pairwise_threshold_grad(const float *gu, const uint8_t *rstar, int64_t items, int64_t tables,
                                        int64_t comparisons, int use_min_margin_ste, void *grad_thresholds,
                                        int grad_dtype, void *workspace, size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::pairwise_threshold_grad_impl(gu, rstar, items, tables, comparisons, use_min_margin_ste,
                                                     grad_thresholds, grad_dtype, workspace, workspace_bytes,
                                                     tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

size_t tropnn_b200_pairwise_backward_workspace_size(int64_t items, int64_t tables, int64_t comparisons,
                                                    int64_t in_features, int use_min_margin_ste) {
  return tropnn_b200::pairwise_backward_workspace(items, tables, comparisons, in_features, use_min_margin_ste);
}

int tropnn_b200_pairwise_backward(const float *grad_out, int64_t items, int64_t out_features, float output_scale,
                                  const int64_t *indices, const float *margins, const int64_t *anchors,
                                  int64_t tables, int64_t comparisons, int64_t in_features, const void *lut,
                                  int lut_dtype, int use_min_margin_ste, int surrogate, float *grad_latent,
                                  void *grad_thresholds, int grad_thresholds_dtype, void *grad_lut, void *workspace,
                                  size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::pairwise_backward_impl(grad_out, items, out_features, output_scale, indices, margins, anchors,
                                               tables, comparisons, in_features, lut, lut_dtype, use_min_margin_ste,
                                               surrogate, grad_latent, grad_thresholds, grad_thresholds_dtype,
                                               grad_lut, workspace, workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
