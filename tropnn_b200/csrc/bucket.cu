// Deterministic gradient scatter for routed layers.
//
// The reference scatters per-row gradients into [group, bucket, width] tables with
// atomics (backends/pairwise_tilelang.py:118-156 `T.atomic_add(grad_lut[...])`,
// backends/triton_backward.py:224-305 `tl.atomic_add(grad_code...)`) or with dense
// one-hot einsums (layers/tropical_exact.py:208-234). Here the scatter is turned into
// a gather: a stable counting sort groups the rows of every (group, bucket), then one
// warp per bucket sums its rows and writes the table entry exactly once. No zeroing,
// no atomics, and the summation order is fixed (ascending row inside a bucket), so
// the result is bit-reproducible run to run.
#include <type_traits>

#include "common.cuh"

namespace tropnn_b200 {

namespace {

constexpr int kSortWarps = 8;
constexpr int kSortThreads = kSortWarps * 32;
constexpr int kMaxBuckets = 4096;

template <typename K>
__device__ __forceinline__ int load_key(const K *keys, int64_t n, int64_t stride, int64_t g, int buckets) {
  int k = static_cast<int>(__ldg(keys + n * stride + g));
  // Keys come from this library's own route kernels and are always < buckets; clamp
  // anyway so that a corrupt key can never write out of bounds.
  return k < 0 ? 0 : (k >= buckets ? buckets - 1 : k);
}

// Exclusive scan of `vals[0..count)` in shared memory by one CTA of kSortThreads
// threads. `tmp` holds kSortThreads ints. Returns the total.
__device__ int block_exclusive_scan(int *vals, int count, int *tmp) {
  const int tid = threadIdx.x;
  const int per = (count + kSortThreads - 1) / kSortThreads;
  const int lo = min(count, tid * per);
  const int hi = min(count, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += vals[i];
  tmp[tid] = local;
  __syncthreads();
  // Hillis-Steele over the per-thread sums (kSortThreads is small).
  for (int off = 1; off < kSortThreads; off <<= 1) {
    int v = (tid >= off) ? tmp[tid - off] : 0;
    __syncthreads();
    tmp[tid] += v;
    __syncthreads();
  }
  int run = tmp[tid] - local;  // exclusive prefix of this thread's range
  const int total = tmp[kSortThreads - 1];
  for (int i = lo; i < hi; ++i) {
    int v = vals[i];
    vals[i] = run;
    run += v;
  }
  __syncthreads();
  return total;
}

// Keys of up to kSortTileRows rows are staged in shared memory (uint16) at a time, with
// every thread issuing independent loads, so the strided key column is read once per
// pass with full memory-level parallelism.
constexpr int kSortTileRows = 16384;

template <typename K>
__device__ __forceinline__ void stage_keys(const K *__restrict__ keys, int64_t tile0, int tile_rows, int64_t stride,
                                           int64_t g, int buckets, uint16_t *keys_s) {
#pragma unroll 8
  for (int i = threadIdx.x; i < tile_rows; i += kSortThreads)
    keys_s[i] = static_cast<uint16_t>(load_key(keys, tile0 + i, stride, g, buckets));
}

// Stable counting sort of one group's rows by key (one CTA per group).
// Pass 1 counts every bucket (shared-memory atomics on integers: order-free), the
// exclusive scan gives the bucket starts. Pass 2 walks the tiles in row order; inside
// a tile warp w owns a contiguous run of rows, so
//   position = bucket start + rows of earlier tiles + rows of earlier warps + rank in warp
// keeps rows of a bucket in ascending order.
template <typename K>
__global__ void __launch_bounds__(kSortThreads) bucket_sort_kernel(const K *__restrict__ keys, int64_t rows,
                                                                   int64_t stride, int buckets,
                                                                   int32_t *__restrict__ perm,
                                                                   int32_t *__restrict__ seg) {
  extern __shared__ int smem[];
  int *counts = smem;                            // [kSortWarps][buckets]
  int *base = counts + kSortWarps * buckets;     // [buckets] running start per bucket
  int *tmp = base + buckets;                     // [kSortThreads]
  uint16_t *keys_s = reinterpret_cast<uint16_t *>(tmp + kSortThreads);  // [kSortTileRows]
  const int64_t g = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int tiles = static_cast<int>((rows + kSortTileRows - 1) / kSortTileRows);

  for (int b = threadIdx.x; b < buckets; b += kSortThreads) base[b] = 0;
  __syncthreads();
  for (int tile = 0; tile < tiles; ++tile) {
    const int64_t tile0 = int64_t(tile) * kSortTileRows;
    const int tile_rows = static_cast<int>(min64(kSortTileRows, rows - tile0));
    if (tiles > 1 || tile == 0) {
      stage_keys(keys, tile0, tile_rows, stride, g, buckets, keys_s);
      __syncthreads();
    }
    for (int i = threadIdx.x; i < tile_rows; i += kSortThreads) atomicAdd(base + keys_s[i], 1);
    __syncthreads();
  }
  block_exclusive_scan(base, buckets, tmp);
  int32_t *my_seg = seg + g * (buckets + 1);
  for (int b = threadIdx.x; b < buckets; b += kSortThreads) my_seg[b] = base[b];
  if (threadIdx.x == 0) my_seg[buckets] = static_cast<int32_t>(rows);

  int32_t *my_perm = perm + g * rows;
  int *my_counts = counts + warp * buckets;
  for (int tile = 0; tile < tiles; ++tile) {
    const int64_t tile0 = int64_t(tile) * kSortTileRows;
    const int tile_rows = static_cast<int>(min64(kSortTileRows, rows - tile0));
    if (tiles > 1) {
      __syncthreads();
      stage_keys(keys, tile0, tile_rows, stride, g, buckets, keys_s);
    }
    for (int i = threadIdx.x; i < kSortWarps * buckets; i += kSortThreads) counts[i] = 0;
    __syncthreads();
    // Contiguous run of the tile per warp, a multiple of 32 rows long.
    const int per_warp = ((tile_rows + kSortWarps - 1) / kSortWarps + 31) & ~31;
    const int start = min(tile_rows, warp * per_warp);
    const int end = min(tile_rows, start + per_warp);
    for (int r0 = start; r0 < end; r0 += 32) {
      const int r = r0 + lane;
      const bool valid = r < end;
      const unsigned active = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int key = keys_s[r];
        const unsigned peers = __match_any_sync(active, key);
        if (lane == __ffs(peers) - 1) my_counts[key] += __popc(peers);
      }
      __syncwarp();
    }
    __syncthreads();
    for (int b = threadIdx.x; b < buckets; b += kSortThreads) {
      int run = base[b];
      for (int w = 0; w < kSortWarps; ++w) {
        const int c = counts[w * buckets + b];
        counts[w * buckets + b] = run;
        run += c;
      }
      base[b] = run;
    }
    __syncthreads();
    for (int r0 = start; r0 < end; r0 += 32) {
      const int r = r0 + lane;
      const bool valid = r < end;
      const unsigned active = __ballot_sync(0xffffffffu, valid);
      int key = 0;
      unsigned peers = 0;
      if (valid) {
        key = keys_s[r];
        peers = __match_any_sync(active, key);
        my_perm[my_counts[key] + __popc(peers & lt_mask)] = static_cast<int32_t>(tile0 + r);
      }
      __syncwarp();
      if (valid && lane == __ffs(peers) - 1) my_counts[key] += __popc(peers);
      __syncwarp();
    }
  }
}

// ---------------------------------------------------------------------------
// segmented row sums
// ---------------------------------------------------------------------------

constexpr int kSegWarps = 4;

template <typename OutT, int VEC>
__device__ __forceinline__ void store_vec(OutT *p, const float *v) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) p[i] = from_f32<OutT>(v[i]);
}
template <>
__device__ __forceinline__ void store_vec<float, 4>(float *p, const float *v) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

struct SegList {
  const int32_t *perm;
  const int32_t *seg;
  const float *coef;
  float sign;
};

template <typename VT, int VEC, int NV>
__device__ __forceinline__ void accumulate_list(const SegList &L, const VT *__restrict__ values, int64_t rows,
                                                int64_t ld, int64_t groups, int buckets, int64_t g, int b,
                                                int64_t col0, int64_t width, float (&acc)[NV][VEC],
                                                float &coef_total) {
  const int lane = threadIdx.x & 31;
  const int32_t *segp = L.seg + g * (buckets + 1);
  const int lo = __ldg(segp + b);
  const int hi = __ldg(segp + b + 1);
  const int32_t *permp = L.perm + g * rows;
  int j = lo;
  // Four rows per pass keep 4*NV vector loads in flight; the accumulation order (ascending
  // position in the bucket) is the same as the one-row loop below.
  for (; j + 4 <= hi; j += 4) {
    int64_t n[4];
    float c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) n[u] = __ldg(permp + j + u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      c[u] = L.coef ? __fmul_rn(L.sign, __ldg(L.coef + n[u] * groups + g)) : L.sign;
      coef_total += c[u];
    }
#pragma unroll
    for (int s = 0; s < NV; ++s) {
      const int64_t col = col0 + int64_t(s) * 32 * VEC + int64_t(lane) * VEC;
      if (col < width) {
        float v[4][VEC];
#pragma unroll
        for (int u = 0; u < 4; ++u) VecLoad<VT, VEC>::load(values + n[u] * ld + col, v[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[s][e] = fmaf(c[u], v[u][e], acc[s][e]);
      }
    }
  }
  for (; j < hi; ++j) {
    const int64_t n = __ldg(permp + j);
    const float c = L.coef ? __fmul_rn(L.sign, __ldg(L.coef + n * groups + g)) : L.sign;
    coef_total += c;
    const VT *vrow = values + n * ld;
#pragma unroll
    for (int s = 0; s < NV; ++s) {
      const int64_t col = col0 + int64_t(s) * 32 * VEC + int64_t(lane) * VEC;
      if (col < width) {
        float v[VEC];
        VecLoad<VT, VEC>::load(vrow + col, v);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[s][e] = fmaf(c, v[e], acc[s][e]);
      }
    }
  }
}

template <typename OutT, int VEC, int NV, typename VT = float>
__global__ void __launch_bounds__(kSegWarps * 32) segment_rowsum_kernel(
    const VT *__restrict__ values, int64_t rows, int64_t width, int64_t ld, int64_t groups, int buckets,
    SegList l0, SegList l1, bool has_l1, float scale, OutT *__restrict__ out, OutT *__restrict__ bucket_sum,
    const uint32_t *__restrict__ absmax = nullptr) {
  // Half-precision values carry the power-of-two gradient scale of *absmax; undone here (exact).
  if (absmax != nullptr) scale = __fmul_rn(scale, pow2_inverse(grad_scale_of(absmax)));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quads = (buckets + kSegWarps - 1) / kSegWarps;
  const int64_t g = blockIdx.x / quads;
  const int b = (blockIdx.x % quads) * kSegWarps + warp;
  if (b >= buckets) return;
  const int64_t col0 = int64_t(blockIdx.y) * (32 * VEC * NV);

  float acc[NV][VEC];
#pragma unroll
  for (int s = 0; s < NV; ++s)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[s][e] = 0.f;
  float coef_total = 0.f;
  accumulate_list<VT, VEC, NV>(l0, values, rows, ld, groups, buckets, g, b, col0, width, acc, coef_total);
  if (has_l1)
    accumulate_list<VT, VEC, NV>(l1, values, rows, ld, groups, buckets, g, b, col0, width, acc, coef_total);

  OutT *orow = out + (g * buckets + b) * width;
#pragma unroll
  for (int s = 0; s < NV; ++s) {
    const int64_t col = col0 + int64_t(s) * 32 * VEC + int64_t(lane) * VEC;
    if (col < width) {
      float v[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) v[e] = __fmul_rn(acc[s][e], scale);
      store_vec<OutT, VEC>(orow + col, v);
    }
  }
  if (bucket_sum != nullptr && blockIdx.y == 0 && lane == 0) {
    bucket_sum[g * buckets + b] = from_f32<OutT>(__fmul_rn(coef_total, scale));
  }
}

template <typename OutT, int VEC, int NV>
int launch_segment_rowsum(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                          int64_t buckets, SegList l0, SegList l1, bool has_l1, float scale, void *out,
                          void *bucket_sum, cudaStream_t stream) {
  const int64_t quads = ceil_div(buckets, kSegWarps);
  const int64_t col_tiles = width > 0 ? ceil_div(width, 32 * VEC * NV) : 1;
  TB_REQUIRE(groups * quads < (int64_t(1) << 31) && col_tiles < 65536, TROPNN_B200_ERR_INVALID,
             "segment_rowsum: grid too large (groups=%lld buckets=%lld width=%lld)", (long long)groups,
             (long long)buckets, (long long)width);
  dim3 grid(static_cast<unsigned>(groups * quads), static_cast<unsigned>(col_tiles));
  segment_rowsum_kernel<OutT, VEC, NV><<<grid, kSegWarps * 32, 0, stream>>>(
      values, rows, width, ld, groups, static_cast<int>(buckets), l0, l1, has_l1, scale,
      static_cast<OutT *>(out), static_cast<OutT *>(bucket_sum));
  return check_launch("segment_rowsum");
}

template <typename OutT>
int dispatch_segment_rowsum(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                            int64_t buckets, SegList l0, SegList l1, bool has_l1, float scale, void *out,
                            void *bucket_sum, cudaStream_t stream) {
  const bool vec4 = (width % 4 == 0) && (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(values) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(out) % (4 * sizeof(OutT)) == 0);
  // Enough CTAs to fill 148 SMs several times over before widening the column tile.
  const int64_t quads = ceil_div(buckets, kSegWarps);
  if (vec4) {
    if (groups * quads * ceil_div(width, 512) >= 4 * 148)
      return launch_segment_rowsum<OutT, 4, 4>(values, rows, width, ld, groups, buckets, l0, l1, has_l1, scale,
                                               out, bucket_sum, stream);
    if (groups * quads * ceil_div(width, 256) >= 4 * 148 || width > 128)
      return launch_segment_rowsum<OutT, 4, 2>(values, rows, width, ld, groups, buckets, l0, l1, has_l1, scale,
                                               out, bucket_sum, stream);
    return launch_segment_rowsum<OutT, 4, 1>(values, rows, width, ld, groups, buckets, l0, l1, has_l1, scale,
                                             out, bucket_sum, stream);
  }
  if (width > 64)
    return launch_segment_rowsum<OutT, 1, 4>(values, rows, width, ld, groups, buckets, l0, l1, has_l1, scale,
                                             out, bucket_sum, stream);
  return launch_segment_rowsum<OutT, 1, 2>(values, rows, width, ld, groups, buckets, l0, l1, has_l1, scale, out,
                                           bucket_sum, stream);
}

}  // namespace

int bucket_sort_impl(const void *keys, int key_dtype, int64_t rows, int64_t groups, int64_t stride,
                     int64_t buckets, int32_t *perm, int32_t *seg, cudaStream_t stream) {
  TB_REQUIRE(rows >= 0 && groups >= 0 && stride >= groups, TROPNN_B200_ERR_INVALID,
             "bucket_sort: bad sizes rows=%lld groups=%lld stride=%lld", (long long)rows, (long long)groups,
             (long long)stride);
  TB_REQUIRE(buckets >= 1 && buckets <= kMaxBuckets, TROPNN_B200_ERR_INVALID,
             "bucket_sort: buckets=%lld outside [1, %d]", (long long)buckets, kMaxBuckets);
  TB_REQUIRE(rows < (int64_t(1) << 31), TROPNN_B200_ERR_INVALID, "bucket_sort: rows=%lld exceeds int32",
             (long long)rows);
  TB_REQUIRE(is_index_dtype(key_dtype), TROPNN_B200_ERR_DTYPE, "bucket_sort: key dtype %s is not an index dtype",
             dtype_name(key_dtype));
  if (groups == 0) return TROPNN_B200_OK;
  TB_REQUIRE(seg != nullptr && ((keys != nullptr && perm != nullptr) || rows == 0), TROPNN_B200_ERR_INVALID,
             "bucket_sort: null pointer");
  const size_t smem = sizeof(int) * (kSortWarps * buckets + buckets + kSortThreads) +
                      sizeof(uint16_t) * static_cast<size_t>(min64(rows, kSortTileRows));
  const int nb = static_cast<int>(buckets);
  const unsigned grid = static_cast<unsigned>(groups);
  switch (key_dtype) {
    case TROPNN_B200_U8:
      TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(bucket_sort_kernel<uint8_t>), smem, "bucket_sort"));
      bucket_sort_kernel<uint8_t><<<grid, kSortThreads, smem, stream>>>(static_cast<const uint8_t *>(keys), rows,
                                                                         stride, nb, perm, seg);
      break;
    case TROPNN_B200_I16:
      TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(bucket_sort_kernel<int16_t>), smem, "bucket_sort"));
      bucket_sort_kernel<int16_t><<<grid, kSortThreads, smem, stream>>>(static_cast<const int16_t *>(keys), rows,
                                                                         stride, nb, perm, seg);
      break;
    default:
      TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(bucket_sort_kernel<int64_t>), smem, "bucket_sort"));
      bucket_sort_kernel<int64_t><<<grid, kSortThreads, smem, stream>>>(static_cast<const int64_t *>(keys), rows,
                                                                         stride, nb, perm, seg);
      break;
  }
  return check_launch("bucket_sort");
}

// segment_rowsum over half-precision values (one list, no coefficients): out[g, b, :] = scale /
// s * sum over the bucket's rows of values[n, :], where the values are x * s rounded to the
// parameter dtype and s is the power-of-two gradient scale of *absmax (tropnn_b200_split_half with
// the same word). Half the bytes of the f32 rows per gathered row; used for the LUT gradient of
// half-precision Pairwise layers, whose result is rounded to that dtype anyway.
int segment_rowsum_half_impl(const void *values, int value_dtype, int64_t rows, int64_t width, int64_t ld,
                             int64_t groups, int64_t buckets, const int32_t *perm, const int32_t *seg, float scale,
                             const uint32_t *absmax, void *out, int out_dtype, cudaStream_t stream) {
  TB_REQUIRE(value_dtype == TROPNN_B200_F16 || value_dtype == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "segment_rowsum_half: value dtype %s unsupported", dtype_name(value_dtype));
  TB_REQUIRE(is_float_dtype(out_dtype), TROPNN_B200_ERR_DTYPE, "segment_rowsum_half: out dtype %s unsupported",
             dtype_name(out_dtype));
  TB_REQUIRE(rows >= 0 && width >= 0 && groups >= 0 && buckets >= 1 && ld >= width && width % 8 == 0 && ld % 8 == 0,
             TROPNN_B200_ERR_INVALID,
             "segment_rowsum_half: bad sizes rows=%lld width=%lld ld=%lld (width and ld multiples of 8)",
             (long long)rows, (long long)width, (long long)ld);
  if (groups == 0 || width == 0) return TROPNN_B200_OK;
  TB_REQUIRE(out != nullptr && seg != nullptr && (rows == 0 || (values != nullptr && perm != nullptr)),
             TROPNN_B200_ERR_INVALID, "segment_rowsum_half: null pointer");
  TB_REQUIRE(reinterpret_cast<uintptr_t>(values) % 16 == 0, TROPNN_B200_ERR_INVALID,
             "segment_rowsum_half: values must be 16-byte aligned");
  const SegList l0{perm, seg, nullptr, 1.f};
  const SegList none{nullptr, nullptr, nullptr, 0.f};
  constexpr int kVec = 8, kNv = 4;
  const int64_t quads = ceil_div(buckets, kSegWarps);
  const int64_t col_tiles = ceil_div(width, int64_t(32 * kVec * kNv));
  TB_REQUIRE(groups * quads < (int64_t(1) << 31) && col_tiles < 65536, TROPNN_B200_ERR_INVALID,
             "segment_rowsum_half: grid too large");
  const dim3 grid(static_cast<unsigned>(groups * quads), static_cast<unsigned>(col_tiles));
  auto go = [&](auto *vt, auto *ot) {
    using VT = std::remove_pointer_t<decltype(vt)>;
    using OT = std::remove_pointer_t<decltype(ot)>;
    segment_rowsum_kernel<OT, kVec, kNv, VT><<<grid, kSegWarps * 32, 0, stream>>>(
        static_cast<const VT *>(values), rows, width, ld, groups, static_cast<int>(buckets), l0, none, false, scale,
        static_cast<OT *>(out), nullptr, absmax);
  };
  const bool f16 = value_dtype == TROPNN_B200_F16;
  switch (out_dtype) {
    case TROPNN_B200_F32:
      f16 ? go(static_cast<__half *>(nullptr), static_cast<float *>(nullptr))
          : go(static_cast<__nv_bfloat16 *>(nullptr), static_cast<float *>(nullptr));
      break;
    case TROPNN_B200_F16:
      f16 ? go(static_cast<__half *>(nullptr), static_cast<__half *>(nullptr))
          : go(static_cast<__nv_bfloat16 *>(nullptr), static_cast<__half *>(nullptr));
      break;
    default:
      f16 ? go(static_cast<__half *>(nullptr), static_cast<__nv_bfloat16 *>(nullptr))
          : go(static_cast<__nv_bfloat16 *>(nullptr), static_cast<__nv_bfloat16 *>(nullptr));
      break;
  }
  return check_launch("segment_rowsum_half");
}

int segment_rowsum_impl(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                        int64_t buckets, const int32_t *perm0, const int32_t *seg0, const float *coef0,
                        float coef_sign0, const int32_t *perm1, const int32_t *seg1, const float *coef1,
                        float coef_sign1, float scale, void *out, int out_dtype, void *bucket_sum,
                        cudaStream_t stream) {
  TB_REQUIRE(rows >= 0 && width >= 0 && groups >= 0 && buckets >= 1 && ld >= width, TROPNN_B200_ERR_INVALID,
             "segment_rowsum: bad sizes rows=%lld width=%lld ld=%lld groups=%lld buckets=%lld", (long long)rows,
             (long long)width, (long long)ld, (long long)groups, (long long)buckets);
  TB_REQUIRE(is_float_dtype(out_dtype), TROPNN_B200_ERR_DTYPE, "segment_rowsum: out dtype %s unsupported",
             dtype_name(out_dtype));
  TB_REQUIRE(seg0 != nullptr && (perm0 != nullptr || rows == 0), TROPNN_B200_ERR_INVALID,
             "segment_rowsum: list0 is required");
  TB_REQUIRE(rows == 0 || (perm1 == nullptr) == (seg1 == nullptr), TROPNN_B200_ERR_INVALID,
             "segment_rowsum: perm1 and seg1 must both be set or both be NULL");
  if (groups == 0 || (width == 0 && bucket_sum == nullptr)) return TROPNN_B200_OK;
  TB_REQUIRE(out != nullptr && (values != nullptr || rows == 0), TROPNN_B200_ERR_INVALID,
             "segment_rowsum: null pointer");
  SegList l0{perm0, seg0, coef0, coef_sign0};
  SegList l1{perm1, seg1, coef1, coef_sign1};
  const bool has_l1 = seg1 != nullptr;
  const int64_t w = width;
  switch (out_dtype) {
    case TROPNN_B200_F32:
      return dispatch_segment_rowsum<float>(values, rows, w, ld, groups, buckets, l0, l1, has_l1, scale, out,
                                            bucket_sum, stream);
    case TROPNN_B200_F16:
      return dispatch_segment_rowsum<__half>(values, rows, w, ld, groups, buckets, l0, l1, has_l1, scale, out,
                                             bucket_sum, stream);
    default:
      return dispatch_segment_rowsum<__nv_bfloat16>(values, rows, w, ld, groups, buckets, l0, l1, has_l1, scale,
                                                    out, bucket_sum, stream);
  }
}

}  // namespace tropnn_b200

extern "C" {

int tropnn_b200_bucket_sort(const void *keys, int key_dtype, int64_t rows, int64_t groups, int64_t key_row_stride,
                            int64_t buckets, int32_t *perm, int32_t *seg, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::bucket_sort_impl(keys, key_dtype, rows, groups, key_row_stride, buckets, perm, seg,
                                         tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_segment_rowsum(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                               int64_t buckets, const int32_t *perm0, const int32_t *seg0, const float *coef0,
                               float coef_sign0, const int32_t *perm1, const int32_t *seg1, const float *coef1,
                               float coef_sign1, float scale, void *out, int out_dtype, void *bucket_sum,
                               void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::segment_rowsum_impl(values, rows, width, ld, groups, buckets, perm0, seg0, coef0,
                                            coef_sign0, perm1, seg1, coef1, coef_sign1, scale, out, out_dtype,
                                            bucket_sum, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_segment_rowsum_half(const void *values, int value_dtype, int64_t rows, int64_t width, int64_t ld,
                                    int64_t groups, int64_t buckets, const int32_t *perm, const int32_t *seg,
                                    float scale, const void *grad_absmax, void *out, int out_dtype, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::segment_rowsum_half_impl(values, value_dtype, rows, width, ld, groups, buckets, perm, seg,
                                                 scale, static_cast<const uint32_t *>(grad_absmax), out, out_dtype,
                                                 tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
