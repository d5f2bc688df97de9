// Sum of a split contraction's slice partials, and the epilogue of the product they belong to.
//
// The tensor-core kernels that cut a long contraction into slices (to give every SM work when
// a batch has few 128-row blocks: the projection, the f32 product, the one-hot code sum and
// router term) write each slice's f32 tile to a workspace in their TMEM-native layout, row
// index fastest: unit u = tile * splits + slice holds float4 partial[u][col / 4][row % 128].
// This kernel, launched after them in stream order, sums the slices of every tile in slice
// order (deterministic) and applies the product's epilogue:
//   kReduceHalf    out[row, col] = half(sum)                 (the projection's z)
//   kReduceF32     out[row, col] = sum + bias[col]           (the f32 product)
//   kReduceHidden  out[row, col] = latent[row, col] + scale * sum   (code sum / router term),
//                  and optionally split[row] = [hi | lo] with hi = half(out), lo = half(out - hi)
//                  (the operand of the output map's f32-input product)
//   kReduceHalfT   out[col, row] = half(sum)                 (the projection's weight gradient,
//                                                             computed transposed)
// A block takes 32 rows x one tile's columns: the slices' loads are coalesced over the rows
// (all of a thread's slices in flight at once), the sums are transposed through shared memory
// and written coalesced over the columns.
#include "common.cuh"

namespace tropnn_b200 {

namespace {

constexpr int kRows = 32;
constexpr int kThreads = 256;
constexpr int kMaxTileCols = 256;
constexpr int kMaxSplits = 16;

template <int MODE, typename OT, typename LT>
__global__ void __launch_bounds__(kThreads) slice_reduce_kernel(const float4 *__restrict__ partial, int splits,
                                                               int n_tiles, int tile_cols, int64_t rows, int64_t cols,
                                                               OT *__restrict__ out, int64_t ldo,
                                                               const float *__restrict__ bias,
                                                               const LT *__restrict__ latent, float scale,
                                                               void *__restrict__ split, int split_f16) {
  __shared__ float tile[kRows][kMaxTileCols + 1];
  const int64_t rb = blockIdx.y;                   // 128-row block
  const int sub = blockIdx.x % 4;                  // which 32 rows of it
  const int nt = blockIdx.x / 4;                   // column tile
  const int quads = tile_cols / 4;
  const int r = threadIdx.x & 31;                  // row within the 32
  const int64_t tile_id = rb * n_tiles + nt;
  const size_t slice_stride = size_t(quads) * 128;
  const float4 *base = partial + size_t(tile_id) * splits * slice_stride + sub * 32 + r;
  for (int q = threadIdx.x >> 5; q < quads; q += kThreads / 32) {
    float4 v[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < splits) v[s] = __ldcg(base + s * slice_stride + size_t(q) * 128);
    float4 acc = v[0];
#pragma unroll
    for (int s = 1; s < kMaxSplits; ++s) {
      if (s < splits) {
        acc.x = __fadd_rn(acc.x, v[s].x);
        acc.y = __fadd_rn(acc.y, v[s].y);
        acc.z = __fadd_rn(acc.z, v[s].z);
        acc.w = __fadd_rn(acc.w, v[s].w);
      }
    }
    tile[r][4 * q] = acc.x;
    tile[r][4 * q + 1] = acc.y;
    tile[r][4 * q + 2] = acc.z;
    tile[r][4 * q + 3] = acc.w;
  }
  __syncthreads();
  const int64_t row0 = rb * 128 + sub * 32;
  const int64_t col0 = int64_t(nt) * tile_cols;
  if constexpr (MODE == kReduceHalfT) {
    // Transposed: a warp writes 32 consecutive rows of one output row (column of the tile).
    for (int e = threadIdx.x; e < kRows * tile_cols; e += kThreads) {
      const int cc = e / kRows, rr = e - cc * kRows;
      const int64_t row = row0 + rr, col = col0 + cc;
      if (row < rows && col < cols) out[col * ldo + row] = from_f32<OT>(tile[rr][cc]);
    }
  } else {
  for (int e = threadIdx.x; e < kRows * tile_cols; e += kThreads) {
    const int rr = e / tile_cols, cc = e - rr * tile_cols;
    const int64_t row = row0 + rr, col = col0 + cc;
    if (row >= rows || col >= cols) continue;
    const float sum = tile[rr][cc];
    if constexpr (MODE == kReduceHalf) {
      out[row * ldo + col] = from_f32<OT>(sum);
    } else if constexpr (MODE == kReduceF32) {
      out[row * ldo + col] = bias != nullptr ? __fadd_rn(sum, __ldg(bias + col)) : sum;
    } else {
      const float h = __fadd_rn(to_f32<LT>(latent[row * cols + col]), __fmul_rn(sum, scale));
      out[row * ldo + col] = h;
      if (split != nullptr) {
        const int64_t o = row * 2 * cols + col;
        if (split_f16) {
          const __half hi = from_f32<__half>(h);
          static_cast<__half *>(split)[o] = hi;
          static_cast<__half *>(split)[o + cols] = from_f32<__half>(__fsub_rn(h, to_f32(hi)));
        } else {
          const __nv_bfloat16 hi = from_f32<__nv_bfloat16>(h);
          static_cast<__nv_bfloat16 *>(split)[o] = hi;
          static_cast<__nv_bfloat16 *>(split)[o + cols] = from_f32<__nv_bfloat16>(__fsub_rn(h, to_f32(hi)));
        }
      }
    }
  }
  }
}

template <int MODE, typename OT, typename LT>
int launch_reduce(const void *partial, int splits, int n_tiles, int tile_cols, int64_t rows, int64_t cols, void *out,
                  int64_t ldo, const float *bias, const void *latent, float scale, cudaStream_t stream,
                  void *split = nullptr, int split_f16 = 0) {
  const int64_t row_blocks = ceil_div(rows, int64_t(128));
  TB_REQUIRE(row_blocks < 65536, TROPNN_B200_ERR_INVALID, "slice_reduce: %lld rows exceed the grid", (long long)rows);
  const dim3 grid(static_cast<unsigned>(4 * n_tiles), static_cast<unsigned>(row_blocks));
  slice_reduce_kernel<MODE, OT, LT><<<grid, kThreads, 0, stream>>>(
      static_cast<const float4 *>(partial), splits, n_tiles, tile_cols, rows, cols, static_cast<OT *>(out), ldo, bias,
      static_cast<const LT *>(latent), scale, split, split_f16);
  return check_launch("slice_reduce");
}

}  // namespace

int slice_reduce_impl(int mode, const void *partial, int splits, int n_tiles, int tile_cols, int64_t rows,
                      int64_t cols, void *out, int out_dtype, int64_t ldo, const float *bias, const void *latent,
                      int latent_dtype, float scale, cudaStream_t stream, void *split, int split_dtype) {
  TB_REQUIRE(splits >= 1 && splits <= kMaxSplits && tile_cols % 4 == 0 && tile_cols >= 4 &&
                 tile_cols <= kMaxTileCols && n_tiles >= 1,
             TROPNN_B200_ERR_INVALID, "slice_reduce: bad geometry splits=%d tile_cols=%d", splits, tile_cols);
  if (rows == 0) return TROPNN_B200_OK;
  switch (mode) {
    case kReduceHalf:
      if (out_dtype == TROPNN_B200_F16)
        return launch_reduce<kReduceHalf, __half, float>(partial, splits, n_tiles, tile_cols, rows, cols, out, ldo,
                                                         nullptr, nullptr, 1.f, stream);
      return launch_reduce<kReduceHalf, __nv_bfloat16, float>(partial, splits, n_tiles, tile_cols, rows, cols, out,
                                                              ldo, nullptr, nullptr, 1.f, stream);
    case kReduceHalfT:
      if (out_dtype == TROPNN_B200_F16)
        return launch_reduce<kReduceHalfT, __half, float>(partial, splits, n_tiles, tile_cols, rows, cols, out, ldo,
                                                          nullptr, nullptr, 1.f, stream);
      return launch_reduce<kReduceHalfT, __nv_bfloat16, float>(partial, splits, n_tiles, tile_cols, rows, cols, out,
                                                               ldo, nullptr, nullptr, 1.f, stream);
    case kReduceF32:
      return launch_reduce<kReduceF32, float, float>(partial, splits, n_tiles, tile_cols, rows, cols, out, ldo, bias,
                                                     nullptr, 1.f, stream);
    default: {
      TB_REQUIRE(split == nullptr || split_dtype == TROPNN_B200_F16 || split_dtype == TROPNN_B200_BF16,
                 TROPNN_B200_ERR_DTYPE, "slice_reduce: split dtype %s unsupported", dtype_name(split_dtype));
      const int f16 = split_dtype == TROPNN_B200_F16 ? 1 : 0;
      if (latent_dtype == TROPNN_B200_F32)
        return launch_reduce<kReduceHidden, float, float>(partial, splits, n_tiles, tile_cols, rows, cols, out, ldo,
                                                          nullptr, latent, scale, stream, split, f16);
      if (latent_dtype == TROPNN_B200_F16)
        return launch_reduce<kReduceHidden, float, __half>(partial, splits, n_tiles, tile_cols, rows, cols, out, ldo,
                                                           nullptr, latent, scale, stream, split, f16);
      return launch_reduce<kReduceHidden, float, __nv_bfloat16>(partial, splits, n_tiles, tile_cols, rows, cols, out,
                                                                ldo, nullptr, latent, scale, stream, split, f16);
    }
  }
}

}  // namespace tropnn_b200
