// LUT gradient of PairwiseLinear in one kernel:
//   grad_lut[t, b, :] = sum over rows n with idx[n, t] == b, in ascending n, of scale * g[n, :]
// (each term added with one fused multiply-add)
// (the reference scatters grad_out into the selected LUT rows: autograd of the gather in
// layers/pairwise.py:99-122, atomics in backends/pairwise_tilelang.py:118-156).
//
// One CTA per (table, 64-column block), 32 warps. Per tile of up to kTileRows rows it
//   1. stages the table's route of every row in shared memory (one byte per row, clamped),
//   2. sorts the rows by bucket in shared memory (stable counting sort: per-warp counts over
//      contiguous row runs, a scan, ranks within a warp from __match_any_sync),
//   3. gathers: warp w owns buckets w, w + 32, ...; lane = two columns; it walks the bucket's
//      rows in ascending order with 8-16 row loads in flight and adds them in registers.
// The accumulators stay in registers across tiles, so the sum is the ascending-row sum
// (deterministic, no atomics, no zero-fill, each entry written once), g is read from L2 once
// per table, and nothing but the result goes back to memory (the two-kernel path it replaces
// wrote and re-read a global row permutation and ran its sort on one CTA per table).
#include "common.cuh"
#include "peer.cuh"

namespace tropnn_b200 {

// Fused all-reduce (world > 1): the peer buffers of one PeerAllReduce set, slot = CTA.
struct LutPeer {
  unsigned char *buf[TROPNN_B200_PEER_MAX_RANKS];
  int world;
  int rank;
  int64_t capacity;  // floats per receive area
  float post_scale;  // 1/world when averaging, else 1
};

namespace {

__device__ int g_lut_grad_error = 0;

constexpr int kWarps = 32;
constexpr int kThreads = 32 * kWarps;
constexpr int kTileRows = 16384;
constexpr int kCols = 64;       // columns per CTA: two per lane
constexpr int kMaxBuckets = 256;

struct LutSmem {
  int count[kWarps][kMaxBuckets];  // per-warp bucket counts, then per-warp write positions
  int start[kMaxBuckets + 1];      // bucket starts in the tile's sorted order
  uint16_t perm[kTileRows];        // tile rows sorted by bucket (stable)
  uint8_t key[kTileRows];          // bucket of every tile row
};

template <typename LT, int BPW, bool VEC2, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1)
    lut_grad_kernel(const float *__restrict__ g, int64_t rows, int out_features, const int64_t *__restrict__ idx,
                    int tables, int buckets, float scale, LT *__restrict__ grad_lut, const LutPeer peer) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LutSmem &S = *reinterpret_cast<LutSmem *>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int t = blockIdx.x;
  const int col = blockIdx.y * kCols + 2 * lane;
  const bool c0_ok = col < out_features, c1_ok = col + 1 < out_features;
  const int bmax = buckets - 1;
  // Row loads in flight per warp (fewer with more accumulators, within 64 registers).
  constexpr int kInflight = BPW <= 2 ? 16 : 8;

  float2 acc[BPW];
#pragma unroll
  for (int j = 0; j < BPW; ++j) acc[j] = make_float2(0.f, 0.f);

  for (int64_t tile0 = 0; tile0 < rows; tile0 += kTileRows) {
    const int tile_rows = static_cast<int>(rows - tile0 < kTileRows ? rows - tile0 : kTileRows);
    // 1. Routes of this table (indices come from this library's forward; clamped anyway so
    //    that a corrupt one cannot address outside the tables).
#pragma unroll 4
    for (int i = threadIdx.x; i < tile_rows; i += kThreads) {
      const int64_t v = __ldg(idx + (tile0 + i) * tables + t);
      S.key[i] = static_cast<uint8_t>(v < 0 ? 0 : (v > bmax ? bmax : v));
    }
    for (int i = threadIdx.x; i < kWarps * kMaxBuckets; i += kThreads) (&S.count[0][0])[i] = 0;
    __syncthreads();

    // 2. Stable counting sort. Warp w owns a contiguous run of rows (a multiple of 32 long).
    const int run = ((tile_rows + kWarps - 1) / kWarps + 31) & ~31;
    const int r_begin = min(tile_rows, warp * run);
    const int r_end = min(tile_rows, r_begin + run);
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
      const int r = r0 + lane;
      const bool valid = r < r_end;
      const unsigned active = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int key = S.key[r];
        const unsigned peers = __match_any_sync(active, key);
        if (lane == __ffs(peers) - 1) S.count[warp][key] += __popc(peers);
      }
      __syncwarp();
    }
    __syncthreads();
    // Bucket totals -> bucket starts (one warp scans up to 256 totals); per-warp positions.
    if (threadIdx.x < buckets) {
      int total = 0;
      for (int w = 0; w < kWarps; ++w) total += S.count[w][threadIdx.x];
      S.start[threadIdx.x + 1] = total;
    }
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      for (int b0 = 0; b0 < buckets; b0 += 32) {
        const int b = b0 + lane;
        int v = b < buckets ? S.start[b + 1] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, off);
          if (lane >= off) v += u;
        }
        if (b < buckets) S.start[b + 1] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
      if (lane == 0) S.start[0] = 0;
    }
    __syncthreads();
    if (threadIdx.x < buckets) {
      int pos = S.start[threadIdx.x];
      for (int w = 0; w < kWarps; ++w) {
        const int c = S.count[w][threadIdx.x];
        S.count[w][threadIdx.x] = pos;
        pos += c;
      }
    }
    __syncthreads();
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
      const int r = r0 + lane;
      const bool valid = r < r_end;
      const unsigned active = __ballot_sync(0xffffffffu, valid);
      int key = 0;
      unsigned peers = 0;
      if (valid) {
        key = S.key[r];
        peers = __match_any_sync(active, key);
        S.perm[S.count[warp][key] + __popc(peers & lt_mask)] = static_cast<uint16_t>(r);
      }
      __syncwarp();
      if (valid && lane == __ffs(peers) - 1) S.count[warp][key] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();

    // 3. Gather-sum in ascending row order per bucket, kInflight loads ahead. Each row adds
    //    grad_out * output_scale (one fused multiply-add; the reference scales, then sums).
    const float *gbase = g + tile0 * out_features + col;
    auto load = [&](uint32_t r) -> float2 {
      const float *p = gbase + size_t(r) * out_features;
      float2 v = make_float2(0.f, 0.f);
      if constexpr (VEC2) {
        if (c0_ok) v = __ldg(reinterpret_cast<const float2 *>(p));
      } else {
        if (c0_ok) v.x = __ldg(p);
        if (c1_ok) v.y = __ldg(p + 1);
      }
      return v;
    };
#pragma unroll
    for (int j = 0; j < BPW; ++j) {
      const int b = warp + j * kWarps;
      if (b >= buckets) continue;
      const int lo = S.start[b], hi = S.start[b + 1];
      int i = lo;
      for (; i + kInflight <= hi; i += kInflight) {
        float2 v[kInflight];
#pragma unroll
        for (int u = 0; u < kInflight; ++u) v[u] = load(S.perm[i + u]);
#pragma unroll
        for (int u = 0; u < kInflight; ++u) {
          acc[j].x = __fmaf_rn(v[u].x, scale, acc[j].x);
          acc[j].y = __fmaf_rn(v[u].y, scale, acc[j].y);
        }
      }
      for (; i < hi; ++i) {
        const float2 v = load(S.perm[i]);
        acc[j].x = __fmaf_rn(v.x, scale, acc[j].x);
        acc[j].y = __fmaf_rn(v.y, scale, acc[j].y);
      }
    }
    __syncthreads();  // the next tile reuses the keys and the permutation
  }

  if constexpr (FUSED) {
    // All-reduce of this CTA's block across the ranks, in the same kernel: push the local sums
    // into every rank's receive area (slot = this CTA, so its call counter orders every reuse
    // of the area), one flag barrier per CTA, then sum the ranks' blocks in rank order from
    // this GPU's own memory (bit-identical on every rank). CTAs push before they wait, so a
    // rank whose CTAs are not all resident still completes.
    __shared__ uint32_t call_s;
    __shared__ int ok_s;
    const int slot = blockIdx.x * gridDim.y + blockIdx.y;
    unsigned char *mine = peer.buf[peer.rank];
    if (threadIdx.x == 0) call_s = peer::counters(mine)[slot] + 1;
    __syncthreads();
    const uint32_t call = call_s, parity = call & 1u;
    const int64_t base = int64_t(slot) * buckets * kCols + 2 * lane;
#pragma unroll
    for (int j = 0; j < BPW; ++j) {
      const int b = warp + j * kWarps;
      if (b >= buckets) continue;
      for (int p = 0; p < peer.world; ++p)
        *reinterpret_cast<float2 *>(peer::recv(peer.buf[p], peer.capacity, parity, peer.rank) + base + b * kCols) =
            acc[j];
    }
    __syncthreads();
    if (threadIdx.x == 0)
      ok_s = peer::slot_barrier(peer.buf, peer.world, peer.rank, slot, call, &g_lut_grad_error) ? 1 : 0;
    __syncthreads();
    if (ok_s) {
#pragma unroll
      for (int j = 0; j < BPW; ++j) {
        const int b = warp + j * kWarps;
        if (b >= buckets) continue;
        float2 sum = __ldcg(reinterpret_cast<const float2 *>(peer::recv(mine, peer.capacity, parity, 0) + base + b * kCols));
        for (int p = 1; p < peer.world; ++p) {
          const float2 v =
              __ldcg(reinterpret_cast<const float2 *>(peer::recv(mine, peer.capacity, parity, p) + base + b * kCols));
          sum.x = __fadd_rn(sum.x, v.x);
          sum.y = __fadd_rn(sum.y, v.y);
        }
        acc[j] = make_float2(__fmul_rn(sum.x, peer.post_scale), __fmul_rn(sum.y, peer.post_scale));
      }
    }
    if (threadIdx.x == 0) peer::counters(mine)[slot] = call;
  }

#pragma unroll
  for (int j = 0; j < BPW; ++j) {
    const int b = warp + j * kWarps;
    if (b >= buckets) continue;
    LT *o = grad_lut + (int64_t(t) * buckets + b) * out_features + col;
    if (c0_ok) o[0] = from_f32<LT>(acc[j].x);
    if (c1_ok) o[1] = from_f32<LT>(acc[j].y);
  }
}

template <typename LT, int BPW>
int launch_bpw(const float *g, int64_t rows, int out_features, const int64_t *idx, int tables, int buckets,
               float scale, LT *grad_lut, const LutPeer *peer, cudaStream_t stream) {
  const size_t smem = sizeof(LutSmem);
  // 8-byte loads of column pairs when every row start is 8-byte aligned.
  const bool vec2 = out_features % 2 == 0 && reinterpret_cast<uintptr_t>(g) % 8 == 0;
  auto kernel = peer != nullptr ? (vec2 ? lut_grad_kernel<LT, BPW, true, true> : lut_grad_kernel<LT, BPW, false, true>)
                                : (vec2 ? lut_grad_kernel<LT, BPW, true, false> : lut_grad_kernel<LT, BPW, false, false>);
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "pairwise_lut_grad"));
  const dim3 grid(static_cast<unsigned>(tables), static_cast<unsigned>(ceil_div(int64_t(out_features), int64_t(kCols))));
  const LutPeer none{};
  kernel<<<grid, kThreads, smem, stream>>>(g, rows, out_features, idx, tables, buckets, scale, grad_lut,
                                           peer != nullptr ? *peer : none);
  return check_launch("pairwise_lut_grad");
}

template <typename LT>
int launch_lut_grad(const float *g, int64_t rows, int out_features, const int64_t *idx, int tables, int buckets,
                    float scale, LT *grad_lut, const LutPeer *peer, cudaStream_t stream) {
  if (buckets <= 32) return launch_bpw<LT, 1>(g, rows, out_features, idx, tables, buckets, scale, grad_lut, peer, stream);
  if (buckets <= 64) return launch_bpw<LT, 2>(g, rows, out_features, idx, tables, buckets, scale, grad_lut, peer, stream);
  if (buckets <= 128) return launch_bpw<LT, 4>(g, rows, out_features, idx, tables, buckets, scale, grad_lut, peer, stream);
  return launch_bpw<LT, 8>(g, rows, out_features, idx, tables, buckets, scale, grad_lut, peer, stream);
}

}  // namespace

bool lut_grad_supported(int64_t tables, int64_t comparisons, int64_t out_features) {
  return tables >= 1 && tables <= (int64_t(1) << 31) - 1 && comparisons >= 1 && comparisons <= 8 &&
         out_features >= 1 && out_features <= (int64_t(1) << 30);
}

int lut_grad_impl(const float *g, int64_t rows, int64_t out_features, const int64_t *indices, int64_t tables,
                  int64_t comparisons, float scale, void *grad_lut, int lut_dtype, const LutPeer *peer,
                  cudaStream_t stream) {
  TB_REQUIRE(lut_grad_supported(tables, comparisons, out_features), TROPNN_B200_ERR_INVALID,
             "pairwise_lut_grad: unsupported shape tables=%lld comparisons=%lld out=%lld (comparisons <= 8)",
             (long long)tables, (long long)comparisons, (long long)out_features);
  TB_REQUIRE(rows >= 0 && rows <= (int64_t(1) << 40), TROPNN_B200_ERR_INVALID, "pairwise_lut_grad: bad row count");
  TB_REQUIRE(is_float_dtype(lut_dtype), TROPNN_B200_ERR_DTYPE, "pairwise_lut_grad: dtype %s unsupported",
             dtype_name(lut_dtype));
  TB_REQUIRE(grad_lut && (rows == 0 || (g && indices)), TROPNN_B200_ERR_INVALID, "pairwise_lut_grad: null pointer");
  TB_REQUIRE(ceil_div(out_features, int64_t(kCols)) <= 65535, TROPNN_B200_ERR_INVALID,
             "pairwise_lut_grad: out_features %lld too large", (long long)out_features);
  const int o = static_cast<int>(out_features), t = static_cast<int>(tables), b = 1 << comparisons;
  switch (lut_dtype) {
    case TROPNN_B200_F32:
      return launch_lut_grad<float>(g, rows, o, indices, t, b, scale, static_cast<float *>(grad_lut), peer, stream);
    case TROPNN_B200_F16:
      return launch_lut_grad<__half>(g, rows, o, indices, t, b, scale, static_cast<__half *>(grad_lut), peer, stream);
    default:
      return launch_lut_grad<__nv_bfloat16>(g, rows, o, indices, t, b, scale,
                                            static_cast<__nv_bfloat16 *>(grad_lut), peer, stream);
  }
}

// Receive-area floats the fused variant needs: one slot of 2^comparisons x 64 floats per CTA.
int64_t lut_grad_peer_floats(int64_t tables, int64_t comparisons, int64_t out_features) {
  return tables * ceil_div(out_features, int64_t(kCols)) * (int64_t(1) << comparisons) * kCols;
}

int read_lut_grad_error(int *value) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_lut_grad_error, sizeof(int));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "reading the device error word: %s", cudaGetErrorString(err));
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_lut_grad_error, &zero, sizeof(int));
  }
  *value = v;
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

int tropnn_b200_pairwise_lut_grad(const float *grad_out, int64_t items, int64_t out_features, const int64_t *indices,
                                  int64_t tables, int64_t comparisons, float scale, void *grad_lut, int lut_dtype,
                                  void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::lut_grad_impl(grad_out, items, out_features, indices, tables, comparisons, scale, grad_lut,
                                      lut_dtype, nullptr, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int64_t tropnn_b200_pairwise_lut_grad_peer_floats(int64_t tables, int64_t comparisons, int64_t out_features) {
  if (!tropnn_b200::lut_grad_supported(tables, comparisons, out_features)) return -1;
  return tropnn_b200::lut_grad_peer_floats(tables, comparisons, out_features);
}

int tropnn_b200_pairwise_lut_grad_allreduce(const float *grad_out, int64_t items, int64_t out_features,
                                            const int64_t *indices, int64_t tables, int64_t comparisons, float scale,
                                            void *grad_lut, int lut_dtype, void *const *buffers, int world, int rank,
                                            int64_t capacity_floats, int average, void *stream) {
  using namespace tropnn_b200;
  TB_CHECK(check_current_device());
  TB_REQUIRE(buffers != nullptr && world >= 1 && world <= TROPNN_B200_PEER_MAX_RANKS && rank >= 0 && rank < world,
             TROPNN_B200_ERR_INVALID, "pairwise_lut_grad_allreduce: rank %d of world %d", rank, world);
  TB_REQUIRE(lut_grad_supported(tables, comparisons, out_features), TROPNN_B200_ERR_INVALID,
             "pairwise_lut_grad_allreduce: unsupported shape");
  const int64_t slots = tables * ceil_div(out_features, int64_t(kCols));
  TB_REQUIRE(slots <= peer::kPeerMaxSlices, TROPNN_B200_ERR_INVALID,
             "pairwise_lut_grad_allreduce: %lld column blocks exceed the %d peer slots", (long long)slots,
             peer::kPeerMaxSlices);
  TB_REQUIRE(capacity_floats >= lut_grad_peer_floats(tables, comparisons, out_features), TROPNN_B200_ERR_INVALID,
             "pairwise_lut_grad_allreduce: peer capacity %lld floats below the %lld needed", (long long)capacity_floats,
             (long long)lut_grad_peer_floats(tables, comparisons, out_features));
  LutPeer peer{};
  for (int p = 0; p < world; ++p) {
    TB_REQUIRE(buffers[p] != nullptr, TROPNN_B200_ERR_INVALID, "pairwise_lut_grad_allreduce: null buffer %d", p);
    peer.buf[p] = static_cast<unsigned char *>(buffers[p]);
  }
  peer.world = world;
  peer.rank = rank;
  peer.capacity = capacity_floats;
  peer.post_scale = average ? 1.f / float(world) : 1.f;
  TB_CHECK(lut_grad_impl(grad_out, items, out_features, indices, tables, comparisons, scale, grad_lut, lut_dtype,
                         world > 1 ? &peer : nullptr, as_stream(stream)));
  return clear_error();
}

}  // extern "C"
