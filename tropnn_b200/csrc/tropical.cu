// TropLinear on sm_100a, fp32-exact SIMT path: route scores + top-2, selected-code
// gather-sum, and the per-row part of the min-face backward. (The f16/bf16 score GEMM
// on the tensor cores lives in score_sm100.cu.)
//
// Reference behaviour (paths inside the tropnn package):
//   scores     backend.py:45-46 (einsum + bias), routing.py:7-10 (topk k=2, margin)
//   hidden     layers/tropical.py:131-138 (gather + sum * code_scale + latent),
//              routing.py:13-15 (min-face mix U(m) = 0.5 / (1 + |m|))
//   backward   layers/tropical_exact.py:204-237 (coefficient form of the autograd of the
//              torch path), backends/triton_backward.py:27-354
//
// Layout: latent f32 [N, D]; router_weight / code [H, K, D] and router_bias [H, K] in
// param dtype; winner/runner [N, H] in the packed index dtype; margins f32 [N, H].
#include "common.cuh"

namespace tropnn_b200 {

int bucket_sort_impl(const void *keys, int key_dtype, int64_t rows, int64_t groups, int64_t stride,
                     int64_t buckets, int32_t *perm, int32_t *seg, cudaStream_t stream);
int segment_rowsum_impl(const float *values, int64_t rows, int64_t width, int64_t ld, int64_t groups,
                        int64_t buckets, const int32_t *perm0, const int32_t *seg0, const float *coef0,
                        float coef_sign0, const int32_t *perm1, const int32_t *seg1, const float *coef1,
                        float coef_sign1, float scale, void *out, int out_dtype, void *bucket_sum,
                        cudaStream_t stream);

bool score_sm100_supported(int64_t D, int64_t K, int pt, int bias_dtype, const void *z, const void *W,
                           const void *bias);
int trop_score_sm100_impl(const void *z, int64_t items, int64_t D, const void *W, const void *bias, int pt, int64_t H,
                          int64_t K, int64_t *w64, uint8_t *win, uint8_t *run, float *m, cudaStream_t stream);
int read_score_error(int *value);
int read_pairwise_error(int *value);
bool score_tf32_supported(int64_t D, int64_t K, int pt, int bias_dtype, const void *z, const void *W,
                          const void *bias);
size_t score_tf32_workspace(int64_t items, int64_t D, int64_t H, int64_t K);
int trop_score_tf32_impl(const float *z, int64_t items, int64_t D, const float *W, const float *bias, int64_t H,
                         int64_t K, int64_t *w64, uint8_t *win, uint8_t *run, float *m, void *ws, size_t ws_bytes,
                         cudaStream_t stream);
bool hidden_sm100_supported(int64_t items, int64_t D, int64_t H, int64_t K, int pt, int zt, int it, const void *latent,
                            const void *code_t, const void *hidden);
int trop_hidden_sm100_impl(const void *latent, int zt, int64_t items, int64_t D, const void *code_t, int pt,
                           int64_t H, int64_t K, const void *win, const void *run, const float *m, float code_scale,
                           int mode, const uint32_t *absmax, float *hidden, void *hidden_split, void *ws, size_t wsb,
                           cudaStream_t stream);
int split_half_impl(const float *x, int64_t rows, int64_t cols, int dtype, const uint32_t *absmax, void *out,
                    cudaStream_t stream);
size_t trop_hidden_sm100_workspace(int64_t items, int64_t D, int64_t H, int64_t K);
int trop_code_transpose_impl(const void *code, int pt, int64_t H, int64_t K, int64_t D, void *code_t,
                             cudaStream_t stream);
int read_hidden_error(int *value);
int read_gemm_error(int *value);
int read_peer_error(int *value);
int read_param_grad_error(int *value);
int read_linear_grad_error(int *value);
int read_lut_grad_error(int *value);
int read_proj_error(int *value);
int read_gemm_tf32_error(int *value);
int trop_gm_sm100_impl(const void *g_split, int64_t rows, int64_t code_dim, const void *code, int dtype, int64_t heads,
                       int64_t cells, const uint8_t *winner, const uint8_t *runner, const float *margins,
                       float code_scale, float *gm, const uint32_t *absmax, cudaStream_t stream);
int trop_param_grad_sm100_impl(int mode, const void *xt, int64_t rows, int64_t D, int pt, int64_t H, int64_t K,
                               const void *win, const void *run, const float *mvals, float code_scale, void *out,
                               void *grad_b, const uint32_t *absmax, cudaStream_t stream);
int transpose_to_half_impl(const void *x, int xt_dtype, int64_t rows, int64_t cols, int pt, void *out,
                           const uint32_t *absmax, cudaStream_t stream);

namespace {

// ---------------------------------------------------------------------------
// route: scores, top-2, margins
// ---------------------------------------------------------------------------
// CTA = 8 warps = 8 heads; lane l owns rows {row0 + l + 32 i, i < RM}. The latent tile
// [32*RM rows, D] sits in shared memory (row pitch D+4 floats keeps the 16-byte lane
// reads conflict-free); router weights are warp-uniform broadcast loads. Cells are
// scored KC at a time with a running top-2, so any cell count works.
constexpr int kRouteWarps = 8;
constexpr int kCellChunk = 8;

// Latent element load: f32, or (ZP) the parameter dtype, upcast exactly.
template <typename PT, bool ZP>
__device__ __forceinline__ float load_latent(const void *z, int64_t i) {
  if constexpr (ZP) {
    return ldg_f32(static_cast<const PT *>(z) + i);
  } else {
    return __ldg(static_cast<const float *>(z) + i);
  }
}

template <typename PT, typename IT, int RM, bool VEC4, bool ZP>
__global__ void __launch_bounds__(kRouteWarps * 32) trop_route_kernel(
    const void *__restrict__ z, int64_t rows, int D, const PT *__restrict__ W, const void *__restrict__ bias, bool bias_f32, int H,
    int K, int64_t *__restrict__ winner_i64, IT *__restrict__ winner, IT *__restrict__ runner,
    float *__restrict__ margins) {
  extern __shared__ float z_s[];
  const int pitch = D + 4;
  const int64_t row0 = int64_t(blockIdx.x) * 32 * RM;
  const int rows_here = static_cast<int>(min64(32 * RM, rows - row0));
  for (int i = threadIdx.x; i < rows_here * D; i += kRouteWarps * 32) {
    const int r = i / D;
    const int d = i - r * D;
    z_s[r * pitch + d] = load_latent<PT, ZP>(z, (row0 + r) * D + d);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.y * kRouteWarps + warp;
  if (h >= H) return;

  float best1[RM], best2[RM];
  int i1[RM], i2[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    best1[r] = -INFINITY; best2[r] = -INFINITY; i1[r] = 0; i2[r] = 1;
  }
  const PT *Wh = W + int64_t(h) * K * D;
  for (int k0 = 0; k0 < K; k0 += kCellChunk) {
    float acc[RM][kCellChunk];
#pragma unroll
    for (int r = 0; r < RM; ++r)
#pragma unroll
      for (int k = 0; k < kCellChunk; ++k) acc[r][k] = 0.f;
    if (VEC4) {
      for (int d = 0; d < D; d += 4) {
        float zv[RM][4];
#pragma unroll
        for (int r = 0; r < RM; ++r) {
          const float4 q = *reinterpret_cast<const float4 *>(z_s + (lane + 32 * r) * pitch + d);
          zv[r][0] = q.x; zv[r][1] = q.y; zv[r][2] = q.z; zv[r][3] = q.w;
        }
#pragma unroll
        for (int k = 0; k < kCellChunk; ++k) {
          if (k0 + k < K) {
            float wv[4];
            const PT *wp = Wh + int64_t(k0 + k) * D + d;
#pragma unroll
            for (int e = 0; e < 4; ++e) wv[e] = ldg_f32(wp + e);
#pragma unroll
            for (int r = 0; r < RM; ++r)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[r][k] = fmaf(zv[r][e], wv[e], acc[r][k]);
          }
        }
      }
    } else {
      for (int d = 0; d < D; ++d) {
        float zv[RM];
#pragma unroll
        for (int r = 0; r < RM; ++r) zv[r] = z_s[(lane + 32 * r) * pitch + d];
#pragma unroll
        for (int k = 0; k < kCellChunk; ++k) {
          if (k0 + k < K) {
            const float wv = ldg_f32(Wh + int64_t(k0 + k) * D + d);
#pragma unroll
            for (int r = 0; r < RM; ++r) acc[r][k] = fmaf(zv[r], wv, acc[r][k]);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kCellChunk; ++k) {
      if (k0 + k < K) {
        const int64_t bi = int64_t(h) * K + k0 + k;
        const float bk = bias_f32 ? __ldg(static_cast<const float *>(bias) + bi) : ldg_f32(static_cast<const PT *>(bias) + bi);
#pragma unroll
        for (int r = 0; r < RM; ++r) {
          const float s = __fadd_rn(acc[r][k], bk);
          // Strict '>' keeps the lowest cell index on exact ties.
          if (s > best1[r]) {
            best2[r] = best1[r]; i2[r] = i1[r]; best1[r] = s; i1[r] = k0 + k;
          } else if (s > best2[r]) {
            best2[r] = s; i2[r] = k0 + k;
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RM; ++r) {
    const int rr = lane + 32 * r;
    if (rr < rows_here) {
      const int64_t o = (row0 + rr) * H + h;
      if (winner_i64) winner_i64[o] = i1[r];
      winner[o] = static_cast<IT>(i1[r]);
      if (runner != nullptr) runner[o] = static_cast<IT>(i2[r]);
      if (margins != nullptr) margins[o] = __fsub_rn(best1[r], best2[r]);
    }
  }
}

template <typename PT, typename IT, int RM>
int launch_route(const void *z, bool zp, int64_t rows, int D, const void *W, const void *b, bool bias_f32, int H,
                 int K, int64_t *w64, void *win, void *run, float *m, cudaStream_t stream) {
  const bool vec4 = (D % 4 == 0);
  const size_t smem = sizeof(float) * 32 * RM * (D + 4);
  TB_REQUIRE(smem <= 200 * 1024, TROPNN_B200_ERR_INVALID, "trop_route: code_dim=%d too large for the SIMT path", D);
  auto kernel = zp ? (vec4 ? trop_route_kernel<PT, IT, RM, true, true> : trop_route_kernel<PT, IT, RM, false, true>)
                   : (vec4 ? trop_route_kernel<PT, IT, RM, true, false> : trop_route_kernel<PT, IT, RM, false, false>);
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), smem, "trop_route"));
  const int64_t row_blocks = ceil_div(rows, 32 * RM);
  TB_REQUIRE(row_blocks < (int64_t(1) << 31) && ceil_div(H, kRouteWarps) < 65536, TROPNN_B200_ERR_INVALID,
             "trop_route: grid too large");
  dim3 grid(static_cast<unsigned>(row_blocks), static_cast<unsigned>(ceil_div(H, kRouteWarps)));
  kernel<<<grid, kRouteWarps * 32, smem, stream>>>(z, rows, D, static_cast<const PT *>(W), b, bias_f32, H, K, w64,
                                                   static_cast<IT *>(win), static_cast<IT *>(run), m);
  return check_launch("trop_route");
}

template <typename PT, typename IT>
int route_by_rows(const void *z, bool zp, int64_t rows, int D, const void *W, const void *b, bool bias_f32, int H,
                  int K, int64_t *w64, void *win, void *run, float *m, cudaStream_t stream) {
  // Four rows per lane once there are enough rows to fill the GPU with 128-row tiles.
  if (ceil_div(rows, 128) * ceil_div(H, kRouteWarps) >= 2 * 148 && 128 * (D + 4) * 4 <= 200 * 1024)
    return launch_route<PT, IT, 4>(z, zp, rows, D, W, b, bias_f32, H, K, w64, win, run, m, stream);
  return launch_route<PT, IT, 1>(z, zp, rows, D, W, b, bias_f32, H, K, w64, win, run, m, stream);
}

// ---------------------------------------------------------------------------
// per-row code kernels: hidden (selected-code gather-sum) and backward rows
// ---------------------------------------------------------------------------
// One CTA of 8 warps per row (and code_dim slice); warp w owns a contiguous range of
// heads. The slice is split in vector slots of VEC elements (16-byte loads when VEC > 1);
// lanes form groups of `lph` lanes, each group takes one head per pass (so a warp covers
// 32/lph heads at once when code_dim is small) and lane l of a group owns slots
// l + j*lph, j < NJ. Per-lane partial sums are combined in a fixed order (warp, then
// lane group), so results are deterministic.
constexpr int kRowWarps = 8;

__device__ __forceinline__ float group_sum(float v, int lph) {
  for (int off = lph >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// hidden = latent + code_scale * sum_h chat_h (the operation order of tropical.py:137).
template <typename PT, typename IT, bool TRAIN, int VEC, int NJ, bool ZP>
__global__ void __launch_bounds__(kRowWarps * 32) trop_hidden_kernel(
    const void *__restrict__ z, int D, const PT *__restrict__ code, int H, int K, const IT *__restrict__ winner,
    const IT *__restrict__ runner, const float *__restrict__ margins, float code_scale, int lph,
    float *__restrict__ hidden) {
  __shared__ float part[kRowWarps * 32 * NJ * VEC];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x;
  const int d_base = blockIdx.y * (32 * NJ * VEC);
  const int slots = min(32 * NJ, (D - d_base + VEC - 1) / VEC);
  const int hpw = 32 / lph;
  const int sub = lane / lph;
  const int l = lane - sub * lph;
  const int hw = (H + kRowWarps - 1) / kRowWarps;
  const int hs = min(H, warp * hw);
  const int he = min(H, hs + hw);
  const IT *wrow = winner + n * H;
  const IT *rrow = runner + n * H;
  const float *mrow = margins + n * H;
  float acc[NJ][VEC];
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = 0.f;
#pragma unroll 4
  for (int h = hs + sub; h < he; h += hpw) {
    const PT *cw = code + (int64_t(h) * K + ld_index(wrow + h)) * D + d_base;
    if (TRAIN) {
      const PT *cr = code + (int64_t(h) * K + ld_index(rrow + h)) * D + d_base;
      const float alpha = __fdiv_rn(0.5f, __fadd_rn(1.f, fabsf(__ldg(mrow + h))));
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int s = l + j * lph;
        if (s < slots) {
          float a[VEC], b[VEC];
          VecLoad<PT, VEC>::load(cw + s * VEC, a);
          VecLoad<PT, VEC>::load(cr + s * VEC, b);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[j][e] = __fadd_rn(acc[j][e], __fadd_rn(a[e], __fmul_rn(alpha, __fsub_rn(b[e], a[e]))));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int s = l + j * lph;
        if (s < slots) {
          float a[VEC];
          VecLoad<PT, VEC>::load(cw + s * VEC, a);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[j][e] = __fadd_rn(acc[j][e], a[e]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) part[((warp * 32 + lane) * NJ + j) * VEC + e] = acc[j][e];
  __syncthreads();
  for (int q = threadIdx.x; q < slots * VEC; q += kRowWarps * 32) {
    const int s = q / VEC;
    const int e = q - s * VEC;
    const int j = s / lph;
    const int ls = s - j * lph;
    float sum = 0.f;
    for (int w = 0; w < kRowWarps; ++w)
      for (int sb = 0; sb < hpw; ++sb) sum = __fadd_rn(sum, part[((w * 32 + sb * lph + ls) * NJ + j) * VEC + e]);
    const int64_t o = n * D + d_base + q;
    hidden[o] = __fadd_rn(load_latent<PT, ZP>(z, o), __fmul_rn(sum, code_scale));
  }
}

// Per-row part of the min-face backward: gm from the group-reduced <g, c_r - c_w>, the
// router term of grad_latent, and the per-row coefficients of the code / router
// scatters. Needs the whole code_dim in one CTA (slots <= 32 * NJ).
template <typename PT, typename IT, bool TRAIN, int VEC, int NJ>
__global__ void __launch_bounds__(kRowWarps * 32) trop_backward_rows_kernel(
    const float *__restrict__ g, int D, const PT *__restrict__ W, const PT *__restrict__ code, int H, int K,
    const IT *__restrict__ winner, const IT *__restrict__ runner, const float *__restrict__ margins, float code_scale,
    int lph, float *__restrict__ grad_z, float *__restrict__ coef_w, float *__restrict__ coef_r,
    float *__restrict__ gm_out) {
  __shared__ float part[kRowWarps * 32 * NJ * VEC];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x;
  const int slots = (D + VEC - 1) / VEC;
  const int hpw = 32 / lph;
  const int sub = lane / lph;
  const int l = lane - sub * lph;
  const int hw = (H + kRowWarps - 1) / kRowWarps;
  const int hs = min(H, warp * hw);
  const int he = min(H, hs + hw);
  const float *grow = g + n * D;
  float gv[NJ][VEC], acc[NJ][VEC];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int s = l + j * lph;
    if (s < slots) {
      VecLoad<float, VEC>::load(grow + s * VEC, gv[j]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) gv[j][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = 0.f;
  }
  // Warp-uniform trip count: every lane takes part in the group shuffles.
  for (int h0 = hs; h0 < he; h0 += hpw) {
    const int h = h0 + sub;
    const bool valid = h < he;
    const int64_t o = n * H + h;
    if (!TRAIN) {
      if (valid && l == 0) coef_w[o] = code_scale;
      continue;
    }
    int w = 0, r = 0;
    float m = 0.f;
    if (valid) {
      w = ld_index(winner + o);
      r = ld_index(runner + o);
      m = __ldg(margins + o);
    }
    const int64_t hk = int64_t(valid ? h : hs) * K;
    const PT *cw = code + (hk + w) * D;
    const PT *cr = code + (hk + r) * D;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int s = l + j * lph;
      if (valid && s < slots) {
        float a[VEC], b[VEC];
        VecLoad<PT, VEC>::load(cw + s * VEC, a);
        VecLoad<PT, VEC>::load(cr + s * VEC, b);
#pragma unroll
        for (int e = 0; e < VEC; ++e) dot = fmaf(__fmul_rn(gv[j][e], code_scale), __fsub_rn(b[e], a[e]), dot);
      }
    }
    dot = group_sum(dot, lph);
    if (!valid) continue;
    const float den = __fadd_rn(1.f, fabsf(m));
    const float alpha = __fdiv_rn(0.5f, den);
    const float sgn = (m > 0.f) ? 1.f : ((m < 0.f) ? -1.f : 0.f);
    // d/dm [0.5 / (1 + |m|)] = -0.5 sign(m) / (1 + |m|)^2
    const float gm = __fmul_rn(dot, __fdiv_rn(__fmul_rn(-0.5f, sgn), __fmul_rn(den, den)));
    const PT *ww = W + (hk + w) * D;
    const PT *wr = W + (hk + r) * D;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int s = l + j * lph;
      if (s < slots) {
        float a[VEC], b[VEC];
        VecLoad<PT, VEC>::load(ww + s * VEC, a);
        VecLoad<PT, VEC>::load(wr + s * VEC, b);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[j][e] = fmaf(gm, __fsub_rn(a[e], b[e]), acc[j][e]);
      }
    }
    if (l == 0) {
      coef_w[o] = __fmul_rn(code_scale, __fsub_rn(1.f, alpha));
      coef_r[o] = __fmul_rn(code_scale, alpha);
      gm_out[o] = gm;
    }
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) part[((warp * 32 + lane) * NJ + j) * VEC + e] = acc[j][e];
  __syncthreads();
  for (int q = threadIdx.x; q < D; q += kRowWarps * 32) {
    const int s = q / VEC;
    const int e = q - s * VEC;
    const int j = s / lph;
    const int ls = s - j * lph;
    float sum = 0.f;
    for (int w = 0; w < kRowWarps; ++w)
      for (int sb = 0; sb < hpw; ++sb) sum = __fadd_rn(sum, part[((w * 32 + sb * lph + ls) * NJ + j) * VEC + e]);
    grad_z[n * D + q] = __fadd_rn(__ldg(grow + q), sum);
  }
}

// Lanes per head: all 32 once a slice has >= 32 slots, else the next power of two.
inline int lanes_per_head(int slots) {
  int lph = 1;
  while (lph < 32 && lph < slots) lph <<= 1;
  return lph;
}

// Vector width of the per-row kernels: 16-byte loads when code_dim allows it.
template <typename PT>
inline bool row_vec_ok(int D, const void *p0, const void *p1, const void *p2) {
  constexpr int V = 16 / sizeof(PT);
  auto al = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return D % V == 0 && al(p0) && al(p1) && al(p2);
}

int validate_trop(int64_t items, int64_t D, int64_t H, int64_t K) {
  TB_REQUIRE(items >= 0 && D >= 1 && H >= 1 && K >= 2, TROPNN_B200_ERR_INVALID,
             "trop: bad sizes items=%lld code_dim=%lld heads=%lld cells=%lld", (long long)items, (long long)D,
             (long long)H, (long long)K);
  TB_REQUIRE(items < (int64_t(1) << 31) && H < (int64_t(1) << 24) && D < (int64_t(1) << 20) && K <= 32767,
             TROPNN_B200_ERR_INVALID, "trop: sizes out of range items=%lld code_dim=%lld heads=%lld cells=%lld",
             (long long)items, (long long)D, (long long)H, (long long)K);
  return TROPNN_B200_OK;
}

int check_index_dtype(int64_t K, int index_dtype) {
  TB_REQUIRE(is_index_dtype(index_dtype), TROPNN_B200_ERR_DTYPE, "trop: index dtype %s unsupported",
             dtype_name(index_dtype));
  TB_REQUIRE(!(index_dtype == TROPNN_B200_U8 && K > 256), TROPNN_B200_ERR_DTYPE,
             "trop: cells=%lld does not fit the u8 index dtype", (long long)K);
  return TROPNN_B200_OK;
}

#define TB_DISPATCH_PT(pt, ...)                              \
  switch (pt) {                                              \
    case TROPNN_B200_F32: { using PT = float; __VA_ARGS__ } break;          \
    case TROPNN_B200_F16: { using PT = __half; __VA_ARGS__ } break;         \
    default: { using PT = __nv_bfloat16; __VA_ARGS__ } break;               \
  }
#define TB_DISPATCH_IT(it, ...)                              \
  switch (it) {                                              \
    case TROPNN_B200_U8: { using IT = uint8_t; __VA_ARGS__ } break;         \
    case TROPNN_B200_I16: { using IT = int16_t; __VA_ARGS__ } break;        \
    default: { using IT = int64_t; __VA_ARGS__ } break;                     \
  }

}  // namespace

int check_latent_dtype(int zt, int pt, const char *what) {
  TB_REQUIRE(zt == TROPNN_B200_F32 || zt == pt, TROPNN_B200_ERR_DTYPE,
             "%s: latent dtype %s must be f32 or the parameter dtype %s", what, dtype_name(zt), dtype_name(pt));
  return TROPNN_B200_OK;
}

// The route's f32 tensor-core path (3xTF32) applies to f32 latent, parameters and bias with u8
// routes and the tile shapes of trop_score_tf32; it needs a workspace for the split operands.
// f32 scores on the tensor cores (3xTF32) from 64 rows on; fewer rows leave an M=128 MMA tile
// mostly empty, and the fp32 FMA kernel answers sooner.
constexpr int64_t kRouteTf32MinItems = 64;

bool route_tf32_applies(int64_t items, int zt, int pt, int bt, int it, int64_t D, int64_t H, int64_t K, const void *z,
                        const void *W, const void *b) {
  return items >= kRouteTf32MinItems && zt == TROPNN_B200_F32 && it == TROPNN_B200_U8 && H * K >= 32 &&
         score_tf32_supported(D, K, pt, bt, z, W, b);
}

size_t trop_route_workspace(int64_t items, int64_t D, int64_t H, int64_t K, int zt, int pt) {
  if (items < 0 || D < 1 || H < 1 || K < 1) return 0;
  if (zt == TROPNN_B200_F32 && pt == TROPNN_B200_F32) return score_tf32_workspace(items, D, H, K);
  return 0;
}

int trop_route_impl(const void *z, int zt, int64_t items, int64_t D, const void *W, const void *b, int bt, int pt,
                    int64_t H, int64_t K, int64_t *w64, void *win, void *run, int it, float *m, void *ws,
                    size_t ws_bytes, cudaStream_t stream) {
  TB_CHECK(validate_trop(items, D, H, K));
  TB_REQUIRE(is_float_dtype(pt), TROPNN_B200_ERR_DTYPE, "trop_route: param dtype %s unsupported", dtype_name(pt));
  TB_CHECK(check_index_dtype(K, it));
  TB_CHECK(check_latent_dtype(zt, pt, "trop_route"));
  TB_REQUIRE(bt == pt || bt == TROPNN_B200_F32, TROPNN_B200_ERR_DTYPE,
             "trop_route: bias dtype %s must be f32 or the parameter dtype %s", dtype_name(bt), dtype_name(pt));
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(z && W && b && win, TROPNN_B200_ERR_INVALID, "trop_route: null pointer");
  // Half-precision latent and parameters: scores on the tensor cores (tcgen05) when the
  // shape fits the kernel's tiles; the SIMT kernel serves everything else.
  const bool zp = zt != TROPNN_B200_F32;
  if (zp && it == TROPNN_B200_U8 && items >= 128 && H * K >= 128 && score_sm100_supported(D, K, pt, bt, z, W, b))
    return trop_score_sm100_impl(z, items, D, W, b, pt, H, K, w64, static_cast<uint8_t *>(win),
                                 static_cast<uint8_t *>(run), m, stream);
  // f32 latent and parameters with room for the split operands: 3xTF32 on the tensor cores.
  if (ws != nullptr && route_tf32_applies(items, zt, pt, bt, it, D, H, K, z, W, b) &&
      ws_bytes >= score_tf32_workspace(items, D, H, K))
    return trop_score_tf32_impl(static_cast<const float *>(z), items, D, static_cast<const float *>(W),
                                static_cast<const float *>(b), H, K, w64, static_cast<uint8_t *>(win),
                                static_cast<uint8_t *>(run), m, ws, ws_bytes, stream);
  int status = TROPNN_B200_OK;
  const bool bias_f32 = bt == TROPNN_B200_F32;
  TB_DISPATCH_PT(pt, TB_DISPATCH_IT(it, status = route_by_rows<PT, IT>(z, zp, items, static_cast<int>(D), W, b,
                                                                       bias_f32, static_cast<int>(H),
                                                                       static_cast<int>(K), w64, win, run, m,
                                                                       stream);))
  return status;
}

template <typename PT, typename IT, int VEC, int NJ, bool ZP>
int launch_hidden(const void *z, int64_t items, int D, const void *code, int H, int K, const void *win,
                  const void *run, const float *m, float code_scale, bool training, float *hidden,
                  cudaStream_t stream) {
  const int slice = 32 * NJ * VEC;
  const int lph = lanes_per_head(std::min(32 * NJ, (D + VEC - 1) / VEC));
  TB_REQUIRE(ceil_div(D, slice) < 65536, TROPNN_B200_ERR_INVALID, "trop_hidden: code_dim=%d too large", D);
  dim3 grid(static_cast<unsigned>(items), static_cast<unsigned>(ceil_div(D, slice)));
  if (training)
    trop_hidden_kernel<PT, IT, true, VEC, NJ, ZP><<<grid, kRowWarps * 32, 0, stream>>>(
        z, D, static_cast<const PT *>(code), H, K, static_cast<const IT *>(win), static_cast<const IT *>(run), m,
        code_scale, lph, hidden);
  else
    trop_hidden_kernel<PT, IT, false, VEC, NJ, ZP><<<grid, kRowWarps * 32, 0, stream>>>(
        z, D, static_cast<const PT *>(code), H, K, static_cast<const IT *>(win), static_cast<const IT *>(win), m,
        code_scale, lph, hidden);
  return check_launch("trop_hidden");
}

template <typename PT, typename IT, bool ZP>
int hidden_by_width(const void *z, int64_t items, int D, const void *code, int H, int K, const void *win,
                    const void *run, const float *m, float code_scale, bool training, float *hidden,
                    cudaStream_t stream) {
  if (row_vec_ok<PT>(D, code, code, code))
    return launch_hidden<PT, IT, 16 / sizeof(PT), 2, ZP>(z, items, D, code, H, K, win, run, m, code_scale, training,
                                                          hidden, stream);
  return launch_hidden<PT, IT, 1, 8, ZP>(z, items, D, code, H, K, win, run, m, code_scale, training, hidden, stream);
}

int trop_hidden_impl(const void *z, int zt, int64_t items, int64_t D, const void *code, const void *code_t, int pt,
                     int64_t H, int64_t K, const void *win, const void *run, int it, const float *m, float code_scale,
                     int training, float *hidden, void *hidden_split, void *ws, size_t wsb, cudaStream_t stream) {
  TB_CHECK(validate_trop(items, D, H, K));
  TB_REQUIRE(hidden_split == nullptr || pt == TROPNN_B200_F16 || pt == TROPNN_B200_BF16, TROPNN_B200_ERR_DTYPE,
             "trop_hidden: hidden_split needs f16/bf16 codes, got %s", dtype_name(pt));
  TB_REQUIRE(is_float_dtype(pt), TROPNN_B200_ERR_DTYPE, "trop_hidden: param dtype %s unsupported", dtype_name(pt));
  TB_CHECK(check_index_dtype(K, it));
  TB_CHECK(check_latent_dtype(zt, pt, "trop_hidden"));
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(z && code && win && hidden && (!training || (run && m)), TROPNN_B200_ERR_INVALID,
             "trop_hidden: null pointer");
  // Half-precision codes with their transpose at hand: one-hot GEMM on the tensor cores.
  if (hidden_sm100_supported(items, D, H, K, pt, zt, it, z, code_t, hidden))
    return trop_hidden_sm100_impl(z, zt, items, D, code_t, pt, H, K, win, run, m, code_scale, training, nullptr, hidden,
                                  hidden_split, ws, wsb, stream);
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H), Ki = static_cast<int>(K);
  const bool train = training != 0;
  const bool zp = zt != TROPNN_B200_F32;
  int status = TROPNN_B200_OK;
  TB_DISPATCH_PT(pt, TB_DISPATCH_IT(it, {
    if constexpr (sizeof(PT) == 2) {
      if (zp) {
        status = hidden_by_width<PT, IT, true>(z, items, Di, code, Hi, Ki, win, run, m, code_scale, train, hidden,
                                               stream);
        break;
      }
    }
    status = hidden_by_width<PT, IT, false>(z, items, Di, code, Hi, Ki, win, run, m, code_scale, train, hidden,
                                            stream);
  }))
  if (status != TROPNN_B200_OK || hidden_split == nullptr) return status;
  return split_half_impl(hidden, items, D, pt, nullptr, hidden_split, stream);
}

template <typename PT, typename IT, int VEC, int NJ>
int launch_backward_rows(const float *g, int64_t items, int D, const void *W, const void *code, int H, int K,
                         const void *win, const void *run, const float *m, float code_scale, bool training, float *gz,
                         float *cw, float *cr, float *gm, cudaStream_t stream) {
  const int slots = (D + VEC - 1) / VEC;
  TB_REQUIRE(slots <= 32 * NJ, TROPNN_B200_ERR_INVALID,
             "trop_backward_rows: code_dim=%d exceeds the per-row limit (%d elements)", D, 32 * NJ * VEC);
  const int lph = lanes_per_head(slots);
  const unsigned blocks = static_cast<unsigned>(items);
  if (training)
    trop_backward_rows_kernel<PT, IT, true, VEC, NJ><<<blocks, kRowWarps * 32, 0, stream>>>(
        g, D, static_cast<const PT *>(W), static_cast<const PT *>(code), H, K, static_cast<const IT *>(win),
        static_cast<const IT *>(run), m, code_scale, lph, gz, cw, cr, gm);
  else
    trop_backward_rows_kernel<PT, IT, false, VEC, NJ><<<blocks, kRowWarps * 32, 0, stream>>>(
        g, D, static_cast<const PT *>(W), static_cast<const PT *>(code), H, K, static_cast<const IT *>(win),
        static_cast<const IT *>(win), m, code_scale, lph, gz, cw, cr, gm);
  return check_launch("trop_backward_rows");
}

int trop_backward_rows_impl(const float *g, int64_t items, int64_t D, const void *W, const void *code, int pt,
                            int64_t H, int64_t K, const void *win, const void *run, int it, const float *m,
                            float code_scale, int training, float *gz, float *cw, float *cr, float *gm,
                            cudaStream_t stream) {
  TB_CHECK(validate_trop(items, D, H, K));
  TB_REQUIRE(is_float_dtype(pt), TROPNN_B200_ERR_DTYPE, "trop_backward_rows: param dtype %s unsupported",
             dtype_name(pt));
  TB_CHECK(check_index_dtype(K, it));
  if (items == 0) return TROPNN_B200_OK;
  TB_REQUIRE(g && code && win && gz && cw && (!training || (W && run && m && cr && gm)), TROPNN_B200_ERR_INVALID,
             "trop_backward_rows: null pointer");
  const int Di = static_cast<int>(D), Hi = static_cast<int>(H), Ki = static_cast<int>(K);
  const bool train = training != 0;
  int status = TROPNN_B200_OK;
  TB_DISPATCH_PT(pt, TB_DISPATCH_IT(it, {
    const bool vec = row_vec_ok<PT>(Di, code, train ? W : code, g) && (reinterpret_cast<uintptr_t>(g) % 16 == 0);
    if (vec)
      status = launch_backward_rows<PT, IT, 16 / sizeof(PT), 2>(g, items, Di, W, code, Hi, Ki, win, run, m,
                                                                 code_scale, train, gz, cw, cr, gm, stream);
    else
      status = launch_backward_rows<PT, IT, 1, 8>(g, items, Di, W, code, Hi, Ki, win, run, m, code_scale, train, gz,
                                                  cw, cr, gm, stream);
  }))
  return status;
}

struct TropBackwardLayout {
  float *coef_w, *coef_r, *gm;
  int32_t *perm_w, *seg_w, *perm_r, *seg_r;
};

static size_t trop_backward_layout(void *ws, size_t bytes, int64_t items, int64_t H, int64_t K, int training,
                                   TropBackwardLayout *L) {
  WorkspaceCarver c(ws, bytes);
  L->coef_w = c.take<float>(size_t(items) * H);
  L->coef_r = training ? c.take<float>(size_t(items) * H) : nullptr;
  L->gm = training ? c.take<float>(size_t(items) * H) : nullptr;
  L->perm_w = c.take<int32_t>(size_t(items) * H);
  L->seg_w = c.take<int32_t>(size_t(H) * (K + 1));
  L->perm_r = training ? c.take<int32_t>(size_t(items) * H) : nullptr;
  L->seg_r = training ? c.take<int32_t>(size_t(H) * (K + 1)) : nullptr;
  return WorkspaceCarver::align(c.used);
}

size_t trop_backward_workspace(int64_t items, int64_t H, int64_t K, int training) {
  if (items < 0 || H < 1 || K < 2) return 0;
  TropBackwardLayout L{};
  return trop_backward_layout(nullptr, 0, items, H, K, training, &L);
}

namespace {

// Parameter gradients of an f32 TropLinear straight from the rows (no bucket sort): CTA =
// (head h, 32-column chunk), 8 warps = 8 row groups of 32 columns; group q takes rows q, q+8,
// ... in order and accumulates in its own shared-memory copy (a warp's lanes update one cell
// row: no bank conflicts)
//   grad_code[h, k, c]   += coef_w[n, h] [w = k] g[n, c] + coef_r[n, h] [r = k] g[n, c]
//   grad_router[h, k, c] += gm[n, h] ([w = k] - [r = k]) z[n, c]
//   grad_bias[h, k]      += gm[n, h] ([w = k] - [r = k])
// (tropical_exact.py:204-237 summed over the batch); the eight copies are then added in group
// order (deterministic). Rows go in chunks of kPgrChunk: the chunk's routes, coefficients and
// g / z column slices are first staged in shared memory with every load in flight at once,
// so the accumulation loop reads shared memory only.
constexpr int kPgrGroups = 8;
constexpr int kPgrCols = 32;
constexpr int kPgrMaxCells = 32;
constexpr int kPgrChunk = 128;

__host__ __device__ inline int pgr_acc_floats(int K, bool code, bool router) {
  return (code ? kPgrGroups * K * kPgrCols : 0) + (router ? kPgrGroups * K * (kPgrCols + 1) : 0);
}

__global__ void __launch_bounds__(kPgrGroups * kPgrCols) trop_param_grad_rows_kernel(
    const float *__restrict__ g, const float *__restrict__ z, int64_t items, int D, int H, int K,
    const uint8_t *__restrict__ win, const uint8_t *__restrict__ run, const float *__restrict__ coef_w,
    const float *__restrict__ coef_r, float coef_const, const float *__restrict__ gm, float *__restrict__ gc,
    float *__restrict__ gW, float *__restrict__ gb) {
  extern __shared__ float pgr_smem[];
  const int h = blockIdx.x;
  const int chunk = blockIdx.y;
  const int q = threadIdx.x >> 5;
  const int cl = threadIdx.x & 31;
  const int col0 = chunk * kPgrCols;
  const bool want_code = gc != nullptr, want_router = gW != nullptr;
  const bool has_run = run != nullptr, has_cr = has_run && coef_r != nullptr;
  float *accC = pgr_smem;                                              // [groups][K][32]
  float *accW = accC + (want_code ? kPgrGroups * K * kPgrCols : 0);    // [groups][K][32]
  float *accB = accW + (want_router ? kPgrGroups * K * kPgrCols : 0);  // [groups][K]
  const int total = pgr_acc_floats(K, want_code, want_router);
  float *s_cw = pgr_smem + total;  // staged per row of the chunk
  float *s_cr = s_cw + kPgrChunk;
  float *s_gm = s_cr + kPgrChunk;
  int *s_route = reinterpret_cast<int *>(s_gm + kPgrChunk);  // w | r << 8 (-1: skip the row)
  float *s_g = reinterpret_cast<float *>(s_route + kPgrChunk);  // [chunk rows][32]
  float *s_z = s_g + kPgrChunk * kPgrCols;                       // [chunk rows][32]
  for (int i = threadIdx.x; i < total; i += blockDim.x) pgr_smem[i] = 0.f;
  float *myC = accC + q * K * kPgrCols + cl;
  float *myW = accW + q * K * kPgrCols + cl;
  float *myB = accB + q * K;
  const bool bias_lane = want_router && cl == 0 && chunk == 0;
  for (int64_t n0 = 0; n0 < items; n0 += kPgrChunk) {
    const int nrows = static_cast<int>(min64(kPgrChunk, items - n0));
    __syncthreads();  // the previous chunk is done with the staging arrays (and the zeroing above)
    for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
      const int64_t nh = (n0 + i) * H + h;
      const int w = __ldg(win + nh);
      const int r = has_run ? __ldg(run + nh) : 0;
      // Not a route of this layer: nothing to add for the row.
      s_route[i] = (w < K && r < K) ? (w | (r << 8)) : -1;
      s_cw[i] = coef_w != nullptr ? __ldg(coef_w + nh) : coef_const;
      s_cr[i] = has_cr ? __ldg(coef_r + nh) : 0.f;
      s_gm[i] = gm != nullptr ? __ldg(gm + nh) : 0.f;
    }
    // The chunk's column slices: consecutive threads read consecutive columns of a row, eight
    // loads of each slice in flight per thread before the stores.
    constexpr int kU = 8;
    const int n_el = nrows * kPgrCols;
    for (int base = threadIdx.x; base < n_el; base += kU * kPgrGroups * kPgrCols) {
      float vg[kU], vz[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = base + u * kPgrGroups * kPgrCols;
        const int64_t n = n0 + (i >> 5);
        const int c = col0 + (i & 31);
        const bool live = i < n_el && c < D;
        vg[u] = (want_code && live) ? __ldg(g + n * D + c) : 0.f;
        vz[u] = (want_router && live) ? __ldg(z + n * D + c) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = base + u * kPgrGroups * kPgrCols;
        if (i < n_el) {
          if (want_code) s_g[i] = vg[u];
          if (want_router) s_z[i] = vz[u];
        }
      }
    }
    __syncthreads();
    for (int j = q; j < nrows; j += kPgrGroups) {
      const int route = s_route[j];
      if (route < 0) continue;
      const int w = route & 0xff, r = route >> 8;
      if (want_code) {
        const float gv = s_g[j * kPgrCols + cl];
        myC[w * kPgrCols] = fmaf(s_cw[j], gv, myC[w * kPgrCols]);
        if (has_cr) myC[r * kPgrCols] = fmaf(s_cr[j], gv, myC[r * kPgrCols]);
      }
      if (want_router) {
        const float zv = s_z[j * kPgrCols + cl];
        const float m = s_gm[j];
        myW[w * kPgrCols] = fmaf(m, zv, myW[w * kPgrCols]);
        myW[r * kPgrCols] = fmaf(-m, zv, myW[r * kPgrCols]);
        if (bias_lane) {
          myB[w] = __fadd_rn(myB[w], m);
          myB[r] = __fsub_rn(myB[r], m);
        }
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < K * kPgrCols; i += blockDim.x) {
    const int k = i / kPgrCols, c = i - k * kPgrCols;
    const int oc = col0 + c;
    if (oc >= D) continue;
    const int64_t o = (int64_t(h) * K + k) * D + oc;
    if (want_code) {
      float s = accC[k * kPgrCols + c];
      for (int p = 1; p < kPgrGroups; ++p) s = __fadd_rn(s, accC[(p * K + k) * kPgrCols + c]);
      gc[o] = s;
    }
    if (want_router) {
      float s = accW[k * kPgrCols + c];
      for (int p = 1; p < kPgrGroups; ++p) s = __fadd_rn(s, accW[(p * K + k) * kPgrCols + c]);
      gW[o] = s;
    }
  }
  if (want_router && chunk == 0 && threadIdx.x < K) {
    float s = accB[threadIdx.x];
    for (int p = 1; p < kPgrGroups; ++p) s = __fadd_rn(s, accB[p * K + threadIdx.x]);
    gb[int64_t(h) * K + threadIdx.x] = s;
  }
}

}  // namespace

bool trop_param_grad_rows_supported(int pt, int it, int64_t K, int64_t H, int64_t D) {
  return pt == TROPNN_B200_F32 && it == TROPNN_B200_U8 && K >= 2 && K <= kPgrMaxCells && H >= 1 && H < 65536 * 1024 &&
         D >= 1 && D <= (1 << 20);
}

int trop_param_grad_rows_impl(const float *g, const float *z, int64_t items, int64_t D, int64_t H, int64_t K,
                              const void *win, const void *run, const float *coef_w, const float *coef_r,
                              float coef_const, const float *gm, float *gc, float *gW, float *gb,
                              cudaStream_t stream) {
  TB_REQUIRE(trop_param_grad_rows_supported(TROPNN_B200_F32, TROPNN_B200_U8, K, H, D), TROPNN_B200_ERR_INVALID,
             "trop_param_grad_rows: unsupported shape heads=%lld cells=%lld code_dim=%lld", (long long)H, (long long)K,
             (long long)D);
  TB_REQUIRE((gW == nullptr) == (gb == nullptr), TROPNN_B200_ERR_INVALID,
             "trop_param_grad_rows: grad_router_weight and grad_router_bias go together");
  TB_REQUIRE(win != nullptr && (gc == nullptr || g != nullptr) &&
                 (gW == nullptr || (z != nullptr && run != nullptr && gm != nullptr)) &&
                 (coef_r == nullptr || run != nullptr),
             TROPNN_B200_ERR_INVALID, "trop_param_grad_rows: null pointer");
  if (gc == nullptr && gW == nullptr) return TROPNN_B200_OK;
  const size_t smem = sizeof(float) * (pgr_acc_floats(static_cast<int>(K), gc != nullptr, gW != nullptr) +
                                       4 * kPgrChunk + 2 * kPgrChunk * kPgrCols);
  TB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(trop_param_grad_rows_kernel), smem,
                               "trop_param_grad_rows"));
  const dim3 grid(static_cast<unsigned>(H), static_cast<unsigned>(ceil_div(D, int64_t(kPgrCols))));
  trop_param_grad_rows_kernel<<<grid, kPgrGroups * kPgrCols, smem, stream>>>(
      g, z, items, static_cast<int>(D), static_cast<int>(H), static_cast<int>(K), static_cast<const uint8_t *>(win),
      static_cast<const uint8_t *>(run), coef_w, coef_r, coef_const, gm, gc, gW, gb);
  return check_launch("trop_param_grad_rows");
}

int trop_backward_impl(const float *g, const float *z, int64_t items, int64_t D, const void *W, const void *code,
                       int pt, int64_t H, int64_t K, const void *win, const void *run, int it, const float *m,
                       float code_scale, int training, float *gz, void *gW, void *gb, void *gc, void *ws,
                       size_t ws_bytes, cudaStream_t stream) {
  TB_CHECK(validate_trop(items, D, H, K));
  TropBackwardLayout L{};
  const size_t need = trop_backward_layout(ws, ws_bytes, items, H, K, training, &L);
  TB_REQUIRE(ws != nullptr && need <= ws_bytes, TROPNN_B200_ERR_WORKSPACE,
             "trop_backward: workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes, need);
  TB_REQUIRE(gz != nullptr, TROPNN_B200_ERR_INVALID, "trop_backward: grad_latent is required");
  TB_CHECK(trop_backward_rows_impl(g, items, D, W, code, pt, H, K, win, run, it, m, code_scale, training, gz,
                                   L.coef_w, L.coef_r, L.gm, stream));
  if (items == 0) return TROPNN_B200_OK;
  if (trop_param_grad_rows_supported(pt, it, K, H, D)) {
    TB_REQUIRE(!(training && (gW != nullptr || gb != nullptr)) || (gW != nullptr && gb != nullptr && z != nullptr),
               TROPNN_B200_ERR_INVALID, "trop_backward: grad_router_weight, grad_router_bias and latent go together");
    return trop_param_grad_rows_impl(g, z, items, D, H, K, win, training ? run : nullptr, L.coef_w,
                                     training ? L.coef_r : nullptr, 1.f, L.gm, static_cast<float *>(gc),
                                     training ? static_cast<float *>(gW) : nullptr,
                                     training ? static_cast<float *>(gb) : nullptr, stream);
  }
  TB_CHECK(bucket_sort_impl(win, it, items, H, H, K, L.perm_w, L.seg_w, stream));
  if (training) TB_CHECK(bucket_sort_impl(run, it, items, H, H, K, L.perm_r, L.seg_r, stream));
  if (gc != nullptr) {
    TB_CHECK(segment_rowsum_impl(g, items, D, D, H, K, L.perm_w, L.seg_w, L.coef_w, 1.f, L.perm_r, L.seg_r,
                                 L.coef_r, 1.f, 1.f, gc, pt, nullptr, stream));
  }
  if (training && (gW != nullptr || gb != nullptr)) {
    TB_REQUIRE(gW != nullptr && gb != nullptr && z != nullptr, TROPNN_B200_ERR_INVALID,
               "trop_backward: grad_router_weight, grad_router_bias and latent go together");
    TB_CHECK(segment_rowsum_impl(z, items, D, D, H, K, L.perm_w, L.seg_w, L.gm, 1.f, L.perm_r, L.seg_r, L.gm, -1.f,
                                 1.f, gW, pt, gb, stream));
  }
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

size_t tropnn_b200_trop_route_workspace_size(int64_t items, int64_t code_dim, int64_t heads, int64_t cells,
                                             int latent_dtype, int param_dtype) {
  return tropnn_b200::trop_route_workspace(items, code_dim, heads, cells, latent_dtype, param_dtype);
}

int tropnn_b200_trop_route(const void *latent, int latent_dtype, int64_t items, int64_t code_dim,
                           const void *router_weight, const void *router_bias, int bias_dtype, int param_dtype,
                           int64_t heads, int64_t cells, int64_t *winner_i64, void *winner, void *runner,
                           int index_dtype, float *margins, void *workspace, size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_route_impl(latent, latent_dtype, items, code_dim, router_weight, router_bias, bias_dtype,
                                        param_dtype, heads, cells, winner_i64, winner, runner, index_dtype, margins,
                                        workspace, workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

size_t tropnn_b200_trop_hidden_workspace_size(int64_t items, int64_t code_dim, int64_t heads, int64_t cells) {
  return tropnn_b200::trop_hidden_sm100_workspace(items, code_dim, heads, cells);
}

int tropnn_b200_trop_hidden(const void *latent, int latent_dtype, int64_t items, int64_t code_dim, const void *code,
                            const void *code_t, int param_dtype, int64_t heads, int64_t cells, const void *winner,
                            const void *runner, int index_dtype, const float *margins, float code_scale, int training,
                            float *hidden, void *hidden_split, void *workspace, size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_hidden_impl(latent, latent_dtype, items, code_dim, code, code_t, param_dtype, heads, cells,
                                         winner, runner, index_dtype, margins, code_scale, training, hidden,
                                         hidden_split, workspace, workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_code_transpose(const void *code, int param_dtype, int64_t heads, int64_t cells, int64_t code_dim,
                                    void *code_t, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_code_transpose_impl(code, param_dtype, heads, cells, code_dim, code_t,
                                                 tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_gm(const void *g_split, int64_t items, int64_t code_dim, const void *code, int param_dtype,
                        int64_t heads, int64_t cells, const void *winner, const void *runner, const float *margins,
                        float code_scale, float *gm, const void *grad_absmax, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  if (items == 0) return tropnn_b200::clear_error();
  TB_CHECK(tropnn_b200::trop_gm_sm100_impl(g_split, items, code_dim, code, param_dtype, heads, cells,
                                           static_cast<const uint8_t *>(winner), static_cast<const uint8_t *>(runner),
                                           margins, code_scale, gm, static_cast<const uint32_t *>(grad_absmax),
                                           tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_router_term(const float *grad_hidden, int64_t items, int64_t code_dim, const void *router_weight_t,
                                 int param_dtype, int64_t heads, int64_t cells, const void *winner, const void *runner,
                                 const float *gm, const void *grad_absmax, float *grad_latent, void *workspace,
                                 size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  if (items == 0) return tropnn_b200::clear_error();
  TB_CHECK(tropnn_b200::trop_hidden_sm100_impl(grad_hidden, TROPNN_B200_F32, items, code_dim, router_weight_t,
                                               param_dtype, heads, cells, winner, runner, gm, 1.0f, 2,
                                               static_cast<const uint32_t *>(grad_absmax), grad_latent, nullptr,
                                               workspace, workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_param_grad(int mode, const void *x_t, int64_t items, int64_t code_dim, int param_dtype,
                                int64_t heads, int64_t cells, const void *winner, const void *runner,
                                const float *values, float code_scale, void *grad, void *grad_bias,
                                const void *grad_absmax, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_param_grad_sm100_impl(mode, x_t, items, code_dim, param_dtype, heads, cells, winner,
                                                   runner, values, code_scale, grad, grad_bias,
                                                   static_cast<const uint32_t *>(grad_absmax),
                                                   tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_transpose_to_half(const void *x, int x_dtype, int64_t rows, int64_t cols, int dtype,
                                  const void *grad_absmax, void *out, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::transpose_to_half_impl(x, x_dtype, rows, cols, dtype, out,
                                               static_cast<const uint32_t *>(grad_absmax),
                                               tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_device_error(int *value) {
  TB_CHECK(tropnn_b200::check_current_device());
  int score = 0, hidden = 0, gemm = 0, peer = 0, pgrad = 0, lgrad = 0, lutg = 0, proj = 0, gtf32 = 0, pair = 0;
  TB_CHECK(tropnn_b200::read_score_error(&score));
  TB_CHECK(tropnn_b200::read_hidden_error(&hidden));
  TB_CHECK(tropnn_b200::read_gemm_error(&gemm));
  TB_CHECK(tropnn_b200::read_peer_error(&peer));
  TB_CHECK(tropnn_b200::read_param_grad_error(&pgrad));
  TB_CHECK(tropnn_b200::read_linear_grad_error(&lgrad));
  TB_CHECK(tropnn_b200::read_lut_grad_error(&lutg));
  TB_CHECK(tropnn_b200::read_proj_error(&proj));
  TB_CHECK(tropnn_b200::read_gemm_tf32_error(&gtf32));
  TB_CHECK(tropnn_b200::read_pairwise_error(&pair));
  *value = score | hidden | gemm | peer | pgrad | lgrad | lutg | proj | gtf32 | pair;
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_backward_rows(const float *grad_hidden, int64_t items, int64_t code_dim,
                                   const void *router_weight, const void *code, int param_dtype, int64_t heads,
                                   int64_t cells, const void *winner, const void *runner, int index_dtype,
                                   const float *margins, float code_scale, int training, float *grad_latent,
                                   float *coef_w, float *coef_r, float *gm, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_backward_rows_impl(grad_hidden, items, code_dim, router_weight, code, param_dtype, heads,
                                                cells, winner, runner, index_dtype, margins, code_scale, training,
                                                grad_latent, coef_w, coef_r, gm, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

int tropnn_b200_trop_param_grad_rows(const float *grad_hidden, const float *latent, int64_t items, int64_t code_dim,
                                     int param_dtype, int64_t heads, int64_t cells, const void *winner,
                                     const void *runner, int index_dtype, const float *coef_w, const float *coef_r,
                                     float coef_const, const float *gm, void *grad_code, void *grad_router_weight,
                                     void *grad_router_bias, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::validate_trop(items, code_dim, heads, cells));
  TB_REQUIRE(tropnn_b200::trop_param_grad_rows_supported(param_dtype, index_dtype, cells, heads, code_dim),
             TROPNN_B200_ERR_INVALID, "trop_param_grad_rows: needs F32 parameters, U8 routes and 2-32 cells");
  if (items == 0) return tropnn_b200::clear_error();
  TB_CHECK(tropnn_b200::trop_param_grad_rows_impl(
      grad_hidden, latent, items, code_dim, heads, cells, winner, runner, coef_w, coef_r, coef_const, gm,
      static_cast<float *>(grad_code), static_cast<float *>(grad_router_weight), static_cast<float *>(grad_router_bias),
      tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

size_t tropnn_b200_trop_backward_workspace_size(int64_t items, int64_t heads, int64_t cells, int training) {
  return tropnn_b200::trop_backward_workspace(items, heads, cells, training);
}

int tropnn_b200_trop_backward(const float *grad_hidden, const float *latent, int64_t items, int64_t code_dim,
                              const void *router_weight, const void *code, int param_dtype, int64_t heads,
                              int64_t cells, const void *winner, const void *runner, int index_dtype,
                              const float *margins, float code_scale, int training, float *grad_latent,
                              void *grad_router_weight, void *grad_router_bias, void *grad_code, void *workspace,
                              size_t workspace_bytes, void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  TB_CHECK(tropnn_b200::trop_backward_impl(grad_hidden, latent, items, code_dim, router_weight, code, param_dtype,
                                           heads, cells, winner, runner, index_dtype, margins, code_scale, training,
                                           grad_latent, grad_router_weight, grad_router_bias, grad_code, workspace,
                                           workspace_bytes, tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
