// Native CPU inference kernels of tropnn — TEST INFRASTRUCTURE ONLY (an extra oracle and an
// optional CPU baseline; the product path, tropnn_b200, never loads this library).
//
// A C++ restatement of the reference's Zig CPU backend (kernels/src/*.zig), which cannot be
// built here (no Zig toolchain):
//   * TropLinear route + selected-code sum, inference only (kernels/src/tropical.zig:5-350):
//     hidden = latent; for every head, the best cell is the first strict maximum of
//     <latent, router_weight[h,c]> + router_bias[h,c]; hidden += code_scale * code[h, best].
//   * PairwiseLinear comparator hash + LUT sum, inference only (kernels/src/lut.zig:5-318):
//     idx_t = sum_r [(x[a] - x[b]) - threshold > 0] << r; out = sum_t lut[t, idx_t] (zeroed first,
//     tables added four at a time: out += ((l0 + l1) + l2) + l3, the rest one at a time).
//   * f16 parameters are widened to f32 per element, f32 accumulation
//     (trop_route_hidden_batch_f16, lut_forward_batch_f16_no_cache).
//   * Rows are split into contiguous ranges, one per thread, the last range on the calling thread
//     (kernels/src/parallel.zig:27-63; at least 128 rows per thread for TropLinear, 64 for
//     Pairwise, as the reference's call sites ask).
// Arithmetic order follows the Zig kernels: dot products in 16 lane accumulators added in lane
// order, then the tail; products and sums rounded separately (built with -ffp-contract=off and
// -march=x86-64-v3; oracle/native.py checks the host CPU before loading it).
// Parity: pinned by the Zig files' own known-answer tests (tropical.zig:352-379,
// lut.zig:320-325) and checked against the numpy oracle on the golden cases
// (tests/test_native_cpu.py).
#include <immintrin.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

constexpr int kLanes = 16;

inline float widen(float v) { return v; }
// f16 bits widened exactly by F16C (vcvtph2ps), as the Zig kernels' f16 -> f32 casts compile on
// such CPUs. The library is built for x86-64-v3 (AVX2, FMA, F16C).
inline float widen(uint16_t v) { return _cvtsh_ss(v); }

// 16-wide vectors, as the Zig kernels' @Vector(16, f32) (two ymm registers on x86-64-v3); 16
// f16 values widen with two vcvtph2ps.
typedef float VecF __attribute__((vector_size(4 * kLanes)));

inline VecF load_vec(const float *p) {
  VecF v;
  std::memcpy(&v, p, sizeof v);
  return v;
}
inline VecF load_vec(const uint16_t *p) {
  const __m256 lo = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i *>(p)));
  const __m256 hi = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i *>(p + 8)));
  VecF v;
  std::memcpy(&v, &lo, sizeof lo);
  std::memcpy(reinterpret_cast<char *>(&v) + sizeof lo, &hi, sizeof hi);
  return v;
}
inline void store_vec(float *p, VecF v) { std::memcpy(p, &v, sizeof v); }

// <a, b> as the Zig kernels form it: a 16-lane accumulator over whole 16-element chunks, its lanes
// added in order; the tail products are returned apart so that the caller can add them before or
// after the bias (the two orders of tropical.zig's generic and small-cell paths).
template <typename P>
inline float lane_sum(const float *a, const P *b, int64_t n, int64_t *tail_start) {
  VecF acc = {};
  int64_t i = 0;
  for (; i + kLanes <= n; i += kLanes) acc = acc + load_vec(a + i) * load_vec(b + i);
  float total = acc[0];
  for (int k = 1; k < kLanes; ++k) total = total + acc[k];
  *tail_start = i;
  return total;
}

template <typename P>
inline float add_tail(float total, const float *a, const P *b, int64_t i, int64_t n) {
  for (; i < n; ++i) total = total + a[i] * widen(b[i]);
  return total;
}

// dest += src * scale (tropical.zig's addScaled / addScaledF16).
template <typename P>
inline void add_scaled(float *dest, const P *src, float scale, int64_t n) {
  int64_t i = 0;
  const VecF sv = scale - VecF{};
  for (; i + kLanes <= n; i += kLanes) store_vec(dest + i, load_vec(dest + i) + load_vec(src + i) * sv);
  for (; i < n; ++i) dest[i] = dest[i] + widen(src[i]) * scale;
}

// dest += ((s0 + s1) + s2) + s3 (lut.zig's four-table step), and dest += s.
template <typename P>
inline void add_four(float *dest, const P *s0, const P *s1, const P *s2, const P *s3, int64_t n) {
  int64_t i = 0;
  for (; i + kLanes <= n; i += kLanes)
    store_vec(dest + i, load_vec(dest + i) + (((load_vec(s0 + i) + load_vec(s1 + i)) + load_vec(s2 + i)) + load_vec(s3 + i)));
  for (; i < n; ++i) dest[i] = dest[i] + (((widen(s0[i]) + widen(s1[i])) + widen(s2[i])) + widen(s3[i]));
}

template <typename P>
inline void add_one(float *dest, const P *s, int64_t n) {
  int64_t i = 0;
  for (; i + kLanes <= n; i += kLanes) store_vec(dest + i, load_vec(dest + i) + load_vec(s + i));
  for (; i < n; ++i) dest[i] = dest[i] + widen(s[i]);
}

template <typename P>
void trop_rows(int64_t r0, int64_t r1, int64_t heads, int64_t cells, int64_t dim, float scale, const float *latent,
               const P *weight, const P *bias, const P *code, float *hidden) {
  for (int64_t n = r0; n < r1; ++n) {
    const float *x = latent + n * dim;
    float *h = hidden + n * dim;
    std::memcpy(h, x, sizeof(float) * size_t(dim));
    for (int64_t hd = 0; hd < heads; ++hd) {
      // 2-4 cells (tropical.zig:29-70): bias added before the tail products, the running best
      // seeded with cell 0. Other cell counts (tropical.zig:5-27): the full dot, then the bias,
      // the running best seeded with -inf. Both keep the first strict maximum.
      const bool small = cells >= 2 && cells <= 4;
      int64_t best = 0;
      float best_score = -std::numeric_limits<float>::infinity();
      for (int64_t c = 0; c < cells; ++c) {
        const P *wc = weight + (hd * cells + c) * dim;
        const float bc = widen(bias[hd * cells + c]);
        int64_t tail = 0;
        const float lanes = lane_sum(x, wc, dim, &tail);
        const float s = small ? add_tail(lanes + bc, x, wc, tail, dim) : add_tail(lanes, x, wc, tail, dim) + bc;
        if ((small && c == 0) || s > best_score) {
          best_score = s;
          best = c;
        }
      }
      add_scaled(h, code + (hd * cells + best) * dim, scale, dim);
    }
  }
}

inline int64_t lut_index(const float *x, const int64_t *anchors, const float *offsets, int64_t t, int64_t C) {
  int64_t idx = 0;
  for (int64_t r = 0; r < C; ++r) {
    const int64_t a = anchors[(t * C + r) * 2], b = anchors[(t * C + r) * 2 + 1];
    const float margin = (x[a] - x[b]) - offsets[t * C + r];
    idx |= int64_t(margin > 0.f) << r;
  }
  return idx;
}

template <typename P>
void lut_rows(int64_t r0, int64_t r1, int64_t tables, int64_t C, int64_t in, int64_t out, const P *weights,
              const int64_t *anchors, const float *offsets, const float *inputs, float *outputs) {
  const int64_t stride = (int64_t(1) << C) * out;
  for (int64_t n = r0; n < r1; ++n) {
    const float *x = inputs + n * in;
    float *o = outputs + n * out;
    std::fill(o, o + out, 0.f);
    int64_t t = 0;
    for (; t + 4 <= tables; t += 4) {
      const P *l0 = weights + t * stride + lut_index(x, anchors, offsets, t, C) * out;
      const P *l1 = weights + (t + 1) * stride + lut_index(x, anchors, offsets, t + 1, C) * out;
      const P *l2 = weights + (t + 2) * stride + lut_index(x, anchors, offsets, t + 2, C) * out;
      const P *l3 = weights + (t + 3) * stride + lut_index(x, anchors, offsets, t + 3, C) * out;
      add_four(o, l0, l1, l2, l3, out);
    }
    for (; t < tables; ++t) {
      add_one(o, weights + t * stride + lut_index(x, anchors, offsets, t, C) * out, out);
    }
  }
}

void trop_range(int64_t r0, int64_t r1, int64_t heads, int64_t cells, int64_t dim, float scale,
                              const float *latent, const void *w, const void *b, const void *c, int f16,
                              float *hidden) {
  if (f16)
    trop_rows(r0, r1, heads, cells, dim, scale, latent, static_cast<const uint16_t *>(w),
              static_cast<const uint16_t *>(b), static_cast<const uint16_t *>(c), hidden);
  else
    trop_rows(r0, r1, heads, cells, dim, scale, latent, static_cast<const float *>(w), static_cast<const float *>(b),
              static_cast<const float *>(c), hidden);
}

void lut_range(int64_t r0, int64_t r1, int64_t tables, int64_t C, int64_t in, int64_t out,
                             const void *weights, int f16, const int64_t *anchors, const float *offsets,
                             const float *inputs, float *outputs) {
  if (f16)
    lut_rows(r0, r1, tables, C, in, out, static_cast<const uint16_t *>(weights), anchors, offsets, inputs, outputs);
  else
    lut_rows(r0, r1, tables, C, in, out, static_cast<const float *>(weights), anchors, offsets, inputs, outputs);
}

int default_threads() {
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : int(std::min(n, 64u));
}

// Contiguous row ranges over `workers` threads (the calling thread takes the last one).
template <typename F>
void parallel_rows(int64_t rows, int64_t min_rows, int threads, F &&fn) {
  if (threads <= 0) threads = default_threads();
  int64_t workers = 1;
  if (rows > min_rows && threads > 1) workers = std::min<int64_t>(threads, (rows + min_rows - 1) / min_rows);
  std::vector<std::thread> pool;
  pool.reserve(size_t(workers - 1));
  int64_t start = 0;
  for (int64_t w = 0; w < workers; ++w) {
    const int64_t end = rows * (w + 1) / workers;
    if (w + 1 == workers)
      fn(start, end);
    else
      pool.emplace_back(fn, start, end);
    start = end;
  }
  for (auto &t : pool) t.join();
}

}  // namespace

extern "C" {

int oracle_cpu_default_threads(void) { return default_threads(); }

// hidden [items, code_dim] from latent [items, code_dim], router_weight / code [heads, cells,
// code_dim] and router_bias [heads, cells] (f32, or f16 bits when param_f16). 0, or -1 for bad sizes.
int oracle_cpu_trop_route_hidden(int64_t items, int64_t heads, int64_t cells, int64_t code_dim, float code_scale,
                                 const float *latent, const void *router_weight, const void *router_bias,
                                 const void *code, int param_f16, float *hidden, int threads) {
  if (items < 0 || heads < 1 || cells < 1 || code_dim < 1) return -1;
  if (items == 0) return 0;
  if (!latent || !router_weight || !router_bias || !code || !hidden) return -1;
  parallel_rows(items, 128, threads, [&](int64_t r0, int64_t r1) {
    trop_range(r0, r1, heads, cells, code_dim, code_scale, latent, router_weight, router_bias, code, param_f16,
               hidden);
  });
  return 0;
}

// outputs [batch, output_dim] = sum over tables of weights[t, idx_t] (f32, or f16 bits when
// weights_f16), idx_t from inputs [batch, input_dim], anchors int64 [tables, comparisons, 2] and
// offsets f32 [tables, comparisons]. 0, or -1 for bad sizes or an anchor outside the input.
int oracle_cpu_lut_forward(int64_t batch, int64_t tables, int64_t comparisons, int64_t input_dim, int64_t output_dim,
                           const void *weights, int weights_f16, const int64_t *anchors, const float *offsets,
                           const float *inputs, float *outputs, int threads) {
  if (batch < 0 || tables < 1 || comparisons < 1 || comparisons > 30 || input_dim < 1 || output_dim < 1) return -1;
  if (!weights || !anchors || !offsets) return -1;
  for (int64_t i = 0; i < tables * comparisons * 2; ++i)
    if (anchors[i] < 0 || anchors[i] >= input_dim) return -1;
  if (batch == 0) return 0;
  if (!inputs || !outputs) return -1;
  parallel_rows(batch, 64, threads, [&](int64_t r0, int64_t r1) {
    lut_range(r0, r1, tables, comparisons, input_dim, output_dim, weights, weights_f16, anchors, offsets, inputs,
              outputs);
  });
  return 0;
}

}  // extern "C"
