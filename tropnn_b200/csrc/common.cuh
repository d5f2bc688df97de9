// Shared helpers of the tropnn_b200 kernels: status plumbing, dtype loads/stores,
// warp reductions. Every .cu of the library includes this header.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/tropnn_b200.h"

namespace tropnn_b200 {

// ----------------------------------------------------------------------------
// host-side status handling
// ----------------------------------------------------------------------------

// Records `fmt` as the calling thread's last error and returns `status`.
int set_error(int status, const char *fmt, ...);
// Clears the last error; returns TROPNN_B200_OK.
int clear_error();
// TROPNN_B200_OK when the current device is sm_100, else an error status.
int check_current_device();
// Maps a pending CUDA launch error to TROPNN_B200_ERR_LAUNCH (with `what` in the message).
int check_launch(const char *what);
// Raises `func`'s dynamic shared-memory limit on the current device to at least `bytes`
// (once per kernel and device; later calls are a table lookup).
int ensure_dynamic_smem(const void *func, size_t bytes, const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Epilogues of slice_reduce_impl (slice_reduce.cu): the sum of a split contraction's slice
// partials (float4 partial[tile * splits + slice][tile_cols / 4][128 rows]) rounded to a half
// dtype (or rounded and written transposed), plus an f32 bias, or added to a latent row times a
// scale (kReduceHidden also writes the [hi | lo] half-precision split of each hidden row to
// `split` [rows, 2 * cols] when it is given).
enum SliceReduceMode { kReduceHalf = 0, kReduceF32 = 1, kReduceHidden = 2, kReduceHalfT = 3 };
int slice_reduce_impl(int mode, const void *partial, int splits, int n_tiles, int tile_cols, int64_t rows,
                      int64_t cols, void *out, int out_dtype, int64_t ldo, const float *bias, const void *latent,
                      int latent_dtype, float scale, cudaStream_t stream, void *split = nullptr,
                      int split_dtype = 0);

// Power-of-two scale that brings a gradient tensor whose largest |value| has the f32 bits
// `absmax_bits` into [16, 32): converted to f16 after it, the gradient neither underflows (f16's
// smallest normal is 6.1e-5) nor overflows in the products formed from it, and the f32 results
// are divided by it again exactly. 1 for a zero or non-finite maximum.
__device__ __forceinline__ float pow2_grad_scale(uint32_t absmax_bits) {
  const int exp_field = static_cast<int>((absmax_bits >> 23) & 0xFFu);
  if (absmax_bits == 0u || exp_field == 0xFF) return 1.f;
  int e = 4 - (exp_field - 127);
  e = e < -126 ? -126 : (e > 126 ? 126 : e);
  return __int_as_float((e + 127) << 23);
}
// 1/s for a power of two s from pow2_grad_scale (exact).
__device__ __forceinline__ float pow2_inverse(float s) {
  const int e = static_cast<int>((__float_as_uint(s) >> 23) & 0xFFu) - 127;
  return __int_as_float((127 - e) << 23);
}
// The scale of pow2_grad_scale for an optional device word (NULL: 1).
__device__ __forceinline__ float grad_scale_of(const uint32_t *absmax) {
  return absmax != nullptr ? pow2_grad_scale(*absmax) : 1.f;
}

#define TB_REQUIRE(cond, status, ...)                  \
  do {                                                 \
    if (!(cond)) return ::tropnn_b200::set_error(status, __VA_ARGS__); \
  } while (0)

#define TB_CHECK(expr)                   \
  do {                                   \
    int _tb_status = (expr);             \
    if (_tb_status != TROPNN_B200_OK) return _tb_status; \
  } while (0)

inline bool is_float_dtype(int dt) {
  return dt == TROPNN_B200_F32 || dt == TROPNN_B200_F16 || dt == TROPNN_B200_BF16;
}
inline bool is_index_dtype(int dt) {
  return dt == TROPNN_B200_U8 || dt == TROPNN_B200_I16 || dt == TROPNN_B200_I64;
}
inline const char *dtype_name(int dt) {
  switch (dt) {
    case TROPNN_B200_F32: return "f32";
    case TROPNN_B200_F16: return "f16";
    case TROPNN_B200_BF16: return "bf16";
    case TROPNN_B200_U8: return "u8";
    case TROPNN_B200_I16: return "i16";
    case TROPNN_B200_I64: return "i64";
    default: return "unknown";
  }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Slice count for a contraction of `kblocks` k blocks per output tile over `tiles` tiles on
// `sms` SMs running one unit (tile, slice) at a time each: the s in [1, max_splits], with at
// least min_kb k blocks a slice, that minimises the critical path, ceil(tiles * s / sms) rounds
// of ceil(kblocks / s) k blocks at kb_us each, plus s slice partials of slice_us each for the
// ordered reduction that follows a split (none for s = 1). Ties go to fewer slices. A count
// just above a multiple of the SMs costs a whole extra round, which the old rule (enough
// slices to reach the SM count) often paid.
inline int balanced_splits(int64_t tiles, int64_t kblocks, int64_t sms, int max_splits, int min_kb, double kb_us,
                           double slice_us) {
  int best = 1;
  double best_cost = double(ceil_div(tiles, sms)) * double(kblocks) * kb_us;
  for (int s = 2; s <= max_splits; ++s) {
    const int64_t kbps = ceil_div(kblocks, s);
    if (kbps < min_kb) break;
    if (ceil_div(kblocks, kbps) != s) continue;  // forms fewer slices: a smaller s covers it
    const double cost = double(ceil_div(tiles * s, sms)) * double(kbps) * kb_us + double(s) * slice_us;
    if (cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// 256-byte aligned carving of a caller-provided workspace.
struct WorkspaceCarver {
  char *base;
  size_t size;
  size_t used = 0;
  WorkspaceCarver(void *b, size_t s) : base(static_cast<char *>(b)), size(s) {}
  static size_t align(size_t v) { return (v + 255) & ~size_t(255); }
  template <typename T>
  T *take(size_t count) {
    size_t off = align(used);
    used = off + count * sizeof(T);
    if (base == nullptr || used > size) return nullptr;
    return reinterpret_cast<T *>(base + off);
  }
};

// ----------------------------------------------------------------------------
// device-side helpers
// ----------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ float ldg_f32(const T *p) { return to_f32<T>(__ldg(p)); }

// Index loads of the packed route payloads (uint8 / int16 / int64).
template <typename I>
__device__ __forceinline__ int ld_index(const I *p) { return static_cast<int>(__ldg(p)); }

// Loads VEC consecutive elements (16 bytes) as floats. Caller guarantees alignment.
template <typename T, int VEC>
struct VecLoad;
template <>
struct VecLoad<float, 4> {
  static __device__ __forceinline__ void load(const float *p, float (&v)[4]) {
    float4 q = __ldg(reinterpret_cast<const float4 *>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
};
template <>
struct VecLoad<__half, 8> {
  static __device__ __forceinline__ void load(const __half *p, float (&v)[8]) {
    uint4 q = __ldg(reinterpret_cast<const uint4 *>(p));
    const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
  }
};
template <>
struct VecLoad<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[8]) {
    uint4 q = __ldg(reinterpret_cast<const uint4 *>(p));
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x; v[2 * i + 1] = f.y;
    }
  }
};
template <>
struct VecLoad<float, 8> {
  static __device__ __forceinline__ void load(const float *p, float (&v)[8]) {
    float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};
template <typename T, int VEC>
struct VecLoad {
  // Scalar fallback (VEC == 1).
  static __device__ __forceinline__ void load(const T *p, float (&v)[VEC]) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = ldg_f32(p + i);
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// fast_sigmoid_odd and izhikevich surrogate derivatives (layers/surrogate.py:9-17),
// evaluated in the same operation order as the reference's torch expressions.
__device__ __forceinline__ float surrogate_grad(float u, int kind) {
  if (kind == TROPNN_B200_SURROGATE_FAST_SIGMOID_ODD) {
    float sgn = (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
    float den = __fadd_rn(1.f, fabsf(u));
    den = __fmul_rn(den, den);
    return __fdiv_rn(__fmul_rn(-0.5f, sgn), den);
  }
  float au = fabsf(u);
  float sig = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-au)));
  float sgn = (u > 0.f) ? -1.f : 1.f;
  return __fmul_rn(__fmul_rn(__fmul_rn(sgn, 2.f), sig), __fsub_rn(1.f, sig));
}

}  // namespace tropnn_b200
