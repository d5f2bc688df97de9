/*
 * tropnn_b200 — C ABI of the sm_100a kernels behind backend="b200".
 *
 * Every entry point takes plain device pointers, int64 sizes, dtype enums and a
 * cudaStream_t passed as `void *` (NULL = legacy default stream). Nothing here
 * allocates or frees device memory: outputs, saved route state and the scratch
 * "workspace" are owned by the caller (the Python host side uses PyTorch's
 * caching allocator). Work is stream-ordered; no entry point synchronises the
 * host. Each returns 0 on success or a negative tropnn_b200_status; the message
 * of the last failure on the calling thread is tropnn_b200_last_error().
 *
 * Reference interfaces replaced (paths inside the tropnn package):
 *   TropLinear route + hidden:   backends/tilelang_route.py:496-585 (_run_trop_forward),
 *                                layers/tropical.py:148-221 (_route_output, torch path)
 *   TropLinear min-face backward: backends/tilelang_route.py:619-677,
 *                                backends/triton_backward.py:357-515,
 *                                layers/tropical_exact.py:164-237
 *   PairwiseLinear forward:      backends/pairwise_tilelang.py:413-457 (_run_forward),
 *                                layers/pairwise.py:99-135
 *   PairwiseLinear STE backward: backends/pairwise_tilelang.py:482-534,
 *                                layers/pairwise.py:137-200
 */
#ifndef TROPNN_B200_H
#define TROPNN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TROPNN_B200_API __attribute__((visibility("default")))
#else
#define TROPNN_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tropnn_b200_status {
  TROPNN_B200_OK = 0,
  TROPNN_B200_ERR_INVALID = -1,   /* bad shape, size, pointer or flag (host raises ValueError) */
  TROPNN_B200_ERR_DTYPE = -2,     /* unsupported dtype (host raises TypeError) */
  TROPNN_B200_ERR_DEVICE = -3,    /* current device is not sm_100 (RuntimeError) */
  TROPNN_B200_ERR_LAUNCH = -4,    /* CUDA launch or runtime error (RuntimeError) */
  TROPNN_B200_ERR_WORKSPACE = -5, /* workspace too small (RuntimeError) */
  TROPNN_B200_ERR_TIMEOUT = -6    /* a bounded device-side wait gave up (RuntimeError) */
} tropnn_b200_status;

/* Element types of parameters and of outputs written in parameter precision. */
typedef enum tropnn_b200_dtype {
  TROPNN_B200_F32 = 0,
  TROPNN_B200_F16 = 1,
  TROPNN_B200_BF16 = 2,
  TROPNN_B200_U8 = 3,  /* packed route indices (cells <= 256) */
  TROPNN_B200_I16 = 4, /* packed route indices (cells <= 32767) */
  TROPNN_B200_I64 = 5  /* route indices otherwise */
} tropnn_b200_dtype;

/* STE surrogates of layers/surrogate.py:9-17. */
typedef enum tropnn_b200_surrogate {
  TROPNN_B200_SURROGATE_FAST_SIGMOID_ODD = 0,
  TROPNN_B200_SURROGATE_IZHIKEVICH = 1
} tropnn_b200_surrogate;

/* ------------------------------------------------------------------ misc */

/* Message of the last failing call on this host thread ("" if none). */
TROPNN_B200_API const char *tropnn_b200_last_error(void);
/* ABI revision; bumped whenever a signature below changes. */
TROPNN_B200_API int tropnn_b200_abi_version(void);
/* TROPNN_B200_OK when `device` is an sm_100 GPU, else TROPNN_B200_ERR_DEVICE. */
TROPNN_B200_API int tropnn_b200_check_device(int device);
/* Kernels this library has launched in this process so far (all devices and threads); a
 * launch recorded into a CUDA graph counts once, when it is recorded. No reference
 * counterpart: instrumentation. */
TROPNN_B200_API unsigned long long tropnn_b200_kernel_launches(void);

/* ------------------------------------------------------- shared machinery */

/*
 * Stable counting sort of rows by route bucket, one group (head or table) at a time.
 * keys[n * key_row_stride + g] (dtype U8/I16/I64) is the bucket of row n in group g.
 * Writes perm[g * rows + j] (row ids, grouped by bucket, ascending row order inside a
 * bucket) and seg[g * (buckets + 1) + b] (start of bucket b; seg[.. + buckets] = rows).
 * buckets <= 4096. This is the gather-side replacement of the scatter-add atomics in
 * backends/pairwise_tilelang.py:118-156 and backends/triton_backward.py:224-305.
 */
TROPNN_B200_API int tropnn_b200_bucket_sort(const void *keys, int key_dtype, int64_t rows, int64_t groups,
                            int64_t key_row_stride, int64_t buckets, int32_t *perm, int32_t *seg,
                            void *stream);

/*
 * Segmented weighted row sum: for every group g, bucket b and column j < width
 *   out[(g*buckets + b)*width + j] = scale * ( sum_{n in list0(g,b)} c0(n,g) * values[n*ld + j]
 *                                            + sum_{n in list1(g,b)} c1(n,g) * values[n*ld + j] )
 * where list_i(g,b) = perm_i[g*rows + seg_i[g*(buckets+1)+b] ..< seg_i[..+b+1]] and
 * c_i(n,g) = coef_sign_i * coef_i[n*groups + g] (or coef_sign_i when coef_i is NULL).
 * perm1/seg1 may be NULL (one list). Every element of `out` is written exactly once
 * (buckets without rows get 0), in out_dtype (F32/F16/BF16). If bucket_sum is not
 * NULL it receives scale * sum of the coefficients per (g, b) in out_dtype.
 * Deterministic: the summation order is fixed by (perm, seg).
 */
TROPNN_B200_API int tropnn_b200_segment_rowsum(const float *values, int64_t rows, int64_t width, int64_t ld,
                               int64_t groups, int64_t buckets,
                               const int32_t *perm0, const int32_t *seg0, const float *coef0, float coef_sign0,
                               const int32_t *perm1, const int32_t *seg1, const float *coef1, float coef_sign1,
                               float scale, void *out, int out_dtype, void *bucket_sum, void *stream);

/*
 * tropnn_b200_segment_rowsum over half-precision values, one list, no coefficients:
 * out[g*buckets + b, :] = scale / s * sum_{j in seg} values[perm[g*rows + j] * ld, :width], with
 * values = x * s rounded to value_dtype (F16/BF16) and s the power-of-two gradient scale of
 * *grad_absmax (tropnn_b200_split_half with the same word; NULL: s = 1). width and ld multiples
 * of 8, values 16-byte aligned. Half the bytes per gathered row of the f32 form: the LUT
 * gradient of half-precision PairwiseLinear layers (rounded to that dtype in any case). The
 * rounding of x to value_dtype adds at most one half-precision unit of relative error per
 * summand. Deterministic.
 */
TROPNN_B200_API int tropnn_b200_segment_rowsum_half(const void *values, int value_dtype, int64_t rows,
                                                    int64_t width, int64_t ld, int64_t groups, int64_t buckets,
                                                    const int32_t *perm, const int32_t *seg, float scale,
                                                    const void *grad_absmax, void *out, int out_dtype,
                                                    void *stream);

/* --------------------------------------------------------- PairwiseLinear */

/*
 * LUT gradient in one kernel (the scatter of layers/pairwise.py:99-122's gather; atomics in
 * backends/pairwise_tilelang.py:118-156):
 *   grad_lut[t, b, :] = sum over rows n with indices[n, t] == b, in ascending n, of
 *                       scale * grad_out[n, :]
 * indices int64 [items, tables] (the forward's), grad_out f32 [items, out_features], grad_lut
 * [tables, 2^comparisons, out_features] in lut_dtype, every entry written once. One CTA per
 * (table, 64 columns) sorts the table's rows by bucket in shared memory and sums each bucket's
 * rows in registers: deterministic, the same order as bucket_sort + segment_rowsum.
 * comparisons <= 8 (the bucket_sort + segment_rowsum pair covers the rest; it is also the faster
 * path above ~1024 columns, where this kernel's per-column-block sorts repeat).
 */
TROPNN_B200_API int tropnn_b200_pairwise_lut_grad(const float *grad_out, int64_t items, int64_t out_features,
                                  const int64_t *indices, int64_t tables, int64_t comparisons, float scale,
                                  void *grad_lut, int lut_dtype, void *stream);

/*
 * tropnn_b200_pairwise_lut_grad with the data-parallel gradient all-reduce fused in (one process
 * per GPU, the peer buffers of tropnn_b200_peer_buffer_create / _open as for
 * tropnn_b200_peer_allreduce_f32, a set used for nothing else): every CTA pushes its block of
 * local sums into every rank's buffer over NVLink as soon as it is computed, meets the other
 * ranks at a per-block flag barrier and writes the rank-order sum (times 1/world when averaging),
 * so the reduction overlaps the other blocks' work. Every rank must make the same calls.
 * tables x ceil(out_features / 64) <= 512 blocks; capacity_floats >=
 * tropnn_b200_pairwise_lut_grad_peer_floats(...) (-1 for unsupported shapes). world = 1 is the
 * plain kernel.
 */
TROPNN_B200_API int64_t tropnn_b200_pairwise_lut_grad_peer_floats(int64_t tables, int64_t comparisons,
                                                                  int64_t out_features);
TROPNN_B200_API int tropnn_b200_pairwise_lut_grad_allreduce(const float *grad_out, int64_t items, int64_t out_features,
                                            const int64_t *indices, int64_t tables, int64_t comparisons,
                                            float scale, void *grad_lut, int lut_dtype, void *const *buffers,
                                            int world, int rank, int64_t capacity_floats, int average,
                                            void *stream);

/*
 * Fused comparator routing + LUT gather-sum (layers/pairwise.py:99-135, base.py:76-77).
 *   u[n,t,r]   = (latent[n,a] - latent[n,b]) - thresholds[t,r],  (a,b) = anchors[t,r,:]
 *   idx[n,t]   = sum_r [u[n,t,r] > 0] << r
 *   out[n,o]   = output_scale * sum_t lut[t, idx[n,t], o]
 * latent f32 [items, in_features]; anchors int64 [tables, comparisons, 2];
 * thresholds [tables, comparisons] and lut [tables, 2^comparisons, out_features] in
 * their own dtypes (F32/F16/BF16). Outputs: out f32 [items, out_features],
 * indices int64 [items, tables], margins f32 [items, tables, comparisons].
 * comparisons <= 12.
 */
TROPNN_B200_API int tropnn_b200_pairwise_forward(const float *latent, int64_t items, int64_t in_features,
                                 const int64_t *anchors, const void *thresholds, int thresholds_dtype,
                                 int64_t tables, int64_t comparisons,
                                 const void *lut, int lut_dtype, int64_t out_features, float output_scale,
                                 float *out, int64_t *indices, float *margins, void *stream);

/*
 * Inverse anchor map used by the STE backward to gather grad_latent without atomics:
 * entries of anchors (flattened, e = (t*comparisons + r)*2 + side) grouped by input
 * feature. feat_start [in_features + 1] int32, feat_entries [tables*comparisons*2] int32.
 * Depends only on the anchors buffer; callers cache it.
 */
TROPNN_B200_API int tropnn_b200_pairwise_anchor_index(const int64_t *anchors, int64_t tables, int64_t comparisons,
                                      int64_t in_features, int32_t *feat_start, int32_t *feat_entries,
                                      void *stream);

/*
 * STE backward rows (layers/pairwise.py:137-200 and their autograd; the surrogate of
 * layers/surrogate.py:9-17): with g = output_scale * grad_out,
 *   min mode:  r* = argmin_r |u[n,t,r]| (first on ties), nb = idx ^ (1<<r*),
 *              gu[n,t] = (sum_o g[n,o] (lut[t,nb,o] - lut[t,idx,o])) * S(u[n,t,r*])
 *   full mode: the same for every r, gu[n,t,r].
 *   grad_latent[n,i] = sum over anchor entries of feature i of +gu (side 0) / -gu (side 1).
 * Writes grad_latent f32 [items, in_features], gu f32 ([items, tables] or
 * [items, tables, comparisons]) and rstar u8 [items, tables] (min mode only).
 */
TROPNN_B200_API int tropnn_b200_pairwise_ste_backward(const float *grad_out, int64_t items, int64_t out_features,
                                      float output_scale, const int64_t *indices, const float *margins,
                                      const int64_t *anchors, int64_t tables, int64_t comparisons,
                                      int64_t in_features, const void *lut, int lut_dtype,
                                      int use_min_margin_ste, int surrogate,
                                      const int32_t *feat_start, const int32_t *feat_entries,
                                      float *grad_latent, float *gu, uint8_t *rstar, void *stream);

/* Bytes of scratch tropnn_b200_pairwise_threshold_grad needs: 0 (the stages meet in shared memory);
 * the query and the workspace arguments stay so that callers need not change. */
TROPNN_B200_API size_t tropnn_b200_pairwise_threshold_grad_workspace_size(int64_t items, int64_t tables,
                                                                          int64_t comparisons);

/*
 * grad_thresholds[t,r] = -sum_n gu (min mode: rows whose r* == r), written in
 * grad_dtype. One launch of 8-CTA clusters: row-slice partial sums combined in a fixed order
 * through distributed shared memory (deterministic). `workspace` may be NULL.
 */
TROPNN_B200_API int tropnn_b200_pairwise_threshold_grad(const float *gu, const uint8_t *rstar, int64_t items,
                                        int64_t tables, int64_t comparisons, int use_min_margin_ste,
                                        void *grad_thresholds, int grad_dtype, void *workspace,
                                        size_t workspace_bytes, void *stream);

/* Bytes of scratch tropnn_b200_pairwise_backward needs. */
TROPNN_B200_API size_t tropnn_b200_pairwise_backward_workspace_size(int64_t items, int64_t tables, int64_t comparisons,
                                                    int64_t in_features, int use_min_margin_ste);

/*
 * Whole PairwiseLinear backward (the autograd backward of pairwise.py:202-248):
 * grad_lut (lut dtype, may be NULL), grad_latent (f32, NULL to skip the STE part) and
 * grad_thresholds (grad_thresholds_dtype, may be NULL). Runs pairwise_lut_grad (up to 8
 * comparisons and 1024 columns; else bucket_sort + segment_rowsum) for the LUT and
 * anchor_index + ste_backward + threshold_grad for the STE terms, all inside `workspace`.
 */
TROPNN_B200_API int tropnn_b200_pairwise_backward(const float *grad_out, int64_t items, int64_t out_features,
                                  float output_scale, const int64_t *indices, const float *margins,
                                  const int64_t *anchors, int64_t tables, int64_t comparisons,
                                  int64_t in_features, const void *lut, int lut_dtype,
                                  int use_min_margin_ste, int surrogate,
                                  float *grad_latent, void *grad_thresholds, int grad_thresholds_dtype,
                                  void *grad_lut, void *workspace, size_t workspace_bytes, void *stream);

/* Size of the fixed scratch buffer behind tropnn_b200_pairwise_backward_noalloc. */
#define TROPNN_B200_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/*
 * tropnn_b200_pairwise_backward without a workspace argument, for callers that cannot
 * allocate device memory (a host with a fixed, fully pre-partitioned memory budget, a
 * foreign-language caller without a CUDA allocator, a loop that must not pay
 * cudaMalloc's implicit synchronisation). No counterpart in the reference: its torch and
 * TileLang paths always allocate their temporaries.
 *
 * Scratch comes from one TROPNN_B200_NOALLOC_SCRATCH_BYTES (8 MiB) device buffer compiled
 * into the library; problems whose tropnn_b200_pairwise_backward_workspace_size() is
 * larger are rejected with TROPNN_B200_ERR_INVALID. The buffer is shared by every call on
 * a GPU: calls that can overlap on that GPU (different streams, threads or processes
 * sharing the context) race on it and must be serialised by the caller. The first call
 * on each device (and again after that device's context was destroyed and recreated)
 * looks up the buffer's device address (cudaGetSymbolAddress) and caches it with the
 * context's id; make that first call before any stream capture. The 8 MiB are reserved on
 * a GPU when the library's module loads there (on first use of its kernels with lazy
 * module loading, the default; at context creation on every device with
 * CUDA_MODULE_LOADING=EAGER), whether or not this entry point is called, and are held
 * until the process exits. Invalid sizes are rejected with TROPNN_B200_ERR_INVALID before
 * the size check. Arguments and results as tropnn_b200_pairwise_backward.
 */
TROPNN_B200_API int tropnn_b200_pairwise_backward_noalloc(const float *grad_out, int64_t items, int64_t out_features,
                                          float output_scale, const int64_t *indices, const float *margins,
                                          const int64_t *anchors, int64_t tables, int64_t comparisons,
                                          int64_t in_features, const void *lut, int lut_dtype,
                                          int use_min_margin_ste, int surrogate,
                                          float *grad_latent, void *grad_thresholds, int grad_thresholds_dtype,
                                          void *grad_lut, void *stream);

/* ------------------------------------------------------------ TropLinear */

/*
 * Route scores, top-2 and margins (backend.py:45-46, routing.py:7-10):
 *   s[n,h,k] = <latent[n,:], router_weight[h,k,:]> + router_bias[h,k]
 *   winner/runner = top-2 cells (lowest index on exact ties), margin = s_w - s_r.
 * latent [items, code_dim] in latent_dtype: F32 (fp32 FMA path, parameters upcast) or
 * the parameter dtype. With F16/BF16 latent and parameters, cells in {2,4,8,16,32},
 * code_dim % 8 == 0 and <= 384, U8 routes and >= 128 rows and score columns, the scores
 * run on the tensor cores (tcgen05, TMEM accumulators, TMA) and only the routes leave
 * the chip; that path needs router_bias in F32 (bias_dtype), which spares its epilogue
 * every conversion. router_weight [heads, cells, code_dim] in param_dtype; router_bias
 * [heads, cells] in bias_dtype (F32 or param_dtype). winner_i64 (int64 [items, heads])
 * may be NULL; winner in index_dtype (U8/I16/I64, the packing of routing.py:18-31);
 * runner (index_dtype) and margins (f32 [items, heads]) may be NULL when not needed.
 * F32 latent, parameters and bias with U8 routes, cells in {2,4,8,16,32}, code_dim a
 * multiple of 4 up to 128 and a `workspace` of tropnn_b200_trop_route_workspace_size() bytes:
 * the scores run on the tensor cores as well, in kind::tf32 with every operand split into two
 * tf32 parts (3xTF32, ~2^-22 relative per product; the split operands go to the workspace).
 * With a NULL or smaller workspace, or fewer than 64 items, those shapes take the fp32 FMA
 * path.
 */
TROPNN_B200_API size_t tropnn_b200_trop_route_workspace_size(int64_t items, int64_t code_dim, int64_t heads,
                                                             int64_t cells, int latent_dtype, int param_dtype);
TROPNN_B200_API int tropnn_b200_trop_route(const void *latent, int latent_dtype, int64_t items, int64_t code_dim,
                           const void *router_weight, const void *router_bias, int bias_dtype, int param_dtype,
                           int64_t heads, int64_t cells,
                           int64_t *winner_i64, void *winner, void *runner, int index_dtype,
                           float *margins, void *workspace,
                           size_t workspace_bytes, void *stream);

/*
 * Input projection z = P(x) (layers/tropical.py:96-99, `proj(x.to(P.dtype))`) for half-precision
 * projection weights: z[n, :] = half(sum_i half(x[n, i]) * P[:, i]) with f32 accumulation,
 * z [items, code_dim] in param_dtype. x f32 [items, in_features] (in_features a multiple of 8),
 * P [code_dim, in_features] in param_dtype (F16/BF16), code_dim in {64, 128, 192, 256}. One
 * tcgen05 GEMM that rounds x to the parameter dtype on chip (no separate cast pass over x).
 * With few row blocks the contraction is split across SMs into slices whose f32 partials go
 * to `workspace` (tropnn_b200_trop_proj_workspace_size bytes; 0 when unsplit) and are summed
 * in slice order (deterministic).
 */
TROPNN_B200_API size_t tropnn_b200_trop_proj_workspace_size(int64_t items, int64_t in_features, int64_t code_dim);
/*
 * Weight gradient of that projection (the reference's half-precision F.linear backward):
 * grad_weight[d, i] = sum_n grad_z[n, d] * half(x[n, i]) for f32 x [items, in_features] and
 * grad_z_t = grad_z transposed to [code_dim, items] in param_dtype (tropnn_b200_transpose_to_half);
 * grad_weight [code_dim, in_features] in param_dtype. f32 accumulation on the tensor cores, x
 * rounded on chip (read once, no cast pass), one rounding of the result; the sample range is cut
 * into slices whose f32 partials go to `workspace` (tropnn_b200_trop_proj_wgrad_workspace_size
 * bytes) and are summed in slice order (deterministic). items and in_features multiples of 8,
 * code_dim in {64, 128, 192, 256}.
 */
TROPNN_B200_API size_t tropnn_b200_trop_proj_wgrad_workspace_size(int64_t items, int64_t in_features,
                                                                  int64_t code_dim);
TROPNN_B200_API int tropnn_b200_trop_proj_wgrad(const float *x, int64_t items, int64_t in_features,
                                                const void *grad_z_t, int param_dtype, int64_t code_dim,
                                                void *grad_weight, void *workspace, size_t workspace_bytes,
                                                void *stream);
TROPNN_B200_API int tropnn_b200_trop_proj(const float *x, int64_t items, int64_t in_features,
                                          const void *proj_weight, int param_dtype, int64_t code_dim, void *z,
                                          void *workspace, size_t workspace_bytes, void *stream);

/*
 * f32 matrix product on the tensor cores, for TropLinear's f32 parameters (the projection
 * tropical.py:96-99 and output map :140-146 with their backward products, and the exact eval
 * path's effective weights and base output, tropical_exact.py:257-358, all f32 GEMMs in the
 * reference): c[i, j] = sum_{l<k} a[i*lda + l] * b[j*ldb + l] (+ bias[j]) for i < m, j < n,
 * written to c[i*ldc + j]. lda and ldb multiples of 4, a and b 16-byte aligned; bias may be
 * NULL. Each operand is split into two tf32 parts and three tcgen05 kind::tf32 products are
 * summed (3xTF32: f32 range, ~2^-22 relative per product). With few 128 x 128 output tiles the
 * contraction is split across SMs; the slices' f32 partials go to `workspace`
 * (tropnn_b200_gemm_tf32x3_workspace_size bytes; 0 when unsplit) and are summed in slice order.
 * Products of at most 32 rows (m <= 32) run as f32 FMA instead (one warp per column of c, no
 * workspace): below one 128-row MMA tile the tensor-core pipeline costs more than the math.
 */
TROPNN_B200_API size_t tropnn_b200_gemm_tf32x3_workspace_size(int64_t m, int64_t n, int64_t k);
TROPNN_B200_API int tropnn_b200_gemm_tf32x3(const float *a, int64_t lda, const float *b, int64_t ldb, int64_t m,
                                            int64_t n, int64_t k, const float *bias, float *c, int64_t ldc,
                                            void *workspace, size_t workspace_bytes, void *stream);
/* out[j*ldo + i] = x[i*ldx + j] for i < rows, j < cols; out[j*ldo + i] = 0 for rows <= i < ldo.
 * A layout step of the f32 products above (no reference counterpart). */
TROPNN_B200_API int tropnn_b200_transpose_f32(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out,
                                              int64_t ldo, void *stream);
/* out[j] = sum_i x[i*ldx + j] in row order (the output-map bias gradient of the f32 path). */
TROPNN_B200_API int tropnn_b200_colsum_f32(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *out,
                                           void *stream);

/*
 * hidden[n,:] = latent[n,:] + code_scale * sum_h chat[n,h,:] with chat = code[h,w] (eval)
 * or code[h,w] + U(m) (code[h,r] - code[h,w]), U(m) = 0.5/(1+|m|) (training)
 * (layers/tropical.py:131-138, routing.py:13-15). code in param_dtype; latent in
 * latent_dtype (F32 or the parameter dtype); hidden f32 [items, code_dim].
 * code_t (may be NULL): code transposed to [code_dim, heads*cells] by
 * tropnn_b200_trop_code_transpose. With it, F16/BF16 codes, U8 routes, cells in
 * {2,4,8,16,32}, code_dim in {64,128,192,256}, heads*cells % 8 == 0 and >= 128 items,
 * the sum runs as a one-hot GEMM on the tensor cores (tcgen05); in training the two
 * mixing weights are then rounded to the parameter dtype. Otherwise a per-row gather.
 * With fewer 128-row blocks than the SMs can take, the tensor-core path splits the
 * (head, cell) contraction into slices when `workspace` holds
 * tropnn_b200_trop_hidden_workspace_size() bytes (their f32 partials, summed in slice order);
 * with a NULL or smaller workspace it runs unsplit. Same for tropnn_b200_trop_router_term.
 * hidden_split (may be NULL; F16/BF16 codes, code_dim % 4 == 0, 16-byte aligned): also
 * written as [items, 2*code_dim] in param_dtype, the [hi | lo] split of each hidden row
 * (tropnn_b200_split_half with a NULL scale) that tropnn_b200_linear_f32out takes for the
 * output map; the tensor-core path forms it in the same epilogue as hidden.
 */
TROPNN_B200_API size_t tropnn_b200_trop_hidden_workspace_size(int64_t items, int64_t code_dim, int64_t heads,
                                                              int64_t cells);
TROPNN_B200_API int tropnn_b200_trop_hidden(const void *latent, int latent_dtype, int64_t items, int64_t code_dim,
                            const void *code, const void *code_t, int param_dtype, int64_t heads, int64_t cells,
                            const void *winner, const void *runner, int index_dtype,
                            const float *margins, float code_scale, int training,
                            float *hidden, void *hidden_split, void *workspace, size_t workspace_bytes,
                            void *stream);

/*
 * code_t[d, h*cells + k] = code[h, k, d]: the K-major right operand of the tensor-core
 * code sum (F16/BF16 only). No reference counterpart: a layout step of this backend.
 */
TROPNN_B200_API int tropnn_b200_trop_code_transpose(const void *code, int param_dtype, int64_t heads, int64_t cells,
                                    int64_t code_dim, void *code_t, void *stream);

/*
 * out[rows, 2*cols] = [hi | lo] per row of the f32 matrix x [rows, cols] times s: hi = x s
 * rounded to dtype (F16/BF16), lo = (x s - hi) rounded to dtype; hi + lo carries x s to
 * ~2^-22 relative (f16). s = 1 when grad_absmax is NULL, else the power-of-two gradient scale
 * of the tensor maximum in *grad_absmax (tropnn_b200_absmax_f32). cols % 4 == 0. Left operand
 * of tropnn_b200_linear_f32out for an f32 input. No reference counterpart: a precision-
 * splitting step of this backend.
 */
TROPNN_B200_API int tropnn_b200_split_half(const float *x, int64_t rows, int64_t cols, int dtype,
                           const void *grad_absmax, void *out, void *stream);

/*
 * tropnn_b200_split_half and its transpose in one pass over x: out_split [rows, 2*cols] as
 * tropnn_b200_split_half writes it, and out_t [cols, rows] = its hi half transposed, equal
 * to tropnn_b200_transpose_to_half of x with the same grad_absmax. rows even, cols % 4 == 0;
 * x 16-byte, out_split 8-byte, out_t 4-byte aligned. The half-precision backward uses it on
 * grad_hidden, whose split feeds tropnn_b200_trop_gm and whose transpose feeds the code
 * gradient. No reference counterpart: a precision-splitting step of this backend.
 */
TROPNN_B200_API int tropnn_b200_split_transpose_half(const float *x, int64_t rows, int64_t cols, int dtype,
                                                     const void *grad_absmax, void *out_split, void *out_t,
                                                     void *stream);

/*
 * Gradient range for the half-precision backward GEMMs: *bits = max(*bits, f32 bits of
 * max_i |x[i]|) (the caller zeroes the 4-byte word first; deterministic). The kernels that take
 * a grad_absmax pointer scale the gradient by s = 2^e bringing that maximum into [16, 32)
 * before rounding it to f16/bf16 and divide their f32 results by s (exact), so gradients far
 * below f16's normal range (6.1e-5) keep their relative precision instead of underflowing; the
 * reference computes these products in f32. x 16-byte aligned.
 */
TROPNN_B200_API int tropnn_b200_absmax_f32(const float *x, int64_t n, void *bits, void *stream);

/*
 * out[n, o] = sum_s sum_k a[n, s*in + k] * weight[o, k] + bias[o] (f32 accumulation on the
 * tensor cores, f32 out [rows, out_features]); a [rows, slices*in] and weight
 * [out_features, in] in dtype (F16/BF16), bias f32 [out_features] or NULL. slices = 2
 * with a from tropnn_b200_split_half is the f32-input linear map of the output projection
 * (layers/tropical.py:140-146: F.linear on the f32 hidden with the weight upcast).
 * in % 64 == 0, slices * in <= 512, out_features % 4 == 0, 16-byte aligned operands.
 */
TROPNN_B200_API int tropnn_b200_linear_f32out(const void *a, int64_t rows, int64_t slices, const void *weight,
                              int64_t out_features, int64_t in_features, int dtype, const float *bias,
                              float *out, void *stream);

/* ------------------------------------------------------------------ multi-GPU */

#define TROPNN_B200_PEER_MAX_RANKS 8
#define TROPNN_B200_PEER_MAX_SEGMENTS 8
#define TROPNN_B200_PEER_HANDLE_BYTES 64

/*
 * Peer buffers for tropnn_b200_peer_allreduce_f32: one per rank (one process per GPU on one
 * node). _create allocates this rank's buffer (cudaMalloc; capacity_floats a multiple of
 * 64) and writes its CUDA IPC handle (TROPNN_B200_PEER_HANDLE_BYTES bytes) to `handle`;
 * the ranks exchange handles, and _open maps another rank's buffer into this process.
 * _close unmaps a peer's buffer, _destroy frees this rank's. These four are the setup of
 * the batch-sharded data parallelism (no reference counterpart: the reference is
 * single-device) and the only entry points that allocate.
 */
TROPNN_B200_API int tropnn_b200_peer_buffer_create(int64_t capacity_floats, void **local, unsigned char *handle);
TROPNN_B200_API int tropnn_b200_peer_buffer_open(const unsigned char *handle, void **peer);
TROPNN_B200_API int tropnn_b200_peer_buffer_close(void *peer);
TROPNN_B200_API int tropnn_b200_peer_buffer_destroy(void *local);

/*
 * In-place sum (average when `average`) of the f32 tensors `segments[s]` (counts[s]
 * floats each, nseg <= TROPNN_B200_PEER_MAX_SEGMENTS, total <= capacity_floats) across
 * `world` ranks over NVLink peer memory: buffers[p] is rank p's peer buffer as mapped in
 * this process (this rank's own at index `rank`). Every rank must make the same calls in
 * the same order. One kernel. Two ranks: each rank stores its tensors into every rank's
 * buffer over NVLink, one flag barrier, then each rank sums the copies from its own memory in
 * rank order. More ranks (two-shot): each rank stores chunk q of its tensors into rank q's
 * buffer, flag barrier, rank q sums chunk q in rank order and stores the result into every
 * rank's buffer, flag barrier, each rank copies the reduced chunks out (2 (W-1)/W of the
 * data sent per rank instead of W-1 copies). Bit-identical results on all ranks; the
 * two-shot and one-shot sums differ only in which rank adds. A rank that does not arrive within 2 s
 * makes the others return with the device error word set (tropnn_b200_device_error).
 * Each peer buffer holds 2 x 8 receive areas of capacity_floats (double-buffered).
 */
TROPNN_B200_API int tropnn_b200_peer_allreduce_f32(void *const *buffers, int world, int rank, int64_t capacity_floats,
                                   float *const *segments, const int64_t *counts, int nseg, int average,
                                   void *stream);

/*
 * Reads and clears the library's device error words: 1 after a tensor-core kernel gave up
 * a bounded wait (its CTA then released its resources and exited). Synchronises with the
 * device; call it off the hot path.
 */
TROPNN_B200_API int tropnn_b200_device_error(int *value);

/*
 * Tensor-core min-face backward for half-precision parameters (layers/tropical_exact.py:
 * 204-237), four GEMMs whose left operand is the (weighted) one-hot route matrix or whose
 * epilogue reads the routes; U8 routes, cells in {2,4,8,16,32}, code_dim in {64,...,256}
 * (a multiple of 64), items a multiple of 8 and >= 128.
 *
 * grad_absmax (every call below; NULL: unscaled) is the word of tropnn_b200_absmax_f32 over
 * grad_hidden: g_split / x_t of grad_hidden and the gm weights are scaled by its power-of-two
 * gradient scale before their rounding to the parameter dtype, and every result (gm included)
 * is scaled back, so tiny gradients keep their precision with f16 parameters.
 * trop_gm: gm[n,h] = code_scale (<g_n, code[h,r]> - <g_n, code[h,w]>) U'(m_nh),
 *   U'(m) = -0.5 sign(m) / (1+|m|)^2, from g_split = [hi | lo] halves of grad_hidden
 *   (tropnn_b200_split_half with the same grad_absmax, [items, 2*code_dim]) against code
 *   ([heads*cells, code_dim]).
 * trop_router_term: grad_latent = grad_hidden + sum_h gm[n,h] (W[h,w] - W[h,r]), with
 *   router_weight_t = router_weight transposed ([code_dim, heads*cells],
 *   tropnn_b200_trop_code_transpose); gm rounded to the parameter dtype in the product.
 * trop_param_grad: grad[h,k,:] = out_scale sum_n (vw [w==k] + vr [r==k]) x[n,:] with x_t =
 *   x transposed to the parameter dtype ([code_dim, items], tropnn_b200_transpose_to_half):
 *   mode 0 (code grad, eval): vw = 1, vr = 0, out_scale = code_scale, x = grad_hidden;
 *   mode 1 (code grad, training): vw = 1-U(m), vr = U(m) (values = margins), out_scale =
 *   code_scale, x = grad_hidden; mode 2 (router grad): vw = gm, vr = -gm (values = gm),
 *   out_scale = 1, x = latent, and grad_bias[h,k] = sum_n gm ([w==k] - [r==k]) when not NULL.
 *   grad / grad_bias in the parameter dtype; x_t's rounding of grad_hidden is within the 2e-2
 *   half-precision tolerance.
 * transpose_to_half: out[c, r] = x[r, c] s rounded to dtype; x in x_dtype (F32 or dtype), s the
 *   gradient scale of grad_absmax (1 when NULL).
 * No reference counterparts as entry points: they restate the reference's backward as GEMMs.
 */
TROPNN_B200_API int tropnn_b200_trop_gm(const void *g_split, int64_t items, int64_t code_dim, const void *code,
                        int param_dtype, int64_t heads, int64_t cells, const void *winner, const void *runner,
                        const float *margins, float code_scale, float *gm, const void *grad_absmax,
                        void *stream);
TROPNN_B200_API int tropnn_b200_trop_router_term(const float *grad_hidden, int64_t items, int64_t code_dim,
                                 const void *router_weight_t, int param_dtype, int64_t heads, int64_t cells,
                                 const void *winner, const void *runner, const float *gm,
                                 const void *grad_absmax, float *grad_latent, void *workspace,
                                 size_t workspace_bytes, void *stream);
TROPNN_B200_API int tropnn_b200_trop_param_grad(int mode, const void *x_t, int64_t items, int64_t code_dim,
                                int param_dtype, int64_t heads, int64_t cells, const void *winner,
                                const void *runner, const float *values, float code_scale, void *grad,
                                void *grad_bias, const void *grad_absmax, void *stream);
TROPNN_B200_API int tropnn_b200_transpose_to_half(const void *x, int x_dtype, int64_t rows, int64_t cols, int dtype,
                                  const void *grad_absmax, void *out, void *stream);

/*
 * Gradients of the f32 output map out = hidden weight^T + bias (layers/tropical.py:140-146,
 * whose F.linear runs in f32 with the half-precision weight upcast) on the tcgen05 tensor
 * cores in tf32 with split operands (x = big + small, three products), which keeps f32
 * accuracy and range. g = grad_out, f32 [rows, out_features]; out_features a multiple of 32;
 * in_features a multiple of 32 in [32, 256].
 * linear_dgrad: grad_hidden[n,i] = sum_o g[n,o] weight32[o,i]; weight32 = the weight widened
 *   to f32 ([out_features, in_features]); grad_hidden f32 [rows, in_features]. With few
 *   128-row blocks the out_features contraction is split across SMs when `workspace` holds
 *   tropnn_b200_linear_dgrad_workspace_size() bytes (slice partials summed in slice order);
 *   NULL runs it unsplit.
 * linear_wgrad: grad_weight[o,i] = sum_n g[n,o] hidden[n,i] rounded to dtype (F16/BF16), and
 *   grad_bias[o] = sum_n g[n,o] in f32 when not NULL; hidden given as its tf32 split
 *   (tropnn_b200_tf32_split). The row range is contracted by a 4-CTA cluster per 128 output
 *   features and the partials summed in a fixed order (deterministic).
 * tf32_split: x = big + small elementwise with big = tf32(x), small = tf32(x - big); count a
 *   multiple of 4, 16-byte aligned pointers.
 */
TROPNN_B200_API size_t tropnn_b200_linear_dgrad_workspace_size(int64_t rows, int64_t out_features,
                                                               int64_t in_features);
TROPNN_B200_API int tropnn_b200_linear_dgrad(const float *g, int64_t rows, int64_t out_features, const float *weight32,
                             int64_t in_features, float *grad_hidden, void *workspace, size_t workspace_bytes,
                             void *stream);
TROPNN_B200_API int tropnn_b200_linear_wgrad(const float *g, int64_t rows, int64_t out_features, const float *hidden_big,
                             const float *hidden_small, int64_t in_features, int dtype, void *grad_weight,
                             float *grad_bias, void *stream);
TROPNN_B200_API int tropnn_b200_tf32_split(const float *x, int64_t count, float *big, float *small, void *stream);

/*
 * Per-row part of the min-face backward (layers/tropical_exact.py:204-237):
 *   training: gm[n,h] = code_scale * U'(m) * sum_d g[n,d] (code[h,r,d] - code[h,w,d]),
 *             U'(m) = -0.5 sign(m) / (1+|m|)^2
 *             grad_latent[n,:] = g[n,:] + sum_h gm[n,h] (W[h,w,:] - W[h,r,:])
 *             coef_w = code_scale (1 - U(m)), coef_r = code_scale U(m)
 *   eval:     grad_latent = g, coef_w = code_scale (gm, coef_r untouched).
 * All per-row outputs f32: grad_latent [items, code_dim], coef_w/coef_r/gm [items, heads].
 */
TROPNN_B200_API int tropnn_b200_trop_backward_rows(const float *grad_hidden, int64_t items, int64_t code_dim,
                                   const void *router_weight, const void *code, int param_dtype,
                                   int64_t heads, int64_t cells,
                                   const void *winner, const void *runner, int index_dtype,
                                   const float *margins, float code_scale, int training,
                                   float *grad_latent, float *coef_w, float *coef_r, float *gm,
                                   void *stream);

/*
 * Parameter gradients of an f32 TropLinear from its rows, without sorting (the batch sums of
 * tropical_exact.py:204-237):
 *   grad_code[h,k,:]   = sum_n coef_w[n,h] [w=k] g[n,:] + coef_r[n,h] [r=k] g[n,:]
 *   grad_router[h,k,:] = sum_n gm[n,h] ([w=k] - [r=k]) z[n,:],  grad_bias[h,k] likewise
 * with coef_w / coef_r / gm from tropnn_b200_trop_backward_rows (coef_w NULL: the constant
 * coef_const; coef_r / runner NULL: no runner-up term, as in eval). F32 parameters, U8
 * routes, 2-32 cells; any output NULL is skipped (the router weight and bias go together).
 * Deterministic (eight row groups summed in group order). tropnn_b200_trop_backward takes this
 * path itself for such layers. No reference counterpart beyond the batch sums it computes.
 */
TROPNN_B200_API int tropnn_b200_trop_param_grad_rows(const float *grad_hidden, const float *latent, int64_t items,
                                     int64_t code_dim, int param_dtype, int64_t heads, int64_t cells,
                                     const void *winner, const void *runner, int index_dtype,
                                     const float *coef_w, const float *coef_r, float coef_const,
                                     const float *gm, void *grad_code, void *grad_router_weight,
                                     void *grad_router_bias, void *stream);

/* Bytes of scratch tropnn_b200_trop_backward needs. */
TROPNN_B200_API size_t tropnn_b200_trop_backward_workspace_size(int64_t items, int64_t heads, int64_t cells, int training);

/*
 * Whole TropLinear route backward (the autograd backward of tropical.py:207-221):
 * grad_latent f32 [items, code_dim]; grad_code [heads, cells, code_dim] and, in
 * training, grad_router_weight / grad_router_bias, all in param_dtype (NULL skips).
 * Runs backward_rows, two bucket sorts and two segment_rowsum passes in `workspace`.
 */
TROPNN_B200_API int tropnn_b200_trop_backward(const float *grad_hidden, const float *latent, int64_t items, int64_t code_dim,
                              const void *router_weight, const void *code, int param_dtype,
                              int64_t heads, int64_t cells,
                              const void *winner, const void *runner, int index_dtype,
                              const float *margins, float code_scale, int training,
                              float *grad_latent, void *grad_router_weight, void *grad_router_bias,
                              void *grad_code, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TROPNN_B200_H */
