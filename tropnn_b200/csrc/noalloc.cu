// Allocation-free variant of the PairwiseLinear backward.
//
// Some callers of this library cannot allocate device memory at all: a host process
// that has already handed all free HBM to its own pool and runs with a fixed budget,
// a foreign-language caller (Go, Java, Rust through the C ABI) that links no CUDA
// allocator of its own, or a latency-critical loop where cudaMalloc's implicit device
// synchronisation would stall other work. tropnn_b200_pairwise_backward needs a
// caller-provided workspace; this entry point instead carves that workspace out of a
// fixed-size buffer compiled into the library, so it calls no cudaMalloc, cudaFree or
// any other allocating routine.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace tropnn_b200 {

int pairwise_backward_impl(const float *g, int64_t items, int64_t out, float out_scale, const int64_t *idx,
                           const float *u, const int64_t *anchors, int64_t tables, int64_t comparisons, int64_t in,
                           const void *lut, int lut_dtype, int use_min, int surrogate, float *gx, void *gthr,
                           int gthr_dtype, void *glut, void *ws, size_t ws_bytes, cudaStream_t stream);
size_t pairwise_backward_workspace(int64_t items, int64_t tables, int64_t comparisons, int64_t in, int use_min);

namespace {

constexpr size_t kScratchBytes = TROPNN_B200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The fixed scratch buffer. Part of the library's device image: it is reserved on a GPU
// when this module loads there (on the first use of the library's kernels with lazy
// module loading, the default; at context creation on every device with
// CUDA_MODULE_LOADING=EAGER) and held until the process exits. In host code `g_noalloc_scratch`
// is only a host-side stand-in for the symbol, never a device address; its device
// address is looked up per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mutex;

// One cached lookup per device: the buffer's address and the id of the context it was
// looked up in. A context that is destroyed and created again (cudaDeviceReset, or a
// caller that manages its own contexts) reloads the library's module, which may place the
// buffer elsewhere, so a lookup is only reused while the same context is current.
struct ScratchEntry {
  void *address;
  unsigned long long context_id;
};
ScratchEntry g_scratch[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

// Process-unique id of the calling thread's current context (cuCtxGetId, through the
// runtime's driver entry points: the library links no -lcuda). Fails when no context is
// current yet.
int current_context_id(unsigned long long *id) {
  static std::once_flag once;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr)
    return set_error(TROPNN_B200_ERR_DEVICE, "pairwise_backward_noalloc: cuCtxGetCurrent/cuCtxGetId unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return set_error(TROPNN_B200_ERR_DEVICE, "pairwise_backward_noalloc: no current CUDA context");
  if (get_id(ctx, id) != CUDA_SUCCESS)
    return set_error(TROPNN_B200_ERR_DEVICE, "pairwise_backward_noalloc: cuCtxGetId failed");
  return TROPNN_B200_OK;
}

// Device address of the scratch buffer in the current device's current context: looked up
// with cudaGetSymbolAddress on the first call made in that context (the set-up step) and
// cached with the context's id.
int scratch_address(void **out) {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_DEVICE, "pairwise_backward_noalloc: cudaGetDevice: %s", cudaGetErrorString(err));
  if (device < 0 || device >= kMaxDevices)
    return set_error(TROPNN_B200_ERR_DEVICE, "pairwise_backward_noalloc: device ordinal %d out of range", device);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchEntry &entry = g_scratch[device];
  unsigned long long ctx_id = 0;
  if (entry.address != nullptr && current_context_id(&ctx_id) == TROPNN_B200_OK && ctx_id == entry.context_id) {
    *out = entry.address;
    return TROPNN_B200_OK;
  }
  void *p = nullptr;
  err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (err != cudaSuccess || p == nullptr)
    return set_error(TROPNN_B200_ERR_LAUNCH, "pairwise_backward_noalloc: cudaGetSymbolAddress on device %d: %s",
                     device, cudaGetErrorString(err));
  TB_CHECK(current_context_id(&ctx_id));  // a context is current once the lookup has run
  entry.address = p;
  entry.context_id = ctx_id;
  *out = p;
  return TROPNN_B200_OK;
}

}  // namespace
}  // namespace tropnn_b200

extern "C" {

int tropnn_b200_pairwise_backward_noalloc(const float *grad_out, int64_t items, int64_t out_features,
                                          float output_scale, const int64_t *indices, const float *margins,
                                          const int64_t *anchors, int64_t tables, int64_t comparisons,
                                          int64_t in_features, const void *lut, int lut_dtype,
                                          int use_min_margin_ste, int surrogate, float *grad_latent,
                                          void *grad_thresholds, int grad_thresholds_dtype, void *grad_lut,
                                          void *stream) {
  TB_CHECK(tropnn_b200::check_current_device());
  const size_t need = tropnn_b200::pairwise_backward_workspace(items, tables, comparisons, in_features,
                                                               use_min_margin_ste);
  if (need == 0) {
    return tropnn_b200::set_error(
        TROPNN_B200_ERR_INVALID,
        "pairwise_backward_noalloc: bad sizes items=%lld tables=%lld comparisons=%lld in_features=%lld",
        (long long)items, (long long)tables, (long long)comparisons, (long long)in_features);
  }
  if (need > tropnn_b200::kScratchBytes) {
    return tropnn_b200::set_error(
        TROPNN_B200_ERR_INVALID,
        "pairwise_backward_noalloc: items=%lld tables=%lld comparisons=%lld in_features=%lld need %zu bytes of "
        "scratch, more than the fixed %zu-byte buffer; call tropnn_b200_pairwise_backward with a workspace instead",
        (long long)items, (long long)tables, (long long)comparisons, (long long)in_features, need,
        tropnn_b200::kScratchBytes);
  }
  void *scratch = nullptr;
  TB_CHECK(tropnn_b200::scratch_address(&scratch));
  // Every scratch byte the backward reads is written earlier in the same call, so the
  // previous call's leftovers need no clearing.
  TB_CHECK(tropnn_b200::pairwise_backward_impl(grad_out, items, out_features, output_scale, indices, margins, anchors,
                                               tables, comparisons, in_features, lut, lut_dtype, use_min_margin_ste,
                                               surrogate, grad_latent, grad_thresholds, grad_thresholds_dtype,
                                               grad_lut, scratch, tropnn_b200::kScratchBytes,
                                               tropnn_b200::as_stream(stream)));
  return tropnn_b200::clear_error();
}

}  // extern "C"
