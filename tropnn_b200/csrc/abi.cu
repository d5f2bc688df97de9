// Status plumbing and device checks shared by every entry point.
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace tropnn_b200 {

namespace {
thread_local std::string g_last_error;
// Compute-capability major per device ordinal, 0 = not queried yet. A benign race
// at worst queries twice.
int g_cc_major[64] = {0};
// Kernels launched by this library in this process (every launch is followed by one
// check_launch).
std::atomic<unsigned long long> g_kernel_launches{0};
}  // namespace

int set_error(int status, const char *fmt, ...) {
  char buf[1024];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  g_last_error = buf;
  return status;
}

int clear_error() {
  g_last_error.clear();
  return TROPNN_B200_OK;
}

static int device_major(int device, int *major) {
  if (device >= 0 && device < 64 && g_cc_major[device] != 0) {
    *major = g_cc_major[device];
    return TROPNN_B200_OK;
  }
  cudaError_t err = cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, device);
  if (err != cudaSuccess) {
    return set_error(TROPNN_B200_ERR_DEVICE, "cudaDeviceGetAttribute(device %d) failed: %s", device,
                     cudaGetErrorString(err));
  }
  if (device >= 0 && device < 64) g_cc_major[device] = *major;
  return TROPNN_B200_OK;
}

int check_current_device() {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    return set_error(TROPNN_B200_ERR_DEVICE, "no CUDA device available: %s", cudaGetErrorString(err));
  }
  int major = 0;
  TB_CHECK(device_major(device, &major));
  if (major != 10) {
    return set_error(TROPNN_B200_ERR_DEVICE,
                     "backend='b200' kernels are built for sm_100a only; device %d has compute capability %d.x",
                     device, major);
  }
  return TROPNN_B200_OK;
}

int check_launch(const char *what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(TROPNN_B200_ERR_LAUNCH, "%s: CUDA error: %s", what, cudaGetErrorString(err));
  }
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return TROPNN_B200_OK;
}

namespace {
struct SmemEntry {
  const void *func;
  int device;
  size_t bytes;
};
std::mutex g_smem_mutex;
std::vector<SmemEntry> g_smem_table;
}  // namespace

int ensure_dynamic_smem(const void *func, size_t bytes, const char *what) {
  if (bytes <= 48 * 1024) return TROPNN_B200_OK;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return set_error(TROPNN_B200_ERR_DEVICE, "%s: cudaGetDevice: %s", what, cudaGetErrorString(err));
  std::lock_guard<std::mutex> lock(g_smem_mutex);
  for (auto &e : g_smem_table) {
    if (e.func == func && e.device == device) {
      if (e.bytes >= bytes) return TROPNN_B200_OK;
      err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
      if (err != cudaSuccess)
        return set_error(TROPNN_B200_ERR_LAUNCH, "%s: %zu bytes of shared memory: %s", what, bytes,
                         cudaGetErrorString(err));
      e.bytes = bytes;
      return TROPNN_B200_OK;
    }
  }
  err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (err != cudaSuccess)
    return set_error(TROPNN_B200_ERR_LAUNCH, "%s: %zu bytes of shared memory: %s", what, bytes, cudaGetErrorString(err));
  g_smem_table.push_back({func, device, bytes});
  return TROPNN_B200_OK;
}

}  // namespace tropnn_b200

extern "C" {

const char *tropnn_b200_last_error(void) { return tropnn_b200::g_last_error.c_str(); }

int tropnn_b200_abi_version(void) { return 20; }

unsigned long long tropnn_b200_kernel_launches(void) {
  return tropnn_b200::g_kernel_launches.load(std::memory_order_relaxed);
}

int tropnn_b200_check_device(int device) {
  int major = 0;
  TB_CHECK(tropnn_b200::device_major(device, &major));
  if (major != 10) {
    return tropnn_b200::set_error(TROPNN_B200_ERR_DEVICE, "device %d has compute capability %d.x, not sm_100",
                                  device, major);
  }
  return tropnn_b200::clear_error();
}

}  // extern "C"
