// C-ABI plumbing: error strings, library version, cached device properties.
#include "common.cuh"

#include <string.h>

namespace specdec {

static thread_local char g_last_error[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int device_info(DeviceInfo* out) {
  static DeviceInfo cache[kMaxDevices];
  static std::atomic<bool> valid[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  SPECDEC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(kInvalidArgument, "device ordinal %d out of range", dev);
  if (!valid[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!valid[dev].load(std::memory_order_relaxed)) {
      DeviceInfo info;
      SPECDEC_CUDA_TRY(cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev));
      SPECDEC_CUDA_TRY(cudaDeviceGetAttribute(&info.max_threads_per_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev));
      SPECDEC_CUDA_TRY(cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
      SPECDEC_CUDA_TRY(cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
      cache[dev] = info;
      valid[dev].store(true, std::memory_order_release);
    }
  }
  *out = cache[dev];
  return kOk;
}

}  // namespace specdec

extern "C" {

const char* specdec_last_error(void) { return specdec::g_last_error; }

int specdec_version(void) { return 1; }

// Returns 1 when the current device is a compute capability 10.0 (B200-class) GPU this library was built for.
int specdec_device_supported(void) {
  specdec::DeviceInfo info;
  if (specdec::device_info(&info) != specdec::kOk) return 0;
  return info.cc_major == 10 && info.cc_minor == 0;
}

}  // extern "C"
