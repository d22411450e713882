// Error plumbing for the C ABI: gfxb_status codes plus a per-thread message,
// the C counterpart of the reference's Status (include/gfxinfer/status.h).
#include <cstdlib>
#include <string>

#include "common.cuh"

namespace gfxb {

namespace {
thread_local std::string g_last_error;
}

void set_error(const char* message) { g_last_error = message != nullptr ? message : ""; }

void set_error_cuda(cudaError_t error, const char* context) {
  g_last_error = std::string(context) + ": " + cudaGetErrorString(error);
}

int fail(int status, const char* message) {
  set_error(message);
  return status;
}

bool pdl_enabled() {
  static const bool enabled = [] {
    const char* value = std::getenv("GFXB_PDL");
    return value == nullptr || value[0] != '0';
  }();
  return enabled;
}

int launch_status(const char* context) {
  const cudaError_t error = cudaGetLastError();
  if (error == cudaSuccess) return GFXB_OK;
  set_error_cuda(error, context);
  return error == cudaErrorMemoryAllocation ? GFXB_OUT_OF_MEMORY : GFXB_CUDA_ERROR;
}

int current_device(int* device) {
  const cudaError_t error = cudaGetDevice(device);
  if (error != cudaSuccess) {
    set_error_cuda(error, "cudaGetDevice failed");
    return GFXB_CUDA_ERROR;
  }
  if (*device < 0 || *device >= kMaxDevices) return fail(GFXB_UNSUPPORTED, "device index beyond the per-device tables");
  return GFXB_OK;
}

int device_sm_count(int* sms) {
  static std::atomic<int> counts[kMaxDevices] = {};
  int device = 0;
  GFXB_TRY(current_device(&device));
  int count = counts[device].load(std::memory_order_relaxed);
  if (count == 0) {
    const cudaError_t error = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
    if (error != cudaSuccess || count <= 0) {
      set_error_cuda(error, "SM count query failed");
      return GFXB_CUDA_ERROR;
    }
    counts[device].store(count, std::memory_order_relaxed);
  }
  *sms = count;
  return GFXB_OK;
}

}  // namespace gfxb

extern "C" const char* gfxb_last_error_message(void) { return gfxb::g_last_error.c_str(); }

extern "C" int gfxb_abi_version(void) { return 1; }

extern "C" int gfxb_require_sm100_device(int device_index, gfxb_device_info* info) {
  int count = 0;
  cudaError_t error = cudaGetDeviceCount(&count);
  if (error != cudaSuccess) {
    gfxb::set_error_cuda(error, "CUDA device enumeration failed");
    return GFXB_CUDA_ERROR;
  }
  if (device_index < 0 || device_index >= count) {
    return gfxb::fail(GFXB_INVALID_ARGUMENT, "requested CUDA device index is out of range");
  }
  cudaDeviceProp properties{};
  error = cudaGetDeviceProperties(&properties, device_index);
  if (error != cudaSuccess) {
    gfxb::set_error_cuda(error, "CUDA device query failed");
    return GFXB_CUDA_ERROR;
  }
  if (info != nullptr) {
    info->index = device_index;
    info->compute_major = properties.major;
    info->compute_minor = properties.minor;
    info->multiprocessors = properties.multiProcessorCount;
    info->global_memory_bytes = properties.totalGlobalMem;
    std::snprintf(info->name, sizeof info->name, "%s", properties.name);
  }
  if (properties.major != 10 || properties.minor != 0) {
    return gfxb::fail(GFXB_UNSUPPORTED, "gfxinfer-b200 requires an sm_100 (B200) device");
  }
  return GFXB_OK;
}
