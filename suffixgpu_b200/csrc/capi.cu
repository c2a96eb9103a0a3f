// Host-side helpers of the C ABI: status strings, error bookkeeping and
// cached device properties.
#include <cuda_runtime.h>

#include "sg_common.cuh"

namespace sg {

static thread_local int g_last_cuda_error = 0;

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

static int device_attr(cudaDeviceAttr attr) {
  int dev = 0;
  cudaGetDevice(&dev);
  int v = 0;
  cudaDeviceGetAttribute(&v, attr, dev);
  return v;
}

int max_dyn_smem() {
  return device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin);
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int num_sms() { return device_attr(cudaDevAttrMultiProcessorCount); }

}  // namespace sg

extern "C" const char* sg_status_string(int status) {
  switch (status) {
    case SG_OK: return "ok";
    case SG_ERR_INVALID: return "invalid argument";
    case SG_ERR_WORKSPACE: return "workspace missing or too small";
    case SG_ERR_CUDA: return "CUDA error";
    case SG_ERR_UNSUPPORTED: return "shape beyond supported limits";
    default: return "unknown status";
  }
}

extern "C" int sg_last_cuda_error(void) { return sg::g_last_cuda_error; }

extern "C" int sg_abi_version(void) { return (1 << 16) | 2; }

extern "C" int sg_mapped_host_ptr(const void* host_ptr, void** device_ptr) {
  if (!host_ptr || !device_ptr) return SG_ERR_INVALID;
  *device_ptr = nullptr;
  cudaPointerAttributes attr{};
  const cudaError_t e = cudaPointerGetAttributes(&attr, host_ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();  // a failed query leaves no sticky error behind
    sg::set_cuda_error(e);
    return SG_ERR_INVALID;
  }
  // page-locked host memory mapped into the device's address space; plain
  // pageable memory reports cudaMemoryTypeUnregistered and is refused
  if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
    return SG_ERR_INVALID;
  *device_ptr = attr.devicePointer;
  return SG_OK;
}
