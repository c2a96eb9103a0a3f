// Shared device/host helpers for the SuffixGPU sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/suffixgpu.h"

#define SG_FULL_MASK 0xffffffffu

#include <nvtx3/nvToolsExt.h>

namespace sg {

// Host-side NVTX range around an entry point: named ranges for nsys / ncu
// (--nvtx) timelines; without an attached tool a push / pop costs a few
// nanoseconds.
struct NvtxScope {
  explicit NvtxScope(const char* name) { nvtxRangePushA(name); }
  ~NvtxScope() { nvtxRangePop(); }
  NvtxScope(const NvtxScope&) = delete;
  NvtxScope& operator=(const NvtxScope&) = delete;
};

// Host-side: remember the last CUDA error seen by an entry point.
void set_cuda_error(cudaError_t e);

inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  return SG_OK;
}

// Reads one device int64 into *out through page-locked memory and
// synchronises `st` (the suffix-array builds' host round trip).
int read_device_i64(const int64_t* dev, int64_t* out, cudaStream_t st);

// Returns the device's max dynamic shared memory per block (opt-in).
int max_dyn_smem();
int num_sms();

int current_device();

// Make `kernel` launchable with `bytes` of dynamic shared memory on the
// current device. `cache` (one slot per device) remembers what was set.
// Static + dynamic shared memory must fit the per-block opt-in limit.
template <class Kernel>
inline int ensure_dyn_smem(Kernel* kernel, size_t bytes, int* cache) {
  if (bytes <= 48 * 1024) return SG_OK;
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return SG_ERR_CUDA;
  if (static_cast<int>(bytes) <= cache[dev]) return SG_OK;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  if (bytes + fa.sharedSizeBytes > static_cast<size_t>(max_dyn_smem()))
    return SG_ERR_UNSUPPORTED;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SG_ERR_CUDA;
  }
  cache[dev] = static_cast<int>(bytes);
  return SG_OK;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

__host__ __device__ inline uint32_t next_pow2_u32(uint32_t v) {
  v--;
  v |= v >> 1;
  v |= v >> 2;
  v |= v >> 4;
  v |= v >> 8;
  v |= v >> 16;
  return v + 1;
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

__device__ __forceinline__ int warp_sum(int v) {
  return __reduce_add_sync(SG_FULL_MASK, v);
}

// Inclusive warp scan of an int.
__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = lane_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(SG_FULL_MASK, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// ---------------------------------------------------------------------------
// mbarrier + TMA bulk copy (cp.async.bulk global -> shared)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
  // Make the initialised barrier visible to the async (TMA) proxy.
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem,
                                         uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Polls of a bounded mbarrier wait: far beyond any bulk copy of resident
// memory (a copy lands within microseconds; 2^22 polls take milliseconds).
constexpr int kWaitPolls = 1 << 22;

// Bounded wait for phase `parity` of `bar`: at most `polls` polls. Returns
// false if the bound ran out (the caller records an error and keeps going).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          int polls = kWaitPolls) {
  const uint32_t addr = smem_u32(bar);
  for (int it = 0; it < polls; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Ampere-style asynchronous 4-byte copy global -> shared (no register
// staging; completion per thread with cp_async_wait_all, which also orders
// the copies against later accesses, so the copy itself carries no memory
// clobber and does not hold back unrelated loads).
__device__ __forceinline__ void cp_async_4(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)),
               "l"(src));
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Bits of the device error word (sg_device_error): a bounded wait of the
// local draft kernel ran out.
constexpr unsigned kDevErrWait = SG_DEVERR_WAIT;

}  // namespace sg
