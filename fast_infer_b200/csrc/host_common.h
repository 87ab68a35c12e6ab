// Host-side helpers shared by the C-ABI entry points: error reporting, tensor-map
// encoding through the driver entry point, device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "fast_infer_b200.h"

namespace fi {

// Record a message for fi_last_error() and return `code`.
int fail(int code, const char* fmt, ...);
// Clear the thread's last-error message.
void clear_error();
// Map a CUDA runtime error to FI_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t e, const char* what);

// cuTensorMapEncodeTiled, resolved once through cudaGetDriverEntryPoint.
// Returns FI_OK or FI_ERR_CUDA / FI_ERR_ALIGNMENT with a message.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle, const char* what);

// Multiprocessor count of the current device (cached per device, thread-safe).
int sm_count();

// Devices whose per-device set-up results are cached; set-up on a device with a
// higher index runs on every call instead.
constexpr int kMaxCachedDevices = 64;

// One-time set-up per device (e.g. cudaFuncSetAttribute, which applies to the
// current device only). run(fn) calls fn once for the current device and returns
// its status; concurrent first calls on one device wait for the one that runs it,
// and a set-up that failed runs again on the next call.
class DeviceOnce {
 public:
  template <typename F>
  cudaError_t run(F&& fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxCachedDevices) return fn();
    if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = fn();
    if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  std::mutex mu_;
  std::atomic<bool> done_[kMaxCachedDevices] = {};
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch is on unless the environment sets FI_PDL=0.
bool pdl_enabled();

// Launches `kernel` allowing it to overlap the tail of the previous kernel on `st`
// (programmatic stream serialization). Only for kernels that call grid_dep_wait()
// before reading another kernel's output or writing global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// launch_pdl for a kernel launched in thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace fi
