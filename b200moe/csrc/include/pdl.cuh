// Programmatic dependent launch: every kernel of this library is launched with
// the programmatic-stream-serialization attribute when B200MOE_PDL=1 and starts
// with pdl_enter(), which waits for the previous grid to complete (and its memory
// to be visible) before touching any global memory.  The hot kernels end with
// pdl_trigger(): once every CTA of the grid has reached it (or exited), the next
// grid in the stream may be scheduled, so its launch and CTA ramp-up overlap this
// grid's tail.  Dependencies are exactly those of plain stream order.  Grids
// launched without the attribute (or by other libraries) are waited for in full,
// and griddepcontrol.wait returns at once in a grid that was not launched
// programmatically.
//
// An earlier placement triggered at kernel entry: the dependents' CTAs then held
// SM slots while the running grid still needed them (decode step 16.93 ms against
// 16.50 ms without PDL).
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>

namespace b200 {

__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next programmatically launched grid be scheduled once every CTA has called it or exited.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B200MOE_PDL");
    return e != nullptr && std::string(e) == "1";
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline void pdl_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("kernel launch: ") + cudaGetErrorString(e));
}

inline int current_device() {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  return dev;
}

// Dynamic shared memory above 48 KB needs an opt-in per kernel AND per device: a
// process that launches on several GPUs sets it once on each (thread-safe).
template <typename... KArgs>
inline void smem_opt_in(void (*kern)(KArgs...), int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;  // (kernel, device, bytes)
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  if (!done.insert({reinterpret_cast<const void*>(kern), dev, bytes}).second) return;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    done.erase({reinterpret_cast<const void*>(kern), dev, bytes});
    throw std::runtime_error(std::string("cudaFuncSetAttribute(max dynamic smem): ") + cudaGetErrorString(e));
  }
}

// SM count of the current device, queried once per device.
inline int device_sm_count() {
  constexpr int kMaxDev = 64;
  static int count[kMaxDev] = {};
  static std::mutex mu;
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDev) throw std::runtime_error("device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (count[dev] == 0) {
    const cudaError_t e = cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) throw std::runtime_error(std::string("SM count: ") + cudaGetErrorString(e));
  }
  return count[dev];
}

}  // namespace b200
