// Cross-GPU epoch flags of the expert-parallel kernels: system-scope release /
// acquire on plain global words (this GPU's memory or a peer's NVLink mapping),
// and a bounded wait that records a status code instead of hanging.
#pragma once
#include <cstdint>

#include "sm100.cuh"

namespace b200 {

// Release / acquire fence at system scope.  The flag protocols here are release /
// acquire patterns (stores -> fence -> flag or counter; counter -> fence -> reads), for
// which acq_rel is enough; the sequentially consistent fence (__threadfence_system)
// also orders store -> load pairs, which none of them needs, and costs more.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= want (wrap-safe compare).  False on timeout (status
// recorded).  The time spent is added to *waited when it is not null.
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t want, int* status,
                                           unsigned long long* waited) {
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  while ((int32_t)(ld_acquire_sys(p) - want) < 0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(status, kStatusTimeoutFlag);
      ok = false;
      break;
    }
    __nanosleep(64);
  }
  if (waited != nullptr) atomicAdd(waited, (unsigned long long)(globaltimer_ns() - t0));
  return ok;
}

}  // namespace b200
