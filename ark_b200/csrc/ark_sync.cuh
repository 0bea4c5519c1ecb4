// ark_sync.cuh -- scoped acquire/release accesses and the global timer used
// by the cross-GPU exchange of the step's partials (P2P stores into peer
// memory mapped through CUDA IPC; every wait is bounded by the timer).
#pragma once

#include <stdint.h>

namespace ark {

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
                 : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
                 : "memory");
}

// Programmatic dependent launch (sm_90 and later).  launch_dependents lets
// the next kernel in the stream, when launched with programmatic stream
// serialization, start its blocks as this grid's blocks retire; wait, in
// that next kernel, returns once this grid has completed and its memory
// operations are visible.  In a kernel launched without the attribute,
// wait returns at once.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace ark
