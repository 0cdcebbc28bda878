// p2p_flags.cuh -- epoch flags of the peer-memory exchange (ep_p2p.cu): release
// stores and acquire loads at system scope, and the bounded wait on them,
// shared by the exchange kernels and the tcgen05 receive front (tgemv.cuh).
#pragma once

#include "common.cuh"

namespace fmb {

__device__ __forceinline__ void flag_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t flag_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// The call's epoch: the explicit one, else one past the device counter (which
// the last kernel of a call advances).
__device__ __forceinline__ uint32_t call_epoch(uint32_t epoch, const uint32_t *ectr) {
    return epoch ? epoch : *reinterpret_cast<const volatile uint32_t *>(ectr) + 1u;
}

// Bounded wait for flag >= epoch; false (and FENCE_TIMEOUT raised) on expiry.
__device__ __forceinline__ bool wait_flag(const uint32_t *flag, uint32_t epoch, uint64_t timeout_ns, int *status) {
    if (flag_acquire(flag) >= epoch) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
        if (flag_acquire(flag) >= epoch) return true;
        if ((it & 63u) == 0 && global_ns() - t0 > timeout_ns) {
            raise_device_status(status, FM_STATUS_FENCE_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
}

// Every thread of the CTA returns once flags[0 .. world) have all reached
// `epoch` (or a wait timed out); threads below `world` do the waiting.
__device__ __forceinline__ void wait_flags_cta(const uint32_t *flags, uint32_t world, uint32_t epoch,
                                               uint64_t timeout_ns, int *status) {
    for (uint32_t s = threadIdx.x; s < world; s += blockDim.x) wait_flag(flags + s, epoch, timeout_ns, status);
    __syncthreads();
}

} // namespace fmb
