// peer.cuh -- the device side of the all-gather channel shared by the GEMV
// kernels (gemv.cu, gemv_strip.cu): system-scope flag stores and loads on
// other GPUs' memory and the bounded wait on a rank's flag array.
//
// A channel is, per rank, a flag array of 2 * world words in device memory
// that every rank can write (slots [0, world): "started call s", [world,
// 2 world): "done call s") and the rank's own channel words sync[4]: sync[0]
// the number of the last call, sync[1] the CTAs of the current call that
// have finished, sync[2] the sticky "failed" mark.
#pragma once

#include <cstdint>

#include "kq_device.cuh"

namespace vkq {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *a) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *a, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
// Bounded wait until flags f[0..count) all equal seq.  Returns 0 on success,
// kStatusPeer at once when a flag is beyond seq (a rank is out of step), and
// kStatusTimeout when the budget runs out.
__device__ __forceinline__ int wait_flags_eq(const unsigned *f, int count, unsigned seq, uint64_t budget_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        bool all = true;
        for (int r = 0; r < count; r++) {
            const int d = (int)(ld_acquire_sys(f + r) - seq);
            if (d > 0) return kStatusPeer;
            all = all && d == 0;
        }
        if (all) return 0;
        if (globaltimer_ns() - t0 > budget_ns) return kStatusTimeout;
        __nanosleep(200);
    }
}

}  // namespace vkq
