// peer.cuh -- the device side of the all-gather channel shared by the GEMV
// kernels (gemv.cu, gemv_strip.cu): flagged-word stores into other GPUs'
// memory and the bounded wait on a rank's own slots.
//
// A channel is, per rank, a channel buffer in device memory that every rank
// can write (256 reserved bytes, then the slots below) and the rank's own
// channel words sync[4]: sync[0] the number of the last call, sync[1] the
// CTAs of the current call that have finished, sync[2] the sticky "failed"
// mark.
#pragma once

#include <cstdint>

#include "kq_device.cuh"

namespace vkq {

// ---- flagged-word exchange (the column-strip all-gather) ----
// From byte kChannelSlotsOffset on, a rank's channel buffer holds two 8-byte
// slots per output element (m, n) of the full [M][N] output, one per parity
// of the call number: (call number << 32) | value bits, written by the rank
// that owns column n with one 64-bit store (single-copy atomic, also over
// NVLink), so the value and its call number arrive together and no fence or
// "done" flag is needed.  Two parities make the "started" handshake needless
// as well: a rank can be at most one call ahead of another (to finish call s
// it must have received every rank's call-s values, which each rank sends
// only after its call s - 1 is complete), so a slot is never overwritten
// before its reader has taken it.
constexpr size_t kChannelSlotsOffset = 256;
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *a, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *a) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t *channel_slot(unsigned *chan, int64_t N, int64_t m, int64_t n, unsigned seq) {
    return reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(chan) + kChannelSlotsOffset) +
           ((m * N + n) * 2 + (seq & 1u));
}
// Bounded wait for the slot of call seq; returns 0 with the value in *v,
// kStatusPeer when the slot carries a later call (a rank out of step),
// kStatusTimeout when the budget runs out, or -1 when *failed turns nonzero
// meanwhile (another thread found the fault and reported it).
__device__ __forceinline__ int wait_slot(const uint64_t *slot, unsigned seq, uint64_t budget_ns,
                                         const unsigned *failed, float *v) {
    uint64_t t0 = 0;
    for (int it = 0;; it++) {
        const uint64_t s = ld_relaxed_sys_u64(slot);
        const int d = (int)((unsigned)(s >> 32) - seq);
        if (d == 0) {
            *v = __uint_as_float((unsigned)s);
            return 0;
        }
        if (d > 0) return kStatusPeer;
        if (it >= 32) {
            if (*reinterpret_cast<const volatile unsigned *>(failed) != 0u) return -1;
            const uint64_t now = globaltimer_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > budget_ns) return kStatusTimeout;
            __nanosleep(64);
        }
    }
}

}  // namespace vkq
