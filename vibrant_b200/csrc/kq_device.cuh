// kq_device.cuh -- device helpers shared by the sm_100a kernels of libvkq.
//
// Super-block layouts follow the reference's parse functions
// (xupit3r/vibrant internal/tensor):
//   Q4_K 144 B: d[0:2] dmin[2:4] scales[4:16] qs[16:144]            quant_q4k.go:137-157
//   Q5_K 176 B: d[0:2] dmin[2:4] scales[4:16] qh[16:48] qs[48:176]  quant_q5k.go:229-252
//   Q6_K 210 B: ql[0:128] qh[128:192] scales[192:208] d[208:210]    quant_q6k.go:134-156
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace vkq {

constexpr int kQ4K = 12, kQ5K = 13, kQ6K = 14;

template <int QT> struct QT_ {};
template <> struct QT_<kQ4K> { static constexpr int BYTES = 144; };
template <> struct QT_<kQ5K> { static constexpr int BYTES = 176; };
template <> struct QT_<kQ6K> { static constexpr int BYTES = 210; };

// Device status word values (mirrors vkq_status).
constexpr int kStatusTimeout = 6;
constexpr int kStatusPeer = 8;  // a peer rank is out of step, or its channel already failed

// ---- float16 -> float32 exactly as the reference does it -----------------
// internal/tensor/tensor.go:629-676: subnormals are normalised exactly,
// 0x8000 gives +0 (the Go constant -0.0 is +0), every NaN gives 0x7FC00000.
__device__ __forceinline__ float go_f16_to_f32(uint32_t h) {
    uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0u) {
        if (mant == 0u) {
            bits = 0u;
        } else {
            // number of shifts until bit 10 is set: clz of the 32-bit mantissa minus 21
            uint32_t shift = __clz(mant) - 21u;
            uint32_t m = (mant << shift) & 0x3FFu;
            bits = (sign << 31) | ((127u - 14u - shift) << 23) | (m << 13);
        }
    } else if (exp == 31u) {
        bits = mant == 0u ? ((sign << 31) | 0x7F800000u) : 0x7FC00000u;
    } else {
        bits = (sign << 31) | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    return __uint_as_float(bits);
}

// Hardware half -> float (IEEE); used where only the matmul tolerance
// applies (it differs from go_f16_to_f32 only in the sign of zero and in
// NaN payloads, neither of which changes a sum of products).
__device__ __forceinline__ float hw_f16_to_f32(uint32_t h) {
    float f;
    asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "r"(h));
    return f;
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions) ------------------------
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// The same operations on float2 through the compiler's builtins, which keep
// each pair in an aligned register pair without moves around every use.
__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) { return __fmul2_rn(a, b); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// 2^23 + (byte in lane J of v), as a float: a byte permute into the exponent
// of 2^23; subtracting 2^23 then gives the byte's value exactly.
template <int J>
__device__ __forceinline__ float byte_as_magic(uint32_t v) {
    return __uint_as_float(prmt(v, 0x4B000000u, 0x7540u | J));
}

// ---- shared memory access -----------------------------------------------
__device__ __forceinline__ uint32_t smem_u32addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- thread-block clusters: rank, barrier, a float of another CTA's shared memory
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem(const float *local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32addr(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// 32-bit word at a 2-byte aligned shared address.
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a) {
    uint32_t base = a & ~3u;
    return __funnelshift_r(lds32(base), lds32(base + 4), (a & 3u) * 8u);
}

// ---- mbarrier / bulk copy / PDL -----------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }"
                 ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Same test, but the thread may sleep (up to hint_ns) until the phase
// completes instead of returning at once, so waiting warps issue few
// instructions.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `budget_ns` and returns false.  Nothing in
// this library waits without a limit on a barrier that another agent fills.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
        if (globaltimer_ns() - t0 > budget_ns) return false;
    }
}

// Bounded wait that polls instead of sleeping: for hand-offs on the
// critical path of a pipeline, where the time a suspended thread takes to
// resume would be paid on every step.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > budget_ns) return false;
    }
}

// Non-blocking test of a phase (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait that polls with test_wait: no suspension, so the thread sees
// the phase complete within a few cycles (a suspended try_wait can take far
// longer to resume).  For hand-offs on the per-step critical path.
__device__ __forceinline__ bool mbar_wait_poll(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > budget_ns) return false;
    }
}

// One-dimensional bulk copy global -> shared (no multicast), completing
// `bytes` of transaction count on `bar`.  dst, src and bytes are multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// 16-byte cp.async global -> shared that reads only `src_bytes` (1..16) of
// the source and zero-fills the rest; src and dst 16-byte aligned.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the arrival is part of the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// allow the next grid in the stream to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace vkq
