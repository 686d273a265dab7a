// umma.cuh -- tcgen05 / TMA helpers shared by the tensor-core kernels of
// libvkq (the prefill GEMM and the tensor-core GEMV): shared-memory matrix and
// instruction descriptors, the MMA and its commit, 2D TMA tile loads, the
// raw super-block words of one 32-value unit, ring positions, and the
// driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "kq_device.cuh"

namespace vkq {

// ---- UMMA descriptors ---------------------------------------------------
// Shared-memory matrix descriptor: start >> 4 in bits [0,14), leading byte
// offset >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1 at
// bit 46, layout type in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// Instruction descriptor for kind::f16: fp32 accumulate (bits 4-5 = 1), A and
// B bf16 (bits 7-9 = 1, 10-12 = 1), A MN-major (bit 15), B K-major (bit 16 =
// 0), N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
            tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- raw super-block words for one 32-value unit --------------------------
// A unit is 32 consecutive n of one k: one sub-block of one super-block,
// since N and the tile origin are multiples of 32.
struct RawUnit {
    uint32_t v[10];
    uint32_t shf;  // Q6_K: byte misalignment of the ql/qh words (0 or 16 bits)
    uint32_t within;
    bool valid;
};

// Reads a unit from a super-block held in shared memory at `blk` (16-byte
// aligned for Q4_K/Q5_K, 2-byte aligned for Q6_K).
template <int QT>
__device__ __forceinline__ void load_unit(uint32_t blk, uint32_t within, bool valid, RawUnit &u) {
    u.valid = valid;
    u.within = within;
    if (!valid) return;
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const uint4 h = lds128(blk);
        const uint4 q = lds128(blk + (QT == kQ4K ? 16u : 48u) + (within >> 1));
        u.v[0] = h.x; u.v[1] = h.y; u.v[2] = h.z; u.v[3] = h.w;
        u.v[4] = q.x; u.v[5] = q.y; u.v[6] = q.z; u.v[7] = q.w;
        if constexpr (QT == kQ5K) u.v[8] = lds32(blk + 16u + (within >> 3));
    } else {
        // ql (offset within/2) and qh (offset 128 + within/4) are multiples of
        // 4 bytes into the block, so both share the block's misalignment
        const uint32_t ql = blk + (within >> 1);
        const uint32_t qh = blk + 128u + (within >> 2);
        u.shf = (ql & 3u) * 8u;
#pragma unroll
        for (int i = 0; i < 5; i++) u.v[i] = lds32((ql & ~3u) + 4u * i);
#pragma unroll
        for (int i = 0; i < 3; i++) u.v[5 + i] = lds32((qh & ~3u) + 4u * i);
        const uint32_t sraw = lds16(blk + 192u + (within >> 4));
        const uint32_t draw = lds16(blk + 208u);
        u.v[8] = sraw | (draw << 16);
    }
}

// Position in a ring of n stages: the stage index, the parity of the phase a
// consumer waits for next (a producer waits for the other one) and the number
// of uses so far; advancing takes no integer division.
struct RingPos {
    uint32_t idx = 0, phase = 0, uses = 0;
    __device__ __forceinline__ void next(uint32_t n) {
        uses++;
        if (++idx == n) {
            idx = 0;
            phase ^= 1u;
        }
    }
};

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// cuTensorMapEncodeTiled from the driver (nullptr when unavailable); defined in gemm.cu.
EncodeTiledFn encode_tiled_fn();

}  // namespace vkq
