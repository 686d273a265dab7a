// gemm.cu -- k-quant dequantize + GEMM on sm_100a tensor cores (tcgen05 / TMEM).
//
// Y[m][n] = sum_k X[m][k] * W[k][n] for M > 8 (prefill), W a Q4_K / Q5_K / Q6_K
// weight in vibrant's orientation (W[k][n] = value k*N + n of the super-block
// stream, internal/gguf/loader.go:24-27).  Replaces matmul_f32
// (internal/gpu/cuda/kernels.cu:11-57, launched for M > 1 by matmulGPU,
// internal/tensor/ops_cuda.go:64-73), which needed the weight expanded to
// float32 first.  Arithmetic: bf16 operands, fp32 accumulate (tolerance class
// 2e-2 of sum_k |x w|).
//
// The product is computed transposed, D[n][m] = W^T[n][k] . X^T[k][m], so
// that the operand built on the fly (the dequantized weight) is the MMA's A:
//  * A tile: 128 n x 64 k bf16, written by the dequant warps straight from the
//    packed blocks into the MN-major 128-byte-swizzled layout (atoms of 64 n x
//    8 k, 1024 bytes; the two 64-n halves 1024 B apart, k groups 2048 B apart).
//    A super-block row gives 256 consecutive n of one k, so MN-major is the
//    natural orientation.
//  * B tile: X converted to bf16 once per call (workspace), loaded by TMA as
//    [mma_n rows of m] x [64 k] with the 128-byte swizzle (K-major, 8-row
//    atoms, SBO 1024 B).  No multicast.
//  * D: fp32 in TMEM, 128 lanes (n) x mma_n columns (m) per accumulator; two
//    accumulators cover 512 rows of X per CTA, so each dequantized W tile
//    feeds 2 x 4 MMAs (128 x 256 x 16) per 64-k step.
// Warp roles (192 threads): warp 0 issues the TMA loads of X, warp 1 owns TMEM
// and issues tcgen05.mma from one thread, warps 2..5 dequantize W into the A
// ring and afterwards drain TMEM to Y (warp w reads TMEM lanes 32*(w%4)..).
// Every mbarrier wait is bounded and reports a timeout through a device
// status word; TMEM is always released.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

static __device__ int g_gemm_status;

constexpr int kGBN = 128;                     // n rows per CTA (MMA M)
constexpr int kGBK = 64;                      // k per stage: one 128-byte swizzle row of bf16
constexpr int kGThreads = 192;                // 6 warps
constexpr int kGDeq = 128;                    // dequant / epilogue threads (warps 2..5)
constexpr int kAStage = kGBN * kGBK * 2;      // 16 KB
constexpr uint64_t kGWaitNs = 2000000000ull;  // bounded waits: 2 s

struct GemmParams {
    const uint8_t *w;
    float *y;
    int64_t K, N, M;
    int mma_n;   // m columns per accumulator (multiple of 32, <= 256: the epilogue drains 32 at a time)
    int nacc;    // accumulators per CTA (1 or 2)
    int stages;  // ring depth
    int ksteps;  // ceil(K / 64)
    int tmem_cols;
};

__device__ __forceinline__ void g_set_status(int c) { atomicExch(&g_gemm_status, c); }

__device__ __forceinline__ void g_wait(uint32_t bar, uint32_t parity) {
    if (!mbar_wait_bounded(bar, parity, kGWaitNs)) g_set_status(kStatusTimeout);
}

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

// ---- raw super-block fetch for one 32-value unit --------------------------
// A unit is 32 consecutive n of one k (one sub-block of one super-block,
// since N and n0 are multiples of 32).
struct RawUnit {
    uint32_t v[10];
    uint32_t shf;  // Q6_K: byte misalignment of ql/qh words (0 or 16 bits)
    uint32_t within;
    bool valid;
};

template <int QT>
__device__ __forceinline__ void fetch_unit(const uint8_t *__restrict__ w, int64_t vidx, bool valid, RawUnit &u) {
    constexpr int B = QT_<QT>::BYTES;
    u.valid = valid;
    u.within = (uint32_t)(vidx & 255);
    if (!valid) return;
    const uint8_t *blk = w + (vidx >> 8) * B;
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const uint4 h = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(blk + (QT == kQ4K ? 16 : 48) + (u.within >> 1)));
        u.v[0] = h.x; u.v[1] = h.y; u.v[2] = h.z; u.v[3] = h.w;
        u.v[4] = q.x; u.v[5] = q.y; u.v[6] = q.z; u.v[7] = q.w;
        if constexpr (QT == kQ5K) u.v[8] = __ldg(reinterpret_cast<const uint32_t *>(blk + 16 + (u.within >> 3)));
    } else {
        // blocks are 2-byte aligned: fetch aligned words and shift later
        const uintptr_t ql = reinterpret_cast<uintptr_t>(blk) + (u.within >> 1);
        const uintptr_t qh = reinterpret_cast<uintptr_t>(blk) + 128 + (u.within >> 2);
        u.shf = (uint32_t)(ql & 3u) * 8u;  // ql and qh share the misalignment (both offsets are even multiples of 4)
        const uint32_t *qlw = reinterpret_cast<const uint32_t *>(ql & ~uintptr_t(3));
        const uint32_t *qhw = reinterpret_cast<const uint32_t *>(qh & ~uintptr_t(3));
#pragma unroll
        for (int i = 0; i < 5; i++) u.v[i] = __ldg(qlw + i);
#pragma unroll
        for (int i = 0; i < 3; i++) u.v[5 + i] = __ldg(qhw + i);
        const uint16_t sraw = __ldg(reinterpret_cast<const uint16_t *>(blk + 192 + (u.within >> 4)));
        const uint16_t draw = __ldg(reinterpret_cast<const uint16_t *>(blk + 208));
        u.v[8] = (uint32_t)sraw | ((uint32_t)draw << 16);
    }
}

// Decode one unit into 32 fp32 values, rounded to bf16 pairs (16 words).
template <int QT>
__device__ __forceinline__ void decode_unit_bf16(const RawUnit &u, uint32_t (&out)[16]) {
    if (!u.valid) {
#pragma unroll
        for (int i = 0; i < 16; i++) out[i] = 0u;
        return;
    }
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const float d = hw_f16_to_f32(u.v[0] & 0xFFFFu), dmin = hw_f16_to_f32(u.v[0] >> 16);
        const int sb = (int)(u.within >> 5);
        const uint32_t sc24 = sb < 4 ? u.v[1] : __funnelshift_r(u.v[1], u.v[2], 24);
        const uint32_t m24 = sb < 4 ? __funnelshift_r(u.v[2], u.v[3], 16) : (u.v[3] >> 8);
        const uint32_t sh = 6u * (sb & 3);
        const float ds = d * (float)((sc24 >> sh) & 63u);
        const float dm = dmin * (float)((m24 >> sh) & 63u);
        const uint32_t qh = (QT == kQ5K) ? u.v[8] : 0u;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int v0 = 2 * i, v1 = 2 * i + 1;
            uint32_t q0 = (u.v[4 + (v0 >> 3)] >> (4 * (v0 & 7))) & 15u;
            uint32_t q1 = (u.v[4 + (v1 >> 3)] >> (4 * (v1 & 7))) & 15u;
            if constexpr (QT == kQ5K) {
                q0 |= ((qh >> v0) & 1u) << 4;
                q1 |= ((qh >> v1) & 1u) << 4;
            }
            out[i] = bf16x2(fmaf(ds, (float)q0, -dm), fmaf(ds, (float)q1, -dm));
        }
    } else {
        uint32_t ql[4], qh[2];
#pragma unroll
        for (int i = 0; i < 4; i++) ql[i] = __funnelshift_r(u.v[i], u.v[i + 1], u.shf);
#pragma unroll
        for (int i = 0; i < 2; i++) qh[i] = __funnelshift_r(u.v[5 + i], u.v[6 + i], u.shf);
        const float d = hw_f16_to_f32(u.v[8] >> 16);
        const float ds0 = d * (float)(int)(int8_t)(u.v[8] & 0xFFu);
        const float ds1 = d * (float)(int)(int8_t)((u.v[8] >> 8) & 0xFFu);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int v0 = 2 * i, v1 = 2 * i + 1;
            const int q0 = (int)(((ql[v0 >> 3] >> (4 * (v0 & 7))) & 15u) | (((qh[v0 >> 4] >> (2 * (v0 & 15))) & 3u) << 4));
            const int q1 = (int)(((ql[v1 >> 3] >> (4 * (v1 & 7))) & 15u) | (((qh[v1 >> 4] >> (2 * (v1 & 15))) & 3u) << 4));
            const float s = (v0 < 16) ? ds0 : ds1;
            out[i] = bf16x2(s * (float)(q0 - 32), s * (float)(q1 - 32));
        }
    }
}

template <int QT>
__global__ void __launch_bounds__(kGThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmx,
                                                            const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32addr(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    const int S = p.stages;
    const uint32_t a_ring = base;                                           // S x 16 KB
    const uint32_t b_stage = (uint32_t)(p.nacc * p.mma_n * 128);             // bytes per B stage
    const uint32_t b_ring = a_ring + (uint32_t)(S * kAStage);
    const uint32_t bars = b_ring + (uint32_t)S * b_stage;                    // a_full, b_full, empty [S], acc_full
    auto a_full = [&](int s) { return bars + 8u * (uint32_t)s; };
    auto b_full = [&](int s) { return bars + 8u * (uint32_t)(S + s); };
    auto st_empty = [&](int s) { return bars + 8u * (uint32_t)(2 * S + s); };
    const uint32_t acc_full = bars + 8u * (uint32_t)(3 * S);
    const uint32_t tmem_slot = acc_full + 8u;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n0 = (int64_t)blockIdx.x * kGBN;
    const int64_t m0 = (int64_t)blockIdx.y * p.nacc * p.mma_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(a_full(s), 4);   // one arrival per dequant warp
            mbar_init(b_full(s), 1);   // TMA expect_tx
            mbar_init(st_empty(s), 1); // tcgen05.commit
        }
        mbar_init(acc_full, 1);
        mbar_init_fence();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
    }
    if (warp == 1) {  // TMEM allocation (whole warp)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = lds32(tmem_slot);

    // weights do not depend on the preceding kernel; X and Y do
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        // ---------------- TMA producer: bf16 X tiles ----------------
        if (lane == 0) {
            for (int ks = 0; ks < p.ksteps; ks++) {
                const int s = ks % S;
                if (ks >= S) g_wait(st_empty(s), (uint32_t)(((ks / S) - 1) & 1));
                mbar_arrive_expect_tx(b_full(s), b_stage);
                for (int a = 0; a < p.nacc; a++)
                    tma_load_2d(b_ring + (uint32_t)s * b_stage + (uint32_t)(a * p.mma_n * 128), &tmx, ks * kGBK,
                                (int)(m0 + a * p.mma_n), b_full(s));
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(kGBN, p.mma_n);
            for (int ks = 0; ks < p.ksteps; ks++) {
                const int s = ks % S;
                const uint32_t par = (uint32_t)((ks / S) & 1);
                g_wait(a_full(s), par);
                g_wait(b_full(s), par);
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t a_s = a_ring + (uint32_t)(s * kAStage);
                const uint32_t b_s = b_ring + (uint32_t)s * b_stage;
#pragma unroll
                for (int kk = 0; kk < kGBK / 16; kk++) {
                    // A: 2 k-groups of 8 per 16-k step (k-group stride 2048 B), n halves 1024 B apart
                    const uint64_t da = smem_desc_sw128(a_s + (uint32_t)(kk * 4096), 1024u, 2048u);
                    for (int a = 0; a < p.nacc; a++) {
                        // B: K-major, 16 k = 32 bytes into each 128-byte row, 8-row atoms 1024 B apart
                        const uint64_t db =
                            smem_desc_sw128(b_s + (uint32_t)(a * p.mma_n * 128) + (uint32_t)(kk * 32), 16u, 1024u);
                        umma_bf16(tmem + (uint32_t)(a * p.mma_n), da, db, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(st_empty(s));  // frees the stage once these MMAs have read it
            }
            umma_commit(acc_full);
        }
    } else {
        // ---------------- dequant warps: W -> bf16 A tiles ----------------
        const int dt = threadIdx.x - 64;  // 0..127
        RawUnit cur[2], nxt[2];
        auto unit_of = [&](int ks, int j, int64_t &vidx) -> bool {
            const int u = dt + j * kGDeq;  // 0..255
            const int kl = u >> 2, sb4 = u & 3;
            const int64_t k = (int64_t)ks * kGBK + kl;
            const int64_t n = n0 + 32 * sb4;
            vidx = k * p.N + n;
            return k < p.K && n < p.N;
        };
        for (int j = 0; j < 2; j++) {
            int64_t vi;
            const bool ok = unit_of(0, j, vi);
            fetch_unit<QT>(p.w, vi, ok, cur[j]);
        }
        for (int ks = 0; ks < p.ksteps; ks++) {
            const int s = ks % S;
            // fetch the next step's raw bytes first (latency overlaps this step)
            if (ks + 1 < p.ksteps) {
                for (int j = 0; j < 2; j++) {
                    int64_t vi;
                    const bool ok = unit_of(ks + 1, j, vi);
                    fetch_unit<QT>(p.w, vi, ok, nxt[j]);
                }
            }
            if (ks >= S) g_wait(st_empty(s), (uint32_t)(((ks / S) - 1) & 1));
            const uint32_t a_s = a_ring + (uint32_t)(s * kAStage);
#pragma unroll
            for (int j = 0; j < 2; j++) {
                uint32_t wv[16];
                decode_unit_bf16<QT>(cur[j], wv);
                const int u = dt + j * kGDeq;
                const int kl = u >> 2, sb4 = u & 3;
                const int g = kl >> 3, kin = kl & 7;
#pragma unroll
                for (int c4 = 0; c4 < 4; c4++) {
                    const int nl = 32 * sb4 + 8 * c4;  // first n of this 16-byte chunk
                    const int h = nl >> 6, c = (nl & 63) >> 3;
                    const uint32_t addr =
                        a_s + (uint32_t)((g * 2 + h) * 1024 + kin * 128 + ((c ^ kin) << 4));
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(wv[4 * c4]),
                                 "r"(wv[4 * c4 + 1]), "r"(wv[4 * c4 + 2]), "r"(wv[4 * c4 + 3])
                                 : "memory");
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full(s));
            cur[0] = nxt[0];
            cur[1] = nxt[1];
        }

        // ---------------- epilogue: TMEM -> Y ----------------
        g_wait(acc_full, 0);
        asm volatile("tcgen05.fence::after_thread_sync;");
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        const int64_t n = n0 + 32 * q + lane;
        for (int a = 0; a < p.nacc; a++) {
            for (int c = 0; c < p.mma_n / 32; c++) {
                uint32_t r[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * p.mma_n + 32 * c);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                      "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                      "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
                      "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
                      "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (n < p.N) {
                    const int64_t mb = m0 + a * p.mma_n + 32 * c;
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (mb + j < p.M) p.y[(mb + j) * p.N + n] = __uint_as_float(r[j]);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols));
    }
}

// X fp32 [M, K] -> bf16 [M, K] (round to nearest even)
__global__ void __launch_bounds__(256) x_to_bf16_kernel(const float *__restrict__ x, uint32_t *__restrict__ xb,
                                                        int64_t npairs) {
    pdl_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npairs;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float2 v = reinterpret_cast<const float2 *>(x)[i];
        xb[i] = bf16x2(v.x, v.y);
    }
    pdl_launch_dependents();
}

// ------------------------------- host side -------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static std::mutex mu;
    static EncodeTiledFn fn = nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

struct GemmPlan {
    int mma_n, nacc, stages, ksteps, tmem_cols;
    int64_t xb_bytes;  // bf16 copy of X in the workspace
    size_t smem;
    dim3 grid;
};

static GemmPlan gemm_plan(const GemvShape &s) {
    GemmPlan g{};
    if (s.M >= 512) {
        g.mma_n = 256;
        g.nacc = 2;
    } else if (s.M > 256) {
        g.mma_n = (int)((((s.M + 1) / 2) + 31) / 32 * 32);
        g.nacc = 2;
    } else {
        g.mma_n = (int)((s.M + 31) / 32 * 32);
        g.nacc = 1;
    }
    const int cols = g.mma_n * g.nacc;
    g.tmem_cols = 32;
    while (g.tmem_cols < cols) g.tmem_cols <<= 1;
    g.ksteps = (int)((s.K + kGBK - 1) / kGBK);
    const size_t stage = (size_t)kAStage + (size_t)g.nacc * g.mma_n * 128;
    g.stages = 4;
    while (g.stages > 2 && 1024 + g.stages * stage + 256 > (size_t)220 * 1024) g.stages--;
    g.smem = 1024 + g.stages * stage + 256;
    g.xb_bytes = ((s.M * s.K * 2) + 255) & ~int64_t(255);
    g.grid = dim3((unsigned)((s.N + kGBN - 1) / kGBN), (unsigned)((s.M + (int64_t)cols - 1) / cols));
    return g;
}

size_t gemm_workspace_bytes(const GemvShape &s) {
    if (s.N % 32 != 0) return 0;
    return (size_t)gemm_plan(s).xb_bytes;
}

template <int QT>
static cudaError_t launch_gemm(const CUtensorMap &tm, const GemmParams &gp, const GemmPlan &g, cudaStream_t st) {
    auto kern = gemm_kernel<QT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = g.grid;
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tm, gp);
}

int gemm_launch(const GemvShape &s, const void *w, const float *x, float *y, void *ws, size_t ws_bytes,
                cudaStream_t stream, int device) {
    (void)device;
    if (s.N % 32 != 0) {
        set_error("the tensor-core GEMM needs N %% 32 == 0 (got N=%lld)", (long long)s.N);
        return 2;
    }
    if (s.K % 8 != 0) {
        set_error("the tensor-core GEMM needs K %% 8 == 0 (got K=%lld): TMA rows of bf16 X must be 16-byte multiples",
                  (long long)s.K);
        return 2;
    }
    if (reinterpret_cast<uintptr_t>(x) & 7u) {
        set_error("the tensor-core GEMM needs x 8-byte aligned");
        return 3;
    }
    const GemmPlan g = gemm_plan(s);
    if (ws == nullptr || ws_bytes < (size_t)g.xb_bytes) {
        set_error("gemm needs a workspace of %lld bytes (got %zu)", (long long)g.xb_bytes, ws_bytes);
        return 4;
    }
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return 5;
    }
    uint32_t *xb = static_cast<uint32_t *>(ws);
    // 1. X -> bf16
    {
        const int64_t npairs = s.M * s.K / 2;
        const int grid = (int)std::min<int64_t>((npairs + 255) / 256, (int64_t)device_sm_count(device) * 8);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)std::max(grid, 1));
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, x_to_bf16_kernel, x, xb, npairs);
        if (e != cudaSuccess) {
            set_error("x to bf16 launch failed: %s", cudaGetErrorString(e));
            return 5;
        }
    }
    // 2. tensor map over the bf16 X: dims {K, M}, box {64, mma_n}, 128-byte swizzle
    CUtensorMap tm;
    const cuuint64_t dims[2] = {(cuuint64_t)s.K, (cuuint64_t)s.M};
    const cuuint64_t strides[1] = {(cuuint64_t)(s.K * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kGBK, (cuuint32_t)g.mma_n};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return 5;
    }
    GemmParams gp{};
    gp.w = static_cast<const uint8_t *>(w);
    gp.y = y;
    gp.K = s.K;
    gp.N = s.N;
    gp.M = s.M;
    gp.mma_n = g.mma_n;
    gp.nacc = g.nacc;
    gp.stages = g.stages;
    gp.ksteps = g.ksteps;
    gp.tmem_cols = g.tmem_cols;
    cudaError_t e;
    switch (s.qtype) {
    case kQ4K: e = launch_gemm<kQ4K>(tm, gp, g, stream); break;
    case kQ5K: e = launch_gemm<kQ5K>(tm, gp, g, stream); break;
    default: e = launch_gemm<kQ6K>(tm, gp, g, stream); break;
    }
    if (e != cudaSuccess) {
        set_error("gemm launch failed: %s", cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int gemm_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
    return v;
}

}  // namespace vkq
