// gemv_tc.cu -- k-quant dequantize + GEMV on the sm_100a tensor cores with
// fp32-class results (the GEMV tolerance, 1e-5 of sum_k |x w|), M <= 4.
//
// y[m][n] = sum_k x[m][k] * W[k][n] for a Q4_K / Q5_K / Q6_K weight in
// vibrant's orientation (W[k][n] is value k*N + n of the super-block stream,
// internal/gguf/loader.go:24-27).  It replaces the fp32 single-row kernel
// behind matmulGPU (internal/gpu/cuda/kernels.cu:61-77 via
// internal/tensor/ops_cuda.go:55-63).
//
// Why tensor cores for a GEMV: on CUDA cores every value costs a decode, an
// fma forming the weight and an fma with x (issue-bound near 7 instructions
// per value).  Here the weight's affine form is split so that the per-value
// work is only the decode:
//   Q4_K/Q5_K  W = s_g * q - mn_g   (s = d*sc, mn = dmin*m per 32-value sub-block g)
//   Q6_K       W = s_g * (q - 32)   (s = d*sc per 16-value group g)
//   y[m][n] = sum_k (x[m][k] * s_kg) * q_kn  -  sum_k corr_kg
// The MMA computes D[n][c] = sum_k A[n][k] * B[k][c] with
//  * A[n][k] = 128 + q_kn as bf16, exact (q < 64): one LOP3 turns two packed
//    nibbles into two bf16 values (0x4300 | q) with no conversion;
//  * B[k][c] = the products a = x[m][k] * s_kg split into three bf16 parts
//    (a = b1 + b2 + b3 to 24 bits), one column per (m, sub-block g, part):
//    each 128-row MMA half covers 4 sub-blocks (Q4_K/Q5_K) or 8 groups (Q6_K)
//    of one super-block row, so the per-(row, sub-block) scale rides in B;
//  * fp32 accumulators in TMEM; the epilogue adds the three part columns of
//    each row's sub-block and subtracts the correction
//      Q4_K/Q5_K: sum_k (128 * a + x * mn),   Q6_K: sum_k 160 * a
//    (128 undoes the bf16 offset, 32 the Q6_K zero point), accumulated on the
//    CUDA cores in fp32 by the thread that built the B entries.
// Work: tiles of 256 output columns (one super-block per k row; when rows
// straddle blocks, two half-blocks) and stages of 64 k; the (tile, stage)
// space is cut into equal contiguous ranges, one per CTA (stream-K), so every
// SM gets the same share; a tile split over CTAs goes through a partials
// buffer and the last CTA to arrive adds the partials in CTA order
// (deterministic).  Roles (704 threads): warp 0 stages raw super-blocks with
// 2D TMA (or 16-byte cp.async when rows have no 16-byte pitch), warp 1 owns
// TMEM and issues the MMAs, warps 2..17 decode one 32-value unit per thread
// per stage (A tile, B entries, corrections), warps 18..21 drain TMEM.
// Every mbarrier wait is bounded; a wait that runs out sets the status word
// and an abort flag, copies in flight are waited for and TMEM is released.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "kq_device.cuh"
#include "umma.cuh"
#include "vkq_internal.h"

namespace vkq {

static __device__ int g_tc_status;

namespace {
constexpr int kTK = 64;                 // k per stage
constexpr int kTN = 256;                // n per tile: two MMA halves of 128
constexpr int kTHalf = 128 * kTK * 2;   // 16 KB: the A operand of one half for a stage
constexpr int kTAStage = 2 * kTHalf;    // 32 KB
constexpr int kTWRaw = 0, kTWMma = 1, kTWDec = 2, kTNDec = 16, kTWEpi = 18, kTNEpi = 4;
constexpr int kTThreads = (kTWEpi + kTNEpi) * 32;  // 704
constexpr int kTMaxStages = 8;
constexpr int kNGrp = 4;                // decode groups: stages j = g (mod 4)
constexpr uint64_t kTWaitNs = 2000000000ull;  // bounded waits: 2 s
constexpr uint64_t kTDrainNs = 20000000ull;   // copies in flight at teardown: 20 ms
}  // namespace

struct TcParams {
    const uint8_t *w;
    int64_t w_bytes;
    int64_t rs, ld, n_base;  // row k of the weight starts at value position k*rs + ((k*ld + n_base) & 255)
    int64_t pitch;           // TMA staging: bytes per weight row (a multiple of 16)
    const float *x;
    float *y;
    int64_t y_ld;
    int64_t K, N;
    int M;
    int tiles, ksteps, per, grid;
    int sr, sa;
    int raw_slot, raw_tma;
    int nc;                  // MMA N: B columns per half
    int nbuf, tmem_cols, acc_stride;
    float *partials;         // [grid][2][MR][256]
    int *counters;           // [tiles][4] (one per row quarter), zero between calls
};

__device__ __forceinline__ void tc_set_status(int c) { atomicExch(&g_tc_status, c); }

__device__ __forceinline__ uint32_t bf16_bits(float f) {
    uint16_t h;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
    return h;
}
// a = b1 + b2 + b3 (bf16 parts; the sum holds 24 significant bits of a) and
// the fp32 value of that sum.
__device__ __forceinline__ void split3(float a, uint32_t &b1, uint32_t &b2, uint32_t &b3, float &ahat) {
    b1 = bf16_bits(a);
    const float f1 = __uint_as_float(b1 << 16);
    const float r1 = a - f1;
    b2 = bf16_bits(r1);
    const float f2 = __uint_as_float(b2 << 16);
    const float r2 = r1 - f2;
    b3 = bf16_bits(r2);
    const float f3 = __uint_as_float(b3 << 16);
    ahat = (f1 + f2) + f3;
}
__device__ __forceinline__ void sts16(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((uint16_t)v) : "memory");
}

template <int QT, int MR>
__global__ void __launch_bounds__(kTThreads, 1) gemv_tc_kernel(const __grid_constant__ CUtensorMap tmw,
                                                               const TcParams p) {
    constexpr int B = QT_<QT>::BYTES;
    constexpr int G = QT == kQ6K ? 8 : 4;   // scale groups per 128-row half
    constexpr int GH = G;                   // scale groups per 128-value row piece
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32addr(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t *const gbase = smem_raw + (base - raw_base);
    const uint32_t b_half = (uint32_t)p.nc * 128u;
    const uint32_t b_stage = 2u * b_half;
    const uint32_t raw_stage = (uint32_t)(kTK * p.raw_slot);
    const uint32_t a_ring = base;
    const uint32_t b_ring = a_ring + (uint32_t)p.sa * kTAStage;
    const uint32_t r_ring = b_ring + (uint32_t)p.sa * b_stage;
    const uint32_t corr_s = (r_ring + (uint32_t)p.sr * raw_stage + 15u) & ~15u;
    constexpr int kCorrPerBuf = kNGrp * 4 * GH * MR;  // floats: [group][warp][scale group][m]
    const uint32_t bars = (corr_s + 2u * kCorrPerBuf * 4u + 7u) & ~7u;
    auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
    const int RF = 0, RE = kTMaxStages, AF = 2 * kTMaxStages, AE = 3 * kTMaxStages, CF = 4 * kTMaxStages,
              CE = CF + 2, KF = CF + 4, KE = CF + 6, DR = CF + 8;
    const uint32_t tmem_slot = bar(DR + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + (tmem_slot - base) + 4);
    float *corr_f = reinterpret_cast<float *>(gbase + (corr_s - base));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t total = (int64_t)p.tiles * p.ksteps;
    const int64_t f0 = (int64_t)blockIdx.x * p.per;
    const int64_t f1 = f0 + p.per < total ? f0 + p.per : total;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.sr; s++) {
            mbar_init(bar(RF + s), p.raw_tma ? 1 : 32);
            mbar_init(bar(RE + s), 4);  // one group's warps
        }
        for (int s = 0; s < p.sa; s++) {
            mbar_init(bar(AF + s), 4);
            mbar_init(bar(AE + s), 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(CF + s), 1);
            mbar_init(bar(CE + s), kTNEpi);
            mbar_init(bar(KF + s), kTNDec);
            mbar_init(bar(KE + s), kTNEpi);
        }
        mbar_init(bar(DR), 1);
        *abort_flag = 0;
        mbar_init_fence();
        if (p.raw_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmw) : "memory");
    }
    // B columns beyond the used ones are never written by the decode: zero them once
    {
        const uint32_t words = (uint32_t)p.sa * b_stage / 16u;
        for (uint32_t i = threadIdx.x; i < words; i += kTThreads)
            asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(b_ring + 16u * i), "r"(0u) : "memory");
    }
    if (warp == kTWMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = lds32(tmem_slot);

    auto wait = [&](uint32_t b, uint32_t parity, bool poll = false) -> bool {
        if (poll ? mbar_wait_spin(b, parity, kTWaitNs) : mbar_wait_bounded(b, parity, kTWaitNs)) return true;
        tc_set_status(kStatusTimeout);
        *abort_flag = 1;
        return false;
    };
    // value position of (k, 0) in the weight stream
    auto row_v = [&](int64_t k) -> int64_t { return k * p.rs + ((k * p.ld + p.n_base) & 255); };

    pdl_launch_dependents();

    if (warp == kTWRaw) {
        // ------------- raw super-blocks: one stage = 64 k rows of one tile -------------
        RingPos rp;
        for (int64_t fa = f0; fa < f1 && !*abort_flag;) {
            const int64_t t = fa / p.ksteps;
            const int64_t fb = (t + 1) * p.ksteps < f1 ? (t + 1) * p.ksteps : f1;
            const int64_t n0 = t * kTN;
            const int64_t nv = p.N - n0 < kTN ? p.N - n0 : kTN;
            bool ok = true;
            for (int64_t f = fa; f < fb; f++, rp.next((uint32_t)p.sr)) {
                const int ks = (int)(f - t * p.ksteps);
                const int s = (int)rp.idx;
                if (rp.uses >= (uint32_t)p.sr && !wait(bar(RE + s), rp.phase ^ 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t st_base = r_ring + (uint32_t)s * raw_stage;
                if (p.raw_tma) {
                    if (lane == 0) {
                        mbar_arrive_expect_tx(bar(RF + s), raw_stage);
                        // uint16 elements: the byte offset of the tile's first block, rounded down to 16
                        tma_load_2d(st_base, &tmw, (int)((((n0 >> 8) * B) & ~int64_t(15)) >> 1), ks * kTK,
                                    bar(RF + s));
                    }
                } else {
                    int64_t lo[2];
                    uint32_t nb[2];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int64_t k = (int64_t)ks * kTK + lane + 32 * h;
                        lo[h] = 0;
                        nb[h] = 0;
                        if (k < p.K) {
                            const int64_t v0 = row_v(k) + n0;
                            const int64_t blk0 = v0 >> 8, blk1 = (v0 + nv - 1) >> 8;
                            lo[h] = (blk0 * B) & ~int64_t(15);
                            nb[h] = (uint32_t)((blk1 + 1) * B - lo[h]);  // <= raw_slot
                        }
                    }
                    const uint32_t c = (uint32_t)lane * 16u;
#pragma unroll 4
                    for (int r = 0; r < kTK; r++) {
                        const int64_t a = __shfl_sync(0xffffffffu, r < 32 ? lo[0] : lo[1], r & 31);
                        const uint32_t n = __shfl_sync(0xffffffffu, r < 32 ? nb[0] : nb[1], r & 31);
                        if (c < n) {
                            const int64_t rem = p.w_bytes - (a + c);  // never reads past the end of w
                            cp_async16(st_base + (uint32_t)(r * p.raw_slot) + c, p.w + a + c,
                                       rem < 16 ? (uint32_t)rem : 16u);
                        }
                    }
                    cp_async_arrive_noinc(bar(RF + s));
                }
            }
            if (!ok) break;
            fa = fb;
        }
        const uint32_t it = rp.uses;
        for (int s = 0; s < p.sr && it > 0; s++) {
            const uint32_t uses = it / (uint32_t)p.sr + ((uint32_t)s < it % (uint32_t)p.sr ? 1u : 0u);
            if (uses > 0) mbar_wait_bounded(bar(RF + s), (uses - 1) & 1u, kTDrainNs);
        }
    } else if (warp == kTWMma) {
        // ------------- MMA issuer -------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, p.nc);
            const uint64_t da0 = smem_desc_sw128(a_ring, 1024u, 2048u);
            const uint64_t db0 = smem_desc_sw128(b_ring, 16u, 1024u);
            RingPos pa;
            uint32_t si = 0;
            for (int64_t fa = f0; fa < f1 && !*abort_flag; si++) {
                const int64_t t = fa / p.ksteps;
                const int64_t fb = (t + 1) * p.ksteps < f1 ? (t + 1) * p.ksteps : f1;
                const uint32_t tb = p.nbuf == 2 ? (si & 1u) : 0u, use = p.nbuf == 2 ? (si >> 1) : si;
                if (use > 0 && !wait(bar(CE + tb), (use - 1) & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t dt0 = tmem + tb * (uint32_t)p.acc_stride, dt1 = dt0 + (uint32_t)p.nc;
                bool ok = true;
                for (int64_t f = fa; f < fb; f++, pa.next((uint32_t)p.sa)) {
                    const int sa = (int)pa.idx;
                    if (!wait(bar(AF + sa), pa.phase, true)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint64_t da = da0 + (uint64_t)((uint32_t)(sa * kTAStage) >> 4);
                    const uint64_t db = db0 + (uint64_t)(((uint32_t)sa * b_stage) >> 4);
                    const uint32_t acc0 = f > fa ? 1u : 0u;
#pragma unroll
                    for (int kk = 0; kk < kTK / 16; kk++) {
                        const uint32_t acc = kk > 0 ? 1u : acc0;
                        umma_bf16(dt0, da + (uint64_t)(kk * 4096 >> 4), db + (uint64_t)(kk * 32 >> 4), idesc, acc);
                        umma_bf16(dt1, da + (uint64_t)((kTHalf + kk * 4096) >> 4),
                                  db + (uint64_t)((b_half + kk * 32) >> 4), idesc, acc);
                    }
                    umma_commit(bar(AE + sa));
                }
                if (!ok) break;
                umma_commit(bar(CF + tb));
                fa = fb;
            }
            umma_commit(bar(DR));
            mbar_wait_bounded(bar(DR), 0, kTDrainNs);
        }
    } else if (warp < kTWEpi) {
        // ------------- decode: raw half-block -> A tile rows, B entries, corrections -------------
        // Four groups of four warps; group g takes the CTA's stages j = g, g+4, ...
        // (so four stages are decoded at once and their latencies overlap).  A
        // thread takes one k row of one MMA half: 128 values of one block half.
        const int dw = warp - kTWDec;
        const int grp = dw >> 2, wq = dw & 3;
        const int h = wq >> 1;                 // MMA half of this thread's row piece
        const int kl = 32 * (wq & 1) + lane;   // k row within the stage
        const uint32_t a_base = (uint32_t)(h * kTHalf + (kl >> 3) * 2048 + (kl & 7) * 128);
        const uint32_t kb2 = 2u * (uint32_t)kl;
        auto b_off = [&](int c) -> uint32_t {
            return (uint32_t)h * b_half +
                   (uint32_t)((c >> 3) * 1024 + (c & 7) * 128 + ((((kb2 >> 4) ^ (uint32_t)(c & 7)) << 4) | (kb2 & 15u)));
        };
        const uint32_t slot_row = r_ring + (uint32_t)(kl * p.raw_slot);
        // ring positions of stage j = grp + 4i (sr, sa >= 4: at most one wrap per step)
        uint32_t ridx = (uint32_t)grp, rph = 0, aidx = (uint32_t)grp, aph = 0;
        int64_t j = grp;  // this group's next stage, counted from f0
        pdl_wait();       // x may come from the preceding kernel
        uint32_t si = 0;
        for (int64_t fa = f0; fa < f1 && !*abort_flag; si++) {
            const int64_t t = fa / p.ksteps;
            const int64_t fb = (t + 1) * p.ksteps < f1 ? (t + 1) * p.ksteps : f1;
            const int64_t n0 = t * kTN;
            const bool n_ok = n0 + 128 * h < p.N;
            const uint32_t x0b = (uint32_t)(((n0 >> 8) * B) & ~int64_t(15));  // TMA box start within a row
            float corr[MR][GH];
#pragma unroll
            for (int m = 0; m < MR; m++)
#pragma unroll
                for (int g = 0; g < GH; g++) corr[m][g] = 0.f;
            const int Ki = (int)p.K;
            bool ok = true;
            // x of the group's next stage is loaded one group step ahead
            float xn[MR];
            auto load_x = [&](int64_t jj, float (&dst)[MR]) {
                const int kx = (int)(f0 + jj - t * p.ksteps) * kTK + kl;
                const bool in = f0 + jj < fb && n_ok && kx < Ki;
#pragma unroll
                for (int m = 0; m < MR; m++) dst[m] = (in && m < p.M) ? __ldg(p.x + (int64_t)m * p.K + kx) : 0.f;
            };
            load_x(j, xn);
            for (; f0 + j < fb; j += kNGrp) {
                const int ks = (int)(f0 + j - t * p.ksteps);
                const int k = ks * kTK + kl;
                const bool valid = n_ok && k < Ki;
                float xv[MR];
#pragma unroll
                for (int m = 0; m < MR; m++) xv[m] = xn[m];
                load_x(j + kNGrp, xn);
                if (!wait(bar(RF + (int)ridx), rph, true)) {
                    ok = false;
                    break;
                }
                // the block half under this row piece, in the raw stage
                uint32_t blk = 0, hb = 0;
                if (valid) {
                    if (p.raw_tma) {
                        const uint32_t u0 = (((uint32_t)k * (uint32_t)p.ld + (uint32_t)p.n_base) & 255u) +
                                            (uint32_t)n0 + 128u * (uint32_t)h;
                        blk = slot_row + ridx * raw_stage + (u0 >> 8) * (uint32_t)B - x0b;
                        hb = (u0 >> 7) & 1u;
                    } else {
                        const int64_t V = row_v(k);
                        const int64_t v = V + n0 + 128 * h;
                        const int64_t lo = (((V + n0) >> 8) * B) & ~int64_t(15);
                        blk = slot_row + ridx * raw_stage + (uint32_t)((v >> 8) * B - lo);
                        hb = (uint32_t)((v >> 7) & 1);
                    }
                }
                uint32_t qw[16], aux[8];  // quants (16 words); Q4_K/Q5_K header + Q5_K high bits, or Q6_K qh
                uint32_t sw[2] = {0u, 0u};  // Q6_K: the 8 int8 group scales
                float d = 0.f, dmin = 0.f;
                if (valid) {
                    if constexpr (QT == kQ4K || QT == kQ5K) {
                        const uint4 hd = lds128(blk);
                        aux[0] = hd.x; aux[1] = hd.y; aux[2] = hd.z; aux[3] = hd.w;
                        const uint32_t qsa = blk + (QT == kQ4K ? 16u : 48u) + 64u * hb;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint4 v4 = lds128(qsa + 16u * i);
                            qw[4 * i] = v4.x; qw[4 * i + 1] = v4.y; qw[4 * i + 2] = v4.z; qw[4 * i + 3] = v4.w;
                        }
                        if constexpr (QT == kQ5K) {
                            const uint4 v4 = lds128(blk + 16u + 16u * hb);
                            aux[4] = v4.x; aux[5] = v4.y; aux[6] = v4.z; aux[7] = v4.w;
                        }
                    } else {
                        // 2-byte aligned block: aligned words and one funnel shift
                        const uint32_t shf = (blk & 3u) * 8u, b4 = blk & ~3u;
                        uint32_t prev = lds32(b4 + 64u * hb);
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const uint32_t nx = lds32(b4 + 64u * hb + 4u * (i + 1));
                            qw[i] = __funnelshift_r(prev, nx, shf);
                            prev = nx;
                        }
                        prev = lds32(b4 + 128u + 32u * hb);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const uint32_t nx = lds32(b4 + 128u + 32u * hb + 4u * (i + 1));
                            aux[i] = __funnelshift_r(prev, nx, shf);
                            prev = nx;
                        }
                        const uint32_t s0 = lds32(b4 + 192u + 8u * hb), s1 = lds32(b4 + 196u + 8u * hb),
                                       s2 = lds32(b4 + 200u + 8u * hb);
                        sw[0] = __funnelshift_r(s0, s1, shf);
                        sw[1] = __funnelshift_r(s1, s2, shf);
                        d = hw_f16_to_f32(lds16(blk + 208u));
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i++) qw[i] = 0u;
#pragma unroll
                    for (int i = 0; i < 8; i++) aux[i] = 0u;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(RE + (int)ridx));
                // per-group scales of this block half
                float sg[GH], mg[GH];
                if constexpr (QT == kQ4K || QT == kQ5K) {
                    d = hw_f16_to_f32(aux[0] & 0xFFFFu);
                    dmin = hw_f16_to_f32(aux[0] >> 16);
                    const uint32_t sc24 = hb ? __funnelshift_r(aux[1], aux[2], 24) : aux[1];
                    const uint32_t m24 = hb ? (aux[3] >> 8) : __funnelshift_r(aux[2], aux[3], 16);
#pragma unroll
                    for (int g = 0; g < GH; g++) {
                        sg[g] = d * (float)((sc24 >> (6 * g)) & 63u);
                        mg[g] = dmin * (float)((m24 >> (6 * g)) & 63u);
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < GH; g++) {
                        sg[g] = d * (float)(int)(int8_t)((sw[g >> 2] >> (8 * (g & 3))) & 0xFFu);
                        mg[g] = 0.f;
                    }
                }
                if (j >= p.sa && !wait(bar(AE + (int)aidx), aph ^ 1u, true)) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = a_ring + aidx * (uint32_t)kTAStage;
                // A: chunk cc holds values 8cc..8cc+7 of the half as bf16 pairs (v_j, v_j+4)
#pragma unroll
                for (int cc = 0; cc < 16; cc++) {
                    const uint32_t W = qw[cc];
                    uint32_t P[4];
                    if constexpr (QT == kQ6K) {
                        const uint32_t b0 = 2u * (uint32_t)(cc & 1);
                        const uint32_t Z = prmt(aux[cc >> 1], 0u, b0 | (4u << 4) | ((b0 + 1u) << 8) | (4u << 12)) << 4;
#pragma unroll
                        for (int jq = 0; jq < 4; jq++)
                            P[jq] = ((W >> (4 * jq)) & 0x000F000Fu) | 0x43004300u | ((Z >> (2 * jq)) & 0x00300030u);
                    } else {
                        uint32_t Y = 0;
                        if constexpr (QT == kQ5K) Y = ((aux[4 + (cc >> 2)] >> (8 * (cc & 3))) & 0xFFu) * 0x10010u;
#pragma unroll
                        for (int jq = 0; jq < 4; jq++) {
                            P[jq] = ((W >> (4 * jq)) & 0x000F000Fu) | 0x43004300u;
                            if constexpr (QT == kQ5K) P[jq] |= (Y >> jq) & 0x00100010u;
                        }
                    }
                    const uint32_t ao = a_base + (uint32_t)((cc >> 3) * 1024) + ((((uint32_t)cc & 7u) ^ ((uint32_t)kl & 7u)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_s + ao), "r"(P[0]), "r"(P[1]),
                                 "r"(P[2]), "r"(P[3])
                                 : "memory");
                }
                // B: per group and m, the product x * s split into three bf16 parts
                const uint32_t b_s = b_ring + aidx * b_stage;
#pragma unroll
                for (int m = 0; m < MR; m++) {
#pragma unroll
                    for (int g = 0; g < GH; g++) {
                        uint32_t b1, b2, b3;
                        float ahat;
                        split3(xv[m] * sg[g], b1, b2, b3, ahat);
                        if constexpr (QT == kQ6K) corr[m][g] = fmaf(160.f, ahat, corr[m][g]);
                        else corr[m][g] = fmaf(128.f, ahat, fmaf(xv[m], mg[g], corr[m][g]));
                        const int c = (m * G + g) * 3;
                        sts16(b_s + b_off(c), b1);
                        sts16(b_s + b_off(c + 1), b2);
                        sts16(b_s + b_off(c + 2), b3);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(AF + (int)aidx));
                ridx += kNGrp;
                if (ridx >= (uint32_t)p.sr) {
                    ridx -= (uint32_t)p.sr;
                    rph ^= 1u;
                }
                aidx += kNGrp;
                if (aidx >= (uint32_t)p.sa) {
                    aidx -= (uint32_t)p.sa;
                    aph ^= 1u;
                }
            }
            if (!ok) break;
            // the segment's corrections of this warp: all 32 lanes (k rows) in a
            // fixed butterfly order, one slot per (group, warp)
            const uint32_t kb = si & 1u;
            if (si >= 2 && !wait(bar(KE + kb), ((si >> 1) - 1) & 1u)) break;
#pragma unroll
            for (int m = 0; m < MR; m++) {
#pragma unroll
                for (int g = 0; g < GH; g++) {
                    float v = corr[m][g];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (lane == 0) corr_f[kb * kCorrPerBuf + ((grp * 4 + wq) * GH + g) * MR + m] = v;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(KF + kb));
            fa = fb;
        }
    } else {
        // ------------- epilogue: TMEM -> y (or the CTA's partials) -------------
        pdl_wait();  // y, the partials and the counters may be used by the preceding kernel
        const int q = warp & 3;  // TMEM lane quarter = 32-row unit of each half
        uint32_t si = 0;
        for (int64_t fa = f0; fa < f1 && !*abort_flag; si++) {
            const int64_t t = fa / p.ksteps;
            const int64_t fb = (t + 1) * p.ksteps < f1 ? (t + 1) * p.ksteps : f1;
            const int64_t n0 = t * kTN;
            const bool whole = fa == t * p.ksteps && fb == (t + 1) * p.ksteps;
            const uint32_t tb = p.nbuf == 2 ? (si & 1u) : 0u, use = p.nbuf == 2 ? (si >> 1) : si;
            if (!wait(bar(CF + tb), use & 1u)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            // parts of this lane's row: Q4_K/Q5_K 3 columns of unit q, Q6_K 6 (two groups)
            float part[MR][2][3];
#pragma unroll
            for (int m = 0; m < MR; m++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + tb * (uint32_t)p.acc_stride +
                                           (uint32_t)(hh * p.nc + (m * G + (QT == kQ6K ? 2 : 1) * q) * 3);
                    uint32_t r[8];
                    if constexpr (QT == kQ6K) {
                        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                                       "=r"(r[6]), "=r"(r[7])
                                     : "r"(taddr));
                    } else {
                        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                                     : "r"(taddr));
                        r[4] = r[5] = r[6] = r[7] = 0u;
                    }
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    const int o = (QT == kQ6K && lane >= 16) ? 3 : 0;  // second group of the unit
#pragma unroll
                    for (int tp = 0; tp < 3; tp++) part[m][hh][tp] = __uint_as_float(r[o + tp]);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(CE + tb));
            const uint32_t kb = si & 1u;
            if (!wait(bar(KF + kb), (si >> 1) & 1u)) break;
            float cs[MR][2];
            const int gq = QT == kQ6K ? 2 * q + (lane >= 16 ? 1 : 0) : q;  // scale group of this lane's row
#pragma unroll
            for (int m = 0; m < MR; m++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    float c = 0.f;
#pragma unroll
                    for (int gr = 0; gr < kNGrp; gr++)
#pragma unroll
                        for (int w2 = 0; w2 < 2; w2++)
                            c += corr_f[kb * kCorrPerBuf + ((gr * 4 + 2 * hh + w2) * GH + gq) * MR + m];
                    cs[m][hh] = c;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(KE + kb));
            // row lane of unit q holds value 8 * (lane / 8) + perm(lane % 8) of the unit
            const int nl = 32 * q + 8 * (lane >> 3) + ((lane & 7) >> 1) + 4 * (lane & 1);
            const int slot = si == 0 ? 0 : 1;
#pragma unroll
            for (int m = 0; m < MR; m++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const float v = ((part[m][hh][0] + part[m][hh][1]) + part[m][hh][2]) - cs[m][hh];
                    const int64_t n = n0 + 128 * hh + nl;
                    if (m < p.M && n < p.N) {
                        if (whole) p.y[(int64_t)m * p.y_ld + n] = v;
                        else p.partials[(((int64_t)blockIdx.x * 2 + slot) * MR + m) * kTN + 128 * hh + nl] = v;
                    }
                }
            }
            if (!whole) {
                // split tile: each epilogue warp counts itself in for its row
                // quarter (after its partial stores); the last CTA to arrive
                // for a quarter adds that quarter's partials in CTA order.  No
                // CTA-wide barrier: every wait here stays bounded.
                const int64_t cf = (t * p.ksteps) / p.per;
                const int64_t cl = ((t + 1) * p.ksteps - 1) / p.per;
                __threadfence();  // this lane's partials, before the warp's arrival is counted
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(p.counters + 4 * t + q, 1) == (int)(cl - cf);
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    const bool cf_slot1 = cf * p.per < t * p.ksteps;
                    float acc[MR][2];
#pragma unroll
                    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = 0.f;
                    constexpr int kBatch = MR >= 4 ? 2 : 4;  // partial rows in flight
                    for (int64_t c0 = cf; c0 <= cl; c0 += kBatch) {
                        float v[kBatch][MR][2];
#pragma unroll
                        for (int u = 0; u < kBatch; u++) {
                            const int64_t cta = c0 + u;
                            const int sl = (cta == cf && cf_slot1) ? 1 : 0;
                            const float *src = p.partials + (cta * 2 + sl) * MR * kTN + nl;
#pragma unroll
                            for (int m = 0; m < MR; m++)
#pragma unroll
                                for (int hh = 0; hh < 2; hh++)
                                    v[u][m][hh] = cta <= cl ? __ldcg(src + m * kTN + 128 * hh) : 0.f;
                        }
#pragma unroll
                        for (int u = 0; u < kBatch; u++)
#pragma unroll
                            for (int m = 0; m < MR; m++)
#pragma unroll
                                for (int hh = 0; hh < 2; hh++)
                                    if (c0 + u <= cl) acc[m][hh] += v[u][m][hh];
                    }
#pragma unroll
                    for (int m = 0; m < MR; m++)
#pragma unroll
                        for (int hh = 0; hh < 2; hh++) {
                            const int64_t n = n0 + 128 * hh + nl;
                            if (m < p.M && n < p.N) p.y[(int64_t)m * p.y_ld + n] = acc[m][hh];
                        }
                    __syncwarp();
                    if (lane == 0) atomicExch(p.counters + 4 * t + q, 0);
                }
            }
            fa = fb;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kTWMma) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols));
    }
}

// ------------------------------- host side -------------------------------
struct TcPlan {
    bool fits;
    int tiles, ksteps, per, grid;
    int sr, sa, raw_slot, raw_tma, nc, nbuf, tmem_cols;
    int64_t pitch;
    size_t smem, part_bytes;
};

static int tc_mr(int64_t M) { return M <= 1 ? 1 : M <= 2 ? 2 : 4; }

static TcPlan tc_plan(const GemvShape &s, const TcLayout &L, int sms) {
    TcPlan g{};
    const int B = s.qtype == kQ4K ? 144 : s.qtype == kQ5K ? 176 : 210;
    const int MR = tc_mr(s.M);
    const int G = s.qtype == kQ6K ? 8 : 4;
    g.tiles = (int)((s.N + kTN - 1) / kTN);
    g.ksteps = (int)((s.K + kTK - 1) / kTK);
    const int64_t total = (int64_t)g.tiles * g.ksteps;
    int64_t grid = std::min<int64_t>(total, sms);
    g.per = (int)((total + grid - 1) / grid);
    g.grid = (int)((total + g.per - 1) / g.per);
    g.nc = (MR * G * 3 + 15) / 16 * 16;
    g.nbuf = 4 * g.nc <= 512 ? 2 : 1;
    g.tmem_cols = 32;
    while (g.tmem_cols < g.nbuf * 2 * g.nc) g.tmem_cols <<= 1;
    // rows of the weight at a 16-byte byte pitch: 2D TMA stages (uint16 elements)
    const bool straddle = (L.ld & 255) != 0 || (L.n_base & 255) != 0;
    g.pitch = (L.rs % 256 == 0) ? L.rs / 256 * B : 0;
    g.raw_tma = g.pitch > 0 && g.pitch % 16 == 0;
    if (g.raw_tma) {
        const int lead = B % 16 == 0 ? 0 : 14;
        g.raw_slot = ((straddle ? 2 * B : B) + lead + 15) & ~15;
    } else {
        g.raw_slot = (2 * B + 15 + 15) & ~15;
    }
    const size_t a_st = kTAStage + 256 * (size_t)g.nc, r_st = (size_t)kTK * g.raw_slot;
    const size_t fixed = 1024 + 2 * (size_t)kNGrp * 4 * G * MR * 4 + 16 + 8 * (4 * kTMaxStages + 12) + 16;
    const size_t budget = 227 * 1024 - fixed;
    // four decode groups work on four stages at once: four A stages, and at
    // least four raw stages, grown while they fit
    g.sa = 4;
    g.sr = 4;
    while (g.sr < kTMaxStages && g.sa * a_st + (g.sr + 1) * r_st <= budget) g.sr++;
    g.fits = g.sa * a_st + g.sr * r_st <= budget;
    g.smem = fixed + g.sa * a_st + g.sr * r_st;
    g.part_bytes = ((size_t)g.grid * 2 * MR * kTN * 4 + 255) & ~size_t(255);
    return g;
}

// K >= 256: the factored form rounds x * s before the minimum is subtracted,
// so its error is bounded relative to sum_k |x| (|s q| + |mn|) rather than
// sum_k |x w|; the two differ only where a column's few terms cancel (s q ~
// mn), which short reductions can hit: those go to the CUDA-core kernel,
// which forms each weight before the product with x.
bool gemv_tc_supported(const GemvShape &s) {
    if (s.M < 1 || s.M > 4 || s.N % 32 != 0 || s.K < 256) return false;
    if (s.qtype == kQ6K && s.M > 2) return false;  // Q6_K's 8 groups x 3 parts x M columns: shared memory
    const int64_t tiles = (s.N + kTN - 1) / kTN;
    return 4 * tiles <= (int64_t)(kWorkspaceCounterHead / 4);  // a counter per tile quarter
}

bool gemv_tc_fits(const GemvShape &s, const TcLayout &L, int device) {
    return gemv_tc_supported(s) && tc_plan(s, L, device_sm_count(device)).fits;
}

size_t gemv_tc_workspace_bytes(const GemvShape &s, const TcLayout &L, int device) {
    if (!gemv_tc_supported(s)) return 0;
    return kWorkspaceCounterHead + tc_plan(s, L, device_sm_count(device)).part_bytes;
}

template <int QT, int MR>
static cudaError_t launch_tc(const CUtensorMap &tm, const TcParams &tp, const TcPlan &g, cudaStream_t st) {
    auto kern = gemv_tc_kernel<QT, MR>;
    cudaError_t e = kernel_smem((const void *)kern, g.smem, false);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)g.grid);
    cfg.blockDim = dim3(kTThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tm, tp);
}

template <int QT>
static cudaError_t dispatch_tc(int mr, const CUtensorMap &tm, const TcParams &tp, const TcPlan &g, cudaStream_t st) {
    switch (mr) {
    case 1: return launch_tc<QT, 1>(tm, tp, g, st);
    case 2: return launch_tc<QT, 2>(tm, tp, g, st);
    default:
        if constexpr (QT == kQ6K) return cudaErrorInvalidValue;  // Q6_K serves M <= 2 (gemv_tc_supported)
        else return launch_tc<QT, 4>(tm, tp, g, st);
    }
}

int gemv_tc_launch(const GemvShape &s, const TcLayout &L, const void *w, int64_t w_bytes, const float *x, float *y,
                   int64_t y_ld, void *ws, size_t ws_bytes, cudaStream_t stream, int device) {
    if (!gemv_tc_supported(s)) {
        set_error("the tensor-core GEMV serves 1 <= M <= 4 and N %% 32 == 0");
        return 2;
    }
    const int sms = device_sm_count(device);
    const TcPlan g = tc_plan(s, L, sms);
    if (!g.fits) {
        set_error("the tensor-core GEMV's stages do not fit in shared memory for this shape");
        return 2;
    }
    const size_t need = kWorkspaceCounterHead + g.part_bytes;
    if (ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) {
        set_error("the tensor-core GEMV needs a 256-byte aligned workspace of %zu bytes (got %zu)", need, ws_bytes);
        return 4;
    }
    CUtensorMap tm;
    memset(&tm, 0, sizeof(tm));
    if (g.raw_tma) {
        EncodeTiledFn enc = encode_tiled_fn();
        if (!enc) {
            set_error("cuTensorMapEncodeTiled is not available from the driver");
            return 5;
        }
        const cuuint64_t dims[2] = {(cuuint64_t)(g.pitch / 2), (cuuint64_t)s.K};
        const cuuint64_t strides[1] = {(cuuint64_t)g.pitch};
        const cuuint32_t box[2] = {(cuuint32_t)(g.raw_slot / 2), (cuuint32_t)kTK};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("cuTensorMapEncodeTiled (tensor-core GEMV weights) failed (%d)", (int)r);
            return 5;
        }
    }
    TcParams tp{};
    tp.w = static_cast<const uint8_t *>(w);
    tp.w_bytes = w_bytes;
    tp.rs = L.rs;
    tp.ld = L.ld;
    tp.n_base = L.n_base;
    tp.pitch = g.pitch;
    tp.x = x;
    tp.y = y;
    tp.y_ld = y_ld;
    tp.K = s.K;
    tp.N = s.N;
    tp.M = (int)s.M;
    tp.tiles = g.tiles;
    tp.ksteps = g.ksteps;
    tp.per = g.per;
    tp.grid = g.grid;
    tp.sr = g.sr;
    tp.sa = g.sa;
    tp.raw_slot = g.raw_slot;
    tp.raw_tma = g.raw_tma;
    tp.nc = g.nc;
    tp.nbuf = g.nbuf;
    tp.tmem_cols = g.tmem_cols;
    tp.acc_stride = 2 * g.nc;
    tp.counters = static_cast<int *>(ws);
    tp.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kWorkspaceCounterHead);
    const int mr = tc_mr(s.M);
    cudaError_t e;
    switch (s.qtype) {
    case kQ4K: e = dispatch_tc<kQ4K>(mr, tm, tp, g, stream); break;
    case kQ5K: e = dispatch_tc<kQ5K>(mr, tm, tp, g, stream); break;
    default: e = dispatch_tc<kQ6K>(mr, tm, tp, g, stream); break;
    }
    if (e != cudaSuccess) {
        set_error("tensor-core GEMV launch failed: %s", cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int gemv_tc_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
    return v;
}

}  // namespace vkq
