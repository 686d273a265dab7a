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
// that the operand built on the fly (the dequantized weight) is the MMA's A
// (M = 128 rows of n) and X is the MMA's B (N = bm columns of m):
//  * raw ring: the super-blocks under a 128 n x 64 k tile (one or two blocks
//    per k row) are streamed from HBM into shared memory by one producer warp,
//    several stages deep: as one 2D TMA tile copy per stage when the k rows
//    have a 16-byte byte pitch (N % 256 == 0 and N/256 * B % 16 == 0), else
//    with 16-byte cp.async, consecutive lanes on consecutive bytes of a row
//    (one bulk copy per 144..420-byte row would be limited by the bulk-copy
//    request rate, ~40 ns per request per SM);
//  * A ring: sixteen dequant warps turn a raw stage into the bf16 A tile, written
//    straight into the MN-major 128-byte-swizzled layout (atoms of 64 n x 8 k,
//    1024 bytes; the two 64-n halves 1024 B apart, k groups 2048 B apart);
//  * B ring: X is converted to bf16 once per call (workspace) and loaded by
//    TMA as [bm rows of m] x [64 k] with the 128-byte swizzle (K-major, 8-row
//    atoms, SBO 1024 B).  No multicast;
//  * D: fp32 in TMEM, 128 lanes (n) x bm columns (m), double-buffered so the
//    epilogue warps drain tile i to Y while the MMA warp accumulates tile i+1.
// Wide units (M > 256): 128 n x 2 bm m, one 16 KB A tile per stage read by
// both MMAs (one per m half, B = the two X tiles), so each weight tile is
// dequantized once for up to 512 rows of m instead of once per 256; each
// dequant thread decodes half a 32-value unit.  Prefill 512 x 2048 x 11008:
// 40 -> 35 us; 2048 x 5120 x 27648: 1.24 PFLOP/s.
// The grid is persistent (at most one CTA per SM); work units are
// (n tile, m tile, k split) taken round-robin.  When the output tiles alone
// cannot fill the machine (narrow N), K is split and the partial products go
// to a workspace that a second kernel adds up in split order (deterministic).
// Warp roles (736 threads): 0 raw-weight producer, 1 X TMA producer, 2 TMEM
// owner + MMA issuer (one thread), 3..18 dequant (one 32-value unit per
// thread per k step; four warps per scheduler hide the decode's latency),
// 19..22 epilogue (warp w reads TMEM lanes 32*(w%4)..+31).  Every mbarrier wait is bounded; a wait that runs
// out sets the device status word and an abort flag that ends every role's
// loop, copies in flight are waited for (bounded) and TMEM is always released.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "kq_device.cuh"
#include "umma.cuh"
#include "vkq_internal.h"

namespace vkq {

static __device__ int g_gemm_status;

constexpr int kGBN = 256;                     // n per tile: one super-block per k row
constexpr int kMmaM = 128;                    // n rows per MMA (two MMAs per tile and 16-k step)
constexpr int kGBK = 64;                      // k per stage: one 128-byte swizzle row of bf16
constexpr int kAHalf = kMmaM * kGBK * 2;      // 16 KB: the A operand of one MMA
constexpr int kAStage = 2 * kAHalf;           // 32 KB
constexpr int kWRaw = 0, kWX = 1, kWMma = 2, kWDeq = 3, kNDeq = 16, kWEpi = 19, kNEpi = 4;
constexpr int kGThreads = (kWEpi + kNEpi) * 32;  // 736
constexpr uint64_t kGWaitNs = 2000000000ull;     // bounded waits: 2 s
constexpr uint64_t kDrainNs = 20000000ull;       // waits for copies in flight at teardown: 20 ms
constexpr int kMaxStages = 8;

struct GemmParams {
    const uint8_t *w;
    int64_t w_bytes;    // valid bytes of w (copies never read past them)
    float *y;           // Y [M][N], or partials [splits][M][N] when splits > 1
    int64_t K, N, M;
    int bm;             // m per tile = MMA N (multiple of 16, <= 256)
    int m_tiles, splits, units;
    int ksteps, kper;   // k steps in all, per split
    int sr, sa, sb;     // raw / A / B ring depths
    int raw_slot;       // bytes per raw row slot (multiple of 16)
    int raw_tma;        // raw stages are 2D tile copies (k rows with a 16-byte pitch)
    int tmem_cols, acc_stride;
    int nbuf;           // TMEM accumulator buffers (2: the epilogue overlaps the next unit)
    int wide;           // units of 128 n x 2*bm m (one dequantized A tile for both MMA halves)
};

__device__ __forceinline__ void g_set_status(int c) { atomicExch(&g_gemm_status, c); }

// A pair of fp32 values rounded to a bf16 pair.
__device__ __forceinline__ uint32_t pair_bf16(float2 w2) { return bf16x2(w2.x, w2.y); }

// Decode one unit into 32 values, rounded to bf16 pairs (16 words).  The
// values come out of the packed bytes as in the fp32 GEMV: nibbles of even
// and odd values are merged into byte lanes E and O, and a byte permute moves
// each quant q into a word of its own, which is used as it is as an fma
// operand: read as a float it is the subnormal q * 2^-149, so with the scale
// pre-multiplied by 2^100 one packed fma gives w * 2^-49 with the single
// rounding of the unscaled fma (every term stays normal: |d*sc| < 2^24).
// Q4_K/Q5_K: w = fma(d*sc, q, -dmin*m), equal to the reference's
// (d*sc)*q - dmin*m because (d*sc)*q is exact; Q6_K: w = (d*s) * (q - 32)
// as fma(d*s, q, -32*d*s).  The 2^-49 is undone by X, which is converted to
// bf16 times 2^49 (x_to_bf16_kernel): every product, and so Y, is unchanged.
constexpr float kWScale = 0x1p100f;  // on d*sc, d*s
constexpr float kWDown = 0x1p-49f;   // w comes out times this
constexpr float kXScale = 0x1p49f;   // X goes into bf16 times this

template <int J>
__device__ __forceinline__ float2 int_pair(uint32_t E, uint32_t O) {
    return make_float2(__uint_as_float(prmt(E, 0u, 0x4440u | J)), __uint_as_float(prmt(O, 0u, 0x4440u | J)));
}

// Moves the second 16 values of a loaded unit to where decode_unit_bf16
// reads the first 16 (quant words, Q5_K fifth bits, Q6_K high bits and
// 16-value scale), so that decode_unit_bf16<QT, 2> yields that half.
template <int QT>
__device__ __forceinline__ void shift_half(RawUnit &u) {
    if constexpr (QT == kQ4K || QT == kQ5K) {
        u.v[4] = u.v[6];
        u.v[5] = u.v[7];
        if constexpr (QT == kQ5K) u.v[8] >>= 16;
    } else {
        u.v[0] = u.v[2];
        u.v[1] = u.v[3];
        u.v[2] = u.v[4];
        u.v[5] = u.v[6];
        u.v[6] = u.v[7];
        u.v[8] = (u.v[8] & 0xFFFF0000u) | ((u.v[8] >> 8) & 0xFFu);
    }
}

// Decodes the first 8 * NC values of a unit (NC = 4: all 32) into 4 * NC
// bf16 pairs.
template <int QT, int NC = 4>
__device__ __forceinline__ void decode_unit_bf16(const RawUnit &u, uint32_t (&out)[4 * NC]) {
    if (!u.valid) {
#pragma unroll
        for (int i = 0; i < 4 * NC; i++) out[i] = 0u;
        return;
    }
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const float d = hw_f16_to_f32(u.v[0] & 0xFFFFu), dmin = hw_f16_to_f32(u.v[0] >> 16);
        const int sb = (int)(u.within >> 5);
        const uint32_t sc24 = sb < 4 ? u.v[1] : __funnelshift_r(u.v[1], u.v[2], 24);
        const uint32_t m24 = sb < 4 ? __funnelshift_r(u.v[2], u.v[3], 16) : (u.v[3] >> 8);
        const uint32_t sh = 6u * (sb & 3);
        const float ds = (d * kWScale) * (float)((sc24 >> sh) & 63u);
        const float ndm = (dmin * -kWDown) * (float)((m24 >> sh) & 63u);
        const float2 s2 = make_float2(ds, ds), nm2 = make_float2(ndm, ndm);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            uint32_t E = u.v[4 + c] & 0x0F0F0F0Fu;
            uint32_t O = (u.v[4 + c] >> 4) & 0x0F0F0F0Fu;
            if constexpr (QT == kQ5K) {
                // bit i of hb is the fifth bit of value 8c+i; bits 0,2,4,6
                // (and 1,3,5,7) go to bit 4 of byte lanes 0..3
                const uint32_t hb = (u.v[8] >> (8 * c)) & 0xFFu;
                E |= ((hb & 0x55u) * 0x410410u) & 0x10101010u;
                O |= (((hb >> 1) & 0x55u) * 0x410410u) & 0x10101010u;
            }
            out[4 * c + 0] = pair_bf16(f2fma(s2, int_pair<0>(E, O), nm2));
            out[4 * c + 1] = pair_bf16(f2fma(s2, int_pair<1>(E, O), nm2));
            out[4 * c + 2] = pair_bf16(f2fma(s2, int_pair<2>(E, O), nm2));
            out[4 * c + 3] = pair_bf16(f2fma(s2, int_pair<3>(E, O), nm2));
        }
    } else {
        uint32_t ql[4], qh[2], qhs[2];
#pragma unroll
        for (int i = 0; i < 4; i++) ql[i] = __funnelshift_r(u.v[i], u.v[i + 1], u.shf);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            qh[i] = __funnelshift_r(u.v[5 + i], u.v[6 + i], u.shf);
            qhs[i] = qh[i] >> 4;
        }
        const float d = hw_f16_to_f32(u.v[8] >> 16) * kWScale;
        const float ds0 = d * (float)(int)(int8_t)(u.v[8] & 0xFFu);
        const float ds1 = d * (float)(int)(int8_t)((u.v[8] >> 8) & 0xFFu);
        // -32 * d*s * 2^-49 = (d*s * 2^100) * -2^-144, exact
        const float o0 = ds0 * -0x1p-144f, o1 = ds1 * -0x1p-144f;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            // byte lane j of X = nibble j of the chunk's 16 qh bits
            //                  = (hi2 of value 2j+1) << 2 | (hi2 of value 2j)
            const uint32_t X = prmt(qh[c >> 1], qhs[c >> 1], (c & 1) ? 0x7362u : 0x5140u) & 0x0F0F0F0Fu;
            const uint32_t E = (ql[c] & 0x0F0F0F0Fu) | ((X & 0x03030303u) << 4);
            const uint32_t O = ((ql[c] >> 4) & 0x0F0F0F0Fu) | ((X << 2) & 0x30303030u);
            const float2 s2 = c < 2 ? make_float2(ds0, ds0) : make_float2(ds1, ds1);
            const float2 o2 = c < 2 ? make_float2(o0, o0) : make_float2(o1, o1);
            out[4 * c + 0] = pair_bf16(f2fma(s2, int_pair<0>(E, O), o2));
            out[4 * c + 1] = pair_bf16(f2fma(s2, int_pair<1>(E, O), o2));
            out[4 * c + 2] = pair_bf16(f2fma(s2, int_pair<2>(E, O), o2));
            out[4 * c + 3] = pair_bf16(f2fma(s2, int_pair<3>(E, O), o2));
        }
    }
}

// Work unit u -> (n tile, m tile, k split); units of one n tile are adjacent
// so that CTAs running at the same time share the weight rows in L2.
struct Unit {
    int64_t n0;
    int m0;
    int kb, ke;  // k steps [kb, ke)
    int split;
};
__device__ __forceinline__ Unit unit_of(const GemmParams &p, int u) {
    Unit r;
    const int split = u % p.splits;
    const int tile = u / p.splits;
    r.n0 = (int64_t)(tile / p.m_tiles) * (p.wide ? kMmaM : kGBN);
    r.m0 = (tile % p.m_tiles) * (p.wide ? 2 * p.bm : p.bm);
    r.kb = split * p.kper;
    r.ke = min(r.kb + p.kper, p.ksteps);
    r.split = split;
    return r;
}

// WIDE: a unit is 128 n x 2 bm m; the A stage is one MMA operand (16 KB), the
// B stage two X tiles (m0 and m0 + bm), and both MMAs of a 16-k step read the
// same A (each weight tile is dequantized once for 2 bm rows of m).
template <int QT, bool WIDE>
__global__ void __launch_bounds__(kGThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmx,
                                                            const __grid_constant__ CUtensorMap tmw,
                                                            const GemmParams p) {
    constexpr int B = QT_<QT>::BYTES;
    constexpr int kA = WIDE ? kAHalf : kAStage;  // bytes of an A stage
    constexpr int kNU = WIDE ? kMmaM : kGBN;     // n per unit
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32addr(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t *const gbase = smem_raw + (base - raw_base);  // generic pointer to `base`
    const uint32_t b_tile = (uint32_t)(p.bm * 128);       // one X tile: bm rows of 64 k
    const uint32_t b_stage = WIDE ? 2u * b_tile : b_tile;
    const uint32_t raw_stage = (uint32_t)(kGBK * p.raw_slot);
    const uint32_t a_ring = base;                                    // sa x kA
    const uint32_t b_ring = a_ring + (uint32_t)(p.sa * kA);          // sb x b_stage
    const uint32_t r_ring = b_ring + (uint32_t)p.sb * b_stage;       // sr x 64*raw_slot
    const uint32_t bars = r_ring + (uint32_t)p.sr * raw_stage;
    auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
    // barrier indices
    const int RF = 0, RE = kMaxStages, AF = 2 * kMaxStages, AE = 3 * kMaxStages, BF = 4 * kMaxStages,
              BE = 5 * kMaxStages, CF = 6 * kMaxStages, CE = CF + 2, DR = CF + 4;
    const uint32_t tmem_slot = bar(DR + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + (tmem_slot - base) + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.sr; s++) {
            mbar_init(bar(RF + s), p.raw_tma ? 1 : 32);  // TMA expect_tx, or one cp.async arrival per lane
            mbar_init(bar(RE + s), kNDeq);  // one arrival per dequant warp
        }
        for (int s = 0; s < p.sa; s++) {
            mbar_init(bar(AF + s), kNDeq);
            mbar_init(bar(AE + s), 1);  // tcgen05.commit
        }
        for (int s = 0; s < p.sb; s++) {
            mbar_init(bar(BF + s), 1);  // TMA expect_tx
            mbar_init(bar(BE + s), 1);  // tcgen05.commit
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(CF + s), 1);      // tcgen05.commit after a unit's last MMA
            mbar_init(bar(CE + s), kNEpi);  // one arrival per epilogue warp
        }
        mbar_init(bar(DR), 1);
        *abort_flag = 0;
        mbar_init_fence();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
        if (p.raw_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmw) : "memory");
    }
    if (warp == kWMma) {  // TMEM allocation (whole warp)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                     "r"(p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = lds32(tmem_slot);

    // A wait that runs out records the timeout and stops every role.  Waits
    // on the per-step critical path (dequant and MMA) poll; the others let
    // the thread sleep so that they take no issue slots from the dequant warps.
    auto wait = [&](uint32_t b, uint32_t parity, bool poll = false) -> bool {
        if (poll ? mbar_wait_spin(b, parity, kGWaitNs) : mbar_wait_bounded(b, parity, kGWaitNs)) return true;
        g_set_status(kStatusTimeout);
        *abort_flag = 1;
        return false;
    };

    // Drains the TMEM accumulator of unit `un` (buffer ab) to Y, or to the
    // split's partials: 16-column chunks of both MMA halves, chunk ci taken by
    // the warp of rank ci % nrank among the warps reading lane quarter q.
    auto drain = [&](const Unit &un, uint32_t ab, int q, int rank, int nrank) {
        float *yb = p.y + (int64_t)un.split * p.M * p.N;
        const int nch = (p.bm + 15) / 16;  // 16-column chunks per MMA half
        for (int ci = rank; ci < 2 * nch; ci += nrank) {
            const int h = ci >= nch ? 1 : 0, c = 16 * (ci - h * nch);
            uint32_t r[16];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + ab * (uint32_t)p.acc_stride +
                                   (uint32_t)(h * p.bm + c);
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            // accumulator half h: n rows 128h.. (or, WIDE, m rows bm*h..)
            const int64_t n = un.n0 + (WIDE ? 0 : kMmaM * h) + 32 * q + lane;
            const int64_t mb = un.m0 + (WIDE ? h * p.bm : 0) + c;
            const int mv = (int)min((int64_t)16, p.M - mb);
            if (n < p.N && mv > 0) {
                float *yp = yb + mb * p.N + n;  // walks down the m rows of this column
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (j < mv) *yp = __uint_as_float(r[j]);
                    yp += p.N;
                }
            }
        }
    };

    pdl_launch_dependents();

    if (warp == kWRaw) {
        // ------------- raw weight producer: two k rows per lane per stage -------------
        // weights do not depend on the preceding kernel: no griddepcontrol.wait
        RingPos rp;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
            const Unit un = unit_of(p, u);
            const int64_t nv = min((int64_t)kNU, p.N - un.n0);
            bool ok = true;
            for (int ks = un.kb; ks < un.ke; ks++, rp.next((uint32_t)p.sr)) {
                const int s = (int)rp.idx;
                if (rp.uses >= (uint32_t)p.sr && !wait(bar(RE + s), rp.phase ^ 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t st_base = r_ring + (uint32_t)s * raw_stage;
                if (p.raw_tma) {
                    // rows of k have a 16-byte pitch: one 2D tile copy of 64 rows x raw_slot bytes
                    if (lane == 0) {
                        mbar_arrive_expect_tx(bar(RF + s), raw_stage);
                        tma_load_2d(st_base, &tmw, (int)(((un.n0 >> 8) * B) & ~int64_t(15)), ks * kGBK, bar(RF + s));
                    }
                } else {
                    // lane l owns the byte ranges of rows l and l + 32; each row is
                    // then copied by consecutive lanes (16 bytes each, coalesced)
                    int64_t lo[2];
                    uint32_t nb[2];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int64_t k = (int64_t)ks * kGBK + lane + 32 * h;
                        lo[h] = 0;
                        nb[h] = 0;
                        if (k < p.K) {
                            const int64_t v0 = k * p.N + un.n0;
                            const int64_t blk0 = v0 >> 8, blk1 = (v0 + nv - 1) >> 8;
                            lo[h] = (blk0 * B) & ~int64_t(15);
                            nb[h] = (uint32_t)((blk1 + 1) * B - lo[h]);  // <= raw_slot <= 32 * 16
                        }
                    }
                    const uint32_t c = (uint32_t)lane * 16u;
#pragma unroll 4
                    for (int r = 0; r < kGBK; r++) {
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
        }
        // copies still in flight land before the CTA exits
        const uint32_t it = rp.uses;
        for (int s = 0; s < p.sr && it > 0; s++) {
            const uint32_t uses = it / (uint32_t)p.sr + ((uint32_t)s < it % (uint32_t)p.sr ? 1u : 0u);
            if (uses > 0) mbar_wait_bounded(bar(RF + s), (uses - 1) & 1u, kDrainNs);
        }
    } else if (warp == kWX) {
        // ------------- X producer: TMA tiles of bf16 X -------------
        if (lane == 0) {
            RingPos rp;
            pdl_wait();  // the bf16 copy of X comes from the preceding kernel
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                const Unit un = unit_of(p, u);
                bool ok = true;
                for (int ks = un.kb; ks < un.ke; ks++, rp.next((uint32_t)p.sb)) {
                    const int s = (int)rp.idx;
                    if (rp.uses >= (uint32_t)p.sb && !wait(bar(BE + s), rp.phase ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(BF + s), b_stage);
                    tma_load_2d(b_ring + (uint32_t)s * b_stage, &tmx, ks * kGBK, un.m0, bar(BF + s));
                    // the second m half (rows past M read as zeros)
                    if (WIDE)
                        tma_load_2d(b_ring + (uint32_t)s * b_stage + b_tile, &tmx, ks * kGBK, un.m0 + p.bm,
                                    bar(BF + s));
                }
                if (!ok) break;
            }
            const uint32_t it = rp.uses;
            for (int s = 0; s < p.sb && it > 0; s++) {
                const uint32_t uses = it / (uint32_t)p.sb + ((uint32_t)s < it % (uint32_t)p.sb ? 1u : 0u);
                if (uses > 0) mbar_wait_bounded(bar(BF + s), (uses - 1) & 1u, kDrainNs);
            }
        }
    } else if (warp == kWMma) {
        // ------------- MMA issuer -------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(kMmaM, p.bm);
            // Descriptors of stage 0; a stage, a 16-k step or an MMA half is
            // reached by adding (byte offset >> 4) to the start-address field
            // (bits 0..13, no carry: shared addresses stay below 256 KB).
            const uint64_t da0 = smem_desc_sw128(a_ring, 1024u, 2048u);
            const uint64_t db0 = smem_desc_sw128(b_ring, 16u, 1024u);
            RingPos pa, pb;
            uint32_t lu = 0;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, lu++) {
                const Unit un = unit_of(p, u);
                const uint32_t ab = p.nbuf == 2 ? (lu & 1u) : 0u, use = p.nbuf == 2 ? (lu >> 1) : lu;
                if (use > 0 && !wait(bar(CE + ab), (use - 1) & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t dt0 = tmem + ab * (uint32_t)p.acc_stride, dt1 = dt0 + (uint32_t)p.bm;
                bool ok = true;
                for (int ks = un.kb; ks < un.ke; ks++, pa.next((uint32_t)p.sa), pb.next((uint32_t)p.sb)) {
                    const int sa = (int)pa.idx, sb = (int)pb.idx;
                    if (!wait(bar(AF + sa), pa.phase, true) || !wait(bar(BF + sb), pb.phase, true)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint64_t da = da0 + (uint64_t)((uint32_t)(sa * kA) >> 4);
                    const uint64_t db = db0 + (uint64_t)(((uint32_t)sb * b_stage) >> 4);
                    const uint32_t acc0 = ks > un.kb ? 1u : 0u;
                    // A half h (n 128h..128h+127): two k groups of 8 per 16-k step
                    // (2048 B apart), 64-n halves 1024 B apart.  B: K-major, 16 k =
                    // 32 bytes into each 128-byte row, 8-row atoms 1024 B apart.
                    // WIDE: one A, and the second MMA takes the second X tile.
                    const uint32_t a1 = WIDE ? 0u : (uint32_t)kAHalf, b1 = WIDE ? b_tile : 0u;
#pragma unroll
                    for (int kk = 0; kk < kGBK / 16; kk++) {
                        const uint32_t acc = kk == 0 ? acc0 : 1u;
                        umma_bf16(dt0, da + (uint64_t)(kk * 4096 >> 4), db + (uint64_t)(kk * 32 >> 4), idesc, acc);
                        umma_bf16(dt1, da + (uint64_t)((a1 + kk * 4096) >> 4), db + (uint64_t)((b1 + kk * 32) >> 4),
                                  idesc, acc);
                    }
                    umma_commit(bar(AE + sa));  // frees the stages once these MMAs have read them
                    umma_commit(bar(BE + sb));
                }
                if (!ok) break;
                umma_commit(bar(CF + ab));
            }
            // every MMA issued has completed before TMEM is released
            umma_commit(bar(DR));
            mbar_wait_bounded(bar(DR), 0, kDrainNs);
        }
    } else if (warp < kWEpi) {
        // ------------- dequant warps: raw stage -> bf16 A tile -------------
        // WIDE: 128 n x 64 k per stage, half a 32-value unit per thread
        constexpr int NC = WIDE ? 2 : 4;                                      // 16-byte A chunks per unit
        constexpr int UPT = WIDE ? 1 : kGBK * (kGBN / 32) / (kNDeq * 32);  // units per thread per stage
        const int dt = threadIdx.x - kWDeq * 32;
        // unit j of the thread in every stage: uu = dt + j * 32 * kNDeq is k row
        // 8 * (uu / 64) + uu % 8 and 32 n starting at 32 * ((uu / 8) % 8)
        // (WIDE: the half (uu / 8) % 2 of the 32 n starting at 32 * ((uu / 16) % 4));
        // the 8 lanes of a shared-memory phase take the 8 k rows of one swizzle
        // atom, so their 16-byte A stores land in 8 different bank groups
        int kl[UPT], c8[UPT], hf[UPT];
        uint32_t a_off[UPT][NC];  // the unit's 16-byte chunks within an A stage
#pragma unroll
        for (int j = 0; j < UPT; j++) {
            const int uu = dt + j * 32 * kNDeq;
            kl[j] = 8 * (uu >> 6) + (uu & 7);
            c8[j] = WIDE ? (uu >> 4) & 3 : (uu >> 3) & 7;
            hf[j] = WIDE ? (uu >> 3) & 1 : 0;
            const int h = WIDE ? 0 : c8[j] >> 2, c32 = c8[j] & 3, g = kl[j] >> 3, kin = kl[j] & 7;
#pragma unroll
            for (int c4 = 0; c4 < NC; c4++) {
                const int nl = 32 * c32 + 16 * hf[j] + 8 * c4;  // first n of the chunk within the MMA half
                const int hh = nl >> 6, c = (nl & 63) >> 3;
                a_off[j][c4] = (uint32_t)(h * kAHalf + (g * 2 + hh) * 1024 + kin * 128 + ((c ^ kin) << 4));
            }
        }
        RingPos pr, pa;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
            const Unit un = unit_of(p, u);
            bool n_ok[UPT];
            uint32_t tma_off[UPT];
#pragma unroll
            for (int j = 0; j < UPT; j++) {
                n_ok[j] = un.n0 + 32 * c8[j] < p.N;
                // TMA stages: one block per k row at the row's slot plus the block's lead
                tma_off[j] = (uint32_t)(kl[j] * p.raw_slot) + (uint32_t)(((un.n0 >> 8) * B) & 15);
            }
            bool ok = true;
            for (int ks = un.kb; ks < un.ke; ks++, pr.next((uint32_t)p.sr), pa.next((uint32_t)p.sa)) {
                const int sr = (int)pr.idx, sa = (int)pa.idx;
                if (!wait(bar(RF + sr), pr.phase, true)) {
                    ok = false;
                    break;
                }
                const uint32_t st_r = r_ring + (uint32_t)sr * raw_stage;
                RawUnit ru[UPT];
#pragma unroll
                for (int j = 0; j < UPT; j++) {
                    const int64_t k = (int64_t)ks * kGBK + kl[j];
                    const bool valid = n_ok[j] && k < p.K;
                    uint32_t blk = 0, within = 0;
                    if (valid) {
                        if (p.raw_tma) {
                            blk = st_r + tma_off[j];
                            within = (uint32_t)(un.n0 & 255) + 32u * (uint32_t)c8[j];
                        } else {
                            const int64_t v0 = k * p.N + un.n0;
                            const int64_t blk0 = v0 >> 8;
                            const int64_t vi = v0 + 32 * c8[j];
                            const uint32_t lead = (uint32_t)((blk0 * B) & 15);
                            blk = st_r + (uint32_t)(kl[j] * p.raw_slot) + lead + (uint32_t)((vi >> 8) - blk0) * B;
                            within = (uint32_t)(vi & 255);
                        }
                    }
                    load_unit<QT>(blk, within, valid, ru[j]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(RE + sr));
                uint32_t wv[UPT][4 * NC];
#pragma unroll
                for (int j = 0; j < UPT; j++) {
                    if (WIDE && hf[j]) shift_half<QT>(ru[j]);
                    decode_unit_bf16<QT, NC>(ru[j], wv[j]);  // before the wait: overlaps the MMAs still reading the stage
                }
                if (pa.uses >= (uint32_t)p.sa && !wait(bar(AE + sa), pa.phase ^ 1u, true)) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = a_ring + (uint32_t)(sa * kA);
#pragma unroll
                for (int j = 0; j < UPT; j++)
#pragma unroll
                    for (int c4 = 0; c4 < NC; c4++)
                        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a_s + a_off[j][c4]),
                                     "r"(wv[j][4 * c4]), "r"(wv[j][4 * c4 + 1]), "r"(wv[j][4 * c4 + 2]),
                                     "r"(wv[j][4 * c4 + 3])
                                     : "memory");
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(AF + sa));
            }
            if (!ok) break;
        }
        // help drain this CTA's last unit
        const int nunits = p.units > (int)blockIdx.x ? (p.units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        if (nunits > 0 && !*abort_flag) {
            const uint32_t lu = (uint32_t)(nunits - 1);
            const uint32_t ab = p.nbuf == 2 ? (lu & 1u) : 0u;
            if (wait(bar(CF + ab), (p.nbuf == 2 ? (lu >> 1) : lu) & 1u)) {
                asm volatile("tcgen05.fence::after_thread_sync;");
                pdl_wait();  // Y may still be read by the preceding kernel
                const Unit un = unit_of(p, (int)blockIdx.x + (int)lu * (int)gridDim.x);
                drain(un, ab, warp & 3, 1 + (warp - kWDeq) / 4, 1 + kNDeq / 4);
            }
        }
    } else {
        // ------------- epilogue: TMEM -> Y (or the split's partials) -------------
        pdl_wait();  // Y may still be read by the preceding kernel
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        uint32_t lu = 0;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, lu++) {
            const Unit un = unit_of(p, u);
            const uint32_t ab = p.nbuf == 2 ? (lu & 1u) : 0u;
            if (!wait(bar(CF + ab), (p.nbuf == 2 ? (lu >> 1) : lu) & 1u)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            // the dequant warps help with the CTA's last unit (they are idle by then)
            const bool last = u + (int)gridDim.x >= p.units;
            drain(un, ab, q, 0, last ? 1 + kNDeq / 4 : 1);
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(CE + ab));
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kWMma) {
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
        xb[i] = bf16x2(v.x * kXScale, v.y * kXScale);  // exact scaling: see decode_unit_bf16
    }
    pdl_launch_dependents();
}

// Y = sum over the k splits of the partial products, in split order.
__global__ void __launch_bounds__(256) split_sum_kernel(const float4 *__restrict__ part, float4 *__restrict__ y,
                                                        int64_t n4, int splits) {
    pdl_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 a = __ldcs(part + i);
        for (int s = 1; s < splits; s++) {
            const float4 b = __ldcs(part + (int64_t)s * n4 + i);
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        y[i] = a;
    }
    pdl_launch_dependents();
}

// ------------------------------- host side -------------------------------
EncodeTiledFn encode_tiled_fn() {
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
    int bm, m_tiles, n_tiles, splits, units, ksteps, kper;
    int sr, sa, sb, raw_slot, raw_tma, tmem_cols, nbuf;
    int wide;  // 128 n x 2 bm m units (see gemm_kernel)
    int64_t xb_bytes, part_bytes;  // workspace after the counter head: bf16 X, then the split partials
    size_t smem;
    int grid;
};

static int block_bytes_of(int qt) { return qt == kQ4K ? 144 : qt == kQ5K ? 176 : 210; }

// Cost model in SM cycles for one unit (256 n x bm m, or WIDE 128 n x 2 bm m)
// and one 64-k step: the two MMAs 128 x bm x 16 of each 16-k step take about
// bm / 2 cycles each (4 * bm per step); dequantizing the stage's weights
// takes about kDeqCycles (256 x 64 values, measured ~1,900 cycles with the
// sixteen dequant warps) or kDeqWide (128 x 64); the SM pulls the raw stage
// and the X tiles out of L2 at about kL2Bytes per cycle.  Units run in waves
// of `sms`; the epilogue writes the unit's floats at about kYBytes per cycle
// and is hidden behind the next unit only when two accumulator buffers fit in
// TMEM (4 * bm <= 512 columns).  Split partials cost a write and a read of
// splits * M * N floats.
static GemmPlan gemm_plan(const GemvShape &s, int sms) {
    constexpr double kDeqCycles = 1900.0, kDeqWide = 1100.0, kL2Bytes = 55.0, kYBytes = 40.0,
                     kUnitOverhead = 1500.0, kBytesPerCycle = 3000.0;
    GemmPlan g{};
    const int B = block_bytes_of(s.qtype);
    // k rows whose byte pitch is a multiple of 16 (N % 256 == 0 and N/256*B % 16
    // == 0) are TMA-copyable as a 2D tile: one block per row (plus the lead of
    // a 2-byte aligned Q6_K block); otherwise up to two blocks plus the lead.
    g.raw_tma = (s.N % 256 == 0) && ((s.N / 256 * B) % 16 == 0);
    if (g.raw_tma) g.raw_slot = (B % 16 == 0) ? B : ((B + 14 + 15) & ~15);
    else g.raw_slot = (2 * B + 15 + 15) & ~15;
    const double raw_stage = (double)kGBK * g.raw_slot;
    g.ksteps = (int)((s.K + kGBK - 1) / kGBK);
    double best = 1e300;
    // WIDE only pays when one m tile of 256 cannot hold M (otherwise its
    // second m half would be empty)
    const size_t ring_budget = 227 * 1024 - (1024 + 8 * (6 * kMaxStages + 8) + 16);
    for (int wide = 0; wide <= (s.M > 256 ? 1 : 0); wide++) {
        const int nu = wide ? kMmaM : kGBN, mh = wide ? 2 : 1;
        const int64_t n_tiles = (s.N + nu - 1) / nu;
        for (int bm = 16; bm <= 256; bm += 16) {
            const int64_t mt = (s.M + mh * bm - 1) / (mh * bm);
            if (bm > 16 && (s.M + mh * (bm - 16) - 1) / (mh * (bm - 16)) == mt) continue;  // bm - 16: same m tiles
            // WIDE needs three A and three raw stages beside two X stages (with
            // two of each the hand-offs, not the work, set the pace: Q6_K rows
            // that are not 16-byte pitched took 127 us at M = 512)
            if (wide && 3 * (size_t)kAHalf + 2 * (size_t)mh * bm * 128 + 3 * (size_t)raw_stage > ring_budget) continue;
            const int64_t tiles = mt * n_tiles;
            const double step = std::max({4.0 * bm, wide ? kDeqWide : kDeqCycles,
                                          (raw_stage + 128.0 * mh * bm) / kL2Bytes});
            const double epi = (double)nu * mh * bm * 4.0 / kYBytes;
            const bool two_bufs = 4 * bm <= 512;
            for (int sp : {1, 2, 3, 4, 6, 8}) {
                if (sp > g.ksteps) break;
                const int kper = (g.ksteps + sp - 1) / sp;
                if ((int64_t)(sp - 1) * kper >= g.ksteps) continue;  // every split gets k steps
                const int64_t units = tiles * sp;
                const int64_t waves = (units + sms - 1) / sms;
                double cost =
                    (double)waves * (kper * step + kUnitOverhead) + (two_bufs ? epi : (double)waves * epi);
                if (sp > 1) cost += 2.0 * sp * (double)s.M * (double)s.N * 4.0 / kBytesPerCycle + kUnitOverhead;
                if (cost < best * 0.999) {
                    best = cost;
                    g.wide = wide;
                    g.n_tiles = (int)n_tiles;
                    g.bm = bm;
                    g.m_tiles = (int)mt;
                    g.splits = sp;
                    g.kper = kper;
                    g.units = (int)units;
                }
            }
        }
    }
    g.nbuf = 4 * g.bm <= 512 ? 2 : 1;
    g.grid = std::min(g.units, sms);
    const size_t a_st = g.wide ? kAHalf : kAStage, b_st = (size_t)(g.wide ? 2 : 1) * g.bm * 128,
                 r_st = (size_t)kGBK * g.raw_slot;
    const size_t fixed = 1024 + 8 * (6 * kMaxStages + 8) + 16;
    const size_t budget = 227 * 1024 - fixed;
    // Ring depths: every stage makes a round trip through several mbarrier
    // hand-offs (about 4000 cycles for the A ring: dequant, MMA issue, MMA
    // execution, commit, dequant again), so two stages leave the tensor cores
    // idle half the time.  Grow A, then X, then the raw weights, round-robin.
    g.sa = 2;
    g.sb = 2;
    g.sr = 2;
    auto used = [&]() { return g.sa * a_st + g.sb * b_st + g.sr * r_st; };
    for (bool grown = true; grown;) {
        grown = false;
        if (g.sa < 4 && used() + a_st <= budget) {
            g.sa++;
            grown = true;
        }
        if (g.sb < 4 && used() + b_st <= budget) {
            g.sb++;
            grown = true;
        }
        if (g.sr < 6 && used() + r_st <= budget) {
            g.sr++;
            grown = true;
        }
    }
    g.smem = fixed + used();
    g.tmem_cols = 32;
    while (g.tmem_cols < g.nbuf * 2 * g.bm) g.tmem_cols <<= 1;
    g.xb_bytes = ((s.M * s.K * 2) + 255) & ~int64_t(255);
    g.part_bytes = g.splits > 1 ? (int64_t)g.splits * s.M * s.N * 4 : 0;
    return g;
}

size_t gemm_workspace_bytes(const GemvShape &s, int device) {
    if (s.N % 32 != 0) return 0;
    const GemmPlan g = gemm_plan(s, device_sm_count(device));
    return kWorkspaceCounterHead + (size_t)(g.xb_bytes + g.part_bytes);
}

template <int QT, bool WIDE>
static cudaError_t launch_gemm(const CUtensorMap &tm, const CUtensorMap &tw, const GemmParams &gp, const GemmPlan &g,
                               cudaStream_t st) {
    auto kern = gemm_kernel<QT, WIDE>;
    cudaError_t e = kernel_smem((const void *)kern, g.smem, false);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)g.grid);
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tm, tw, gp);
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::max(grid, 1));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

int gemm_launch(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y, void *ws,
                size_t ws_bytes, cudaStream_t stream, int device) {
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
    const int sms = device_sm_count(device);
    const GemmPlan g = gemm_plan(s, sms);
    const size_t need = kWorkspaceCounterHead + (size_t)(g.xb_bytes + g.part_bytes);
    if (ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) {
        set_error("gemm needs a 256-byte aligned workspace of %zu bytes (got %zu)", need, ws_bytes);
        return 4;
    }
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return 5;
    }
    // after the GEMV's counter head, which this call leaves untouched
    uint32_t *xb = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) + kWorkspaceCounterHead);
    float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kWorkspaceCounterHead + g.xb_bytes);
    // 1. X -> bf16
    {
        const int64_t npairs = s.M * s.K / 2;
        const int grid = (int)std::min<int64_t>((npairs + 255) / 256, (int64_t)sms * 8);
        cudaError_t e = launch_pdl(x_to_bf16_kernel, grid, stream, x, xb, npairs);
        if (e != cudaSuccess) {
            set_error("x to bf16 launch failed: %s", cudaGetErrorString(e));
            return 5;
        }
    }
    // 2. tensor map over the bf16 X: dims {K, M}, box {64, bm}, 128-byte swizzle
    CUtensorMap tm;
    const cuuint64_t dims[2] = {(cuuint64_t)s.K, (cuuint64_t)s.M};
    const cuuint64_t strides[1] = {(cuuint64_t)(s.K * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kGBK, (cuuint32_t)g.bm};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return 5;
    }
    // tensor map over the weight bytes as [K rows][N/256*B bytes], box {raw_slot, 64}
    CUtensorMap tw = tm;  // unused unless raw_tma
    if (g.raw_tma) {
        const int B = block_bytes_of(s.qtype);
        const cuuint64_t wd[2] = {(cuuint64_t)(s.N / 256 * B), (cuuint64_t)s.K};
        const cuuint64_t ws_[1] = {(cuuint64_t)(s.N / 256 * B)};
        const cuuint32_t wbox[2] = {(cuuint32_t)g.raw_slot, (cuuint32_t)kGBK};
        r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), wd, ws_, wbox, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
            return 5;
        }
    }
    GemmParams gp{};
    gp.w = static_cast<const uint8_t *>(w);
    gp.w_bytes = w_bytes;
    gp.y = g.splits > 1 ? part : y;
    gp.K = s.K;
    gp.N = s.N;
    gp.M = s.M;
    gp.bm = g.bm;
    gp.m_tiles = g.m_tiles;
    gp.splits = g.splits;
    gp.units = g.units;
    gp.ksteps = g.ksteps;
    gp.kper = g.kper;
    gp.sr = g.sr;
    gp.sa = g.sa;
    gp.sb = g.sb;
    gp.raw_slot = g.raw_slot;
    gp.raw_tma = g.raw_tma;
    gp.tmem_cols = g.tmem_cols;
    gp.acc_stride = 2 * g.bm;
    gp.nbuf = g.nbuf;
    gp.wide = g.wide;
    cudaError_t e;
    switch (s.qtype) {
    case kQ4K: e = g.wide ? launch_gemm<kQ4K, true>(tm, tw, gp, g, stream) : launch_gemm<kQ4K, false>(tm, tw, gp, g, stream); break;
    case kQ5K: e = g.wide ? launch_gemm<kQ5K, true>(tm, tw, gp, g, stream) : launch_gemm<kQ5K, false>(tm, tw, gp, g, stream); break;
    default: e = g.wide ? launch_gemm<kQ6K, true>(tm, tw, gp, g, stream) : launch_gemm<kQ6K, false>(tm, tw, gp, g, stream); break;
    }
    if (e != cudaSuccess) {
        set_error("gemm launch failed: %s", cudaGetErrorString(e));
        return 5;
    }
    if (g.splits > 1) {
        const int64_t n4 = s.M * s.N / 4;
        const int grid = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)sms * 8);
        e = launch_pdl(split_sum_kernel, grid, stream, reinterpret_cast<const float4 *>(part),
                       reinterpret_cast<float4 *>(y), n4, g.splits);
        if (e != cudaSuccess) {
            set_error("split-K sum launch failed: %s", cudaGetErrorString(e));
            return 5;
        }
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
