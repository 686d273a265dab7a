// gemv.cu -- fused k-quant dequantize + GEMV on sm_100a, fp32 accumulate.
//
// Computes y[m][n] = sum_k x[m][k] * W[k][n] for 1 <= M <= 8, where W is a
// Q4_K / Q5_K / Q6_K weight in vibrant's orientation: W[k][n] is value
// k*N + n of the super-block stream (internal/gguf/loader.go:24-27,
// internal/tensor/matmul_quant.go:87-89).  It replaces the fp32 single-row
// kernel behind matmulGPU (internal/gpu/cuda/kernels.cu:61-77 via
// internal/tensor/ops_cuda.go:55-63), which needed the weight expanded to
// float32 on the host first.
//
// Design (HBM-bound; algorithmic bytes per call = weight bytes + x + y):
//  * The output columns are cut into tiles of TN = 32*VPT values; a row
//    chunk (one k, TN columns) is a contiguous run of super-blocks.  The
//    (tile, k) space is flattened and split evenly over a grid of 2 CTAs per
//    SM ("stream-K" over rows), so every shape fills the machine.
//  * Each of the 8 warps of a CTA takes every 8th row of the CTA's range and
//    streams its own rows into a private shared-memory ring (STAGES slots,
//    one mbarrier each): lane 0 issues one cp.async.bulk (no multicast) per
//    row chunk, refilling a slot right after its row is decoded.  There is
//    no producer warp and no cross-warp wait outside the tile flushes.  The
//    first STAGES rows are requested before griddepcontrol.wait, so the
//    weight stream overlaps the tail of the previous kernel when launched
//    with programmatic stream serialization.  x for 32 rows at a time sits
//    one value per lane and reaches each row through a shuffle.
//  * Lane l decodes VPT consecutive values of the row (64 for M == 1 on wide
//    matrices, else 32 / 32 / 16 / 8 for M = 1 / 2 / 4 / 8), in groups of at
//    most 32 that never straddle a super-block, straight from the packed
//    bytes: nibbles are merged into byte lanes, each value is moved into a
//    word of its own by one byte permute and used as a float as it is (the
//    integer q is the subnormal q * 2^-149; the multipliers carry a
//    power-of-two scale that undoes it), and accumulated with packed fp32x2
//    FMAs: a = x*(d*scale) times q per value (Q6_K; 32*a once per row and
//    lane into a correction sum applied at the flush), or w = (d*sc)*q -
//    dmin*m formed per value and then multiplied by x (Q4_K/Q5_K: keeps the
//    error relative to |x*w| where the two terms cancel).
//  * Partial sums of the 8 warps are added through shared memory in a fixed
//    tree order; tiles split over several CTAs go through a small partials
//    buffer and the last CTA to arrive (an atomic counter per tile, reset
//    after use) adds the partials in CTA order, so results are deterministic.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "kq_device.cuh"
#include "peer.cuh"
#include "vkq_internal.h"

namespace vkq {

static __device__ int g_gemv_status;

constexpr int kNW = 8;                       // warps per CTA, each streaming its own rows
constexpr int kThreads = kNW * 32;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s
constexpr int kSmemPerCta = 112 * 1024;      // two CTAs per SM
constexpr int kRedSlots = 4;                 // [MR][TN] partial-sum slots of the tree warp reduction
// Tiles of at most 1024 values (all rows m) reduce across the 8 warps in one
// step through 8 slots (fewer barriers); larger ones through a tree over
// kRedSlots slots (less shared memory).
__host__ __device__ constexpr bool flat_reduction(int mr, int vpt) { return mr * 32 * vpt <= 1024; }
constexpr int kMaxStages = 12;               // ring slots per warp
constexpr int kMinStages = 3;
constexpr int kCombineLoads = 8;             // partial loads in flight per thread in the split-K sum
constexpr int kMaxFanIn = 32;                // CTAs per tile summed in one level
constexpr int kGroup = 16;                   // CTAs per first-level group above that

struct GemvParams {
    const uint8_t *w;
    int64_t w_bytes;    // valid bytes of w
    int64_t w_floor16;  // bytes that bulk copies may read
    const float *x;
    float *y;
    int64_t K, N;        // N: the output columns this launch computes
    int M;
    int ntiles;
    int grid;
    int64_t rows_total;  // ntiles * K
    int64_t rpc;         // rows (tile, k) per CTA
    float *partials;     // [grid][2][MR][TN]: per-CTA sums of shared tiles
    float *gpartials;    // [ntiles + ngroups][MR][TN]: per-group sums (two-level split-K)
    int *counters;       // [ntiles] per tile, then [ntiles + ngroups] per (tile + group)
    int group;           // CTAs per first-level group of the split-K sum
    int row_cap;         // bytes per ring row slot (multiple of 16)
    int stages;
};

// Row-sharded all-gather: column n of this launch's columns is stored into
// every rank's output [M][y_ld] at column col_off + n.  A separate kernel
// parameter (growing GemvParams changes the plain kernel's code generation).
//
// The weight is this rank's row-block shard (vkq_shard_weight): row k of the
// shard holds the super-blocks that cover columns [n_base, n_base + N) of row
// k of the full [K, ld] weight, starting at the block that holds column
// n_base, in rs / 256 block slots.  Value n of row k therefore sits at
// position k * rs + ((k * ld + n_base) & 255) + n of the shard's stream, which
// keeps every value at the in-block position it had in the full weight (a
// block that straddles two rows or two shards is copied whole and the values
// outside the row's columns are never read).
//
// Protocol (every rank makes the same sequence of calls on one channel; the
// flagged-word exchange of peer.cuh):
//  * seq = sync[0] + 1 is this call's number (read after
//    griddepcontrol.wait, once the preceding work is complete);
//  * every finished output value goes into this rank's output and, as one
//    64-bit store of (seq, value bits), into its slot in every other rank's
//    channel buffer;
//  * at the end every thread of the grid polls a share of this rank's slots
//    for the other ranks' columns of call seq and copies them into the
//    output, so the kernel's completion means the whole result is in place;
//    the last CTA to finish records seq in sync[0];
//  * a slot of a later call (a rank out of step) or a wait that runs out
//    marks the channel failed (sync[2], sticky): a failed channel sends and
//    waits no more, every later call keeps to its own columns and reports
//    VKQ_ERR_PEER until the host resets it.
constexpr int kMaxPeers = 8;
struct GatherParams {
    float *peer_y[kMaxPeers];         // every rank's output buffer (addresses valid on this device)
    unsigned *peer_flags[kMaxPeers];  // every rank's flags: [0, world) started, [world, 2 world) done
    unsigned *sync;                   // this rank's [last call, finished CTAs, failed]
    int world, rank;
    int64_t y_ld, col_off;
    int64_t rs, ld, n_base;           // shard row stride (values), full row length, first column
    uint64_t wait_ns;                 // budget of each wait on the peers
};

__device__ __forceinline__ void set_status(int code) { atomicExch(&g_gemv_status, code); }

// Output stores of the all-gather: this rank's output buffer and, unless
// the channel has failed (peers == false), the value's slot in every other
// rank's channel buffer.
__device__ __forceinline__ void store_peers(const GatherParams &g, bool peers, unsigned seq, int64_t m, int64_t c,
                                            float v) {
    g.peer_y[g.rank][m * g.y_ld + g.col_off + c] = v;
    if (!peers) return;
    const uint64_t word = ((uint64_t)seq << 32) | __float_as_uint(v);
#pragma unroll 1
    for (int r = 0; r < g.world; r++)
        if (r != g.rank) st_relaxed_sys_u64(channel_slot(g.peer_flags[r], g.y_ld, m, g.col_off + c, seq), word);
}
__device__ __forceinline__ void store_peers4(const GatherParams &g, bool peers, unsigned seq, int64_t m, int64_t c,
                                             float4 v) {
    // 16-byte aligned: widths and offsets are multiples of 32
    *reinterpret_cast<float4 *>(g.peer_y[g.rank] + m * g.y_ld + g.col_off + c) = v;
    if (!peers) return;
    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll 1
    for (int r = 0; r < g.world; r++) {
        if (r == g.rank) continue;
#pragma unroll
        for (int i = 0; i < 4; i++)
            st_relaxed_sys_u64(channel_slot(g.peer_flags[r], g.y_ld, m, g.col_off + c + i, seq),
                               ((uint64_t)seq << 32) | __float_as_uint(e[i]));
    }
}
__device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Integer weights as subnormal floats.  A 6-bit quant q isolated in the low
// bits of a 32-bit word is, read as a float, the subnormal q * 2^-149: one
// byte permute per value makes an fma operand, with no conversion.
//  * Q6_K: fma(a * 2^76, word, acc) adds a * q * 2^-73 with the single
//    rounding of fma(a, float(q), acc * 2^73); the flush multiplies by 2^73.
//    Exact while |a| < 2^52 (a * 2^76 finite) and |a * q| >= 2^-53 or 0.
//  * Q4_K / Q5_K: fma(d*sc * 2^100, word, -dmin*m * 2^-49) is the weight
//    w = d*sc*q - dmin*m times 2^-49 with one rounding (all three terms stay
//    normal for f16 d, dmin and 6-bit sc, m), and x * 2^49 restores the scale
//    in the product with x.
constexpr float kQ6Scale = 0x1p76f;     // Q6_K per-row multipliers
constexpr float kQ6Unscale = 0x1p73f;   // Q6_K accumulators at the flush
constexpr float kQ45Scale = 0x1p100f;   // Q4_K / Q5_K d*sc
constexpr float kQ45Down = 0x1p-49f;    // Q4_K / Q5_K -dmin*m (and 1 / the x scale)
constexpr float kQ45XScale = 0x1p49f;   // Q4_K / Q5_K x
// Q6_K takes the subnormal product with a correction sum for MR <= 2 and
// the exact 2^23 form for MR >= 4 (accum_chunk_magic).
template <int MR> constexpr bool kQ6Split = MR <= 2;
constexpr float kQ6MagicScale = 0x1p-73f;  // Q6_K per-row multipliers of the 2^23 form

// Q6_K: acc[m][pair0 + j] += a[m] * (value 2j, value 2j+1) of an 8-value
// chunk; byte lane j of E / O holds value 2j / 2j+1.
template <int MR, int NP>
__device__ __forceinline__ void accum_chunk_scaled(float2 (&acc)[MR][NP], int pair0, uint32_t E, uint32_t O,
                                                   const float (&a)[MR]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 q2 = make_float2(__uint_as_float(prmt(E, 0u, 0x4440u | j)),
                                      __uint_as_float(prmt(O, 0u, 0x4440u | j)));
#pragma unroll
        for (int m = 0; m < MR; m++) acc[m][pair0 + j] = f2fma(make_float2(a[m], a[m]), q2, acc[m][pair0 + j]);
    }
}

// Q6_K for MR >= 4, where the correction sums would cost registers the MR
// accumulators need and one more packed add per pair is small beside the MR
// FMAs: acc[m] += a'[m] * (q - 32) with the value q - 32 formed exactly by a
// byte permute into the exponent of 2^23 and one packed add of -(2^23 + 32);
// a' = a * 2^-73 (kQ6MagicScale) so that the flush treats both forms alike.
template <int MR, int NP>
__device__ __forceinline__ void accum_chunk_magic(float2 (&acc)[MR][NP], int pair0, uint32_t E, uint32_t O,
                                                  const float (&a)[MR]) {
    const float2 neg = make_float2(-8388640.0f, -8388640.0f);  // -(2^23 + 32)
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 q2 = f2add(make_float2(__uint_as_float(prmt(E, 0x4B000000u, 0x7440u | j)),
                                            __uint_as_float(prmt(O, 0x4B000000u, 0x7440u | j))), neg);
#pragma unroll
        for (int m = 0; m < MR; m++) acc[m][pair0 + j] = f2fma(make_float2(a[m], a[m]), q2, acc[m][pair0 + j]);
    }
}

// Q4_K / Q5_K: w = scale * q - min formed per value (one rounding, as close
// to the reference's two roundings as one fma gets), then acc[m] += x[m] * w.
// Forming w first keeps the error relative to |x*w| even where scale*q and
// min nearly cancel.
template <int MR, int NP>
__device__ __forceinline__ void accum_chunk_affine(float2 (&acc)[MR][NP], int pair0, uint32_t E, uint32_t O,
                                                   float2 s2, float2 nm2, const float (&xs)[MR]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 q2 = make_float2(__uint_as_float(prmt(E, 0u, 0x4440u | j)),
                                      __uint_as_float(prmt(O, 0u, 0x4440u | j)));
        const float2 w2 = f2fma(s2, q2, nm2);
#pragma unroll
        for (int m = 0; m < MR; m++) acc[m][pair0 + j] = f2fma(make_float2(xs[m], xs[m]), w2, acc[m][pair0 + j]);
    }
}

// Decode VPT values of one super-block (shared address blk, first value
// `within`) and accumulate x[m] * W into acc.  Q6_K, w = (d*scale)*(q - 32):
// acc gets a*q with a = x*d*scale (scaled by 2^76) and corr[m] (one
// component per 16-value scale group) the sum of a, taken 32 times at the
// flush.  Q4_K / Q5_K accumulate x*w directly (corr unused).
template <int QT, int MR, int VPT>
__device__ __forceinline__ void decode_accum(uint32_t blk, int within, const float (&xv)[MR],
                                             float2 (&acc)[MR][VPT / 2], float2 (&corr)[MR]) {
    constexpr int NCH = VPT / 8;  // chunks of 8 values
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const uint4 hdr = lds128(blk);
        const float d = hw_f16_to_f32(hdr.x & 0xFFFFu), dmin = hw_f16_to_f32(hdr.x >> 16);
        const int sb = within >> 5;
        const uint32_t sc24 = sb < 4 ? hdr.y : __funnelshift_r(hdr.y, hdr.z, 24);
        const uint32_t m24 = sb < 4 ? __funnelshift_r(hdr.z, hdr.w, 16) : (hdr.w >> 8);
        const uint32_t sh = 6u * (sb & 3);
        const float ds = (d * kQ45Scale) * (float)((sc24 >> sh) & 63u);
        const float ndm = (dmin * -kQ45Down) * (float)((m24 >> sh) & 63u);
        const float2 s2 = make_float2(ds, ds), nm2 = make_float2(ndm, ndm);
        float xs[MR];
#pragma unroll
        for (int m = 0; m < MR; m++) xs[m] = xv[m] * kQ45XScale;
        const uint32_t qs = blk + (QT == kQ4K ? 16 : 48) + (within >> 1);
        uint32_t wq[NCH];
        if constexpr (NCH == 4) {
            uint4 t = lds128(qs);
            wq[0] = t.x; wq[1] = t.y; wq[2] = t.z; wq[3] = t.w;
        } else if constexpr (NCH == 2) {
            uint2 t = lds64(qs);
            wq[0] = t.x; wq[1] = t.y;
        } else {
            wq[0] = lds32(qs);
        }
        uint32_t qh = 0;
        if constexpr (QT == kQ5K) {
            const uint32_t qha = blk + 16 + (within >> 3);
            if constexpr (NCH == 4) qh = lds32(qha);
            else if constexpr (NCH == 2) qh = lds16(qha);
            else qh = lds16(qha & ~1u) >> (8 * (qha & 1u));
        }
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            uint32_t E = wq[c] & 0x0F0F0F0Fu;
            uint32_t O = (wq[c] >> 4) & 0x0F0F0F0Fu;
            if constexpr (QT == kQ5K) {
                // bit i of hb is the fifth bit of value 8c+i; spread bits
                // 0,2,4,6 (and 1,3,5,7) to bit 4 of byte lanes 0..3.
                const uint32_t hb = (qh >> (8 * c)) & 0xFFu;
                E |= ((hb & 0x55u) * 0x410410u) & 0x10101010u;
                O |= (((hb >> 1) & 0x55u) * 0x410410u) & 0x10101010u;
            }
            accum_chunk_affine<MR, VPT / 2>(acc, 4 * c, E, O, s2, nm2, xs);
        }
    } else {  // Q6_K: blk is only 2-byte aligned in shared memory
        const float d = hw_f16_to_f32(lds16(blk + 208)) * (kQ6Split<MR> ? kQ6Scale : kQ6MagicScale);
        const int g0 = within >> 4;  // first 16-value scale group
        const uint32_t sraw = lds16(blk + 192 + (g0 & ~1));
        const int s0 = (int)(int8_t)((g0 & 1) ? (sraw >> 8) : sraw);
        const int s1 = (int)(int8_t)(sraw >> 8);
        float a0[MR], a1[MR];
        const float ds0 = d * (float)s0, ds1 = d * (float)s1;
#pragma unroll
        for (int m = 0; m < MR; m++) {
            a0[m] = xv[m] * ds0;
            a1[m] = xv[m] * ds1;
            if constexpr (kQ6Split<MR>) {
                if constexpr (NCH == 4) corr[m] = f2add(corr[m], make_float2(a0[m], a1[m]));
                else corr[m].x += a0[m];
            }
        }
        const uint32_t ql = blk + (within >> 1);
        const uint32_t qha = blk + 128 + (within >> 2);
        uint32_t wq[NCH];
        // ql and (for groups of >= 16 values) qh lie at the same offset
        // modulo 4: one shift serves both
        const uint32_t shf = (ql & 3u) * 8u;
        {
            const uint32_t base = ql & ~3u;
            uint32_t wv[NCH + 1];
#pragma unroll
            for (int i = 0; i <= NCH; i++) wv[i] = lds32(base + 4 * i);
#pragma unroll
            for (int i = 0; i < NCH; i++) wq[i] = __funnelshift_r(wv[i], wv[i + 1], shf);
        }
        uint32_t qh[(NCH + 1) / 2];
        if constexpr (NCH >= 2) {
            const uint32_t base = qha & ~3u;
            uint32_t hv[NCH / 2 + 1];
#pragma unroll
            for (int i = 0; i <= NCH / 2; i++) hv[i] = lds32(base + 4 * i);
#pragma unroll
            for (int i = 0; i < NCH / 2; i++) qh[i] = __funnelshift_r(hv[i], hv[i + 1], shf);
        } else {
            qh[0] = lds16(qha);
        }
        uint32_t qhs[(NCH + 1) / 2];
#pragma unroll
        for (int i = 0; i < (NCH + 1) / 2; i++) qhs[i] = qh[i] >> 4;
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            // the low nibble of byte lane j of X is nibble j of the chunk's
            // 16 qh bits = (hi2 of value 2j+1) << 2 | (hi2 of value 2j)
            const uint32_t X = prmt(qh[c >> 1], qhs[c >> 1], (c & 1) ? 0x7362u : 0x5140u);
            const uint32_t E = (wq[c] & 0x0F0F0F0Fu) | ((X << 4) & 0x30303030u);
            const uint32_t O = ((wq[c] >> 4) & 0x0F0F0F0Fu) | ((X << 2) & 0x30303030u);
            if constexpr (kQ6Split<MR>) {
                if (NCH == 4 && c >= 2) accum_chunk_scaled<MR, VPT / 2>(acc, 4 * c, E, O, a1);
                else accum_chunk_scaled<MR, VPT / 2>(acc, 4 * c, E, O, a0);
            } else {
                accum_chunk_magic<MR, VPT / 2>(acc, 4 * c, E, O, a0);  // MR >= 4: VPT <= 16, one group
            }
        }
    }
}

// XOR swizzle of a lane's float4 slots in the reduction buffer: the 8 lanes
// of a quarter warp store to 8 different 16-byte bank groups.
template <int VPT>
__device__ __forceinline__ int red_swz(int lane) {
    constexpr int F = VPT / 4;  // float4 per lane
    if constexpr (F >= 8) return lane & 7;
    else return (lane / (8 / F)) & (F - 1);
}

// G: the all-gather variant (outputs stored into every rank's buffer, with
// the start / done handshakes); the plain kernel carries none of it.
template <int QT, int MR, int VPT, bool G>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvParams p, const GatherParams gq) {
    constexpr int B = QT_<QT>::BYTES;
    constexpr int TN = 32 * VPT;
    constexpr bool kFlatRed = flat_reduction(MR, VPT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = p.stages;
    // [kNW][S] mbarriers | 2 flag words | ring [kNW][S][row_cap] | red [8 or kRedSlots][MR][TN]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    int *flag = reinterpret_cast<int *>(full + kNW * S);
    const int hdr_bytes = ((8 * kNW * S + 8) + 127) & ~127;
    uint8_t *ring = smem + hdr_bytes;
    float *red = reinterpret_cast<float *>(ring + (size_t)kNW * S * p.row_cap);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tid = threadIdx.x;  // 0..255
    const int64_t f0 = (int64_t)blockIdx.x * p.rpc;
    const int64_t f1 = imin64(f0 + p.rpc, p.rows_total);
    const int nrows = (int)(f1 - f0);
    // this warp's rows: f0 + warp + kNW * j for j < nw
    const int nw = nrows > warp ? (nrows - warp + kNW - 1) / kNW : 0;
    const int64_t K = p.K, N = p.N;
    const uint32_t Ku = (uint32_t)K, Nu = (uint32_t)N;

    uint64_t *my_full = full + warp * S;
    uint8_t *my_ring = ring + (size_t)warp * S * p.row_cap;
    const uint32_t my_ring_u32 = smem_u32addr(my_ring);
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(smem_u32addr(&my_full[s]), 1);
        mbar_init_fence();
    }
    __syncwarp();

    // Per-row parameters are computed 32 rows at a time, one row per lane,
    // and reach the lane that uses them through a shuffle.
    //   issue side: byte offset of the row chunk's 16-byte aligned span of
    //   super-blocks and its length (bulk copy), plus the < 16 bytes past the
    //   last 16-byte boundary of w (copied by hand);
    //   decode side: the low 32 bits of v0 = k*N + n0, or the shard position
    //   k*rs + ((k*ld + n_base) & 255) + n0 of the all-gather (in-block
    //   offset of the row's first value and the 16-byte lead of its first
    //   block), the first column n0 of the row's tile, and x of the row.
    auto row_tk = [&](int r, uint32_t &t, uint32_t &k) {
        const uint32_t f = (uint32_t)(f0 + warp) + (uint32_t)(kNW * r);  // rows_total < 2^31
        t = f / Ku;
        k = f - t * Ku;
    };
    uint32_t i_src = 0, i_len = 0;  // issue parameters of row ib + lane
    auto issue_batch = [&](int ib) {
        const int r = ib + lane;
        i_src = 0;
        i_len = 0;
        if (r < nw) {
            uint32_t t, k;
            row_tk(r, t, k);
            const int64_t n0 = (int64_t)t * TN, n1 = imin64(n0 + TN, N);
            const int64_t base = G ? (int64_t)k * gq.rs + (((int64_t)k * gq.ld + gq.n_base) & 255) : (int64_t)k * N;
            const int64_t a_lo = (((base + n0) >> 8) * B) & ~int64_t(15);
            const int64_t byte_hi = ((base + n1 + 255) >> 8) * B;
            int64_t c_hi = imin64((byte_hi + 15) & ~int64_t(15), p.w_floor16);
            if (c_hi < a_lo) c_hi = a_lo;
            i_src = (uint32_t)a_lo;  // weights are below 4 GiB on this path
            const int64_t tail = byte_hi > c_hi ? byte_hi - c_hi : 0;  // < 16
            i_len = (uint32_t)(c_hi - a_lo) | ((uint32_t)tail << 24);
        }
    };
    // Lane 0 streams this warp's row ji into ring slot sl.
    int ji = 0;
    auto issue_next = [&](int sl) {
        if ((ji & 31) == 0) issue_batch(ji);
        const uint32_t src = __shfl_sync(0xffffffffu, i_src, ji & 31);
        const uint32_t len = __shfl_sync(0xffffffffu, i_len, ji & 31);
        if (lane == 0) {
            const uint32_t bytes = len & 0xFFFFFFu, tail = len >> 24;
            uint8_t *dst = my_ring + (size_t)sl * p.row_cap;
            for (uint32_t b = 0; b < tail; b++) dst[bytes + b] = p.w[(int64_t)src + bytes + b];
            const uint32_t bar = smem_u32addr(&my_full[sl]);
            mbar_arrive_expect_tx(bar, bytes);
            if (bytes > 0) bulk_g2s(my_ring_u32 + (uint32_t)(sl * p.row_cap), p.w + src, bytes, bar);
        }
        ji++;
    };
    // the weights do not depend on the preceding kernel: fill the ring first
    for (int s = 0; s < S && ji < nw; s++) issue_next(s);
    pdl_launch_dependents();
    pdl_wait();  // x, y and the workspace may belong to the preceding kernel

    uint32_t c_n0 = 0, c_v0 = 0;  // decode parameters of row jb + lane
    auto decode_batch = [&](int jb) {
        const int r = jb + lane;
        if (r < nw) {
            uint32_t t, k;
            row_tk(r, t, k);
            c_n0 = t * TN;
            if constexpr (G) c_v0 = k * (uint32_t)gq.rs + ((k * (uint32_t)gq.ld + (uint32_t)gq.n_base) & 255u) + c_n0;
            else c_v0 = k * Nu + c_n0;
        }
    };
    auto load_x = [&](int jb, float (&xr)[MR]) {
        const int r = jb + lane;
        uint32_t kx = 0;
        if (r < nw) kx = ((uint32_t)(f0 + warp) + (uint32_t)(kNW * r)) % Ku;
#pragma unroll
        for (int m = 0; m < MR; m++) xr[m] = (r < nw && m < p.M) ? __ldg(p.x + (int64_t)m * K + kx) : 0.0f;
    };
    float xcur[MR], xnext[MR];
    load_x(0, xcur);
    load_x(32, xnext);
    decode_batch(0);

    const uint32_t red_base = smem_u32addr(red);
    // H groups of VH <= 32 consecutive values per lane (two for VPT = 64);
    // a group never straddles a super-block
    constexpr int H = VPT > 32 ? VPT / 32 : 1;
    constexpr int VH = VPT / H;
    float2 acc[H][MR][VH / 2];
    float2 corr[H][MR];
#pragma unroll
    for (int h = 0; h < H; h++) {
#pragma unroll
        for (int m = 0; m < MR; m++) {
#pragma unroll
            for (int i = 0; i < VH / 2; i++) acc[h][m][i] = make_float2(0.f, 0.f);
            corr[h][m] = make_float2(0.f, 0.f);
        }
    }

    // All-gather: this call's number, and whether the channel failed
    // earlier (then this rank keeps to its own columns and waits for none).
    // flag[1] carries seq, flag[2] whether values go to the other ranks.
    unsigned seq = 0;
    bool peers_ok = true;
    if (G && gq.world > 1) {
        if (tid == 0) {
            const unsigned sq = *reinterpret_cast<volatile unsigned *>(&gq.sync[0]) + 1u;
            const bool failed = *reinterpret_cast<volatile unsigned *>(&gq.sync[2]) != 0u;
            if (failed) set_status(kStatusPeer);
            flag[1] = (int)sq;
            flag[2] = failed ? 0 : 1;
        }
        named_bar_sync(1, kNW * 32);
        seq = (unsigned)flag[1];
        peers_ok = flag[2] != 0;
    } else if (G) {
        peers_ok = false;  // one rank: its own buffer only
    }

    const int64_t first_tile = f0 / K;
    const int64_t last_tile = (f1 - 1) / K;
    int64_t cur_tile = first_tile;
    bool pend_first = false, pend_last = false;  // shared tiles written as partials
    int old_first = 0, old_last = 0;             // their first-level counts (thread 0)
    int64_t next_boundary = (cur_tile + 1) * K - f0;

    // this lane's float4 i (of VPT / 4) of row m in slot sl of the reduction buffer
    auto red_addr = [&](int sl, int m, int i) {
        return red_base + (uint32_t)(((sl * MR + m) * TN + lane * VPT + 4 * (i ^ red_swz<VPT>(lane))) * 4);
    };
    auto store_red = [&](int sl) {
#pragma unroll
        for (int m = 0; m < MR; m++) {
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                const float2 u = acc[i / (VH / 4)][m][2 * (i % (VH / 4))];
                const float2 v = acc[i / (VH / 4)][m][2 * (i % (VH / 4)) + 1];
                asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(red_addr(sl, m, i)), "f"(u.x), "f"(u.y),
                             "f"(v.x), "f"(v.y));
            }
        }
    };
    auto add_red = [&](int sl) {
#pragma unroll
        for (int m = 0; m < MR; m++) {
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                float4 t4;
                asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                             : "=f"(t4.x), "=f"(t4.y), "=f"(t4.z), "=f"(t4.w) : "r"(red_addr(sl, m, i)));
                float2 &u = acc[i / (VH / 4)][m][2 * (i % (VH / 4))];
                float2 &v = acc[i / (VH / 4)][m][2 * (i % (VH / 4)) + 1];
                u = f2add(u, make_float2(t4.x, t4.y));
                v = f2add(v, make_float2(t4.z, t4.w));
            }
        }
    };

    auto flush = [&](int64_t tile) {
        // 1. Q6_K: value = acc * 2^73 - 32 * sum(a) (one rounding), in place
        if constexpr (QT == kQ6K) {
#pragma unroll
            for (int h = 0; h < H; h++) {
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    const float c_lo = corr[h][m].x * -0x1p-71f;  // -32 * sum(a) / 2^76, values [0, 16)
                    const float c_hi = corr[h][m].y * -0x1p-71f;  // values [16, 32) of the group
#pragma unroll
                    for (int i = 0; i < VH / 2; i++) {
                        const float c = (VH == 32 && i >= 8) ? c_hi : c_lo;
                        acc[h][m][i] = make_float2(fmaf(acc[h][m][i].x, kQ6Unscale, c),
                                                   fmaf(acc[h][m][i].y, kQ6Unscale, c));
                    }
                    corr[h][m] = make_float2(0.f, 0.f);
                }
            }
        }
        // 2. sum over the 8 warps in a fixed order.  Small tiles: every warp
        //    stores its slot and step 3 adds the 8 slots.  Large tiles
        //    (kRedSlots slots only): w += w + 4, then w += w + 2, and warps
        //    0 and 1 leave the two halves in slots 0 and 1.
        if constexpr (kFlatRed) {
            store_red(warp);
        } else {
            if (warp >= 4) store_red(warp - 4);
            named_bar_sync(1, kNW * 32);
            if (warp < 4) add_red(warp);
            named_bar_sync(1, kNW * 32);
            if (warp >= 2 && warp < 4) store_red(warp - 2);
            named_bar_sync(1, kNW * 32);
            if (warp < 2) add_red(warp);
            named_bar_sync(1, kNW * 32);
            if (warp < 2) store_red(warp);
        }
#pragma unroll
        for (int h = 0; h < H; h++) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
#pragma unroll
                for (int i = 0; i < VH / 2; i++) acc[h][m][i] = make_float2(0.f, 0.f);
            }
        }
        const bool whole = (tile * K >= f0) && ((tile + 1) * K <= f1);
        named_bar_sync(1, kNW * 32);
        // 3. the slots added in order, stored coalesced
        const int64_t n0 = tile * TN;
        const int ncols = (int)imin64(TN, N - n0);
        const int slot = (tile == first_tile) ? 0 : 1;
        for (int idx = tid; idx < MR * TN; idx += kNW * 32) {
            const int m = idx / TN, c = idx % TN;
            if (m >= p.M || c >= ncols) continue;
            const int L = c / VPT, i = (c % VPT) / 4;
            const int phys = L * VPT + 4 * (i ^ red_swz<VPT>(L)) + (c & 3);
            float sum = red[m * TN + phys] + red[(MR + m) * TN + phys];
            if constexpr (kFlatRed) {
#pragma unroll
                for (int w = 2; w < kNW; w++) sum += red[(w * MR + m) * TN + phys];
            }
            if (whole) {
                if constexpr (G) store_peers(gq, peers_ok, seq, m, n0 + c, sum);
                else p.y[(int64_t)m * N + n0 + c] = sum;
            }
            else p.partials[(((int64_t)blockIdx.x * 2 + slot) * MR + m) * TN + c] = sum;
        }
        named_bar_sync(1, kNW * 32);
        // A tile shared with other CTAs (only the first and the last tile of
        // this CTA's rows): count this CTA in at once (thread 0 keeps the
        // counter's old value; the atomic's latency overlaps the rows that
        // follow), and sum after this CTA's last row, when the accumulators
        // are free.
        if (!whole) {
            __threadfence();
            named_bar_sync(1, kNW * 32);
            if (tid == 0) {
                const int64_t g = blockIdx.x / p.group;
                const int old = atomicAdd(p.counters + p.ntiles + tile + g, 1);
                if (tile == first_tile) old_first = old;
                else old_last = old;
            }
            if (tile == first_tile) pend_first = true;
            else pend_last = true;
        }
    };

    // Split-K sum of a shared tile, in two levels so that no CTA reads more
    // than about `group` partial rows: the CTAs of the tile are cut into
    // groups of p.group consecutive CTAs; the last CTA of a group to get here
    // adds the group's partials in CTA order, and the last group to finish
    // adds the group sums in group order (deterministic).  A tile whose CTAs
    // all lie in one group is finished by the first level.
    auto sum_rows = [&](int64_t tile, auto src, int count, auto sink) {
        const int64_t n0 = tile * TN;
        const int ncols = (int)imin64(TN, N - n0);
        for (int idx4 = tid; idx4 < MR * TN / 4; idx4 += kNW * 32) {
            const int m = (idx4 * 4) / TN, c = (idx4 * 4) % TN;
            if (m >= p.M || c >= ncols) continue;
            float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j0 = 0; j0 < count; j0 += kCombineLoads) {
                float4 v[kCombineLoads];
#pragma unroll
                for (int u = 0; u < kCombineLoads; u++)
                    if (j0 + u < count) v[u] = __ldcg(reinterpret_cast<const float4 *>(src(j0 + u) + (size_t)m * TN + c));
#pragma unroll
                for (int u = 0; u < kCombineLoads; u++) {
                    if (j0 + u < count) {
                        acc4.x += v[u].x; acc4.y += v[u].y; acc4.z += v[u].z; acc4.w += v[u].w;
                    }
                }
            }
            sink(m, c, acc4);
        }
    };
    auto to_output = [&](int64_t tile) {
        const int64_t n0 = tile * TN;
        const bool peers = peers_ok;
        return [=, &gq, &p](int m, int c, float4 v) {
            if constexpr (G) {
                store_peers4(gq, peers, seq, m, n0 + c, v);
            } else {
                float *yo = p.y + (int64_t)m * N + n0 + c;
                yo[0] = v.x; yo[1] = v.y; yo[2] = v.z; yo[3] = v.w;
            }
        };
    };
    auto combine = [&](int64_t tile, int old1) {  // old1: thread 0's first-level count
        const int64_t cf = (tile * K) / p.rpc;
        const int64_t cl = imin64(((tile + 1) * K - 1) / p.rpc, p.grid - 1);
        const int64_t gl = cf / p.group, gh = cl / p.group, g = blockIdx.x / p.group;
        const int64_t c_lo = cf > g * p.group ? cf : g * p.group;
        const int64_t c_hi = imin64(cl, g * p.group + p.group - 1);
        int *cnt1 = p.counters + p.ntiles + tile + g;
        named_bar_sync(1, kNW * 32);
        if (tid == 0) flag[0] = (old1 == (int)(c_hi - c_lo));
        named_bar_sync(1, kNW * 32);
        if (!flag[0]) return;
        __threadfence();
        // a CTA holds this tile in slot 0 if the tile is its first, else in
        // slot 1: only CTA cf can start before the tile
        const bool cf_slot1 = cf * p.rpc < tile * K;
        auto part = [&](int j) {
            const int64_t cta = c_lo + j;
            const int sl = (cta == cf && cf_slot1) ? 1 : 0;
            return p.partials + (size_t)(cta * 2 + sl) * MR * TN;
        };
        const int n1 = (int)(c_hi - c_lo + 1);
        if (gl == gh) {
            sum_rows(tile, part, n1, to_output(tile));
            named_bar_sync(1, kNW * 32);
            if (tid == 0) atomicExch(cnt1, 0);
            return;
        }
        float *gdst = p.gpartials + (size_t)(tile + g) * MR * TN;
        sum_rows(tile, part, n1, [&](int m, int c, float4 v) {
            *reinterpret_cast<float4 *>(gdst + (size_t)m * TN + c) = v;
        });
        __threadfence();
        named_bar_sync(1, kNW * 32);
        if (tid == 0) {
            atomicExch(cnt1, 0);
            flag[0] = (atomicAdd(&p.counters[tile], 1) == (int)(gh - gl));
        }
        named_bar_sync(1, kNW * 32);
        if (!flag[0]) return;
        __threadfence();
        auto gpart = [&](int j) { return p.gpartials + (size_t)(tile + gl + j) * MR * TN; };
        sum_rows(tile, gpart, (int)(gh - gl + 1), to_output(tile));
        named_bar_sync(1, kNW * 32);
        if (tid == 0) atomicExch(&p.counters[tile], 0);
    };

    // this warp's next row j: CTA-local index pl, its ring slot / phase
    int pl = warp;
    int nb32 = (int)next_boundary;
    int slot = 0;
    uint32_t phase = 0;
    int islot = ji % S;  // ring slot of the next row to stream

    // Decode row j (its parameters sit in lane j % 32 of the current batch)
    // from ring slot sl.
    auto decode_row = [&](int jj, int sl) {
        float xv[MR];
#pragma unroll
        for (int m = 0; m < MR; m++) xv[m] = __shfl_sync(0xffffffffu, xcur[m], jj);
        const uint32_t n0 = __shfl_sync(0xffffffffu, c_n0, jj);
        const uint32_t v0 = __shfl_sync(0xffffffffu, c_v0, jj);
        if (n0 + lane * VPT < Nu) {
            const uint32_t lead = (((v0 >> 8) & 15u) * (uint32_t)B) & 15u;
            const uint32_t wl = (v0 & 255u) + lane * VPT;
            const uint32_t row = my_ring_u32 + (uint32_t)(sl * p.row_cap) + lead;
#pragma unroll
            for (int h = 0; h < H; h++) {
                const uint32_t wh = wl + h * VH;
                // (N is a multiple of 32: a lane's second group may lie past N)
                if (h == 0 || n0 + lane * VPT + h * VH < Nu)
                    decode_accum<QT, MR, VH>(row + (wh >> 8) * B, (int)(wh & 255u), xv, acc[h], corr[h]);
            }
        }
    };

    for (int j = 0; j < nw;) {
        while (pl >= nb32) {
            flush(cur_tile);
            cur_tile++;
            nb32 += (int)K;
        }
        // Two rows at a time when both lie in the current tile and in the
        // current parameter batch: one straight run of decode code for both
        // (more independent work in flight, loop costs shared).
        const int jj = j & 31;
        const bool pair = (j + 1 < nw) && (pl + kNW < nb32) && (jj != 31);
        if (!mbar_wait_bounded(smem_u32addr(&my_full[slot]), phase, kWaitNs)) set_status(kStatusTimeout);
        int used = 1;
        if (pair) {
            const int slot1 = slot + 1 == S ? 0 : slot + 1;
            const uint32_t phase1 = slot + 1 == S ? phase ^ 1u : phase;
            if (!mbar_wait_bounded(smem_u32addr(&my_full[slot1]), phase1, kWaitNs)) set_status(kStatusTimeout);
            decode_row(jj, slot);
            decode_row(jj + 1, slot1);
            used = 2;
        } else {
            decode_row(jj, slot);
        }
        j += used;
        pl += used * kNW;
        slot += used;
        if (slot >= S) {
            slot -= S;
            phase ^= 1u;
        }
        if ((j & 31) == 0 && j < nw) {  // next batch of 32 rows
#pragma unroll
            for (int m = 0; m < MR; m++) xcur[m] = xnext[m];
            load_x(j + 32, xnext);
            decode_batch(j);
        }
        // Refill the slots of all but the last decoded row (every lane has
        // long finished reading them): up to S - 1 rows ahead.
        __syncwarp();
        while (ji < nw && ji < j - 1 + S) {
            issue_next(islot);
            if (++islot == S) islot = 0;
        }
    }
    while (cur_tile <= last_tile) {
        flush(cur_tile);
        cur_tile++;
    }
    if (pend_first) combine(first_tile, old_first);
    if (pend_last) combine(last_tile, old_last);
    // All-gather: the other ranks' columns from this rank's slots into its
    // output (every thread of the grid takes a share), then the last CTA to
    // finish records the call number.
    if (G && gq.world > 1) {
        if (peers_ok) {
            const int64_t n_all = gq.y_ld, rest = n_all - N;
            const int64_t total = (int64_t)p.M * rest;
            int bad = 0;
            for (int64_t e = (int64_t)blockIdx.x * kThreads + tid; e < total && bad == 0;
                 e += (int64_t)p.grid * kThreads) {
                const int64_t m = e / rest, j = e % rest, n = j < gq.col_off ? j : j + N;
                float v;
                bad = wait_slot(channel_slot(gq.peer_flags[gq.rank], n_all, m, n, seq), seq, gq.wait_ns,
                                &gq.sync[2], &v);
                if (bad == 0) gq.peer_y[gq.rank][m * n_all + n] = v;
            }
            // the first thread to find a fault reports it and marks the
            // channel failed, which stops every other waiting thread
            if (bad > 0 && atomicExch(&gq.sync[2], 1u) == 0u) set_status(bad);
        }
        named_bar_sync(1, kNW * 32);
        if (tid == 0) {
            const unsigned old = atomicAdd(&gq.sync[1], 1u);
            if (old == (unsigned)p.grid - 1u) {  // every CTA has read this call's number
                gq.sync[1] = 0u;
                gq.sync[0] = seq;
            }
        }
    }
}

// -------- generic path (N % 32 != 0): one thread per output column ---------
template <int QT>
__device__ __forceinline__ float value_at(const uint8_t *blk, int i) {
    if constexpr (QT == kQ6K) {
        uint32_t lo = blk[i >> 1];
        lo = (i & 1) ? (lo >> 4) : (lo & 0x0Fu);
        uint32_t hi = (blk[128 + (i >> 2)] >> ((i & 3) * 2)) & 3u;
        float d = hw_f16_to_f32(blk[208] | (uint32_t)blk[209] << 8);
        return d * (float)(int8_t)blk[192 + (i >> 4)] * (float)((int)(lo | hi << 4) - 32);
    } else {
        float d = hw_f16_to_f32(blk[0] | (uint32_t)blk[1] << 8);
        float dmin = hw_f16_to_f32(blk[2] | (uint32_t)blk[3] << 8);
        const int sb = i >> 5, g = sb >> 2, sh = 6 * (sb & 3);
        const uint8_t *s = blk + 4;
        uint32_t a = s[3 * g] | (uint32_t)s[3 * g + 1] << 8 | (uint32_t)s[3 * g + 2] << 16;
        uint32_t b = s[6 + 3 * g] | (uint32_t)s[7 + 3 * g] << 8 | (uint32_t)s[8 + 3 * g] << 16;
        const uint8_t *qs = blk + (QT == kQ4K ? 16 : 48);
        uint32_t q = qs[i >> 1];
        q = (i & 1) ? (q >> 4) : (q & 0x0Fu);
        if constexpr (QT == kQ5K) q |= ((blk[16 + (i >> 3)] >> (i & 7)) & 1u) << 4;
        return d * (float)((a >> sh) & 63u) * (float)q - dmin * (float)((b >> sh) & 63u);
    }
}

template <int QT>
__global__ void __launch_bounds__(128) gemv_generic_kernel(const uint8_t *__restrict__ w, const float *__restrict__ x,
                                                           float *__restrict__ y, int64_t K, int64_t N, int M) {
    constexpr int B = QT_<QT>::BYTES;
    pdl_wait();
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t k = 0; k < K; k++) {
        const int64_t v = k * N + n;
        const float wv = value_at<QT>(w + (v >> 8) * B, (int)(v & 255));
#pragma unroll
        for (int m = 0; m < 8; m++)
            if (m < M) acc[m] = fmaf(__ldg(x + (int64_t)m * K + k), wv, acc[m]);
    }
    for (int m = 0; m < M; m++) y[(int64_t)m * N + n] = acc[m];
}

// ------------------------------- host side -------------------------------
struct Plan {
    int mr, vpt, tn;
    int ntiles, grid, stages, row_cap;
    int64_t rpc;
    size_t smem;
    int group, ngroups;  // CTAs per first-level split-K group, and the group count
    size_t part1_bytes, partial_bytes, counter_bytes;
    bool generic;
};

static int block_bytes(int qt) { return qt == kQ4K ? 144 : qt == kQ5K ? 176 : 210; }

static Plan make_plan(const GemvShape &s, int device) {
    Plan pl{};
    // the fast path keeps byte offsets of the weight in 32 bits
    const int64_t wbytes = ((s.K * s.N + 255) / 256) * block_bytes(s.qtype);
    pl.generic = (s.N % 32) != 0 || wbytes >= (int64_t(1) << 32) - 4096;
    if (pl.generic) return pl;
    if (s.M <= 1) {
        // 64 values per lane (2048-column tiles) halve the per-row work and
        // the bulk copies per value; taken when the ragged last tile wastes
        // little and there are enough tiles to keep the split-K fan-in low
        const int64_t nt64 = (s.N + 2047) / 2048;
        const bool wide = nt64 >= 12 && (nt64 * 2048 - s.N) * 25 <= s.N;
        pl.mr = 1;
        pl.vpt = wide ? 64 : 32;
    } else if (s.M <= 2) { pl.mr = 2; pl.vpt = 32; }
    else if (s.M <= 4) { pl.mr = 4; pl.vpt = 16; }
    else { pl.mr = 8; pl.vpt = 8; }
    pl.tn = 32 * pl.vpt;
    if ((s.N + pl.tn - 1) / pl.tn > (int64_t)(kWorkspaceCounterHead / 4)) {
        pl.generic = true;  // more tile counters than the workspace head holds
        return pl;
    }
    pl.ntiles = (int)((s.N + pl.tn - 1) / pl.tn);
    const int64_t rows_total = (int64_t)pl.ntiles * s.K;
    if (rows_total >= (int64_t(1) << 31) || s.N >= (int64_t(1) << 31)) {
        pl.generic = true;  // row indices and columns are kept in 32 bits
        return pl;
    }
    const int sms = device_sm_count(device);
    int64_t grid = (int64_t)sms * 2;
    if (grid > rows_total) grid = rows_total;
    pl.rpc = (rows_total + grid - 1) / grid;
    pl.grid = (int)((rows_total + pl.rpc - 1) / pl.rpc);
    const int B = block_bytes(s.qtype);
    pl.row_cap = (((pl.tn / 256 + 1) * B + 16 + 16) + 15) & ~15;
    const size_t red = (size_t)(flat_reduction(pl.mr, pl.vpt) ? kNW : kRedSlots) * pl.mr * pl.tn * 4;
    auto smem_for = [&](int st) {
        return (size_t)(((8 * kNW * st + 8) + 127) & ~127) + (size_t)kNW * st * pl.row_cap + red;
    };
    int stages = kMaxStages;
    while (stages > kMinStages && smem_for(stages) > (size_t)kSmemPerCta) stages--;
    pl.stages = stages;
    pl.smem = smem_for(stages);
    // split-K: a tile is shared by up to ceil(K / rpc) + 1 CTAs; above
    // kMaxFanIn the sum goes through groups of kGroup CTAs
    const int64_t fan_in = (s.K + pl.rpc - 1) / pl.rpc + 1;
    pl.group = fan_in > kMaxFanIn ? kGroup : pl.grid;
    pl.ngroups = (pl.grid + pl.group - 1) / pl.group;
    if (2 * (int64_t)pl.ntiles + pl.ngroups > (int64_t)(kWorkspaceCounterHead / 4)) {
        pl.generic = true;  // more split-K counters than the workspace head holds
        return pl;
    }
    pl.part1_bytes = ((size_t)pl.grid * 2 * pl.mr * pl.tn * 4 + 255) & ~size_t(255);
    const size_t gpart = pl.group < pl.grid ? (size_t)(pl.ntiles + pl.ngroups) * pl.mr * pl.tn * 4 : 0;
    pl.partial_bytes = pl.part1_bytes + ((gpart + 255) & ~size_t(255));
    pl.counter_bytes = ((size_t)(2 * pl.ntiles + pl.ngroups) * 4 + 255) & ~size_t(255);
    return pl;
}

// Which kernel serves a plain GEMV (vkq_set_gemv_path): 0 chooses, 1 the
// CUDA-core kernel of this file, 2 the tensor-core kernel (gemv_tc.cu), 3 the
// column-strip kernel (gemv_strip.cu); a kernel that does not serve the shape
// leaves the choice to the automatic order.
static int g_gemv_path = 0;

int set_gemv_path(int path) {
    const int old = g_gemv_path;
    g_gemv_path = path;
    return old;
}

// The tensor-core kernel serves weights whose rows start on super-block
// boundaries (N % 256 == 0: every 256-column tile is one block per row);
// rows that straddle blocks (the vocabulary projection, N % 256 == 128) are
// the CUDA-core kernel's, which streams whole row chunks.
static bool use_tensor_cores(const GemvShape &s, int device) {
    if (g_gemv_path == 1 || s.N % 256 != 0) return false;
    // single-row Q6_K (the 11008 -> 2048 down projection: 16.7 us here
    // against 18.5 us on tensor cores) stays on the CUDA cores
    if (g_gemv_path == 0 && s.qtype == kQ6K && s.M == 1) return false;
    return gemv_tc_fits(s, TcLayout{s.N, 0, 0}, device);
}

// Single-row Q4_K GEMVs with N % 256 == 0 go to the column-strip kernel (no
// workspace, no cross-CTA sums; as fast as the tensor-core kernel or faster
// on every 3B and 14B layer shape measured), M = 2..4 to the tensor-core
// kernel, unless a kernel is selected.  (Weight pointers are 16-byte
// aligned: the entry points check it.)
static bool use_strips(const GemvShape &s, int device) {
    if (g_gemv_path == 1 || g_gemv_path == 2 || s.N % 256 != 0) return false;
    if (g_gemv_path == 0 && s.M != 1) return false;
    return gemv_strip_fits(s, StripLayout{s.N, 0}, device);
}

// Enough workspace for whichever kernel serves the shape (the CUDA-core
// and tensor-core kernels check their own need; the column-strip kernel
// needs none).
size_t gemv_workspace_bytes(const GemvShape &s, int device) {
    Plan pl = make_plan(s, device);
    const size_t simt = pl.generic ? 0 : kWorkspaceCounterHead + pl.partial_bytes;
    const size_t tc = gemv_tc_workspace_bytes(s, TcLayout{s.N, 0, 0}, device);
    return simt > tc ? simt : tc;
}

template <int QT, int MR, int VPT, bool G>
static cudaError_t launch_fast(const GemvParams &gp, const GatherParams &gq, const Plan &pl, cudaStream_t stream) {
    auto kern = gemv_kernel<QT, MR, VPT, G>;
    // two CTAs per SM need the largest shared-memory carveout
    cudaError_t e = kernel_smem((const void *)kern, pl.smem, true);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, gp, gq);
}

template <int QT>
static cudaError_t dispatch_mr(const GemvParams &gp, const GatherParams &gq, const Plan &pl, cudaStream_t st) {
    const bool gather = gq.world > 0;
    switch (pl.mr) {
    case 1:
        if (pl.vpt == 64)
            return gather ? launch_fast<QT, 1, 64, true>(gp, gq, pl, st) : launch_fast<QT, 1, 64, false>(gp, gq, pl, st);
        return gather ? launch_fast<QT, 1, 32, true>(gp, gq, pl, st) : launch_fast<QT, 1, 32, false>(gp, gq, pl, st);
    case 2: return gather ? launch_fast<QT, 2, 32, true>(gp, gq, pl, st) : launch_fast<QT, 2, 32, false>(gp, gq, pl, st);
    case 4: return gather ? launch_fast<QT, 4, 16, true>(gp, gq, pl, st) : launch_fast<QT, 4, 16, false>(gp, gq, pl, st);
    default: return gather ? launch_fast<QT, 8, 8, true>(gp, gq, pl, st) : launch_fast<QT, 8, 8, false>(gp, gq, pl, st);
    }
}

int gemv_launch(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y, void *ws,
                size_t ws_bytes, cudaStream_t stream, int device, const GatherArgs *gather) {
    if (!gather && use_strips(s, device))
        return gemv_strip_launch(s, StripLayout{s.N, 0}, w, w_bytes, x, y, s.N, 0, stream, device);
    // the all-gather of a Q4_K shard with block-aligned rows: column strips
    if (gather && g_gemv_path != 1 && g_gemv_path != 2 && s.qtype == kQ4K && s.M <= 4 &&
        gemv_strip_gather_fits(s, *gather, device))
        return gemv_strip_gather(s, w, w_bytes, x, *gather, stream, device);
    if (!gather && use_tensor_cores(s, device))
        return gemv_tc_launch(s, TcLayout{s.N, 0, 0}, w, w_bytes, x, y, s.N, ws, ws_bytes, stream, device);
    Plan pl = make_plan(s, device);
    cudaError_t e;
    if (pl.generic && gather) {
        set_error("the all-gather GEMV needs a shard width that is a multiple of 32 (got %lld)", (long long)s.N);
        return 2;
    }
    if (pl.generic) {
        const uint8_t *wp = static_cast<const uint8_t *>(w);
        dim3 grid((unsigned)((s.N + 127) / 128));
        switch (s.qtype) {
        case kQ4K: gemv_generic_kernel<kQ4K><<<grid, 128, 0, stream>>>(wp, x, y, s.K, s.N, (int)s.M); break;
        case kQ5K: gemv_generic_kernel<kQ5K><<<grid, 128, 0, stream>>>(wp, x, y, s.K, s.N, (int)s.M); break;
        default: gemv_generic_kernel<kQ6K><<<grid, 128, 0, stream>>>(wp, x, y, s.K, s.N, (int)s.M); break;
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) {
            set_error("gemv (generic) launch failed: %s", cudaGetErrorString(e));
            return 5;
        }
        return 0;
    }
    const size_t need = kWorkspaceCounterHead + pl.partial_bytes;
    if (ws == nullptr || ws_bytes < need) {
        set_error("gemv needs a workspace of %zu bytes (got %zu)", need, ws_bytes);
        return 4;
    }
    GemvParams gp{};
    gp.w = static_cast<const uint8_t *>(w);
    gp.w_bytes = w_bytes;
    gp.w_floor16 = w_bytes & ~int64_t(15);
    gp.x = x;
    gp.y = y;
    gp.K = s.K;
    gp.N = s.N;
    gp.M = (int)s.M;
    gp.ntiles = pl.ntiles;
    gp.grid = pl.grid;
    gp.rows_total = (int64_t)pl.ntiles * s.K;
    gp.rpc = pl.rpc;
    gp.counters = static_cast<int *>(ws);
    // partials after the fixed counter head: a later call with more tiles
    // must find its counters at zero, never overwritten by these partials
    gp.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kWorkspaceCounterHead);
    gp.gpartials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + kWorkspaceCounterHead + pl.part1_bytes);
    gp.group = pl.group;
    gp.row_cap = pl.row_cap;
    gp.stages = pl.stages;
    GatherParams gq{};
    gq.world = 0;  // 0: the plain kernel
    if (gather) {
        if (gather->world < 1 || gather->world > kMaxPeers) {
            set_error("the all-gather serves 1 to %d ranks (got %d)", kMaxPeers, gather->world);
            return 1;
        }
        for (int r = 0; r < gather->world; r++) {
            gq.peer_y[r] = gather->peer_y[r];
            gq.peer_flags[r] = gather->peer_flags[r];
        }
        gq.sync = gather->sync;
        gq.world = gather->world;
        gq.rank = gather->rank;
        gq.y_ld = gather->y_ld;
        gq.col_off = gather->col_off;
        gq.rs = gather->rs;
        gq.ld = gather->ld;
        gq.n_base = gather->n_base;
        gq.wait_ns = gather->wait_ns;
    }
    switch (s.qtype) {
    case kQ4K: e = dispatch_mr<kQ4K>(gp, gq, pl, stream); break;
    case kQ5K: e = dispatch_mr<kQ5K>(gp, gq, pl, stream); break;
    default: e = dispatch_mr<kQ6K>(gp, gq, pl, stream); break;
    }
    if (e != cudaSuccess) {
        set_error("gemv launch failed: %s", cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

// ---- fixed device-resident scratch (vkq_gemv_noalloc) ----------------------
// For callers that cannot allocate device memory themselves, the split-K
// partial sums and tile counters can live in this file-scope array instead of
// a caller-provided workspace.  It is part of the module image, so every GPU
// that loads the library keeps these bytes until the process exits.  In host
// code the name g_gemv_scratch is only a stand-in for the symbol; the device
// address comes from cudaGetSymbolAddress, looked up once per device.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) uint8_t g_gemv_scratch[kNoAllocScratchBytes];

static void *noalloc_scratch_address(int device) {
    static std::mutex mu;
    static void *addr[64] = {nullptr};
    int dev = device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    if (dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (addr[dev] == nullptr) {
        void *ptr = nullptr;
        // the device is current here (the entry point made it so)
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemv_scratch);
        if (e != cudaSuccess) {
            set_error("cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = ptr;
    }
    return addr[dev];
}

int gemv_launch_noalloc(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y,
                        cudaStream_t stream, int device) {
    if (use_strips(s, device)) return gemv_launch(s, w, w_bytes, x, y, nullptr, 0, stream, device);
    Plan pl = make_plan(s, device);
    const bool tc = use_tensor_cores(s, device);
    if (pl.generic && !tc) return gemv_launch(s, w, w_bytes, x, y, nullptr, 0, stream, device);
    const size_t need = gemv_workspace_bytes(s, device);
    if (need > kNoAllocScratchBytes) {
        set_error("this GEMV needs %zu bytes of scratch; the fixed scratch of vkq_gemv_noalloc holds %zu", need,
                  kNoAllocScratchBytes);
        return 4;
    }
    void *base = noalloc_scratch_address(device);
    if (base == nullptr) {
        if (vkq_last_error_empty()) set_error("cannot locate the fixed scratch on device %d", device);
        return 5;
    }
    // the tile counters must start at zero; the array keeps the last call's bytes
    const size_t tc_counters = (size_t)((s.N + 255) / 256) * 16;
    const size_t clear = tc && tc_counters > pl.counter_bytes ? tc_counters : pl.counter_bytes;
    cudaError_t e = cudaMemsetAsync(base, 0, clear, stream);
    if (e != cudaSuccess) {
        set_error("clearing the fixed scratch: %s", cudaGetErrorString(e));
        return 5;
    }
    return gemv_launch(s, w, w_bytes, x, y, base, kNoAllocScratchBytes, stream, device);
}

int gemv_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(int));
    return v;
}

}  // namespace vkq
