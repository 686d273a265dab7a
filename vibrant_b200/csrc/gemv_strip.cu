// gemv_strip.cu -- Q4_K dequantize + GEMV in column strips on sm_100a, for
// weights whose stored rows start on a super-block boundary (the N % 256 == 0
// layers of a transformer and their row-block shards), with the fused forms
// of a decode step's linears: several weights over one input (q, k and v),
// gate and up with a SiLU(gate) * up epilogue, and an RMSNorm prologue.
//
// y[m][n] = sum_k h[m][k] * W[k][n], 1 <= M <= 4, fp32 accumulate, with the
// per-value arithmetic of the CUDA-core GEMV in gemv.cu: the weight
// w = (d*sc)*q - dmin*m is formed with one rounding, then h*w accumulated.
// h = x, or with the prologue h = x / sqrt(mean(x^2) + eps) * g (the
// reference's rms_norm_f32, internal/gpu/cuda/kernels.cu:209-288, applied by
// internal/transformer/layer.go before attention and before the FFN): the
// product is linear in h, so the kernel accumulates (x*g)*w and multiplies
// each output by 1/rms, the sum of squares coming from the x values the
// kernel reads anyway.
// Q4_K layout (internal/tensor/quant_q4k.go:137-157, values as in
// DequantizeQ4_K, quant_q4k.go:37-79): d, dmin (f16), 12 bytes of 6-bit
// scales and mins in four little-endian 24-bit groups (sc[0..3], sc[4..7],
// m[0..3], m[4..7]), then 128 bytes of quants, value v in byte v/2 (low
// nibble for even v).  A 32-value sub-block is therefore 16 contiguous quant
// bytes under one (scale, min) pair.
//
// Design (HBM-bound; algorithmic bytes per call = weights + x + y):
//  * A lane-column is V consecutive output columns of one weight: one
//    sub-block (V = 32, 16 quant bytes; M <= 2) or half of one (V = 16,
//    8 bytes; M >= 3).  The lane-columns of all the launch's weights, in
//    order (or gate and up alternating, for the SiLU epilogue), are dealt out
//    in contiguous runs to column groups.  A group is one CTA, or a
//    thread-block cluster of S CTAs that split K into S ranges and add their
//    sums through distributed shared memory: no partial sum leaves the SM, so
//    there is no global workspace, atomic or memory fence, and small matrices
//    finish in one pass of the machine.
//  * Thread t of a CTA owns lane-column t % nlc of its group and every R-th
//    row (R = 512 / nlc) of the CTA's k range.  Per row it copies the
//    16-byte block header, its quant bytes, x[m][k] (and g[k]) into a ring of
//    kStripDepth slots of its own in shared memory with cp.async (L2 256-byte
//    prefetch), kStripDepth rows ahead of their use: the bytes in flight take
//    no registers, and as each thread reads only its own slots, no barrier is
//    needed (cp.async.wait_group per thread).  Lanes of one warp take
//    adjacent lane-columns, so a warp's copies cover contiguous runs of each
//    row.  The first rows' weight bytes are requested before
//    griddepcontrol.wait (the weights do not depend on the preceding kernel;
//    x and y do).
//  * Per row: d and dmin, the sub-block's 6-bit scale and min (one funnel
//    shift each out of the header words), then per pair of values one byte
//    permute per value and two packed fp32x2 FMAs (w, then h*w; the quant is
//    used as the subnormal float q * 2^-149 with the multipliers scaled by
//    powers of two, exactly as in gemv.cu).
//  * Sums: the CTA's threads add through shared memory in a fixed order
//    (rows strided over threads, then the strides), the cluster's CTAs
//    through DSMEM in CTA-rank order, so results are run-to-run identical.
//  * Row-sharded all-gather (weight 0, or the gate|up pair; further weights
//    stay whole and local, as k and v of a sharded q): the launch computes
//    this rank's columns from its row-block shard and sends each value to
//    every other rank as one 64-bit store of (call number, value bits) into
//    that rank's channel slots (peer.cuh); then every thread of the grid
//    polls a share of this rank's slots for the other ranks' columns of this
//    call and copies them into the output.  No fence, no "started" or
//    "done" flag: the slot carries its own call number, and two parities per
//    element suffice because no rank can be two calls ahead of another.  A wait that runs out
//    or a slot of a later call marks the channel failed (sticky); a failed
//    channel sends and waits no more and keeps the launch to its own columns.
#include <cstdint>
#include <mutex>

#include "kq_device.cuh"
#include "peer.cuh"
#include "vkq_internal.h"

namespace vkq {

static __device__ int g_strip_status;
__device__ __forceinline__ void strip_status(int code) { atomicExch(&g_strip_status, code); }

constexpr int kStripThreads = 512;  // one CTA per SM
constexpr int kStripMaxCluster = 8;
// Rows in flight per thread.  Measured on the 3B/14B shapes with 8, 6, 4, 3
// and 2: the shallowest ring was fastest nearly everywhere (2048 -> 11008:
// 13.6 -> 10.7 us; 3B decode step 496 -> 529 tokens/s) -- a smaller prologue
// on the critical path of CTAs that start late, and more of the SM's memory
// left to L1.
constexpr int kStripDepth = 2;
constexpr int kStripSlot = 48;      // ring slot: header [0,16), quants [16,32), x[0..M) then g [32,48)

// Multipliers of the subnormal-quant form (the values gemv.cu uses).
constexpr float kStripScale = 0x1p100f;   // d*sc
constexpr float kStripDown = 0x1p-49f;    // -dmin*m
constexpr float kStripXScale = 0x1p49f;   // x

struct StripSegP {
    const uint8_t *w;  // stored rows of row_bytes each
    float *y;          // [M][y_ld], columns from col_off
    int64_t row_bytes, y_ld, col_off;
    int c0;            // in-block position of the weight's first column (multiple of V)
    int lane_end;      // one past the weight's last lane-column in the launch's lane order
};

// The all-gather channel of a launch (world == 0: none).
struct StripGatherP {
    unsigned *peer_flags[kMaxRanks];  // every rank's channel buffer (addresses valid on this device)
    unsigned *sync;                   // this rank's channel words
    int world, rank;
    uint64_t wait_ns;
};

struct StripParams {
    StripSegP seg[kMaxStripSegs];
    const float *x;       // [M][K]
    const float *norm_w;  // RMSNorm weight g[K], or null
    int64_t K, k_per;     // k_per: rows per cluster rank
    float eps;
    int nseg;
    int silu;             // 1: lanes alternate gate (seg 0) and up (seg 1); y0 = SiLU(gate) * up
    int lanes;            // lane-columns of the launch
    int groups;           // column groups
    int unit;             // lane-columns per indivisible unit (2 for the SiLU pairs)
    int S;                // CTAs per cluster
};

// cp.async global -> shared of 16, 8 or 4 bytes; the 16- and 8-byte copies
// ask L2 to fetch the whole 256-byte sector group (the neighbouring
// lane-columns of other CTAs read the rest of it).
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global.L2::256B [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// The cluster's sum of one shared-memory float, in CTA-rank order.
__device__ __forceinline__ float cluster_sum(const float *local, int S) {
    if (S == 1) return *local;
    float s = ld_dsmem(local, 0);
    for (int r = 1; r < S; r++) s += ld_dsmem(local, (uint32_t)r);
    return s;
}

// Sum of n floats a[0], a[stride], ... in four interleaved partial sums (the
// loads of one pass are independent, so they overlap instead of waiting on
// each other); a fixed order for a given n.
__device__ __forceinline__ float strided_sum(const float *a, int n, int stride) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
        s0 += a[(i + 0) * stride];
        s1 += a[(i + 1) * stride];
        s2 += a[(i + 2) * stride];
        s3 += a[(i + 3) * stride];
    }
    for (; i < n; i++) s0 += a[i * stride];
    return (s0 + s1) + (s2 + s3);
}

// Weight and in-weight lane-column of launch lane-column gl.
__device__ __forceinline__ void strip_lane(const StripParams &p, int gl, int &si, int &ll) {
    if (p.silu) {
        si = gl & 1;
        ll = gl >> 1;
        return;
    }
    int start = 0;
    si = 0;
    while (si + 1 < p.nseg && gl >= p.seg[si].lane_end) {
        start = p.seg[si].lane_end;
        si++;
    }
    ll = gl - start;
}

// The quant words of one lane-column row (V / 8 words of 8 values), read
// from a ring slot.
template <int V> struct QWords;
template <> struct QWords<32> {
    uint4 v;
    __device__ __forceinline__ void read(uint32_t a) { v = lds128(a); }
    __device__ __forceinline__ uint32_t operator[](int i) const {
        return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    }
};
template <> struct QWords<16> {
    uint2 v;
    __device__ __forceinline__ void read(uint32_t a) { v = lds64(a); }
    __device__ __forceinline__ uint32_t operator[](int i) const { return i == 0 ? v.x : v.y; }
};

template <int M> constexpr int strip_v() { return M <= 2 ? 32 : 16; }

template <int M>
__global__ void __launch_bounds__(kStripThreads, 1) gemv_strip_kernel(const StripParams p, const StripGatherP gq) {
    constexpr int V = strip_v<M>();
    constexpr int D = kStripDepth;
    constexpr int MV = M * V;
    constexpr int RS = MV + 4;  // padded row of the sums buffer (see below)
    constexpr int NP = V / 2;   // value pairs per lane-column
    // ring[D][kStripThreads] slots during the main loop; afterwards the same
    // bytes hold red[kStripThreads][RS] and red2[kStripThreads]
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float ssq_cta[4];  // this CTA's share of sum_k x[m][k]^2 (RMSNorm prologue)
    __shared__ unsigned chan[2];  // all-gather: this call's number; 2 unchecked, 1 peers ok, 0 own buffer only
    float *red = reinterpret_cast<float *>(smem);
    float *red2 = red + kStripThreads * RS;

    const int t = threadIdx.x;
    const int S = p.S;
    const bool norm = p.norm_w != nullptr;
    const int crank = S > 1 ? (int)cluster_ctarank() : 0;
    const int g = (int)(blockIdx.x / (unsigned)S);
    // groups of q + 1 units first, then groups of q: the larger groups start
    // on the SMs that the previous launch frees first, the smaller ones on the
    // SMs its slowest CTAs hold longest
    const int units = p.lanes / p.unit;
    const int uq = units / p.groups, ur = units % p.groups;
    const int lo = (g * uq + (g < ur ? g : ur)) * p.unit;
    const int nlc = (uq + (g < ur ? 1 : 0)) * p.unit;
    const int R = kStripThreads / nlc;  // row groups (threads per lane-column)
    const int lcl = t % nlc, rg = t / nlc;
    const int64_t k0 = (int64_t)crank * p.k_per;
    const int64_t span = (p.K - k0 < p.k_per ? p.K - k0 : p.k_per);
    const int nr = (rg < R && span > rg) ? (int)((span - rg + R - 1) / R) : 0;
    const bool track_ssq = norm && lcl == 0;  // lane-column 0's threads see every row of the range once

    // this thread's lane-column: weight si, block b of its stored row, first value `within`
    int si, ll;
    strip_lane(p, lo + lcl, si, ll);
    const int64_t row_bytes = p.seg[si].row_bytes;
    const int pos = p.seg[si].c0 + ll * V;
    const int64_t b = pos >> 8;
    const int within = pos & 255;
    const int j = within >> 5;  // sub-block
    // 6-bit fields in header words 1..3: scale at bit 24*(j/4) + 6*(j%4), min 48 bits later
    const int o_sc = 24 * (j >> 2) + 6 * (j & 3), o_m = o_sc + 48;
    const bool sc_hi = o_sc >= 32, m_hi = o_m >= 64;
    const uint32_t s_sc = (uint32_t)(o_sc & 31), s_m = (uint32_t)(o_m & 31);
    const int qoff = 16 + (within >> 1);

    const int64_t step = (int64_t)R * row_bytes;
    const uint8_t *pw = p.seg[si].w + (k0 + rg) * row_bytes + b * 144;  // header of the next row to request
    const float *px = p.x + k0 + rg;                                      // x[0][next row]
    const float *pg = norm ? p.norm_w + k0 + rg : nullptr;                // g[next row]
    const uint32_t slot0 = smem_u32addr(smem) + (uint32_t)(t * kStripSlot);
    constexpr uint32_t kSlotStride = kStripThreads * kStripSlot;

    auto request_w = [&](int u) {
        const uint32_t a = slot0 + (uint32_t)u * kSlotStride;
        cp_async_16(a, pw);
        if constexpr (V == 32) cp_async_16(a + 16, pw + qoff);
        else cp_async_8(a + 16, pw + qoff);
        pw += step;
    };
    auto request_x = [&](int u) {
        const uint32_t a = slot0 + (uint32_t)u * kSlotStride + 32;
#pragma unroll
        for (int m = 0; m < M; m++) cp_async_4(a + 4 * m, px + (int64_t)m * p.K);
        px += R;
        if (norm) {
            cp_async_4(a + 4 * M, pg);
            pg += R;
        }
    };
    // prologue: the weight bytes of the first D rows, then (once the
    // preceding kernel is complete) their x; one commit group per row
#pragma unroll
    for (int u = 0; u < D; u++)
        if (u < nr) request_w(u);
    pdl_wait();  // x (and y) may belong to the preceding kernel
    pdl_launch_dependents();
#pragma unroll
    for (int u = 0; u < D; u++) {
        if (u < nr) request_x(u);
        cp_async_commit();
    }
    const bool gather = gq.world > 1;
    if (gather && t == 0) {  // this call's number, and whether the channel failed earlier
        const unsigned seq = *reinterpret_cast<volatile unsigned *>(&gq.sync[0]) + 1u;
        const bool failed = *reinterpret_cast<volatile unsigned *>(&gq.sync[2]) != 0u;
        if (failed) strip_status(kStatusPeer);
        chan[0] = seq;
        chan[1] = failed ? 0u : 1u;
    }

    float2 acc[M][NP];
#pragma unroll
    for (int m = 0; m < M; m++)
#pragma unroll
        for (int i = 0; i < NP; i++) acc[m][i] = make_float2(0.f, 0.f);
    float ssq[M];
#pragma unroll
    for (int m = 0; m < M; m++) ssq[m] = 0.f;

    for (int i0 = 0; i0 < nr; i0 += D) {
#pragma unroll
        for (int u = 0; u < D; u++) {
            if (i0 + u < nr) {
                cp_async_wait<D - 1>();  // row i0 + u (commit group i0 + u) has landed
                const uint32_t a = slot0 + (uint32_t)u * kSlotStride;
                const uint4 h = lds128(a);
                QWords<V> q;
                q.read(a + 16);
                float xr[M];
                const uint4 xq = lds128(a + 32);
                const uint32_t xw[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
                for (int m = 0; m < M; m++) xr[m] = __uint_as_float(xw[m]);
                if (norm) {
                    const float gk = __uint_as_float(M == 1 ? xq.y : M == 2 ? xq.z : xq.w);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        if (track_ssq) ssq[m] = fmaf(xr[m], xr[m], ssq[m]);
                        xr[m] *= gk;
                    }
                }
                if (i0 + u + D < nr) {  // refill this slot with the row D ahead
                    request_w(u);
                    request_x(u);
                }
                cp_async_commit();
                const float d = hw_f16_to_f32(h.x & 0xFFFFu), dmin = hw_f16_to_f32(h.x >> 16);
                const uint32_t sa = sc_hi ? h.z : h.y, sb = sc_hi ? h.w : h.z;
                const uint32_t ma = m_hi ? h.w : h.z, mb = m_hi ? 0u : h.w;
                const float ds = (d * kStripScale) * (float)(__funnelshift_r(sa, sb, s_sc) & 63u);
                const float ndm = (dmin * -kStripDown) * (float)(__funnelshift_r(ma, mb, s_m) & 63u);
                const float2 s2 = make_float2(ds, ds), nm2 = make_float2(ndm, ndm);
                float2 xs[M];
#pragma unroll
                for (int m = 0; m < M; m++) {
                    const float xm = xr[m] * kStripXScale;
                    xs[m] = make_float2(xm, xm);
                }
#pragma unroll
                for (int c = 0; c < V / 8; c++) {
                    // byte lane i of E / O holds value 8c + 2i / 8c + 2i + 1
                    const uint32_t E = q[c] & 0x0F0F0F0Fu, O = (q[c] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 q2 = make_float2(__uint_as_float(prmt(E, 0u, 0x4440u | i)),
                                                      __uint_as_float(prmt(O, 0u, 0x4440u | i)));
                        const float2 w2 = f2fma(s2, q2, nm2);
#pragma unroll
                        for (int m = 0; m < M; m++) acc[m][4 * c + i] = f2fma(xs[m], w2, acc[m][4 * c + i]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring's bytes become the sums' buffer

    // ---- sums over the CTA's row groups ----
    // red[t][m*V + v] with rows padded to RS = MV + 4 floats, so the 16-byte
    // stores of 8 consecutive threads fall on distinct banks; the padding of
    // lane-column 0's rows carries the sums of squares
    if (rg < R) {
        float *row = red + t * RS;
        float4 *mine = reinterpret_cast<float4 *>(row);
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int i = 0; i < NP; i += 2)
                mine[(m * V + 2 * i) / 4] = make_float4(acc[m][i].x, acc[m][i].y, acc[m][i + 1].x, acc[m][i + 1].y);
        if (track_ssq) {
#pragma unroll
            for (int m = 0; m < M; m++) row[MV + m] = ssq[m];
        }
    }
    __syncthreads();
    // output e = lcl*MV + mv: the row group r of lane-column lcl wrote it at
    // red[(r*nlc + lcl)*RS + mv]; the sum goes to row group 0's element
    // (lcl*RS + mv), which no other output reads
    const int E = nlc * MV;
    const int rstride = nlc * RS;
    const int P = E >= kStripThreads ? 1 : kStripThreads / E;  // threads per output
    if (P == 1) {
        for (int e = t; e < E; e += kStripThreads) {
            const int at = (e / MV) * RS + e % MV;
            red[at] = strided_sum(red + at, R, rstride);
        }
    } else {
        const int e = t % E, part = t / E;
        const int at = (e / MV) * RS + e % MV;
        if (part < P) red2[part * E + e] = strided_sum(red + part * rstride + at, (R - part + P - 1) / P, P * rstride);
        __syncthreads();
        if (t < E) red[at] = strided_sum(red2 + t, P, E);
    }
    if (norm && t < M) ssq_cta[t] = strided_sum(red + MV + t, R, rstride);
    __syncthreads();

    // ---- the cluster's CTAs add their sums in rank order and store y ----
    const bool peers = gather && chan[1] == 1u;
    const unsigned seq = gather ? chan[0] : 0u;
    // an output value into its place in y (for the all-gather, weight 0's y
    // is this rank's output buffer) and, for the gathered weight unless the
    // channel has failed, into its slot in every other rank's channel buffer
    auto put = [&](const StripSegP &sg, int m, int64_t col, float v, bool gathered) {
        const int64_t off = (int64_t)m * sg.y_ld + sg.col_off + col;
        sg.y[off] = v;
        if (gathered && peers) {
            const uint64_t word = ((uint64_t)seq << 32) | __float_as_uint(v);
#pragma unroll 1
            for (int r = 0; r < gq.world; r++)
                if (r != gq.rank) st_relaxed_sys_u64(channel_slot(gq.peer_flags[r], sg.y_ld, m, sg.col_off + col, seq), word);
        }
    };
    if (S > 1) cluster_sync_all();
    float inv[M];  // 1 / rms of each row of x (1 without the prologue)
#pragma unroll
    for (int m = 0; m < M; m++) {
        inv[m] = 1.f;
        if (norm) inv[m] = 1.f / sqrtf(cluster_sum(&ssq_cta[m], S) / (float)p.K + p.eps);
    }
    if (!p.silu) {
        const int e_lo = crank * E / S, e_hi = (crank + 1) * E / S;
        for (int e = e_lo + t; e < e_hi; e += kStripThreads) {
            const int lc = e / MV, m = (e % MV) / V, v = e % V;
            const float s = cluster_sum(red + lc * RS + e % MV, S);
            int s_i, s_ll;
            strip_lane(p, lo + lc, s_i, s_ll);
            const StripSegP &sg = p.seg[s_i];
            put(sg, m, (int64_t)s_ll * V + v, s * (M == 1 ? inv[0] : inv[m]), s_i == 0);
        }
    } else {
        // gate lane 2i, up lane 2i + 1 of the CTA hold pair i (lo is even)
        const int E2 = (nlc / 2) * MV;
        const int e_lo = crank * E2 / S, e_hi = (crank + 1) * E2 / S;
        for (int e = e_lo + t; e < e_hi; e += kStripThreads) {
            const int pl = e / MV, mv = e % MV, m = mv / V, v = mv % V;
            const float sc = M == 1 ? inv[0] : inv[m];
            const float gv = cluster_sum(red + (2 * pl) * RS + mv, S) * sc;
            const float uv = cluster_sum(red + (2 * pl + 1) * RS + mv, S) * sc;
            const StripSegP &sg = p.seg[0];
            put(sg, m, (int64_t)(lo / 2 + pl) * V + v, gv / (1.0f + expf(-gv)) * uv, true);
        }
    }
    if (S > 1) cluster_sync_all();  // no CTA leaves while the others read its shared memory
    // All-gather: the other ranks' columns from this rank's slots into its
    // output (every thread of the grid takes a share), then the last CTA to
    // finish records the call number.
    if (gather) {
        if (peers) {
            // weight 0 (with the SiLU epilogue: the gate|up pair) is the sharded one
            const StripSegP &sg = p.seg[0];
            const int64_t width = (int64_t)(p.silu ? p.lanes / 2 : p.seg[0].lane_end) * V;
            const int64_t n_all = sg.y_ld, rest = n_all - width;
            const int64_t total = (int64_t)M * rest;
            int bad = 0;
            for (int64_t e = (int64_t)blockIdx.x * kStripThreads + t; e < total && bad == 0;
                 e += (int64_t)gridDim.x * kStripThreads) {
                const int m = (int)(e / rest);
                const int64_t j = e % rest, n = j < sg.col_off ? j : j + width;
                float v;
                bad = wait_slot(channel_slot(gq.peer_flags[gq.rank], n_all, m, n, seq), seq, gq.wait_ns,
                                &gq.sync[2], &v);
                if (bad == 0) sg.y[m * n_all + n] = v;
            }
            // the first thread to find a fault reports it and marks the
            // channel failed, which stops every other waiting thread
            if (bad > 0 && atomicExch(&gq.sync[2], 1u) == 0u) strip_status(bad);
        }
        __syncthreads();
        if (t == 0) {
            const unsigned old = atomicAdd(&gq.sync[1], 1u);
            if (old == gridDim.x - 1u) {  // every CTA has read this call's number
                gq.sync[1] = 0u;
                gq.sync[0] = chan[0];
            }
        }
    }
}

// ------------------------------- host side -------------------------------
struct StripPlan {
    int V = 0, S = 1, groups = 0, lanes = 0, unit = 1;
    int64_t k_per = 0;
    size_t smem = 0;
};

static size_t strip_smem(int M) {
    const size_t ring = (size_t)kStripDepth * kStripThreads * kStripSlot;
    const size_t sums = (size_t)kStripThreads * (M * (M <= 2 ? 32 : 16) + 5) * sizeof(float);
    return ring > sums ? ring : sums;
}

static const void *strip_kernel(int M) {
    switch (M) {
    case 1: return (const void *)gemv_strip_kernel<1>;
    case 2: return (const void *)gemv_strip_kernel<2>;
    case 3: return (const void *)gemv_strip_kernel<3>;
    default: return (const void *)gemv_strip_kernel<4>;
    }
}

static cudaError_t strip_prepare(const void *fn, size_t smem) { return kernel_smem(fn, smem, true); }

// CTAs of clusters of S that the device runs at once (max active clusters x S).
static int strip_capacity(int M, int S, int device) {
    static std::mutex mu;
    static int cache[16][5][kStripMaxCluster + 1];  // [device][M][S], 0 = not asked
    const int sms = device_sm_count(device);
    if (S == 1) return sms;
    if (device < 0 || device >= 16) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int &c = cache[device][M][S];
    if (c == 0) {
        const void *fn = strip_kernel(M);
        const size_t smem = strip_smem(M);
        int n = 0;
        if (strip_prepare(fn, smem) == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3((unsigned)(S * (sms / S)));
            cfg.blockDim = dim3(kStripThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute a[1];
            a[0].id = cudaLaunchAttributeClusterDimension;
            a[0].val.clusterDim.x = (unsigned)S;
            a[0].val.clusterDim.y = 1;
            a[0].val.clusterDim.z = 1;
            cfg.attrs = a;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
        }
        cudaGetLastError();
        c = n > 0 ? n * S : -1;
    }
    return c > 0 ? c : 0;
}

// Estimated cycles of one launch: the busiest CTA's issue time (thread
// instructions per lane-column row, 32 threads per warp instruction, four
// schedulers at ~2/3 issue), or its longest thread's chain of rows, plus
// fixed costs (DRAM latency and the sums; the cluster barriers, which grow
// with the cluster).
static double strip_cost(int M, int V, int S, int nlc, int64_t rows) {
    const double per_row = V * (2.4 + 0.5 * M) + 34 + 4 * M;
    const double issue = (double)nlc * (double)rows * per_row / (32 * 4 * 0.67);
    const int R = kStripThreads / nlc;
    const double chain = (double)((rows + R - 1) / R) * (per_row + 40);
    return (issue > chain ? issue : chain) + 2500 + (S > 1 ? 2000 + 600 * S : 0);
}

static StripPlan strip_plan(int M, int64_t K, int64_t lanes, int unit, int device) {
    StripPlan best;
    const int V = M <= 2 ? 32 : 16;
    const int64_t units = lanes / unit;
    double best_cost = 0;
    for (int S = 1; S <= kStripMaxCluster; S++) {
        if (S == 5 || S == 7) continue;
        if ((int64_t)S > K) break;
        const int cap = strip_capacity(M, S, device);
        int64_t groups = cap / S;
        if (groups <= 0) continue;
        if (groups > units) groups = units;
        const int64_t nlc = (units + groups - 1) / groups * unit;
        if (nlc > kStripThreads) continue;
        const int64_t k_per = (K + S - 1) / S;
        if ((int64_t)(S - 1) * k_per >= K) continue;  // every rank gets rows
        const double c = strip_cost(M, V, S, (int)nlc, k_per);
        if (best.V == 0 || c < best_cost) {
            best_cost = c;
            best.V = V;
            best.S = S;
            best.groups = (int)groups;
            best.lanes = (int)lanes;
            best.unit = unit;
            best.k_per = k_per;
            best.smem = strip_smem(M);
        }
    }
    return best;
}

// Lane-columns of one weight, or 0 when the layout does not suit the kernel.
static int64_t strip_lanes(const StripSeg &g, int V) {
    if (g.N < V || g.N % V != 0 || g.rs % 256 != 0 || g.c0 < 0 || g.c0 >= 256 || g.c0 % V != 0 ||
        g.c0 + g.N > g.rs || g.N / V >= (int64_t(1) << 28))
        return 0;
    return g.N / V;
}

bool gemv_strip_supported(const GemvShape &s) {
    return s.qtype == kQ4K && s.M >= 1 && s.M <= 4 && s.K >= 1 && s.N >= 16;
}

bool gemv_strip_fits(const GemvShape &s, const StripLayout &L, int device) {
    if (!gemv_strip_supported(s)) return false;
    const int64_t lanes = strip_lanes(StripSeg{nullptr, 0, s.N, L.rs, L.c0, nullptr, 0, 0}, s.M <= 2 ? 32 : 16);
    return lanes > 0 && strip_plan((int)s.M, s.K, lanes, 1, device).V != 0;
}

int gemv_strip_multi(int M, int64_t K, const StripSeg *segs, int nseg, bool silu, const float *x,
                     const float *norm_w, float eps, cudaStream_t stream, int device, const GatherArgs *gather) {
    const int V = M <= 2 ? 32 : 16;
    if (M < 1 || M > 4 || nseg < 1 || nseg > kMaxStripSegs || K < 1 || (silu && nseg != 2) ||
        (norm_w && M > 3)) {
        set_error("the column-strip GEMV serves 1..%d weights, M <= 4 (M <= 3 with the RMSNorm prologue)",
                  kMaxStripSegs);
        return 3;
    }
    StripParams p{};
    int64_t lanes = 0;
    for (int i = 0; i < nseg; i++) {
        const int64_t n = strip_lanes(segs[i], V);
        if (n == 0) {
            set_error("weight %d (N=%lld, row stride %lld values, offset %lld) does not suit the column-strip GEMV", i,
                      (long long)segs[i].N, (long long)segs[i].rs, (long long)segs[i].c0);
            return 3;
        }
        const int64_t row_bytes = segs[i].rs / 256 * 144;
        if (segs[i].w_bytes < K * row_bytes) {
            set_error("weight %d: buffer of %lld bytes for %lld rows of %lld", i, (long long)segs[i].w_bytes,
                      (long long)K, (long long)row_bytes);
            return 2;
        }
        lanes += n;
        StripSegP &q = p.seg[i];
        q.w = static_cast<const uint8_t *>(segs[i].w);
        q.y = segs[i].y;
        q.row_bytes = row_bytes;
        q.y_ld = segs[i].y_ld;
        q.col_off = segs[i].col_off;
        q.c0 = (int)segs[i].c0;
        q.lane_end = (int)lanes;
    }
    if (silu && segs[0].N != segs[1].N) {
        set_error("SiLU(gate) * up needs gate and up of one width (%lld, %lld)", (long long)segs[0].N,
                  (long long)segs[1].N);
        return 3;
    }
    const StripPlan pl = strip_plan(M, K, lanes, silu ? 2 : 1, device);
    if (pl.V == 0) {
        set_error("the column-strip GEMV has no plan for this shape");
        return 3;
    }
    p.x = x;
    p.norm_w = norm_w;
    p.K = K;
    p.k_per = pl.k_per;
    p.eps = eps;
    p.nseg = nseg;
    p.silu = silu ? 1 : 0;
    p.lanes = pl.lanes;
    p.groups = pl.groups;
    p.unit = pl.unit;
    p.S = pl.S;
    StripGatherP gq{};
    if (gather) {
        // weight 0 (and for SiLU weight 1) is this rank's shard, gathered;
        // the other weights are whole and stay local
        if (gather->world < 1 || gather->world > kMaxRanks ||
            (gather->world > 1 && gather->slot_elems < (int64_t)M * segs[0].y_ld)) {
            set_error("the column-strip all-gather serves 1 to %d ranks with channel slots for every output", kMaxRanks);
            return 3;
        }
        for (int r = 0; r < gather->world; r++) {
            gq.peer_flags[r] = gather->peer_flags[r];
        }
        gq.sync = gather->sync;
        gq.world = gather->world;
        gq.rank = gather->rank;
        gq.wait_ns = gather->wait_ns;
    }
    const void *fn = strip_kernel(M);
    cudaError_t e = strip_prepare(fn, pl.smem);
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)(pl.groups * pl.S));
        cfg.blockDim = dim3(kStripThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = stream;
        cudaLaunchAttribute a[2];
        a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        a[0].val.programmaticStreamSerializationAllowed = 1;
        int na = 1;
        if (pl.S > 1) {
            a[1].id = cudaLaunchAttributeClusterDimension;
            a[1].val.clusterDim.x = (unsigned)pl.S;
            a[1].val.clusterDim.y = 1;
            a[1].val.clusterDim.z = 1;
            na = 2;
        }
        cfg.attrs = a;
        cfg.numAttrs = (unsigned)na;
        void *args[] = {&p, &gq};
        e = cudaLaunchKernelExC(&cfg, fn, args);
    }
    if (e != cudaSuccess) {
        set_error("column-strip gemv launch failed: %s", cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int gemv_strip_launch(const GemvShape &s, const StripLayout &L, const void *w, int64_t w_bytes, const float *x,
                      float *y, int64_t y_ld, int64_t col_off, cudaStream_t stream, int device) {
    if (!gemv_strip_supported(s)) {
        set_error("the column-strip GEMV serves Q4_K with 1 <= M <= 4");
        return 3;
    }
    const StripSeg g{w, w_bytes, s.N, L.rs, L.c0, y, y_ld, col_off};
    return gemv_strip_multi((int)s.M, s.K, &g, 1, false, x, nullptr, 0.f, stream, device, nullptr);
}

bool gemv_strip_gather_fits(const GemvShape &s, const GatherArgs &g, int device) {
    // the channel buffers hold a slot pair for every output element
    if (g.world > 1 && g.slot_elems < s.M * g.y_ld) return false;
    // the shard's rows start at one in-block position: every row of the full
    // weight starts on a block boundary (ld % 256 == 0), or there is one row
    if ((g.ld & 255) != 0 && s.K != 1) return false;
    return gemv_strip_fits(s, StripLayout{g.rs, g.n_base & 255}, device);
}

int gemv_strip_gather(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, const GatherArgs &g,
                      cudaStream_t stream, int device) {
    const StripSeg seg{w, w_bytes, s.N, g.rs, g.n_base & 255, g.peer_y[g.rank], g.y_ld, g.col_off};
    return gemv_strip_multi((int)s.M, s.K, &seg, 1, false, x, nullptr, 0.f, stream, device, &g);
}

int gemv_strip_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_strip_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_strip_status, &zero, sizeof(int));
    return v;
}

}  // namespace vkq
