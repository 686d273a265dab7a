// gemv_rows.cu -- the decode GEMV for weights in the upstream GGUF
// orientation, on sm_100a.
//
// vibrant reads a [K, N] weight as W[k][n] = value k*N + n of the
// super-block stream (internal/gguf/loader.go:24-27): the blocks run along
// the output dimension, and every other kernel of this library follows it.
// GGUF files as other engines write them store a linear layer's weight as
// [out][in]: row n holds the K/256 blocks of output n, so W[n][k] = value
// n*K + k.  This kernel serves that orientation (vkq_matmul_upstream):
//
//   y[m][n] = sum_k x[m][k] * W[n][k],  K % 256 == 0, fp32 accumulate.
//
// A row's blocks are contiguous, so a warp takes whole output rows: lane l
// takes the 32-value units l, l + 32, ... of the row (unit u = sub-block u % 8
// of block u / 8), loads its header and quant bytes straight from HBM (the 8
// lanes of one block read its header once and 128 contiguous quant bytes),
// decodes the unit into fp32 pairs and multiplies them with the matching x
// pairs by packed fp32x2 FMA; a shuffle tree adds the lanes' sums.  Each value
// is formed as in the other kernels: Q4_K / Q5_K w = (d*sc)*q - dmin*m and
// Q6_K w = (d*s)*(q - 32), each with one rounding, from the quant used as the
// subnormal float q * 2^-149 with the multipliers scaled by powers of two.
#include <cstdint>

#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

constexpr int kRowThreads = 512;              // 16 warps, one CTA per SM
constexpr int kRowWarps = kRowThreads / 32;
constexpr size_t kRowStageBytes = 96 * 1024;  // x rows staged in shared memory up to this size
constexpr float kRowWScale = 0x1p100f;        // on d*sc, d*s
constexpr float kRowWDown = 0x1p-49f;         // w comes out times this
constexpr float kRowXScale = 0x1p49f;         // and x goes in times this

template <int QT> struct RowBlock;
template <> struct RowBlock<kQ4K> { static constexpr int BYTES = 144; };
template <> struct RowBlock<kQ5K> { static constexpr int BYTES = 176; };
template <> struct RowBlock<kQ6K> { static constexpr int BYTES = 210; };

// Read-only loads through the non-coherent path, left to the compiler to
// schedule (the weights do not change during a launch).
__device__ __forceinline__ uint4 ldg128(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ uint32_t ldg32(const void *p) { return __ldg(reinterpret_cast<const unsigned int *>(p)); }
__device__ __forceinline__ uint32_t ldg16(const void *p) { return __ldg(reinterpret_cast<const unsigned short *>(p)); }

// The raw words of one 32-value unit (value `within` .. within + 31 of a
// block at global address blk): Q4_K / Q5_K header, quant words (and fifth
// bits); Q6_K ql, qh words (from the 4-byte aligned address below, shifted by
// shf bits) and the unit's two 16-value scales with d.
struct RowUnit {
    uint32_t v[10];
    uint32_t shf;
};

template <int QT>
__device__ __forceinline__ void row_load(const uint8_t *blk, int within, RowUnit &u) {
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const uint4 h = ldg128(blk);
        const uint4 q = ldg128(blk + (QT == kQ4K ? 16 : 48) + (within >> 1));
        u.v[0] = h.x; u.v[1] = h.y; u.v[2] = h.z; u.v[3] = h.w;
        u.v[4] = q.x; u.v[5] = q.y; u.v[6] = q.z; u.v[7] = q.w;
        if constexpr (QT == kQ5K) u.v[8] = ldg32(blk + 16 + (within >> 3));
    } else {
        // ql (offset within/2) and qh (offset 128 + within/4) share the
        // block's misalignment modulo 4
        const uintptr_t ql = reinterpret_cast<uintptr_t>(blk) + (within >> 1);
        const uintptr_t qh = reinterpret_cast<uintptr_t>(blk) + 128 + (within >> 2);
        u.shf = (uint32_t)(ql & 3u) * 8u;
        const uint8_t *qlw = reinterpret_cast<const uint8_t *>(ql & ~uintptr_t(3));
        const uint8_t *qhw = reinterpret_cast<const uint8_t *>(qh & ~uintptr_t(3));
#pragma unroll
        for (int i = 0; i < 5; i++) u.v[i] = ldg32(qlw + 4 * i);
#pragma unroll
        for (int i = 0; i < 3; i++) u.v[5 + i] = ldg32(qhw + 4 * i);
        u.v[8] = ldg16(blk + 192 + (within >> 4)) | (ldg16(blk + 208) << 16);
    }
}

template <int J>
__device__ __forceinline__ float2 row_pair(uint32_t E, uint32_t O) {
    return make_float2(__uint_as_float(prmt(E, 0u, 0x4440u | J)), __uint_as_float(prmt(O, 0u, 0x4440u | J)));
}

// The unit's 32 values times 2^-49 as 16 pairs: w[4c + j] holds values
// 8c + 2j and 8c + 2j + 1.
template <int QT>
__device__ __forceinline__ void row_decode(const RowUnit &u, int within, float2 (&w)[16]) {
    if constexpr (QT == kQ4K || QT == kQ5K) {
        const float d = hw_f16_to_f32(u.v[0] & 0xFFFFu), dmin = hw_f16_to_f32(u.v[0] >> 16);
        const int sb = within >> 5;
        const uint32_t sc24 = sb < 4 ? u.v[1] : __funnelshift_r(u.v[1], u.v[2], 24);
        const uint32_t m24 = sb < 4 ? __funnelshift_r(u.v[2], u.v[3], 16) : (u.v[3] >> 8);
        const uint32_t sh = 6u * (sb & 3);
        const float ds = (d * kRowWScale) * (float)((sc24 >> sh) & 63u);
        const float ndm = (dmin * -kRowWDown) * (float)((m24 >> sh) & 63u);
        const float2 s2 = make_float2(ds, ds), nm2 = make_float2(ndm, ndm);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t E = u.v[4 + c] & 0x0F0F0F0Fu;
            uint32_t O = (u.v[4 + c] >> 4) & 0x0F0F0F0Fu;
            if constexpr (QT == kQ5K) {
                // bit i of hb is the fifth bit of value 8c + i
                const uint32_t hb = (u.v[8] >> (8 * c)) & 0xFFu;
                E |= ((hb & 0x55u) * 0x410410u) & 0x10101010u;
                O |= (((hb >> 1) & 0x55u) * 0x410410u) & 0x10101010u;
            }
            w[4 * c + 0] = f2fma(s2, row_pair<0>(E, O), nm2);
            w[4 * c + 1] = f2fma(s2, row_pair<1>(E, O), nm2);
            w[4 * c + 2] = f2fma(s2, row_pair<2>(E, O), nm2);
            w[4 * c + 3] = f2fma(s2, row_pair<3>(E, O), nm2);
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
        const float d = hw_f16_to_f32(u.v[8] >> 16) * kRowWScale;
        const float ds0 = d * (float)(int)(int8_t)(u.v[8] & 0xFFu);
        const float ds1 = d * (float)(int)(int8_t)((u.v[8] >> 8) & 0xFFu);
        // -32 * d*s * 2^-49 = (d*s * 2^100) * -2^-144, exact
        const float o0 = ds0 * -0x1p-144f, o1 = ds1 * -0x1p-144f;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            // byte lane j of X = (hi2 of value 2j+1) << 2 | (hi2 of value 2j)
            const uint32_t X = prmt(qh[c >> 1], qhs[c >> 1], (c & 1) ? 0x7362u : 0x5140u) & 0x0F0F0F0Fu;
            const uint32_t E = (ql[c] & 0x0F0F0F0Fu) | ((X & 0x03030303u) << 4);
            const uint32_t O = ((ql[c] >> 4) & 0x0F0F0F0Fu) | ((X << 2) & 0x30303030u);
            const float2 s2 = c < 2 ? make_float2(ds0, ds0) : make_float2(ds1, ds1);
            const float2 o2 = c < 2 ? make_float2(o0, o0) : make_float2(o1, o1);
            w[4 * c + 0] = f2fma(s2, row_pair<0>(E, O), o2);
            w[4 * c + 1] = f2fma(s2, row_pair<1>(E, O), o2);
            w[4 * c + 2] = f2fma(s2, row_pair<2>(E, O), o2);
            w[4 * c + 3] = f2fma(s2, row_pair<3>(E, O), o2);
        }
    }
}

// Rows n = warp, warp + (warps of the grid), ...; MR rows of x at once.
// x is 16-byte aligned and K % 256 == 0, so every unit's 32 x values are
// eight aligned float4 loads (L1 serves the CTA's warps after the first).
template <int QT, int MR>
__global__ void __launch_bounds__(kRowThreads, 1)
    gemv_rows_kernel(const uint8_t *__restrict__ w, int64_t K, int64_t N, int64_t row_bytes, const float *x,
                     float *__restrict__ y, int64_t y_ld, int stage_x) {
    constexpr int B = RowBlock<QT>::BYTES;
    extern __shared__ __align__(16) float xs_sm[];  // x [MR][K] when it fits (stage_x), else unused
    pdl_wait();  // x (and y) may belong to the preceding kernel
    pdl_launch_dependents();
    if (stage_x) {  // every warp reads all of x: one copy per CTA in shared memory
        const int64_t n4 = (int64_t)MR * K / 4;
        for (int64_t i = threadIdx.x; i < n4; i += kRowThreads)
            reinterpret_cast<float4 *>(xs_sm)[i] = __ldg(reinterpret_cast<const float4 *>(x) + i);
        __syncthreads();
        x = xs_sm;
    }
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    const int64_t nw = (int64_t)gridDim.x * kRowWarps;
    const int units = (int)(K >> 5);  // 32-value units per row
    // RPW rows per warp at a time (n, n + nw, ...): each lane's loads for all
    // of them are in flight before the first is used
    constexpr int RPW = MR == 1 ? 4 : MR == 2 ? 2 : 1;
    for (int64_t n0 = gw; n0 < N; n0 += RPW * nw) {
        float2 acc[RPW][MR];
#pragma unroll
        for (int r = 0; r < RPW; r++)
#pragma unroll
            for (int m = 0; m < MR; m++) acc[r][m] = make_float2(0.f, 0.f);
#pragma unroll 2
        for (int u = lane; u < units; u += 32) {
            const int b = u >> 3, within = (u & 7) << 5;
            RowUnit ru[RPW];
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                const int64_t n = n0 + r * nw < N ? n0 + r * nw : n0;  // a row past N repeats row n0 (not stored)
                row_load<QT>(w + n * row_bytes + (int64_t)b * B, within, ru[r]);
            }
            // the unit's 32 x values (times 2^49) of each row of x, read once
            // for all RPW weight rows
            const float *xk = x + (int64_t)b * 256 + within;
            float2 xp[MR][16];
#pragma unroll
            for (int m = 0; m < MR; m++)
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    // a generic load: x is the shared-memory copy or global memory
                    const float4 xv = reinterpret_cast<const float4 *>(xk + (int64_t)m * K)[c];
                    xp[m][2 * c] = make_float2(xv.x * kRowXScale, xv.y * kRowXScale);
                    xp[m][2 * c + 1] = make_float2(xv.z * kRowXScale, xv.w * kRowXScale);
                }
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                float2 wv[16];
                row_decode<QT>(ru[r], within, wv);
#pragma unroll
                for (int m = 0; m < MR; m++)
#pragma unroll
                    for (int j = 0; j < 16; j++) acc[r][m] = f2fma(xp[m][j], wv[j], acc[r][m]);
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const int64_t n = n0 + r * nw;
#pragma unroll
            for (int m = 0; m < MR; m++) {
                float s = acc[r][m].x + acc[r][m].y;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0 && n < N) y[(int64_t)m * y_ld + n] = s;
            }
        }
    }
}

template <int QT, int MR>
static cudaError_t rows_launch_mr(const uint8_t *w, int64_t K, int64_t N, const float *x, float *y, int64_t y_ld,
                                  cudaStream_t s, int device) {
    const int64_t row_bytes = K / 256 * RowBlock<QT>::BYTES;
    const int64_t need = (N + kRowWarps - 1) / kRowWarps;
    const int grid = (int)(need < device_sm_count(device) ? need : device_sm_count(device));
    const size_t xbytes = (size_t)MR * (size_t)K * sizeof(float);
    const int stage_x = xbytes <= kRowStageBytes ? 1 : 0;
    if (stage_x) {
        const cudaError_t e = kernel_smem((const void *)gemv_rows_kernel<QT, MR>, xbytes, false);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kRowThreads);
    cfg.dynamicSmemBytes = stage_x ? xbytes : 0;
    cfg.stream = s;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_rows_kernel<QT, MR>, w, K, N, row_bytes, x, y, y_ld, stage_x);
}

template <int QT>
static cudaError_t rows_launch_qt(const uint8_t *w, int64_t K, int64_t N, const float *x, int64_t M, float *y,
                                  cudaStream_t s, int device) {
    // four rows of x per launch: the accumulators of more would crowd out
    // the loads in flight
    for (int64_t m0 = 0; m0 < M; m0 += 4) {
        const int64_t mr = M - m0 < 4 ? M - m0 : 4;
        const float *xm = x + m0 * K;
        float *ym = y + m0 * N;
        cudaError_t e;
        switch (mr) {
        case 1: e = rows_launch_mr<QT, 1>(w, K, N, xm, ym, N, s, device); break;
        case 2: e = rows_launch_mr<QT, 2>(w, K, N, xm, ym, N, s, device); break;
        case 3: e = rows_launch_mr<QT, 3>(w, K, N, xm, ym, N, s, device); break;
        default: e = rows_launch_mr<QT, 4>(w, K, N, xm, ym, N, s, device); break;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t gemv_rows_launch(int qtype, const void *w, int64_t K, int64_t N, const float *x, int64_t M, float *y,
                             cudaStream_t s, int device) {
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    switch (qtype) {
    case kQ4K: return rows_launch_qt<kQ4K>(wb, K, N, x, M, y, s, device);
    case kQ5K: return rows_launch_qt<kQ5K>(wb, K, N, x, M, y, s, device);
    default: return rows_launch_qt<kQ6K>(wb, K, N, x, M, y, s, device);
    }
}

}  // namespace vkq
