// dequant.cu -- bit-exact k-quant -> float32 expansion on sm_100a.
//
// vkq_dequantize_f32 replaces the CPU expansion that vibrant performs before
// uploading a quantized weight (dequantizeForGPU -> DequantizeQ*_KTensor,
// internal/tensor/tensor_cuda_api.go:39-53); vkq_dequant_transpose_f32
// replaces DequantTransposeQ4K/Q5K/Q6K (internal/tensor/dequant_transpose.go:15-157).
//
// Bit-exactness: the reference computes scale = d*float32(sc), min =
// dmin*float32(m), out = scale*float32(q) - min (Q4_K/Q5_K) and
// out = (d*float32(s))*float32(q-32) (Q6_K), each operation rounded to
// float32 with no fused multiply-add (default GOAMD64).  The kernels use
// __fmul_rn / __fsub_rn, which are never contracted, and no flush-to-zero.
#include <cstdint>

#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

// Scale/min of sub-block sb from the 12 packed bytes: four 6-bit fields per
// little-endian 24-bit group (extractScalesAndMins, quant_q5k.go:97-120).
__device__ __forceinline__ void scale_min_6bit(const uint8_t *s, int sb, uint32_t &sc, uint32_t &m) {
    int g = sb >> 2, sh = 6 * (sb & 3);
    uint32_t a = s[3 * g] | (uint32_t)s[3 * g + 1] << 8 | (uint32_t)s[3 * g + 2] << 16;
    uint32_t b = s[6 + 3 * g] | (uint32_t)s[7 + 3 * g] << 8 | (uint32_t)s[8 + 3 * g] << 16;
    sc = (a >> sh) & 63u;
    m = (b >> sh) & 63u;
}

// Value i (0..255) of one super-block, exactly as the reference computes it.
template <int QT>
__device__ __forceinline__ float dequant_value(const uint8_t *blk, int i) {
    if constexpr (QT == kQ6K) {
        uint32_t lo = blk[i >> 1];
        lo = (i & 1) ? (lo >> 4) : (lo & 0x0Fu);
        uint32_t hi = (blk[128 + (i >> 2)] >> ((i & 3) * 2)) & 3u;
        int q = (int)(lo | (hi << 4));
        float d = go_f16_to_f32(blk[208] | (uint32_t)blk[209] << 8);
        float s = (float)(int8_t)blk[192 + (i >> 4)];
        return __fmul_rn(__fmul_rn(d, s), (float)(q - 32));
    } else {
        float d = go_f16_to_f32(blk[0] | (uint32_t)blk[1] << 8);
        float dmin = go_f16_to_f32(blk[2] | (uint32_t)blk[3] << 8);
        uint32_t sc, m;
        scale_min_6bit(blk + 4, i >> 5, sc, m);
        const uint8_t *qs = blk + (QT == kQ4K ? 16 : 48);
        uint32_t q = qs[i >> 1];
        q = (i & 1) ? (q >> 4) : (q & 0x0Fu);
        if constexpr (QT == kQ5K) q |= ((blk[16 + (i >> 3)] >> (i & 7)) & 1u) << 4;
        float scale = __fmul_rn(d, (float)sc);
        float mn = __fmul_rn(dmin, (float)m);
        return __fsub_rn(__fmul_rn(scale, (float)q), mn);
    }
}

// One warp per super-block; lane l produces values 8l..8l+7.
template <int QT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t *__restrict__ w, int64_t nblocks,
                                                      float *__restrict__ out) {
    constexpr int B = QT_<QT>::BYTES;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const uint8_t *blk = w + b * B;
        float v[8];
        if constexpr (QT == kQ6K) {
            float d = go_f16_to_f32(blk[208] | (uint32_t)blk[209] << 8);
            float ds = __fmul_rn(d, (float)(int8_t)blk[192 + (lane >> 1)]);
            uint32_t qlw = blk[4 * lane] | (uint32_t)blk[4 * lane + 1] << 8 |
                           (uint32_t)blk[4 * lane + 2] << 16 | (uint32_t)blk[4 * lane + 3] << 24;
            uint32_t qh = blk[128 + 2 * lane] | (uint32_t)blk[129 + 2 * lane] << 8;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                uint32_t lo = (qlw >> (4 * i)) & 0xFu;
                uint32_t hi = (qh >> (2 * i)) & 3u;
                v[i] = __fmul_rn(ds, (float)((int)(lo | hi << 4) - 32));
            }
        } else {
            float d = go_f16_to_f32(blk[0] | (uint32_t)blk[1] << 8);
            float dmin = go_f16_to_f32(blk[2] | (uint32_t)blk[3] << 8);
            uint32_t sc, m;
            scale_min_6bit(blk + 4, lane >> 2, sc, m);
            float scale = __fmul_rn(d, (float)sc);
            float mn = __fmul_rn(dmin, (float)m);
            const uint8_t *qs = blk + (QT == kQ4K ? 16 : 48) + 4 * lane;
            uint32_t qw = *reinterpret_cast<const uint32_t *>(qs);  // 16-byte aligned blocks
            uint32_t qh = (QT == kQ5K) ? blk[16 + lane] : 0u;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                uint32_t q = ((qw >> (4 * i)) & 0xFu) | (((qh >> i) & 1u) << 4);
                v[i] = __fsub_rn(__fmul_rn(scale, (float)q), mn);
            }
        }
        float *o = out + b * 256 + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = v[i];
    }
}

// Q4_K/Q5_K blocks are 16-byte multiples; the word loads above need a
// 4-byte aligned weight pointer.  Unaligned pointers use the per-value path.
template <int QT>
__global__ void __launch_bounds__(256) dequant_any_align_kernel(const uint8_t *__restrict__ w, int64_t nvalues,
                                                                float *__restrict__ out) {
    constexpr int B = QT_<QT>::BYTES;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvalues;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = dequant_value<QT>(w + (i >> 8) * B, (int)(i & 255));
}

// out[n*K + k] = W[k][n] for the first (K*N/256)*256 values; the rest stays 0
// (dequant_transpose.go:26,34-52).  32x32 tiles through shared memory so that
// both the (per-value) reads and the transposed writes are coalesced.
template <int QT>
__global__ void __launch_bounds__(256) dequant_transpose_kernel(const uint8_t *__restrict__ w, int64_t K,
                                                                int64_t N, float *__restrict__ out) {
    constexpr int B = QT_<QT>::BYTES;
    __shared__ float tile[32][33];
    const int64_t limit = (K * N / 256) * 256;
    const int64_t tiles_k = (K + 31) / 32, tiles_n = (N + 31) / 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows of 32
    for (int64_t t = blockIdx.x; t < tiles_k * tiles_n; t += gridDim.x) {
        const int64_t k0 = (t / tiles_n) * 32, n0 = (t % tiles_n) * 32;
#pragma unroll
        for (int r = 0; r < 32; r += 8) {
            int64_t k = k0 + ty + r, n = n0 + tx;
            float v = 0.0f;
            if (k < K && n < N) {
                int64_t idx = k * N + n;
                if (idx < limit) v = dequant_value<QT>(w + (idx >> 8) * B, (int)(idx & 255));
            }
            tile[ty + r][tx] = v;
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 32; r += 8) {
            int64_t n = n0 + ty + r, k = k0 + tx;
            if (n < N && k < K) out[n * K + k] = tile[tx][ty + r];
        }
        __syncthreads();
    }
}

static int grid_for(int64_t work, int per_cta, int device) {
    int sms = device_sm_count(device);
    int64_t g = (work + per_cta - 1) / per_cta;
    int64_t cap = (int64_t)sms * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

template <int QT>
static cudaError_t launch_dequant(const void *w, int64_t nblocks, float *out, cudaStream_t s, int device) {
    const uint8_t *wp = static_cast<const uint8_t *>(w);
    bool aligned = (reinterpret_cast<uintptr_t>(w) & 3u) == 0;
    if (QT == kQ6K || aligned) {
        dequant_kernel<QT><<<grid_for(nblocks, 8, device), 256, 0, s>>>(wp, nblocks, out);
    } else {
        dequant_any_align_kernel<QT><<<grid_for(nblocks * 256, 256, device), 256, 0, s>>>(wp, nblocks * 256, out);
    }
    return cudaGetLastError();
}

cudaError_t dequantize_f32(int qtype, const void *w, int64_t nblocks, float *out, cudaStream_t s, int device) {
    switch (qtype) {
    case kQ4K: return launch_dequant<kQ4K>(w, nblocks, out, s, device);
    case kQ5K: return launch_dequant<kQ5K>(w, nblocks, out, s, device);
    default: return launch_dequant<kQ6K>(w, nblocks, out, s, device);
    }
}

template <int QT>
static cudaError_t launch_dt(const void *w, int64_t K, int64_t N, float *out, cudaStream_t s, int device) {
    int64_t tiles = ((K + 31) / 32) * ((N + 31) / 32);
    dequant_transpose_kernel<QT><<<grid_for(tiles, 1, device), 256, 0, s>>>(static_cast<const uint8_t *>(w), K, N, out);
    return cudaGetLastError();
}

cudaError_t dequant_transpose_f32(int qtype, const void *w, int64_t K, int64_t N, float *out, cudaStream_t s,
                                  int device) {
    switch (qtype) {
    case kQ4K: return launch_dt<kQ4K>(w, K, N, out, s, device);
    case kQ5K: return launch_dt<kQ5K>(w, K, N, out, s, device);
    default: return launch_dt<kQ6K>(w, K, N, out, s, device);
    }
}

}  // namespace vkq
