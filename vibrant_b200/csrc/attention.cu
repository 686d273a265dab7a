// attention.cu -- decode attention on sm_100a: one query token per sequence
// against its KV cache, fp32.
//
// The reference computes attention on the CPU per (batch, head)
// (computeAttention, internal/transformer/attention.go:316-363) after
// appending the new token's K and V to the cache (:147-162) and expanding
// grouped KV heads (expandKVHeads, :280-314):
//   scores[j] = (q . k_j) * float32(1 / sqrt(D))            (scaleScores :413-427)
//   no mask: one query row against len key rows              (applyCausalMask :429-460)
//   p = exp(scores - max) / sum, normalised by multiplying   (applySoftmax :462-527)
//   o = p . V
// Here one CTA takes one (head, sequence): its 8 warps take keys j, j + 8, ...
// for the scores (a warp per key: the lanes split head_dim, so each key row is
// one coalesced read, then a shuffle sum), the block reduces the max and the
// sum in fixed orders, and for o each warp sums p_j * v_j over its keys with
// the lanes again splitting head_dim; the 8 partial rows are added in warp
// order.  Query head h reads KV head h / (heads / kv_heads).  The caches are
// [batch][kv_heads][cache_len][head_dim] with the first len rows valid.
#include <cmath>
#include <cstdint>

#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;

template <int D>
__global__ void __launch_bounds__(kAttnThreads)
    attn_decode_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
                       float *__restrict__ o, int heads, int kv_heads, int64_t len, int64_t cache_len, float scale) {
    constexpr int DPL = D / 32;  // head_dim values per lane
    extern __shared__ __align__(16) float sm[];
    float *scores = sm;                    // [len]
    __shared__ float part[kAttnWarps][D];  // per-warp partial outputs
    __shared__ float red[kAttnWarps];
    pdl_wait();  // q and the caches may come from the preceding kernel
    pdl_launch_dependents();
    const int h = blockIdx.x, b = blockIdx.y;
    const int kvh = h / (heads / kv_heads);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *qh = q + ((int64_t)b * heads + h) * D;
    const int64_t kv0 = ((int64_t)b * kv_heads + kvh) * cache_len * D;
    float qv[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) qv[i] = qh[lane * DPL + i];

    // scores and their maximum
    float mx = -__int_as_float(0x7f800000);
    for (int64_t j = warp; j < len; j += kAttnWarps) {
        const float *kr = kc + kv0 + j * D + lane * DPL;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; i++) s = fmaf(qv[i], kr[i], s);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        s *= scale;
        if (lane == 0) scores[j] = s;
        mx = fmaxf(mx, s);
    }
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kAttnWarps; w++) mx = fmaxf(mx, red[w]);
    __syncthreads();

    // exp(score - max) and the sum, in a fixed order (threads over keys, then warps)
    float sum = 0.f;
    for (int64_t j = threadIdx.x; j < len; j += kAttnThreads) {
        const float e = expf(scores[j] - mx);
        scores[j] = e;
        sum += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) total += red[w];
    const float inv = 1.0f / total;

    // o = sum_j (e_j * inv) v_j: warp w over keys w, w + 8, ...
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[i] = 0.f;
    for (int64_t j = warp; j < len; j += kAttnWarps) {
        const float p = scores[j] * inv;
        const float *vr = vc + kv0 + j * D + lane * DPL;
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[i] = fmaf(p, vr[i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < DPL; i++) part[warp][lane * DPL + i] = acc[i];
    __syncthreads();
    float *oh = o + ((int64_t)b * heads + h) * D;
    for (int d = threadIdx.x; d < D; d += kAttnThreads) {
        float s = part[0][d];
#pragma unroll
        for (int w = 1; w < kAttnWarps; w++) s += part[w][d];
        oh[d] = s;
    }
}

size_t attention_max_len() { return (size_t)(200 * 1024) / sizeof(float); }

cudaError_t attention_decode(const float *q, const float *kc, const float *vc, float *o, int64_t batch, int64_t heads,
                             int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim, cudaStream_t s) {
    const size_t smem = (size_t)len * sizeof(float);
    const void *fn = head_dim == 64 ? (const void *)attn_decode_kernel<64> : (const void *)attn_decode_kernel<128>;
    cudaError_t e = kernel_smem(fn, smem, false);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)heads, (unsigned)batch);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    const int h = (int)heads, kvh = (int)kv_heads;
    const float scale = (float)(1.0 / std::sqrt((double)head_dim));  // as scaleScores: float32(1 / sqrt(D))
    void *args[] = {(void *)&q, (void *)&kc, (void *)&vc, (void *)&o, (void *)&h, (void *)&kvh,
                    (void *)&len, (void *)&cache_len, (void *)&scale};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace vkq
