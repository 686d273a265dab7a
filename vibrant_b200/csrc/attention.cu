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
// Query head h reads KV head h / (heads / kv_heads).  The caches are
// [batch][kv_heads][cache_len][head_dim] with the first len rows valid.
//
// One (head, sequence) is one thread-block cluster of S CTAs (S = 1, 2, 4 or
// 8) that split the len keys into S contiguous chunks, so that a decode step
// with few heads still spreads its cache reads over many SMs.  In each CTA
// the 8 warps take the chunk's keys j, j + 8, ..., four at a time with their
// loads in flight together: for a score the lanes split head_dim (each key
// row one coalesced read) and a shuffle butterfly adds them.  The softmax
// keeps the reference's single global maximum: every CTA posts its chunk's
// maximum in shared memory, and after a cluster barrier each reads all S of
// them (distributed shared memory) to get the max over all keys; the sum of
// exp(score - max) goes the same way, added in CTA-rank order.  Each CTA then
// forms its chunk's share of p . V (warp partials added in warp order), and
// after one more barrier CTA r adds the S shares of dims [r D/S, (r+1) D/S)
// in rank order and stores them.  A last barrier keeps every CTA's shared
// memory alive until the others have read it.  Nothing is allocated: the
// scores live in the CTA's dynamic shared memory (at most kAttnChunk keys a
// CTA, so len <= 8 kAttnChunk).
#include <cmath>
#include <cstdint>

#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnUnroll = 4;                                 // keys a warp has in flight
constexpr int64_t kAttnChunk = (200 * 1024) / sizeof(float);  // keys a CTA holds scores for
constexpr int kAttnMaxCluster = 8;
constexpr int64_t kAttnMinKeys = 64;  // a chunk is not split below this many keys

// DPL consecutive floats of one lane: one vector load when the row is
// aligned for it (VEC), else DPL scalar loads.
template <int DPL, bool VEC>
__device__ __forceinline__ void load_lane(const float *p, float (&r)[DPL]) {
    if constexpr (VEC && DPL == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(p);
        r[0] = t.x, r[1] = t.y, r[2] = t.z, r[3] = t.w;
    } else if constexpr (VEC && DPL == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        r[0] = t.x, r[1] = t.y;
    } else {
#pragma unroll
        for (int i = 0; i < DPL; i++) r[i] = p[i];
    }
}

template <int D, bool VEC>
__global__ void __launch_bounds__(kAttnThreads)
    attn_decode_kernel(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
                       float *__restrict__ o, int heads, int kv_heads, int64_t len, int64_t cache_len, int chunk,
                       float scale) {
    constexpr int DPL = D / 32;  // head_dim values per lane
    constexpr int U = kAttnUnroll;
    extern __shared__ __align__(16) float sm[];
    float *scores = sm;                    // [chunk]: this CTA's keys
    __shared__ float part[kAttnWarps][D];  // per-warp partial outputs
    __shared__ float red[kAttnWarps];
    __shared__ float stat[2];   // this CTA's maximum and sum, read by the cluster
    __shared__ float share[D];  // this CTA's share of o, read by the cluster
    pdl_wait();  // q and the caches may come from the preceding kernel
    pdl_launch_dependents();
    const int S = (int)gridDim.x, c = (int)blockIdx.x;  // the cluster spans x: rank c
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / (heads / kv_heads);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t lo = (int64_t)c * chunk;
    const int n = lo < len ? (int)(len - lo < chunk ? len - lo : chunk) : 0;
    const float *qh = q + ((int64_t)b * heads + h) * D;
    const int64_t kv0 = (((int64_t)b * kv_heads + kvh) * cache_len + lo) * D + lane * DPL;
    const float *kb = kc + kv0, *vb = vc + kv0;
    float qv[DPL];
    load_lane<DPL, VEC>(qh + lane * DPL, qv);

    // scores of this chunk and their maximum
    float mx = -__int_as_float(0x7f800000);
    for (int j0 = warp; j0 < n; j0 += kAttnWarps * U) {
        float s[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            float kr[DPL];
            if (j < n) {
                load_lane<DPL, VEC>(kb + (int64_t)j * D, kr);
            } else {
#pragma unroll
                for (int i = 0; i < DPL; i++) kr[i] = 0.f;
            }
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < DPL; i++) a = fmaf(qv[i], kr[i], a);
            s[u] = a;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            if (j < n) {
                const float v = s[u] * scale;
                if (lane == 0) scores[j] = v;
                mx = fmaxf(mx, v);
            }
        }
    }
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kAttnWarps; w++) mx = fmaxf(mx, red[w]);
    if (S > 1) {
        if (threadIdx.x == 0) stat[0] = mx;
        cluster_sync_all();
        mx = ld_dsmem(&stat[0], 0);
        for (int r = 1; r < S; r++) mx = fmaxf(mx, ld_dsmem(&stat[0], (uint32_t)r));
    }
    __syncthreads();  // red is reused below

    // exp(score - max) and the sum: threads over keys, then warps, then CTAs
    float sum = 0.f;
    for (int j = threadIdx.x; j < n; j += kAttnThreads) {
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
    if (S > 1) {
        if (threadIdx.x == 0) stat[1] = total;
        cluster_sync_all();
        total = ld_dsmem(&stat[1], 0);
        for (int r = 1; r < S; r++) total += ld_dsmem(&stat[1], (uint32_t)r);
    }
    const float inv = 1.0f / total;

    // this chunk's share of o = sum_j (e_j * inv) v_j: warp w over keys w, w + 8, ...
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[i] = 0.f;
    for (int j0 = warp; j0 < n; j0 += kAttnWarps * U) {
        float vr[U][DPL];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            if (j < n) {
                load_lane<DPL, VEC>(vb + (int64_t)j * D, vr[u]);
            } else {
#pragma unroll
                for (int i = 0; i < DPL; i++) vr[u][i] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            const float p = j < n ? scores[j] * inv : 0.f;
#pragma unroll
            for (int i = 0; i < DPL; i++) acc[i] = fmaf(p, vr[u][i], acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < DPL; i++) part[warp][lane * DPL + i] = acc[i];
    __syncthreads();
    float *oh = o + ((int64_t)b * heads + h) * D;
    if (S == 1) {
        for (int d = threadIdx.x; d < D; d += kAttnThreads) {
            float s = part[0][d];
#pragma unroll
            for (int w = 1; w < kAttnWarps; w++) s += part[w][d];
            oh[d] = s;
        }
        return;
    }
    for (int d = threadIdx.x; d < D; d += kAttnThreads) {
        float s = part[0][d];
#pragma unroll
        for (int w = 1; w < kAttnWarps; w++) s += part[w][d];
        share[d] = s;
    }
    cluster_sync_all();
    const int per = D / S;  // D is 64 or 128 and S divides 8
    for (int d = c * per + (int)threadIdx.x; d < (c + 1) * per; d += kAttnThreads) {
        float s = ld_dsmem(&share[d], 0);
        for (int r = 1; r < S; r++) s += ld_dsmem(&share[d], (uint32_t)r);
        oh[d] = s;
    }
    cluster_sync_all();  // no CTA leaves while the others read its shared memory
}

size_t attention_max_len() { return (size_t)(kAttnMaxCluster * kAttnChunk); }

// CTAs per (head, sequence): enough that every chunk's scores fit, then
// doubled while the grid is under two CTAs per SM and a chunk keeps at least
// kAttnMinKeys keys.
static int attention_cluster(int64_t len, int64_t ctas, int sms) {
    int S = 1;
    while (S < kAttnMaxCluster && (len + S - 1) / S > kAttnChunk) S *= 2;
    while (S < kAttnMaxCluster && ctas * S < 2 * (int64_t)sms && len / (2 * S) >= kAttnMinKeys) S *= 2;
    return S;
}

cudaError_t attention_decode(const float *q, const float *kc, const float *vc, float *o, int64_t batch, int64_t heads,
                             int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int S = attention_cluster(len, batch * heads, device_sm_count(dev));
    const int chunk = (int)((len + S - 1) / S);
    const size_t smem = (size_t)chunk * sizeof(float);
    // whole lane vectors: q, the caches and o aligned to head_dim/32 floats
    const uintptr_t vec = (uintptr_t)(head_dim / 32) * sizeof(float) - 1;
    const bool aligned = (((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc) & vec) == 0;
    const void *fn = head_dim == 64 ? (aligned ? (const void *)attn_decode_kernel<64, true>
                                               : (const void *)attn_decode_kernel<64, false>)
                                    : (aligned ? (const void *)attn_decode_kernel<128, true>
                                               : (const void *)attn_decode_kernel<128, false>);
    e = kernel_smem(fn, smem, false);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)S, (unsigned)heads, (unsigned)batch);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute a[2];
    a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a[0].val.programmaticStreamSerializationAllowed = 1;
    unsigned na = 1;
    if (S > 1) {
        a[1].id = cudaLaunchAttributeClusterDimension;
        a[1].val.clusterDim.x = (unsigned)S;
        a[1].val.clusterDim.y = 1;
        a[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = a;
    cfg.numAttrs = na;
    const int h = (int)heads, kvh = (int)kv_heads;
    const float scale = (float)(1.0 / std::sqrt((double)head_dim));  // as scaleScores: float32(1 / sqrt(D))
    void *args[] = {(void *)&q, (void *)&kc, (void *)&vc, (void *)&o, (void *)&h, (void *)&kvh,
                    (void *)&len, (void *)&cache_len, (void *)&chunk, (void *)&scale};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace vkq
