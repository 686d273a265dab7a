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
// the 8 warps take the chunk's keys j, j + 8, ..., eight at a time: for a
// score the lanes split head_dim (each key row one coalesced read) and a
// shuffle butterfly adds them, while the V rows of the same keys are
// prefetched into L2.  The softmax
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
//
// The fused decode step (attention_decode_rope) is the reference's whole
// Attention.Forward after the projections for one new token
// (attention.go:141-172): RoPE on q and on the new k (ApplyRotation,
// rope.go:49-124, the arithmetic of rope_kernel), the new K and V appended
// at row len - 1 of the caches (concatenateSeqDim), and the attention above,
// in one launch.  Every CTA rotates its own head's q; the CTA holding the
// last chunk takes key len - 1 from the rotated k_new and from v_new instead
// of the cache, and the first query head of each KV group stores that row,
// so no CTA of the launch reads a row another one writes.
#include <cmath>
#include <cstdint>

#include "../../include/vkq.h"
#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnUnroll = 8;                                 // keys a warp has in flight
constexpr int64_t kAttnChunk = (200 * 1024) / sizeof(float);  // keys a CTA holds scores for
constexpr int kAttnMaxCluster = 8;
constexpr int64_t kAttnMinKeys = 64;  // a chunk is not split below this many keys

// VKQ_ERR_INVALID_ARGUMENT when a fused step met a position outside its tables.
static __device__ int g_attn_status;

struct AttnParams {
    const float *q, *kc, *vc;
    float *o;
    int heads, kv_heads;
    int64_t len, cache_len;
    int chunk;
    float scale;
    // the fused decode step (ROPE): the new token's q (in q), k and v before
    // rotation, the tables and positions, and the caches to append to
    const float *k_new, *v_new, *cos_t, *sin_t;
    const int *pos;
    int64_t max_seq;
    float *kc_out, *vc_out;
};

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

// Rotate the lane's DPL values (whole interleaved pairs) by the table entries
// of position ps: each product and sum rounded on its own, as rope_kernel.
template <int D, int DPL>
__device__ __forceinline__ void rotate_lane(float (&x)[DPL], const float *cos_t, const float *sin_t, int ps,
                                            int lane) {
    const int64_t tb = (int64_t)ps * (D / 2) + lane * (DPL / 2);
#pragma unroll
    for (int t = 0; t < DPL / 2; t++) {
        const float c = cos_t[tb + t], sn = sin_t[tb + t];
        const float x0 = x[2 * t], x1 = x[2 * t + 1];
        x[2 * t] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        x[2 * t + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    return s;
}

template <int D, bool VEC, bool ROPE>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
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
    const int g = p.heads / p.kv_heads, kvh = h / g;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t lo = (int64_t)c * p.chunk;
    const int n = lo < p.len ? (int)(p.len - lo < p.chunk ? p.len - lo : p.chunk) : 0;
    const float *qh = p.q + ((int64_t)b * p.heads + h) * D;
    const int64_t row0 = ((int64_t)b * p.kv_heads + kvh) * p.cache_len;
    const int64_t kv0 = (row0 + lo) * D + lane * DPL;
    const float *kb = p.kc + kv0, *vb = p.vc + kv0;
    float qv[DPL];
    load_lane<DPL, VEC>(qh + lane * DPL, qv);

    // The fused step: the new token is key len - 1, the last of the last
    // chunk.  Its K and V come rotated from k_new and v_new (this launch
    // never reads that cache row); one CTA of each KV head stores them there.
    int ps = 0;
    bool has_new = false;
    float kn[DPL], vn[DPL];
    if constexpr (ROPE) {
        ps = p.pos[b];
        if (ps < 0 || ps >= p.max_seq) {  // the same for every CTA of the cluster: all leave
            if (threadIdx.x == 0 && c == 0) atomicExch(&g_attn_status, VKQ_ERR_INVALID_ARGUMENT);
            return;
        }
        rotate_lane<D, DPL>(qv, p.cos_t, p.sin_t, ps, lane);
        has_new = n > 0 && lo + n == p.len;
        if (has_new && warp == 0) {
            const int64_t nb = ((int64_t)b * p.kv_heads + kvh) * D + lane * DPL;
            load_lane<DPL, VEC>(p.k_new + nb, kn);
            load_lane<DPL, VEC>(p.v_new + nb, vn);
            rotate_lane<D, DPL>(kn, p.cos_t, p.sin_t, ps, lane);
            if (h % g == 0) {
                const int64_t r = (row0 + p.len - 1) * D + lane * DPL;
#pragma unroll
                for (int i = 0; i < DPL; i++) p.kc_out[r + i] = kn[i], p.vc_out[r + i] = vn[i];
            }
        }
    }
    const int nc = n - (has_new ? 1 : 0);  // keys read from the cache

    // scores of this chunk and their maximum; the V rows are prefetched into
    // L2 meanwhile (a lane per 128-byte line)
    float mx = -__int_as_float(0x7f800000);
    for (int j0 = warp; j0 < nc; j0 += kAttnWarps * U) {
        float s[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            float kr[DPL];
            if (j < nc) {
                load_lane<DPL, VEC>(kb + (int64_t)j * D, kr);
                if ((lane * DPL) % 32 == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (int64_t)j * D));
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
        for (int u = 0; u < U; u++) s[u] = warp_sum(s[u]);
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            if (j < nc) {
                const float v = s[u] * p.scale;
                if (lane == 0) scores[j] = v;
                mx = fmaxf(mx, v);
            }
        }
    }
    if (ROPE && has_new && warp == 0) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; i++) a = fmaf(qv[i], kn[i], a);
        const float v = warp_sum(a) * p.scale;
        if (lane == 0) scores[nc] = v;
        mx = fmaxf(mx, v);
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
    sum = warp_sum(sum);
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
    for (int j0 = warp; j0 < nc; j0 += kAttnWarps * U) {
        float vr[U][DPL];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            if (j < nc) {
                load_lane<DPL, VEC>(vb + (int64_t)j * D, vr[u]);
            } else {
#pragma unroll
                for (int i = 0; i < DPL; i++) vr[u][i] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * kAttnWarps;
            const float pj = j < nc ? scores[j] * inv : 0.f;
#pragma unroll
            for (int i = 0; i < DPL; i++) acc[i] = fmaf(pj, vr[u][i], acc[i]);
        }
    }
    if (ROPE && has_new && warp == 0) {
        const float pj = scores[nc] * inv;
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[i] = fmaf(pj, vn[i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < DPL; i++) part[warp][lane * DPL + i] = acc[i];
    __syncthreads();
    float *oh = p.o + ((int64_t)b * p.heads + h) * D;
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

template <int D, bool ROPE>
static const void *attn_kernel(bool vec) {
    return vec ? (const void *)attn_decode_kernel<D, true, ROPE> : (const void *)attn_decode_kernel<D, false, ROPE>;
}

// Cluster size, chunk, kernel variant and launch; p.chunk is filled in here.
static cudaError_t attention_launch(AttnParams p, int64_t batch, int64_t head_dim, bool rope, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int S = attention_cluster(p.len, batch * p.heads, device_sm_count(dev));
    p.chunk = (int)((p.len + S - 1) / S);
    const size_t smem = (size_t)p.chunk * sizeof(float);
    // whole lane vectors: the buffers a lane reads aligned to head_dim/32 floats
    const uintptr_t vec = (uintptr_t)(head_dim / 32) * sizeof(float) - 1;
    uintptr_t bits = (uintptr_t)p.q | (uintptr_t)p.kc | (uintptr_t)p.vc;
    if (rope) bits |= (uintptr_t)p.k_new | (uintptr_t)p.v_new;
    const bool aligned = (bits & vec) == 0;
    const void *fn = head_dim == 64 ? (rope ? attn_kernel<64, true>(aligned) : attn_kernel<64, false>(aligned))
                                    : (rope ? attn_kernel<128, true>(aligned) : attn_kernel<128, false>(aligned));
    e = kernel_smem(fn, smem, false);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)S, (unsigned)p.heads, (unsigned)batch);
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
    void *args[] = {(void *)&p};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

static AttnParams attention_params(const float *q, const float *kc, const float *vc, float *o, int64_t heads,
                                   int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim) {
    AttnParams p{};
    p.q = q, p.kc = kc, p.vc = vc, p.o = o;
    p.heads = (int)heads, p.kv_heads = (int)kv_heads;
    p.len = len, p.cache_len = cache_len;
    p.scale = (float)(1.0 / std::sqrt((double)head_dim));  // as scaleScores: float32(1 / sqrt(D))
    return p;
}

cudaError_t attention_decode(const float *q, const float *kc, const float *vc, float *o, int64_t batch, int64_t heads,
                             int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim, cudaStream_t s) {
    return attention_launch(attention_params(q, kc, vc, o, heads, kv_heads, len, cache_len, head_dim), batch,
                            head_dim, false, s);
}

cudaError_t attention_decode_rope(const float *q, const float *k_new, const float *v_new, const float *cos_t,
                                  const float *sin_t, const int *positions, float *kc, float *vc, float *o,
                                  int64_t batch, int64_t heads, int64_t kv_heads, int64_t len, int64_t cache_len,
                                  int64_t head_dim, int64_t max_seq, cudaStream_t s) {
    AttnParams p = attention_params(q, kc, vc, o, heads, kv_heads, len, cache_len, head_dim);
    p.k_new = k_new, p.v_new = v_new, p.cos_t = cos_t, p.sin_t = sin_t, p.pos = positions;
    p.max_seq = max_seq;
    p.kc_out = kc, p.vc_out = vc;
    return attention_launch(p, batch, head_dim, true, s);
}

int attention_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int));
    return v;
}

}  // namespace vkq
