// elementwise.cu -- the activation and normalisation steps between the
// linear layers of a decode step, on sm_100a.
//
//  * silu_mul: out = SiLU(gate) * up = gate / (1 + exp(-gate)) * up, one pass
//    over both inputs (the reference runs silu_f32 then mul_f32,
//    internal/gpu/cuda/kernels.cu:306-341, as tensor.SiLU and tensor.Mul in
//    internal/transformer/feedforward.go:92-94);
//  * rms_norm: out[r] = (x[r] / sqrt(mean(x[r]^2) + eps)) * weight, one CTA
//    per row with a fixed-order reduction (kernels.cu:209-288).
// Both are HBM-bound streams of a few tens of KB in a decode step: their cost
// is the launch, so they take part in programmatic dependent launch like the
// GEMV (the next kernel's prologue overlaps their tail).
#include <cstdint>

#include "../../include/vkq.h"
#include "kq_device.cuh"
#include "vkq_internal.h"

namespace vkq {

__global__ void __launch_bounds__(256) silu_mul_kernel(const float *__restrict__ gate, const float *__restrict__ up,
                                                       float *__restrict__ out, int64_t n) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 g = reinterpret_cast<const float4 *>(gate)[i];
        const float4 u = reinterpret_cast<const float4 *>(up)[i];
        float4 o;
        o.x = g.x / (1.0f + expf(-g.x)) * u.x;
        o.y = g.y / (1.0f + expf(-g.y)) * u.y;
        o.z = g.z / (1.0f + expf(-g.z)) * u.z;
        o.w = g.w / (1.0f + expf(-g.w)) * u.w;
        reinterpret_cast<float4 *>(out)[i] = o;
    }
    for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = gate[i] / (1.0f + expf(-gate[i])) * up[i];
}

constexpr int kNormThreads = 512;

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ weight,
                                                                float *__restrict__ out, int64_t n, float eps) {
    __shared__ float part[kNormThreads / 32];
    __shared__ float rms;
    pdl_wait();
    pdl_launch_dependents();
    const float *xr = x + (int64_t)blockIdx.x * n;
    float *yr = out + (int64_t)blockIdx.x * n;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += kNormThreads) s = fmaf(xr[i], xr[i], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < kNormThreads / 32; w++) t += part[w];
        rms = sqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float r = rms;
    for (int64_t i = threadIdx.x; i < n; i += kNormThreads) yr[i] = (xr[i] / r) * weight[i];
}

static __device__ int g_elem_status;

// Rotary position embedding over interleaved pairs, as the reference's
// rope_f32 (internal/gpu/cuda/kernels.cu:363-414) and its CPU path
// RoPE.ApplyRotation (internal/transformer/rope.go:49-124): x and out are
// [rows][half pairs] with rows = batch * heads * seq and seq the fastest of
// the three ([batch][head][seq][dim]); pair i of a token at position p is
// rotated by cos/sin table entry p * half + i:
//   out[2i] = x[2i]*c - x[2i+1]*s,  out[2i+1] = x[2i]*s + x[2i+1]*c,
// each product and each sum rounded on its own (no fused multiply-add), as
// the reference's float32 arithmetic does, so the results are bit-identical.
// A position outside [0, max_seq) leaves its pairs unwritten and records
// VKQ_ERR_INVALID_ARGUMENT in the status word.  x and out may be the same.
__global__ void __launch_bounds__(256) rope_kernel(const float2 *x, float2 *out, const float *__restrict__ cos_t,
                                                   const float *__restrict__ sin_t, const int *__restrict__ pos,
                                                   int64_t pairs, int64_t seq, int64_t half, int64_t max_seq) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = p % half, s = (p / half) % seq;
        const int ps = pos[s];
        if (ps < 0 || ps >= max_seq) {
            atomicExch(&g_elem_status, VKQ_ERR_INVALID_ARGUMENT);
            continue;
        }
        const float c = cos_t[(int64_t)ps * half + i], sn = sin_t[(int64_t)ps * half + i];
        const float2 v = x[p];
        out[p] = make_float2(__fsub_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, sn)),
                             __fadd_rn(__fmul_rn(v.x, sn), __fmul_rn(v.y, c)));
    }
}

int elem_read_status() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_elem_status, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_elem_status, &zero, sizeof(int));
    return v;
}

// dst[0..n) = src[0..n), src being pinned host memory that the device reads
// through its mapping.  The loads do not depend on the preceding kernel and
// are issued before griddepcontrol.wait; only the stores into dst (which the
// preceding kernel may still be reading) wait for it.  Each thread moves up
// to four floats.
__global__ void __launch_bounds__(256) stage_in_kernel(const float *__restrict__ src, float *__restrict__ dst,
                                                       int64_t n) {
    pdl_launch_dependents();
    const int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec && i0 + 4 <= n) {
        const float4 q = __ldcv(reinterpret_cast<const float4 *>(src + i0));
        v[0] = q.x;
        v[1] = q.y;
        v[2] = q.z;
        v[3] = q.w;
    } else {
        for (int j = 0; j < 4; j++)
            if (i0 + j < n) v[j] = __ldcv(src + i0 + j);
    }
    pdl_wait();
    if (vec && i0 + 4 <= n) {
        *reinterpret_cast<float4 *>(dst + i0) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        for (int j = 0; j < 4; j++)
            if (i0 + j < n) dst[i0 + j] = v[j];
    }
}

static cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, cudaStream_t s, void **args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t silu_mul(const float *gate, const float *up, float *out, int64_t n, cudaStream_t s, int device) {
    const int sms = device_sm_count(device);
    int64_t blocks = (n / 4 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 4 * sms) blocks = 4 * sms;
    void *args[] = {(void *)&gate, (void *)&up, (void *)&out, (void *)&n};
    return launch_pdl((const void *)silu_mul_kernel, dim3((unsigned)blocks), dim3(256), s, args);
}

cudaError_t rope(const float *x, float *out, const float *cos_t, const float *sin_t, const int *positions,
                 int64_t rows, int64_t seq, int64_t head_dim, int64_t max_seq, cudaStream_t s, int device) {
    const int64_t half = head_dim / 2, pairs = rows * half;
    int64_t blocks = (pairs + 255) / 256;
    const int64_t cap = 8 * (int64_t)device_sm_count(device);
    if (blocks > cap) blocks = cap;
    void *args[] = {(void *)&x, (void *)&out, (void *)&cos_t, (void *)&sin_t, (void *)&positions,
                    (void *)&pairs, (void *)&seq, (void *)&half, (void *)&max_seq};
    return launch_pdl((const void *)rope_kernel, dim3((unsigned)blocks), dim3(256), s, args);
}

cudaError_t stage_in(const float *src_mapped, float *dst, int64_t n, cudaStream_t s) {
    const int64_t blocks = (n + 1023) / 1024;
    void *args[] = {(void *)&src_mapped, (void *)&dst, (void *)&n};
    return launch_pdl((const void *)stage_in_kernel, dim3((unsigned)blocks), dim3(256), s, args);
}

cudaError_t rms_norm(const float *x, const float *weight, float *out, int64_t rows, int64_t n, float eps,
                     cudaStream_t s) {
    void *args[] = {(void *)&x, (void *)&weight, (void *)&out, (void *)&n, (void *)&eps};
    return launch_pdl((const void *)rms_norm_kernel, dim3((unsigned)rows), dim3(kNormThreads), s, args);
}

}  // namespace vkq
