// capi.cu -- extern "C" entry points of libvkq.so (declared in include/vkq.h).
//
// Each entry point makes `device` current on the calling thread, validates
// its arguments the way vibrant's cgo wrappers do before launching
// (internal/gpu/cuda/library.go:95-100: null pointers and non-positive
// dimensions are rejected), launches on the caller's stream and reports
// errors as a status code plus a thread-local message instead of the
// reference's "return nil and fall back to the CPU" (ops_cuda.go:34-38,75-84):
// this path has no CPU fallback.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/vkq.h"
#include "vkq_internal.h"

namespace vkq {

static thread_local char t_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

int device_sm_count(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 64) dev = 63;
    std::lock_guard<std::mutex> g(mu);
    if (cache[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cache[dev] = v;
    }
    return cache[dev];
}

bool vkq_last_error_empty() { return t_err[0] == '\0'; }

cudaError_t kernel_smem(const void *fn, size_t smem, bool carveout) {
    struct Entry {
        const void *fn;
        int dev;
        size_t smem;
    };
    static std::mutex mu;
    static Entry table[512];
    static int used = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(mu);
    int i = 0;
    while (i < used && (table[i].fn != fn || table[i].dev != dev)) i++;
    if (i < used && table[i].smem >= smem) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && carveout) e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (i == used && used < 512) table[used++] = Entry{fn, dev, smem};
    else if (i < used) table[i].smem = smem;
    return cudaSuccess;
}

static int block_bytes(int qt) {
    switch (qt) {
    case VKQ_Q4_K: return 144;
    case VKQ_Q5_K: return 176;
    case VKQ_Q6_K: return 210;
    default: return 0;
    }
}

// Makes the device current and checks it is a compute capability 10.x part
// (the kernels are built for sm_100a only).
static int enter(int device) {
    t_err[0] = '\0';
    int dev = device;
    int cur = -1;
    if (device >= 0 && (cudaGetDevice(&cur) != cudaSuccess || cur != device)) {
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) {
            set_error("cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
            return VKQ_ERR_CUDA;
        }
    } else if (cudaGetDevice(&dev) != cudaSuccess) {
        set_error("no current CUDA device");
        return VKQ_ERR_CUDA;
    }
    static int cc_major[64] = {0};
    int d = dev < 64 ? dev : 63;
    if (cc_major[d] == 0) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
            set_error("cannot query device %d", dev);
            return VKQ_ERR_CUDA;
        }
        cc_major[d] = major;
    }
    if (cc_major[d] != 10) {
        set_error("device %d has compute capability %d.x; libvkq is built for sm_100a only", dev, cc_major[d]);
        return VKQ_ERR_UNSUPPORTED;
    }
    return VKQ_OK;
}

static int check_launch(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return VKQ_ERR_CUDA;
    }
    return VKQ_OK;
}

// Largest x or y that vkq_matmul_host moves through the host mapping.
constexpr size_t kStageBytes = 1 << 20;

// The device address of pinned host memory mapped into the current device's
// address space, or null for any other memory.
static void *mapped_host(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

static int check_matmul_args(int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
                             int64_t M, float *y) {
    int bb = block_bytes(qtype);
    if (bb == 0) {
        set_error("unsupported qtype %d (expected 12, 13 or 14)", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!w || !x || !y) {
        set_error("null pointer passed to matmul");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (K <= 0 || N <= 0 || M <= 0) {
        set_error("invalid dimensions: M=%lld, N=%lld, K=%lld", (long long)M, (long long)N, (long long)K);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (K > (int64_t(1) << 40) / N) {
        set_error("weight too large: K=%lld N=%lld", (long long)K, (long long)N);
        return VKQ_ERR_UNSUPPORTED;
    }
    const int64_t need = ((K * N + 255) / 256) * bb;
    if (w_bytes < need) {
        set_error("weight buffer holds %lld bytes, a [%lld x %lld] weight needs %lld", (long long)w_bytes,
                  (long long)K, (long long)N, (long long)need);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (reinterpret_cast<uintptr_t>(w) & 15u) {
        set_error("weight pointer must be 16-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 3u) {
        set_error("x and y must be 4-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    return VKQ_OK;
}

}  // namespace vkq

using namespace vkq;

extern "C" {

int vkq_abi_version(void) { return VKQ_ABI_VERSION; }

const char *vkq_status_string(int status) {
    switch (status) {
    case VKQ_OK: return "ok";
    case VKQ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case VKQ_ERR_UNSUPPORTED: return "unsupported";
    case VKQ_ERR_MISALIGNED: return "misaligned pointer";
    case VKQ_ERR_WORKSPACE: return "workspace missing or too small";
    case VKQ_ERR_CUDA: return "CUDA error";
    case VKQ_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case VKQ_ERR_NCCL: return "NCCL error";
    case VKQ_ERR_PEER: return "a peer rank is out of step, or the channel failed earlier";
    default: return "unknown status";
    }
}

const char *vkq_last_error(void) { return t_err; }

int64_t vkq_block_bytes(int qtype) { return block_bytes(qtype); }

int vkq_weight_bytes(int qtype, int64_t K, int64_t N, int64_t *bytes) {
    t_err[0] = '\0';
    int bb = block_bytes(qtype);
    if (bb == 0) {
        set_error("unsupported qtype %d", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!bytes || K <= 0 || N <= 0) {
        set_error("invalid arguments to vkq_weight_bytes");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    *bytes = ((K * N + 255) / 256) * bb;
    return VKQ_OK;
}

int vkq_dequantize_f32(int device, int qtype, const void *w, int64_t nblocks, float *out, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (block_bytes(qtype) == 0) {
        set_error("unsupported qtype %d", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!w || !out || nblocks <= 0) {
        set_error("invalid arguments to vkq_dequantize_f32");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (reinterpret_cast<uintptr_t>(out) & 3u) {
        set_error("out must be 4-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(dequantize_f32(qtype, w, nblocks, out, (cudaStream_t)stream, device), "dequantize");
}

int vkq_dequant_transpose_f32(int device, int qtype, const void *w, int64_t K, int64_t N, float *out,
                              void *stream) {
    int st = enter(device);
    if (st) return st;
    if (block_bytes(qtype) == 0) {
        set_error("unsupported qtype %d", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!w || !out || K <= 0 || N <= 0) {
        set_error("invalid arguments to vkq_dequant_transpose_f32");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    return check_launch(dequant_transpose_f32(qtype, w, K, N, out, (cudaStream_t)stream, device),
                        "dequant_transpose");
}

int vkq_matmul_workspace_bytes(int device, int qtype, int64_t M, int64_t K, int64_t N, size_t *bytes) {
    int st = enter(device);
    if (st) return st;
    if (!bytes || M <= 0 || K <= 0 || N <= 0 || block_bytes(qtype) == 0) {
        set_error("invalid arguments to vkq_matmul_workspace_bytes");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    GemvShape s{qtype, K, N, M};
    if (M <= 8) {
        *bytes = gemv_workspace_bytes(s, device);
        return VKQ_OK;
    }
    // tensor-core GEMM (bf16 copy of x), or 8-row GEMV chunks for shapes it does not serve
    GemvShape s8{qtype, K, N, 8};
    size_t a = gemm_workspace_bytes(s, device), b = gemv_workspace_bytes(s8, device);
    *bytes = a > b ? a : b;
    return VKQ_OK;
}

int vkq_gemv(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
             int64_t M, float *y, void *workspace, size_t workspace_bytes, void *stream) {
    int st = enter(device);
    if (st) return st;
    st = check_matmul_args(qtype, w, w_bytes, K, N, x, M, y);
    if (st) return st;
    if (M > 8) {
        set_error("vkq_gemv serves 1 <= M <= 8 (got %lld)", (long long)M);
        return VKQ_ERR_UNSUPPORTED;
    }
    GemvShape s{qtype, K, N, M};
    return gemv_launch(s, w, w_bytes, x, y, workspace, workspace_bytes, (cudaStream_t)stream, device);
}

int vkq_gemv_noalloc(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
                     int64_t M, float *y, void *stream) {
    int st = enter(device);
    if (st) return st;
    st = check_matmul_args(qtype, w, w_bytes, K, N, x, M, y);
    if (st) return st;
    if (M > 8) {
        set_error("vkq_gemv_noalloc serves 1 <= M <= 8 (got %lld)", (long long)M);
        return VKQ_ERR_UNSUPPORTED;
    }
    GemvShape s{qtype, K, N, M};
    return gemv_launch_noalloc(s, w, w_bytes, x, y, (cudaStream_t)stream, device);
}

int vkq_gemm(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
             int64_t M, float *y, void *workspace, size_t workspace_bytes, void *stream) {
    int st = enter(device);
    if (st) return st;
    st = check_matmul_args(qtype, w, w_bytes, K, N, x, M, y);
    if (st) return st;
    GemvShape s{qtype, K, N, M};
    return gemm_launch(s, w, w_bytes, x, y, workspace, workspace_bytes, (cudaStream_t)stream, device);
}

int vkq_matmul(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
               int64_t M, float *y, void *workspace, size_t workspace_bytes, void *stream) {
    if (M <= 8) return vkq_gemv(device, qtype, w, w_bytes, K, N, x, M, y, workspace, workspace_bytes, stream);
    int st = enter(device);
    if (st) return st;
    st = check_matmul_args(qtype, w, w_bytes, K, N, x, M, y);
    if (st) return st;
    if (N % 32 == 0 && K % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 7u) == 0)
        return vkq_gemm(device, qtype, w, w_bytes, K, N, x, M, y, workspace, workspace_bytes, stream);
    // shapes the tensor-core kernel does not serve: fp32 GEMV over 8-row chunks
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int64_t mc = (M - m0) < 8 ? (M - m0) : 8;
        GemvShape s{qtype, K, N, mc};
        st = gemv_launch(s, w, w_bytes, x + m0 * K, y + m0 * N, workspace, workspace_bytes, (cudaStream_t)stream,
                         device);
        if (st) return st;
    }
    return VKQ_OK;
}

int vkq_matmul_upstream(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, const float *x,
                        int64_t M, float *y, void *stream) {
    int st = enter(device);
    if (st) return st;
    st = check_matmul_args(qtype, w, w_bytes, K, N, x, M, y);  // the same blocks: ceil(K*N/256)
    if (st) return st;
    if (K % 256 != 0) {
        set_error("vkq_matmul_upstream needs K %% 256 == 0 (rows of whole super-blocks), got K=%lld", (long long)K);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (reinterpret_cast<uintptr_t>(x) & 15u) {
        set_error("vkq_matmul_upstream needs x 16-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(gemv_rows_launch(qtype, w, K, N, x, M, y, (cudaStream_t)stream, device),
                        "upstream-orientation GEMV launch");
}

int vkq_matmul_host(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                    const float *x_host, int64_t M, float *y_host, float *x_dev, float *y_dev, void *workspace,
                    size_t workspace_bytes, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!x_host || !y_host) {
        set_error("vkq_matmul_host: null host buffer");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    st = check_matmul_args(qtype, w, w_bytes, K, N, x_dev, M, y_dev);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t xb = (size_t)(M * K) * sizeof(float), yb = (size_t)(M * N) * sizeof(float);
    // Pinned host buffers are reached through their device mapping: a small
    // kernel reads x (before the preceding kernel ends) and the GEMV stores y
    // straight into host memory, with no copy-engine round trips; other host
    // memory, and larger prefill inputs and outputs, go by cudaMemcpyAsync.
    const float *x_map = xb <= kStageBytes ? static_cast<const float *>(mapped_host(x_host)) : nullptr;
    float *y_map = (M <= 8 && yb <= kStageBytes) ? static_cast<float *>(mapped_host(y_host)) : nullptr;
    if (x_map)
        st = check_launch(stage_in(x_map, x_dev, M * K, s), "reading x from the host");
    else
        st = check_launch(cudaMemcpyAsync(x_dev, x_host, xb, cudaMemcpyHostToDevice, s), "copying x to the device");
    if (st) return st;
    st = vkq_matmul(device, qtype, w, w_bytes, K, N, x_dev, M, y_map ? y_map : y_dev, workspace, workspace_bytes,
                    stream);
    if (st || y_map) return st;
    return check_launch(cudaMemcpyAsync(y_host, y_dev, yb, cudaMemcpyDeviceToHost, s), "copying y to the host");
}

int vkq_ipc_alloc(int device, size_t bytes, void **ptr, unsigned char handle[64]) {
    int st = enter(device);
    if (st) return st;
    if (!ptr || !handle || bytes == 0) {
        set_error("invalid arguments to vkq_ipc_alloc");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return check_launch(e, "vkq_ipc_alloc");
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle, &h, 64);
    *ptr = p;
    return VKQ_OK;
}

int vkq_ipc_open(int device, const unsigned char handle[64], void **ptr) {
    int st = enter(device);
    if (st) return st;
    if (!ptr || !handle) {
        set_error("invalid arguments to vkq_ipc_open");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    return check_launch(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "vkq_ipc_open");
}

int vkq_ipc_close(int device, void *ptr) {
    int st = enter(device);
    if (st) return st;
    return check_launch(cudaIpcCloseMemHandle(ptr), "vkq_ipc_close");
}

int vkq_ipc_free(int device, void *ptr) {
    int st = enter(device);
    if (st) return st;
    return check_launch(cudaFree(ptr), "vkq_ipc_free");
}

int vkq_gemv_allgather(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, int64_t col_lo,
                       int64_t col_hi, const float *x, int64_t M, void *const *peer_out, void *const *peer_flags,
                       void *sync, int world, int rank, void *workspace, size_t workspace_bytes, void *stream) {
    int st = enter(device);
    if (st) return st;
    const int bb = block_bytes(qtype);
    if (bb == 0) {
        set_error("unsupported qtype %d (expected 12, 13 or 14)", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!w || !x || !sync || !peer_out || !peer_flags || K <= 0 || N <= 0 || M <= 0) {
        set_error("vkq_gemv_allgather: null pointer or non-positive size");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (M > 8) {
        set_error("vkq_gemv_allgather serves 1 <= M <= 8 (got %lld)", (long long)M);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || N % 32 != 0 || col_lo < 0 || col_hi > N ||
        col_hi <= col_lo || col_lo % 32 != 0 || col_hi % 32 != 0) {
        set_error("vkq_gemv_allgather: invalid world/rank (%d/%d, at most %d ranks) or columns [%lld, %lld) of "
                  "N=%lld (multiples of 32 needed)",
                  world, rank, kMaxRanks, (long long)col_lo, (long long)col_hi, (long long)N);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (reinterpret_cast<uintptr_t>(w) & 15u) {
        set_error("weight pointer must be 16-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    const int64_t rb = shard_row_blocks(K, N, col_lo, col_hi);
    if (w_bytes < K * rb * bb) {
        set_error("the shard holds %lld bytes; columns [%lld, %lld) of a [%lld x %lld] weight need %lld "
                  "(vkq_shard_bytes)",
                  (long long)w_bytes, (long long)col_lo, (long long)col_hi, (long long)K, (long long)N,
                  (long long)(K * rb * bb));
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    GatherArgs g{};
    for (int r = 0; r < world; r++) {
        if (!peer_out[r] || !peer_flags[r]) {
            set_error("vkq_gemv_allgather: null peer buffer for rank %d", r);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        g.peer_y[r] = static_cast<float *>(peer_out[r]);
        g.peer_flags[r] = static_cast<unsigned *>(peer_flags[r]);
    }
    if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(g.peer_y[rank]) & 15u)) {
        set_error("x must be 4-byte and the output buffers 16-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    g.sync = static_cast<unsigned *>(sync);
    g.world = world;
    g.rank = rank;
    g.y_ld = N;
    g.col_off = col_lo;
    g.rs = rb * 256;
    g.ld = N;
    g.n_base = col_lo;
    g.wait_ns = peer_wait_ns();
    g.slot_elems = M * N;  // the channel buffers hold vkq_gather_channel_bytes(M, N) (the contract)
    GemvShape s{qtype, K, col_hi - col_lo, M};
    return gemv_launch(s, w, w_bytes, x, nullptr, workspace, workspace_bytes, (cudaStream_t)stream, device, &g);
}

int vkq_set_gemv_path(int path) {
    t_err[0] = '\0';
    if (path < 0 || path > 3) {
        set_error("vkq_set_gemv_path: 0 (automatic), 1 (CUDA cores), 2 (tensor cores) or 3 (column strips)");
        return -1;
    }
    return set_gemv_path(path);
}

int vkq_silu_mul(int device, const float *gate, const float *up, float *out, int64_t n, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!gate || !up || !out || n <= 0) {
        set_error("invalid arguments to vkq_silu_mul");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(out)) &
        15u) {
        set_error("vkq_silu_mul needs 16-byte aligned buffers");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(silu_mul(gate, up, out, n, (cudaStream_t)stream, device), "silu_mul");
}

int vkq_rms_norm(int device, const float *x, const float *weight, float *out, int64_t rows, int64_t n, float eps,
                 void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!x || !weight || !out || rows <= 0 || n <= 0 || rows > 0x7FFFFFFF || !(eps >= 0.0f)) {
        set_error("invalid arguments to vkq_rms_norm");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out)) &
        3u) {
        set_error("vkq_rms_norm needs 4-byte aligned buffers");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(rms_norm(x, weight, out, rows, n, eps, (cudaStream_t)stream), "rms_norm");
}

int vkq_rope_f32(int device, const float *x, float *out, const float *cos_table, const float *sin_table,
                 const int32_t *positions, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t max_seq,
                 void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!x || !out || !cos_table || !sin_table || !positions || batch <= 0 || heads <= 0 || seq <= 0 ||
        head_dim <= 0 || head_dim % 2 != 0 || max_seq <= 0 || batch * heads * seq > (int64_t(1) << 40) / head_dim) {
        set_error("invalid arguments to vkq_rope_f32 (head_dim must be even, every count positive)");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 7u) {
        set_error("vkq_rope_f32 needs x and out 8-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(rope(x, out, cos_table, sin_table, positions, batch * heads * seq, seq, head_dim, max_seq,
                             (cudaStream_t)stream, device),
                        "rope");
}

int vkq_attention_decode_f32(int device, const float *q, const float *k_cache, const float *v_cache, float *out,
                             int64_t batch, int64_t heads, int64_t kv_heads, int64_t len, int64_t cache_len,
                             int64_t head_dim, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!q || !k_cache || !v_cache || !out || batch <= 0 || batch > 65535 || heads <= 0 || heads > 65535 ||
        kv_heads <= 0 || heads % kv_heads != 0 || len <= 0 || cache_len < len ||
        (uint64_t)len > attention_max_len()) {
        set_error("invalid arguments to vkq_attention_decode_f32 (heads a multiple of kv_heads, 0 < len <= "
                  "cache_len, len <= %zu)",
                  attention_max_len());
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (head_dim != 64 && head_dim != 128) {
        set_error("vkq_attention_decode_f32 serves head_dim 64 or 128 (got %lld)", (long long)head_dim);
        return VKQ_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(out)) &
        3u) {
        set_error("vkq_attention_decode_f32 needs 4-byte aligned buffers");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(attention_decode(q, k_cache, v_cache, out, batch, heads, kv_heads, len, cache_len, head_dim,
                                         (cudaStream_t)stream),
                        "decode attention");
}

int vkq_attention_rope_decode_f32(int device, const float *q, const float *k_new, const float *v_new,
                                  const float *cos_table, const float *sin_table, const int32_t *positions,
                                  float *k_cache, float *v_cache, float *out, int64_t batch, int64_t heads,
                                  int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim, int64_t max_seq,
                                  void *stream) {
    int st = enter(device);
    if (st) return st;
    if (!q || !k_new || !v_new || !cos_table || !sin_table || !positions || !k_cache || !v_cache || !out ||
        batch <= 0 || batch > 65535 || heads <= 0 || heads > 65535 || kv_heads <= 0 || heads % kv_heads != 0 ||
        len <= 0 || cache_len < len || (uint64_t)len > attention_max_len() || max_seq <= 0) {
        set_error("invalid arguments to vkq_attention_rope_decode_f32 (heads a multiple of kv_heads, 0 < len <= "
                  "cache_len, len <= %zu, max_seq > 0)",
                  attention_max_len());
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (head_dim != 64 && head_dim != 128) {
        set_error("vkq_attention_rope_decode_f32 serves head_dim 64 or 128 (got %lld)", (long long)head_dim);
        return VKQ_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
         reinterpret_cast<uintptr_t>(cos_table) | reinterpret_cast<uintptr_t>(sin_table) |
         reinterpret_cast<uintptr_t>(positions) | reinterpret_cast<uintptr_t>(k_cache) |
         reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out)) &
        3u) {
        set_error("vkq_attention_rope_decode_f32 needs 4-byte aligned buffers");
        return VKQ_ERR_MISALIGNED;
    }
    return check_launch(attention_decode_rope(q, k_new, v_new, cos_table, sin_table, positions, k_cache, v_cache, out,
                                              batch, heads, kv_heads, len, cache_len, head_dim, max_seq,
                                              (cudaStream_t)stream),
                        "fused decode attention");
}

size_t vkq_gather_channel_bytes(int64_t m_max, int64_t N) {
    return m_max > 0 && N > 0 ? gather_channel_bytes(m_max, N) : 0;
}

int vkq_linear_fused(int device, int qtype, int nweights, const void *const *w, const int64_t *w_bytes, int64_t K,
                     const int64_t *N, const float *x, int64_t M, const float *norm_w, float eps, int epilogue,
                     float *const *y, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (qtype != VKQ_Q4_K) {
        set_error("vkq_linear_fused serves Q4_K weights (got qtype %d)", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!w || !w_bytes || !N || !y || !x || K <= 0 || M < 1 || M > 4 || nweights < 1 ||
        nweights > kMaxStripSegs || (epilogue != VKQ_EPI_NONE && epilogue != VKQ_EPI_SILU_MUL) ||
        (epilogue == VKQ_EPI_SILU_MUL && nweights != 2) || (norm_w && (M > 3 || !(eps >= 0.0f)))) {
        set_error("invalid arguments to vkq_linear_fused");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(norm_w)) & 3u) {
        set_error("x and norm_w must be 4-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    StripSeg segs[kMaxStripSegs];
    for (int i = 0; i < nweights; i++) {
        const bool out = i == 0 || epilogue == VKQ_EPI_NONE;
        if (!w[i] || N[i] <= 0 || N[i] % 256 != 0 || (out && !y[i])) {
            set_error("weight %d: null pointer or N=%lld not a positive multiple of 256", i, (long long)N[i]);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        if (K > (int64_t(1) << 40) / N[i] || w_bytes[i] < K * N[i] / 256 * 144) {
            set_error("weight %d: buffer of %lld bytes for a [%lld x %lld] Q4_K weight", i, (long long)w_bytes[i],
                      (long long)K, (long long)N[i]);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        if ((reinterpret_cast<uintptr_t>(w[i]) & 15u) || (out && (reinterpret_cast<uintptr_t>(y[i]) & 3u))) {
            set_error("weight %d: weights must be 16-byte and outputs 4-byte aligned", i);
            return VKQ_ERR_MISALIGNED;
        }
        segs[i] = StripSeg{w[i], w_bytes[i], N[i], N[i], 0, out ? y[i] : nullptr, N[i], 0};
    }
    const int r = gemv_strip_multi((int)M, K, segs, nweights, epilogue == VKQ_EPI_SILU_MUL, x, norm_w, eps,
                                   (cudaStream_t)stream, device);
    return r == 0 ? VKQ_OK : r == 2 ? VKQ_ERR_INVALID_ARGUMENT : r == 3 ? VKQ_ERR_UNSUPPORTED : VKQ_ERR_CUDA;
}

int vkq_linear_fused_allgather(int device, int qtype, int nweights, const void *const *w, const int64_t *w_bytes,
                               int64_t K, int64_t N, int64_t col_lo, int64_t col_hi, const int64_t *N_local,
                               const float *x, int64_t M, const float *norm_w, float eps, int epilogue,
                               float *const *y_local, void *const *peer_out, void *const *peer_flags, void *sync,
                               int world, int rank, void *stream) {
    int st = enter(device);
    if (st) return st;
    if (qtype != VKQ_Q4_K) {
        set_error("vkq_linear_fused_allgather serves Q4_K weights (got qtype %d)", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    const bool silu = epilogue == VKQ_EPI_SILU_MUL;
    if (!w || !w_bytes || !x || !sync || !peer_out || !peer_flags || K <= 0 || M < 1 || M > 4 || nweights < 1 ||
        nweights > kMaxStripSegs || (epilogue != VKQ_EPI_NONE && !silu) || (silu && nweights != 2) ||
        (!silu && nweights > 1 && (!N_local || !y_local)) || (norm_w && (M > 3 || !(eps >= 0.0f)))) {
        set_error("invalid arguments to vkq_linear_fused_allgather");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || N <= 0 || N % 256 != 0 || col_lo < 0 ||
        col_hi > N || col_hi <= col_lo || col_lo % 32 != 0 || col_hi % 32 != 0) {
        set_error("vkq_linear_fused_allgather: invalid world/rank (%d/%d) or columns [%lld, %lld) of N=%lld "
                  "(N a multiple of 256, columns of 32)",
                  world, rank, (long long)col_lo, (long long)col_hi, (long long)N);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(norm_w)) & 3u) {
        set_error("x and norm_w must be 4-byte aligned");
        return VKQ_ERR_MISALIGNED;
    }
    GatherArgs g{};
    for (int r = 0; r < world; r++) {
        if (!peer_out[r] || !peer_flags[r]) {
            set_error("vkq_linear_fused_allgather: null peer buffer for rank %d", r);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        g.peer_y[r] = static_cast<float *>(peer_out[r]);
        g.peer_flags[r] = static_cast<unsigned *>(peer_flags[r]);
    }
    const int64_t rb = shard_row_blocks(K, N, col_lo, col_hi);
    StripSeg segs[kMaxStripSegs];
    for (int i = 0; i < nweights; i++) {
        const bool shard = i == 0 || silu;
        const int64_t n_i = shard ? N : N_local[i];
        const int64_t need = shard ? K * rb * 144 : (n_i > 0 ? K * n_i / 256 * 144 : 0);
        if (!w[i] || n_i <= 0 || n_i % 256 != 0 || (!shard && !y_local[i]) || w_bytes[i] < need) {
            set_error("weight %d: null pointer, N not a multiple of 256, or a buffer of %lld bytes (needs %lld)", i,
                      (long long)w_bytes[i], (long long)need);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        if ((reinterpret_cast<uintptr_t>(w[i]) & 15u) || (!shard && (reinterpret_cast<uintptr_t>(y_local[i]) & 3u))) {
            set_error("weight %d: weights must be 16-byte and outputs 4-byte aligned", i);
            return VKQ_ERR_MISALIGNED;
        }
        segs[i] = shard ? StripSeg{w[i], w_bytes[i], col_hi - col_lo, rb * 256, col_lo & 255, g.peer_y[rank], N, col_lo}
                        : StripSeg{w[i], w_bytes[i], n_i, n_i, 0, y_local[i], n_i, 0};
    }
    g.sync = static_cast<unsigned *>(sync);
    g.world = world;
    g.rank = rank;
    g.y_ld = N;
    g.col_off = col_lo;
    g.rs = rb * 256;
    g.ld = N;
    g.n_base = col_lo;
    g.wait_ns = peer_wait_ns();
    g.slot_elems = M * N;  // the channel buffers hold vkq_gather_channel_bytes(M, N) (the contract)
    const int r = gemv_strip_multi((int)M, K, segs, nweights, silu, x, norm_w, eps, (cudaStream_t)stream, device, &g);
    return r == 0 ? VKQ_OK : r == 2 ? VKQ_ERR_INVALID_ARGUMENT : r == 3 ? VKQ_ERR_UNSUPPORTED : VKQ_ERR_CUDA;
}

int vkq_device_status(int device, int *code) {
    int st = enter(device);
    if (st) return st;
    if (!code) {
        set_error("null code pointer");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return check_launch(e, "cudaDeviceSynchronize");
    int g = gemv_read_status();
    const int g2 = gemm_read_status();
    const int g3 = gemv_tc_read_status();
    const int g4 = gemv_strip_read_status();
    const int g5 = elem_read_status();
    const int g6 = attention_read_status();
    if (g == 0) g = g2;
    if (g == 0) g = g3;
    if (g == 0) g = g4;
    if (g == 0) g = g5;
    if (g == 0) g = g6;
    if (g < 0 || g2 < 0 || g3 < 0 || g4 < 0 || g5 < 0 || g6 < 0) {
        set_error("cannot read the device status word");
        return VKQ_ERR_CUDA;
    }
    *code = g ? g : VKQ_OK;
    return VKQ_OK;
}

}  // extern "C"
