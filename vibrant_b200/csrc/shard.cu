// shard.cu -- row-sharded matmul across the GPUs of one node: the column
// plan, the row-block shard encoding of a quantized weight, and the
// in-process communicator (one process driving every GPU, as vibrant's host
// does: internal/gpu/cuda.go:33-46 keeps one CUDA device per process today).
//
// Sharding follows the output columns n (vibrant's orientation: W[k][n] is
// value k*N + n of the super-block stream, internal/gguf/loader.go:24-27).
// Rank r owns columns [lo, hi) with equal widths rounded up to 32.  Its shard
// keeps, for every row k, the super-blocks that cover columns [lo, hi) of
// that row, copied whole, in a fixed number of block slots per row; the
// GEMV reads value n of row k at k*rs + ((k*N + lo) & 255) + n (see
// GatherParams in gemv.cu).  Blocks that straddle two rows (N % 256 != 0, the
// vocabulary projection) or two shards are duplicated; values outside the
// rank's columns are never read.  When N and the shard bounds are multiples
// of 256 the shard is exactly the [K, hi - lo] stream of the shard's columns.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/vkq.h"
#include "vkq_internal.h"

namespace vkq {

uint64_t peer_wait_ns() {
    static uint64_t v = [] {
        const char *e = getenv("VKQ_PEER_WAIT_MS");
        long ms = e ? strtol(e, nullptr, 10) : 0;
        if (ms <= 0 || ms > 60000) ms = 2000;
        return (uint64_t)ms * 1000000ull;
    }();
    return v;
}

static int qtype_block_bytes(int qt) { return qt == VKQ_Q4_K ? 144 : qt == VKQ_Q5_K ? 176 : qt == VKQ_Q6_K ? 210 : 0; }

// Column range of a rank: equal widths, rounded up to a multiple of 32.
static bool plan_columns(int64_t N, int world, int rank, int64_t &lo, int64_t &hi) {
    if (N <= 0 || world < 1 || rank < 0 || rank >= world) return false;
    int64_t width = (N + world - 1) / world;
    width = (width + 31) / 32 * 32;
    lo = rank * width < N ? rank * width : N;
    hi = (rank + 1) * width < N ? (rank + 1) * width : N;
    return hi > lo;
}

// Block slots per shard row for columns [lo, hi): the largest count of
// blocks any row's columns touch.  (k*N + lo) mod 256 repeats with a period
// of at most 256 rows.
int64_t shard_row_blocks(int64_t K, int64_t N, int64_t lo, int64_t hi) {
    int64_t maxoff = 0;
    const int64_t rows = K < 256 ? K : 256;
    for (int64_t k = 0; k < rows; k++) {
        const int64_t off = (k * N + lo) & 255;
        if (off > maxoff) maxoff = off;
    }
    return (maxoff + (hi - lo) - 1) / 256 + 1;
}

}  // namespace vkq

using namespace vkq;

struct vkq_comm {
    int world;
    int dev[kMaxRanks];
    unsigned *flags[kMaxRanks];  // per device: channel buffer (flag words, then flagged-word slots)
    unsigned *sync[kMaxRanks];   // per device: channel words (last call, finished CTAs, failed)
    size_t chan_bytes;           // bytes of each channel buffer
};

// Grows every device's channel buffer to hold the slots of an [M][N]
// output (zero-filled; between calls, never inside a stream capture).
static int comm_reserve(vkq_comm *c, int64_t M, int64_t N) {
    const size_t need = gather_channel_bytes(M, N);
    if (need <= c->chan_bytes) return VKQ_OK;
    for (int i = 0; i < c->world; i++) {
        cudaError_t e = cudaSetDevice(c->dev[i]);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaFree(c->flags[i]);
        if (e == cudaSuccess) {
            c->flags[i] = nullptr;
            e = cudaMalloc(&c->flags[i], need);
        }
        if (e == cudaSuccess) e = cudaMemset(c->flags[i], 0, need);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            set_error("growing the channel buffer on device %d: %s", c->dev[i], cudaGetErrorString(e));
            return VKQ_ERR_CUDA;
        }
    }
    c->chan_bytes = need;
    return VKQ_OK;
}

extern "C" {

int vkq_shard_columns(int64_t N, int world, int rank, int64_t *lo, int64_t *hi) {
    if (!lo || !hi) {
        set_error("null output pointer");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) {
        set_error("invalid world/rank %d/%d (1 to %d ranks)", world, rank, kMaxRanks);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (N % 32 != 0 || !plan_columns(N, world, rank, *lo, *hi)) {
        set_error("N=%lld cannot be split over %d ranks in column ranges of multiples of 32", (long long)N, world);
        return VKQ_ERR_UNSUPPORTED;
    }
    return VKQ_OK;
}

int vkq_shard_bytes(int qtype, int64_t K, int64_t N, int64_t col_lo, int64_t col_hi, int64_t *row_blocks,
                    int64_t *bytes) {
    const int bb = qtype_block_bytes(qtype);
    if (bb == 0) {
        set_error("unsupported qtype %d", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (!bytes || K <= 0 || N <= 0 || col_lo < 0 || col_hi > N || col_hi <= col_lo) {
        set_error("invalid arguments to vkq_shard_bytes");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    const int64_t rb = shard_row_blocks(K, N, col_lo, col_hi);
    if (row_blocks) *row_blocks = rb;
    *bytes = K * rb * bb;
    return VKQ_OK;
}

int vkq_shard_weight(int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, int64_t col_lo,
                     int64_t col_hi, void *out, int64_t out_bytes) {
    const int bb = qtype_block_bytes(qtype);
    int64_t rb = 0, need = 0;
    int st = vkq_shard_bytes(qtype, K, N, col_lo, col_hi, &rb, &need);
    if (st) return st;
    if (!w || !out) {
        set_error("null pointer passed to vkq_shard_weight");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (out_bytes < need) {
        set_error("shard buffer holds %lld bytes, needs %lld", (long long)out_bytes, (long long)need);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    if (w_bytes < ((K * N + 255) / 256) * bb) {
        set_error("weight buffer holds %lld bytes, a [%lld x %lld] weight needs %lld", (long long)w_bytes,
                  (long long)K, (long long)N, (long long)(((K * N + 255) / 256) * bb));
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    const uint8_t *src = static_cast<const uint8_t *>(w);
    uint8_t *dst = static_cast<uint8_t *>(out);
    const int64_t width = col_hi - col_lo;
    for (int64_t k = 0; k < K; k++) {
        const int64_t v0 = k * N + col_lo;
        const int64_t b0 = v0 >> 8;
        const int64_t count = ((v0 & 255) + width - 1) / 256 + 1;
        uint8_t *row = dst + k * rb * bb;
        memcpy(row, src + b0 * bb, (size_t)(count * bb));
        if (count < rb) memset(row + count * bb, 0, (size_t)((rb - count) * bb));
    }
    return VKQ_OK;
}

int vkq_comm_init(int world, const int *devices, vkq_comm **comm) {
    set_error("%s", "");
    if (!comm || !devices || world < 1 || world > kMaxRanks) {
        set_error("vkq_comm_init: 1 to %d devices", kMaxRanks);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    *comm = nullptr;
    for (int i = 0; i < world; i++)
        for (int j = 0; j < i; j++)
            if (devices[i] == devices[j]) {
                set_error("vkq_comm_init: device %d listed twice", devices[i]);
                return VKQ_ERR_INVALID_ARGUMENT;
            }
    vkq_comm *c = new vkq_comm();
    c->world = world;
    c->chan_bytes = 256 + 8 * (size_t)world;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < world && e == cudaSuccess; i++) {
        c->dev[i] = devices[i];
        e = cudaSetDevice(devices[i]);
        int major = 0;
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, devices[i]);
        if (e == cudaSuccess && major != 10) {
            set_error("device %d has compute capability %d.x; libvkq is built for sm_100a only", devices[i], major);
            for (int r = 0; r < i; r++) {
                cudaSetDevice(c->dev[r]);
                cudaFree(c->flags[r]);
                cudaFree(c->sync[r]);
            }
            delete c;
            return VKQ_ERR_UNSUPPORTED;
        }
        for (int j = 0; j < world && e == cudaSuccess; j++) {
            if (j == i) continue;
            int can = 0;
            e = cudaDeviceCanAccessPeer(&can, devices[i], devices[j]);
            if (e == cudaSuccess && !can) {
                set_error("device %d cannot access device %d's memory", devices[i], devices[j]);
                e = cudaErrorPeerAccessUnsupported;
                break;
            }
            e = cudaDeviceEnablePeerAccess(devices[j], 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) {
                cudaGetLastError();
                e = cudaSuccess;
            }
        }
        if (e == cudaSuccess) e = cudaMalloc(&c->flags[i], 256 + 8 * (size_t)world);
        if (e == cudaSuccess) e = cudaMalloc(&c->sync[i], 256);
        if (e == cudaSuccess) e = cudaMemset(c->flags[i], 0, 256 + 8 * (size_t)world);
        if (e == cudaSuccess) e = cudaMemset(c->sync[i], 0, 256);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    if (e != cudaSuccess) {
        if (vkq_last_error_empty()) set_error("vkq_comm_init: %s", cudaGetErrorString(e));
        for (int i = 0; i < world; i++) {
            if (c->flags[i] || c->sync[i]) {
                cudaSetDevice(c->dev[i]);
                if (c->flags[i]) cudaFree(c->flags[i]);
                if (c->sync[i]) cudaFree(c->sync[i]);
            }
        }
        delete c;
        return e == cudaErrorPeerAccessUnsupported ? VKQ_ERR_UNSUPPORTED : VKQ_ERR_CUDA;
    }
    *comm = c;
    return VKQ_OK;
}

int vkq_comm_reset(vkq_comm *comm) {
    set_error("%s", "");
    if (!comm) {
        set_error("null communicator");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    for (int i = 0; i < comm->world; i++) {
        cudaError_t e = cudaSetDevice(comm->dev[i]);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemset(comm->flags[i], 0, comm->chan_bytes);
        if (e == cudaSuccess) e = cudaMemset(comm->sync[i], 0, 256);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            set_error("vkq_comm_reset on device %d: %s", comm->dev[i], cudaGetErrorString(e));
            return VKQ_ERR_CUDA;
        }
    }
    return VKQ_OK;
}

int vkq_comm_destroy(vkq_comm *comm) {
    set_error("%s", "");
    if (!comm) return VKQ_OK;
    int st = VKQ_OK;
    for (int i = 0; i < comm->world; i++) {
        cudaError_t e = cudaSetDevice(comm->dev[i]);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaFree(comm->flags[i]);
        if (e == cudaSuccess) e = cudaFree(comm->sync[i]);
        if (e != cudaSuccess) {
            set_error("vkq_comm_destroy on device %d: %s", comm->dev[i], cudaGetErrorString(e));
            st = VKQ_ERR_CUDA;
        }
    }
    delete comm;
    return st;
}

int vkq_comm_size(const vkq_comm *comm) { return comm ? comm->world : 0; }

int vkq_gemv_sharded(vkq_comm *comm, int qtype, const void *const *w_shards, const int64_t *w_bytes, int64_t K,
                     int64_t N, const float *const *x, int64_t M, float *const *y, void *const *workspaces,
                     const size_t *workspace_bytes, void *const *streams) {
    set_error("%s", "");
    if (!comm || !w_shards || !w_bytes || !x || !y || !workspace_bytes || !workspaces || !streams) {
        set_error("vkq_gemv_sharded: null argument array");
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    const int world = comm->world;
    const int bb = qtype_block_bytes(qtype);
    if (bb == 0) {
        set_error("unsupported qtype %d", qtype);
        return VKQ_ERR_UNSUPPORTED;
    }
    if (M < 1 || M > 8 || K <= 0 || N <= 0 || N % 32 != 0) {
        set_error("vkq_gemv_sharded: 1 <= M <= 8 and N a multiple of 32 (M=%lld, N=%lld)", (long long)M,
                  (long long)N);
        return VKQ_ERR_UNSUPPORTED;
    }
    for (int r = 0; r < world; r++) {
        int64_t lo, hi;
        if (!plan_columns(N, world, r, lo, hi)) {
            set_error("N=%lld leaves rank %d of %d without columns", (long long)N, r, world);
            return VKQ_ERR_UNSUPPORTED;
        }
        if (!w_shards[r] || !x[r] || !y[r]) {
            set_error("vkq_gemv_sharded: null pointer for rank %d", r);
            return VKQ_ERR_INVALID_ARGUMENT;
        }
    }
    const int rs = comm_reserve(comm, M, N);
    if (rs) return rs;
    for (int r = 0; r < world; r++) {
        int64_t lo, hi;
        plan_columns(N, world, r, lo, hi);
        const int64_t rb = shard_row_blocks(K, N, lo, hi);
        if (w_bytes[r] < K * rb * bb) {
            set_error("rank %d's shard holds %lld bytes, needs %lld", r, (long long)w_bytes[r],
                      (long long)(K * rb * bb));
            return VKQ_ERR_INVALID_ARGUMENT;
        }
        cudaError_t e = cudaSetDevice(comm->dev[r]);
        if (e != cudaSuccess) {
            set_error("cudaSetDevice(%d): %s", comm->dev[r], cudaGetErrorString(e));
            return VKQ_ERR_CUDA;
        }
        GatherArgs g{};
        for (int i = 0; i < world; i++) {
            g.peer_y[i] = y[i];
            g.peer_flags[i] = comm->flags[i];
        }
        g.sync = comm->sync[r];
        g.world = world;
        g.rank = r;
        g.y_ld = N;
        g.col_off = lo;
        g.rs = rb * 256;
        g.ld = N;
        g.n_base = lo;
        g.wait_ns = peer_wait_ns();
        g.slot_elems = (int64_t)((comm->chan_bytes - 256) / 16);
        GemvShape s{qtype, K, hi - lo, M};
        const int st = gemv_launch(s, w_shards[r], w_bytes[r], x[r], nullptr, workspaces[r], workspace_bytes[r],
                                   (cudaStream_t)streams[r], comm->dev[r], &g);
        if (st) return st;
    }
    return VKQ_OK;
}

}  // extern "C"
