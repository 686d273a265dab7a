// gguf.cu -- GGUF weights to the device, still quantized (host code).
//
// Replaces the GPU upload route of the reference: gguf.ParseGGUF
// (internal/gguf/parser.go:15-64) + GGUFFile.LoadTensor (loader.go:11-73) +
// Tensor.ToDevice, which expands every k-quant tensor to float32 on the host
// first (dequantizeForGPU, internal/tensor/tensor_cuda_api.go:16-53).  Here
// the file is memory-mapped, the header, metadata and tensor infos are parsed
// with bounds checks (metadata values are skipped; the reader keeps only
// what the matmul path needs), and a tensor's raw super-blocks go to device
// memory through pinned staging buffers and cudaMemcpyAsync: 0.56 / 0.69 /
// 0.82 bytes per weight instead of 4.  A rank can load only its row-block
// shard (vkq_shard_weight's layout) straight from the mapping.
//
// Layout facts followed (the reference's reading of the format): magic
// "GGUF", versions 2 and 3, u64 counts, length-prefixed strings, the tensor
// data section at the end of the tensor infos rounded up to 32 bytes
// (parser.go:53-60), shape = the GGUF dims in file order (loader.go:24-27),
// and calculateTensorSize's byte counts (metadata.go:170-204), which -- unlike
// LoadTensor's expectedSize (loader.go:35-48) -- covers Q4_K.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/vkq.h"
#include "vkq_internal.h"

namespace vkq {

struct GgufTensor {
    std::string name;
    uint32_t n_dims;
    int64_t dims[4];
    uint32_t type;
    uint64_t offset;  // relative to the data section
    int64_t bytes;
};

// calculateTensorSize (internal/gguf/metadata.go:170-204); -1 for a type it does not size
static int64_t ggml_bytes(uint32_t type, int64_t elements) {
    switch (type) {
    case 0: return elements * 4;                   // F32
    case 1: return elements * 2;                   // F16
    case 2: return (elements + 31) / 32 * 18;      // Q4_0
    case 8: return (elements + 31) / 32 * 34;      // Q8_0
    case 12: return (elements + 255) / 256 * 144;  // Q4_K
    case 13: return (elements + 255) / 256 * 176;  // Q5_K
    case 14: return (elements + 255) / 256 * 210;  // Q6_K
    case 15: return (elements + 255) / 256 * 292;  // Q8_K
    default: return -1;
    }
}

}  // namespace vkq

using namespace vkq;

struct vkq_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t data_offset = 0;
    std::vector<GgufTensor> tensors;
};

namespace {

struct Reader {
    const uint8_t *p;
    size_t n, pos = 0;
    bool ok = true;
    bool take(void *dst, size_t k) {
        if (!ok || k > n - pos) return ok = false;
        memcpy(dst, p + pos, k);
        pos += k;
        return true;
    }
    bool skip(uint64_t k) {
        if (!ok || k > n - pos) return ok = false;
        pos += (size_t)k;
        return true;
    }
    template <typename T> bool get(T &v) { return take(&v, sizeof(T)); }
    bool str(std::string *out, uint64_t limit) {
        uint64_t len = 0;
        if (!get(len) || len > limit || len > n - pos) return ok = false;
        if (out) out->assign(reinterpret_cast<const char *>(p + pos), (size_t)len);
        pos += (size_t)len;
        return true;
    }
    // a metadata value of type vt (parser.go readMetadataValue / readArray)
    bool value(uint32_t vt, int depth) {
        static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -1, 8, 8, 8};  // types 0..12
        if (vt > 12 || depth > 4) return ok = false;
        if (vt == 8) return str(nullptr, uint64_t(1) << 30);
        if (vt == 9) {
            uint32_t et = 0;
            uint64_t len = 0;
            if (!get(et) || !get(len) || len > (uint64_t(1) << 28)) return ok = false;
            if (et <= 12 && sizes[et] > 0) return skip(len * (uint64_t)sizes[et]);
            for (uint64_t i = 0; i < len && ok; i++) value(et, depth + 1);
            return ok;
        }
        return skip((uint64_t)sizes[vt]);
    }
};

int fail(int code, const char *msg);

// Host bytes -> device through two pinned staging buffers (the copy of one
// chunk into pinned memory overlaps the DMA of the previous one); nothing
// is expanded.  `gather` fills a staging chunk [off, off + n) of the output.
template <typename Gather>
int upload(int device, void *dst, int64_t total, cudaStream_t stream, Gather gather) {
    constexpr size_t kChunk = size_t(8) << 20;
    void *stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaError_t e = cudaSetDevice(device);
    for (int i = 0; i < 2 && e == cudaSuccess; i++) {
        e = cudaHostAlloc(&stage[i], kChunk, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
    }
    int64_t off = 0;
    for (int i = 0; e == cudaSuccess && off < total; i ^= 1) {
        const size_t n = (size_t)(total - off) < kChunk ? (size_t)(total - off) : kChunk;
        e = cudaEventSynchronize(done[i]);  // the buffer's previous copy has landed
        if (e != cudaSuccess) break;
        gather(static_cast<uint8_t *>(stage[i]), off, n);
        e = cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, stage[i], n, cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaEventRecord(done[i], stream);
        off += (int64_t)n;
    }
    for (int i = 0; i < 2; i++) {
        if (done[i]) {
            if (e == cudaSuccess) e = cudaEventSynchronize(done[i]);
            cudaEventDestroy(done[i]);
        }
        if (stage[i]) cudaFreeHost(stage[i]);
    }
    if (e != cudaSuccess) {
        set_error("uploading GGUF tensor data: %s", cudaGetErrorString(e));
        return VKQ_ERR_CUDA;
    }
    return VKQ_OK;
}

int fail(int code, const char *msg) {
    set_error("%s", msg);
    return code;
}

}  // namespace

extern "C" {

int vkq_gguf_tensor_bytes(int ggml_type, int n_dims, const int64_t *dims, int64_t *bytes) {
    set_error("%s", "");
    if (!dims || !bytes || n_dims < 1 || n_dims > 4) return fail(VKQ_ERR_INVALID_ARGUMENT, "invalid dims");
    int64_t e = 1;
    for (int i = 0; i < n_dims; i++) {
        if (dims[i] < 0 || (dims[i] > 0 && e > (int64_t(1) << 50) / dims[i]))
            return fail(VKQ_ERR_INVALID_ARGUMENT, "tensor too large");
        e *= dims[i];
    }
    const int64_t b = ggml_bytes((uint32_t)ggml_type, e);
    if (b < 0) return fail(VKQ_ERR_UNSUPPORTED, "tensor type without a size rule");
    *bytes = b;
    return VKQ_OK;
}

int vkq_gguf_open(const char *path, vkq_gguf **out) {
    set_error("%s", "");
    if (!path || !out) return fail(VKQ_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_error("cannot open %s", path);
        return VKQ_ERR_INVALID_ARGUMENT;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return fail(VKQ_ERR_INVALID_ARGUMENT, "not a GGUF file (too short)");
    }
    void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        close(fd);
        return fail(VKQ_ERR_INVALID_ARGUMENT, "cannot map the file");
    }
    vkq_gguf *g = new vkq_gguf();
    g->fd = fd;
    g->map = static_cast<const uint8_t *>(m);
    g->size = (size_t)st.st_size;
    Reader r{g->map, g->size};
    uint32_t magic = 0;
    uint64_t n_tensors = 0, n_kv = 0;
    int code = VKQ_OK;
    const char *why = nullptr;
    if (!r.get(magic) || magic != 0x46554747u) {
        code = VKQ_ERR_INVALID_ARGUMENT;
        why = "invalid magic (not GGUF)";
    } else if (!r.get(g->version) || g->version < 2 || g->version > 3) {
        code = VKQ_ERR_UNSUPPORTED;
        why = "unsupported GGUF version (2 and 3 are read)";
    } else if (!r.get(n_tensors) || !r.get(n_kv) || n_tensors > (uint64_t(1) << 24) || n_kv > (uint64_t(1) << 24)) {
        code = VKQ_ERR_INVALID_ARGUMENT;
        why = "bad tensor or metadata count";
    }
    for (uint64_t i = 0; code == VKQ_OK && i < n_kv; i++) {
        uint32_t vt = 0;
        if (!r.str(nullptr, uint64_t(1) << 30) || !r.get(vt) || !r.value(vt, 0)) {
            code = VKQ_ERR_INVALID_ARGUMENT;
            why = "truncated or malformed metadata";
        }
    }
    for (uint64_t i = 0; code == VKQ_OK && i < n_tensors; i++) {
        GgufTensor t{};
        if (!r.str(&t.name, uint64_t(1) << 16) || !r.get(t.n_dims) || t.n_dims < 1 || t.n_dims > 4) {
            code = VKQ_ERR_INVALID_ARGUMENT;
            why = "malformed tensor info";
            break;
        }
        for (uint32_t d = 0; d < t.n_dims; d++) {
            uint64_t v = 0;
            r.get(v);
            t.dims[d] = (int64_t)v;
        }
        r.get(t.type);
        r.get(t.offset);
        if (!r.ok) {
            code = VKQ_ERR_INVALID_ARGUMENT;
            why = "truncated tensor info";
            break;
        }
        int64_t e = 1;
        bool big = false;
        for (uint32_t d = 0; d < t.n_dims; d++) {
            if (t.dims[d] < 0 || (t.dims[d] > 0 && e > (int64_t(1) << 50) / t.dims[d])) big = true;
            else e *= t.dims[d];
        }
        t.bytes = big ? -1 : ggml_bytes(t.type, e);
        g->tensors.push_back(std::move(t));
    }
    if (code == VKQ_OK) {
        g->data_offset = ((uint64_t)r.pos + 31) & ~uint64_t(31);
        for (const GgufTensor &t : g->tensors) {
            if (t.bytes >= 0 && (t.offset > g->size || g->data_offset + t.offset + (uint64_t)t.bytes > g->size)) {
                code = VKQ_ERR_INVALID_ARGUMENT;
                why = "a tensor's data lies past the end of the file";
                break;
            }
        }
    }
    if (code != VKQ_OK) {
        munmap(const_cast<uint8_t *>(g->map), g->size);
        close(fd);
        delete g;
        return fail(code, why);
    }
    *out = g;
    return VKQ_OK;
}

int vkq_gguf_close(vkq_gguf *g) {
    set_error("%s", "");
    if (!g) return VKQ_OK;
    munmap(const_cast<uint8_t *>(g->map), g->size);
    close(g->fd);
    delete g;
    return VKQ_OK;
}

int64_t vkq_gguf_tensor_count(const vkq_gguf *g) { return g ? (int64_t)g->tensors.size() : -1; }

int vkq_gguf_find(const vkq_gguf *g, const char *name, int64_t *index) {
    set_error("%s", "");
    if (!g || !name || !index) return fail(VKQ_ERR_INVALID_ARGUMENT, "null argument");
    for (size_t i = 0; i < g->tensors.size(); i++)
        if (g->tensors[i].name == name) {
            *index = (int64_t)i;
            return VKQ_OK;
        }
    set_error("tensor %s not found in GGUF file", name);
    return VKQ_ERR_INVALID_ARGUMENT;
}

int vkq_gguf_tensor_info(const vkq_gguf *g, int64_t index, const char **name, int *ggml_type, int *n_dims,
                         int64_t dims[4], int64_t *data_offset, int64_t *bytes) {
    set_error("%s", "");
    if (!g || index < 0 || index >= (int64_t)g->tensors.size()) return fail(VKQ_ERR_INVALID_ARGUMENT, "bad index");
    const GgufTensor &t = g->tensors[(size_t)index];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = (int)t.type;
    if (n_dims) *n_dims = (int)t.n_dims;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = d < (int)t.n_dims ? t.dims[d] : 1;
    if (data_offset) *data_offset = (int64_t)(g->data_offset + t.offset);
    if (bytes) *bytes = t.bytes;
    return VKQ_OK;
}

int vkq_gguf_load_tensor(vkq_gguf *g, int64_t index, int device, void *dst, int64_t dst_bytes, void *stream) {
    set_error("%s", "");
    if (!g || !dst || index < 0 || index >= (int64_t)g->tensors.size())
        return fail(VKQ_ERR_INVALID_ARGUMENT, "bad argument to vkq_gguf_load_tensor");
    const GgufTensor &t = g->tensors[(size_t)index];
    if (t.bytes < 0) return fail(VKQ_ERR_UNSUPPORTED, "tensor type without a size rule");
    if (dst_bytes < t.bytes) return fail(VKQ_ERR_INVALID_ARGUMENT, "destination smaller than the tensor");
    const uint8_t *src = g->map + g->data_offset + t.offset;
    return upload(device, dst, t.bytes, (cudaStream_t)stream,
                  [&](uint8_t *stage, int64_t off, size_t n) { memcpy(stage, src + off, n); });
}

int vkq_gguf_load_shard(vkq_gguf *g, int64_t index, int64_t col_lo, int64_t col_hi, int device, void *dst,
                        int64_t dst_bytes, void *stream) {
    set_error("%s", "");
    if (!g || !dst || index < 0 || index >= (int64_t)g->tensors.size())
        return fail(VKQ_ERR_INVALID_ARGUMENT, "bad argument to vkq_gguf_load_shard");
    const GgufTensor &t = g->tensors[(size_t)index];
    const int bb = t.type == 12 ? 144 : t.type == 13 ? 176 : t.type == 14 ? 210 : 0;
    if (bb == 0 || t.n_dims != 2) return fail(VKQ_ERR_UNSUPPORTED, "shards are for 2D k-quant weights");
    const int64_t K = t.dims[0], N = t.dims[1];
    int64_t rb = 0, need = 0;
    int st = vkq_shard_bytes((int)t.type, K, N, col_lo, col_hi, &rb, &need);
    if (st) return st;
    if (dst_bytes < need) return fail(VKQ_ERR_INVALID_ARGUMENT, "destination smaller than the shard");
    const uint8_t *src = g->map + g->data_offset + t.offset;
    const int64_t width = col_hi - col_lo, row_bytes = rb * bb;
    // the shard row by row, as vkq_shard_weight lays it out
    return upload(device, dst, need, (cudaStream_t)stream, [&](uint8_t *stage, int64_t off, size_t n) {
        for (int64_t o = off; o < off + (int64_t)n;) {
            const int64_t k = o / row_bytes, in_row = o % row_bytes;
            const int64_t v0 = k * N + col_lo;
            const int64_t have = (((v0 & 255) + width - 1) / 256 + 1) * bb;  // bytes of real blocks
            const int64_t take = std::min<int64_t>(row_bytes - in_row, off + (int64_t)n - o);
            const int64_t real = std::max<int64_t>(0, std::min<int64_t>(have - in_row, take));
            if (real > 0) memcpy(stage + (o - off), src + (v0 >> 8) * bb + in_row, (size_t)real);
            if (take > real) memset(stage + (o - off) + real, 0, (size_t)(take - real));
            o += take;
        }
    });
}

}  // extern "C"
