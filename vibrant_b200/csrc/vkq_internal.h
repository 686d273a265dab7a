// vkq_internal.h -- host-side declarations shared by the translation units of
// libvkq.so (not part of the public ABI; see include/vkq.h for that).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace vkq {

int device_sm_count(int device);
// Raises a kernel's dynamic shared-memory limit on the current device to at
// least `smem` bytes (with `carveout`, also its preferred carveout to the
// maximum); the driver is asked only when a launch needs more than the last
// limit set for that kernel and device.
cudaError_t kernel_smem(const void *fn, size_t smem, bool carveout);

cudaError_t dequantize_f32(int qtype, const void *w, int64_t nblocks, float *out, cudaStream_t s, int device);
cudaError_t dequant_transpose_f32(int qtype, const void *w, int64_t K, int64_t N, float *out, cudaStream_t s,
                                  int device);

// Layout of a caller's matmul workspace: the first kWorkspaceCounterHead bytes
// hold the GEMV's split-K tile counters, which every call leaves at zero (the
// GEMV fast path serves at most kWorkspaceCounterHead / 4 tiles); every other
// kernel keeps its scratch after them, so any call may follow any other on
// one workspace.
constexpr size_t kWorkspaceCounterHead = 64 * 1024;

// fp32 CUDA-core GEMV (1 <= M <= 8).
struct GemvShape {
    int qtype;
    int64_t K, N, M;
};
// Workspace bytes the GEMV plan needs (0 when it needs none).
size_t gemv_workspace_bytes(const GemvShape &s, int device);
// Row-sharded all-gather through peer memory: the launch computes columns
// [n_base, n_base + N) of a [K, ld] weight from this rank's row-block shard
// (row stride rs values) and stores column n_base + n of the result into every
// rank's output [M][y_ld] at column col_off + n; see vkq_gemv_allgather.
constexpr int kMaxRanks = 8;
struct GatherArgs {
    float *peer_y[kMaxRanks];         // every rank's output buffer (device addresses usable here)
    unsigned *peer_flags[kMaxRanks];  // every rank's flag array (2 * world words each)
    unsigned *sync;                   // this rank's channel words (4 uint32)
    int world, rank;
    int64_t y_ld, col_off;
    int64_t rs, ld, n_base;
    uint64_t wait_ns;
    // output elements (m, n) the channel buffers' flagged-word slots hold
    // (0: none; the column-strip all-gather needs M * y_ld)
    int64_t slot_elems;
};
// Bytes of a channel buffer (flag words, then two 8-byte slots per output
// element of an [m_max][N] output).
inline size_t gather_channel_bytes(int64_t m_max, int64_t N) { return 256 + (size_t)m_max * (size_t)N * 16; }
// Budget of each wait on peer ranks (ns): VKQ_PEER_WAIT_MS, default 2000 ms.
uint64_t peer_wait_ns();
// Block slots per row of the row-block shard of columns [lo, hi).
int64_t shard_row_blocks(int64_t K, int64_t N, int64_t lo, int64_t hi);
// Returns a vkq_status code; on failure writes a message with set_error.
int gemv_launch(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y, void *ws,
                size_t ws_bytes, cudaStream_t stream, int device, const GatherArgs *gather = nullptr);
// Same GEMV with its scratch in a fixed device array of the library (no
// workspace argument, nothing allocated); see vkq_gemv_noalloc.
int gemv_launch_noalloc(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y,
                        cudaStream_t stream, int device);
int gemv_read_status();
// Selects the kernel of plain GEMVs: 0 automatic, 1 CUDA cores (gemv.cu), 2
// tensor cores (gemv_tc.cu), 3 column strips (gemv_strip.cu); returns the
// previous choice.
int set_gemv_path(int path);

// Tensor-core GEMV (gemv_tc.cu), fp32-class results, 1 <= M <= 4, N % 32 == 0.
// Row k of the weight starts at value position k*rs + ((k*ld + n_base) & 255)
// of its super-block stream: {N, 0, 0} for a plain [K, N] weight, {rb*256, N,
// lo} for a row-block shard of columns [lo, ...).
struct TcLayout {
    int64_t rs, ld, n_base;
};
bool gemv_tc_supported(const GemvShape &s);
// supported, and its pipeline stages fit in shared memory for this layout
bool gemv_tc_fits(const GemvShape &s, const TcLayout &L, int device);
size_t gemv_tc_workspace_bytes(const GemvShape &s, const TcLayout &L, int device);
int gemv_tc_launch(const GemvShape &s, const TcLayout &L, const void *w, int64_t w_bytes, const float *x, float *y,
                   int64_t y_ld, void *ws, size_t ws_bytes, cudaStream_t stream, int device);
int gemv_tc_read_status();

// Q4_K column-strip GEMV (gemv_strip.cu), 1 <= M <= 4, for stored rows that
// start on a super-block boundary: row k of the weight is rs / 256 blocks,
// and column n of the launch is value c0 + n of its stored row ({N, 0} for
// a plain [K, N] weight with N % 256 == 0; {rb*256, lo & 255} for the
// row-block shard of columns [lo, ...) of such a weight).  Needs no workspace.
struct StripLayout {
    int64_t rs, c0;
};
bool gemv_strip_supported(const GemvShape &s);
bool gemv_strip_fits(const GemvShape &s, const StripLayout &L, int device);
int gemv_strip_launch(const GemvShape &s, const StripLayout &L, const void *w, int64_t w_bytes, const float *x,
                      float *y, int64_t y_ld, int64_t col_off, cudaStream_t stream, int device);
// One launch over several Q4_K weights [K, N_i] that share x [M, K]: weight
// i (layout {rs, c0} as above) writes y_i[m][col_off + n]; with silu two
// weights of one width (gate, up) write SiLU(gate) * up into y_0; with
// norm_w the input is RMSNorm(x) * norm_w (row-wise, eps), M <= 3.
constexpr int kMaxStripSegs = 4;
struct StripSeg {
    const void *w;
    int64_t w_bytes, N, rs, c0;
    float *y;
    int64_t y_ld, col_off;
};
int gemv_strip_multi(int M, int64_t K, const StripSeg *segs, int nseg, bool silu, const float *x,
                     const float *norm_w, float eps, cudaStream_t stream, int device,
                     const GatherArgs *gather = nullptr);
// The row-sharded all-gather of one Q4_K weight through the column-strip
// kernel (a row-block shard of an N % 256 == 0 weight; see GatherArgs).
bool gemv_strip_gather_fits(const GemvShape &s, const GatherArgs &g, int device);
int gemv_strip_gather(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, const GatherArgs &g,
                      cudaStream_t stream, int device);
int gemv_strip_read_status();  // reads and clears the column-strip kernel's device status word

// fp32 GEMV for weights in the upstream GGUF orientation (gemv_rows.cu):
// y[m][n] = sum_k x[m][k] * W[n][k], W[n][k] = value n*K + k; K % 256 == 0,
// x 16-byte aligned, any M (four rows of x per launch).
cudaError_t gemv_rows_launch(int qtype, const void *w, int64_t K, int64_t N, const float *x, int64_t M, float *y,
                             cudaStream_t s, int device);

// bf16 tensor-core GEMM (tcgen05), any M; needs N % 32 == 0 and K % 8 == 0.
size_t gemm_workspace_bytes(const GemvShape &s, int device);
int gemm_launch(const GemvShape &s, const void *w, int64_t w_bytes, const float *x, float *y, void *ws,
                size_t ws_bytes, cudaStream_t stream, int device);
int gemm_read_status();  // reads and clears this TU's device status word (synchronous)

// SiLU(gate) * up and row-wise RMSNorm (elementwise.cu); 16-byte aligned buffers.
cudaError_t silu_mul(const float *gate, const float *up, float *out, int64_t n, cudaStream_t s, int device);
cudaError_t rms_norm(const float *x, const float *weight, float *out, int64_t rows, int64_t n, float eps,
                     cudaStream_t s);
// Decode attention (attention.cu): q [batch][heads][D], caches
// [batch][kv_heads][cache_len][D] with len valid rows, out [batch][heads][D];
// D = 64 or 128, len <= attention_max_len().
size_t attention_max_len();
cudaError_t attention_decode(const float *q, const float *kc, const float *vc, float *o, int64_t batch, int64_t heads,
                             int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim, cudaStream_t s);
// The fused decode step: q [batch][heads][D] and k_new, v_new
// [batch][kv_heads][D] before RoPE; rotates q and k_new at positions[b],
// stores the rotated k_new and v_new at row len - 1 of the caches and
// attends over rows 0 .. len-1.  A position outside [0, max_seq) skips its
// sequence and sets the status word attention_read_status() returns.
cudaError_t attention_decode_rope(const float *q, const float *k_new, const float *v_new, const float *cos_t,
                                  const float *sin_t, const int *positions, float *kc, float *vc, float *o,
                                  int64_t batch, int64_t heads, int64_t kv_heads, int64_t len, int64_t cache_len,
                                  int64_t head_dim, int64_t max_seq, cudaStream_t s);
int attention_read_status();  // reads and clears the attention kernels' status word
// Rotary position embedding over interleaved pairs (elementwise.cu): x and
// out [rows][head_dim] with rows = batch * heads * seq, seq the fastest;
// tables [max_seq][head_dim / 2]; 8-byte aligned x, out.
cudaError_t rope(const float *x, float *out, const float *cos_t, const float *sin_t, const int *positions,
                 int64_t rows, int64_t seq, int64_t head_dim, int64_t max_seq, cudaStream_t s, int device);
int elem_read_status();  // reads and clears the elementwise kernels' status word
// dst[0..n) = src[0..n) from pinned host memory through its device mapping
// (elementwise.cu), as a kernel that takes part in programmatic dependent launch.
cudaError_t stage_in(const float *src_mapped, float *dst, int64_t n, cudaStream_t s);

void set_error(const char *fmt, ...);
bool vkq_last_error_empty();

}  // namespace vkq
