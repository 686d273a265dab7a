/*
 * vkq.h -- C ABI of the B200 (sm_100a) k-quant dequantize-and-matmul path.
 *
 * Drop-in boundary for xupit3r/vibrant's GPU matmul path.  Every entry point
 * is extern "C", takes plain pointers and sizes, returns an int status
 * (0 = VKQ_OK) and never throws.  On failure vkq_last_error() gives a
 * thread-local message.  Device pointers are owned by the caller (vibrant's
 * gpu.Buffer, internal/gpu/buffer.go:6-29; the raw pointer comes from
 * Buffer.Ptr(), internal/gpu/cuda.go:250-254).
 *
 * Conventions shared by all entry points
 *  - device: CUDA ordinal made current on the calling thread before any CUDA
 *    call (Go may run a cgo call on any OS thread); pass -1 to keep the
 *    thread's current device.
 *  - stream: a cudaStream_t passed as void*; NULL is the legacy default
 *    stream, which is what vibrant's kernels use today
 *    (internal/tensor/ops_cuda.go:62,71).  Calls are asynchronous: nothing
 *    synchronizes the host, so the caller keeps its Device.Sync()
 *    (ops_cuda.go:81) where it needs one.
 *  - qtype: GGML type code of the weight, as in internal/gguf/metadata.go:21-23.
 *  - Weight orientation follows the reference: a quantized weight is
 *    logically row-major [K, N] = [in, out] (internal/gguf/loader.go:24-27);
 *    W[k][n] is dequantized value k*N + n of the byte stream, and the stream
 *    holds ceil(K*N/256) super-blocks (calculateTensorSize,
 *    internal/gguf/metadata.go:170-204).  x is float32 [M, K] row-major and
 *    y is float32 [M, N] row-major.
 *  - There is no CPU fallback: when the GPU path cannot run, the call fails.
 */
#ifndef VKQ_H
#define VKQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VKQ_ABI_VERSION 5

#if defined(__GNUC__)
#define VKQ_API __attribute__((visibility("default")))
#else
#define VKQ_API
#endif

/* GGML type codes, internal/gguf/metadata.go:21-23. */
enum vkq_qtype { VKQ_Q4_K = 12, VKQ_Q5_K = 13, VKQ_Q6_K = 14 };

enum vkq_status {
    VKQ_OK = 0,
    VKQ_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, short buffer */
    VKQ_ERR_UNSUPPORTED = 2,      /* unknown qtype, or a shape/device no kernel serves */
    VKQ_ERR_MISALIGNED = 3,       /* a pointer lacks the alignment the kernel needs */
    VKQ_ERR_WORKSPACE = 4,        /* workspace missing or smaller than required */
    VKQ_ERR_CUDA = 5,             /* CUDA runtime error (message in vkq_last_error) */
    VKQ_ERR_DEVICE_TIMEOUT = 6,   /* a bounded device-side wait gave up */
    VKQ_ERR_NCCL = 7,             /* collective failure in the sharded path */
    VKQ_ERR_PEER = 8              /* a peer rank is out of step, or its channel failed earlier */
};

/* Version of this ABI (VKQ_ABI_VERSION of the built library). */
VKQ_API int vkq_abi_version(void);
/* Static text for a status code. */
VKQ_API const char *vkq_status_string(int status);
/* Message of the last failing call made on this thread ("" if none). */
VKQ_API const char *vkq_last_error(void);

/* Bytes of one super-block: 144 / 176 / 210 (Q4_K_BLOCK_SIZE,
 * quant_q4k.go:9-11; Q5_K_BLOCK_SIZE, quant_q5k.go:9-13; Q6_K_BLOCK_SIZE,
 * quant_q6k.go:9-11).  0 for an unknown type. */
VKQ_API int64_t vkq_block_bytes(int qtype);

/* Byte size of a [K, N] weight: ceil(K*N/256) blocks.  Replaces
 * calculateTensorSize for the k-quant types (internal/gguf/metadata.go:170-204). */
VKQ_API int vkq_weight_bytes(int qtype, int64_t K, int64_t N, int64_t *bytes);

/* Dequantize nblocks super-blocks to float32 (nblocks*256 values), bit-exact
 * with the reference Go decoders: every non-NaN result has the same bits as
 * DequantizeQ4_K / Q5_K / Q6_K (quant_q4k.go:37-79, quant_q5k.go:39-88,
 * quant_q6k.go:39-80) including float16ToFloat32's choices (tensor.go:629-676);
 * NaN results are NaN.  Replaces the CPU expansion done before upload by
 * dequantizeForGPU (internal/tensor/tensor_cuda_api.go:39-53).
 * w: device, any alignment; out: device, 4-byte aligned. */
VKQ_API int vkq_dequantize_f32(int device, int qtype, const void *w, int64_t nblocks, float *out,
                       void *stream);

/* Fused dequantize + transpose: quantized [K, N] -> float32 [N, K], bit-exact
 * with DequantTransposeQ4K / Q5K / Q6K (internal/tensor/dequant_transpose.go:15-157)
 * as used by GetOrDequantTranspose (internal/tensor/tensor.go:535-588),
 * including its handling of a trailing partial block (left zero). */
VKQ_API int vkq_dequant_transpose_f32(int device, int qtype, const void *w, int64_t K, int64_t N,
                              float *out, void *stream);

/* Workspace needed by vkq_matmul / vkq_gemv / vkq_gemm for this problem on
 * this device.  The workspace is caller-owned device memory, at least
 * 256-byte aligned, zero-filled before its first use; every call leaves it
 * ready for the next one.  Calls that may run concurrently need separate
 * workspaces. */
VKQ_API int vkq_matmul_workspace_bytes(int device, int qtype, int64_t M, int64_t K, int64_t N,
                               size_t *bytes);

/* y[M,N] = x[M,K] . W[K,N] with W quantized (qtype), float32 in and out.
 * Dispatch: M <= 8 runs vkq_gemv (fp32 accumulate, max relative error 1e-5
 * against the reference's float32 CPU MatMul); larger M runs vkq_gemm (bf16
 * tensor cores, 2e-2) when N % 32 == 0 and K % 8 == 0, else vkq_gemv over
 * 8-row chunks.  w_bytes is the size of the weight buffer (at least
 * vkq_weight_bytes).  w must be 16-byte aligned.
 * Replaces matmul_f32_single_row_launch (internal/gpu/cuda/launch.cu:37-48,
 * M == 1) and matmul_f32_launch (launch.cu:25-35, M > 1) as called by
 * matmulGPU (internal/tensor/ops_cuda.go:16-101), with the weight kept
 * quantized on the device instead of expanded to float32. */
VKQ_API int vkq_matmul(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
               const float *x, int64_t M, float *y, void *workspace, size_t workspace_bytes,
               void *stream);

/* vkq_matmul for a caller whose activations live in host memory (the
 * reference's MatMul on a CPU activation and a device weight: the upload of
 * x, the product, the download of y, as Tensor.ToDevice / EnsureCPUData do
 * around matmulGPU, internal/tensor/tensor_cuda_api.go and
 * internal/tensor/tensor.go:482-524): moves x_host [M, K] into the device
 * buffer x_dev, runs vkq_matmul and delivers y [M, N] to y_host, all
 * enqueued on `stream`.  Pinned host buffers (cudaHostAlloc, mapped into the
 * device's address space) up to 1 MiB are reached through the mapping: a
 * small kernel reads x, and for M <= 8 the GEMV stores y straight into
 * y_host (y_dev is then unused); other host memory, and larger buffers, are
 * copied with cudaMemcpyAsync (synchronously for pageable memory).  Same
 * arguments and errors as vkq_matmul otherwise. */
VKQ_API int vkq_matmul_host(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                            const float *x_host, int64_t M, float *y_host, float *x_dev, float *y_dev,
                            void *workspace, size_t workspace_bytes, void *stream);

/* The upstream GGUF orientation, behind an entry point of its own: a weight
 * stored [N rows][K] as GGUF files written by other engines hold a linear
 * layer ([out][in]: row n is the K/256 super-blocks of output n along K, so
 * W[n][k] = value n*K + k of the stream), where vibrant's loader reads value
 * k*N + n as W[k][n] (internal/gguf/loader.go:24-27) and every other entry
 * point of this library follows vibrant.  y[m][n] = sum_k x[m][k] * W[n][k],
 * fp32 accumulate within max relative error 1e-5 of sum_k |x w|; needs
 * K % 256 == 0 and x 16-byte aligned; any M (a warp per output row, four
 * rows of x per launch); no workspace. */
VKQ_API int vkq_matmul_upstream(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                                const float *x, int64_t M, float *y, void *stream);

/* The fp32-class GEMV path of vkq_matmul, for 1 <= M <= 8 (decode): the
 * Q4_K column-strip kernel (M == 1, N % 256 == 0), the tensor-core kernel
 * (M <= 4; dequantized quants and per-sub-block scaled x split into three
 * bf16 parts, fp32 accumulate) or the CUDA-core kernel; all within max
 * relative error 1e-5 of sum_k |x w|. */
VKQ_API int vkq_gemv(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
             const float *x, int64_t M, float *y, void *workspace, size_t workspace_bytes,
             void *stream);

/* The bf16 tensor-core (tcgen05/TMEM) GEMM path of vkq_matmul for any M >= 1:
 * bf16 operands, fp32 accumulate, max relative error 2e-2 of sum_k |x w|.
 * Needs N % 32 == 0, K % 8 == 0 and x 8-byte aligned; the workspace holds a
 * bf16 copy of x.  Replaces matmul_f32 (internal/gpu/cuda/kernels.cu:11-57)
 * on the prefill path of matmulGPU (internal/tensor/ops_cuda.go:64-73). */
VKQ_API int vkq_gemm(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                     const float *x, int64_t M, float *y, void *workspace, size_t workspace_bytes,
                     void *stream);

/* Selects the kernel that serves vkq_gemv / vkq_matmul for 1 <= M <= 8,
 * process-wide: 0 automatic (the default), 1 the CUDA-core kernel, 2 the
 * tensor-core kernel (M <= 4), 3 the Q4_K column-strip kernel (M <= 4,
 * N % 256 == 0); all in the 1e-5 tolerance class, and a kernel that does not
 * serve a shape leaves it to the automatic choice.  Returns
 * the previous choice, or -1 for an invalid one.  No counterpart in the
 * reference (it has one fp32 kernel, internal/gpu/cuda/kernels.cu:61-77);
 * for tests and measurements. */
VKQ_API int vkq_set_gemv_path(int path);

/* The fp32 GEMV of vkq_gemv without a workspace argument, for callers that
 * cannot allocate device memory: a host whose allocator owns every byte of
 * the device budget, a plugin whose memory plan is fixed before it runs, or a
 * caller that must avoid cudaMalloc's device-wide synchronisation.  No
 * counterpart in the reference.  The split-K scratch lives in a fixed 8 MiB
 * device array inside the library, which every GPU that loads the library
 * holds until the process exits; a problem needing more scratch is rejected
 * with VKQ_ERR_WORKSPACE.  The call allocates nothing.  Its first call on a
 * device looks the array up (cudaGetSymbolAddress) -- make that first call
 * before any stream capture.  All calls share the one array: calls that
 * overlap on the GPU (different streams, or different host threads on one
 * device) race and must be serialised by the caller.  1 <= M <= 8. */
VKQ_API int vkq_gemv_noalloc(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                             const float *x, int64_t M, float *y, void *stream);

/* The steps between the linear layers of a decode step (float32, device
 * buffers).  out = SiLU(gate) * up elementwise, SiLU(g) = g / (1 + exp(-g)):
 * replaces silu_f32 followed by mul_f32 (internal/gpu/cuda/kernels.cu:306-341)
 * as FeedForward.Forward applies them (internal/transformer/feedforward.go:92-94);
 * buffers 16-byte aligned.  vkq_rms_norm: out[r] = (x[r] / sqrt(mean(x[r]^2)
 * + eps)) * weight for each of `rows` rows of n values: replaces
 * rms_norm_f32 / rms_norm_batched_f32 (kernels.cu:209-288). */
VKQ_API int vkq_silu_mul(int device, const float *gate, const float *up, float *out, int64_t n, void *stream);
VKQ_API int vkq_rms_norm(int device, const float *x, const float *weight, float *out, int64_t rows, int64_t n,
                         float eps, void *stream);

/* Rotary position embedding over interleaved pairs: replaces rope_f32
 * (internal/gpu/cuda/kernels.cu:363-414, launched by LaunchRoPEKernel,
 * internal/gpu/cuda/library.go:397-415) with the arithmetic of
 * RoPE.ApplyRotation (internal/transformer/rope.go:49-124).  x and out are
 * [batch][heads][seq][head_dim] float32 (8-byte aligned, may be the same
 * buffer); cos_table and sin_table [max_seq][head_dim / 2] (as NewRoPE,
 * rope.go:19-43, builds them); positions[seq] (int32) the position of each
 * token.  Pair i of a token at position p: out[2i] = x[2i]*c - x[2i+1]*s,
 * out[2i+1] = x[2i]*s + x[2i+1]*c with c, s at table entry p*head_dim/2 + i,
 * each product and sum rounded on its own: bit-identical to the reference's
 * float32 results.  A position outside [0, max_seq) leaves its pairs
 * unwritten; vkq_device_status then reports VKQ_ERR_INVALID_ARGUMENT. */
VKQ_API int vkq_rope_f32(int device, const float *x, float *out, const float *cos_table, const float *sin_table,
                         const int32_t *positions, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                         int64_t max_seq, void *stream);

/* Decode attention, one query token per sequence against its KV cache:
 * replaces computeAttention (internal/transformer/attention.go:316-363) for
 * the reference's decode step, where the new token's K and V are appended to
 * the cache (:147-162), grouped KV heads are shared (expandKVHeads, :280-314)
 * and no mask applies (applyCausalMask :429-460, one query row):
 *   o[b][h] = softmax(q[b][h] . K[b][h / g]^T * float32(1/sqrt(D))) . V[b][h / g]
 * with g = heads / kv_heads.  q and out are [batch][heads][D]; the caches are
 * [batch][kv_heads][cache_len][D] with rows 0 .. len-1 valid (cache_len is
 * the allocated length, >= len).  D = 64 or 128; len <= 409600.  fp32, within
 * 1e-5 of sum_j p_j |v_j| of the reference's arithmetic.  Allocates nothing. */
VKQ_API int vkq_attention_decode_f32(int device, const float *q, const float *k_cache, const float *v_cache,
                                     float *out, int64_t batch, int64_t heads, int64_t kv_heads, int64_t len,
                                     int64_t cache_len, int64_t head_dim, void *stream);

/* The decode branch of Attention.Forward after its projections, in one
 * launch: replaces, for one new token per sequence, ApplyRotation on q and k
 * (internal/transformer/attention.go:141-143, rope.go:49-124), the cache
 * concatenation (attention.go:146-162, concatenateSeqDim) and
 * expandKVHeads + computeAttention (:164-172).  q [batch][heads][D], k_new
 * and v_new [batch][kv_heads][D] are the projections before RoPE;
 * positions[batch] (int32) the new token's position, cos_table and
 * sin_table [max_seq][D / 2] as for vkq_rope_f32.  q and k_new are rotated
 * with vkq_rope_f32's arithmetic (bit-identical), the rotated k_new and
 * v_new are stored at row len - 1 of k_cache and v_cache
 * ([batch][kv_heads][cache_len][D], rows 0 .. len-2 already valid), and out
 * [batch][heads][D] is vkq_attention_decode_f32 over rows 0 .. len-1, within
 * the same 1e-5 of sum_j p_j |v_j|.  Same limits as vkq_attention_decode_f32;
 * 4-byte aligned buffers; allocates nothing.  A position outside
 * [0, max_seq) leaves that sequence's out and cache rows unwritten, and
 * vkq_device_status then reports VKQ_ERR_INVALID_ARGUMENT. */
VKQ_API int vkq_attention_rope_decode_f32(int device, const float *q, const float *k_new, const float *v_new,
                                          const float *cos_table, const float *sin_table, const int32_t *positions,
                                          float *k_cache, float *v_cache, float *out, int64_t batch, int64_t heads,
                                          int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim,
                                          int64_t max_seq, void *stream);

/* The fused linears of a decode step: one launch over `nweights` Q4_K
 * weights [K, N_i] (N_i % 256 == 0, 16-byte aligned) that share the input
 * x [M, K] (4-byte aligned):
 *   h = x, or with norm_w != NULL h = x / sqrt(mean(x^2) + eps) * norm_w
 *       row by row (the RMSNorm prologue, M <= 3);
 *   VKQ_EPI_NONE:     y[i] = h . W_i for every weight (1..4: q, k and v);
 *   VKQ_EPI_SILU_MUL: y[0] = SiLU(h . W_0) * (h . W_1) (two weights of one
 *                     width: gate and up).
 * w, w_bytes, N and y are host arrays of nweights entries; y[i] is a device
 * buffer [M, N_i] (y[0] alone for VKQ_EPI_SILU_MUL).  fp32 accumulate, the
 * GEMV's 1e-5 tolerance class; 1 <= M <= 4; no workspace.  Replaces, for one
 * token, the RMSNorm of TransformerLayer.Forward (internal/transformer/
 * layer.go:111, rms_norm_f32 of internal/gpu/cuda/kernels.cu:209-288) with the
 * MatMul calls that follow it: q, k, v in Attention.Forward
 * (internal/transformer/attention.go:120,124,128) and gate, up, SiLU, Mul in
 * FeedForward.Forward (internal/transformer/feedforward.go:87-95).  Other
 * qtypes give VKQ_ERR_UNSUPPORTED. */
#define VKQ_EPI_NONE 0
#define VKQ_EPI_SILU_MUL 1
VKQ_API int vkq_linear_fused(int device, int qtype, int nweights, const void *const *w, const int64_t *w_bytes,
                             int64_t K, const int64_t *N, const float *x, int64_t M, const float *norm_w, float eps,
                             int epilogue, float *const *y, void *stream);

/* ---- Row-sharded matmul across the GPUs of one node ----
 * The reference runs on a single device (internal/gpu/cuda/cuda.go:33-46);
 * these entry points implement the multi-GPU layout of the same MatMul.  The
 * output columns of a [K, N] weight are split over `world` ranks (at most 8)
 * in equal ranges rounded up to multiples of 32 (vkq_shard_columns); each
 * rank holds only its row-block shard of the weight (vkq_shard_weight) and
 * the result is all-gathered inside the GEMV kernel through peer memory over
 * NVLink (plain stores into every rank's output, no collective library).
 *
 * Channel protocol, shared by both forms below: every rank makes the same
 * sequence of calls on a channel, each rank on one stream.  A call stores
 * into another rank's output only after that rank has started the same call
 * (so it has finished with the previous contents); when it completes on the
 * stream every rank's columns are in this rank's output.  Every wait is
 * bounded (VKQ_PEER_WAIT_MS in the environment, default 2000): a rank that
 * never arrives makes the others give up with VKQ_ERR_DEVICE_TIMEOUT, a rank
 * whose call number differs makes them give up at once with VKQ_ERR_PEER
 * (both read with vkq_device_status).  A failed call stores nothing into
 * other ranks' outputs, and every later call on that channel fails at once
 * (VKQ_ERR_PEER, no waits) until the channel is reset. */

/* Output columns [*lo, *hi) of rank `rank`; N a multiple of 32. */
VKQ_API int vkq_shard_columns(int64_t N, int world, int rank, int64_t *lo, int64_t *hi);
/* Size of the row-block shard of columns [col_lo, col_hi) of a [K, N] weight:
 * K rows of *row_blocks super-block slots (*bytes = K * row_blocks * block
 * bytes).  Host-only. */
VKQ_API int vkq_shard_bytes(int qtype, int64_t K, int64_t N, int64_t col_lo, int64_t col_hi, int64_t *row_blocks,
                            int64_t *bytes);
/* Builds the row-block shard of columns [col_lo, col_hi) from the full raw
 * weight (HOST memory, e.g. the mmapped GGUF bytes of
 * internal/gguf/loader.go:11-73): row k holds the super-blocks covering
 * values k*N + col_lo .. k*N + col_hi - 1, copied byte for byte (blocks that
 * straddle rows or shards are duplicated), zero-padded to row_blocks slots.
 * The caller uploads the result (raw blocks, no float32 expansion). */
VKQ_API int vkq_shard_weight(int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N, int64_t col_lo,
                             int64_t col_hi, void *out, int64_t out_bytes);

/* In-process form: one process drives every GPU (vibrant's host is one Go
 * process).  vkq_comm_init enables peer access between the listed devices
 * and allocates each device's channel flags; one communicator is one channel. */
typedef struct vkq_comm vkq_comm;
VKQ_API int vkq_comm_init(int world, const int *devices, vkq_comm **comm);
/* Zeroes every device's channel (after synchronising them): the recovery
 * from a failed call; no call may be in flight. */
VKQ_API int vkq_comm_reset(vkq_comm *comm);
VKQ_API int vkq_comm_destroy(vkq_comm *comm);
VKQ_API int vkq_comm_size(const vkq_comm *comm);
/* y[r] = x[r] . W on every device r, computed as rank r's columns of the
 * shards w_shards[r] (each on device r, built for the columns of
 * vkq_shard_columns(N, world, r)) and all-gathered into every y[r] (device r,
 * float32 [M, N], 16-byte aligned).  Arrays are HOST arrays of `world`
 * entries; workspaces[r] holds vkq_matmul_workspace_bytes(M, K, hi - lo) on
 * device r; streams[r] is a stream of device r.  Launches on every device
 * and returns; 1 <= M <= 8.  The first call with a larger M * N grows the
 * communicator's channel buffers (it synchronizes every device and
 * allocates: make it before any stream capture). */
VKQ_API int vkq_gemv_sharded(vkq_comm *comm, int qtype, const void *const *w_shards, const int64_t *w_bytes,
                             int64_t K, int64_t N, const float *const *x, int64_t M, float *const *y,
                             void *const *workspaces, const size_t *workspace_bytes, void *const *streams);

/* Multi-process form (one process per GPU): device buffers shared between
 * processes.  vkq_ipc_alloc allocates `bytes` of zero-filled device memory and
 * returns a 64-byte handle another process passes to vkq_ipc_open to map the
 * same buffer (peer access is enabled on the mapping).  vkq_ipc_close unmaps,
 * vkq_ipc_free releases the owner's buffer (after every mapping of it has
 * been closed). */
VKQ_API int vkq_ipc_alloc(int device, size_t bytes, void **ptr, unsigned char handle[64]);
VKQ_API int vkq_ipc_open(int device, const unsigned char handle[64], void **ptr);
VKQ_API int vkq_ipc_close(int device, void *ptr);
VKQ_API int vkq_ipc_free(int device, void *ptr);

/* This rank's part of a sharded y[M, N] = x[M, K] . W[K, N]: columns
 * [col_lo, col_hi) (multiples of 32) computed with the fp32 GEMV of vkq_gemv
 * from the rank's row-block shard w (vkq_shard_weight for the same columns,
 * w_bytes >= vkq_shard_bytes) and stored into every rank's output y[M][N].
 * peer_out and peer_flags are HOST arrays of `world` device pointers usable
 * on this device: every rank's output buffer and channel buffer (own entry
 * included); a channel buffer holds vkq_gather_channel_bytes(M, N) bytes or
 * more (flag words, then the flagged-word slots through which the Q4_K
 * column-strip kernel exchanges values) and starts at zero; sync points to
 * this rank's 4 uint32 channel words (zero at first; zero them on every rank,
 * with the channel buffers, to reset a failed channel).
 * 1 <= M <= 8; the workspace is vkq_matmul_workspace_bytes(M, K, col_hi - col_lo). */
VKQ_API int vkq_gemv_allgather(int device, int qtype, const void *w, int64_t w_bytes, int64_t K, int64_t N,
                               int64_t col_lo, int64_t col_hi, const float *x, int64_t M, void *const *peer_out,
                               void *const *peer_flags, void *sync, int world, int rank, void *workspace,
                               size_t workspace_bytes, void *stream);
/* Bytes of a channel buffer for outputs of up to m_max rows of N columns:
 * 256 bytes of flag words, then two 8-byte slots per output element. */
VKQ_API size_t vkq_gather_channel_bytes(int64_t m_max, int64_t N);

/* vkq_linear_fused on a row-sharded model (Q4_K, N % 256 == 0): w[0] is this
 * rank's row-block shard of columns [col_lo, col_hi) of a [K, N] weight
 * (vkq_shard_columns), and its output is all-gathered like
 * vkq_gemv_allgather's into every rank's peer_out[rank] [M][N];
 *   VKQ_EPI_NONE:     w[1..] are whole weights [K, N_local[i]] computed on
 *                     every rank into y_local[i] (k and v beside a sharded q);
 *   VKQ_EPI_SILU_MUL: nweights == 2, w[1] the shard of the same columns of
 *                     the up weight; the gathered output is SiLU(gate) * up.
 * norm_w / eps as in vkq_linear_fused; channel buffers of
 * vkq_gather_channel_bytes(M, N); 1 <= M <= 4; every rank makes the same
 * sequence of calls on a channel (vkq_gemv_allgather's protocol). */
VKQ_API int vkq_linear_fused_allgather(int device, int qtype, int nweights, const void *const *w,
                                       const int64_t *w_bytes, int64_t K, int64_t N, int64_t col_lo, int64_t col_hi,
                                       const int64_t *N_local, const float *x, int64_t M, const float *norm_w,
                                       float eps, int epilogue, float *const *y_local, void *const *peer_out,
                                       void *const *peer_flags, void *sync, int world, int rank, void *stream);

/* ---- GGUF weights to the device, still quantized ----
 * Replaces the GPU upload route of the reference: ParseGGUF
 * (internal/gguf/parser.go:15-64) + LoadTensor (internal/gguf/loader.go:11-73)
 * + Tensor.ToDevice, which expands k-quant tensors to float32 on the host
 * (internal/tensor/tensor_cuda_api.go:16-53).  vkq_gguf_open memory-maps the
 * file and parses its header, metadata (skipped) and tensor infos, with
 * bounds checks; the tensor data section starts at the end of the infos
 * rounded up to 32 bytes (parser.go:53-60).  Host-only except the loads. */
typedef struct vkq_gguf vkq_gguf;
VKQ_API int vkq_gguf_open(const char *path, vkq_gguf **gguf);
VKQ_API int vkq_gguf_close(vkq_gguf *gguf);
VKQ_API int64_t vkq_gguf_tensor_count(const vkq_gguf *gguf);
VKQ_API int vkq_gguf_find(const vkq_gguf *gguf, const char *name, int64_t *index);
/* Name (valid while the file is open), GGML type, dims in file order (unused
 * entries 1; vibrant's [K, N] = [dims[0], dims[1]], loader.go:24-27), the
 * absolute file offset of the data and its byte size (-1 for a type without
 * a size rule). */
VKQ_API int vkq_gguf_tensor_info(const vkq_gguf *gguf, int64_t index, const char **name, int *ggml_type,
                                 int *n_dims, int64_t dims[4], int64_t *data_offset, int64_t *bytes);
/* Byte size of a tensor: calculateTensorSize (internal/gguf/metadata.go:170-204),
 * which covers Q4_K where LoadTensor's expectedSize (loader.go:35-48) does not. */
VKQ_API int vkq_gguf_tensor_bytes(int ggml_type, int n_dims, const int64_t *dims, int64_t *bytes);
/* Copies a tensor's raw bytes to device memory `dst` (dst_bytes >= its size)
 * through pinned staging buffers on `stream`; returns when the copy is done. */
VKQ_API int vkq_gguf_load_tensor(vkq_gguf *gguf, int64_t index, int device, void *dst, int64_t dst_bytes,
                                 void *stream);
/* Copies the row-block shard of columns [col_lo, col_hi) of a 2D k-quant
 * weight (the layout of vkq_shard_weight) to device memory, gathering it from
 * the mapping: each rank reads and uploads only its shard. */
VKQ_API int vkq_gguf_load_shard(vkq_gguf *gguf, int64_t index, int64_t col_lo, int64_t col_hi, int device,
                                void *dst, int64_t dst_bytes, void *stream);

/* Reads and clears the device-side status word of this library on a device
 * (set when a bounded wait inside a kernel gave up, or a peer was out of
 * step).  Synchronizes with the device.  *code receives VKQ_OK,
 * VKQ_ERR_DEVICE_TIMEOUT or VKQ_ERR_PEER. */
VKQ_API int vkq_device_status(int device, int *code);

#ifdef __cplusplus
}
#endif
#endif /* VKQ_H */
