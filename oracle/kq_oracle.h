/*
 * kq_oracle.h -- CPU oracle for the k-quant dequantize-and-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * Go arithmetic of xupit3r/vibrant's internal/tensor package.  It is used as
 * the checker by tests/, by __graft_entry__.smoke() and as the timed CPU
 * baseline by bench.py.  The product library (libvkq.so) never links or
 * calls it; there is no CPU fallback in the product path.
 *
 * Parity pins: the known-answer values of the reference's own tests
 * (internal/tensor/float16_test.go, quant_q6k_test.go,
 * quant_q6k_integration_test.go, quant_q5k_test.go, dequant_transpose_test.go,
 * tensor_cuda_test.go) are checked in tests/test_oracle_golden.py, and an
 * independent numpy restatement (tests/golden/make_golden.py) produced the
 * committed fixtures the oracle is compared with.  The decode-attention and
 * RoPE restatements (internal/transformer) are checked in
 * tests/test_oracle_attention.py against the values of
 * internal/transformer/transformer_test.go that it holds and against numpy
 * restatements; that test file's header says what it pins.
 *
 * Compiled with -ffp-contract=off: the reference is built for the default
 * GOAMD64 level, where the Go compiler does not fuse a*b+c into an FMA, so
 * every product and every sum is rounded to float32 separately.
 *
 * Orientation: a quantized weight is logically row-major [K, N] (in, out);
 * element W[k][n] is dequantized value number k*N + n of the byte stream, and
 * a 256-value super-block covers consecutive n of one row k
 * (internal/gguf/loader.go:24-27, internal/tensor/matmul_quant.go:87-89).
 */
#ifndef KQ_ORACLE_H
#define KQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Super-block geometry (internal/tensor/quant_q5k.go:9-13, quant_q4k.go:9-11,
 * quant_q6k.go:9-11). */
#define KO_QK_K 256
#define KO_Q4K_BYTES 144
#define KO_Q5K_BYTES 176
#define KO_Q6K_BYTES 210

/* Type codes shared with include/vkq.h (VKQ_Q4_K etc.). */
#define KO_Q4_K 12
#define KO_Q5_K 13
#define KO_Q6_K 14

int ko_block_bytes(int qtype);

/* internal/tensor/tensor.go:629-676 */
float ko_f16_to_f32(uint16_t h);
/* internal/tensor/tensor.go:606-627 (used by the reference's test quantizers) */
uint16_t ko_f32_to_f16(float f);

/* internal/tensor/quant_q5k.go:97-120 */
void ko_extract_scales_mins(const uint8_t scales[12], uint8_t sc[8], uint8_t m[8]);

/* One super-block -> 256 float32, internal/tensor/block_cache.go:222-248
 * (Q4_K), :82-122 (Q5_K), :158-186 (Q6_K); byte offsets from
 * parseQ4_KBlock quant_q4k.go:137-157, parseQ5_KBlock quant_q5k.go:229-252,
 * parseQ6_KBlock quant_q6k.go:134-156. */
void ko_dequant_block_q4k(const uint8_t *blk, float out[256]);
void ko_dequant_block_q5k(const uint8_t *blk, float out[256]);
void ko_dequant_block_q6k(const uint8_t *blk, float out[256]);

/* DequantizeQ*_KTensor (quant_q4k.go:161-211, quant_q5k.go:256-307,
 * quant_q6k.go:160-210): nblocks blocks -> nblocks*256 floats. */
int ko_dequantize(int qtype, const uint8_t *data, int64_t nblocks, float *out);

/* DequantTransposeQ4K/Q5K/Q6K (dequant_transpose.go:15-157): quantized
 * [M, N] -> float32 [N, M].  Only the first (M*N)/256 whole blocks are
 * expanded, as in the reference; the remaining tail stays zero. */
int ko_dequant_transpose(int qtype, const uint8_t *data, int64_t M, int64_t N, float *out);

/* simd_ops.go:60-78 -- eight strided partial sums, tail into s0, then
 * s0+s1+...+s7 left to right. */
float ko_vector_dot(const float *a, const float *b, int64_t n);
/* simd_ops.go:82-98 -- dst[i] += src[i]*scale */
void ko_vector_scale_add(float *dst, const float *src, int64_t n, float scale);

/* matmul_simd.go:150-201, transposed branch (:165-188): y[j] = dot(x, wt[j,:]),
 * columns split over nthreads workers like the goroutine fan-out. */
void ko_matmul_single_row_t(const float *x, const float *wt, int64_t K, int64_t N,
                            float *y, int nthreads);
/* matmul_simd.go:189-199, untransposed branch (the LM-head path): outer
 * product over k, skipping x[k] == 0, single threaded as in the reference. */
void ko_matmul_single_row_u(const float *x, const float *w, int64_t K, int64_t N,
                            float *y);
/* matmul_simd.go:13-69 with a pre-transposed B (ops < 1024). */
void ko_matmul_simd_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N, float *c);
/* matmul_simd.go:72-146, transposed branch (1024 <= ops < 1<<20). */
void ko_matmul_blocked_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N, float *c);
/* matmul_simd.go:204-276 with a pre-transposed B (ops >= 1<<20), rows split
 * over nthreads workers. */
void ko_matmul_parallel_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N,
                          float *c, int nthreads);

/* tensor.MatMul(a, b) for a float32 a [M,K] and a quantized b [K,N]
 * (matmul.go:46-99): b.GetOrDequantTranspose() (tensor.go:535-588) followed by
 * the size dispatch.  wt_scratch must hold N*K floats (the cached transposed
 * copy); it is filled here.  nthreads stands in for runtime.NumCPU(). */
int ko_matmul_quant(int qtype, const float *a, int64_t M, int64_t K,
                    const uint8_t *bq, int64_t N, float *c, float *wt_scratch, int nthreads);

/* The LM-head route (internal/transformer/model.go:389-403): tensor.Dequantize
 * of the whole weight (untransposed float32 [K,N]) and then MatMul, which for
 * an untransposed float32 B and M == 1 takes the outer-product branch and for
 * M > 1 the size dispatch on the untransposed B.  w_scratch holds
 * ceil(K*N/256)*256 floats. */
int ko_matmul_dequant_untransposed(int qtype, const float *a, int64_t M, int64_t K,
                                   const uint8_t *bq, int64_t N, float *c, float *w_scratch,
                                   int nthreads);

/* MatMulQ5K / MatMulQ6K (matmul_quant.go:30-191): c[i,j] = sequential
 * float32 sum over k of a[i,k] * deq(k*N + j); all three types. */
int ko_matmul_quant_sequential(int qtype, const float *a, int64_t M, int64_t K, const uint8_t *bq, int64_t N,
                               float *c);

/* The reference's test quantizers (QuantizeQ4_K quant_q4k.go:215-282,
 * QuantizeQ6_K quant_q6k.go:214-294), serialized as QuantizeQ4_KTensor /
 * QuantizeQ6_KTensor do (matmul_quant_helpers.go:62-145): n floats ->
 * ceil(n/256) blocks. */
int ko_quantize_q4k(const float *in, int64_t n, uint8_t *out);
int ko_quantize_q6k(const float *in, int64_t n, uint8_t *out);

/* ---- decode attention and RoPE (internal/transformer) ---------------------- */

/* NewRoPE (internal/transformer/rope.go:19-43): tables [max_seq][head_dim/2],
 * angle = pos * (1 / pow(freq_base, 2i / head_dim)) in double, then cos and
 * sin rounded to float.  (This libm may differ from Go's math package in the
 * last bit of a double, which float rounding almost always hides.) */
void ko_rope_tables(int64_t head_dim, double freq_base, int64_t max_seq, float *cos_t, float *sin_t);

/* RoPE.ApplyRotation, CPU branch (rope.go:49-124): x and out
 * [batch][heads][seq][head_dim] (out may be x), positions[seq].  Pair i of a
 * token at position p: out[2i] = x0*c - x1*s, out[2i+1] = x0*s + x1*c, every
 * product and sum rounded to float.  Returns -1 (out untouched) if a position
 * lies outside [0, max_seq). */
int ko_rope_apply(const float *x, float *out, const float *cos_t, const float *sin_t, const int32_t *positions,
                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t max_seq);

/* concatenateSeqDim (attention.go:529-569) into a preallocated cache: the
 * n_new rows of new_rows [batch][kv_heads][n_new][head_dim] become rows
 * row0 .. row0+n_new-1 of cache [batch][kv_heads][cache_len][head_dim].
 * Returns -1 if they do not fit. */
int ko_kv_append(float *cache, const float *new_rows, int64_t batch, int64_t kv_heads, int64_t cache_len,
                 int64_t row0, int64_t n_new, int64_t head_dim);

/* The decode branch of Attention.Forward after RoPE and the append
 * (attention.go:164-172): expandKVHeads (:280-314, query head h reads KV
 * head h / (heads / kv_heads)), then computeAttention (:316-363) for one
 * query row against rows 0 .. len-1 of the caches:
 *   scores = MatMul(q, Transpose(K)): Transpose copies (ops.go:445-468), so
 *     MatMul (matmul.go:46-99) takes matmulSIMDSingleRow's untransposed
 *     outer-product branch (matmul_simd.go:189-199);
 *   scaleScores (:413-427) by float(1 / sqrt(head_dim));
 *   applyCausalMask (:429-460) masks nothing for one query row;
 *   applySoftmax (:462-527): max, float(exp(double(s - max))), float sum,
 *     then a multiply by 1/sum;
 *   out = MatMul(p, V), the same outer-product branch.
 * q, out [batch][heads][head_dim]; caches [batch][kv_heads][cache_len][head_dim].
 * Returns -1 on bad sizes, -2 if scratch cannot be allocated. */
int ko_attention_decode(const float *q, const float *kc, const float *vc, float *out, int64_t batch, int64_t heads,
                        int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim);

#ifdef __cplusplus
}
#endif
#endif
