/*
 * kq_oracle.c -- CPU oracle (test infrastructure only) for the k-quant
 * dequantize-and-matmul path.  A plain-C restatement of the reference Go
 * arithmetic; see kq_oracle.h for the scope and for what pins it.  Every
 * function cites the reference file:line it follows (paths relative to the
 * root of xupit3r/vibrant).
 *
 * Build: oracle/Makefile (-O2 -ffp-contract=off -fno-tree-vectorize; the Go
 * compiler emits scalar code, and lane-wise vector code would give the same
 * bits anyway, so the flag only keeps the timing honest).
 */
#include "kq_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline float bits_to_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static inline uint32_t f32_to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

int ko_block_bytes(int qtype) {
    switch (qtype) {
    case KO_Q4_K: return KO_Q4K_BYTES;
    case KO_Q5_K: return KO_Q5K_BYTES;
    case KO_Q6_K: return KO_Q6K_BYTES;
    default: return 0;
    }
}

/* internal/tensor/tensor.go:629-676.  Two deliberate departures from IEEE
 * half->single conversion are reproduced: 0x8000 yields +0 (the Go constant
 * -0.0 is +0, tensor.go:637-639) and every NaN yields float32(math.NaN()),
 * whose bits are 0x7FC00000 (tensor.go:669-670). */
float ko_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    if (exp == 0) {
        if (mant == 0) return bits_to_f32(0u); /* both zeros -> +0 */
        uint32_t shift = 0, m = mant;
        while ((m & 0x400u) == 0) {           /* tensor.go:647-652 */
            m <<= 1;
            shift++;
        }
        m &= 0x3FFu;
        uint32_t exp32 = 127u - 14u - shift;  /* tensor.go:656 */
        return bits_to_f32((sign << 31) | (exp32 << 23) | (m << 13));
    }
    if (exp == 31) {
        if (mant == 0) return bits_to_f32((sign << 31) | 0x7F800000u);
        return bits_to_f32(0x7FC00000u);
    }
    return bits_to_f32((sign << 31) | ((exp - 15u + 127u) << 23) | (mant << 13));
}

/* internal/tensor/tensor.go:606-627: truncating conversion used only by the
 * reference's test quantizers. */
uint16_t ko_f32_to_f16(float f) {
    if (f == 0.0f) return 0;
    uint32_t bits = f32_to_bits(f);
    uint32_t sign = (bits >> 31) & 1u;
    int32_t exp = (int32_t)((bits >> 23) & 0xFFu) - 127 + 15;
    uint32_t mant = (bits >> 13) & 0x3FFu;
    if (exp <= 0) return (uint16_t)(sign << 15);
    if (exp >= 31) return (uint16_t)((sign << 15) | 0x7C00u);
    return (uint16_t)((sign << 15) | ((uint32_t)exp << 10) | mant);
}

/* internal/tensor/quant_q5k.go:97-120 */
void ko_extract_scales_mins(const uint8_t s[12], uint8_t sc[8], uint8_t m[8]) {
    sc[0] = s[0] & 0x3F;
    sc[1] = (uint8_t)((s[0] >> 6) | (s[1] << 2)) & 0x3F;
    sc[2] = (uint8_t)((s[1] >> 4) | (s[2] << 4)) & 0x3F;
    sc[3] = (s[2] >> 2) & 0x3F;
    sc[4] = s[3] & 0x3F;
    sc[5] = (uint8_t)((s[3] >> 6) | (s[4] << 2)) & 0x3F;
    sc[6] = (uint8_t)((s[4] >> 4) | (s[5] << 4)) & 0x3F;
    sc[7] = (s[5] >> 2) & 0x3F;
    m[0] = s[6] & 0x3F;
    m[1] = (uint8_t)((s[6] >> 6) | (s[7] << 2)) & 0x3F;
    m[2] = (uint8_t)((s[7] >> 4) | (s[8] << 4)) & 0x3F;
    m[3] = (s[8] >> 2) & 0x3F;
    m[4] = s[9] & 0x3F;
    m[5] = (uint8_t)((s[9] >> 6) | (s[10] << 2)) & 0x3F;
    m[6] = (uint8_t)((s[10] >> 4) | (s[11] << 4)) & 0x3F;
    m[7] = (s[11] >> 2) & 0x3F;
}

static inline uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* dequantizeQ4KBlockBatch, internal/tensor/block_cache.go:222-248 (same math
 * as DequantizeQ4_K, quant_q4k.go:37-79).  Layout quant_q4k.go:137-157:
 * d[0:2] dmin[2:4] scales[4:16] qs[16:144]. */
void ko_dequant_block_q4k(const uint8_t *blk, float out[256]) {
    float d = ko_f16_to_f32(le16(blk + 0));
    float dmin = ko_f16_to_f32(le16(blk + 2));
    uint8_t sc[8], m[8];
    ko_extract_scales_mins(blk + 4, sc, m);
    const uint8_t *qs = blk + 16;
    for (int sb = 0; sb < 8; sb++) {
        float scale = d * (float)sc[sb];
        float mn = dmin * (float)m[sb];
        for (int i = 0; i < 32; i++) {
            int v = sb * 32 + i;
            uint8_t bits = qs[v / 2];
            uint8_t q = (v % 2 == 0) ? (bits & 0x0F) : (bits >> 4);
            out[v] = scale * (float)q - mn;
        }
    }
}

/* dequantizeQ5KBlockBatch, internal/tensor/block_cache.go:82-122 (same math
 * as DequantizeQ5_K, quant_q5k.go:39-88).  Layout quant_q5k.go:229-252:
 * d[0:2] dmin[2:4] scales[4:16] qh[16:48] qs[48:176]. */
void ko_dequant_block_q5k(const uint8_t *blk, float out[256]) {
    float d = ko_f16_to_f32(le16(blk + 0));
    float dmin = ko_f16_to_f32(le16(blk + 2));
    uint8_t sc[8], m[8];
    ko_extract_scales_mins(blk + 4, sc, m);
    const uint8_t *qh = blk + 16;
    const uint8_t *qs = blk + 48;
    for (int sb = 0; sb < 8; sb++) {
        float scale = d * (float)sc[sb];
        float mn = dmin * (float)m[sb];
        for (int i = 0; i < 32; i++) {
            int v = sb * 32 + i;
            uint8_t lo = qs[v / 2];
            lo = (v % 2 == 0) ? (lo & 0x0F) : (lo >> 4);
            uint8_t hi = (qh[v / 8] >> (v % 8)) & 0x01;
            uint8_t q = lo | (uint8_t)(hi << 4);
            out[v] = scale * (float)q - mn;
        }
    }
}

/* dequantizeQ6KBlockBatch, internal/tensor/block_cache.go:158-186 (same math
 * as DequantizeQ6_K, quant_q6k.go:39-80).  Layout quant_q6k.go:134-156:
 * ql[0:128] qh[128:192] scales[192:208] (int8) d[208:210]. */
void ko_dequant_block_q6k(const uint8_t *blk, float out[256]) {
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *scales = (const int8_t *)(blk + 192);
    float d = ko_f16_to_f32(le16(blk + 208));
    for (int i = 0; i < 256; i++) {
        uint8_t lo = ql[i / 2];
        lo = (i % 2 == 0) ? (lo & 0x0F) : (lo >> 4);
        uint8_t hi = (qh[i / 4] >> ((i % 4) * 2)) & 0x03;
        uint8_t q = lo | (uint8_t)(hi << 4);
        float scale = (float)scales[i / 16];
        out[i] = d * scale * (float)((int)q - 32); /* (d*scale)*(q-32) */
    }
}

static void dequant_block(int qtype, const uint8_t *blk, float out[256]) {
    switch (qtype) {
    case KO_Q4_K: ko_dequant_block_q4k(blk, out); break;
    case KO_Q5_K: ko_dequant_block_q5k(blk, out); break;
    default: ko_dequant_block_q6k(blk, out); break;
    }
}

/* DequantizeQ4_KTensor / Q5_K / Q6_K (quant_q4k.go:161-211,
 * quant_q5k.go:256-307, quant_q6k.go:160-210). */
int ko_dequantize(int qtype, const uint8_t *data, int64_t nblocks, float *out) {
    int bb = ko_block_bytes(qtype);
    if (bb == 0 || nblocks < 0) return -1;
    for (int64_t b = 0; b < nblocks; b++) dequant_block(qtype, data + b * bb, out + b * 256);
    return 0;
}

/* DequantTransposeQ4K/Q5K/Q6K, internal/tensor/dequant_transpose.go:15-157:
 * numBlocks = M*N/256 (integer division), each block scattered to the
 * transposed position out[col*M + row] (:44-51). */
int ko_dequant_transpose(int qtype, const uint8_t *data, int64_t M, int64_t N, float *out) {
    int bb = ko_block_bytes(qtype);
    if (bb == 0 || M <= 0 || N <= 0) return -1;
    int64_t total = M * N;
    int64_t nblocks = total / 256;
    memset(out, 0, (size_t)total * sizeof(float));
    float buf[256];
    for (int64_t bi = 0; bi < nblocks; bi++) {
        dequant_block(qtype, data + bi * bb, buf);
        int64_t g = bi * 256;
        for (int k = 0; k < 256; k++) {
            int64_t src = g + k;
            int64_t row = src / N, col = src % N;
            out[col * M + row] = buf[k];
        }
    }
    return 0;
}

/* internal/tensor/simd_ops.go:60-78 */
float ko_vector_dot(const float *a, const float *b, int64_t n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
    int64_t i = 0;
    for (; i + 7 < n; i += 8) {
        s0 += a[i] * b[i];
        s1 += a[i + 1] * b[i + 1];
        s2 += a[i + 2] * b[i + 2];
        s3 += a[i + 3] * b[i + 3];
        s4 += a[i + 4] * b[i + 4];
        s5 += a[i + 5] * b[i + 5];
        s6 += a[i + 6] * b[i + 6];
        s7 += a[i + 7] * b[i + 7];
    }
    for (; i < n; i++) s0 += a[i] * b[i];
    return s0 + s1 + s2 + s3 + s4 + s5 + s6 + s7;
}

/* internal/tensor/simd_ops.go:82-98 */
void ko_vector_scale_add(float *dst, const float *src, int64_t n, float scale) {
    int64_t i = 0;
    for (; i + 7 < n; i += 8) {
        dst[i] += src[i] * scale;
        dst[i + 1] += src[i + 1] * scale;
        dst[i + 2] += src[i + 2] * scale;
        dst[i + 3] += src[i + 3] * scale;
        dst[i + 4] += src[i + 4] * scale;
        dst[i + 5] += src[i + 5] * scale;
        dst[i + 6] += src[i + 6] * scale;
        dst[i + 7] += src[i + 7] * scale;
    }
    for (; i < n; i++) dst[i] += src[i] * scale;
}

/* ---- worker fan-out standing in for the goroutines ---------------------- */

typedef struct {
    const float *a, *wt;
    float *c;
    int64_t M, K, N, lo, hi;
} ko_job;

static void *single_row_worker(void *p) {
    ko_job *j = (ko_job *)p;
    for (int64_t col = j->lo; col < j->hi; col++)
        j->c[col] = ko_vector_dot(j->a, j->wt + col * j->K, j->K);
    return NULL;
}

static void *parallel_rows_worker(void *p) {
    ko_job *j = (ko_job *)p;
    for (int64_t i = j->lo; i < j->hi; i++) {
        const float *arow = j->a + i * j->K;
        float *crow = j->c + i * j->N;
        for (int64_t col = 0; col < j->N; col++)
            crow[col] = ko_vector_dot(arow, j->wt + col * j->K, j->K);
    }
    return NULL;
}

static void run_jobs(void *(*fn)(void *), ko_job *jobs, int n) {
    if (n == 1) {
        fn(&jobs[0]);
        return;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n);
    int *started = (int *)calloc((size_t)n, sizeof(int));
    for (int w = 0; w < n; w++) started[w] = pthread_create(&th[w], NULL, fn, &jobs[w]) == 0;
    for (int w = 0; w < n; w++) {
        if (started[w]) pthread_join(th[w], NULL);
        else fn(&jobs[w]);
    }
    free(started);
    free(th);
}

/* matmul_simd.go:150-201, transposed branch :165-188.  numWorkers =
 * min(NumCPU, N); colsPerWorker = ceil(N/numWorkers). */
void ko_matmul_single_row_t(const float *x, const float *wt, int64_t K, int64_t N, float *y,
                            int nthreads) {
    int64_t workers = nthreads < 1 ? 1 : nthreads;
    if (workers > N) workers = N;
    int64_t per = (N + workers - 1) / workers;
    ko_job *jobs = (ko_job *)calloc((size_t)workers, sizeof(ko_job));
    for (int64_t w = 0; w < workers; w++) {
        int64_t lo = w * per, hi = lo + per;
        if (hi > N) hi = N;
        if (lo > hi) lo = hi;
        ko_job j = {x, wt, y, 1, K, N, lo, hi};
        jobs[w] = j;
    }
    run_jobs(single_row_worker, jobs, (int)workers);
    free(jobs);
}

/* matmul_simd.go:189-199: c starts at zero (Zeros, :157); rows with
 * x[k] == 0 are skipped. */
void ko_matmul_single_row_u(const float *x, const float *w, int64_t K, int64_t N, float *y) {
    memset(y, 0, (size_t)N * sizeof(float));
    for (int64_t k = 0; k < K; k++) {
        float av = x[k];
        if (av == 0) continue;
        ko_vector_scale_add(y, w + k * N, N, av);
    }
}

/* matmul_simd.go:13-69 (B pre-transposed or transposed into the pool buffer;
 * either way c[i][j] = dot(a_i, bT_j)). */
void ko_matmul_simd_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N, float *c) {
    for (int64_t i = 0; i < M; i++)
        for (int64_t col = 0; col < N; col++)
            c[i * N + col] = ko_vector_dot(a + i * K, wt + col * K, K);
}

/* matmul_simd.go:72-146, transposed branch :91-112: 64-wide blocks over
 * (i, j, k); each k-chunk's sum is added into c (which starts at zero). */
void ko_matmul_blocked_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N, float *c) {
    const int64_t bs = 64;
    memset(c, 0, (size_t)(M * N) * sizeof(float));
    for (int64_t i0 = 0; i0 < M; i0 += bs)
        for (int64_t j0 = 0; j0 < N; j0 += bs)
            for (int64_t k0 = 0; k0 < K; k0 += bs) {
                int64_t iM = i0 + bs < M ? i0 + bs : M;
                int64_t jM = j0 + bs < N ? j0 + bs : N;
                int64_t kM = k0 + bs < K ? k0 + bs : K;
                for (int64_t i = i0; i < iM; i++)
                    for (int64_t j = j0; j < jM; j++) {
                        float sum = 0;
                        for (int64_t k = k0; k < kM; k++) sum += a[i * K + k] * wt[j * K + k];
                        c[i * N + j] += sum;
                    }
            }
}

/* matmul_simd.go:204-276: rowsPerWorker = ceil(M/NumCPU). */
void ko_matmul_parallel_t(const float *a, const float *wt, int64_t M, int64_t K, int64_t N, float *c,
                          int nthreads) {
    int64_t workers = nthreads < 1 ? 1 : nthreads;
    int64_t per = (M + workers - 1) / workers;
    ko_job *jobs = (ko_job *)calloc((size_t)workers, sizeof(ko_job));
    for (int64_t w = 0; w < workers; w++) {
        int64_t lo = w * per, hi = lo + per;
        if (hi > M) hi = M;
        if (lo > hi) lo = hi;
        ko_job j = {a, wt, c, M, K, N, lo, hi};
        jobs[w] = j;
    }
    run_jobs(parallel_rows_worker, jobs, (int)workers);
    free(jobs);
}

/* The size dispatch of MatMul (matmul.go:75-89) once B is float32 and
 * transposed ([N,K]); HasAVX2() is always true on amd64 (simd.go:27-34). */
static void dispatch_transposed(const float *a, const float *wt, int64_t M, int64_t K, int64_t N,
                                float *c, int nthreads) {
    if (M == 1) {
        ko_matmul_single_row_t(a, wt, K, N, c, nthreads);
        return;
    }
    int64_t ops = M * N * K;
    if (ops < 1024) ko_matmul_simd_t(a, wt, M, K, N, c);
    else if (ops < 1024 * 1024) ko_matmul_blocked_t(a, wt, M, K, N, c);
    else ko_matmul_parallel_t(a, wt, M, K, N, c, nthreads);
}

/* tensor.MatMul with a quantized B, matmul.go:46-99 + GetOrDequantTranspose
 * tensor.go:535-588 (fused dequant-transpose for 2-D tensors). */
int ko_matmul_quant(int qtype, const float *a, int64_t M, int64_t K, const uint8_t *bq, int64_t N,
                    float *c, float *wt_scratch, int nthreads) {
    if (ko_block_bytes(qtype) == 0 || M <= 0 || K <= 0 || N <= 0) return -1;
    if (ko_dequant_transpose(qtype, bq, K, N, wt_scratch) != 0) return -1;
    dispatch_transposed(a, wt_scratch, M, K, N, c, nthreads);
    return 0;
}

/* LM-head route, internal/transformer/model.go:389-403: Dequantize
 * (ops.go:486-530, untransposed [K,N]) then MatMul.  For an untransposed
 * float32 B, GetOrDequantTranspose returns B unchanged (tensor.go:543-547);
 * M == 1 takes the outer-product branch (matmul_simd.go:189-199); larger M
 * transposes B into a pool buffer (matmul_simd.go:36-45, :227-237) or walks
 * its columns (:113-138) with the same arithmetic as the transposed kernels. */
int ko_matmul_dequant_untransposed(int qtype, const float *a, int64_t M, int64_t K,
                                   const uint8_t *bq, int64_t N, float *c, float *w_scratch,
                                   int nthreads) {
    if (ko_block_bytes(qtype) == 0 || M <= 0 || K <= 0 || N <= 0) return -1;
    int64_t nblocks = (K * N + 255) / 256;
    if (ko_dequantize(qtype, bq, nblocks, w_scratch) != 0) return -1;
    if (M == 1) {
        ko_matmul_single_row_u(a, w_scratch, K, N, c);
        return 0;
    }
    float *wt = (float *)malloc((size_t)(K * N) * sizeof(float));
    if (!wt) return -2;
    for (int64_t k = 0; k < K; k++)
        for (int64_t n = 0; n < N; n++) wt[n * K + k] = w_scratch[k * N + n];
    dispatch_transposed(a, wt, M, K, N, c, nthreads);
    free(wt);
    return 0;
}

/* QuantizeQ4_K (internal/tensor/quant_q4k.go:215-282), serialized in the
 * byte order of QuantizeQ4_KTensor (matmul_quant_helpers.go:116-145): per
 * block min/max, scale = (max - min) / 15 (at least 1e-10), D = f16(scale),
 * Dmin = f16(min), the scale bytes 0 and 6 set to 32 and the rest zero, and
 * q = uint8((x - min) / scale) clamped to 15, packed low nibble first.  The
 * reference's test quantizer: only sub-block 0 gets a non-zero scale. */
int ko_quantize_q4k(const float *in, int64_t n, uint8_t *out) {
    if (n <= 0) return -1;
    const int64_t nb = (n + 255) / 256;
    memset(out, 0, (size_t)(nb * KO_Q4K_BYTES));
    for (int64_t b = 0; b < nb; b++) {
        uint8_t *blk = out + b * KO_Q4K_BYTES;
        const int64_t off = b * 256, end = off + 256 < n ? off + 256 : n;
        float mn = FLT_MAX, mx = -FLT_MAX;
        for (int64_t i = off; i < end; i++) {
            if (in[i] < mn) mn = in[i];
            if (in[i] > mx) mx = in[i];
        }
        float scale = (mx - mn) / 15.0f;
        if (scale < 1e-10f) scale = 1e-10f;
        const uint16_t d = ko_f32_to_f16(scale), dm = ko_f32_to_f16(mn);
        blk[0] = (uint8_t)d;
        blk[1] = (uint8_t)(d >> 8);
        blk[2] = (uint8_t)dm;
        blk[3] = (uint8_t)(dm >> 8);
        blk[4 + 0] = 32;
        blk[4 + 6] = 32;
        for (int64_t i = off; i < end; i++) {
            const int64_t idx = i - off;
            uint8_t q = (uint8_t)((in[i] - mn) / scale);
            if (q > 15) q = 15;
            if (idx % 2 == 0) blk[16 + idx / 2] = q & 0x0F;
            else blk[16 + idx / 2] |= (uint8_t)((q & 0x0F) << 4);
        }
    }
    return 0;
}

/* QuantizeQ6_K (internal/tensor/quant_q6k.go:214-294), serialized in the
 * byte order of QuantizeQ6_KTensor (matmul_quant_helpers.go:62-92): d =
 * max(|max|, |min|) / 32 (at least 1e-10), D = f16(d), every group scale 1,
 * q = int(x / d + 32.5) clamped to [0, 63]: low nibbles into Ql, high bit
 * pairs into Qh. */
int ko_quantize_q6k(const float *in, int64_t n, uint8_t *out) {
    if (n <= 0) return -1;
    const int64_t nb = (n + 255) / 256;
    memset(out, 0, (size_t)(nb * KO_Q6K_BYTES));
    for (int64_t b = 0; b < nb; b++) {
        uint8_t *blk = out + b * KO_Q6K_BYTES;
        const int64_t off = b * 256, end = off + 256 < n ? off + 256 : n;
        float mn = FLT_MAX, mx = -FLT_MAX;
        for (int64_t i = off; i < end; i++) {
            if (in[i] < mn) mn = in[i];
            if (in[i] > mx) mx = in[i];
        }
        const double amax = fabs((double)mx) > fabs((double)mn) ? fabs((double)mx) : fabs((double)mn);
        float d = (float)amax / 32.0f;
        if (d < 1e-10f) d = 1e-10f;
        const uint16_t dh = ko_f32_to_f16(d);
        for (int j = 0; j < 16; j++) blk[192 + j] = 1;
        blk[208] = (uint8_t)dh;
        blk[209] = (uint8_t)(dh >> 8);
        for (int64_t i = off; i < end; i++) {
            const int64_t idx = i - off;
            const float scale = 1.0f;  /* Scales[idx / 16] */
            const float scaled = in[i] / (d * scale);
            int q = (int)(scaled + 32.5f);
            if (q < 0) q = 0;
            if (q > 63) q = 63;
            if (idx % 2 == 0) blk[idx / 2] = (uint8_t)(q & 0x0F);
            else blk[idx / 2] |= (uint8_t)((q & 0x0F) << 4);
            blk[128 + idx / 4] |= (uint8_t)(((q >> 4) & 0x03) << ((idx % 4) * 2));
        }
    }
    return 0;
}

/* MatMulQ5K / MatMulQ6K (internal/tensor/matmul_quant.go:30-191): the
 * reference's fused route, every output a float32 sum over k in sequential
 * order of a[i,k] * deq(k*N + j) (the per-element dequantization equals the
 * block dequantization bit for bit, quant_q4k_test.go:48-91).  Restated for
 * all three types; M*N outputs of K terms each. */
int ko_matmul_quant_sequential(int qtype, const float *a, int64_t M, int64_t K, const uint8_t *bq, int64_t N,
                               float *c) {
    if (ko_block_bytes(qtype) == 0 || M <= 0 || K <= 0 || N <= 0) return -1;
    const int64_t nblocks = (K * N + 255) / 256;
    float *w = (float *)malloc((size_t)(nblocks * 256) * sizeof(float));
    if (!w) return -2;
    if (ko_dequantize(qtype, bq, nblocks, w) != 0) {
        free(w);
        return -1;
    }
    for (int64_t i = 0; i < M; i++) {
        for (int64_t j = 0; j < N; j++) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; k++) sum += a[i * K + k] * w[k * N + j];
            c[i * N + j] = sum;
        }
    }
    free(w);
    return 0;
}

/* ---- decode attention and RoPE (internal/transformer) ---------------------- */

/* NewRoPE, internal/transformer/rope.go:19-43. */
void ko_rope_tables(int64_t head_dim, double freq_base, int64_t max_seq, float *cos_t, float *sin_t) {
    const int64_t half = head_dim / 2;
    for (int64_t pos = 0; pos < max_seq; pos++) {
        for (int64_t i = 0; i < half; i++) {
            const double freq = 1.0 / pow(freq_base, (double)(2 * i) / (double)head_dim);
            const double angle = (double)pos * freq;
            cos_t[pos * half + i] = (float)cos(angle);
            sin_t[pos * half + i] = (float)sin(angle);
        }
    }
}

/* RoPE.ApplyRotation, CPU branch, rope.go:49-124 (the loop :98-118). */
int ko_rope_apply(const float *x, float *out, const float *cos_t, const float *sin_t, const int32_t *positions,
                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t max_seq) {
    const int64_t half = head_dim / 2;
    for (int64_t s = 0; s < seq; s++)
        if (positions[s] < 0 || positions[s] >= max_seq) return -1;
    for (int64_t b = 0; b < batch; b++) {
        for (int64_t h = 0; h < heads; h++) {
            for (int64_t s = 0; s < seq; s++) {
                const int64_t off = ((b * heads + h) * seq + s) * head_dim;
                const int64_t t = (int64_t)positions[s] * half;
                for (int64_t i = 0; i < half; i++) {
                    const float c = cos_t[t + i], sn = sin_t[t + i];
                    const float x0 = x[off + 2 * i], x1 = x[off + 2 * i + 1];
                    const float p0 = x0 * c, p1 = x1 * sn, p2 = x0 * sn, p3 = x1 * c;
                    out[off + 2 * i] = p0 - p1;
                    out[off + 2 * i + 1] = p2 + p3;
                }
            }
        }
    }
    return 0;
}

/* concatenateSeqDim, attention.go:529-569: the cached rows stay where they
 * are and the new rows follow them. */
int ko_kv_append(float *cache, const float *new_rows, int64_t batch, int64_t kv_heads, int64_t cache_len,
                 int64_t row0, int64_t n_new, int64_t head_dim) {
    if (row0 < 0 || n_new < 0 || row0 + n_new > cache_len) return -1;
    for (int64_t b = 0; b < batch; b++) {
        for (int64_t h = 0; h < kv_heads; h++) {
            float *dst = cache + ((b * kv_heads + h) * cache_len + row0) * head_dim;
            const float *src = new_rows + (b * kv_heads + h) * n_new * head_dim;
            memcpy(dst, src, (size_t)(n_new * head_dim) * sizeof(float));
        }
    }
    return 0;
}

/* expandKVHeads (attention.go:280-314) and computeAttention (:316-363) for one
 * query row: scaleScores :413-427, applyCausalMask :429-460 (nothing masked
 * when rows < cols, and a 1x1 score has nothing above its diagonal),
 * applySoftmax :462-527, both products through matmulSIMDSingleRow's
 * untransposed branch (matmul_simd.go:189-199, ko_matmul_single_row_u). */
int ko_attention_decode(const float *q, const float *kc, const float *vc, float *out, int64_t batch, int64_t heads,
                        int64_t kv_heads, int64_t len, int64_t cache_len, int64_t head_dim) {
    if (batch <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || len <= 0 || cache_len < len ||
        head_dim <= 0)
        return -1;
    const int64_t group = heads / kv_heads, D = head_dim;
    float *kt = (float *)malloc((size_t)(D * len) * sizeof(float));
    float *row = (float *)malloc((size_t)len * sizeof(float));
    if (!kt || !row) {
        free(kt);
        free(row);
        return -2;
    }
    const float scale = (float)(1.0 / sqrt((double)D));
    const float neg_inf = -INFINITY;
    for (int64_t b = 0; b < batch; b++) {
        for (int64_t h = 0; h < heads; h++) {
            const int64_t kvh = h / group;
            const float *kr = kc + (b * kv_heads + kvh) * cache_len * D;
            const float *vr = vc + (b * kv_heads + kvh) * cache_len * D;
            const float *qh = q + (b * heads + h) * D;
            /* Transpose (ops.go:445-468): kt[d][j] = K[j][d] */
            for (int64_t j = 0; j < len; j++)
                for (int64_t d = 0; d < D; d++) kt[d * len + j] = kr[j * D + d];
            ko_matmul_single_row_u(qh, kt, D, len, row);
            for (int64_t j = 0; j < len; j++) row[j] *= scale;
            float mx = row[0];
            for (int64_t j = 0; j < len; j++)
                if (row[j] > mx) mx = row[j];
            float sum = 0.0f;
            for (int64_t j = 0; j < len; j++) {
                if (row[j] == neg_inf) {
                    row[j] = 0.0f;
                } else {
                    row[j] = (float)exp((double)(row[j] - mx));
                    sum += row[j];
                }
            }
            if (sum > 0.0f) {
                const float inv = 1.0f / sum;
                for (int64_t j = 0; j < len; j++) row[j] *= inv;
            }
            ko_matmul_single_row_u(row, vr, len, D, out + (b * heads + h) * D);
        }
    }
    free(kt);
    free(row);
    return 0;
}
