/*
 * oracle.c - CPU restatement of the reference's int8 GEMM path and decoder
 * block ops.  TEST INFRASTRUCTURE ONLY (see oracle.h): the B200 library never
 * links or calls this file.
 *
 * Built with -ffp-contract=off: every fused multiply-add is an explicit
 * fmaf() that mirrors a fusion GCC performs in the reference's
 * target("avx2,fma") kernels (the reference builds with -ffp-contract=fast,
 * Makefile CXXFLAGS).  Those fusions were confirmed bit-for-bit against the
 * reference library compiled from source (tests/test_oracle.py).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* Epilogue math (src/internal.h:87-136)                                      */
/* ------------------------------------------------------------------------- */

static const float kLog2e = 1.4426950408889634f;
static const float kC1 = 0.6931471805599453f;
static const float kC2 = 0.2402265069591007f;
static const float kC3 = 0.05550410866482158f;
static const float kC4 = 0.009618129107628477f;
static const float kC5 = 0.0013333558146428443f;

/* 2^f for f in [0,1): the reference's degree-5 polynomial.  In the AVX2
 * kernels every "c + f*(...)" step of the Horner chain becomes one FMA. */
static float exp2_poly(float f, int form)
{
    if (form != ORACLE_FORM_SCALAR) {
        float p = fmaf(f, kC5, kC4);
        p = fmaf(f, p, kC3);
        p = fmaf(f, p, kC2);
        p = fmaf(f, p, kC1);
        return fmaf(f, p, 1.0f);
    }
    return 1.0f + f * (kC1 + f * (kC2 + f * (kC3 + f * (kC4 + f * kC5))));
}

/* fast_expf, src/internal.h:87-108. */
float oracle_fast_expf(float x, int form)
{
    if (x < -80.0f) return 0.0f;
    if (x > 80.0f) return INFINITY;
    float z = x * kLog2e;
    float zi = floorf(z);
    float f = z - zi;
    return ldexpf(exp2_poly(f, form), (int)zi);
}

/* exp256_ps, src/kernels/llm.cpp:32-56: clamps to [-80,80] instead of the
 * scalar cut-offs, FMA Horner, 2^n from exponent bits (exact for the clamped
 * range, n in [-116,116]). */
static float exp256_lane(float x)
{
    if (x < -80.0f) x = -80.0f;
    if (x > 80.0f) x = 80.0f;
    float z = x * kLog2e;
    float zi = floorf(z);
    float f = z - zi;
    return ldexpf(exp2_poly(f, ORACLE_FORM_AVX2), (int)zi);
}

static float silu_f(float x, int form)
{
    return x / (1.0f + oracle_fast_expf(-x, form));
}

/* gelu_tanh, src/internal.h:113-120.  In the AVX2 kernels x + k1*x3 fuses. */
static float gelu_tanh_f(float x, int form)
{
    const float k0 = 0.7978845608028654f;
    const float k1 = 0.035677408136300125f;
    float x3 = x * x * x;
    float inner = form != ORACLE_FORM_SCALAR ? k0 * fmaf(k1, x3, x)
                                             : k0 * (x + k1 * x3);
    float t = 2.0f / (1.0f + oracle_fast_expf(-2.0f * inner, form)) - 1.0f;
    return 0.5f * x * (1.0f + t);
}

float oracle_epilogue(float v, uint32_t epilogue, int form)
{
    switch (epilogue) {
    case 1: return v > 0.0f ? v : 0.0f;              /* RELU */
    case 2: return silu_f(v, form);                  /* SILU */
    case 3:                                          /* GELU_TANH */
    case 4: return gelu_tanh_f(v, form);             /* GELU_ERF aliases tanh */
    default: return v;
    }
}

/* ------------------------------------------------------------------------- */
/* MATMUL_I8 (src/kernels/kernels.cpp:526-550)                                */
/* ------------------------------------------------------------------------- */

void oracle_gemm_i8_acc(const int8_t *A, uint32_t lda, const int8_t *B,
                        uint32_t ldb, int32_t *acc, uint32_t M, uint32_t K,
                        uint32_t N)
{
    /* int32 accumulation over all of K is exact and order-free, so a rank-1
     * update order (vectorisable) gives the same integers as the reference's
     * dot-product order. */
    for (uint32_t m = 0; m < M; ++m) {
        int32_t *row = acc + (size_t)m * N;
        memset(row, 0, sizeof(int32_t) * N);
        const int8_t *a = A + (size_t)m * lda;
        for (uint32_t k = 0; k < K; ++k) {
            const int32_t av = a[k];
            if (!av) continue;
            const int8_t *b = B + (size_t)k * ldb;
            for (uint32_t n = 0; n < N; ++n) row[n] += av * (int32_t)b[n];
        }
    }
}

/* store_i8_c, src/kernels/kernels.cpp:526-535.
 *   out = (float)dot * sa * sb      (left to right, IEEE)
 *   out += bias                     (AVX2 register-block kernels: fused,
 *                                    fmaf(t, sb, bias); decode streams and
 *                                    scalar: two roundings)
 *   out = apply_epilogue(out)       (polynomial fused except in scalar) */
float oracle_dequant(int32_t acc, float sa, float sb, const float *bias_n,
                     uint32_t epilogue, int form)
{
    float t = (float)acc * sa;
    float out;
    if (bias_n)
        out = form == ORACLE_FORM_AVX2 ? fmaf(t, sb, *bias_n) : t * sb + *bias_n;
    else
        out = t * sb;
    return oracle_epilogue(out, epilogue, form);
}

void oracle_matmul_i8(const int8_t *A, uint32_t lda, const int8_t *B,
                      const float *scale_a, const float *scale_b,
                      const float *bias, float *C, uint32_t ldc, uint32_t M,
                      uint32_t K, uint32_t N, uint32_t epilogue, int form)
{
    int32_t *row = (int32_t *)malloc(sizeof(int32_t) * (N ? N : 1));
    if (!row) return;
    for (uint32_t m = 0; m < M; ++m) {
        oracle_gemm_i8_acc(A + (size_t)m * lda, lda, B, N, row, 1, K, N);
        const float sa = scale_a ? scale_a[m] : 1.0f;
        for (uint32_t n = 0; n < N; ++n) {
            const float sb = scale_b ? scale_b[n] : 1.0f;
            C[(size_t)m * ldc + n] = oracle_dequant(row[n], sa, sb,
                                                    bias ? bias + n : NULL,
                                                    epilogue, form);
        }
    }
    free(row);
}

/* ------------------------------------------------------------------------- */
/* MATMUL_I8 as a reference device computes it: which kernel owns each      */
/* output element, and so which form its dequant epilogue is rounded in.     */
/* ------------------------------------------------------------------------- */

/* Per-worker scratch the reference kernels stage into (VNPU_LOCAL_STORE_BYTES,
 * include/vnpu.h:51); thread_scratch() hands out that plus one cache line and
 * each kernel asks for its bytes plus one cache line, so the cache lines
 * cancel in every "fits" test below. */
#define ORACLE_LOCAL_STORE 262144u

/* decode_max_tile_columns, src/core/scheduler.cpp:75-93: the widest decode
 * column tile, half of L2 shared by `rows` int32 staging rows, bounded by the
 * scratch, rounded down to 32 columns, at least 256. */
static uint32_t i8_decode_cap(uint64_t l2_bytes, uint32_t rows)
{
    uint64_t l2 = l2_bytes ? l2_bytes : 512u * 1024u;
    uint64_t cols = l2 / (8u * (uint64_t)rows);
    uint64_t scratch = ORACLE_LOCAL_STORE / (4u * (uint64_t)rows);
    if (cols > scratch) cols = scratch;
    cols &= ~(uint64_t)31u;
    if (cols < 256u) cols = 256u;
    if (cols > 0x7fffffffu) cols = 0x7fffffffu;
    return (uint32_t)cols;
}

void oracle_i8_tile_geometry(uint32_t unit, uint32_t M, uint32_t N,
                             uint32_t threads, uint32_t tile_m,
                             uint32_t tile_n, int pack_b, uint64_t l2_bytes,
                             uint32_t *tm_out, uint32_t *tn_out)
{
    const uint32_t units = threads ? threads : 1;
    uint32_t tk;
    /* Decode rows (src/core/scheduler.cpp:107-175): M <= 3 rows of int8 get
     * one contiguous column slice per worker once a worker's share of N
     * reaches 1024 columns; every other case is the F32 geometry. */
    if (M <= 3 && (unit == 0 || unit == 1) && N / units >= 1024u) {
        uint32_t tiles = N / 256u;
        if (tiles < 1) tiles = 1;
        if (tiles > units) tiles = units;
        const uint32_t cap = i8_decode_cap(l2_bytes, M);
        if ((N + tiles - 1) / tiles > cap) {
            tiles = (N + cap - 1) / cap;
            tiles = (tiles + units - 1) / units * units;
        }
        uint32_t wide = ((N + tiles - 1) / tiles + 31u) & ~31u;
        if (wide < 1) wide = 1;
        *tm_out = M;
        *tn_out = wide < N ? wide : N;
        return;
    }
    oracle_f32_tile_geometry(unit, M, N, threads, tile_m, 1, tile_n, pack_b,
                             tm_out, &tk, tn_out);
}

/* The form of output element (m, n), gemm_i8_dispatch_tile
 * (src/kernels/kernels.cpp:922-978) applied to the tile (m, n) falls in.
 * The AVX2 kernels round store_i8_c differently depending on where GCC
 * inlined and fused it (found element by element against the reference
 * build, tests/test_oracle.py):
 *   2x32 register blocks, packed or not (:634-700, :779-842)   block
 *   rank-2/3 streams (:581-632), the rank-1 row stream (:746-764) stream
 *   the scalar tile for the column tail of a row pair           stream
 *   the scalar tile for the column tail of a single row         scalar
 * and the scalar ISA and the Cell unit (:880-920) are scalar throughout. */
int oracle_i8_element_form(uint32_t unit, int avx2, int pack_b, uint32_t K,
                           uint32_t M, uint32_t N, uint32_t tm, uint32_t tn,
                           uint32_t m, uint32_t n)
{
    if (!avx2 || unit == 3) return ORACLE_FORM_SCALAR;
    const uint32_t m0 = m / tm * tm, n0 = n / tn * tn;
    const uint32_t rows = M - m0 < tm ? M - m0 : tm;
    const uint32_t cols = N - n0 < tn ? N - n0 : tn;
    const int tail = n - n0 >= (cols & ~31u);
    const int single = (rows & 1u) && m - m0 == rows - 1u;
    const uint64_t stride8 = ((uint64_t)cols + 7u) & ~(uint64_t)7u;
    if (cols >= 1024u && (rows == 2u || rows == 3u) &&
        stride8 * rows * 4u <= ORACLE_LOCAL_STORE)
        return ORACLE_FORM_STREAM;                      /* rank-R stream */
    if (pack_b && rows >= 3u && (uint64_t)K * cols <= ORACLE_LOCAL_STORE) {
        if (!tail) return ORACLE_FORM_AVX2;             /* packed panel blocks */
        return single ? ORACLE_FORM_SCALAR : ORACLE_FORM_STREAM;
    }
    if (!single) return tail ? ORACLE_FORM_STREAM : ORACLE_FORM_AVX2;
    if ((uint64_t)cols * 4u <= ORACLE_LOCAL_STORE) return ORACLE_FORM_STREAM;
    /* no room to stage the row: the 1x32 blocked walk, scalar tail */
    return tail ? ORACLE_FORM_SCALAR : ORACLE_FORM_AVX2;
}

void oracle_i8_form_map(uint32_t unit, uint32_t M, uint32_t K, uint32_t N,
                        uint32_t threads, uint32_t tile_m, uint32_t tile_n,
                        int pack_b, int avx2, uint64_t l2_bytes, int32_t *forms)
{
    uint32_t tm, tn;
    if (unit == 0) unit = 1;
    oracle_i8_tile_geometry(unit, M, N, threads, tile_m, tile_n, pack_b,
                            l2_bytes, &tm, &tn);
    for (uint32_t m = 0; m < M; ++m)
        for (uint32_t n = 0; n < N; ++n)
            forms[(size_t)m * N + n] = oracle_i8_element_form(
                unit, avx2, pack_b, K, M, N, tm, tn, m, n);
}

void oracle_matmul_i8_device(const int8_t *A, uint32_t lda, const int8_t *B,
                             const float *scale_a, const float *scale_b,
                             const float *bias, float *C, uint32_t ldc,
                             uint32_t M, uint32_t K, uint32_t N,
                             uint32_t epilogue, uint32_t unit,
                             uint32_t threads, uint32_t tile_m,
                             uint32_t tile_n, int pack_b, int avx2,
                             uint64_t l2_bytes)
{
    uint32_t tm, tn;
    if (unit == 0) unit = 1;  /* choose_unit: AUTO resolves to VOODOO */
    oracle_i8_tile_geometry(unit, M, N, threads, tile_m, tile_n, pack_b,
                            l2_bytes, &tm, &tn);
    int32_t *row = (int32_t *)malloc(sizeof(int32_t) * (N ? N : 1));
    if (!row) return;
    for (uint32_t m = 0; m < M; ++m) {
        oracle_gemm_i8_acc(A + (size_t)m * lda, lda, B, N, row, 1, K, N);
        const float sa = scale_a ? scale_a[m] : 1.0f;
        for (uint32_t n = 0; n < N; ++n) {
            const float sb = scale_b ? scale_b[n] : 1.0f;
            const int form = oracle_i8_element_form(unit, avx2, pack_b, K, M,
                                                    N, tm, tn, m, n);
            C[(size_t)m * ldc + n] = oracle_dequant(row[n], sa, sb,
                                                    bias ? bias + n : NULL,
                                                    epilogue, form);
        }
    }
    free(row);
}

/* ------------------------------------------------------------------------- */
/* QUANTIZE_I8 (src/kernels/llm.cpp:387-436)                                  */
/* ------------------------------------------------------------------------- */

/* quantize_value, src/kernels/llm.cpp:387-393: std::round is half away from
 * zero (roundf), clamp to [-128, 127]. */
static int8_t quantize_value(float x, float inv)
{
    float q = roundf(x * inv);
    if (q > 127.0f) q = 127.0f;
    if (q < -128.0f) q = -128.0f;
    return (int8_t)(int)q;
}

/* scale = maxabs/127 with the reference's guard (llm.cpp:403-404).  NaN
 * elements never win std::max(maxabs, |x|), so they are skipped. */
static float scale_of(float maxabs)
{
    float scale = maxabs / 127.0f;
    if (scale <= 0.0f || !isfinite(scale)) scale = 1.0f;
    return scale;
}

static float absmax_step(float m, float x)
{
    float a = fabsf(x);
    return m < a ? a : m;   /* std::max(m, a) */
}

int oracle_quantize_i8(const float *X, int8_t *Y, float *scales, uint64_t rows,
                       uint64_t cols, uint32_t axis)
{
    if (!X || !Y || !scales || !rows || !cols || axis > 2) return -1;
    if (axis == 0) {
        for (uint64_t r = 0; r < rows; ++r) {
            const float *x = X + r * cols;
            float m = 0.0f;
            for (uint64_t j = 0; j < cols; ++j) m = absmax_step(m, x[j]);
            float scale = scale_of(m);
            float inv = 1.0f / scale;
            scales[r] = scale;
            for (uint64_t j = 0; j < cols; ++j) Y[r * cols + j] = quantize_value(x[j], inv);
        }
    } else if (axis == 1) {
        float *m = (float *)calloc(cols, sizeof(float));
        if (!m) return -2;
        for (uint64_t r = 0; r < rows; ++r)
            for (uint64_t c = 0; c < cols; ++c) m[c] = absmax_step(m[c], X[r * cols + c]);
        for (uint64_t c = 0; c < cols; ++c) scales[c] = scale_of(m[c]);
        for (uint64_t r = 0; r < rows; ++r)
            for (uint64_t c = 0; c < cols; ++c)
                Y[r * cols + c] = quantize_value(X[r * cols + c], 1.0f / scales[c]);
        free(m);
    } else {
        /* Per tensor (src/core/scheduler.cpp:441-460, llm.cpp:430-436):
         * scales[0] = maxabs/127, then inv = 1/(scales[0] > 0 ? scales[0] : 1). */
        uint64_t n = rows * cols;
        float m = 0.0f;
        for (uint64_t i = 0; i < n; ++i) m = absmax_step(m, X[i]);
        scales[0] = scale_of(m);
        float inv = 1.0f / (scales[0] > 0.0f ? scales[0] : 1.0f);
        for (uint64_t i = 0; i < n; ++i) Y[i] = quantize_value(X[i], inv);
    }
    return 0;
}

/* vnpu_pack_weights_i8, src/core/scheduler.cpp:783-805: canonical KxN copy
 * and int32 column sums. */
void oracle_column_sums(const int8_t *B, uint32_t K, uint32_t N, uint32_t ldb,
                        uint32_t trans_b, int32_t *sums, int8_t *canonical)
{
    uint32_t ld = ldb ? ldb : (trans_b ? K : N);
    for (uint32_t n = 0; n < N; ++n) sums[n] = 0;
    for (uint32_t k = 0; k < K; ++k)
        for (uint32_t n = 0; n < N; ++n) {
            int8_t v = trans_b ? B[(size_t)n * ld + k] : B[(size_t)k * ld + n];
            if (canonical) canonical[(size_t)k * N + n] = v;
            sums[n] += v;
        }
}

/* ------------------------------------------------------------------------- */
/* Block ops (src/kernels/llm.cpp)                                            */
/* ------------------------------------------------------------------------- */

/* hsum256, src/kernels/llm.cpp:19-28: (lo+hi), then two horizontal adds. */
static float hsum8(const float v[8])
{
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    return (s0 + s1) + (s2 + s3);
}

/* dot_avx2, src/kernels/llm.cpp:332-343. */
static float dot_avx2(const float *a, const float *b, uint32_t n)
{
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float sum = hsum8(acc);
    for (; i < n; ++i) sum = fmaf(a[i], b[i], sum);
    return sum;
}

/* RMSNorm: scalar src/kernels/llm.cpp:64-77; AVX2 :80-106. */
void oracle_rmsnorm(const float *X, const float *W, float *Y, uint32_t rows,
                    uint32_t cols, float eps, int form)
{
    float e = eps > 0.0f ? eps : 1e-5f;
    for (uint32_t r = 0; r < rows; ++r) {
        const float *x = X + (size_t)r * cols;
        float *y = Y + (size_t)r * cols;
        float ss;
        if (form == ORACLE_FORM_AVX2) {
            ss = dot_avx2(x, x, cols);
        } else {
            ss = 0.0f;
            for (uint32_t j = 0; j < cols; ++j) ss += x[j] * x[j];
        }
        float inv = 1.0f / sqrtf(ss / (float)cols + e);
        uint32_t vec_end = form == ORACLE_FORM_AVX2 ? (cols / 8u) * 8u : 0u;
        for (uint32_t j = 0; j < cols; ++j) {
            float w = W ? W[j] : 1.0f;
            y[j] = j < vec_end ? (x[j] * w) * inv : x[j] * inv * w;
        }
    }
}

/* rotate_vector, src/kernels/llm.cpp:188-217. */
static void rotate_vector(float *x, uint32_t dim, float position,
                          float theta_base, float scaling, int interleaved)
{
    if (!x || dim < 2) return;
    position *= scaling;
    if (interleaved) {
        for (uint32_t j = 0; j + 1 < dim; j += 2) {
            float inv = 1.0f / powf(theta_base, (float)j / (float)dim);
            float angle = position * inv;
            float c = cosf(angle), s = sinf(angle);
            float x0 = x[j], x1 = x[j + 1];
            x[j] = x0 * c - x1 * s;
            x[j + 1] = x0 * s + x1 * c;
        }
    } else {
        uint32_t half = dim / 2;
        for (uint32_t j = 0; j < half; ++j) {
            float inv = 1.0f / powf(theta_base, 2.0f * (float)j / (float)dim);
            float angle = position * inv;
            float c = cosf(angle), s = sinf(angle);
            float x0 = x[j], x1 = x[j + half];
            x[j] = x0 * c - x1 * s;
            x[j + half] = x0 * s + x1 * c;
        }
    }
}

/* kernel_rope_tokens, src/kernels/llm.cpp:576-602. */
void oracle_rope(float *Q, float *K, const int32_t *positions, uint32_t batch,
                 uint32_t heads, uint32_t q_seq, uint32_t k_seq,
                 uint32_t head_dim, uint32_t position_offset,
                 uint32_t interleaved, float theta_base, float scaling)
{
    if (!Q && !K) return;
    uint32_t seq = q_seq > k_seq ? q_seq : k_seq;
    uint64_t total = (uint64_t)batch * heads * seq;
    float theta = theta_base > 0.0f ? theta_base : 10000.0f;
    float sc = scaling > 0.0f ? scaling : 1.0f;
    for (uint64_t idx = 0; idx < total; ++idx) {
        uint64_t bh = idx / seq;
        uint32_t t = (uint32_t)(idx % seq);
        float position = (float)(positions ? positions[t]
                                           : (int32_t)(t + position_offset));
        if (Q && t < q_seq)
            rotate_vector(Q + (bh * q_seq + t) * head_dim, head_dim, position,
                          theta, sc, interleaved != 0);
        if (K && t < k_seq)
            rotate_vector(K + (bh * k_seq + t) * head_dim, head_dim, position,
                          theta, sc, interleaved != 0);
    }
}

/* SwiGLU: AVX2 src/kernels/llm.cpp:289-306 (exp256 lanes), scalar :240-246. */
void oracle_swiglu(const float *gate, const float *up, float *Y,
                   uint64_t count, float alpha, int form)
{
    float a = alpha == 0.0f ? 1.0f : alpha;
    for (uint64_t i = 0; i < count; ++i) {
        float g = gate[i];
        if (form == ORACLE_FORM_AVX2) {
            float s = g / (1.0f + exp256_lane(-g));
            Y[i] = (s * up[i]) * a;
        } else {
            Y[i] = silu_f(g, ORACLE_FORM_SCALAR) * up[i] * a;
        }
    }
}

/* ADD: AVX2 src/kernels/llm.cpp:256-271 fma(x, alpha, y*beta); scalar :223-230. */
void oracle_add(const float *A, const float *B, float *Y, uint64_t count,
                float alpha, float beta, int form)
{
    int dflt = alpha == 0.0f && beta == 0.0f;
    float al = dflt ? 1.0f : alpha;
    float be = dflt ? 1.0f : beta;
    for (uint64_t i = 0; i < count; ++i)
        Y[i] = form == ORACLE_FORM_AVX2 ? fmaf(A[i], al, B[i] * be)
                                        : al * A[i] + be * B[i];
}

/* attention_range, src/kernels/llm.cpp:442-546: 16-query x 64-key blocks,
 * online softmax with fast_expf (the function is compiled without FMA, so the
 * scalar form), dot products and V accumulation through the AVX2 helpers. */
void oracle_attention(const float *Q, const float *K, const float *V,
                      const float *mask, float *O, uint32_t batch,
                      uint32_t heads, uint32_t seq_q, uint32_t seq_k,
                      uint32_t head_dim, uint32_t causal, float scale_in)
{
    enum { BQ = 16, BK = 64 };
    const uint32_t D = head_dim;
    const float scale = scale_in > 0.0f ? scale_in : 1.0f / sqrtf((float)D);
    const uint32_t causal_offset = seq_k > seq_q ? seq_k - seq_q : 0;
    float *scores = (float *)malloc(sizeof(float) * BQ * BK);
    float *acc = (float *)malloc(sizeof(float) * BQ * D);
    float m[BQ], l[BQ];
    if (!scores || !acc) { free(scores); free(acc); return; }
    for (uint64_t bh = 0; bh < (uint64_t)batch * heads; ++bh) {
        const float *Qh = Q + bh * seq_q * D;
        const float *Kh = K + bh * seq_k * D;
        const float *Vh = V + bh * seq_k * D;
        const float *Mh = mask ? mask + bh * seq_q * seq_k : NULL;
        float *Oh = O + bh * seq_q * D;
        for (uint32_t q0 = 0; q0 < seq_q; q0 += BQ) {
            uint32_t qc = seq_q - q0 < BQ ? seq_q - q0 : BQ;
            for (uint32_t i = 0; i < qc; ++i) {
                m[i] = -INFINITY;
                l[i] = 0.0f;
                memset(acc + (size_t)i * D, 0, sizeof(float) * D);
            }
            for (uint32_t k0 = 0; k0 < seq_k; k0 += BK) {
                uint32_t kc = seq_k - k0 < BK ? seq_k - k0 : BK;
                for (uint32_t i = 0; i < qc; ++i) {
                    uint32_t qi = q0 + i;
                    for (uint32_t j = 0; j < kc; ++j) {
                        uint32_t ki = k0 + j;
                        float s;
                        if (causal && ki > qi + causal_offset) {
                            s = -INFINITY;
                        } else {
                            s = dot_avx2(Qh + (size_t)qi * D, Kh + (size_t)ki * D, D) * scale;
                            if (Mh) s += Mh[(size_t)qi * seq_k + ki];
                        }
                        scores[i * BK + j] = s;
                    }
                }
                for (uint32_t i = 0; i < qc; ++i) {
                    float bmax = -INFINITY;
                    for (uint32_t j = 0; j < kc; ++j)
                        bmax = bmax < scores[i * BK + j] ? scores[i * BK + j] : bmax;
                    if (!isfinite(bmax)) continue;
                    float nm = m[i] < bmax ? bmax : m[i];
                    float alpha = oracle_fast_expf(m[i] - nm, ORACLE_FORM_SCALAR);
                    float sum_p = 0.0f;
                    for (uint32_t j = 0; j < kc; ++j) {
                        float p = oracle_fast_expf(scores[i * BK + j] - nm, ORACLE_FORM_SCALAR);
                        scores[i * BK + j] = p;
                        sum_p += p;
                    }
                    l[i] = l[i] * alpha + sum_p;
                    float *row = acc + (size_t)i * D;
                    for (uint32_t d = 0; d < D; ++d) row[d] *= alpha;
                    for (uint32_t j = 0; j < kc; ++j) {
                        float p = scores[i * BK + j];
                        if (p == 0.0f) continue;
                        const float *v = Vh + (size_t)(k0 + j) * D;
                        for (uint32_t d = 0; d < D; ++d) row[d] = fmaf(v[d], p, row[d]);
                    }
                    m[i] = nm;
                }
            }
            for (uint32_t i = 0; i < qc; ++i) {
                float inv = l[i] > 0.0f ? 1.0f / l[i] : 0.0f;
                for (uint32_t d = 0; d < D; ++d)
                    Oh[(size_t)(q0 + i) * D + d] = acc[(size_t)i * D + d] * inv;
            }
        }
    }
    free(scores);
    free(acc);
}

/* ------------------------------------------------------------------------- */
/* MATMUL_F32 (src/kernels/kernels.cpp:19-331,480-520;                        */
/*             src/core/scheduler.cpp:95-207,208-262,274-352)                 */
/* ------------------------------------------------------------------------- */

/* tile_geometry for F32 (int8 = false), src/core/scheduler.cpp:95-207.  The
 * reference's tile sizes depend on its thread count, its tile defaults and
 * VNPU_PACK; which kernel computes an output element, and so the rounding it
 * sees, depends on the tile it falls in. */
void oracle_f32_tile_geometry(uint32_t unit, uint32_t M, uint32_t N,
                              uint32_t threads, uint32_t tile_m,
                              uint32_t tile_k, uint32_t tile_n, int pack_b,
                              uint32_t *tm_out, uint32_t *tk_out,
                              uint32_t *tn_out)
{
    uint32_t tm = tile_m ? tile_m : 1, tk = tile_k ? tile_k : 1;
    uint32_t tn = tile_n ? tile_n : 1;
    const uint32_t units = threads ? threads : 1;
    const int voodoo = unit == 1 || unit == 0;
    if (M <= 8 && voodoo) {
        /* decode rows: one row block; F32 keeps the 32..64 column tile */
        tm = M;
        tn = tn < 32 ? 32 : (tn > 64 ? 64 : tn);
        if (tn > N) tn = N;
        goto done;
    }
    if (pack_b && voodoo && M >= 3 && (N + 63) / 64 >= 2 * units) {
        tm = M;
        tn = 64;
        goto done;
    }
    if (unit == 2) {            /* WILDCAT */
        if (tm > 32) tm = 32;
        if (tn > 64) tn = 64;
        if (tk > 128) tk = 128;
    } else if (unit == 3) {     /* CELL */
        if (tm > 16) tm = 16;
        if (tn > 64) tn = 64;
        if (tk > 64) tk = 64;
    }
    {
        const uint64_t target = (uint64_t)units * 64;
        uint64_t tiles = (uint64_t)((M + tm - 1) / tm) * ((N + tn - 1) / tn);
        while (tiles > target && (tm < M || tn < N)) {
            if (tm < M) tm = 2 * tm < M ? 2 * tm : M;
            if (tn < N) tn = 2 * tn < N ? 2 * tn : N;
            tiles = (uint64_t)((M + tm - 1) / tm) * ((N + tn - 1) / tn);
        }
    }
done:
    *tm_out = tm;
    *tk_out = tk;
    *tn_out = tn;
}

typedef struct {
    const float *A, *B, *bias;
    float *C;
    uint32_t K, lda, ldb, ldc, trans_a, trans_b, epilogue;
    float alpha, beta;
} F32Op;

static float f32_a(const F32Op *p, uint32_t m, uint32_t k)
{
    return p->trans_a ? p->A[(size_t)k * p->lda + m] : p->A[(size_t)m * p->lda + k];
}

static float f32_b(const F32Op *p, uint32_t k, uint32_t n)
{
    return p->trans_b ? p->B[(size_t)n * p->ldb + k] : p->B[(size_t)k * p->ldb + n];
}

/* store_c, src/kernels/kernels.cpp:43-50: alpha*v, + bias, + beta*C,
 * epilogue.  How GCC fuses it depends on the kernel it is inlined into:
 *   F32_STORE_BLOCK  - register blocks and row stream: alpha*v+bias and
 *                      beta*C+out both fused
 *   F32_STORE_PANEL  - first K panel of the packed tile, and the B^T dot
 *                      kernel: bias added unfused, beta*C+out fused
 *   F32_STORE_SCALAR - scalar / Cell kernels: every step rounded. */
enum { F32_STORE_BLOCK = 0, F32_STORE_PANEL = 1, F32_STORE_SCALAR = 2, F32_STORE_DOT = 3 };

static float f32_store(const F32Op *p, uint32_t m, uint32_t n, float v, int store)
{
    float *dst = p->C + (size_t)m * p->ldc + n;
    float out;
    if (p->bias && store == F32_STORE_BLOCK) out = fmaf(p->alpha, v, p->bias[n]);
    else if (p->bias) out = p->alpha * v + p->bias[n];
    else out = p->alpha * v;
    if (p->beta != 0.0f)
        out = store >= F32_STORE_SCALAR ? out + p->beta * *dst : fmaf(p->beta, *dst, out);
    return oracle_epilogue(out, p->epilogue,
                           store == F32_STORE_SCALAR ? ORACLE_FORM_SCALAR : ORACLE_FORM_AVX2);
}

enum { F32_FMA = 0, F32_CHUNKED = 1, F32_UNFUSED = 2, F32_NT8 = 3 };

/* One output element in the given accumulation form. */
static void f32_element(const F32Op *p, uint32_t m, uint32_t n, int kind)
{
    float *dst = p->C + (size_t)m * p->ldc + n;
    if (kind == F32_UNFUSED) {       /* scalar tile :65-76, Cell tile :409-454 */
        float acc = 0.0f;
        for (uint32_t k = 0; k < p->K; ++k) acc = acc + f32_a(p, m, k) * f32_b(p, k, n);
        *dst = f32_store(p, m, n, acc, F32_STORE_SCALAR);
    } else if (kind == F32_NT8) {    /* B^T dot products :331-352 */
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        uint32_t k = 0;
        for (; k + 8 <= p->K; k += 8)
            for (int l = 0; l < 8; ++l)
                lane[l] = fmaf(f32_a(p, m, k + l), f32_b(p, k + l, n), lane[l]);
        float dot = hsum8(lane);
        /* The scalar tail as GCC -O3 compiles it: whole groups of four take
         * one SSE multiply and in-order unfused adds, the last 0-3 terms
         * fuse (checked for every tail length 1-7 against the reference). */
        const uint32_t quad_end = k + (p->K - k) / 4 * 4;
        for (; k < quad_end; ++k) dot = dot + f32_a(p, m, k) * f32_b(p, k, n);
        for (; k < p->K; ++k) dot = fmaf(f32_a(p, m, k), f32_b(p, k, n), dot);
        *dst = f32_store(p, m, n, dot, F32_STORE_PANEL);
    } else if (kind == F32_CHUNKED) { /* packed panel tile :241-329, kc = 128 */
        for (uint32_t k0 = 0; k0 < p->K; k0 += 128) {
            const uint32_t k1 = p->K - k0 < 128 ? p->K : k0 + 128;
            float part = 0.0f;
            for (uint32_t k = k0; k < k1; ++k) part = fmaf(f32_a(p, m, k), f32_b(p, k, n), part);
            *dst = k0 == 0 ? f32_store(p, m, n, part, F32_STORE_PANEL)
                           : fmaf(p->alpha, part, *dst);
        }
    } else {                         /* register blocks :167-239, row stream :98-145 */
        float acc = 0.0f;
        for (uint32_t k = 0; k < p->K; ++k) acc = fmaf(f32_a(p, m, k), f32_b(p, k, n), acc);
        *dst = f32_store(p, m, n, acc, F32_STORE_BLOCK);
    }
}

/* Which form computes (m, n) of a tile, gemm_f32_dispatch_tile :480-520. */
static int f32_kind(uint32_t unit, int avx2, int pack_b, uint32_t trans_a,
                    uint32_t trans_b, uint32_t m0, uint32_t rows, uint32_t n0,
                    uint32_t cols, uint32_t m)
{
    (void)n0;
    if (unit == 3 || !avx2 || trans_a) return F32_UNFUSED;
    if (trans_b) return F32_NT8;
    if (pack_b && cols % 32 == 0 && rows >= 3 &&
        (uint64_t)128 * cols * sizeof(float) <= 256u * 1024u + 64u)
        return m < m0 + rows / 3 * 3 ? F32_CHUNKED : F32_FMA;
    return F32_FMA;
}

void oracle_matmul_f32(const float *A, const float *B, const float *bias,
                       float *C, uint32_t M, uint32_t K, uint32_t N,
                       uint32_t lda, uint32_t ldb, uint32_t ldc,
                       uint32_t trans_a, uint32_t trans_b, float alpha,
                       float beta, uint32_t epilogue, uint32_t unit,
                       const uint8_t *tile_mask, uint32_t mask_tile_m,
                       uint32_t mask_tile_n, uint32_t threads,
                       uint32_t tile_m, uint32_t tile_k, uint32_t tile_n,
                       int pack_b, int avx2)
{
    F32Op p;
    p.A = A; p.B = B; p.bias = bias; p.C = C;
    p.K = K;
    p.lda = lda ? lda : (trans_a ? M : K);
    p.ldb = ldb ? ldb : (trans_b ? K : N);
    p.ldc = ldc ? ldc : N;
    p.trans_a = trans_a; p.trans_b = trans_b;
    p.alpha = alpha == 0.0f ? 1.0f : alpha;
    p.beta = beta;
    p.epilogue = epilogue;
    uint32_t tm, tk, tn;
    oracle_f32_tile_geometry(unit, M, N, threads, tile_m, tile_k, tile_n, pack_b, &tm, &tk, &tn);
    const uint32_t mt = (M + tm - 1) / tm, nt = (N + tn - 1) / tn;
    for (uint32_t mi = 0; mi < mt; ++mi) {
        const uint32_t m0 = mi * tm, rows = M - m0 < tm ? M - m0 : tm;
        for (uint32_t ni = 0; ni < nt; ++ni) {
            const uint32_t n0 = ni * tn, cols = N - n0 < tn ? N - n0 : tn;
            int cull = 0;
            if (tile_mask && mask_tile_m && mask_tile_n) {   /* :234-243 */
                uint32_t mm = (uint32_t)(((uint64_t)mi * mask_tile_m) / mt);
                uint32_t nn = (uint32_t)(((uint64_t)ni * mask_tile_n) / nt);
                if (mm > mask_tile_m - 1) mm = mask_tile_m - 1;
                if (nn > mask_tile_n - 1) nn = mask_tile_n - 1;
                cull = tile_mask[(size_t)mm * mask_tile_n + nn] == 0;
            }
            for (uint32_t m = m0; m < m0 + rows; ++m) {
                for (uint32_t n = n0; n < n0 + cols; ++n) {
                    if (cull) {                              /* zero_c_tile :52-62 */
                        float *dst = C + (size_t)m * p.ldc + n;
                        float out = bias ? bias[n] : 0.0f;
                        if (beta != 0.0f) out = out + beta * *dst;
                        *dst = oracle_epilogue(out, epilogue, ORACLE_FORM_SCALAR);
                        continue;
                    }
                    f32_element(&p, m, n, f32_kind(unit, avx2, pack_b, trans_a, trans_b,
                                                   m0, rows, n0, cols, m));
                }
            }
        }
    }
}
