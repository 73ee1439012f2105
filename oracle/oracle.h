/*
 * oracle.h - CPU restatement of the reference's arithmetic for the int8 GEMM
 * hot path and the decoder-block ops.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker.
 * The shipped B200 library never links, loads or calls it.
 *
 * Each function names the reference file:line it restates (paths relative to
 * the reference checkout).  The restatement is pinned two ways: against the
 * reference library itself built from its own sources (oracle/_ref, see
 * oracle/Makefile), and against committed golden vectors produced by that
 * build (tests/golden/).
 *
 * Floating-point "forms": the reference is compiled with -ffp-contract=fast,
 * and its AVX2 kernels carry target("avx2,fma"), so GCC fuses some a*b+c into
 * one FMA there while the scalar kernels (no FMA available) never fuse.
 *   ORACLE_FORM_AVX2   - the fusions GCC performs in the AVX2 register-block
 *                        kernels (bias add and polynomial both fused)
 *   ORACLE_FORM_SCALAR - plain IEEE operations, no fusion
 *   ORACLE_FORM_STREAM - the AVX2 rank-1 / rank-R decode streams: bias added
 *                        unfused, polynomial fused (MATMUL_I8 epilogue only)
 * This file is built with -ffp-contract=off, so each fmaf() below is the only
 * fusion that happens.
 */
#ifndef VNPU_ORACLE_H
#define VNPU_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_FORM_AVX2 = 0, ORACLE_FORM_SCALAR = 1, ORACLE_FORM_STREAM = 2 };

/* fast_expf (src/internal.h:87-108) in the given form. */
float oracle_fast_expf(float x, int form);
/* apply_epilogue (src/internal.h:110-136): NONE/RELU/SILU/GELU_TANH/GELU_ERF. */
float oracle_epilogue(float v, uint32_t epilogue, int form);

/* int32 accumulators of A(MxK, lda) . B(KxN row-major, ldb) into acc (MxN). */
void oracle_gemm_i8_acc(const int8_t *A, uint32_t lda, const int8_t *B,
                        uint32_t ldb, int32_t *acc, uint32_t M, uint32_t K,
                        uint32_t N);

/* MATMUL_I8 (src/kernels/kernels.cpp:526-550 store_i8_c + scalar tile).
 * B is the canonical row-major KxN int8 matrix the reference keeps in
 * vnpu_packed_weights::original; scale_b NULL means 1.0 (the reference pads
 * its scales with 1.0f, src/core/scheduler.cpp:795). */
void oracle_matmul_i8(const int8_t *A, uint32_t lda, const int8_t *B,
                      const float *scale_a, const float *scale_b,
                      const float *bias, float *C, uint32_t ldc, uint32_t M,
                      uint32_t K, uint32_t N, uint32_t epilogue, int form);

/* MATMUL_I8 tile sizes (src/core/scheduler.cpp:75-207, int8 branch) for a
 * reference device with `threads` workers, tile defaults tile_m / tile_n,
 * VNPU_PACK = pack_b and an L2 of l2_bytes (0: the reference's 512 KiB
 * default); unit as resolved by choose_unit (1 VOODOO, 2 WILDCAT, 3 CELL). */
void oracle_i8_tile_geometry(uint32_t unit, uint32_t M, uint32_t N,
                             uint32_t threads, uint32_t tile_m,
                             uint32_t tile_n, int pack_b, uint64_t l2_bytes,
                             uint32_t *tm, uint32_t *tn);

/* ORACLE_FORM_* of output element (m, n) of an M x K x N MATMUL_I8 on tiles
 * tm x tn (gemm_i8_dispatch_tile, src/kernels/kernels.cpp:922-978). */
int oracle_i8_element_form(uint32_t unit, int avx2, int pack_b, uint32_t K,
                           uint32_t M, uint32_t N, uint32_t tm, uint32_t tn,
                           uint32_t m, uint32_t n);

/* The form of every element (M x N int32, row-major) of the same product. */
void oracle_i8_form_map(uint32_t unit, uint32_t M, uint32_t K, uint32_t N,
                        uint32_t threads, uint32_t tile_m, uint32_t tile_n,
                        int pack_b, int avx2, uint64_t l2_bytes, int32_t *forms);

/* MATMUL_I8 exactly as the reference device described by threads /
 * tile_m, tile_n / pack_b / avx2 (0 = VNPU_FORCE_ISA=scalar) / l2_bytes
 * computes it with no flags: each element in its kernel's form.  unit 0
 * (AUTO) resolves to VOODOO. */
void oracle_matmul_i8_device(const int8_t *A, uint32_t lda, const int8_t *B,
                             const float *scale_a, const float *scale_b,
                             const float *bias, float *C, uint32_t ldc,
                             uint32_t M, uint32_t K, uint32_t N,
                             uint32_t epilogue, uint32_t unit,
                             uint32_t threads, uint32_t tile_m,
                             uint32_t tile_n, int pack_b, int avx2,
                             uint64_t l2_bytes);

/* Dequant epilogue for one accumulator (store_i8_c). */
float oracle_dequant(int32_t acc, float sa, float sb, const float *bias_n,
                     uint32_t epilogue, int form);

/* QUANTIZE_I8 (src/kernels/llm.cpp:387-436, src/core/scheduler.cpp:430-473).
 * axis 0 = per row, 1 = per column, 2 = per tensor. */
int oracle_quantize_i8(const float *X, int8_t *Y, float *scales, uint64_t rows,
                       uint64_t cols, uint32_t axis);

/* PACK_WEIGHTS_I8 column sums (src/core/scheduler.cpp:783-805). */
void oracle_column_sums(const int8_t *B, uint32_t K, uint32_t N, uint32_t ldb,
                        uint32_t trans_b, int32_t *sums, int8_t *canonical);

/* RMSNORM_F32 (src/kernels/llm.cpp:64-108). */
void oracle_rmsnorm(const float *X, const float *W, float *Y, uint32_t rows,
                    uint32_t cols, float eps, int form);

/* ROPE_F32 (src/kernels/llm.cpp:188-217 rotate_vector, :576-602 tokens). */
void oracle_rope(float *Q, float *K, const int32_t *positions, uint32_t batch,
                 uint32_t heads, uint32_t q_seq, uint32_t k_seq,
                 uint32_t head_dim, uint32_t position_offset,
                 uint32_t interleaved, float theta_base, float scaling);

/* SWIGLU_F32 (src/kernels/llm.cpp:240-246 scalar, :289-306 AVX2). */
void oracle_swiglu(const float *gate, const float *up, float *Y,
                   uint64_t count, float alpha, int form);

/* ADD_F32 (src/kernels/llm.cpp:223-230 scalar, :256-271 AVX2). */
void oracle_add(const float *A, const float *B, float *Y, uint64_t count,
                float alpha, float beta, int form);

/* ATTENTION_F32 (src/kernels/llm.cpp:442-546 attention_range). */
void oracle_attention(const float *Q, const float *K, const float *V,
                      const float *mask, float *O, uint32_t batch,
                      uint32_t heads, uint32_t seq_q, uint32_t seq_k,
                      uint32_t head_dim, uint32_t causal, float scale);

/* MATMUL_F32 tile sizes (src/core/scheduler.cpp:95-207, F32 branch) for a
 * reference device with `threads` worker threads and tile defaults
 * tile_m/k/n (128/128/64 on AVX2 hosts, 32/64/32 scalar); unit is the unit
 * choose_unit resolved (1 VOODOO, 2 WILDCAT, 3 CELL). */
void oracle_f32_tile_geometry(uint32_t unit, uint32_t M, uint32_t N,
                              uint32_t threads, uint32_t tile_m,
                              uint32_t tile_k, uint32_t tile_n, int pack_b,
                              uint32_t *tm, uint32_t *tk, uint32_t *tn);

/* MATMUL_F32 (src/kernels/kernels.cpp:19-331,480-520) as the reference
 * device described by threads / tile_m,k,n / pack_b (VNPU_PACK) / avx2
 * (0 = VNPU_FORCE_ISA=scalar) computes it, element by element in the
 * rounding of the kernel that owns the element's tile. */
void oracle_matmul_f32(const float *A, const float *B, const float *bias,
                       float *C, uint32_t M, uint32_t K, uint32_t N,
                       uint32_t lda, uint32_t ldb, uint32_t ldc,
                       uint32_t trans_a, uint32_t trans_b, float alpha,
                       float beta, uint32_t epilogue, uint32_t unit,
                       const uint8_t *tile_mask, uint32_t mask_tile_m,
                       uint32_t mask_tile_n, uint32_t threads,
                       uint32_t tile_m, uint32_t tile_k, uint32_t tile_n,
                       int pack_b, int avx2);

#ifdef __cplusplus
}
#endif

#endif /* VNPU_ORACLE_H */
