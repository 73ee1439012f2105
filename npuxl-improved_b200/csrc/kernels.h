// kernels.h - host-side launch interface of the sm_100a kernels.
//
// The runtime (runtime.cpp) validates a command, resolves its pointers to
// device memory and calls one of these; each enqueues its kernel(s) on
// ctx.stream and returns the launch status.  Nothing here synchronises.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace vnpu_b200 {

// Error codes written (atomicOr) into the per-stream device error word.
enum DeviceError : uint32_t {
    kErrNone = 0,
    kErrWaitTimeout = 1u << 0,   // an mbarrier / flag wait ran out of time
    kErrBadConfig = 1u << 1,     // a kernel saw a launch shape it cannot run
    kErrTmemAlloc = 1u << 2,     // tensor memory allocation returned nonsense
};

// Dequant epilogue forms (vnpu_b200.h: block / stream / scalar); kFormMixed
// marks a FormMap whose form varies from element to element.
enum EpiForm : uint32_t { kFormBlock = 0, kFormStream = 1, kFormScalar = 2, kFormMixed = 3 };

// The rounding form of each element of a MATMUL_I8 output.  The reference
// device rounds an element's dequant epilogue in the form of the CPU kernel
// that owns its tile (src/kernels/kernels.cpp:922-978), and its tile grid
// (src/core/scheduler.cpp:75-207) depends on M, N, its thread count, its tile
// defaults and VNPU_PACK.  runtime.cpp builds the map from the same rules:
// either one form for the whole output (form != kFormMixed, the usual case),
// or a 16-entry table of 2-bit forms indexed by the element's row class
// (last row tile?, the odd row of its tile?) and column class (last column
// tile?, in the tile's column tail past its last whole 32 columns?).
struct FormMap {
    uint32_t form = kFormBlock;   // every element's form, or kFormMixed
    uint32_t tm = 1, tn = 1;      // the reference's tile rows / columns
    uint32_t M = 0, N = 0;        // the whole output those tiles cover
    uint32_t col_base = 0;        // whole-output column of the launch's column 0
    uint32_t table = 0;           // form of class (row * 4 + column) at bits 2i..2i+1
    uint32_t reserved = 0;
};

struct LaunchCtx {
    cudaStream_t stream = nullptr;
    uint32_t *err = nullptr;        // per-stream device error word
    int num_sms = 148;
    uint64_t wait_limit_ns = 2000000000ull;  // bound of every device-side wait
    uint64_t *launch_counter = nullptr;      // host counter, +1 per kernel launch
};

// ---- QUANTIZE_I8 (src/kernels/llm.cpp:387-436) ------------------------------
cudaError_t quantize_rows(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                          uint64_t rows, uint64_t cols);
cudaError_t quantize_columns(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                             uint64_t rows, uint64_t cols);
// Per tensor needs a device scratch word for the running absmax (4 bytes).
cudaError_t quantize_tensor(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                            uint64_t rows, uint64_t cols, uint32_t *absmax_scratch);

// ---- PACK_WEIGHTS_I8 (src/core/scheduler.cpp:763-836) -------------------------
// B (K x N, or N x K when trans_b) with row stride ldb -> Bt[N][k_stride]
// (K-major, zero padded to k_stride) and column_sums[N].
cudaError_t pack_weights(const LaunchCtx &ctx, const int8_t *B, uint32_t K, uint32_t N,
                         uint32_t ldb, uint32_t trans_b, int8_t *Bt, uint32_t k_stride,
                         int32_t *column_sums);

// ---- MATMUL_I8 ----------------------------------------------------------------
struct MatmulI8 {
    const int8_t *A = nullptr;      // M x K, row stride lda (bytes)
    uint32_t lda = 0;
    const int8_t *Bt = nullptr;     // N x k_stride, K-major packed weights
    uint32_t k_stride = 0;
    const float *scale_a = nullptr; // M or NULL (1.0)
    const float *scale_b = nullptr; // N (device copy in the packed handle)
    const float *bias = nullptr;    // N or NULL
    float *C = nullptr;             // M x N, row stride ldc (floats)
    uint32_t ldc = 0;
    uint32_t M = 0, K = 0, N = 0;
    uint32_t epilogue = 0;
    FormMap fmap;                   // rounding form of each output element
    const CUtensorMap *tmap_b = nullptr;     // TMA map of Bt (box 128 x 256, SW128)
    const CUtensorMap *tmap_b128 = nullptr;  // same, box 128 x 128 (CTA-pair kernel)
    // Scatter mode (MATMUL_I8_SCATTER): the shard is written into ndst full
    // [M][ldd] outputs at column col_offset instead of C.
    float *dst[8] = {};
    uint32_t ndst = 0;
    uint32_t ldd = 0;
    uint32_t col_offset = 0;
    // Residual (MATMUL_I8_RESIDUAL): C = R + out, R [M][ldr]; taken only by
    // matmul_i8_split_residual.
    const float *R = nullptr;
    uint32_t ldr = 0;
    // The residual GEMVs (M = 1) only: *advance_pos += advance once the
    // previous kernels of the stream are complete.
    int32_t *advance_pos = nullptr;
    int32_t advance = 0;
};

enum class MatmulKernel { kTcgen05, kGemv, kSimt };

// MATMUL_I8 with the residual add (p.R) folded into the split-K finish
// kernel of the CTA-pair GEMM; cudaErrorNotSupported, with nothing launched,
// when the shape does not take that path (the caller then adds separately).
cudaError_t matmul_i8_split_residual(const LaunchCtx &ctx, const MatmulI8 &p);

// MATMUL_I8 with the scatter epilogue (CTA-pair kernel; TMA-aligned A required).
cudaError_t matmul_i8_scatter(const LaunchCtx &ctx, const MatmulI8 &p);

// Which kernel a shape goes to (pure function of the arguments).
MatmulKernel choose_matmul_kernel(uint32_t M, uint32_t K, uint32_t N, uint32_t lda,
                                  const void *A);
const char *matmul_kernel_name(MatmulKernel k);
// Kernel the most recent MATMUL_I8 launch used (any thread, any device).
const char *last_matmul_kernel();

cudaError_t matmul_i8(const LaunchCtx &ctx, const MatmulI8 &p);
// The M <= 2 GEMV with each warp's column landed in shared memory before the
// programmatic wait (gemv_stream.cu): 16-byte aligned A and lda, 8 x
// cols_per_warp x k_stride bytes of shared memory per CTA (<= 200 KiB).
// R: C = R + out.
bool gemv_stream_supported(const MatmulI8 &p, uint32_t cols_per_warp);
// The gate/up GEMV (M <= 2) with the SwiGLU epilogue: B is [K][2I].
cudaError_t matmul_i8_swiglu_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p, float *Y,
                                         uint32_t ldy, uint32_t I, float alpha);
// MATMUL_I8 of a [K][2I] gate/up weight followed by SWIGLU_F32 of its halves
// into Y (rows x I, row stride ldy): the SwiGLU in the GEMM's epilogue where
// the CTA-pair kernel or the streaming GEMV takes the shape, else MATMUL_I8
// into stream-ordered scratch and swiglu_rows.
cudaError_t matmul_i8_swiglu(const LaunchCtx &ctx, const MatmulI8 &p, float *Y, uint32_t ldy,
                             float alpha);
// M <= 8 with the products on mma.sync (gemv_stream.cu); groups = 8-column
// groups per CTA (1, 2 or 4).
bool gemv_mma_supported(const MatmulI8 &p);
bool gemv_mma_preferred(const MatmulI8 &p);
cudaError_t matmul_i8_gemv_mma(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                               uint32_t ldr, uint32_t groups);
cudaError_t matmul_i8_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p, const float *R = nullptr,
                                  uint32_t ldr = 0);

// Individual kernels (tests pin each against the oracle).
cudaError_t matmul_i8_tcgen05(const LaunchCtx &ctx, const MatmulI8 &p);
cudaError_t matmul_i8_gemv(const LaunchCtx &ctx, const MatmulI8 &p);
cudaError_t matmul_i8_simt(const LaunchCtx &ctx, const MatmulI8 &p);

// TMA tensor maps (driver entry point resolved once through the runtime).
bool encode_tmap_kmajor_i8(CUtensorMap *map, const void *base, uint64_t k_extent,
                           uint64_t rows, uint64_t row_stride_bytes, uint32_t box_k,
                           uint32_t box_rows);
bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t dim0,
                    uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swizzle);

// QKV projection epilogue (VNPU_B200_OP_QKV_ROPE_APPEND): where the rotated
// Q/K and the V of each token go.  Token t has position (*position or
// position_offset) + t, used for the rotation and as its cache slot.
struct QkvRope {
    float *Q = nullptr;         // [heads][T][head_dim]
    float *K_out = nullptr;     // [heads][T][head_dim] or NULL
    float *V_out = nullptr;     // [heads][T][head_dim] or NULL
    float *K_cache = nullptr;   // [heads][capacity][head_dim]
    float *V_cache = nullptr;
    float *mask = nullptr;      // [heads][capacity] or NULL
    const int32_t *position = nullptr;
    uint32_t heads = 0, head_dim = 0, capacity = 0, position_offset = 0;
    float scaling = 1.0f;
    const float *inv_freq = nullptr;   // host, head_dim/2 entries (ROPE_F32's table)
};
// One token (M = 1): the streaming GEMV with the rotation pairs in one warp.
cudaError_t qkv_rope_append_gemv(const LaunchCtx &ctx, const MatmulI8 &p, const QkvRope &q);
// The same on the shared-memory streaming GEMV (gemv_stream.cu).
cudaError_t qkv_rope_append_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p, const QkvRope &q);
// Any T: C is the MATMUL_I8 output [T][3*heads*head_dim] already computed.
cudaError_t qkv_split_rope_append(const LaunchCtx &ctx, const float *C, uint32_t T,
                                  const QkvRope &q);
// C = R + MATMUL_I8 for M = 1 in the GEMV's epilogue.
cudaError_t matmul_i8_gemv_residual(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                                    uint32_t ldr);

// ---- MATMUL_F32 (src/kernels/kernels.cpp:19-352,480-520) -----------------------
// Accumulation form of the reference kernel a command's elements take
// (gemm_f32.cu has the rules).
enum F32Mode : uint32_t { kF32Block = 0, kF32Unfused = 1, kF32Dot8 = 2 };

struct MatmulF32 {
    const float *A = nullptr;       // M x K (K x M when trans_a), row stride lda
    const float *B = nullptr;       // K x N (N x K when trans_b), row stride ldb
    const float *bias = nullptr;    // N or NULL
    float *C = nullptr;             // M x N, row stride ldc; read when beta != 0
    uint32_t M = 0, K = 0, N = 0, lda = 0, ldb = 0, ldc = 0;
    uint32_t trans_a = 0, trans_b = 0;
    float alpha = 1.0f, beta = 0.0f;
    uint32_t epilogue = 0;
    uint32_t mode = kF32Block;
    // The reference's tile geometry for this GEMM (tile_m x tile_n grid) and
    // whether its packed-panel kernel may own tiles (AVX2, VNPU_PACK, NN).
    uint32_t tile_m = 1, tile_n = 1;
    uint32_t packed = 0;
    const uint8_t *mask = nullptr;  // Wildcat cull mask, mask_m x mask_n bytes
    uint32_t mask_m = 0, mask_n = 0;
};

cudaError_t matmul_f32(const LaunchCtx &ctx, const MatmulF32 &p);

// ---- decoder-block ops (src/kernels/llm.cpp) -----------------------------------
cudaError_t rmsnorm(const LaunchCtx &ctx, const float *X, const float *W, float *Y,
                    uint32_t rows, uint32_t cols, float eps);
// inv_freq: host-computed 1/theta^(2j/dim) (or j/dim interleaved), head_dim/2 entries.
// RMSNORM_F32 then QUANTIZE_I8 per row in one pass (Y may be NULL).
cudaError_t rmsnorm_quantize(const LaunchCtx &ctx, const float *X, const float *W, float *Y,
                             int8_t *Q, float *scales, uint32_t rows, uint32_t cols, float eps);
// SWIGLU_F32 then QUANTIZE_I8 per row in one pass (Y may be NULL); gate and
// up rows are ld elements apart (ld >= cols), Y, Q dense.
cudaError_t swiglu_quantize(const LaunchCtx &ctx, const float *gate, const float *up, float *Y,
                            int8_t *Q, float *scales, uint32_t rows, uint32_t cols, uint32_t ld,
                            float alpha);
// KV-cache append (VNPU_B200_OP_KV_APPEND); position may be a device pointer.
cudaError_t kv_append(const LaunchCtx &ctx, const float *K, const float *V, float *K_cache,
                      float *V_cache, float *mask, const int32_t *position, uint32_t heads,
                      uint32_t T, uint32_t head_dim, uint32_t capacity, uint32_t position_offset);
cudaError_t rope(const LaunchCtx &ctx, float *Q, float *K, const int32_t *positions,
                 uint32_t batch, uint32_t heads, uint32_t q_seq, uint32_t k_seq,
                 uint32_t head_dim, uint32_t position_offset, uint32_t interleaved,
                 float scaling, const float *inv_freq_host);
// The decoder block driver's device-side position (set or advance) and the
// -inf fill of its cache mask.
cudaError_t block_position(const LaunchCtx &ctx, int32_t *pos, int32_t value, bool advance);
cudaError_t fill_neg_inf(const LaunchCtx &ctx, float *p, uint64_t n);
// Y[r][j] = swiglu(C[r][j], C[r][I + j]) * alpha, the SWIGLU_F32 expression.
cudaError_t swiglu_rows(const LaunchCtx &ctx, const float *C, uint32_t ldc, float *Y, uint32_t ldy,
                        uint32_t rows, uint32_t I, float alpha);
cudaError_t swiglu(const LaunchCtx &ctx, const float *gate, const float *up, float *Y,
                   uint64_t count, float alpha);
cudaError_t add(const LaunchCtx &ctx, const float *A, const float *B, float *Y, uint64_t count,
                float alpha, float beta);
// o_token_major: O as [batch][seq_q][heads][head_dim] instead of the
// reference's [batch][heads][seq_q][head_dim] (VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR).
cudaError_t attention(const LaunchCtx &ctx, const float *Q, const float *K, const float *V,
                      const float *mask, float *O, uint32_t batch, uint32_t heads,
                      uint32_t seq_q, uint32_t seq_k, uint32_t head_dim, uint32_t causal,
                      float scale, bool o_token_major = false);

// ---- device-wait self test -------------------------------------------------------
cudaError_t wait_timeout_probe(const LaunchCtx &ctx, const uint32_t *flag, uint64_t limit_ns);

}  // namespace vnpu_b200
