/*
 * vnpu_b200.h - B200 extensions to the vnpu v1 ABI.
 *
 * Everything here is additive, in the way the reference's ABI rules allow
 * (reference include/vnpu.h:14: "new capabilities are added via opcodes/flags,
 * not by changing v1 structs").  An engine that only knows vnpu.h never needs
 * this header.
 */
#ifndef VNPU_B200_H
#define VNPU_B200_H

#include "vnpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Dequant epilogue rounding of MATMUL_I8 and the int8 B200 opcodes.  With a
 * bias and/or an activation, the reference's outputs differ in the last bits
 * between its own CPU kernels, and which kernel computes an element depends
 * on the tile it falls in (src/core/scheduler.cpp:75-207 tile grid from M, N,
 * the worker-thread count, the tile defaults and VNPU_PACK;
 * src/kernels/kernels.cpp:922-978 kernel per tile):
 *
 *   block    out = fmaf(float(acc)*sa, sb, bias), activation polynomial
 *            evaluated with FMAs: the register-block AVX2 kernels (2x32 /
 *            1x32 blocks, packed panel; kernels.cpp:634-701,779-869).
 *   stream   out = (float(acc)*sa)*sb + bias (two roundings), FMA
 *            polynomial: the rank-1 / rank-R decode streams
 *            (kernels.cpp:581-632,702-767) and the column tail of a row pair.
 *   scalar   no fused operation anywhere: the column tail of a single row,
 *            the Cell unit, VNPU_FORCE_ISA=scalar and VNPU_MODE=reference
 *            (kernels.cpp:537-550).
 *
 * By default every element takes the form the reference device of the same
 * configuration (vnpu_config_t.num_threads, else the host's physical cores;
 * tile_m / tile_n; VNPU_PACK; VNPU_FORCE_ISA / VNPU_MODE; the host L2 size)
 * gives it, so an unflagged command returns the reference's bits.  These
 * command flags (no reference counterpart) force one form for every element
 * instead; VNPU_B200_EPILOGUE=block|stream|scalar in the environment does the
 * same for devices created afterwards.  Without bias and with epilogue NONE
 * or RELU all forms are the same bits.
 */
#define VNPU_CMD_FLAG_EPI_STREAM   (1u << 8)
#define VNPU_CMD_FLAG_EPI_SCALAR   (1u << 9)
#define VNPU_CMD_FLAG_EPI_BLOCK    (1u << 11)

/*
 * ATTENTION_F32 output layout (no reference counterpart): with this flag O is
 * written token-major, [batch][seq_q][heads][head_dim], the row layout the
 * next projection reads, instead of the reference's head-major
 * [batch][heads][seq_q][head_dim] (reference include/vnpu.h attention args).
 * The values are the same bits; only their places differ.  Q, K, V and the
 * mask keep the reference's layouts.
 */
#define VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR (1u << 10)

/*
 * Fused row prologues for MATMUL_I8 (no reference counterpart; the reference
 * submits RMSNORM_F32 or SWIGLU_F32 and then QUANTIZE_I8 per row).  Opcodes
 * outside the reference's range, as its ABI rules allow (reference
 * include/vnpu.h:14); the arguments travel in vnpu_command_t.args.raw
 * (memcpy the struct there).  Q (rows x cols int8) and scales (rows f32) are
 * the bits QUANTIZE_I8 per row gives for the f32 result; Y, when not NULL,
 * receives that f32 result (the bits RMSNORM_F32 / SWIGLU_F32 give).
 * cols <= 49152.  eps <= 0 means 1e-5 and alpha == 0 means 1, as in the
 * stand-alone commands.
 */
#define VNPU_B200_OP_RMSNORM_QUANTIZE_I8  0x100u
#define VNPU_B200_OP_SWIGLU_QUANTIZE_I8   0x101u

typedef struct vnpu_b200_rmsnorm_quantize_args_t {
    const float *X;      /* rows x cols */
    const float *W;      /* cols, or NULL (1.0) */
    float *Y;            /* rows x cols f32 result, or NULL */
    int8_t *Q;           /* rows x cols */
    float *scales;       /* rows */
    uint32_t rows;
    uint32_t cols;
    float eps;
    uint32_t reserved0;
} vnpu_b200_rmsnorm_quantize_args_t;

typedef struct vnpu_b200_swiglu_quantize_args_t {
    const float *gate;   /* rows x cols, row stride ld */
    const float *up;     /* rows x cols, row stride ld */
    float *Y;            /* rows x cols f32 result (dense), or NULL */
    int8_t *Q;           /* rows x cols */
    float *scales;       /* rows */
    uint32_t rows;
    uint32_t cols;
    float alpha;
    uint32_t ld;         /* elements between rows of gate and up; 0 = cols.  gate and up
                            may be the two halves of one [rows][2*cols] GEMM output */
} vnpu_b200_swiglu_quantize_args_t;

/*
 * KV-cache append for KV-cached decoding (no reference counterpart: the
 * reference has no KV cache).  Copies head-major K and V ([heads][T][head_dim]
 * f32, as ROPE_F32 leaves them) into slots pos .. pos+T-1 of the caches
 * ([heads][capacity][head_dim]) and sets those slots of the additive mask
 * ([heads][capacity], may be NULL) to 0, so ATTENTION_F32 over the whole
 * capacity with that mask attends to the filled slots only.  pos is *position
 * (a device int32, read when the command runs: a captured graph can advance
 * it) or position_offset when position is NULL.  Slots at or past capacity are
 * not written: VNPU_ERR_INVALID_ARGUMENT when pos is known on the host, the
 * stream's device error otherwise.
 */
#define VNPU_B200_OP_KV_APPEND  0x102u

typedef struct vnpu_b200_kv_append_args_t {
    const float *K;
    const float *V;
    float *K_cache;
    float *V_cache;
    float *mask;
    const int32_t *position;
    uint32_t heads;
    uint32_t T;
    uint32_t head_dim;
    uint32_t capacity;
    uint32_t position_offset;
    uint32_t reserved0;
} vnpu_b200_kv_append_args_t;

/*
 * Column-sharded MATMUL_I8 fused with the all-gather of its output (no
 * reference counterpart; the reference's multi-device split is by rows and
 * F32 only).  The rank's shard C[:, 0:N) is written straight into every
 * destination's full output at columns col_offset .. col_offset+N-1, tile by
 * tile from the GEMM epilogue with plain stores (peer destinations over
 * NVLink), instead of a separate all-gather after the GEMM.
 *
 * dst[0..ndst-1] are device memory: this GPU's, or another GPU's mapped with
 * vnpu_b200_ipc_open (not staged).  Each is a [M][ldd] f32 matrix; ldd,
 * col_offset and the dst addresses are multiples of 4 floats / 16 bytes.
 * Other arguments as vnpu_matmul_i8_args_t (A on this GPU, TMA-aligned:
 * 16-byte aligned A and lda % 16 == 0).  A destination on another GPU is
 * complete once the writing rank's command has completed: order the readers
 * after it (a barrier across the ranks).
 */
#define VNPU_B200_OP_MATMUL_I8_SCATTER  0x103u
#define VNPU_B200_SCATTER_MAX  8

typedef struct vnpu_b200_matmul_i8_scatter_args_t {
    const int8_t *A;
    vnpu_packed_weights_t *B;
    const float *scale_a;
    const float *bias;
    float *dst[VNPU_B200_SCATTER_MAX];
    uint32_t M;
    uint32_t K;
    uint32_t N;          /* columns of this shard (the packed weights' N) */
    uint32_t lda;        /* 0 = K */
    uint32_t ldd;        /* row stride of every destination, floats */
    uint32_t col_offset; /* first destination column of this shard */
    uint32_t ndst;       /* 1 .. VNPU_B200_SCATTER_MAX */
    uint32_t epilogue;
} vnpu_b200_matmul_i8_scatter_args_t;

/*
 * QKV projection with RoPE and the KV-cache append in its epilogue (the
 * reference builds this from MATMUL_I8, a host split into head-major Q/K/V,
 * ROPE_F32 and a cache copy, tools/llm_bench.cpp:256-311).  Same bits as
 * MATMUL_I8 of A (T x K) with the packed QKV weights B (N = 3 * heads *
 * head_dim, columns [Q | K | V], each head-contiguous), then ROPE_F32
 * (non-interleaved, theta_base / scaling as vnpu_rope_f32_args_t) of the Q and
 * K parts, then VNPU_B200_OP_KV_APPEND of K and V.  Token t has position
 * p = pos + t, pos being *position (device int32, read when the command runs)
 * or position_offset when position is NULL: p is both its rotation position
 * and its cache slot.
 *   Q       [heads][T][head_dim]    rotated queries (required)
 *   K_out   [heads][T][head_dim]    rotated keys, or NULL
 *   V_out   [heads][T][head_dim]    values, or NULL
 *   K_cache, V_cache [heads][capacity][head_dim], mask [heads][capacity]
 *           (mask may be NULL): slot p of every head written, mask slot 0.
 * head_dim even, <= 512.  Slots outside the capacity are not written (the
 * stream's device error).  One kernel when T = 1 (the decode step's GEMV
 * computes each rotation pair in one warp); otherwise MATMUL_I8 plus one
 * split / rotate / append kernel.
 */
#define VNPU_B200_OP_QKV_ROPE_APPEND  0x104u

typedef struct vnpu_b200_qkv_rope_append_args_t {
    const int8_t *A;
    vnpu_packed_weights_t *B;
    const float *scale_a;
    const float *bias;
    float *Q;
    float *K_out;
    float *V_out;
    float *K_cache;
    float *V_cache;
    float *mask;
    const int32_t *position;
    uint32_t T;
    uint32_t K;
    uint32_t heads;
    uint32_t head_dim;
    uint32_t capacity;
    uint32_t position_offset;
    float theta_base;   /* <= 0: 10000 */
    float scaling;      /* <= 0: 1 */
    uint32_t epilogue;  /* MATMUL_I8 epilogue of the projection */
    uint32_t reserved0;
} vnpu_b200_qkv_rope_append_args_t;

/*
 * MATMUL_I8 plus a residual: C = R + matmul_i8(A, B) with one rounding of the
 * sum, the bits of ADD_F32 (alpha = beta = 1) of R and the MATMUL_I8 output
 * (the decoder block's x + proj, tools/llm_bench.cpp:296-326).  R may be C
 * (in place).  M <= 8 with a 16-byte aligned A runs it in the GEMV's
 * epilogue; other shapes run MATMUL_I8 into C and then the addition.
 */
#define VNPU_B200_OP_MATMUL_I8_RESIDUAL  0x105u

typedef struct vnpu_b200_matmul_i8_residual_args_t {
    const int8_t *A;
    vnpu_packed_weights_t *B;
    const float *scale_a;
    const float *bias;
    const float *R;     /* M x N residual, row stride ldr */
    float *C;
    uint32_t M;
    uint32_t K;
    uint32_t N;
    uint32_t lda;       /* 0 = K */
    uint32_t ldr;       /* 0 = N */
    uint32_t ldc;       /* 0 = N */
    uint32_t epilogue;
    uint32_t reserved0;
} vnpu_b200_matmul_i8_residual_args_t;

/*
 * Position advance (a B200 command flag; no reference counterpart).  With
 * VNPU_B200_CMD_FLAG_ADVANCE_POSITION, VNPU_B200_OP_MATMUL_I8_RESIDUAL also
 * adds advance to the device int32 *position once the stream's earlier
 * commands are complete: the decode step's position, which QKV_ROPE_APPEND
 * and KV_APPEND read, moves on in the step's last command instead of a
 * launch of its own (for one row the GEMV does it; other shapes run a
 * one-thread kernel after the product).  The fields sit at byte
 * VNPU_B200_ADVANCE_OFFSET of vnpu_command_t.args.raw, after the command's
 * own arguments.  The flag is an argument error on other commands.
 */
#define VNPU_B200_CMD_FLAG_ADVANCE_POSITION  (1u << 14)
#define VNPU_B200_ADVANCE_OFFSET             128u

typedef struct vnpu_b200_advance_t {
    int32_t *position;      /* device int32 */
    int32_t advance;
    uint32_t reserved;
} vnpu_b200_advance_t;

/*
 * The gate/up projection with its SwiGLU (no reference counterpart; the
 * reference block runs MATMUL_I8 on the [K][2I] gate/up weight, splits the
 * [T][2I] output into gate and up on the host and submits SWIGLU_F32:
 * tools/llm_bench.cpp:298-311).  B holds 2I columns (gate 0..I-1, up
 * I..2I-1); Y (M x I, row stride ldy) receives the bits SWIGLU_F32 (with
 * alpha) gives for the halves of that MATMUL_I8's output, each element of
 * which keeps the rounding form it has in the 2I-wide product.  The SwiGLU
 * runs in the GEMM's epilogue where the CTA-pair tensor-core GEMM (M > 128)
 * or the streaming decode GEMV (M <= 2) takes the shape, so the 2I-wide
 * product never reaches memory; elsewhere the product goes to stream-ordered
 * scratch first.  alpha == 0 means 1, as in SWIGLU_F32.
 */
#define VNPU_B200_OP_MATMUL_I8_SWIGLU  0x108u

typedef struct vnpu_b200_matmul_i8_swiglu_args_t {
    const int8_t *A;
    vnpu_packed_weights_t *B;   /* K x 2I */
    const float *scale_a;
    const float *bias;          /* 2I entries or NULL */
    float *Y;                   /* M x I */
    uint32_t M;
    uint32_t K;
    uint32_t N;                 /* 2I, the columns of B */
    uint32_t lda;               /* 0 = K */
    uint32_t ldy;               /* 0 = I */
    uint32_t epilogue;          /* of the MATMUL_I8, before the SwiGLU */
    float alpha;
    uint32_t reserved0;
} vnpu_b200_matmul_i8_swiglu_args_t;

/*
 * MATMUL_I8 of one column shard of a wider product (no reference
 * counterpart; the reference has no int8 multi-device split).  B holds the
 * shard's N columns, which are columns col_base .. col_base + N - 1 of an
 * M x K x n_full product; C receives the shard (M x N, row stride ldc).
 * Every element is rounded in the form the reference device gives that
 * element of the whole n_full-wide product, so shards assembled side by side
 * are the bits of one MATMUL_I8 of the whole weight.  bias holds the shard's
 * N entries.  n_full = 0 means N (a whole product).
 */
#define VNPU_B200_OP_MATMUL_I8_SHARD  0x106u

typedef struct vnpu_b200_matmul_i8_shard_args_t {
    const int8_t *A;
    vnpu_packed_weights_t *B;
    const float *scale_a;
    const float *bias;
    float *C;
    uint32_t M;
    uint32_t K;
    uint32_t N;
    uint32_t lda;       /* 0 = K */
    uint32_t ldc;       /* 0 = N */
    uint32_t epilogue;
    uint32_t n_full;    /* columns of the whole product (0 = N) */
    uint32_t col_base;  /* whole-product column of the shard's column 0 */
} vnpu_b200_matmul_i8_shard_args_t;

/*
 * Column-sharded int8 GEMM over a local cluster's devices (no reference
 * counterpart: the reference's cluster splits MATMUL_F32 rows only,
 * src/cluster/cluster.cpp:437-546).  cache_weights_i8 splits the K x N int8
 * weights B (host memory, row stride ldb; scales N floats or NULL = 1.0) by
 * columns over the cluster's devices, in proportion to their weights and in
 * multiples of 256 columns, and packs each device's shard into that
 * device's HBM.  matmul_i8 runs every device's shard in parallel
 * (VNPU_B200_OP_MATMUL_I8_SHARD; A M x K int8 with per-row scale_a, bias N
 * floats or NULL, all host memory) and places each shard's columns in C
 * (M x N f32, row stride ldc, host memory or any device's memory).  The
 * result is the bits of one vnpu_matmul_i8 of the whole weight on one device.
 * Also in the backend table's reserved[6] and reserved[7].
 */
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_cache_weights_i8(vnpu_cluster_t *cluster,
                                                              const char *key,
                                                              const int8_t *B,
                                                              const float *scales, uint32_t K,
                                                              uint32_t N, uint32_t ldb,
                                                              vnpu_weight_handle_t **out);
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_matmul_i8(vnpu_cluster_t *cluster,
                                                       vnpu_weight_handle_t *weights,
                                                       const int8_t *A, const float *scale_a,
                                                       const float *bias, float *C, uint32_t M,
                                                       uint32_t K, uint32_t N, uint32_t ldc,
                                                       uint32_t epilogue);

/* CUDA IPC between the processes of one node (for scatter destinations):
 * get_handle exports the cudaMalloc allocation whose base is device_ptr
 * (vnpu_buffer_alloc memory qualifies) as 64 opaque bytes; open maps such a
 * handle from another process on `device` (peer access enabled);
 * close unmaps it. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_get_handle(const void *device_ptr,
                                                         uint8_t handle[64]);
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_open(int device, const uint8_t handle[64],
                                                   void **out_ptr);
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_close(void *ptr);

/* The cudaStream_t behind a vnpu stream (as void*), so callers can order
 * their own CUDA work and timing events against its kernels.  Copies of host
 * operands run on two further streams of the vnpu stream (uploads, downloads)
 * joined to this one by events: work ordered after this handle sees a
 * command's kernels but not the download of its host outputs, which vnpu
 * events and vnpu_stream_sync do cover. */
VNPU_API void * VNPU_CALL vnpu_b200_stream_handle(vnpu_stream_t *stream);

/* CUDA device ordinal of a vnpu device. */
VNPU_API int VNPU_CALL vnpu_b200_device_ordinal(const vnpu_device_t *device);

/* Number of kernels this library has launched on the device so far. */
VNPU_API uint64_t VNPU_CALL vnpu_b200_kernel_launches(const vnpu_device_t *device);

/* The reference device whose rounding this device reproduces (no reference
 * counterpart): MATMUL_I8's per-element epilogue form and MATMUL_F32's
 * per-tile accumulation order are those of a reference device
 * (src/core/runtime.cpp:858-938) with these settings.  epilogue_forced != 0
 * when VNPU_B200_EPILOGUE fixed one form (epilogue_form: 0 block, 1 stream,
 * 2 scalar) for every element instead. */
typedef struct vnpu_b200_reference_model {
    uint32_t num_threads;          /* worker threads */
    uint32_t tile_m, tile_k, tile_n;
    uint32_t pack_b;               /* VNPU_PACK */
    uint32_t scalar_isa;           /* VNPU_FORCE_ISA=scalar or VNPU_MODE=reference */
    uint64_t l2_bytes;             /* the host L2 size it reads */
    uint32_t epilogue_forced;
    uint32_t epilogue_form;
} vnpu_b200_reference_model_t;

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_reference_model(const vnpu_device_t *device,
                                                          vnpu_b200_reference_model_t *out);

/* Device address of the packed K-major weight matrix ([N][k_stride] int8)
 * and of its scales, for callers that fuse their own kernels around it. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_packed_weights_device(
    const vnpu_packed_weights_t *weights, const int8_t **bt, uint32_t *k_stride,
    const float **scales);

/* Which MATMUL_I8 kernel the dispatcher picks for a shape, by name
 * ("tcgen05", "gemv", "simt"); for tests and the bench. */
VNPU_API const char * VNPU_CALL vnpu_b200_matmul_i8_kernel(uint32_t M, uint32_t K, uint32_t N,
                                                          uint32_t lda, const void *A);

/* Name of the kernel the most recent MATMUL_I8 launch in this process used
 * ("gemm_i8_tcgen05_pair_wide_kernel", "gemm_i8_tcgen05_pair_kernel",
 * "gemm_i8_tcgen05_kernel", "gemv_i8_tcgen05_kernel", "gemv_i8_kernel",
 * "gemm_i8_simt_kernel"; "none" before the first); for tests and the bench. */
VNPU_API const char * VNPU_CALL vnpu_b200_last_matmul_kernel(void);

/* Device-side wait self-test: launches a kernel that waits on a flag nothing
 * sets, bounded by timeout_us, and returns VNPU_ERR_TIMEOUT when the bound is
 * hit (VNPU_OK would mean the flag was seen).  It exercises the same bounded
 * wait and error-word path the GEMM pipeline uses, without faulting the GPU. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_selftest_wait_timeout(vnpu_stream_t *stream,
                                                                uint32_t timeout_us);

/*
 * CUDA-graph capture of a command stream (no reference counterpart: the
 * reference's stream worker has no launch cost to amortise).  Commands
 * submitted between capture_begin and capture_end are recorded, not run;
 * graph_launch replays them on any stream of the same device with one launch.
 * While capturing, every operand must already be in device memory (host
 * operands would need a host copy at replay time): such commands, and
 * PACK_WEIGHTS_I8, fail with VNPU_ERR_INVALID_ARGUMENT, and vnpu_stream_sync
 * returns VNPU_ERR_DEVICE_BUSY.  Packed weights used by a graph must outlive it.
 */
typedef struct vnpu_b200_graph vnpu_b200_graph_t;
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_capture_begin(vnpu_stream_t *stream);
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_capture_end(vnpu_stream_t *stream,
                                                      vnpu_b200_graph_t **out_graph);
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_graph_launch(vnpu_b200_graph_t *graph,
                                                       vnpu_stream_t *stream);
VNPU_API void VNPU_CALL vnpu_b200_graph_destroy(vnpu_b200_graph_t *graph);

/*
 * The decoder block of the reference's synthetic LLM benchmark (no reference
 * counterpart as an API: the reference drives it from its tool,
 * tools/llm_bench.cpp:213-326, with host vectors, and has no KV cache; its
 * "decode" re-runs the block).  Here the block lives in the library: weights
 * quantized per column and packed in HBM, a KV cache of `capacity` slots
 * ([heads][capacity][head_dim] f32 each, zero, with an additive mask of -inf
 * on the slots not yet written), activations in HBM, and every op a vnpu
 * command on the block's stream, so a C engine can run prefill and KV-cached
 * decode without any other runtime.  The op sequence and its bits are the
 * reference block's: RMSNorm (eps) -> QUANTIZE_I8 -> MATMUL_I8 (QKV) -> RoPE
 * (theta_base) on Q, K -> causal ATTENTION_F32 -> QUANTIZE_I8 -> MATMUL_I8
 * (O) -> ADD -> RMSNorm -> QUANTIZE_I8 -> MATMUL_I8 (gate/up) -> SWIGLU_F32 ->
 * QUANTIZE_I8 -> MATMUL_I8 (down) -> ADD, run as the B200 opcodes that give
 * the same bits (RMSNORM_QUANTIZE_I8, QKV_ROPE_APPEND, MATMUL_I8_RESIDUAL,
 * MATMUL_I8_SWIGLU, or SWIGLU_QUANTIZE_I8 with VNPU_B200_BLOCK_SWIGLU_PROLOGUE).
 */
#define VNPU_B200_BLOCK_SWIGLU_PROLOGUE  (1u << 0)

typedef struct vnpu_b200_block_config_t {
    uint32_t d_model;      /* heads * head_dim */
    uint32_t heads;
    uint32_t inter;        /* SwiGLU hidden width I */
    uint32_t capacity;     /* KV-cache slots; also the largest prefill */
    float eps;             /* RMSNorm epsilon; <= 0: 1e-5, as RMSNORM_F32 */
    float theta_base;      /* RoPE; <= 0: 10000 */
    uint32_t flags;        /* VNPU_B200_BLOCK_* */
    uint32_t reserved0;
} vnpu_b200_block_config_t;

typedef struct vnpu_b200_block vnpu_b200_block_t;

/* Creates the block on `stream`'s device.  Weights are f32, host or device
 * memory, row-major: w_qkv d x 3d (columns [Q | K | V], head-contiguous),
 * w_o d x d, w_gate_up d x 2I (columns [gate | up]), w_down I x d, norm1 and
 * norm2 d entries.  They are quantized per column (QUANTIZE_I8) and packed;
 * the f32 arrays are not kept.  Synchronous. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_create(
    vnpu_stream_t *stream, const vnpu_b200_block_config_t *config, const float *w_qkv,
    const float *w_o, const float *w_gate_up, const float *w_down, const float *norm1,
    const float *norm2, vnpu_b200_block_t **out_block);

/* T tokens x (T x d f32, device) at positions pos .. pos+T-1 -> y (T x d f32,
 * device; may not alias x).  T > 1 is a prefill from an empty cache (pos must
 * be 0; the tokens attend causally to each other, as the reference block
 * does); T = 1 attends to every filled cache slot.  Sets the device-side
 * position to pos + T.  Enqueued on the block's stream. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_forward(vnpu_b200_block_t *block, const float *x,
                                                        uint32_t T, uint32_t pos, float *y);

/* One decode token at the device-side position, which then advances by one,
 * as one CUDA-graph launch: the first call (and any call whose x or y differs
 * from the previous one) records the step, later calls replay it.  x and y
 * are 1 x d f32 device memory.  Enqueued on the block's stream. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_decode(vnpu_b200_block_t *block, const float *x,
                                                       float *y);

/* Empties the cache (zero K/V, mask -inf) and sets the position to 0. */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_reset(vnpu_b200_block_t *block);

VNPU_API void VNPU_CALL vnpu_b200_block_destroy(vnpu_b200_block_t *block);

/*
 * Per-tensor QUANTIZE_I8 (VNPU_QUANT_PER_TENSOR) that allocates nothing.  No
 * reference counterpart: the reference quantizes on host memory it already
 * owns.  Same bits as vnpu_quantize_i8 with axis PER_TENSOR (reference
 * src/kernels/llm.cpp:421-436).
 *
 * For callers that cannot allocate device memory at the point of the call and
 * hold no vnpu stream (whose creation allocates its error and scratch words):
 * an engine that reserved all of HBM for weights and its KV-cache pool at
 * start-up, or code on an out-of-memory path.  The scratch is a static device
 * array inside this library (65,792 bytes per device); the call makes no
 * cudaMalloc/cudaMallocAsync/cudaFree and no allocating library call.
 *
 * X (rows*cols f32), Y (rows*cols int8) and scale (1 f32) are device memory of
 * CUDA device `device`; cuda_stream is a cudaStream_t of that device (NULL =
 * its legacy default stream).  The work is enqueued on the stream; nothing
 * synchronises.  The device is made current for the call and the caller's
 * current device is restored.
 *
 * Limits and errors (VNPU_ERR_INVALID_ARGUMENT, with a line on stderr, before
 * anything is enqueued): rows*cols above 2^28 elements (the static scratch
 * holds one partial maximum per 2^14 elements, for 2^14 chunks), a zero size,
 * a NULL or host pointer, or a pointer on another device.
 *
 * The first call on each device looks up the scratch address
 * (cudaGetSymbolAddress, with that device current) and zeroes its counter
 * word with a synchronous cudaMemset; make that first call before any stream
 * capture on the device.
 *
 * There is one scratch per device and process: calls that can overlap on the
 * same device (different streams with no ordering between them, or several
 * host threads) race on it and give wrong results.  Order such calls.
 */
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_quantize_i8_tensor_noalloc(
    int device, void *cuda_stream, const float *X, int8_t *Y, float *scale, uint64_t rows,
    uint64_t cols);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VNPU_B200_H */
