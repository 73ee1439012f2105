// block.cpp - the decoder block of the reference's synthetic LLM benchmark
// (tools/llm_bench.cpp:213-326) as a library object with a KV cache: weights
// packed in HBM, activations and cache in HBM, every op a vnpu command on the
// block's stream, one decode token replayed as a CUDA graph.  The reference
// drives the same op sequence from its tool with host vectors and no cache;
// here it runs as the B200 opcodes that give the same bits:
//   RMSNORM_QUANTIZE_I8 -> QKV_ROPE_APPEND -> ATTENTION_F32 -> QUANTIZE_I8 ->
//   MATMUL_I8_RESIDUAL (O) -> RMSNORM_QUANTIZE_I8 -> MATMUL_I8_SWIGLU ->
//   QUANTIZE_I8 -> MATMUL_I8_RESIDUAL (down)
// (or MATMUL_I8 + SWIGLU_QUANTIZE_I8 for the gate/up step with
// VNPU_B200_BLOCK_SWIGLU_PROLOGUE).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/vnpu.h"
#include "../../include/vnpu_b200.h"
#include "kernels.h"
#include "runtime.h"

struct vnpu_b200_block {
    vnpu_stream_t *stream = nullptr;
    vnpu_b200_block_config_t cfg{};
    uint32_t head_dim = 0;
    vnpu_packed_weights_t *w_qkv = nullptr, *w_o = nullptr, *w_gu = nullptr, *w_down = nullptr;
    float *norm1 = nullptr, *norm2 = nullptr;
    float *kc = nullptr, *vc = nullptr, *mask = nullptr;  // [heads][capacity][head_dim], [heads][capacity]
    int32_t *pos = nullptr;                               // device-side position
    // activations, `capacity` rows each
    int8_t *a8 = nullptr;
    float *sa = nullptr, *q = nullptr, *kt = nullptr, *vt = nullptr, *o = nullptr, *x1 = nullptr;
    float *ff = nullptr, *gu = nullptr;
    std::vector<void *> allocs;
    vnpu_b200_graph_t *graph = nullptr;
    const float *graph_x = nullptr;
    float *graph_y = nullptr;
};

namespace {

using vnpu_b200::LaunchCtx;

template <typename T>
vnpu_status_t dev_alloc(vnpu_b200_block_t *b, T **p, uint64_t count) {
    void *v = nullptr;
    if (cudaMalloc(&v, count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_OUT_OF_MEMORY;
    }
    b->allocs.push_back(v);
    *p = static_cast<T *>(v);
    return VNPU_OK;
}

template <typename A>
vnpu_command_t b200_cmd(uint32_t opcode, const A &args, uint32_t flags = 0) {
    static_assert(sizeof(A) <= sizeof(vnpu_command_t::args), "arguments fit the command");
    vnpu_command_t c;
    std::memset(&c, 0, sizeof(c));
    c.opcode = opcode;
    c.flags = flags;
    std::memcpy(c.args.raw, &args, sizeof(args));
    return c;
}

// VNPU_B200_CMD_FLAG_ADVANCE_POSITION with its fields after the command's own
// arguments.
void with_advance(vnpu_command_t &c, int32_t *position, int32_t advance) {
    c.flags |= VNPU_B200_CMD_FLAG_ADVANCE_POSITION;
    const vnpu_b200_advance_t a{position, advance, 0};
    std::memcpy(c.args.raw + VNPU_B200_ADVANCE_OFFSET, &a, sizeof(a));
}

// Launch context for the block's own small kernels on the stream; launches
// are counted like the commands' (into the capture while capturing).
LaunchCtx block_ctx(vnpu_stream_t *s, uint64_t *counter) {
    LaunchCtx c;
    c.stream = s->cs;
    c.err = s->d_err;
    c.num_sms = s->device->num_sms;
    c.wait_limit_ns = s->device->wait_limit_ns;
    c.launch_counter = counter;
    return c;
}

void count_block_launches(vnpu_stream_t *s, uint64_t n) {
    if (s->capturing)
        s->captured_launches += n;
    else
        s->device->launches.fetch_add(n);
}

// f32 weight (K x N, host or device) -> QUANTIZE_I8 per column -> packed.
vnpu_status_t pack_f32(vnpu_b200_block_t *b, const float *w, uint32_t K, uint32_t N,
                       vnpu_packed_weights_t **out) {
    int8_t *q = nullptr;
    float *s = nullptr;
    if (cudaMalloc(reinterpret_cast<void **>(&q), static_cast<uint64_t>(K) * N) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&s), sizeof(float) * N) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(q);
        return VNPU_ERR_OUT_OF_MEMORY;
    }
    vnpu_command_t c;
    std::memset(&c, 0, sizeof(c));
    c.opcode = VNPU_OP_QUANTIZE_I8;
    c.args.quantize_i8 = vnpu_quantize_i8_args_t{w, q, s, K, N, VNPU_QUANT_PER_COLUMN, 0};
    vnpu_status_t rc = vnpu_stream_submit(b->stream, &c, 1, nullptr);
    if (rc == VNPU_OK) rc = vnpu_stream_sync(b->stream);
    if (rc == VNPU_OK) rc = vnpu_pack_weights_i8(b->stream->device, q, s, K, N, N, 0, out);
    cudaFree(q);
    cudaFree(s);
    return rc;
}

}  // namespace

namespace {

// The block's commands for T tokens: x (T x d) -> y.  position: the device
// position (decode replay) or NULL (host pos).
std::vector<vnpu_command_t> block_commands(vnpu_b200_block_t *b, const float *x, uint32_t T,
                                           uint32_t pos, const int32_t *position, float *y) {
    const vnpu_b200_block_config_t &c = b->cfg;
    const uint32_t d = c.d_model, I = c.inter, H = c.heads, hd = b->head_dim;
    std::vector<vnpu_command_t> cmds;
    // RMSNorm -> QUANTIZE_I8 (per row) of x
    cmds.push_back(b200_cmd(VNPU_B200_OP_RMSNORM_QUANTIZE_I8,
                            vnpu_b200_rmsnorm_quantize_args_t{x, b->norm1, nullptr, b->a8, b->sa, T,
                                                              d, c.eps, 0}));
    // QKV projection, RoPE on Q and K, K/V appended at slots pos..pos+T-1
    cmds.push_back(b200_cmd(
        VNPU_B200_OP_QKV_ROPE_APPEND,
        vnpu_b200_qkv_rope_append_args_t{b->a8, b->w_qkv, b->sa, nullptr, b->q,
                                         T > 1 ? b->kt : nullptr, T > 1 ? b->vt : nullptr, b->kc,
                                         b->vc, b->mask, position, T, d, H, hd, c.capacity, pos,
                                         c.theta_base, 1.0f, 0, 0}));
    // attention: a prefill over its own tokens (causal), a decode token over
    // the cache (the mask hides the empty slots); O token-major [T][d]
    vnpu_command_t att;
    std::memset(&att, 0, sizeof(att));
    att.opcode = VNPU_OP_ATTENTION_F32;
    if (T > 1) {
        att.args.attention = vnpu_attention_f32_args_t{b->q, b->kt, b->vt, nullptr, b->o, nullptr, 0,
                                                       1, H, T, T, hd, 1, 0.0f, 0};
        att.flags = VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR;
    } else {
        att.args.attention = vnpu_attention_f32_args_t{b->q, b->kc, b->vc, b->mask, b->o, nullptr,
                                                       0, 1, H, 1, c.capacity, hd, 0, 0.0f, 0};
    }
    cmds.push_back(att);
    // O projection + residual: x1 = x + O W_o
    vnpu_command_t qo;
    std::memset(&qo, 0, sizeof(qo));
    qo.opcode = VNPU_OP_QUANTIZE_I8;
    qo.args.quantize_i8 = vnpu_quantize_i8_args_t{b->o, b->a8, b->sa, T, d, VNPU_QUANT_PER_ROW, 0};
    cmds.push_back(qo);
    cmds.push_back(b200_cmd(VNPU_B200_OP_MATMUL_I8_RESIDUAL,
                            vnpu_b200_matmul_i8_residual_args_t{b->a8, b->w_o, b->sa, nullptr, x,
                                                                b->x1, T, d, d, 0, 0, 0, 0, 0}));
    // RMSNorm -> QUANTIZE_I8 of x1
    cmds.push_back(b200_cmd(VNPU_B200_OP_RMSNORM_QUANTIZE_I8,
                            vnpu_b200_rmsnorm_quantize_args_t{b->x1, b->norm2, nullptr, b->a8, b->sa,
                                                              T, d, c.eps, 0}));
    if (c.flags & VNPU_B200_BLOCK_SWIGLU_PROLOGUE) {
        // gate/up product [T][2I], then SwiGLU -> QUANTIZE_I8 reading its halves
        vnpu_command_t gu;
        std::memset(&gu, 0, sizeof(gu));
        gu.opcode = VNPU_OP_MATMUL_I8;
        gu.args.matmul_i8 = vnpu_matmul_i8_args_t{b->a8, b->w_gu, b->sa, nullptr, b->gu, T, d,
                                                  2 * I, 0, 0, 0, 0};
        cmds.push_back(gu);
        cmds.push_back(b200_cmd(VNPU_B200_OP_SWIGLU_QUANTIZE_I8,
                                vnpu_b200_swiglu_quantize_args_t{b->gu, b->gu + I, nullptr, b->a8,
                                                                 b->sa, T, I, 1.0f, 2 * I}));
    } else {
        // gate/up with the SwiGLU in its epilogue, then QUANTIZE_I8
        cmds.push_back(b200_cmd(VNPU_B200_OP_MATMUL_I8_SWIGLU,
                                vnpu_b200_matmul_i8_swiglu_args_t{b->a8, b->w_gu, b->sa, nullptr,
                                                                  b->ff, T, d, 2 * I, 0, 0, 0,
                                                                  1.0f, 0}));
        vnpu_command_t qf;
        std::memset(&qf, 0, sizeof(qf));
        qf.opcode = VNPU_OP_QUANTIZE_I8;
        qf.args.quantize_i8 = vnpu_quantize_i8_args_t{b->ff, b->a8, b->sa, T, I, VNPU_QUANT_PER_ROW, 0};
        cmds.push_back(qf);
    }
    // down projection + residual: y = x1 + ff W_down; a decode step also
    // advances the device position there
    vnpu_command_t dc = b200_cmd(VNPU_B200_OP_MATMUL_I8_RESIDUAL,
                                 vnpu_b200_matmul_i8_residual_args_t{b->a8, b->w_down, b->sa,
                                                                     nullptr, b->x1, y, T, I, d, 0,
                                                                     0, 0, 0, 0});
    if (position) with_advance(dc, b->pos, static_cast<int32_t>(T));
    cmds.push_back(dc);
    return cmds;
}

vnpu_status_t set_position(vnpu_b200_block_t *b, int32_t value, bool advance) {
    uint64_t n = 0;
    const LaunchCtx ctx = block_ctx(b->stream, &n);
    const cudaError_t e = vnpu_b200::block_position(ctx, b->pos, value, advance);
    count_block_launches(b->stream, n);
    return e == cudaSuccess ? VNPU_OK : VNPU_ERR_DEVICE_ERROR;
}

}  // namespace

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_create(
    vnpu_stream_t *stream, const vnpu_b200_block_config_t *config, const float *w_qkv,
    const float *w_o, const float *w_gate_up, const float *w_down, const float *norm1,
    const float *norm2, vnpu_b200_block_t **out_block) {
    if (!out_block) return VNPU_ERR_INVALID_ARGUMENT;
    *out_block = nullptr;
    if (!stream || !config || !w_qkv || !w_o || !w_gate_up || !w_down || !config->heads ||
        !config->d_model || config->d_model % config->heads || !config->inter ||
        !config->capacity || (config->d_model / config->heads) % 2 ||
        config->d_model / config->heads > 512)
        return VNPU_ERR_INVALID_ARGUMENT;
    cudaSetDevice(stream->device->ordinal);
    auto *b = new vnpu_b200_block_t();
    b->stream = stream;
    b->cfg = *config;
    b->head_dim = config->d_model / config->heads;
    const uint32_t d = config->d_model, I = config->inter, H = config->heads, cap = config->capacity;
    const uint64_t cache = static_cast<uint64_t>(H) * cap * b->head_dim;
    const uint64_t rows = cap;
    vnpu_status_t rc = VNPU_OK;
    auto step = [&](vnpu_status_t r) {
        if (rc == VNPU_OK) rc = r;
    };
    step(pack_f32(b, w_qkv, d, 3 * d, &b->w_qkv));
    step(pack_f32(b, w_o, d, d, &b->w_o));
    step(pack_f32(b, w_gate_up, d, 2 * I, &b->w_gu));
    step(pack_f32(b, w_down, I, d, &b->w_down));
    step(dev_alloc(b, &b->norm1, d));
    step(dev_alloc(b, &b->norm2, d));
    step(dev_alloc(b, &b->kc, cache));
    step(dev_alloc(b, &b->vc, cache));
    step(dev_alloc(b, &b->mask, static_cast<uint64_t>(H) * cap));
    step(dev_alloc(b, &b->pos, 1));
    step(dev_alloc(b, &b->a8, rows * (d > I ? d : I)));
    step(dev_alloc(b, &b->sa, rows));
    step(dev_alloc(b, &b->q, rows * d));
    step(dev_alloc(b, &b->kt, rows * d));
    step(dev_alloc(b, &b->vt, rows * d));
    step(dev_alloc(b, &b->o, rows * d));
    step(dev_alloc(b, &b->x1, rows * d));
    if (config->flags & VNPU_B200_BLOCK_SWIGLU_PROLOGUE)
        step(dev_alloc(b, &b->gu, rows * 2 * I));
    else
        step(dev_alloc(b, &b->ff, rows * I));
    if (rc == VNPU_OK) {
        // RMSNorm weights (host or device; NULL = 1.0)
        std::vector<float> ones(d, 1.0f);
        for (auto [dst, src] : {std::pair<float *, const float *>{b->norm1, norm1},
                                std::pair<float *, const float *>{b->norm2, norm2}})
            if (cudaMemcpy(dst, src ? src : ones.data(), sizeof(float) * d, cudaMemcpyDefault) !=
                cudaSuccess)
                rc = VNPU_ERR_INVALID_ARGUMENT;
    }
    if (rc == VNPU_OK) rc = vnpu_b200_block_reset(b);
    if (rc == VNPU_OK) rc = vnpu_stream_sync(stream);
    if (rc != VNPU_OK) {
        cudaGetLastError();
        vnpu_b200_block_destroy(b);
        return rc;
    }
    *out_block = b;
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_reset(vnpu_b200_block_t *block) {
    if (!block) return VNPU_ERR_INVALID_ARGUMENT;
    vnpu_stream_t *s = block->stream;
    cudaSetDevice(s->device->ordinal);
    const uint64_t cache = static_cast<uint64_t>(block->cfg.heads) * block->cfg.capacity *
                           block->head_dim * sizeof(float);
    if (cudaMemsetAsync(block->kc, 0, cache, s->cs) != cudaSuccess ||
        cudaMemsetAsync(block->vc, 0, cache, s->cs) != cudaSuccess)
        return VNPU_ERR_DEVICE_ERROR;
    uint64_t n = 0;
    const LaunchCtx ctx = block_ctx(s, &n);
    if (vnpu_b200::fill_neg_inf(ctx, block->mask,
                                static_cast<uint64_t>(block->cfg.heads) * block->cfg.capacity) !=
        cudaSuccess)
        return VNPU_ERR_DEVICE_ERROR;
    count_block_launches(s, n);
    return set_position(block, 0, false);
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_forward(vnpu_b200_block_t *block, const float *x,
                                                        uint32_t T, uint32_t pos, float *y) {
    if (!block || !x || !y || !T || T > block->cfg.capacity || (T > 1 && pos != 0) ||
        static_cast<uint64_t>(pos) + T > block->cfg.capacity || x == y)
        return VNPU_ERR_INVALID_ARGUMENT;
    cudaSetDevice(block->stream->device->ordinal);
    const std::vector<vnpu_command_t> cmds = block_commands(block, x, T, pos, nullptr, y);
    const vnpu_status_t rc = vnpu_stream_submit(block->stream, cmds.data(), cmds.size(), nullptr);
    if (rc != VNPU_OK) return rc;
    return set_position(block, static_cast<int32_t>(pos + T), false);
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_block_decode(vnpu_b200_block_t *block, const float *x,
                                                       float *y) {
    if (!block || !x || !y || x == y) return VNPU_ERR_INVALID_ARGUMENT;
    vnpu_stream_t *s = block->stream;
    cudaSetDevice(s->device->ordinal);
    if (!block->graph || block->graph_x != x || block->graph_y != y) {
        if (block->graph) {
            vnpu_b200_graph_destroy(block->graph);
            block->graph = nullptr;
        }
        vnpu_status_t rc = vnpu_b200_capture_begin(s);
        if (rc != VNPU_OK) return rc;
        const std::vector<vnpu_command_t> cmds = block_commands(block, x, 1, 0, block->pos, y);
        rc = vnpu_stream_submit(s, cmds.data(), cmds.size(), nullptr);
        vnpu_b200_graph_t *g = nullptr;
        const vnpu_status_t rc_end = vnpu_b200_capture_end(s, &g);
        if (rc == VNPU_OK) rc = rc_end;
        if (rc != VNPU_OK) {
            if (g) vnpu_b200_graph_destroy(g);
            return rc;
        }
        block->graph = g;
        block->graph_x = x;
        block->graph_y = y;
    }
    return vnpu_b200_graph_launch(block->graph, s);
}

VNPU_API void VNPU_CALL vnpu_b200_block_destroy(vnpu_b200_block_t *block) {
    if (!block) return;
    cudaSetDevice(block->stream->device->ordinal);
    vnpu_stream_sync(block->stream);
    if (block->graph) vnpu_b200_graph_destroy(block->graph);
    for (vnpu_packed_weights_t *w : {block->w_qkv, block->w_o, block->w_gu, block->w_down})
        if (w) vnpu_packed_weights_destroy(w);
    for (void *p : block->allocs) cudaFree(p);
    delete block;
}
