// block_ops.cu - decoder-block operators on sm_100a: RMSNORM_F32, ROPE_F32,
// SWIGLU_F32, ADD_F32, ATTENTION_F32 (src/kernels/llm.cpp).
//
// Each restates the arithmetic of the reference's AVX2 build in the same
// order of operations where the order is cheap to keep (RMSNorm's 8-lane
// sum, SwiGLU's exp256, ADD's FMA, attention's 16x64 blocking with its
// 8-lane dot products and in-order probability sums), so on identical inputs
// they reproduce the reference bit for bit; RoPE uses the device sinf/cosf
// (<= 2 ulp from glibc) with the reference's inverse frequencies computed on
// the host with the same libm powf.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "quant_common.cuh"

namespace vnpu_b200 {
namespace {

inline void count_launch(const LaunchCtx &ctx, uint64_t n = 1) {
    if (ctx.launch_counter) *ctx.launch_counter += n;
}

// ---------------------------------------------------------------------------
// RMSNorm (llm.cpp:80-106, AVX2): ss = 8-lane FMA partial sums over full
// 8-element groups, hsum256 order, scalar FMA tail; inv = 1/sqrt(ss/cols+eps);
// y = (x*w)*inv on the vector part, x*inv*w on the tail.
// One warp per row; lanes 0..7 run the eight partial-sum chains.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *__restrict__ X,
                                                      const float *__restrict__ W,
                                                      float *__restrict__ Y, uint32_t rows,
                                                      uint32_t cols, float eps) {
    pdl_enter();
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *x = X + static_cast<uint64_t>(warp) * cols;
    float *y = Y + static_cast<uint64_t>(warp) * cols;
    const uint32_t full = cols & ~7u;
    float part = 0.0f;
    if (lane < 8)
        for (uint32_t j = lane; j < full; j += 8) part = __fmaf_rn(x[j], x[j], part);
    // hsum256: ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7))
    const float hi = __shfl_down_sync(0xffffffffu, part, 4);
    const float s = __fadd_rn(part, hi);             // lane i<4: v_i + v_{i+4}
    const float s1 = __shfl_down_sync(0xffffffffu, s, 1);
    const float s01 = __fadd_rn(s, s1);              // lane 0: s0+s1, lane 2: s2+s3
    const float s23 = __shfl_down_sync(0xffffffffu, s01, 2);
    float sum = __fadd_rn(s01, s23);                 // lane 0
    if (lane == 0)
        for (uint32_t j = full; j < cols; ++j) sum = __fmaf_rn(x[j], x[j], sum);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(cols)), eps)));
    for (uint32_t j = lane; j < cols; j += 32) {
        const float w = W ? W[j] : 1.0f;
        y[j] = j < full ? __fmul_rn(__fmul_rn(x[j], w), inv) : __fmul_rn(__fmul_rn(x[j], inv), w);
    }
}

// The same arithmetic with one CTA per row: the row is staged in shared
// memory by coalesced loads, so the eight sequential chains (lanes 0..7 of
// warp 0) read it at shared-memory latency instead of global.
constexpr uint32_t kRmsRowThreads = 256;
constexpr uint32_t kRmsRowMaxCols = 48 * 1024;   // 192 KiB staged row

// Stage row x into xs (CTA-wide) and return 1/sqrt(ss/cols + eps) with ss in
// the reference's AVX2 order, computed by lanes 0..7 of warp 0 from xs.
__device__ __forceinline__ float stage_row_rms_inv(const float *__restrict__ x, float *xs,
                                                   uint32_t cols, float eps, bool vec,
                                                   float *inv_sh) {
    const uint32_t tid = threadIdx.x;
    if (vec) {
        for (uint32_t i = tid; i < cols / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(xs)[i] = __ldg(reinterpret_cast<const float4 *>(x) + i);
    } else {
        for (uint32_t i = tid; i < cols; i += blockDim.x) xs[i] = __ldg(x + i);
    }
    __syncthreads();
    const uint32_t full = cols & ~7u;
    if (tid < 32) {
        float part = 0.0f;
        if (tid < 8) {
            // 16 loads ahead of the dependent FMAs, so the chain runs at FMA
            // latency rather than shared-memory latency.
            const uint32_t steps = full / 8;
            uint32_t k = 0;
            for (; k + 16 <= steps; k += 16) {
                float v[16];
#pragma unroll
                for (uint32_t u = 0; u < 16; ++u) v[u] = xs[tid + 8 * (k + u)];
#pragma unroll
                for (uint32_t u = 0; u < 16; ++u) part = __fmaf_rn(v[u], v[u], part);
            }
            for (; k < steps; ++k) part = __fmaf_rn(xs[tid + 8 * k], xs[tid + 8 * k], part);
        }
        const float hi = __shfl_down_sync(0xffffffffu, part, 4);
        const float s = __fadd_rn(part, hi);
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1);
        const float s01 = __fadd_rn(s, s1);
        const float s23 = __shfl_down_sync(0xffffffffu, s01, 2);
        if (tid == 0) {
            float sum = __fadd_rn(s01, s23);
            for (uint32_t j = full; j < cols; ++j) sum = __fmaf_rn(xs[j], xs[j], sum);
            *inv_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(cols)), eps)));
        }
    }
    __syncthreads();
    return *inv_sh;
}

__global__ void __launch_bounds__(kRmsRowThreads) rmsnorm_row_kernel(
    const float *__restrict__ X, const float *__restrict__ W, float *__restrict__ Y,
    uint32_t cols, float eps, bool vec) {
    pdl_enter();
    extern __shared__ __align__(16) float xs[];
    __shared__ float inv_sh;
    const uint32_t tid = threadIdx.x;
    const float *x = X + static_cast<uint64_t>(blockIdx.x) * cols;
    float *y = Y + static_cast<uint64_t>(blockIdx.x) * cols;
    const uint32_t full = cols & ~7u;
    const float inv = stage_row_rms_inv(x, xs, cols, eps, vec, &inv_sh);
    if (vec && W && (reinterpret_cast<uintptr_t>(W) & 15u) == 0u) {
        // cols % 8 == 0 here (vec requires it): every element is in the vector part
        for (uint32_t i = tid; i < cols / 4; i += kRmsRowThreads) {
            const float4 xv = reinterpret_cast<const float4 *>(xs)[i];
            const float4 wv = __ldg(reinterpret_cast<const float4 *>(W) + i);
            reinterpret_cast<float4 *>(y)[i] =
                make_float4(__fmul_rn(__fmul_rn(xv.x, wv.x), inv), __fmul_rn(__fmul_rn(xv.y, wv.y), inv),
                            __fmul_rn(__fmul_rn(xv.z, wv.z), inv), __fmul_rn(__fmul_rn(xv.w, wv.w), inv));
        }
    } else {
        for (uint32_t j = tid; j < cols; j += kRmsRowThreads) {
            const float w = W ? W[j] : 1.0f;
            y[j] = j < full ? __fmul_rn(__fmul_rn(xs[j], w), inv) : __fmul_rn(__fmul_rn(xs[j], inv), w);
        }
    }
}

// ---------------------------------------------------------------------------
// Fused row prologues for the next MATMUL_I8 (no reference counterpart: the
// reference runs RMSNORM_F32 / SWIGLU_F32 and then QUANTIZE_I8 per row).  One
// CTA per row: the f32 result is formed in shared memory exactly as the
// stand-alone kernels form it (and optionally written out), then quantized per
// row from those same values - the bits of the two-command sequence.
// ---------------------------------------------------------------------------
// A row is split over a cluster of C CTAs (C = 1 when there are rows enough to
// fill the GPU): CTA `rank` forms and quantizes columns [c0, c1); the row's
// absmax is the max of the CTAs' maxima, exchanged through distributed shared
// memory (a max is order-free, so the scale is the stand-alone one).
constexpr uint32_t kFqThreads = 256;
constexpr uint32_t kFqMaxCluster = 8;
constexpr uint32_t kFqPerThread = 8;    // elements in flight per thread and pass

__device__ __forceinline__ void fq_slice(uint32_t cols, uint32_t &c0, uint32_t &c1) {
    const uint32_t C = cluster_nctarank(), rank = cluster_ctarank();
    const uint32_t per = ((cols + C - 1) / C + 15u) & ~15u;   // 16-aligned slices
    c0 = min(cols, rank * per);
    c1 = min(cols, c0 + per);
}

// Finish a row: the CTA's slice of f32 values is in ys[0 .. c1-c0), its
// largest |y| in `m`; exchange maxima, quantize the slice.
__device__ __forceinline__ void fq_quantize_slice(const float *ys, uint32_t c0, uint32_t c1,
                                                  float m, int8_t *__restrict__ q,
                                                  float *__restrict__ scale_out, float *red,
                                                  float *maxes) {
    const uint32_t tid = threadIdx.x;
    const uint32_t C = cluster_nctarank(), rank = cluster_ctarank();
    m = block_max(m, red);
    float rowmax = m;   // >= 0, never NaN (fmaxf from 0)
    if (C > 1) {        // a row over several CTAs: exchange their maxima
        if (tid < C) st_shared_cluster_f32(mapa_shared(smem_addr(maxes + rank), tid), m);
        cluster_sync_all();
        rowmax = 0.0f;
        for (uint32_t r = 0; r < C; ++r) rowmax = fmaxf(rowmax, maxes[r]);
    }
    const float scale = scale_from_absmax(rowmax);
    const float inv = __fdiv_rn(1.0f, scale);
    if (tid == 0 && rank == 0) *scale_out = scale;
    const uint32_t n = c1 - c0;
    if ((reinterpret_cast<uintptr_t>(q + c0) & 3u) == 0u) {
        for (uint32_t i = tid; i < n / 4; i += kFqThreads) {
            const float4 v = reinterpret_cast<const float4 *>(ys)[i];
            reinterpret_cast<uint32_t *>(q + c0)[i] = pack4(v.x, v.y, v.z, v.w, inv);
        }
        for (uint32_t j = (n & ~3u) + tid; j < n; j += kFqThreads) q[c0 + j] = quantize_value(ys[j], inv);
    } else {
        for (uint32_t j = tid; j < n; j += kFqThreads) q[c0 + j] = quantize_value(ys[j], inv);
    }
}

__global__ void __launch_bounds__(kFqThreads) rmsnorm_quantize_kernel(
    const float *__restrict__ X, const float *__restrict__ W, float *__restrict__ Y,
    int8_t *__restrict__ Q, float *__restrict__ scales, uint32_t cols, float eps, bool vec) {
    pdl_enter();
    extern __shared__ __align__(16) float xs[];   // the whole row
    __shared__ __align__(16) float maxes[kFqMaxCluster];
    __shared__ float inv_sh;
    __shared__ float red[32];
    const uint32_t tid = threadIdx.x;
    const uint64_t row = blockIdx.x / cluster_nctarank();
    // Every CTA stages the row and runs the same in-order chains (no broadcast).
    const float inv = stage_row_rms_inv(X + row * cols, xs, cols, eps, vec, &inv_sh);
    uint32_t c0, c1;
    fq_slice(cols, c0, c1);
    const uint32_t full = cols & ~7u;
    float *y = Y ? Y + row * cols : nullptr;
    float m = 0.0f;
    for (uint32_t base = c0 + tid; base < c1; base += kFqThreads * kFqPerThread) {
        float wv[kFqPerThread];
#pragma unroll
        for (uint32_t e = 0; e < kFqPerThread; ++e) {
            const uint32_t j = base + e * kFqThreads;
            wv[e] = (W && j < c1) ? __ldg(W + j) : 1.0f;
        }
#pragma unroll
        for (uint32_t e = 0; e < kFqPerThread; ++e) {
            const uint32_t j = base + e * kFqThreads;
            if (j < c1) {
                const float v = j < full ? __fmul_rn(__fmul_rn(xs[j], wv[e]), inv)
                                         : __fmul_rn(__fmul_rn(xs[j], inv), wv[e]);
                xs[j] = v;   // in place: each element is read once, by its own thread
                m = fmaxf(m, fabsf(v));
                if (y) y[j] = v;
            }
        }
    }
    __syncthreads();
    fq_quantize_slice(xs + c0, c0, c1, m, Q + row * cols, scales + row, red, maxes);
}

__global__ void __launch_bounds__(kFqThreads) swiglu_quantize_kernel(
    const float *__restrict__ G, const float *__restrict__ U, float *__restrict__ Y,
    int8_t *__restrict__ Q, float *__restrict__ scales, uint32_t cols, uint32_t ld, float alpha) {
    pdl_enter();
    extern __shared__ __align__(16) float ys[];   // this CTA's slice
    __shared__ __align__(16) float maxes[kFqMaxCluster];
    __shared__ float red[32];
    const uint32_t tid = threadIdx.x;
    const uint64_t row = blockIdx.x / cluster_nctarank();
    uint32_t c0, c1;
    fq_slice(cols, c0, c1);
    const float *g = G + row * ld;
    const float *u = U + row * ld;
    float *y = Y ? Y + row * cols : nullptr;
    float m = 0.0f;
    for (uint32_t base = c0 + tid; base < c1; base += kFqThreads * kFqPerThread) {
        float gv[kFqPerThread], uv[kFqPerThread];
#pragma unroll
        for (uint32_t e = 0; e < kFqPerThread; ++e) {
            const uint32_t j = base + e * kFqThreads;
            gv[e] = j < c1 ? __ldg(g + j) : 0.0f;
            uv[e] = j < c1 ? __ldg(u + j) : 0.0f;
        }
#pragma unroll
        for (uint32_t e = 0; e < kFqPerThread; ++e) {
            const uint32_t j = base + e * kFqThreads;
            if (j < c1) {
                const float v = __fmul_rn(
                    __fmul_rn(__fdiv_rn(gv[e], __fadd_rn(1.0f, ref_exp256_lane(-gv[e]))), uv[e]), alpha);
                ys[j - c0] = v;
                m = fmaxf(m, fabsf(v));
                if (y) y[j] = v;
            }
        }
    }
    __syncthreads();
    fq_quantize_slice(ys, c0, c1, m, Q + row * cols, scales + row, red, maxes);
}

// ---------------------------------------------------------------------------
// RoPE (llm.cpp:188-217, :576-602): one thread per (batch*head, token, pair).
// ---------------------------------------------------------------------------
constexpr uint32_t kRopeMaxPairs = 256;
struct RopeFreq {
    float inv[kRopeMaxPairs];
};

__device__ __forceinline__ void rotate_pair(float *x, uint32_t i0, uint32_t i1, float angle) {
    float s, c;
    sincosf(angle, &s, &c);
    const float x0 = x[i0], x1 = x[i1];
    x[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    x[i1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void rope_kernel(float *__restrict__ Q, float *__restrict__ K,
                            const int32_t *__restrict__ positions, uint32_t bh_count,
                            uint32_t q_seq, uint32_t k_seq, uint32_t head_dim,
                            uint32_t position_offset, uint32_t interleaved, float scaling,
                            const RopeFreq freq) {
    pdl_enter();
    const uint32_t pairs = head_dim / 2;
    const uint32_t seq = max(q_seq, k_seq);
    const uint64_t total = static_cast<uint64_t>(bh_count) * seq * pairs;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t j = static_cast<uint32_t>(i % pairs);
        const uint64_t tok = i / pairs;
        const uint32_t t = static_cast<uint32_t>(tok % seq);
        const uint64_t bh = tok / seq;
        const float position = __fmul_rn(
            static_cast<float>(positions ? positions[t] : static_cast<int32_t>(t + position_offset)),
            scaling);
        const float angle = __fmul_rn(position, freq.inv[j]);
        const uint32_t i0 = interleaved ? 2 * j : j;
        const uint32_t i1 = interleaved ? 2 * j + 1 : j + pairs;
        if (Q && t < q_seq) rotate_pair(Q + (bh * q_seq + t) * head_dim, i0, i1, angle);
        if (K && t < k_seq) rotate_pair(K + (bh * k_seq + t) * head_dim, i0, i1, angle);
    }
}

// ---------------------------------------------------------------------------
// SwiGLU (llm.cpp:289-306, AVX2): s = g / (1 + exp256(-g)); y = (s*u)*alpha.
// ADD (llm.cpp:256-271, AVX2): y = fma(a, alpha, b*beta).
// ---------------------------------------------------------------------------
__global__ void swiglu_kernel(const float *__restrict__ G, const float *__restrict__ U,
                              float *__restrict__ Y, uint64_t n, float alpha) {
    pdl_enter();
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float g = G[i];
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, ref_exp256_lane(-g)));
        Y[i] = __fmul_rn(__fmul_rn(s, U[i]), alpha);
    }
}

// Y[r][j] = swiglu(C[r][j], C[r][I + j]) * alpha: the gate/up halves of one
// [rows][2I] projection output (row stride ldc), the same expression.
__global__ void swiglu_rows_kernel(const float *__restrict__ C, uint32_t ldc, float *__restrict__ Y,
                                   uint32_t ldy, uint32_t rows, uint32_t I, float alpha) {
    pdl_enter();
    const uint64_t n = static_cast<uint64_t>(rows) * I;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = i / I;
        const uint32_t j = static_cast<uint32_t>(i - r * I);
        const float g = C[r * ldc + j];
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, ref_exp256_lane(-g)));
        Y[r * ldy + j] = __fmul_rn(__fmul_rn(s, C[r * ldc + I + j]), alpha);
    }
}

__global__ void swiglu_vec_kernel(const float4 *__restrict__ G, const float4 *__restrict__ U,
                                  float4 *__restrict__ Y, uint64_t n4, float alpha) {
    pdl_enter();
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float4 g = G[i], u = U[i];
        float4 y;
        y.x = __fmul_rn(__fmul_rn(__fdiv_rn(g.x, __fadd_rn(1.0f, ref_exp256_lane(-g.x))), u.x), alpha);
        y.y = __fmul_rn(__fmul_rn(__fdiv_rn(g.y, __fadd_rn(1.0f, ref_exp256_lane(-g.y))), u.y), alpha);
        y.z = __fmul_rn(__fmul_rn(__fdiv_rn(g.z, __fadd_rn(1.0f, ref_exp256_lane(-g.z))), u.z), alpha);
        y.w = __fmul_rn(__fmul_rn(__fdiv_rn(g.w, __fadd_rn(1.0f, ref_exp256_lane(-g.w))), u.w), alpha);
        Y[i] = y;
    }
}

__global__ void add_kernel(const float *__restrict__ A, const float *__restrict__ B,
                           float *__restrict__ Y, uint64_t n, float alpha, float beta) {
    pdl_enter();
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        Y[i] = __fmaf_rn(A[i], alpha, __fmul_rn(B[i], beta));
}

__global__ void add_vec_kernel(const float4 *__restrict__ A, const float4 *__restrict__ B,
                               float4 *__restrict__ Y, uint64_t n4, float alpha, float beta) {
    pdl_enter();
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float4 a = A[i], b = B[i];
        Y[i] = make_float4(__fmaf_rn(a.x, alpha, __fmul_rn(b.x, beta)),
                           __fmaf_rn(a.y, alpha, __fmul_rn(b.y, beta)),
                           __fmaf_rn(a.z, alpha, __fmul_rn(b.z, beta)),
                           __fmaf_rn(a.w, alpha, __fmul_rn(b.w, beta)));
    }
}

// ---------------------------------------------------------------------------
// Attention (llm.cpp:442-546).  One CTA (16 warps) per (batch*head, block of
// 16 queries); keys in blocks of 64 as in the reference.
//   scores : thread (key, chain) holds chain c of K[key] (elements 8t+c) in
//            registers and runs the FMA chain against each query;
//            the eight chains are combined in hsum256 order, the D%8 tail is
//            FMA'd after, then *scale (+mask); causal keys are -inf.
//   softmax: warp q: block max; skip the block if it is not finite;
//            alpha = fast_expf(m - new_m), p = fast_expf(s - new_m) (the
//            reference's attention is compiled without FMA: unfused
//            polynomial); l = l*alpha + (in-order sum of p).
//   values : thread (q, d): acc = acc*alpha, then acc = fma(V[j][d], p_j, acc)
//            for j in order, skipping p == 0.
// ---------------------------------------------------------------------------
constexpr uint32_t kAttBQ = 16;
constexpr uint32_t kAttBK = 64;
constexpr uint32_t kAttThreads = 512;
constexpr uint32_t kAttMaxD = 256;
constexpr uint32_t kAttMaxChain = kAttMaxD / 8;

// Chain-major Q tile: chain c of a query starts at c * att_chain_stride; the
// stride is 4 mod 8 floats so the eight chains fall in eight distinct groups
// of four banks (16-byte reads conflict-free).
__host__ __device__ constexpr uint32_t att_chain_stride(uint32_t chains) {
    return chains + ((4u + 8u - (chains & 7u)) & 7u);
}
__host__ __device__ constexpr uint32_t att_q_stride(uint32_t D) {
    return 8u * att_chain_stride(D / 8u) + (D & 7u);
}

struct AttParams {
    const float *Q, *K, *V, *mask;
    float *O;
    uint32_t heads, seq_q, seq_k, D, causal;
    float scale;
    uint32_t *err;       // stream error word (bounded waits)
    uint64_t wait_ns;    // bound of every device-side wait
    uint32_t o_tokens = 0;   // 1: O is [batch][seq_q][heads][D] (token-major rows)
};

// Output row of query qi of (batch * heads + h) = bh: head-major as the
// reference lays it out, or token-major (VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR).
// With seq_q == 1 the two are the same addresses.
__device__ __forceinline__ float *att_out_row(const AttParams &p, uint32_t bh, uint32_t qi) {
    if (!p.o_tokens) return p.O + (static_cast<uint64_t>(bh) * p.seq_q + qi) * p.D;
    const uint32_t b = bh / p.heads, h = bh - b * p.heads;
    return p.O + ((static_cast<uint64_t>(b) * p.seq_q + qi) * p.heads + h) * p.D;
}

// Layout in shared memory:
//   Qs [16 q][8 chains][D/8] - chain-major, so a thread reads its chain of a
//                              query with 16-byte loads (plus the D%8 tail
//                              [16 q][D%8] after it);
//   Vs [64 keys][D];  S [16 q][64 keys] scores, then probabilities.
// Warp q (0..15) owns query q in the softmax and value phases: its online
// softmax state lives in registers and the two phases need no block barrier.
template <bool VEC>
__global__ void __launch_bounds__(kAttThreads) attention_kernel(const AttParams p) {
    pdl_enter();
    extern __shared__ float att_smem[];
    const uint32_t D = p.D;
    const uint32_t chains = D / 8, full = chains * 8, tail = D - full;
    const uint32_t cstride = att_chain_stride(chains);     // padded: conflict-free chains
    const uint32_t qstride = att_q_stride(D);
    float *Qs = att_smem;                                  // 16*qstride
    float *Vs = Qs + kAttBQ * qstride;                     // 64*D
    float *S = Vs + kAttBK * D;                            // 16*64

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bh = blockIdx.y;
    const uint32_t q0 = blockIdx.x * kAttBQ;
    const uint32_t qc = min(kAttBQ, p.seq_q - q0);
    const uint64_t head_q = static_cast<uint64_t>(bh) * p.seq_q * D;
    const uint64_t head_k = static_cast<uint64_t>(bh) * p.seq_k * D;
    const float *Qh = p.Q + head_q;
    const float *Kh = p.K + head_k;
    const float *Vh = p.V + head_k;
    const float *Mh = p.mask ? p.mask + static_cast<uint64_t>(bh) * p.seq_q * p.seq_k : nullptr;
    const uint32_t causal_offset = p.seq_k > p.seq_q ? p.seq_k - p.seq_q : 0;

    for (uint32_t i = tid; i < kAttBQ * D; i += kAttThreads) {
        const uint32_t q = i / D, e = i % D;
        const float v = q < qc ? Qh[static_cast<uint64_t>(q0 + q) * D + e] : 0.0f;
        // element e = 8t + c of the vector part goes to chain c, position t;
        // the D%8 tail follows the eight chains
        const uint32_t dst = e < full ? q * qstride + (e & 7u) * cstride + (e >> 3)
                                      : q * qstride + 8u * cstride + (e - full);
        Qs[dst] = v;
    }

    // Per-query state of the query this warp owns (lane-uniform).
    float m_run = -__int_as_float(0x7f800000), l_run = 0.0f;
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    float acc_s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};

    uint32_t k_end = p.seq_k;
    if (p.causal) k_end = min(p.seq_k, q0 + qc - 1 + causal_offset + 1);

    const uint32_t my_key = tid >> 3, my_chain = tid & 7;
    for (uint32_t k0 = 0; k0 < k_end; k0 += kAttBK) {
        const uint32_t kc = min(kAttBK, p.seq_k - k0);
        __syncthreads();  // previous block's V and probabilities consumed
        if (VEC) {
            const float4 *src = reinterpret_cast<const float4 *>(Vh + static_cast<uint64_t>(k0) * D);
            float4 *dst = reinterpret_cast<float4 *>(Vs);
            for (uint32_t i = tid; i < kc * D / 4; i += kAttThreads) dst[i] = __ldg(src + i);
        } else {
            for (uint32_t i = tid; i < kc * D; i += kAttThreads)
                Vs[i] = Vh[static_cast<uint64_t>(k0) * D + i];
        }
        // ---- scores: thread (key, chain) keeps its chain of K[key] in registers
        float kreg[kAttMaxChain];
        const bool key_ok = my_key < kc;
        const float *krow = Kh + static_cast<uint64_t>(k0 + (key_ok ? my_key : 0)) * D;
#pragma unroll
        for (uint32_t t = 0; t < kAttMaxChain; ++t)
            kreg[t] = (key_ok && t < chains) ? __ldg(krow + 8 * t + my_chain) : 0.0f;
        __syncthreads();  // Qs (first block) and Vs visible
        for (uint32_t q = 0; q < qc; ++q) {
            const float *qchain = Qs + q * qstride + my_chain * cstride;
            float part = 0.0f;
            if (VEC && (chains & 3u) == 0u) {
#pragma unroll
                for (uint32_t t = 0; t < kAttMaxChain; t += 4) {
                    if (t < chains) {
                        const float4 qv = *reinterpret_cast<const float4 *>(qchain + t);
                        part = __fmaf_rn(qv.x, kreg[t + 0], part);
                        part = __fmaf_rn(qv.y, kreg[t + 1], part);
                        part = __fmaf_rn(qv.z, kreg[t + 2], part);
                        part = __fmaf_rn(qv.w, kreg[t + 3], part);
                    }
                }
            } else {
#pragma unroll
                for (uint32_t t = 0; t < kAttMaxChain; ++t)
                    if (t < chains) part = __fmaf_rn(qchain[t], kreg[t], part);
            }
            // hsum256 within the 8-lane group
            const float hi = __shfl_down_sync(0xffffffffu, part, 4, 8);
            const float s = __fadd_rn(part, hi);
            const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
            const float s01 = __fadd_rn(s, s1);
            const float s23 = __shfl_down_sync(0xffffffffu, s01, 2, 8);
            if (my_chain == 0 && key_ok) {
                float dot = __fadd_rn(s01, s23);
                for (uint32_t i = 0; i < tail; ++i)
                    dot = __fmaf_rn(Qs[q * qstride + 8u * cstride + i], krow[full + i], dot);
                const uint32_t qi = q0 + q, ki = k0 + my_key;
                float sc;
                if (p.causal && ki > qi + causal_offset) {
                    sc = -__int_as_float(0x7f800000);
                } else {
                    sc = __fmul_rn(dot, p.scale);
                    if (Mh) sc = __fadd_rn(sc, Mh[static_cast<uint64_t>(qi) * p.seq_k + ki]);
                }
                S[q * kAttBK + my_key] = sc;
            }
        }
        __syncthreads();  // all scores of the block written
        if (warp >= qc) continue;
        // ---- online softmax of query `warp` (llm.cpp:516-538)
        float *srow = S + warp * kAttBK;
        float bmax = -__int_as_float(0x7f800000);
        for (uint32_t j = lane; j < kc; j += 32) bmax = fmaxf(bmax, srow[j]);
        for (int o = 16; o > 0; o >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
        if (!isfinite(bmax)) continue;  // fully masked block: skipped, as in the reference
        const float nm = fmaxf(m_run, bmax);
        const float p_lo = lane < kc ? ref_fast_expf(__fsub_rn(srow[lane], nm), false) : 0.0f;
        const float p_hi = lane + 32 < kc ? ref_fast_expf(__fsub_rn(srow[lane + 32], nm), false) : 0.0f;
        if (lane < kc) srow[lane] = p_lo;
        if (lane + 32 < kc) srow[lane + 32] = p_hi;
        const float alpha = ref_fast_expf(__fsub_rn(m_run, nm), false);
        __syncwarp();
        // the in-order sum of p over the block's keys, walked through shuffles
        float sum_p = 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < 32; ++j) {
            const float v = __shfl_sync(0xffffffffu, p_lo, j);
            if (j < kc) sum_p = __fadd_rn(sum_p, v);
        }
#pragma unroll
        for (uint32_t j = 0; j < 32; ++j) {
            const float v = __shfl_sync(0xffffffffu, p_hi, j);
            if (j + 32 < kc) sum_p = __fadd_rn(sum_p, v);
        }
        l_run = __fadd_rn(__fmul_rn(l_run, alpha), sum_p);
        m_run = nm;
        // ---- values: acc = acc*alpha, then acc = fma(V[j], p_j, acc) in key order
        if (VEC) {
#pragma unroll
            for (uint32_t r = 0; r < 2; ++r) {
                const uint32_t d4 = lane + 32u * r;
                if (d4 * 4u >= D) break;
                float4 a = acc[r];
                a.x = __fmul_rn(a.x, alpha);
                a.y = __fmul_rn(a.y, alpha);
                a.z = __fmul_rn(a.z, alpha);
                a.w = __fmul_rn(a.w, alpha);
                for (uint32_t j = 0; j < kc; ++j) {
                    const float pj = srow[j];
                    if (pj == 0.0f) continue;
                    const float4 v = *reinterpret_cast<const float4 *>(Vs + j * D + 4u * d4);
                    a.x = __fmaf_rn(v.x, pj, a.x);
                    a.y = __fmaf_rn(v.y, pj, a.y);
                    a.z = __fmaf_rn(v.z, pj, a.z);
                    a.w = __fmaf_rn(v.w, pj, a.w);
                }
                acc[r] = a;
            }
        } else {
#pragma unroll
            for (uint32_t r = 0; r < 8; ++r) {
                const uint32_t d = lane + 32u * r;
                if (d >= D) break;
                float a = __fmul_rn(acc_s[r], alpha);
                for (uint32_t j = 0; j < kc; ++j) {
                    const float pj = srow[j];
                    if (pj == 0.0f) continue;
                    a = __fmaf_rn(Vs[j * D + d], pj, a);
                }
                acc_s[r] = a;
            }
        }
    }
    if (warp < qc) {
        const float inv = l_run > 0.0f ? __fdiv_rn(1.0f, l_run) : 0.0f;
        float *orow = att_out_row(p, bh, q0 + warp);
        if (VEC) {
#pragma unroll
            for (uint32_t r = 0; r < 2; ++r) {
                const uint32_t d4 = lane + 32u * r;
                if (d4 * 4u >= D) break;
                reinterpret_cast<float4 *>(orow)[d4] =
                    make_float4(__fmul_rn(acc[r].x, inv), __fmul_rn(acc[r].y, inv),
                                __fmul_rn(acc[r].z, inv), __fmul_rn(acc[r].w, inv));
            }
        } else {
#pragma unroll
            for (uint32_t r = 0; r < 8; ++r) {
                const uint32_t d = lane + 32u * r;
                if (d >= D) break;
                orow[d] = __fmul_rn(acc_s[r], inv);
            }
        }
    }
}

// a = fma(v, p, a) when p != 0, else a unchanged (the reference skips zero
// probabilities); a predicated FMA keeps the test off the dependency chain.
__device__ __forceinline__ float fma_if_nonzero(float v, float p, float a) {
    asm("{\n\t.reg .pred q;\n\tsetp.ne.f32 q, %2, 0f00000000;\n\t@q fma.rn.f32 %0, %1, %2, %0;\n\t}"
        : "+f"(a)
        : "f"(v), "f"(p));
    return a;
}

// Prefill attention for head_dim 128: the same arithmetic again, tiled for
// the CUDA cores.  One CTA (8 warps) per (batch*head, 64 queries), one CTA
// per SM, the CTAs with the most causal keys first; K and V blocks of 64
// keys double-buffered in shared memory by cp.async.  Warp w owns queries
// 8w..8w+7 through all three phases, so only the block loads need the whole
// CTA in step:
//   scores : lane (c, kg) = (lane%8, lane/8) runs AVX2 chain c of the warp's
//            8 queries x keys 8kg..8kg+7 of a 32-key half (Q and K rows
//            chain-major in shared memory: 16 loaded floats per 64 FMAs), then
//            three shuffle steps add the chains in hsum256 order; *scale
//            (+mask);
//   softmax: lane (q, quarter) = (lane/4, lane%4) holds keys 16*quarter..+15
//            of query q: causal and ragged keys -inf, block max, skip if not
//            finite, fast_expf, the in-order sum handed from quarter to
//            quarter, l = l*alpha + sum;
//   values : lane l owns dims 4l..4l+3 of all 8 queries: acc = acc*alpha,
//            then fma(V[j][d], p_j, acc) in key order.  The reference skips
//            zero probabilities; where every query's nonzero probabilities
//            are a prefix of the block (all keys, or a causal diagonal), the
//            FMAs below the shortest prefix need no test.
constexpr uint32_t kApThreads = 256;
constexpr uint32_t kApBQ = 64;
constexpr uint32_t kApD = 128;
// Q and K rows are kept chain-major: element d of a row at (d % 8) * kApCS + d / 8,
// so a lane reads four steps of its chain with one 16-byte load; the chain
// stride of 20 floats puts the eight chains in distinct bank groups.
constexpr uint32_t kApCS = 20;
constexpr uint32_t kApTRow = 8 * kApCS;   // floats per chain-major row
// K rows go in pairs, interleaved: keys 2i and 2i+1 of chain c at step t sit
// side by side, so a 16-byte load gives two steps of a key pair as two f32x2
// operands; 36 floats per chain keep the eight chains in distinct bank groups.
constexpr uint32_t kApKCS = 36;
constexpr uint32_t kApKPRow = 8 * kApKCS;   // floats per key pair
constexpr uint32_t kApKStage = (kAttBK / 2) * kApKPRow;
constexpr size_t kApSmemFloats = static_cast<size_t>(kApBQ) * kApTRow + 2u * kApKStage +
                                 2u * kAttBK * kApD + static_cast<size_t>(kApBQ) * kAttBK;

// 64 rows of 128 floats (rows >= valid zero) into chain-major rows, by
// 4-byte copies (a warp reads 128 contiguous bytes and writes 32 distinct banks).
__device__ __forceinline__ void ap_load_rows_t(float *T, const float *src, uint32_t valid,
                                               uint32_t tid) {
#pragma unroll 4
    for (uint32_t e = tid; e < 64u * kApD; e += kApThreads) {
        const uint32_t row = e >> 7, d = e & 127u;
        const bool ok = row < valid;
        cp_async_4_zfill(T + row * kApTRow + (d & 7u) * kApCS + (d >> 3),
                         src + static_cast<uint64_t>(ok ? row : 0u) * kApD + d, ok);
    }
}

// Block k0 of K (chain-major, key pairs interleaved) and V (64 rows; rows
// past seq_k zero) into one stage.
__device__ __forceinline__ void ap_load_kv(float *Ks, float *Vs, const float *Kh, const float *Vh,
                                           uint32_t k0, uint32_t seq_k, uint32_t tid) {
    const uint32_t valid = min(64u, seq_k - k0);
    const float *src = Kh + static_cast<uint64_t>(k0) * kApD;
#pragma unroll 4
    for (uint32_t e = tid; e < 64u * kApD; e += kApThreads) {
        const uint32_t row = e >> 7, d = e & 127u;
        const bool ok = row < valid;
        cp_async_4_zfill(Ks + (row >> 1) * kApKPRow + (d & 7u) * kApKCS + (d >> 3) * 2u + (row & 1u),
                         src + static_cast<uint64_t>(ok ? row : 0u) * kApD + d, ok);
    }
#pragma unroll
    for (uint32_t i = tid; i < kAttBK * kApD / 4; i += kApThreads) {
        const uint32_t j = i >> 5, c4 = i & 31u;
        const bool ok = j < valid;
        const uint64_t row = ok ? k0 + j : k0;
        cp_async_16_zfill(Vs + j * kApD + 4 * c4, Vh + row * kApD + 4 * c4, ok);
    }
}

// a += v * p for four dims held as two f32 pairs: fma(v[d], p, a[d]) each,
// two per fma.rn.f32x2.
__device__ __forceinline__ void fma4x2(uint64_t (&a)[2], const ulonglong2 &v, float p) {
    const uint64_t pp = pack_f32x2(p, p);
    a[0] = fma_f32x2(v.x, pp, a[0]);
    a[1] = fma_f32x2(v.y, pp, a[1]);
}

__global__ void __launch_bounds__(kApThreads, 1) attention_prefill_kernel(const AttParams p) {
    pdl_enter();
    extern __shared__ __align__(16) float ap_smem[];
    float *Qs = ap_smem;                          // [64][kApTRow] chain-major
    float *Kst = Qs + kApBQ * kApTRow;            // [2][32 key pairs][kApKPRow]
    float *Vst = Kst + 2 * kApKStage;             // [2][64][128]
    float *S = Vst + 2 * kAttBK * kApD;           // [64][64] scores, then probabilities

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t bh = blockIdx.x;
    const uint32_t q0 = (gridDim.y - 1 - blockIdx.y) * kApBQ;
    const uint32_t qc = min(kApBQ, p.seq_q - q0);
    const uint64_t head_q = static_cast<uint64_t>(bh) * p.seq_q * kApD;
    const uint64_t head_k = static_cast<uint64_t>(bh) * p.seq_k * kApD;
    const float *Kh = p.K + head_k;
    const float *Vh = p.V + head_k;
    const float *Mh = p.mask ? p.mask + static_cast<uint64_t>(bh) * p.seq_q * p.seq_k : nullptr;
    const uint32_t causal_offset = p.seq_k > p.seq_q ? p.seq_k - p.seq_q : 0;
    const float ninf = -__int_as_float(0x7f800000);

    uint32_t k_end = p.seq_k;
    if (p.causal) k_end = min(p.seq_k, q0 + qc - 1 + causal_offset + 1);
    const uint32_t nblk = (k_end + kAttBK - 1) / kAttBK;

    // Q rows (zero past seq_q) and the first K/V block: copy group 0.
    ap_load_rows_t(Qs, p.Q + head_q + static_cast<uint64_t>(q0) * kApD, qc, tid);
    if (nblk > 0) ap_load_kv(Kst, Vst, Kh, Vh, 0, p.seq_k, tid);
    cp_async_commit();

    // softmax lanes: state of query row 8*warp + lane/4 (the four lanes agree)
    const uint32_t sq = lane >> 2, quarter = lane & 3u;
    const uint32_t srow = 8 * warp + sq;
    const uint32_t sqi = q0 + srow;
    float m_run = ninf, l_run = 0.0f;
    // value lanes: dims 4*lane..4*lane+3 of the warp's 8 queries
    // as pairs (dims 0-1, 2-3) for fma.rn.f32x2: two independent fmaf per instruction
    uint64_t acc[8][2];
#pragma unroll
    for (uint32_t q = 0; q < 8; ++q) acc[q][0] = acc[q][1] = 0ull;

    const uint32_t wq_last = q0 + 8 * warp + 7;   // last query row of the warp
    // score lanes: chain c = lane % 8; slot r holds query 8*warp + (r ^ mq)
    const uint32_t c_ = lane & 7u;
    const uint32_t mq = ((c_ >> 2) & 1u) * 4u + (c_ & 1u) * 2u + ((c_ >> 1) & 1u);
    const float *qptr[8];
#pragma unroll
    for (uint32_t r = 0; r < 8; ++r) qptr[r] = Qs + (8 * warp + (r ^ mq)) * kApTRow + c_ * kApCS;
    for (uint32_t b = 0; b < nblk; ++b) {
        const uint32_t k0 = b * kAttBK;
        const uint32_t kc = min(kAttBK, p.seq_k - k0);
        if (b + 1 < nblk) {
            const uint32_t nx = (b + 1) & 1u;
            ap_load_kv(Kst + nx * kApKStage, Vst + nx * kAttBK * kApD, Kh, Vh, k0 + kAttBK,
                       p.seq_k, tid);
            cp_async_commit();
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();   // block b (and Q) visible to every warp
        const float *Ks = Kst + (b & 1u) * kApKStage;
        const float *Vs = Vst + (b & 1u) * kAttBK * kApD;

        // ---- scores: lane (c, kg) runs chain c of the warp's 8 queries x keys
        // jb + 8kg + u (u < 8), then the eight chains of each pair are summed
        // across lanes in hsum256 order
        {
            const uint32_t c = lane & 7u, kg = lane >> 3;
#pragma unroll 1
            for (uint32_t jb = 0; jb < kAttBK; jb += 32) {
                // a half whose keys are past kc, or causal-masked for every
                // query of the warp, is left out (the softmax masks it)
                if (jb >= kc || (p.causal && k0 + jb > wq_last + causal_offset)) break;
                // acc2[r][i]: keys 2i, 2i+1 of slot r, one fma.rn.f32x2 per step
                uint64_t acc2[8][4];
#pragma unroll
                for (uint32_t r = 0; r < 8; ++r)
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) acc2[r][i] = 0ull;
                const float *kp_ = Ks + (jb / 2u + 4u * kg) * kApKPRow + c * kApKCS;
#pragma unroll 1
                for (uint32_t tg = 0; tg < 4; ++tg) {
                    float4 qv[8];
#pragma unroll
                    for (uint32_t r = 0; r < 8; ++r)
                        qv[r] = *reinterpret_cast<const float4 *>(qptr[r] + 4 * tg);
                    // kk[i][0] = steps 4tg, 4tg+1 of key pair i; kk[i][1] = steps 4tg+2, 4tg+3
                    ulonglong2 kk[4][2];
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) {
                        kk[i][0] = *reinterpret_cast<const ulonglong2 *>(kp_ + i * kApKPRow + 8 * tg);
                        kk[i][1] = *reinterpret_cast<const ulonglong2 *>(kp_ + i * kApKPRow + 8 * tg + 4);
                    }
#pragma unroll
                    for (uint32_t r = 0; r < 8; ++r) {
                        const float qs[4] = {qv[r].x, qv[r].y, qv[r].z, qv[r].w};
#pragma unroll
                        for (uint32_t st = 0; st < 4; ++st) {
                            const uint64_t qq = pack_f32x2(qs[st], qs[st]);
#pragma unroll
                            for (uint32_t i = 0; i < 4; ++i) {
                                const uint64_t kpair = st == 0 ? kk[i][0].x : st == 1 ? kk[i][0].y
                                                     : st == 2 ? kk[i][1].x : kk[i][1].y;
                                acc2[r][i] = fma_f32x2(qq, kpair, acc2[r][i]);
                            }
                        }
                    }
                }
                float acc[8][8];
#pragma unroll
                for (uint32_t r = 0; r < 8; ++r)
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) {
                        acc[r][2 * i] = half_f32x2(acc2[r][i], 0);
                        acc[r][2 * i + 1] = half_f32x2(acc2[r][i], 1);
                    }
                // Slot r of lane c holds query r ^ mq: each step keeps the
                // lower slots and adds the partner's upper ones, which hold
                // the same queries; partners c^4, c^1, c^2 give
                // ((c0+c4)+(c1+c5))+((c2+c6)+(c3+c7)) (each add commutes).
#pragma unroll
                for (uint32_t r = 0; r < 4; ++r)
#pragma unroll
                    for (uint32_t u = 0; u < 8; ++u)
                        acc[r][u] = __fadd_rn(acc[r][u], __shfl_xor_sync(0xffffffffu, acc[r + 4][u], 4));
#pragma unroll
                for (uint32_t r = 0; r < 2; ++r)
#pragma unroll
                    for (uint32_t u = 0; u < 8; ++u)
                        acc[r][u] = __fadd_rn(acc[r][u], __shfl_xor_sync(0xffffffffu, acc[r + 2][u], 1));
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u)
                    acc[0][u] = __fadd_rn(acc[0][u], __shfl_xor_sync(0xffffffffu, acc[1][u], 2));
                const uint32_t q = 8 * warp + mq;
                const uint32_t qi = q0 + q;
                float sc[8];
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u) {
                    const uint32_t jj = jb + 8u * kg + u;
                    sc[u] = __fmul_rn(acc[0][u], p.scale);
                    if (Mh && qi < p.seq_q && jj < kc)
                        sc[u] = __fadd_rn(sc[u], Mh[static_cast<uint64_t>(qi) * p.seq_k + k0 + jj]);
                }
                float4 *srow4 = reinterpret_cast<float4 *>(S + q * kAttBK + jb + 8u * kg);
                srow4[0] = make_float4(sc[0], sc[1], sc[2], sc[3]);
                srow4[1] = make_float4(sc[4], sc[5], sc[6], sc[7]);
            }
        }
        __syncwarp();

        // ---- online softmax, lane (sq, quarter)
        float alpha = 1.0f;
        uint32_t info;   // bit 0 active, bit 1 nonzero keys form a prefix, bits 2.. their count
        {
            float *Sr = S + srow * kAttBK + 16 * quarter;
            float s[16];
#pragma unroll
            for (uint32_t i4 = 0; i4 < 4; ++i4) {
                const float4 v = *reinterpret_cast<const float4 *>(Sr + 4 * i4);
                s[4 * i4] = v.x;
                s[4 * i4 + 1] = v.y;
                s[4 * i4 + 2] = v.z;
                s[4 * i4 + 3] = v.w;
            }
            float bmax = ninf;
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) {
                const uint32_t j = 16 * quarter + i;
                if (j >= kc || (p.causal && k0 + j > sqi + causal_offset)) s[i] = ninf;
                bmax = fmaxf(bmax, s[i]);
            }
            bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
            bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
            const bool act = isfinite(bmax);   // fully masked block: skipped, as in the reference
            const float nm = fmaxf(m_run, bmax);
            float pr[16];
            uint32_t nzm = 0;
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) {
                pr[i] = act && 16 * quarter + i < kc ? ref_fast_expf(__fsub_rn(s[i], nm), false)
                                                     : 0.0f;
                nzm |= (pr[i] != 0.0f ? 1u : 0u) << i;
            }
            if (act) alpha = ref_fast_expf(__fsub_rn(m_run, nm), false);
            float run = 0.0f;
#pragma unroll
            for (uint32_t ph = 0; ph < 4; ++ph) {
                if (quarter == ph && act) {
#pragma unroll
                    for (uint32_t i = 0; i < 16; ++i)
                        if (16 * ph + i < kc) run = __fadd_rn(run, pr[i]);
                }
                run = __shfl_sync(0xffffffffu, run, (lane & ~3u) | ph);
            }
            if (act) {
                l_run = __fadd_rn(__fmul_rn(l_run, alpha), run);
                m_run = nm;
            }
#pragma unroll
            for (uint32_t i4 = 0; i4 < 4; ++i4)
                *reinterpret_cast<float4 *>(Sr + 4 * i4) =
                    make_float4(pr[4 * i4], pr[4 * i4 + 1], pr[4 * i4 + 2], pr[4 * i4 + 3]);
            uint64_t nz = 0;
#pragma unroll
            for (uint32_t x = 0; x < 4; ++x)
                nz |= static_cast<uint64_t>(__shfl_sync(0xffffffffu, nzm, (lane & ~3u) | x)) << (16 * x);
            const uint32_t n = static_cast<uint32_t>(__popcll(nz));
            const bool prefix = nz == (n == 64 ? ~0ull : ((1ull << n) - 1ull));
            info = (act ? 1u : 0u) | (prefix ? 2u : 0u) | (n << 2);
        }
        __syncwarp();

        // ---- values, lane = dims 4*lane..4*lane+3 of the warp's 8 queries
        {
            uint32_t nq[8];
            uint32_t nmin = kAttBK, nmax = 0;
            bool allpre = true;
#pragma unroll
            for (uint32_t q = 0; q < 8; ++q) {
                const uint32_t iq = __shfl_sync(0xffffffffu, info, 4 * q);
                const float aq = __shfl_sync(0xffffffffu, alpha, 4 * q);
                nq[q] = iq >> 2;
                nmin = min(nmin, nq[q]);
                nmax = max(nmax, nq[q]);
                allpre = allpre && (iq & 2u);
                if (iq & 1u) {
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h)
                        acc[q][h] = pack_f32x2(__fmul_rn(half_f32x2(acc[q][h], 0), aq),
                                               __fmul_rn(half_f32x2(acc[q][h], 1), aq));
                }
            }
            const float *vcol = Vs + 4 * lane;
            const float *Pw = S + 8 * warp * kAttBK;
            if (allpre) {
                uint32_t j = 0;
#pragma unroll 2
                for (; j + 4 <= nmin; j += 4) {
                    ulonglong2 v[4];
#pragma unroll
                    for (uint32_t u = 0; u < 4; ++u)
                        v[u] = *reinterpret_cast<const ulonglong2 *>(vcol + (j + u) * kApD);
#pragma unroll
                    for (uint32_t q = 0; q < 8; ++q) {
                        const float4 pp = *reinterpret_cast<const float4 *>(Pw + q * kAttBK + j);
                        fma4x2(acc[q], v[0], pp.x);
                        fma4x2(acc[q], v[1], pp.y);
                        fma4x2(acc[q], v[2], pp.z);
                        fma4x2(acc[q], v[3], pp.w);
                    }
                }
#pragma unroll 1
                for (; j < nmax; ++j) {
                    const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(vcol + j * kApD);
#pragma unroll
                    for (uint32_t q = 0; q < 8; ++q)
                        if (j < nq[q]) fma4x2(acc[q], v, Pw[q * kAttBK + j]);
                }
            } else {
#pragma unroll 1
                for (uint32_t j = 0; j < kc; ++j) {
                    const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(vcol + j * kApD);
#pragma unroll
                    for (uint32_t q = 0; q < 8; ++q) {
                        const float pq = Pw[q * kAttBK + j];
                        if (pq != 0.0f) fma4x2(acc[q], v, pq);
                    }
                }
            }
        }
        __syncthreads();   // stage b & 1 is refilled by the next iteration
    }
#pragma unroll
    for (uint32_t q = 0; q < 8; ++q) {
        const float lq = __shfl_sync(0xffffffffu, l_run, 4 * q);
        const uint32_t qi = q0 + 8 * warp + q;
        if (qi >= p.seq_q) continue;
        const float inv = lq > 0.0f ? __fdiv_rn(1.0f, lq) : 0.0f;
        reinterpret_cast<float4 *>(att_out_row(p, bh, qi))[lane] =
            make_float4(__fmul_rn(half_f32x2(acc[q][0], 0), inv),
                        __fmul_rn(half_f32x2(acc[q][0], 1), inv),
                        __fmul_rn(half_f32x2(acc[q][1], 0), inv),
                        __fmul_rn(half_f32x2(acc[q][1], 1), inv));
    }
}

// Decode attention (one query per head): the same arithmetic as
// attention_kernel, reorganised for latency.  One CTA per (batch, head):
//   A. every score of the row at once: thread (key, chain) runs its 16-step
//      chain (query chain in registers, K from global), hsum256 over the 8
//      chains, *scale (+mask); keys past the causal limit are -inf;
//   B. warp 0 walks the 64-key blocks in order: block max, skip if not
//      finite, p = fast_expf(s - m), alpha, in-order sum; p and alpha are
//      kept in shared memory;
//   C. thread d accumulates acc = acc*alpha_b, then fma(V[j][d], p_j, acc)
//      over the keys in order - the reference's order for every output d.
constexpr uint32_t kDecThreads = 512;
constexpr uint32_t kDecMaxKeys = 8192;

__global__ void __launch_bounds__(kDecThreads) attention_decode_kernel(const AttParams p) {
    pdl_enter();
    extern __shared__ float dec_smem[];
    const uint32_t D = p.D;
    const uint32_t chains = D / 8, full = chains * 8, tail = D - full;
    const uint32_t nblk = (p.seq_k + kAttBK - 1) / kAttBK;
    float *S = dec_smem;                          // [seq_k] scores, then probabilities
    float *alpha_b = S + p.seq_k;                 // [nblk]
    int *active_b = reinterpret_cast<int *>(alpha_b + nblk);  // [nblk]
    float *l_sh = reinterpret_cast<float *>(active_b + nblk); // [1]
    float *qv = l_sh + 1;                          // [D]

    const uint32_t tid = threadIdx.x, lane = tid & 31;
    const uint32_t bh = blockIdx.x;
    const float *Qh = p.Q + static_cast<uint64_t>(bh) * D;     // seq_q == 1
    const float *Kh = p.K + static_cast<uint64_t>(bh) * p.seq_k * D;
    const float *Vh = p.V + static_cast<uint64_t>(bh) * p.seq_k * D;
    const float *Mh = p.mask ? p.mask + static_cast<uint64_t>(bh) * p.seq_k : nullptr;
    const uint32_t causal_offset = p.seq_k - 1;   // seq_k > seq_q == 1

    for (uint32_t i = tid; i < D; i += kDecThreads) qv[i] = Qh[i];
    __syncthreads();
    // ---- A. scores
    const uint32_t my_chain = tid & 7, key_lane = tid >> 3;   // 64 keys per pass
    float qreg[kAttMaxChain];
#pragma unroll
    for (uint32_t t = 0; t < kAttMaxChain; ++t) qreg[t] = t < chains ? qv[8 * t + my_chain] : 0.0f;
    for (uint32_t base = 0; base < p.seq_k; base += kDecThreads / 8) {
        const uint32_t ki = base + key_lane;
        const bool key_ok = ki < p.seq_k;
        const float *krow = Kh + static_cast<uint64_t>(key_ok ? ki : 0) * D;
        float part = 0.0f;
#pragma unroll
        for (uint32_t t = 0; t < kAttMaxChain; ++t)
            if (t < chains) part = __fmaf_rn(qreg[t], key_ok ? __ldg(krow + 8 * t + my_chain) : 0.0f, part);
        const float hi = __shfl_down_sync(0xffffffffu, part, 4, 8);
        const float s = __fadd_rn(part, hi);
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
        const float s01 = __fadd_rn(s, s1);
        const float s23 = __shfl_down_sync(0xffffffffu, s01, 2, 8);
        if (my_chain == 0 && key_ok) {
            float dot = __fadd_rn(s01, s23);
            for (uint32_t i = 0; i < tail; ++i) dot = __fmaf_rn(qv[full + i], krow[full + i], dot);
            float sc;
            if (p.causal && ki > causal_offset) {
                sc = -__int_as_float(0x7f800000);
            } else {
                sc = __fmul_rn(dot, p.scale);
                if (Mh) sc = __fadd_rn(sc, Mh[ki]);
            }
            S[ki] = sc;
        }
    }
    __syncthreads();
    // ---- B. online softmax over the blocks, in order (warp 0)
    if (tid < 32) {
        float m_run = -__int_as_float(0x7f800000), l_run = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b) {
            const uint32_t k0 = b * kAttBK, kc = min(kAttBK, p.seq_k - k0);
            float *srow = S + k0;
            float bmax = -__int_as_float(0x7f800000);
            for (uint32_t j = lane; j < kc; j += 32) bmax = fmaxf(bmax, srow[j]);
            for (int o = 16; o > 0; o >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
            if (!isfinite(bmax)) {
                if (lane == 0) active_b[b] = 0;
                continue;
            }
            const float nm = fmaxf(m_run, bmax);
            for (uint32_t j = lane; j < kc; j += 32) srow[j] = ref_fast_expf(__fsub_rn(srow[j], nm), false);
            const float alpha = ref_fast_expf(__fsub_rn(m_run, nm), false);
            __syncwarp();
            float sum_p = 0.0f;
            if (lane == 0) {
                for (uint32_t j = 0; j < kc; ++j) sum_p = __fadd_rn(sum_p, srow[j]);
                alpha_b[b] = alpha;
                active_b[b] = 1;
            }
            sum_p = __shfl_sync(0xffffffffu, sum_p, 0);
            l_run = __fadd_rn(__fmul_rn(l_run, alpha), sum_p);
            m_run = nm;
            __syncwarp();
        }
        if (lane == 0) *l_sh = l_run;
    }
    __syncthreads();
    // ---- C. values, thread d, keys in order
    const float l = *l_sh;
    const float inv = l > 0.0f ? __fdiv_rn(1.0f, l) : 0.0f;
    for (uint32_t d = tid; d < D; d += kDecThreads) {
        float a = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b) {
            if (!active_b[b]) continue;
            a = __fmul_rn(a, alpha_b[b]);
            const uint32_t k0 = b * kAttBK, kc = min(kAttBK, p.seq_k - k0);
#pragma unroll 8
            for (uint32_t j = 0; j < kc; ++j) {
                const float pj = S[k0 + j];
                const float v = __ldg(Vh + static_cast<uint64_t>(k0 + j) * D + d);
                if (pj != 0.0f) a = __fmaf_rn(v, pj, a);
            }
        }
        p.O[static_cast<uint64_t>(bh) * D + d] = __fmul_rn(a, inv);
    }
}

// Decode attention on a cluster of kDcCluster CTAs per (batch, head), same
// arithmetic again.  The row's keys are split across the cluster for the
// scores and its dims for the values:
//   0. every thread starts cp.async copies of this CTA's V slice (all keys,
//      dims [d0, d0 + dslice)) into shared memory;
//   A. thread = key of this CTA's key range: the eight chains of the dot
//      product (K row streamed with 16-byte loads), hsum256 order, *scale
//      (+mask); each CTA then gathers the other ranges through distributed
//      shared memory;
//   B. warp 0 replays the online softmax over the 64-key blocks in order
//      (every CTA of the cluster does, identically);
//   C. thread = dim of the slice: acc = acc*alpha_b, fma(V[j][d], p_j, acc)
//      over the keys in order, from shared memory.
// Requires D % 16 == 0 and 16-byte aligned V (the caller checks).
// The in-order value chain of one dim: acc = acc*alpha_b per active block,
// then acc = fma(V[j][d], p_j, acc) over its keys (p_j == 0 skipped).  With
// kSlice > 0 the V row stride is a compile-time constant and 16 keys' loads
// are issued ahead of their FMAs.
template <uint32_t kSlice>
__device__ __forceinline__ float value_chain(const float *Vs, const float *S, const float *alpha_b,
                                             const int *active_b, uint32_t nblk, uint32_t L,
                                             uint32_t d, uint32_t dslice = kSlice) {
    const uint32_t stride = kSlice ? kSlice : dslice;
    float a = 0.0f;
    for (uint32_t b = 0; b < nblk; ++b) {
        if (!active_b[b]) continue;
        a = __fmul_rn(a, alpha_b[b]);
        const uint32_t k0 = b * kAttBK, kc = min(kAttBK, L - k0);
        const float *vcol = Vs + static_cast<size_t>(k0) * stride + d;
        const float *prow = S + k0;
        uint32_t j = 0;
        for (; j + 16 <= kc; j += 16) {
            float pv[16], vv[16];
#pragma unroll
            for (uint32_t u = 0; u < 16; u += 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(prow + j + u);
                pv[u] = p4.x;
                pv[u + 1] = p4.y;
                pv[u + 2] = p4.z;
                pv[u + 3] = p4.w;
            }
#pragma unroll
            for (uint32_t u = 0; u < 16; ++u) vv[u] = vcol[(j + u) * stride];
#pragma unroll
            for (uint32_t u = 0; u < 16; ++u) a = fma_if_nonzero(vv[u], pv[u], a);
        }
        for (; j < kc; ++j) a = fma_if_nonzero(vcol[j * stride], prow[j], a);
    }
    return a;
}

constexpr uint32_t kDcCluster = 4;
constexpr uint32_t kDcThreads = 256;
constexpr size_t kDcMaxSmem = 200 * 1024;

// The dot product of one query and one key in the reference's AVX2 order:
// chain c (c = 0..7) accumulates elements 8t + c in t order, then
// ((c0+c4) + (c1+c5)) + ((c2+c6) + (c3+c7)).  kT > 0: D = 8 kT, every K load
// issued before the first FMA.
template <uint32_t kT>
__device__ __forceinline__ float dot_hsum256(const float *qs, const float *krow, uint32_t D) {
    float c[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const float4 *k4 = reinterpret_cast<const float4 *>(krow);
    const float4 *q4 = reinterpret_cast<const float4 *>(qs);
    if constexpr (kT > 0) {
        float4 kr[2 * kT];
#pragma unroll
        for (uint32_t i = 0; i < 2 * kT; ++i) kr[i] = __ldg(k4 + i);
#pragma unroll
        for (uint32_t t = 0; t < kT; ++t) {
            const float4 ka = kr[2 * t], kb = kr[2 * t + 1];
            const float4 qa = q4[2 * t], qb = q4[2 * t + 1];
            c[0] = __fmaf_rn(qa.x, ka.x, c[0]);
            c[1] = __fmaf_rn(qa.y, ka.y, c[1]);
            c[2] = __fmaf_rn(qa.z, ka.z, c[2]);
            c[3] = __fmaf_rn(qa.w, ka.w, c[3]);
            c[4] = __fmaf_rn(qb.x, kb.x, c[4]);
            c[5] = __fmaf_rn(qb.y, kb.y, c[5]);
            c[6] = __fmaf_rn(qb.z, kb.z, c[6]);
            c[7] = __fmaf_rn(qb.w, kb.w, c[7]);
        }
        return __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[4]), __fadd_rn(c[1], c[5])),
                         __fadd_rn(__fadd_rn(c[2], c[6]), __fadd_rn(c[3], c[7])));
    }
#pragma unroll 4
    for (uint32_t t = 0; t < D / 8; ++t) {
        const float4 ka = __ldg(k4 + 2 * t), kb = __ldg(k4 + 2 * t + 1);
        const float4 qa = q4[2 * t], qb = q4[2 * t + 1];
        c[0] = __fmaf_rn(qa.x, ka.x, c[0]);
        c[1] = __fmaf_rn(qa.y, ka.y, c[1]);
        c[2] = __fmaf_rn(qa.z, ka.z, c[2]);
        c[3] = __fmaf_rn(qa.w, ka.w, c[3]);
        c[4] = __fmaf_rn(qb.x, kb.x, c[4]);
        c[5] = __fmaf_rn(qb.y, kb.y, c[5]);
        c[6] = __fmaf_rn(qb.z, kb.z, c[6]);
        c[7] = __fmaf_rn(qb.w, kb.w, c[7]);
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[4]), __fadd_rn(c[1], c[5])),
                     __fadd_rn(__fadd_rn(c[2], c[6]), __fadd_rn(c[3], c[7])));
}

// dot_hsum256 with the key row in shared memory (plain loads).
__device__ __forceinline__ float dot_hsum256_shared(const float *qs, const float *krow,
                                                    uint32_t D) {
    float c[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const float4 *k4 = reinterpret_cast<const float4 *>(krow);
    const float4 *q4 = reinterpret_cast<const float4 *>(qs);
#pragma unroll 4
    for (uint32_t t = 0; t < D / 8; ++t) {
        const float4 ka = k4[2 * t], kb = k4[2 * t + 1];
        const float4 qa = q4[2 * t], qb = q4[2 * t + 1];
        c[0] = __fmaf_rn(qa.x, ka.x, c[0]);
        c[1] = __fmaf_rn(qa.y, ka.y, c[1]);
        c[2] = __fmaf_rn(qa.z, ka.z, c[2]);
        c[3] = __fmaf_rn(qa.w, ka.w, c[3]);
        c[4] = __fmaf_rn(qb.x, kb.x, c[4]);
        c[5] = __fmaf_rn(qb.y, kb.y, c[5]);
        c[6] = __fmaf_rn(qb.z, kb.z, c[6]);
        c[7] = __fmaf_rn(qb.w, kb.w, c[7]);
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[4]), __fadd_rn(c[1], c[5])),
                     __fadd_rn(__fadd_rn(c[2], c[6]), __fadd_rn(c[3], c[7])));
}

// Shared memory of the decode cluster kernel, in floats (the host sizes it
// with the same function): V slice [L][D/4], K rows of this CTA's key range
// [span][D+4], q [D], S [L], the compacted nonzero keys and probabilities
// [L] + [L], then per-block words and two mbarriers.
constexpr uint32_t kDcVBox = 64;   // V rows per TMA box
// This CTA's K rows, [span][D+4] (padded: no bank conflicts in the scores).
__host__ __device__ inline size_t dc_region_floats(uint32_t L, uint32_t D) {
    const size_t span = (L + kDcCluster - 1) / kDcCluster;
    return span * (D + 4);
}
__host__ __device__ inline size_t dc_smem_floats(uint32_t L, uint32_t D) {
    const size_t nblk = (L + kAttBK - 1) / kAttBK;
    const size_t vrows = (L + kDcVBox - 1) / kDcVBox * kDcVBox;   // whole boxes
    const size_t words = vrows * (D / kDcCluster) + dc_region_floats(L, D) + D + 3 * L + 6 * nblk + 1;
    return (words + 3) / 4 * 4 + 4;   // + two 8-byte mbarriers, 16-byte aligned
}

__global__ void __cluster_dims__(kDcCluster, 1, 1) __launch_bounds__(kDcThreads)
    attention_decode_cluster_kernel(const AttParams p, const __grid_constant__ CUtensorMap vmap) {
    pdl_enter();
    extern __shared__ __align__(16) float dc_smem[];
    const uint32_t D = p.D, L = p.seq_k;
    const uint32_t nblk = (L + kAttBK - 1) / kAttBK;
    const uint32_t dslice = D / kDcCluster;
    const uint32_t span = (L + kDcCluster - 1) / kDcCluster;
    const uint32_t kld = D + 4;                            // padded K row: no bank conflicts
    const uint32_t vboxes = (L + kDcVBox - 1) / kDcVBox;
    float *Vs = dc_smem;                                   // [vboxes * 64][dslice]
    float *Ks = Vs + static_cast<size_t>(vboxes) * kDcVBox * dslice;   // [span][kld]
    float *qs = Ks + dc_region_floats(L, D);               // [D]
    float *S = qs + D;                                     // [L]
    float *nz_p = S + L;                                   // [L] nonzero probabilities, per block
    int *nz_k = reinterpret_cast<int *>(nz_p + L);         // [L] their keys
    float *alpha_b = reinterpret_cast<float *>(nz_k + L);  // [nblk]
    int *active_b = reinterpret_cast<int *>(alpha_b + nblk);
    int *nz_cnt = active_b + nblk;                         // [nblk]
    float *nm_b = reinterpret_cast<float *>(nz_cnt + nblk);   // [nblk]
    float *sum_b = nm_b + nblk;                            // [nblk]
    float *l_sh = sum_b + nblk;
    uint64_t *bars = reinterpret_cast<uint64_t *>(dc_smem + dc_smem_floats(L, D) - 4);

    const uint32_t tid = threadIdx.x, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t bh = blockIdx.x / kDcCluster;
    const float *Qh = p.Q + static_cast<uint64_t>(bh) * D;
    const float *Kh = p.K + static_cast<uint64_t>(bh) * L * D;
    const float *Vh = p.V + static_cast<uint64_t>(bh) * L * D;
    const float *Mh = p.mask ? p.mask + static_cast<uint64_t>(bh) * L : nullptr;
    const uint32_t d0 = rank * dslice;
    const uint32_t k_lo = min(L, rank * span), k_hi = min(L, k_lo + span);
    const uint32_t krows = k_hi - k_lo;

    // 0. The TMA unit copies this CTA's K rows (one bulk copy per row, into
    //    padded rows) and its V slice (64-row boxes of the [rows][D] tensor
    //    map: the rows of this head, columns [d0, d0 + dslice)) into shared
    //    memory; bars[0] counts the K bytes, bars[1] the V bytes.
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bars[0], krows * D * 4u);
        mbar_arrive_expect_tx(&bars[1], vboxes * kDcVBox * dslice * 4u);
        for (uint32_t v = 0; v < vboxes; ++v)
            tma_load_2d(Vs + static_cast<size_t>(v) * kDcVBox * dslice, &vmap, &bars[1],
                        static_cast<int32_t>(d0), static_cast<int32_t>(bh * L + v * kDcVBox));
    }
    __syncthreads();
    for (uint32_t r = tid; r < krows; r += kDcThreads)
        bulk_load_1d(Ks + static_cast<size_t>(r) * kld, Kh + static_cast<uint64_t>(k_lo + r) * D,
                     D * 4u, &bars[0]);
    (void)Vh;
    for (uint32_t i = tid; i < D; i += kDcThreads) qs[i] = Qh[i];
    __syncthreads();
    // A timed-out wait leaves an error in the stream's word; the CTA carries
    // on to the cluster barriers so that its partners do not wait for it.
    mbar_wait(&bars[0], 0, p.wait_ns, p.err, nullptr);

    // A. scores of keys [k_lo, k_hi), from the K rows in shared memory
    for (uint32_t r = tid; r < krows; r += kDcThreads) {
        const float dot = dot_hsum256_shared(qs, Ks + static_cast<size_t>(r) * kld, D);
        float sc = __fmul_rn(dot, p.scale);
        if (Mh) sc = __fadd_rn(sc, Mh[k_lo + r]);
        S[k_lo + r] = sc;   // decode: the causal limit seq_k - 1 masks no key
    }
    cluster_sync_all();   // every range written
    for (uint32_t ki = tid; ki < L; ki += kDcThreads) {
        const uint32_t owner = ki / span;
        if (owner != rank) S[ki] = ld_shared_cluster_f32(mapa_shared(smem_addr(S + ki), owner));
    }
    cluster_sync_all();   // every gather done before S is overwritten below

    // B. online softmax.  The running max before block b is the max of the
    // finite block maxima up to b, so: (1) warps find every block's max;
    // (2) thread 0 walks the blocks for the running max and alpha;
    // (3) warps exponentiate and sum their blocks (each sum in key order)
    //     and list each block's nonzero probabilities in key order;
    // (4) thread 0 folds l = l*alpha + sum over the blocks in order.
    const uint32_t warp = tid >> 5;
    const float ninf = -__int_as_float(0x7f800000);
    for (uint32_t b = warp; b < nblk; b += kDcThreads / 32) {
        const uint32_t k0 = b * kAttBK, kc = min(kAttBK, L - k0);
        const float s_lo = lane < kc ? S[k0 + lane] : ninf;
        const float s_hi = lane + 32 < kc ? S[k0 + lane + 32] : ninf;
        float bmax = fmaxf(s_lo, s_hi);
        for (int o = 16; o > 0; o >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
        if (lane == 0) nm_b[b] = bmax;
    }
    __syncthreads();
    if (tid == 0) {
        float m_run = ninf;
        for (uint32_t b = 0; b < nblk; ++b) {
            const float bmax = nm_b[b];
            if (!isfinite(bmax)) {
                active_b[b] = 0;
                continue;
            }
            const float nm = fmaxf(m_run, bmax);
            alpha_b[b] = ref_fast_expf(__fsub_rn(m_run, nm), false);
            active_b[b] = 1;
            nm_b[b] = nm;
            m_run = nm;
        }
    }
    __syncthreads();
    for (uint32_t b = warp; b < nblk; b += kDcThreads / 32) {
        if (!active_b[b]) continue;
        const uint32_t k0 = b * kAttBK, kc = min(kAttBK, L - k0);
        const float nm = nm_b[b];
        const float p_lo = lane < kc ? ref_fast_expf(__fsub_rn(S[k0 + lane], nm), false) : 0.0f;
        const float p_hi =
            lane + 32 < kc ? ref_fast_expf(__fsub_rn(S[k0 + lane + 32], nm), false) : 0.0f;
        if (lane < kc) S[k0 + lane] = p_lo;
        if (lane + 32 < kc) S[k0 + lane + 32] = p_hi;
        float sum_p = 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < 32; ++j) {
            const float v = __shfl_sync(0xffffffffu, p_lo, j);
            if (j < kc) sum_p = __fadd_rn(sum_p, v);
        }
#pragma unroll
        for (uint32_t j = 0; j < 32; ++j) {
            const float v = __shfl_sync(0xffffffffu, p_hi, j);
            if (j + 32 < kc) sum_p = __fadd_rn(sum_p, v);
        }
        // The value chain skips p == 0 (as the reference does): keep the
        // others, in key order.
        const uint32_t m_lo = __ballot_sync(0xffffffffu, lane < kc && p_lo != 0.0f);
        const uint32_t m_hi = __ballot_sync(0xffffffffu, lane + 32 < kc && p_hi != 0.0f);
        const uint32_t below = (1u << lane) - 1u;
        if ((m_lo >> lane) & 1u) {
            const uint32_t at = k0 + __popc(m_lo & below);
            nz_p[at] = p_lo;
            nz_k[at] = static_cast<int>(k0 + lane);
        }
        if ((m_hi >> lane) & 1u) {
            const uint32_t at = k0 + __popc(m_lo) + __popc(m_hi & below);
            nz_p[at] = p_hi;
            nz_k[at] = static_cast<int>(k0 + lane + 32);
        }
        if (lane == 0) {
            sum_b[b] = sum_p;
            nz_cnt[b] = static_cast<int>(__popc(m_lo) + __popc(m_hi));
        }
    }
    __syncthreads();
    if (tid == 0) {
        float l_run = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b)
            if (active_b[b]) l_run = __fadd_rn(__fmul_rn(l_run, alpha_b[b]), sum_b[b]);
        *l_sh = l_run;
    }
    mbar_wait(&bars[1], 0, p.wait_ns, p.err, nullptr);
    __syncthreads();

    // C. values of dims [d0, d0 + dslice): acc = acc*alpha_b per active
    // block, then fma(V[k][d], p_k, acc) over the block's keys in order,
    // skipping p == 0: blocks without a zero run a plain FMA chain, the
    // others walk their list of nonzero keys.
    if (tid < dslice) {
        const float l = *l_sh;
        const float inv = l > 0.0f ? __fdiv_rn(1.0f, l) : 0.0f;
        const float *vcol = Vs + tid;   // V[k][d0 + tid] = vcol[k * dslice]
        float a = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b) {
            if (!active_b[b]) continue;
            a = __fmul_rn(a, alpha_b[b]);
            const uint32_t k0 = b * kAttBK, kc = min(kAttBK, L - k0);
            if (static_cast<uint32_t>(nz_cnt[b]) == kc) {
                // 16-key chunks, the next chunk's V values and probabilities
                // loaded while the current one runs through the chain.
                const uint32_t chunks = kc / 16;
                float vv[2][16], pv[2][16];
                auto load = [&](uint32_t c, float *v, float *pp) {
                    const uint32_t k = k0 + c * 16;
#pragma unroll
                    for (uint32_t u = 0; u < 16; ++u) v[u] = vcol[static_cast<size_t>(k + u) * dslice];
#pragma unroll
                    for (uint32_t q = 0; q < 4; ++q) {
                        const float4 p4 = *reinterpret_cast<const float4 *>(S + k + 4 * q);
                        pp[4 * q] = p4.x;
                        pp[4 * q + 1] = p4.y;
                        pp[4 * q + 2] = p4.z;
                        pp[4 * q + 3] = p4.w;
                    }
                };
                if (chunks) load(0, vv[0], pv[0]);
                for (uint32_t c = 0; c < chunks; c += 2) {
                    if (c + 1 < chunks) load(c + 1, vv[1], pv[1]);
#pragma unroll
                    for (uint32_t u = 0; u < 16; ++u) a = __fmaf_rn(vv[0][u], pv[0][u], a);
                    if (c + 1 >= chunks) break;
                    if (c + 2 < chunks) load(c + 2, vv[0], pv[0]);
#pragma unroll
                    for (uint32_t u = 0; u < 16; ++u) a = __fmaf_rn(vv[1][u], pv[1][u], a);
                }
                for (uint32_t k = k0 + chunks * 16; k < k0 + kc; ++k)
                    a = __fmaf_rn(vcol[static_cast<size_t>(k) * dslice], S[k], a);
                continue;
            }
            const uint32_t n = static_cast<uint32_t>(nz_cnt[b]);
            // Groups of 8 keys, the next group's keys, probabilities and V
            // values loaded while the current one runs through the chain.
            const uint32_t groups = n / 8;
            float pv[2][8], vv[2][8];
            auto load = [&](uint32_t g, float *pp, float *vp) {
                int kk[8];
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u) kk[u] = nz_k[k0 + g * 8 + u];
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u) {
                    pp[u] = nz_p[k0 + g * 8 + u];
                    vp[u] = vcol[static_cast<size_t>(kk[u]) * dslice];
                }
            };
            if (groups) load(0, pv[0], vv[0]);
            for (uint32_t g = 0; g < groups; g += 2) {
                if (g + 1 < groups) load(g + 1, pv[1], vv[1]);
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u) a = __fmaf_rn(vv[0][u], pv[0][u], a);
                if (g + 1 >= groups) break;
                if (g + 2 < groups) load(g + 2, pv[0], vv[0]);
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u) a = __fmaf_rn(vv[1][u], pv[1][u], a);
            }
            for (uint32_t i = groups * 8; i < n; ++i)
                a = __fmaf_rn(vcol[static_cast<size_t>(nz_k[k0 + i]) * dslice], nz_p[k0 + i], a);
        }
        p.O[static_cast<uint64_t>(bh) * D + d0 + tid] = __fmul_rn(a, inv);
    }
}

// QKV split + RoPE + KV append for T tokens (VNPU_B200_OP_QKV_ROPE_APPEND,
// T > 1): thread (head, pair j) of block (head group, part, token run) reads
// columns j and j + D/2 of the MATMUL_I8 output C [T][3*heads*D] for
// kQsTokens tokens, rotates Q and K exactly as rope_kernel does and writes
// the head-major outputs and the cache slot.  The inverse frequencies are
// copied to shared memory once per block (lanes index them by pair).
constexpr uint32_t kQsThreads = 256;
constexpr uint32_t kQsTokens = 8;

__global__ void __launch_bounds__(kQsThreads) qkv_split_rope_append_kernel(
    const float *__restrict__ C, uint32_t T, float *__restrict__ Q, float *__restrict__ Kout,
    float *__restrict__ Vout, float *__restrict__ Kc, float *__restrict__ Vc,
    float *__restrict__ mask, const int32_t *__restrict__ position, uint32_t heads, uint32_t D,
    uint32_t cap, uint32_t pos0, float scaling, const RopeFreq freq, uint32_t *err) {
    pdl_enter();
    __shared__ float inv_s[kRopeMaxPairs];
    const uint32_t half = D / 2;
    const uint32_t sec = blockIdx.y;
    if (sec < 2)
        for (uint32_t i = threadIdx.x; i < half; i += kQsThreads) inv_s[i] = freq.inv[i];
    __syncthreads();
    const uint32_t per_block = kQsThreads / half;          // heads per block (half <= 256)
    const uint32_t hl = threadIdx.x / half;
    const uint32_t j = threadIdx.x - hl * half;
    const uint32_t h = blockIdx.x * per_block + hl;
    if (hl >= per_block || h >= heads) return;
    const int32_t base = position ? *position : static_cast<int32_t>(pos0);
    const float inv = sec < 2 ? inv_s[j] : 0.0f;
    float *out = sec == 0 ? Q : (sec == 1 ? Kout : Vout);
    float *cache = sec == 1 ? Kc : Vc;
    const uint64_t ldc = 3ull * heads * D;
    const uint32_t t1 = min(T, (blockIdx.z + 1) * kQsTokens);
    for (uint32_t t = blockIdx.z * kQsTokens; t < t1; ++t) {
        const float *row = C + t * ldc + (static_cast<uint64_t>(sec) * heads + h) * D;
        float x0 = row[j], x1 = row[j + half];
        const int32_t pos = base + static_cast<int32_t>(t);
        if (sec < 2) {
            float v[2] = {x0, x1};
            rotate_pair(v, 0, 1, __fmul_rn(__fmul_rn(static_cast<float>(pos), scaling), inv));
            x0 = v[0];
            x1 = v[1];
        }
        const uint64_t o = (static_cast<uint64_t>(h) * T + t) * D + j;
        if (out) {
            out[o] = x0;
            out[o + half] = x1;
        }
        if (sec == 0) continue;
        if (pos < 0 || static_cast<uint32_t>(pos) >= cap) {
            if (sec == 1 && j == 0) record_error(err, kErrBadConfig);
            continue;
        }
        const uint64_t c = (static_cast<uint64_t>(h) * cap + static_cast<uint32_t>(pos)) * D + j;
        cache[c] = x0;
        cache[c + half] = x1;
        if (sec == 1 && j == 0 && mask)
            mask[static_cast<uint64_t>(h) * cap + static_cast<uint32_t>(pos)] = 0.0f;
    }
}

// KV-cache append: element (h, t, d) of K/V goes to slot pos + t of head h.
__global__ void kv_append_kernel(const float *__restrict__ K, const float *__restrict__ V,
                                 float *__restrict__ Kc, float *__restrict__ Vc,
                                 float *__restrict__ mask, const int32_t *__restrict__ position,
                                 uint32_t heads, uint32_t T, uint32_t D, uint32_t cap,
                                 uint32_t pos0, bool vec, uint32_t *err) {
    pdl_enter();
    const int64_t pos = position ? static_cast<int64_t>(*position) : static_cast<int64_t>(pos0);
    const uint32_t w = vec ? D / 4 : D;   // units per (h, t) row
    const uint64_t total = static_cast<uint64_t>(heads) * T * w;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t ht = i / w;
        const uint32_t u = static_cast<uint32_t>(i - ht * w);
        const uint32_t h = static_cast<uint32_t>(ht / T), t = static_cast<uint32_t>(ht % T);
        const int64_t slot = pos + t;
        if (slot < 0 || slot >= static_cast<int64_t>(cap)) {
            if (u == 0) record_error(err, kErrBadConfig);
            continue;
        }
        const uint64_t dst = (static_cast<uint64_t>(h) * cap + static_cast<uint64_t>(slot)) * w + u;
        if (vec) {
            reinterpret_cast<float4 *>(Kc)[dst] = __ldg(reinterpret_cast<const float4 *>(K) + i);
            reinterpret_cast<float4 *>(Vc)[dst] = __ldg(reinterpret_cast<const float4 *>(V) + i);
        } else {
            Kc[dst] = __ldg(K + i);
            Vc[dst] = __ldg(V + i);
        }
        if (mask && u == 0) mask[static_cast<uint64_t>(h) * cap + static_cast<uint64_t>(slot)] = 0.0f;
    }
}

// Spins on a flag nothing sets, bounded by limit_ns: the device-side wait
// pattern of the GEMM pipeline, exercised on its own.
__global__ void wait_probe_kernel(const uint32_t *flag, uint64_t limit_ns, uint32_t *err) {
    const uint64_t start = global_timer_ns();
    while (true) {
        if (*reinterpret_cast<const volatile uint32_t *>(flag) != 0u) return;
        if (global_timer_ns() - start > limit_ns) {
            record_error(err, kErrWaitTimeout);
            return;
        }
        __nanosleep(1000);
    }
}

unsigned grid_for(uint64_t n, int num_sms, unsigned threads) {
    const uint64_t want = (n + threads - 1) / threads;
    const uint64_t cap = static_cast<uint64_t>(num_sms) * 16;
    return static_cast<unsigned>(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

cudaError_t rmsnorm(const LaunchCtx &ctx, const float *X, const float *W, float *Y,
                    uint32_t rows, uint32_t cols, float eps) {
    if (cols <= kRmsRowMaxCols && std::getenv("VNPU_B200_RMSNORM_WARP") == nullptr) {
        const size_t smem = sizeof(float) * cols;
        if (smem > 48 * 1024) {
            static bool configured[64] = {};
            int dev = 0;
            cudaGetDevice(&dev);
            if (dev >= 0 && dev < 64 && !configured[dev]) {
                const cudaError_t e = cudaFuncSetAttribute(
                    rmsnorm_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                    static_cast<int>(sizeof(float) * kRmsRowMaxCols));
                if (e != cudaSuccess) return e;
                configured[dev] = true;
            }
        }
        const bool vec = cols % 8 == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(Y) & 15u) == 0;
        VNPU_LAUNCH(launch_pdl(ctx.stream, rmsnorm_row_kernel, dim3(rows), dim3(kRmsRowThreads), smem, X, W, Y, cols, eps, vec));
    } else {
        const unsigned blocks = (rows + 7) / 8;
        VNPU_LAUNCH(launch_pdl(ctx.stream, rmsnorm_kernel, dim3(blocks), dim3(256), 0, X, W, Y, rows, cols, eps));
    }
    count_launch(ctx);
    return cudaGetLastError();
}

namespace {
// Cluster size for a fused row prologue: split rows only while there are too
// few of them to occupy the SMs.
uint32_t fq_cluster(const LaunchCtx &ctx, uint32_t rows) {
    if (const char *e = std::getenv("VNPU_B200_FUSED_CLUSTER")) {
        const unsigned long c = std::strtoul(e, nullptr, 10);
        if (c == 1 || c == 2 || c == 4 || c == 8) return static_cast<uint32_t>(c);
    }
    if (rows >= static_cast<uint32_t>(ctx.num_sms)) return 1;
    if (rows * 2 >= static_cast<uint32_t>(ctx.num_sms)) return 2;
    if (rows * 4 >= static_cast<uint32_t>(ctx.num_sms)) return 4;
    return kFqMaxCluster;
}

template <typename Kernel, typename... Args>
cudaError_t launch_fq(const LaunchCtx &ctx, Kernel kernel, uint32_t rows, uint32_t csize,
                      size_t smem, Args... args) {
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows * csize, 1, 1);
    cfg.blockDim = dim3(kFqThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_allowed() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}
}  // namespace

cudaError_t rmsnorm_quantize(const LaunchCtx &ctx, const float *X, const float *W, float *Y,
                             int8_t *Q, float *scales, uint32_t rows, uint32_t cols, float eps) {
    if (cols > kRmsRowMaxCols || rows == 0 || rows > 0x0fffffffu) return cudaErrorInvalidValue;
    const uint32_t csize = fq_cluster(ctx, rows);
    const bool vec = cols % 8 == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0;
    const cudaError_t e = launch_fq(ctx, rmsnorm_quantize_kernel, rows, csize, sizeof(float) * cols,
                                    X, W, Y, Q, scales, cols, eps, vec);
    count_launch(ctx);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t swiglu_quantize(const LaunchCtx &ctx, const float *gate, const float *up, float *Y,
                            int8_t *Q, float *scales, uint32_t rows, uint32_t cols, uint32_t ld,
                            float alpha) {
    if (cols > kRmsRowMaxCols || rows == 0 || rows > 0x0fffffffu || ld < cols)
        return cudaErrorInvalidValue;
    const uint32_t csize = fq_cluster(ctx, rows);
    const size_t slice = ((cols + csize - 1) / csize + 15u) & ~15u;
    const cudaError_t e = launch_fq(ctx, swiglu_quantize_kernel, rows, csize, sizeof(float) * slice,
                                    gate, up, Y, Q, scales, cols, ld, alpha);
    count_launch(ctx);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t rope(const LaunchCtx &ctx, float *Q, float *K, const int32_t *positions,
                 uint32_t batch, uint32_t heads, uint32_t q_seq, uint32_t k_seq,
                 uint32_t head_dim, uint32_t position_offset, uint32_t interleaved,
                 float scaling, const float *inv_freq_host) {
    if (head_dim / 2 > kRopeMaxPairs) return cudaErrorInvalidValue;
    RopeFreq f;
    for (uint32_t j = 0; j < head_dim / 2; ++j) f.inv[j] = inv_freq_host[j];
    const uint64_t total = static_cast<uint64_t>(batch) * heads * (q_seq > k_seq ? q_seq : k_seq) *
                           (head_dim / 2);
    VNPU_LAUNCH(launch_pdl(ctx.stream, rope_kernel, dim3(grid_for(total, ctx.num_sms, 256)), dim3(256), 0, 
        Q, K, positions, batch * heads, q_seq, k_seq, head_dim, position_offset, interleaved,
        scaling, f));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t qkv_split_rope_append(const LaunchCtx &ctx, const float *C, uint32_t T,
                                  const QkvRope &q) {
    if (q.head_dim == 0 || (q.head_dim & 1u) || q.head_dim / 2 > kRopeMaxPairs || T == 0)
        return cudaErrorInvalidValue;
    RopeFreq f;
    for (uint32_t j = 0; j < q.head_dim / 2; ++j) f.inv[j] = q.inv_freq[j];
    const uint32_t per_block = kQsThreads / (q.head_dim / 2);
    const uint32_t runs = (T + kQsTokens - 1) / kQsTokens;
    if (runs > 65535u) return cudaErrorInvalidValue;
    const dim3 grid((q.heads + per_block - 1) / per_block, 3, runs);
    VNPU_LAUNCH(launch_pdl(ctx.stream, qkv_split_rope_append_kernel, grid, dim3(kQsThreads), 0,
                           C, T, q.Q, q.K_out, q.V_out, q.K_cache, q.V_cache, q.mask, q.position,
                           q.heads, q.head_dim, q.capacity, q.position_offset, q.scaling, f,
                           ctx.err));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t swiglu_rows(const LaunchCtx &ctx, const float *C, uint32_t ldc, float *Y, uint32_t ldy,
                        uint32_t rows, uint32_t I, float alpha) {
    const uint64_t n = static_cast<uint64_t>(rows) * I;
    if (n == 0) return cudaSuccess;
    if (ctx.launch_counter) ++*ctx.launch_counter;
    return launch_pdl(ctx.stream, swiglu_rows_kernel, dim3(grid_for(n, ctx.num_sms, 256)), dim3(256),
                      0, C, ldc, Y, ldy, rows, I, alpha);
}

cudaError_t swiglu(const LaunchCtx &ctx, const float *gate, const float *up, float *Y,
                   uint64_t count, float alpha) {
    const bool vec = count % 4 == 0 && (reinterpret_cast<uintptr_t>(gate) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(up) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(Y) & 15) == 0;
    if (vec)
        VNPU_LAUNCH(launch_pdl(ctx.stream, swiglu_vec_kernel, dim3(grid_for(count / 4, ctx.num_sms, 256)), dim3(256), 0, 
            reinterpret_cast<const float4 *>(gate), reinterpret_cast<const float4 *>(up),
            reinterpret_cast<float4 *>(Y), count / 4, alpha));
    else
        VNPU_LAUNCH(launch_pdl(ctx.stream, swiglu_kernel, dim3(grid_for(count, ctx.num_sms, 256)), dim3(256), 0, gate, up, Y,
                                                                                 count, alpha));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t add(const LaunchCtx &ctx, const float *A, const float *B, float *Y, uint64_t count,
                float alpha, float beta) {
    const bool vec = count % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(B) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(Y) & 15) == 0;
    if (vec)
        VNPU_LAUNCH(launch_pdl(ctx.stream, add_vec_kernel, dim3(grid_for(count / 4, ctx.num_sms, 256)), dim3(256), 0, 
            reinterpret_cast<const float4 *>(A), reinterpret_cast<const float4 *>(B),
            reinterpret_cast<float4 *>(Y), count / 4, alpha, beta));
    else
        VNPU_LAUNCH(launch_pdl(ctx.stream, add_kernel, dim3(grid_for(count, ctx.num_sms, 256)), dim3(256), 0, A, B, Y, count,
                                                                              alpha, beta));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t attention(const LaunchCtx &ctx, const float *Q, const float *K, const float *V,
                      const float *mask, float *O, uint32_t batch, uint32_t heads,
                      uint32_t seq_q, uint32_t seq_k, uint32_t head_dim, uint32_t causal,
                      float scale, bool o_token_major) {
    if (head_dim > kAttMaxD || head_dim == 0) return cudaErrorInvalidValue;
    const size_t smem =
        sizeof(float) * (kAttBQ * att_q_stride(head_dim) + kAttBK * head_dim + kAttBQ * kAttBK);
    const bool vec = head_dim % 4 == 0 && (reinterpret_cast<uintptr_t>(V) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(O) & 15) == 0;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const int max_smem = static_cast<int>(sizeof(float) * (kAttBQ * att_q_stride(kAttMaxD) +
                                                               kAttBK * kAttMaxD + kAttBQ * kAttBK));
        cudaError_t e = cudaFuncSetAttribute(attention_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attention_kernel<false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    AttParams ap;
    ap.Q = Q;
    ap.K = K;
    ap.V = V;
    ap.mask = mask;
    ap.O = O;
    ap.heads = heads;
    ap.seq_q = seq_q;
    ap.seq_k = seq_k;
    ap.D = head_dim;
    ap.causal = causal;
    ap.scale = scale;
    ap.o_tokens = o_token_major ? 1u : 0u;
    ap.err = ctx.err;
    ap.wait_ns = ctx.wait_limit_ns;
    const char *attn_env = std::getenv("VNPU_B200_ATTN");   // general | decode | cluster
    const bool force_general = attn_env && !std::strcmp(attn_env, "general");
    const bool allow_cluster = !(attn_env && !std::strcmp(attn_env, "decode"));
    const size_t dc_smem = sizeof(float) * dc_smem_floats(seq_k, head_dim);
    if (seq_q == 1 && !force_general && allow_cluster && head_dim % 16 == 0 &&
        (reinterpret_cast<uintptr_t>(V) & 15) == 0 && (reinterpret_cast<uintptr_t>(K) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(Q) & 15) == 0 && dc_smem <= kDcMaxSmem) {
        static bool dc_configured[64] = {};
        if (dev >= 0 && dev < 64 && !dc_configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(attention_decode_cluster_kernel,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(kDcMaxSmem));
            if (e != cudaSuccess) return e;
            dc_configured[dev] = true;
        }
        CUtensorMap vmap;
        if (!encode_tmap_2d(&vmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, V, head_dim,
                            static_cast<uint64_t>(batch) * heads * seq_k, head_dim * 4ull,
                            head_dim / kDcCluster, kDcVBox, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
        VNPU_LAUNCH(launch_pdl(ctx.stream, attention_decode_cluster_kernel,
                               dim3(batch * heads * kDcCluster), dim3(kDcThreads), dc_smem, ap,
                               vmap));
        count_launch(ctx);
        return cudaGetLastError();
    }
    if (seq_q == 1 && seq_k <= kDecMaxKeys && !force_general) {
        const uint32_t nblk = (seq_k + kAttBK - 1) / kAttBK;
        const size_t dsmem = sizeof(float) * (seq_k + nblk + nblk + 1 + head_dim);
        static bool dec_configured[64] = {};
        if (dev >= 0 && dev < 64 && !dec_configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(
                attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                static_cast<int>(sizeof(float) * (kDecMaxKeys + 2 * (kDecMaxKeys / kAttBK) + 1 +
                                                  kAttMaxD)));
            if (e != cudaSuccess) return e;
            dec_configured[dev] = true;
        }
        VNPU_LAUNCH(launch_pdl(ctx.stream, attention_decode_kernel, dim3(batch * heads), dim3(kDecThreads), dsmem, ap));
        count_launch(ctx);
        return cudaGetLastError();
    }
    dim3 grid((seq_q + kAttBQ - 1) / kAttBQ, batch * heads);
    const bool aligned_all = ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
                               reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(O)) &
                              15u) == 0;
    if (head_dim == kApD && aligned_all && (seq_q + kApBQ - 1) / kApBQ <= 65535u &&
        !(attn_env && !std::strcmp(attn_env, "general"))) {
        // (batch*head, 64-query block): blocks are dispatched x-fastest, so
        // every head's longest causal block comes before any shorter one
        const dim3 ap_grid(batch * heads, (seq_q + kApBQ - 1) / kApBQ);
        const size_t ap_smem = sizeof(float) * kApSmemFloats;
        static bool ap_configured[64] = {};
        if (dev >= 0 && dev < 64 && !ap_configured[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(
                attention_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                static_cast<int>(ap_smem));
            if (e != cudaSuccess) return e;
            ap_configured[dev] = true;
        }
        VNPU_LAUNCH(launch_pdl(ctx.stream, attention_prefill_kernel, ap_grid, dim3(kApThreads),
                               ap_smem, ap));
        count_launch(ctx);
        return cudaGetLastError();
    }
    if (vec)
        VNPU_LAUNCH(launch_pdl(ctx.stream, attention_kernel<true>, dim3(grid), dim3(kAttThreads), smem, ap));
    else
        VNPU_LAUNCH(launch_pdl(ctx.stream, attention_kernel<false>, dim3(grid), dim3(kAttThreads), smem, ap));
    count_launch(ctx);
    return cudaGetLastError();
}

// The decoder block's device-side position: *pos = value (set) or *pos +=
// value (advance), one thread; and the cache mask filled with -inf.
__global__ void block_position_kernel(int32_t *pos, int32_t value, uint32_t advance) {
    pdl_enter();
    if (threadIdx.x == 0) *pos = advance ? *pos + value : value;
}

__global__ void fill_neg_inf_kernel(float *p, uint64_t n) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        p[i] = -INFINITY;
}

cudaError_t block_position(const LaunchCtx &ctx, int32_t *pos, int32_t value, bool advance) {
    count_launch(ctx);
    return launch_pdl(ctx.stream, block_position_kernel, dim3(1), dim3(32), 0, pos, value,
                      advance ? 1u : 0u);
}

cudaError_t fill_neg_inf(const LaunchCtx &ctx, float *p, uint64_t n) {
    if (n == 0) return cudaSuccess;
    count_launch(ctx);
    fill_neg_inf_kernel<<<grid_for(n, ctx.num_sms, 256), 256, 0, ctx.stream>>>(p, n);
    return cudaGetLastError();
}

cudaError_t kv_append(const LaunchCtx &ctx, const float *K, const float *V, float *K_cache,
                      float *V_cache, float *mask, const int32_t *position, uint32_t heads,
                      uint32_t T, uint32_t head_dim, uint32_t capacity, uint32_t position_offset) {
    const bool vec = head_dim % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V) |
                       reinterpret_cast<uintptr_t>(K_cache) | reinterpret_cast<uintptr_t>(V_cache)) &
                      15u) == 0;
    const uint64_t total = static_cast<uint64_t>(heads) * T * (vec ? head_dim / 4 : head_dim);
    VNPU_LAUNCH(launch_pdl(ctx.stream, kv_append_kernel, dim3(grid_for(total, ctx.num_sms, 256)), dim3(256), 0, 
        K, V, K_cache, V_cache, mask, position, heads, T, head_dim, capacity, position_offset, vec,
        ctx.err));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t wait_timeout_probe(const LaunchCtx &ctx, const uint32_t *flag, uint64_t limit_ns) {
    wait_probe_kernel<<<1, 1, 0, ctx.stream>>>(flag, limit_ns, ctx.err);
    count_launch(ctx);
    return cudaGetLastError();
}

}  // namespace vnpu_b200
