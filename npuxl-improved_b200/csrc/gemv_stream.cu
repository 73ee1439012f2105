// gemv_stream.cu - MATMUL_I8 for M <= 8 (the decode GEMV) with the weights
// landed in shared memory by cp.async before the programmatic wait for the
// previous kernel: one column per warp with __dp4a products (M <= 2), and
// 8-column groups with the products on mma.sync (M <= 8, below).
//
// Bound: HBM.  A decode GEMV reads every weight byte once (K*N int8) plus a
// few KB of activations, so its time is the weight stream plus fixed costs
// per launch: the launch itself, the first DRAM round trip and the wait for
// the previous kernel.  In a chain of kernels on one stream (programmatic
// dependent launch, triggered at entry) this kernel's CTAs become resident
// while the previous kernel still runs, and each warp issues the copies of
// its whole column (k_stride bytes, 16 bytes a lane per cp.async) into its
// own slice of shared memory at once: the weights do not depend on the
// previous kernel, the activations and the output do.  A warp waits only for
// the copies it issued itself, reads back only the chunks it copied
// (k = lane * 16 + 512 j), multiplies them with the activation row(s) by
// __dp4a (exact int32), reduces over its lanes and applies store_i8_c's
// dequant epilogue (src/kernels/kernels.cpp:526-535) in the element's
// reference form.  Shared memory rather than registers holds the prefetched
// bytes, so the next kernel of the stream also fits beside this one.
//
// Epilogue variants: plain, residual (C = R + out, ADD_F32's rounding), and
// the QKV projection of one token (VNPU_B200_OP_QKV_ROPE_APPEND), where a
// warp owns the two columns of a rotation pair (j, j + D/2 of one head) so
// lane 0 can rotate them as ROPE_F32 does and place them as KV_APPEND does.
//
// Measured alternatives (B200, 4096 x 4096, graph of 32 launches over 32
// weight copies): registers as the landing buffer 3.6-4.0 us; a producer
// warp feeding a ring of shared-memory stages (TMA cp.async.bulk or cp.async,
// consumer warps splitting K) 11.5 us; L2 prefetch at entry then loads from
// L2 4.2 us; a K split where each thread copies its own chunks of every
// column of a CTA-wide range 4.5 us; this kernel 3.6 us with a bare store and
// 3.95 us with the full dequant epilogue (the epilogue is on the critical
// path of a chain of dependent kernels), against 3.96 us for the register-
// streaming GEMV; at 4096 x 12288 / 4096 x 22016 10.2 / 15.9 us against
// 10.9 / 16.1 us.  The activation chunks are read by plain batched loads and
// the epilogue's scales and bias are fetched before the products: byte-wise
// guarded loads and fetching them after cost 4.4 -> 3.95 us and 14.8 ->
// 10.8 us at K = 11008.
//
// The mma.sync kernel (graph of launches over distinct weights, bias, no
// activation): 4096 x 4096 at M = 1 / 4 / 8 3.73 / 3.71 / 3.89 us, against
// 3.91 us for the one-column kernel at M = 1 and 6.5 / 7.3 us for the
// tcgen05 swap-AB GEMV at M = 4 / 8; 4096 x 12288 and 4096 x 22016 at M = 8
// 11.2 / 18.1 us with one group per CTA.  Activations staged in shared
// memory instead of registers, four warps per CTA, or four groups per CTA
// all measured slower; K = 11008 (88 KiB of weights per 8 columns) is
// faster on the register-streaming GEMV.  Landing only the first 7/8, 6/8 or
// 5/8 of each warp's chunks before the programmatic wait (the rest read from
// global memory after it, 64 registers, four CTAs per SM, so every CTA of
// the next launch fits beside this one's) took 4.7 / 6.8 / 7.3 us at
// 4096 x 4096, M = 1, against 3.63 us landing all of it: the loads after the
// wait put a DRAM round trip on the critical path behind the previous kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace vnpu_b200 {

namespace {

constexpr uint32_t kGsWarps = 8;                      // warps (columns) per CTA
constexpr uint32_t kGsThreads = kGsWarps * 32;
constexpr uint32_t kGsMaxSmem = 200u * 1024u;         // largest shared slice set per CTA
constexpr uint32_t kGsMaxPairs = 256;                 // head_dim / 2 of the QKV variant

struct GsParams {
    const int8_t *A;
    uint32_t lda;
    const int8_t *Bt;
    uint32_t k_stride;
    const float *scale_a;
    const float *scale_b;
    const float *bias;
    float *C;
    uint32_t ldc;
    uint32_t M, K, N;
    uint32_t epilogue;
    FormMap fmap;
};

struct GsPlain {};
// C = R + out; *advance_pos += advance (when not NULL) once the previous
// kernels of the stream are complete (MATMUL_I8_RESIDUAL's
// VNPU_B200_CMD_FLAG_ADVANCE_POSITION).
struct GsResidual {
    const float *R;
    uint32_t ldr;
    int32_t *advance_pos;
    int32_t advance;
};

template <typename Extra>
__device__ __forceinline__ void gs_advance(const Extra &x) {
    if constexpr (std::is_same<Extra, GsResidual>::value)
        if (x.advance_pos && blockIdx.x == 0 && threadIdx.x == 0) *x.advance_pos += x.advance;
}
struct GsQkv {
    float *Q, *Kout, *Vout, *Kc, *Vc, *mask;
    const int32_t *position;
    uint32_t *err;
    uint32_t heads, D, cap, pos0;
    float scaling;
    float inv[kGsMaxPairs];   // 1 / theta^(2j/D), computed on the host like ROPE_F32
};

// 16 activation bytes of row m at k (zeros past K; the packed weights are zero there too).
__device__ __forceinline__ int4 gs_act16(const GsParams &p, uint32_t m, uint32_t k) {
    if (k >= p.K) return make_int4(0, 0, 0, 0);
    const int8_t *row = p.A + static_cast<uint64_t>(m) * p.lda;
    if (k + 16u <= p.K) return __ldg(reinterpret_cast<const int4 *>(row + k));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (uint32_t b = 0; b < 16u; ++b)
        if (k + b < p.K)
            w[b >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(row[k + b])) << (8u * (b & 3u));
    return make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]), static_cast<int>(w[2]),
                     static_cast<int>(w[3]));
}

// The gate/up projection with its SwiGLU (VNPU_B200_OP_MATMUL_I8_SWIGLU): a
// warp owns gate column j and up column I + j of the [K][2I] weight and
// writes Y[m][j] = swiglu(gate, up) * alpha.
struct GsSwiglu {
    float *Y;
    uint32_t ldy;
    uint32_t I;
    float alpha;
};

// The rotation pair a warp of the QKV variant owns: section (Q, K, V), head,
// index j < D/2, and the first column (the second is D/2 further).
__device__ __forceinline__ void gs_qkv_pair(const GsQkv &x, uint32_t pair, uint32_t &sec,
                                            uint32_t &h, uint32_t &j, uint32_t &n0) {
    const uint32_t half = x.D / 2, per_sec = x.heads * half;
    sec = pair / per_sec;
    const uint32_t r = pair - sec * per_sec;
    h = r / half;
    j = r - h * half;
    n0 = sec * x.heads * x.D + h * x.D + j;
}

// kC columns per warp (2 for the QKV variant), kM rows.  Dynamic shared
// memory: kGsWarps * kC slices of k_stride bytes.
template <int kM, int kC, typename Extra>
__global__ void __launch_bounds__(kGsThreads) gemv_i8_stream_kernel(const GsParams p,
                                                                   const Extra x) {
    constexpr bool kQkv = std::is_same<Extra, GsQkv>::value;
    constexpr bool kSw = std::is_same<Extra, GsSwiglu>::value;
    static_assert(!kQkv || (kM == 1 && kC == 2), "the QKV epilogue is one token, column pairs");
    static_assert(!kSw || kC == 2, "the SwiGLU epilogue pairs a gate and an up column");
    extern __shared__ __align__(16) uint8_t gs_smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t ncol[kC];
    bool warp_valid = true;
    uint32_t q_sec = 0, q_h = 0, q_j = 0;
    if constexpr (kQkv) {
        const uint32_t pair = blockIdx.x * kGsWarps + warp;
        warp_valid = pair < 3u * x.heads * (x.D / 2u);
        uint32_t n0 = 0;
        if (warp_valid) gs_qkv_pair(x, pair, q_sec, q_h, q_j, n0);
        ncol[0] = n0;
        ncol[1] = n0 + x.D / 2u;
    } else if constexpr (kSw) {
        const uint32_t j = blockIdx.x * kGsWarps + warp;
        warp_valid = j < x.I;
        ncol[0] = j;
        ncol[1] = x.I + j;
    } else {
#pragma unroll
        for (int c = 0; c < kC; ++c) ncol[c] = (blockIdx.x * kGsWarps + warp) * kC + c;
    }
    // Copy this warp's columns; every lane copies (and later reads) only its
    // own 16-byte chunks, so no lane waits for another's data.
    uint8_t *slice = gs_smem + static_cast<size_t>(warp) * kC * p.k_stride;
#pragma unroll
    for (int c = 0; c < kC; ++c) {
        if (warp_valid && ncol[c] < p.N) {
            const int8_t *src = p.Bt + static_cast<uint64_t>(ncol[c]) * p.k_stride;
            for (uint32_t k = lane * 16u; k < p.k_stride; k += 512u)
                cp_async_16(slice + c * p.k_stride + k, src + k);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // The stream's next kernel may start now; the activations, the scales,
    // the bias and C may belong to the previous one.
    pdl_enter();
    gs_advance(x);
    // Lane 0 fetches the epilogue's operands now, so their latency overlaps
    // the products instead of following them.
    const bool has_bias = p.bias != nullptr;
    float e_sa[kM], e_sb[kC], e_bias[kC];
    int32_t e_pos = 0;
    if (lane == 0 && warp_valid) {
#pragma unroll
        for (int m = 0; m < kM; ++m) e_sa[m] = p.scale_a ? __ldg(p.scale_a + m) : 1.0f;
#pragma unroll
        for (int c = 0; c < kC; ++c) {
            const uint32_t n = ncol[c] < p.N ? ncol[c] : 0u;
            e_sb[c] = __ldg(p.scale_b + n);
            e_bias[c] = has_bias ? __ldg(p.bias + n) : 0.0f;
        }
        if constexpr (kQkv) e_pos = x.position ? *x.position : static_cast<int32_t>(x.pos0);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    int32_t acc[kC][kM];
#pragma unroll
    for (int c = 0; c < kC; ++c)
#pragma unroll
        for (int m = 0; m < kM; ++m) acc[c][m] = 0;
    // Whole 16-byte chunks by plain loads the compiler can batch; the ragged
    // chunk past the last multiple of 16 (if any) byte by byte.
    const uint32_t k16 = p.K & ~15u;
    auto mac = [&](const int4 (&a)[kM], uint32_t k) {
#pragma unroll
        for (int c = 0; c < kC; ++c) {
            const int4 w = *reinterpret_cast<const int4 *>(slice + c * p.k_stride + k);
#pragma unroll
            for (int m = 0; m < kM; ++m) {
                int s = acc[c][m];
                s = __dp4a(a[m].x, w.x, s);
                s = __dp4a(a[m].y, w.y, s);
                s = __dp4a(a[m].z, w.z, s);
                s = __dp4a(a[m].w, w.w, s);
                acc[c][m] = s;
            }
        }
    };
#pragma unroll 4
    for (uint32_t k = lane * 16u; k < k16; k += 512u) {
        int4 a[kM];
#pragma unroll
        for (int m = 0; m < kM; ++m)
            a[m] = __ldg(reinterpret_cast<const int4 *>(p.A + static_cast<uint64_t>(m) * p.lda + k));
        mac(a, k);
    }
    if (k16 < p.K && lane == (k16 / 16u) % 32u) {
        int4 a[kM];
#pragma unroll
        for (int m = 0; m < kM; ++m) a[m] = gs_act16(p, m, k16);
        mac(a, k16);
    }
#pragma unroll
    for (int c = 0; c < kC; ++c)
#pragma unroll
        for (int m = 0; m < kM; ++m)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                acc[c][m] += __shfl_xor_sync(0xffffffffu, acc[c][m], o);
    if (lane != 0 || !warp_valid) return;
    if constexpr (kQkv) {
        // Both columns of the pair: dequantize as MATMUL_I8 would, rotate Q/K
        // as ROPE_F32 does (src/kernels/llm.cpp:188-217), place as KV_APPEND.
        float v[2];
#pragma unroll
        for (int c = 0; c < 2; ++c)
            v[c] = ref_dequant(acc[c][0], e_sa[0], e_sb[c], has_bias, e_bias[c], p.epilogue,
                               form_at(p.fmap, 0u, ncol[c]));
        const int32_t pos = e_pos;
        if (q_sec < 2) {
            const float angle = __fmul_rn(__fmul_rn(static_cast<float>(pos), x.scaling), x.inv[q_j]);
            float sn, cs;
            sincosf(angle, &sn, &cs);
            const float x0 = v[0], x1 = v[1];
            v[0] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            v[1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        const uint64_t row = static_cast<uint64_t>(q_h) * x.D + q_j;   // [h][t = 0][j]
        const uint32_t half = x.D / 2;
        if (q_sec == 0) {
            x.Q[row] = v[0];
            x.Q[row + half] = v[1];
            return;
        }
        float *out = q_sec == 1 ? x.Kout : x.Vout;
        if (out) {
            out[row] = v[0];
            out[row + half] = v[1];
        }
        if (pos < 0 || static_cast<uint32_t>(pos) >= x.cap) {
            if (q_sec == 1 && q_j == 0) record_error(x.err, kErrBadConfig);
            return;
        }
        const uint64_t slot = (static_cast<uint64_t>(q_h) * x.cap + static_cast<uint32_t>(pos)) * x.D + q_j;
        float *cache = q_sec == 1 ? x.Kc : x.Vc;
        cache[slot] = v[0];
        cache[slot + half] = v[1];
        if (q_sec == 1 && q_j == 0 && x.mask)
            x.mask[static_cast<uint64_t>(q_h) * x.cap + static_cast<uint32_t>(pos)] = 0.0f;
        return;
    } else if constexpr (kSw) {
        // Gate and up dequantised as MATMUL_I8 would, then SWIGLU_F32's
        // expression (src/kernels/llm.cpp:289-306).
#pragma unroll
        for (int m = 0; m < kM; ++m) {
            const float g = ref_dequant(acc[0][m], e_sa[m], e_sb[0], has_bias, e_bias[0],
                                        p.epilogue, form_at(p.fmap, static_cast<uint32_t>(m), ncol[0]));
            const float u = ref_dequant(acc[1][m], e_sa[m], e_sb[1], has_bias, e_bias[1],
                                        p.epilogue, form_at(p.fmap, static_cast<uint32_t>(m), ncol[1]));
            const float s = __fdiv_rn(g, __fadd_rn(1.0f, ref_exp256_lane(-g)));
            x.Y[static_cast<uint64_t>(m) * x.ldy + ncol[0]] = __fmul_rn(__fmul_rn(s, u), x.alpha);
        }
    } else {
#pragma unroll
        for (int c = 0; c < kC; ++c) {
            const uint32_t n = ncol[c];
            if (n >= p.N) continue;
#pragma unroll
            for (int m = 0; m < kM; ++m) {
                float out = ref_dequant(acc[c][m], e_sa[m], e_sb[c], has_bias, e_bias[c],
                                        p.epilogue, form_at(p.fmap, static_cast<uint32_t>(m), n));
                if constexpr (std::is_same<Extra, GsResidual>::value)
                    out = __fadd_rn(x.R[static_cast<uint64_t>(m) * x.ldr + n], out);
                p.C[static_cast<uint64_t>(m) * p.ldc + n] = out;
            }
        }
    }
}

template <int kM, int kC, typename Extra>
cudaError_t gs_launch(const LaunchCtx &ctx, const GsParams &g, uint32_t grid, const Extra &x) {
    static std::mutex mu;
    static bool opted[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    {
        std::lock_guard<std::mutex> l(mu);
        if (dev < 0 || dev >= 64 || !opted[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(gemv_i8_stream_kernel<kM, kC, Extra>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(kGsMaxSmem));
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) opted[dev] = true;
        }
    }
    const uint32_t smem = kGsWarps * kC * g.k_stride;
    if (ctx.launch_counter) ++*ctx.launch_counter;
    return launch_pdl(ctx.stream, gemv_i8_stream_kernel<kM, kC, Extra>, dim3(grid),
                      dim3(kGsThreads), smem, g, x);
}

// ---------------------------------------------------------------------------
// M = 3..8: the products on the tensor core by mma.sync m16n8k32 (s8 x s8 ->
// s32, exact like __dp4a), the activation rows as the A operand (rows 0..7,
// 8..15 zero) and 8 weight columns as the B operand.  Eight warps split K
// into 64-byte chunks (chunk c to warp c % 8); a CTA owns 8 * kG columns.
// Which physical k a fragment slot holds is free as long as both operands
// agree, so lane (g, t) = (lane / 4, lane % 4) reads 16 contiguous bytes of
// its activation row g and of weight column g at k = 64 c + 16 t: the bytes
// 0-7 feed the first mma of the chunk, 8-15 the second.  Each lane lands its
// own weight bytes by cp.async before the programmatic wait, as above; the
// warps' partial sums meet in shared memory and one thread per output
// applies the element's dequant epilogue.
// ---------------------------------------------------------------------------
constexpr uint32_t kGmWarps = 8;
constexpr uint32_t kGmThreads = kGmWarps * 32;

__device__ __forceinline__ void mma_s8_m16n8k32(int32_t (&d)[4], uint32_t a0, uint32_t a2,
                                                uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// kNci: chunks per warp at most (K <= 64 * 8 * kNci).  Dynamic shared
// memory: the weight slots (8 warps x nci chunks x kG groups x 512 bytes)
// then the partial sums (8 warps x kG x 64 int32).
template <int kG, int kNci, typename Extra>
__global__ void __launch_bounds__(kGmThreads) gemv_i8_mma_kernel(const GsParams p, const Extra x) {
    extern __shared__ __align__(16) uint8_t gm_smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t g = lane >> 2, t = lane & 3;
    const uint32_t n0 = blockIdx.x * 8u * kG;
    const uint32_t nch = (p.k_stride + 63u) / 64u;
    const uint32_t nci = (nch + kGmWarps - 1u) / kGmWarps;
    uint8_t *wslots = gm_smem + static_cast<size_t>(warp) * nci * kG * 512u;
#pragma unroll
    for (int i = 0; i < kNci; ++i) {
        const uint32_t c = warp + kGmWarps * i;
        const uint32_t k = c * 64u + t * 16u;
        if (c < nch && k < p.k_stride) {
#pragma unroll
            for (int q = 0; q < kG; ++q) {
                const uint32_t n = n0 + 8u * q + g;
                if (n < p.N)
                    cp_async_16(wslots + (i * kG + q) * 512u + lane * 16u,
                                p.Bt + static_cast<uint64_t>(n) * p.k_stride + k);
            }
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    pdl_enter();
    gs_advance(x);
    // This thread's output (if any): its epilogue operands now.
    const uint32_t o = threadIdx.x;
    const uint32_t oq = o / 64u, orr = o % 64u, oln = orr / 2u;
    const uint32_t om = oln >> 2, on = n0 + 8u * oq + 2u * (oln & 3u) + (orr & 1u);
    const bool has_out = o < 64u * kG && om < p.M && on < p.N;
    const bool has_bias = p.bias != nullptr;
    float e_sa = 1.0f, e_sb = 1.0f, e_bias = 0.0f;
    if (has_out) {
        e_sa = p.scale_a ? __ldg(p.scale_a + om) : 1.0f;
        e_sb = __ldg(p.scale_b + on);
        e_bias = has_bias ? __ldg(p.bias + on) : 0.0f;
    }
    int4 a[kNci];
#pragma unroll
    for (int i = 0; i < kNci; ++i) {
        const uint32_t k = (warp + kGmWarps * i) * 64u + t * 16u;
        if (g < p.M && k + 16u <= p.K)
            a[i] = __ldg(reinterpret_cast<const int4 *>(p.A + static_cast<uint64_t>(g) * p.lda + k));
        else if (g < p.M && k < p.K)
            a[i] = gs_act16(p, g, k);
        else
            a[i] = make_int4(0, 0, 0, 0);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    int32_t acc[kG][4];
#pragma unroll
    for (int q = 0; q < kG; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0;
#pragma unroll
    for (int i = 0; i < kNci; ++i) {
        if (warp + kGmWarps * i < nch) {
#pragma unroll
            for (int q = 0; q < kG; ++q) {
                const int4 w = *reinterpret_cast<const int4 *>(wslots + (i * kG + q) * 512u + lane * 16u);
                mma_s8_m16n8k32(acc[q], a[i].x, a[i].y, w.x, w.y);
                mma_s8_m16n8k32(acc[q], a[i].z, a[i].w, w.z, w.w);
            }
        }
    }
    // Partial sums of (row g, columns 8q + 2t, 8q + 2t + 1) to shared memory.
    int32_t *red = reinterpret_cast<int32_t *>(gm_smem + static_cast<size_t>(kGmWarps) * nci * kG * 512u);
#pragma unroll
    for (int q = 0; q < kG; ++q) {
        red[(warp * kG + q) * 64u + lane * 2u] = acc[q][0];
        red[(warp * kG + q) * 64u + lane * 2u + 1u] = acc[q][1];
    }
    __syncthreads();
    if (!has_out) return;
    int32_t s = 0;
#pragma unroll
    for (uint32_t w = 0; w < kGmWarps; ++w) s += red[(w * kG + oq) * 64u + orr];
    float out = ref_dequant(s, e_sa, e_sb, has_bias, e_bias, p.epilogue, form_at(p.fmap, om, on));
    if constexpr (std::is_same<Extra, GsResidual>::value)
        out = __fadd_rn(x.R[static_cast<uint64_t>(om) * x.ldr + on], out);
    p.C[static_cast<uint64_t>(om) * p.ldc + on] = out;
}

template <int kG, int kNci, typename Extra>
cudaError_t gm_launch(const LaunchCtx &ctx, const GsParams &g, const Extra &x) {
    static std::mutex mu;
    static bool opted[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    {
        std::lock_guard<std::mutex> l(mu);
        if (dev < 0 || dev >= 64 || !opted[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(gemv_i8_mma_kernel<kG, kNci, Extra>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(kGsMaxSmem));
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) opted[dev] = true;
        }
    }
    const uint32_t nch = (g.k_stride + 63u) / 64u;
    const uint32_t nci = (nch + kGmWarps - 1u) / kGmWarps;
    const uint32_t smem = kGmWarps * nci * kG * 512u + kGmWarps * kG * 64u * 4u;
    const uint32_t grid = (g.N + 8u * kG - 1u) / (8u * kG);
    if (ctx.launch_counter) ++*ctx.launch_counter;
    return launch_pdl(ctx.stream, gemv_i8_mma_kernel<kG, kNci, Extra>, dim3(grid),
                      dim3(kGmThreads), smem, g, x);
}

template <typename Extra>
cudaError_t gm_dispatch(const LaunchCtx &ctx, const GsParams &g, uint32_t groups, const Extra &x) {
    const bool short_k = g.k_stride <= 64u * kGmWarps * 8u;
    switch (groups) {
    case 2: return short_k ? gm_launch<2, 8>(ctx, g, x) : gm_launch<2, 16>(ctx, g, x);
    case 4: return short_k ? gm_launch<4, 8>(ctx, g, x) : gm_launch<4, 16>(ctx, g, x);
    default: return short_k ? gm_launch<1, 8>(ctx, g, x) : gm_launch<1, 16>(ctx, g, x);
    }
}

GsParams gs_params(const MatmulI8 &p) {
    GsParams g;
    g.A = p.A;
    g.lda = p.lda;
    g.Bt = p.Bt;
    g.k_stride = p.k_stride;
    g.scale_a = p.scale_a;
    g.scale_b = p.scale_b;
    g.bias = p.bias;
    g.C = p.C;
    g.ldc = p.ldc;
    g.M = p.M;
    g.K = p.K;
    g.N = p.N;
    g.epilogue = p.epilogue;
    g.fmap = p.fmap;
    return g;
}

}  // namespace

// K up to 8192: past that (e.g. 11008, 88 KiB of columns per CTA, two CTAs
// per SM) the register-streaming GEMV measured faster (9.9 against 10.7 us
// at 11008 x 4096).
bool gemv_stream_supported(const MatmulI8 &p, uint32_t cols_per_warp) {
    return p.M >= 1 && p.M <= 2 && p.K >= 1 && p.k_stride <= 8192u && p.k_stride % 16u == 0u &&
           static_cast<uint64_t>(kGsWarps) * cols_per_warp * p.k_stride <= kGsMaxSmem &&
           (reinterpret_cast<uintptr_t>(p.A) % 16u) == 0u && p.lda % 16u == 0u &&
           (reinterpret_cast<uintptr_t>(p.Bt) % 16u) == 0u;
}

cudaError_t matmul_i8_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                                  uint32_t ldr) {
    if (!gemv_stream_supported(p, 1)) return cudaErrorInvalidValue;
    const GsParams g = gs_params(p);
    const uint32_t grid = (p.N + kGsWarps - 1) / kGsWarps;
    if (p.advance_pos && !R) return cudaErrorNotSupported;
    if (R) {
        const GsResidual x{R, ldr, p.advance_pos, p.advance};
        return p.M == 1 ? gs_launch<1, 1>(ctx, g, grid, x) : gs_launch<2, 1>(ctx, g, grid, x);
    }
    return p.M == 1 ? gs_launch<1, 1>(ctx, g, grid, GsPlain{})
                    : gs_launch<2, 1>(ctx, g, grid, GsPlain{});
}

cudaError_t matmul_i8_swiglu_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p, float *Y,
                                         uint32_t ldy, uint32_t I, float alpha) {
    if (p.N != 2u * I || I == 0 || !gemv_stream_supported(p, 2)) return cudaErrorInvalidValue;
    const GsSwiglu x{Y, ldy, I, alpha};
    const uint32_t grid = (I + kGsWarps - 1) / kGsWarps;
    return p.M == 1 ? gs_launch<1, 2>(ctx, gs_params(p), grid, x)
                    : gs_launch<2, 2>(ctx, gs_params(p), grid, x);
}

bool gemv_mma_supported(const MatmulI8 &p) {
    return p.M >= 1 && p.M <= 8 && p.K >= 1 && p.k_stride <= 8192u && p.k_stride % 16u == 0u &&
           (reinterpret_cast<uintptr_t>(p.A) % 16u) == 0u && p.lda % 16u == 0u &&
           (reinterpret_cast<uintptr_t>(p.Bt) % 16u) == 0u;
}

// Two 8-column groups per CTA while every CTA of the launch and of the next
// one fit on the GPU at once (N <= 32 x 148, K <= 4096); one group past that.
static bool gemv_mma_small(const MatmulI8 &p) {
    return p.N <= 32u * 148u && p.k_stride <= 4096u;
}

// The mma GEMV for M = 2..8 wherever it takes the shape, and for M = 1 at the
// small shapes where it measured faster than the one-column-per-warp kernel
// (4096 x 4096: 3.73 against 3.91 us; 4096 x 12288: 10.8 against 10.2 us).
bool gemv_mma_preferred(const MatmulI8 &p) {
    if (!gemv_mma_supported(p)) return false;
    return p.M >= 2 || gemv_mma_small(p);
}

cudaError_t matmul_i8_gemv_mma(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                               uint32_t ldr, uint32_t groups) {
    if (!gemv_mma_supported(p)) return cudaErrorInvalidValue;
    if (groups == 0) groups = gemv_mma_small(p) ? 2u : 1u;
    const GsParams g = gs_params(p);
    if (p.advance_pos && !R) return cudaErrorNotSupported;
    if (R) return gm_dispatch(ctx, g, groups, GsResidual{R, ldr, p.advance_pos, p.advance});
    return gm_dispatch(ctx, g, groups, GsPlain{});
}

cudaError_t qkv_rope_append_gemv_stream(const LaunchCtx &ctx, const MatmulI8 &p,
                                        const QkvRope &q) {
    if (p.M != 1 || q.head_dim == 0 || (q.head_dim & 1u) || q.head_dim / 2 > kGsMaxPairs ||
        p.N != 3u * q.heads * q.head_dim || !gemv_stream_supported(p, 2))
        return cudaErrorInvalidValue;
    GsQkv x;
    x.Q = q.Q;
    x.Kout = q.K_out;
    x.Vout = q.V_out;
    x.Kc = q.K_cache;
    x.Vc = q.V_cache;
    x.mask = q.mask;
    x.position = q.position;
    x.err = ctx.err;
    x.heads = q.heads;
    x.D = q.head_dim;
    x.cap = q.capacity;
    x.pos0 = q.position_offset;
    x.scaling = q.scaling;
    for (uint32_t j = 0; j < q.head_dim / 2; ++j) x.inv[j] = q.inv_freq[j];
    const uint32_t pairs = 3u * q.heads * (q.head_dim / 2u);
    return gs_launch<1, 2>(ctx, gs_params(p), (pairs + kGsWarps - 1) / kGsWarps, x);
}

}  // namespace vnpu_b200
