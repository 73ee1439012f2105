// gemm_f32.cu - MATMUL_F32 on the B200's CUDA cores, bit-exact with the
// reference's CPU kernels (src/kernels/kernels.cpp:19-352,480-520).
//
// The reference defines every output as one sequential float chain over k,
// rounded the way the CPU kernel that owns the element's tile rounds it.
// tf32 / bf16 tensor-core MMAs round the operands and sum in an order of
// their own, so this path is a register-tiled SIMT GEMM instead: each thread
// keeps its outputs' chains in registers and walks k in order, so the chain
// of every element is exactly the reference's.  The forms:
//   kF32Block   - AVX2 register blocks and row stream (:98-239): fmaf chain
//                 over all of K.  Rows the reference's packed-panel kernel
//                 owns (:241-329) restart the chain every 128 k and fold each
//                 panel in with C = fmaf(alpha, panel, C).
//   kF32Unfused - scalar ISA, Cell unit, transposed A (:65-76, :409-454):
//                 acc + a*b with both roundings.
//   kF32Dot8    - transposed B (:331-352): 8 fmaf chains over k mod 8, the
//                 AVX2 horizontal sum, then the scalar tail (whole groups of
//                 four unfused, the last 0-3 terms fused, as GCC -O3 builds
//                 it).
// The host (runtime.cpp) restates the reference's tile geometry for the
// device's configuration; the kernel derives each element's form and its
// store rounding (store_c, :43-50) from that geometry.
#include <cstdint>

#include "common.cuh"

namespace vnpu_b200 {
namespace {

constexpr int kF32Threads = 256;
constexpr int kF32BK = 8;          // k per shared-memory stage
constexpr int kF32Panel = 128;     // packed-panel depth, kernels.cpp:247
// packed kernel needs a 128 x tn float panel in 256 KiB + 64 B of scratch
constexpr uint32_t kF32PanelMaxCols = (256u * 1024u + 64u) / (128u * 4u);

inline void count_launch(const LaunchCtx &ctx, uint64_t n = 1) {
    if (ctx.launch_counter) *ctx.launch_counter += n;
}

// store_c roundings (kernels.cpp:43-50) by owning kernel.
__device__ __forceinline__ float store_block(float v, const MatmulF32 &p, uint32_t n, float dst) {
    float out = p.bias ? __fmaf_rn(p.alpha, v, p.bias[n]) : __fmul_rn(p.alpha, v);
    if (p.beta != 0.0f) out = __fmaf_rn(p.beta, dst, out);
    return ref_activation(out, p.epilogue, true);
}
__device__ __forceinline__ float store_panel(float v, const MatmulF32 &p, uint32_t n, float dst) {
    float out = __fmul_rn(p.alpha, v);
    if (p.bias) out = __fadd_rn(out, p.bias[n]);
    if (p.beta != 0.0f) out = __fmaf_rn(p.beta, dst, out);
    return ref_activation(out, p.epilogue, true);
}
__device__ __forceinline__ float store_scalar(float v, const MatmulF32 &p, uint32_t n, float dst) {
    float out = __fmul_rn(p.alpha, v);
    if (p.bias) out = __fadd_rn(out, p.bias[n]);
    if (p.beta != 0.0f) out = __fadd_rn(out, __fmul_rn(p.beta, dst));
    return ref_activation(out, p.epilogue, false);
}
// zero_c_tile (kernels.cpp:52-62): a culled tile's outputs.
__device__ __forceinline__ float store_culled(const MatmulF32 &p, uint32_t n, float dst) {
    float out = p.bias ? p.bias[n] : 0.0f;
    if (p.beta != 0.0f) out = __fadd_rn(out, __fmul_rn(p.beta, dst));
    return ref_activation(out, p.epilogue, false);
}

// Tile-mask cull of the reference tile that holds (m, n)
// (src/core/scheduler.cpp:234-243).
__device__ __forceinline__ bool culled(const MatmulF32 &p, uint32_t m, uint32_t n) {
    if (!p.mask) return false;
    const uint32_t mt = (p.M + p.tile_m - 1) / p.tile_m, nt = (p.N + p.tile_n - 1) / p.tile_n;
    const uint32_t mi = m / p.tile_m, ni = n / p.tile_n;
    uint32_t mm = static_cast<uint32_t>(static_cast<uint64_t>(mi) * p.mask_m / mt);
    uint32_t nn = static_cast<uint32_t>(static_cast<uint64_t>(ni) * p.mask_n / nt);
    mm = min(mm, p.mask_m - 1);
    nn = min(nn, p.mask_n - 1);
    return p.mask[static_cast<uint64_t>(mm) * p.mask_n + nn] == 0;
}

// Row m lies in a full 3-row block of its reference tile (kernels.cpp:252).
__device__ __forceinline__ bool panel_row(const MatmulF32 &p, uint32_t m) {
    const uint32_t m0 = m / p.tile_m * p.tile_m;
    const uint32_t rows = min(p.tile_m, p.M - m0);
    return rows >= 3 && m < m0 + rows / 3 * 3;
}
// Column n's reference tile takes the packed-panel kernel (kernels.cpp:498-505).
__device__ __forceinline__ bool panel_col(const MatmulF32 &p, uint32_t n) {
    const uint32_t n0 = n / p.tile_n * p.tile_n;
    const uint32_t cols = min(p.tile_n, p.N - n0);
    return cols % 32 == 0 && cols <= kF32PanelMaxCols;
}

__device__ __forceinline__ float load_a(const MatmulF32 &p, uint32_t m, uint32_t k) {
    return p.trans_a ? p.A[static_cast<uint64_t>(k) * p.lda + m]
                     : p.A[static_cast<uint64_t>(m) * p.lda + k];
}
__device__ __forceinline__ float load_b(const MatmulF32 &p, uint32_t k, uint32_t n) {
    return p.trans_b ? p.B[static_cast<uint64_t>(n) * p.ldb + k]
                     : p.B[static_cast<uint64_t>(k) * p.ldb + n];
}

// One CTA computes a BM x BN block of C; 16 x 16 threads, each TM x TN
// outputs (rows ty*4.. and 64+ty*4.. when TM = 8).  A and B stages live in
// shared memory k-major (As[k][m], Bs[k][n]) so the inner loop reads
// float4s; the next stage is prefetched into registers while the current one
// is consumed.
template <int kMode>
__global__ void __launch_bounds__(kF32Threads, 1) gemm_f32_kernel(MatmulF32 p) {
    constexpr int BM = kMode == kF32Dot8 ? 64 : 128;
    constexpr int BN = BM;
    constexpr int TM = BM / 16, TN = BN / 16;
    constexpr int LA = BM * kF32BK / kF32Threads;   // A elements per thread per stage
    constexpr int LB = BN * kF32BK / kF32Threads;
    constexpr int CH = kMode == kF32Dot8 ? 8 : 1;   // chains per output
    __shared__ __align__(16) float As[2][kF32BK][BM + 4];
    __shared__ __align__(16) float Bs[2][kF32BK][BN + 4];

    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const uint32_t m_base = blockIdx.y * BM, n_base = blockIdx.x * BN;
    auto row_of = [&](int i) -> uint32_t {
        return m_base + (TM == 8 ? (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4) : ty * 4 + i);
    };
    auto col_of = [&](int j) -> uint32_t {
        return n_base + (TN == 8 ? (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4) : tx * 4 + j);
    };

    // Stage loader: element e of the BM x 8 (A) / 8 x BN (B) stage, mapped so
    // consecutive threads walk the operand's contiguous dimension.
    float ra[LA], rb[LB];
    auto fetch = [&](uint32_t k0) {
#pragma unroll
        for (int q = 0; q < LA; ++q) {
            const int e = tid + q * kF32Threads;
            const int mm = p.trans_a ? e % BM : e / kF32BK;
            const int kk = p.trans_a ? e / BM : e % kF32BK;
            const uint32_t m = m_base + mm, k = k0 + kk;
            ra[q] = (m < p.M && k < p.K) ? load_a(p, m, k) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < LB; ++q) {
            const int e = tid + q * kF32Threads;
            const int nn = p.trans_b ? e / kF32BK : e % BN;
            const int kk = p.trans_b ? e % kF32BK : e / BN;
            const uint32_t n = n_base + nn, k = k0 + kk;
            rb[q] = (n < p.N && k < p.K) ? load_b(p, k, n) : 0.0f;
        }
    };
    auto deposit = [&](int buf) {
#pragma unroll
        for (int q = 0; q < LA; ++q) {
            const int e = tid + q * kF32Threads;
            const int mm = p.trans_a ? e % BM : e / kF32BK;
            const int kk = p.trans_a ? e / BM : e % kF32BK;
            As[buf][kk][mm] = ra[q];
        }
#pragma unroll
        for (int q = 0; q < LB; ++q) {
            const int e = tid + q * kF32Threads;
            const int nn = p.trans_b ? e / kF32BK : e % BN;
            const int kk = p.trans_b ? e % kF32BK : e / BN;
            Bs[buf][kk][nn] = rb[q];
        }
    };

    float acc[TM][TN][CH];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j)
#pragma unroll
            for (int c = 0; c < CH; ++c) acc[i][j][c] = 0.0f;

    // Packed-panel rows (kF32Block only): bit i*TN+j set when the element's
    // chain restarts every 128 k.  fold[] holds the folded panels.
    uint64_t panel_bits = 0;
    if (kMode == kF32Block && p.packed) {
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const uint32_t m = row_of(i);
            if (m >= p.M || !panel_row(p, m)) continue;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const uint32_t n = col_of(j);
                if (n < p.N && panel_col(p, n)) panel_bits |= 1ull << (i * TN + j);
            }
        }
    }
    float fold[kMode == kF32Block ? TM : 1][kMode == kF32Block ? TN : 1];
    if (kMode == kF32Block) {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) fold[i][j] = 0.0f;
    }

    // kF32Dot8 runs the 8-lane chains over whole stages only; the tail k >=
    // K8 is summed after the horizontal add.
    const uint32_t k_main = kMode == kF32Dot8 ? p.K / 8 * 8 : p.K;
    const uint32_t stages = (k_main + kF32BK - 1) / kF32BK;
    if (stages) {
        fetch(0);
        deposit(0);
        __syncthreads();
    }
    for (uint32_t t = 0; t < stages; ++t) {
        const int buf = t & 1;
        if (t + 1 < stages) fetch((t + 1) * kF32BK);
        const uint32_t kcount = min(static_cast<uint32_t>(kF32BK), k_main - t * kF32BK);
#pragma unroll
        for (int kk = 0; kk < kF32BK; ++kk) {
            if (kk < static_cast<int>(kcount)) {
                float a[TM], b[TN];
#pragma unroll
                for (int h = 0; h < TM / 4; ++h) {
                    const float4 v = *reinterpret_cast<const float4 *>(&As[buf][kk][h * 64 + ty * 4]);
                    a[h * 4 + 0] = v.x; a[h * 4 + 1] = v.y; a[h * 4 + 2] = v.z; a[h * 4 + 3] = v.w;
                }
#pragma unroll
                for (int h = 0; h < TN / 4; ++h) {
                    const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][kk][h * 64 + tx * 4]);
                    b[h * 4 + 0] = v.x; b[h * 4 + 1] = v.y; b[h * 4 + 2] = v.z; b[h * 4 + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) {
                        if (kMode == kF32Unfused)
                            acc[i][j][0] = __fadd_rn(acc[i][j][0], __fmul_rn(a[i], b[j]));
                        else
                            acc[i][j][kMode == kF32Dot8 ? kk : 0] =
                                __fmaf_rn(a[i], b[j], acc[i][j][kMode == kF32Dot8 ? kk : 0]);
                    }
            }
        }
        if (kMode == kF32Block && panel_bits) {
            const uint32_t k_done = (t + 1) * kF32BK;
            if (k_done % kF32Panel == 0 || t + 1 == stages) {
                const bool first = k_done <= kF32Panel;
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) {
                        if (!((panel_bits >> (i * TN + j)) & 1)) continue;
                        const uint32_t m = row_of(i), n = col_of(j);
                        if (first) {
                            const float dst = p.beta != 0.0f
                                ? p.C[static_cast<uint64_t>(m) * p.ldc + n] : 0.0f;
                            fold[i][j] = store_panel(acc[i][j][0], p, n, dst);
                        } else {
                            fold[i][j] = __fmaf_rn(p.alpha, acc[i][j][0], fold[i][j]);
                        }
                        acc[i][j][0] = 0.0f;
                    }
            }
        }
        if (t + 1 < stages) {
            deposit(buf ^ 1);
            __syncthreads();
        }
    }

    // Store.
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const uint32_t m = row_of(i);
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const uint32_t n = col_of(j);
            if (n >= p.N) continue;
            float *dst = p.C + static_cast<uint64_t>(m) * p.ldc + n;
            const float old = p.beta != 0.0f ? *dst : 0.0f;
            float out;
            if (culled(p, m, n)) {
                out = store_culled(p, n, old);
            } else if (kMode == kF32Unfused) {
                out = store_scalar(acc[i][j][0], p, n, old);
            } else if (kMode == kF32Dot8) {
                const float s0 = __fadd_rn(acc[i][j][0], acc[i][j][4 % CH]);
                const float s1 = __fadd_rn(acc[i][j][1 % CH], acc[i][j][5 % CH]);
                const float s2 = __fadd_rn(acc[i][j][2 % CH], acc[i][j][6 % CH]);
                const float s3 = __fadd_rn(acc[i][j][3 % CH], acc[i][j][7 % CH]);
                float dot = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
                uint32_t k = k_main;
                const uint32_t quad_end = k + (p.K - k) / 4 * 4;
                for (; k < quad_end; ++k)
                    dot = __fadd_rn(dot, __fmul_rn(load_a(p, m, k), load_b(p, k, n)));
                for (; k < p.K; ++k) dot = __fmaf_rn(load_a(p, m, k), load_b(p, k, n), dot);
                out = store_panel(dot, p, n, old);
            } else if ((panel_bits >> (i * TN + j)) & 1) {
                out = fold[i][j];
            } else {
                out = store_block(acc[i][j][0], p, n, old);
            }
            *dst = out;
        }
    }
}

}  // namespace

cudaError_t matmul_f32(const LaunchCtx &ctx, const MatmulF32 &p) {
    if (!p.M || !p.N || !p.K || !p.tile_m || !p.tile_n) return cudaErrorInvalidValue;
    if (p.mask && (!p.mask_m || !p.mask_n)) return cudaErrorInvalidValue;
    const uint32_t bm = p.mode == kF32Dot8 ? 64 : 128;
    const uint64_t gx = (p.N + bm - 1) / bm, gy = (p.M + bm - 1) / bm;
    if (gx > 0x7fffffffull || gy > 65535ull) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<uint32_t>(gx), static_cast<uint32_t>(gy));
    switch (p.mode) {
    case kF32Block: gemm_f32_kernel<kF32Block><<<grid, kF32Threads, 0, ctx.stream>>>(p); break;
    case kF32Unfused: gemm_f32_kernel<kF32Unfused><<<grid, kF32Threads, 0, ctx.stream>>>(p); break;
    case kF32Dot8: gemm_f32_kernel<kF32Dot8><<<grid, kF32Threads, 0, ctx.stream>>>(p); break;
    default: return cudaErrorInvalidValue;
    }
    count_launch(ctx);
    return cudaGetLastError();
}

}  // namespace vnpu_b200
