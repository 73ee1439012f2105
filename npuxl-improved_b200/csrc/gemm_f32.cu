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
#include <atomic>
#include <cstdint>

#include "common.cuh"

namespace vnpu_b200 {
namespace {

constexpr int kF32Threads = 256;
constexpr int kF32BK = 16;         // k per shared-memory stage
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

// 4-byte asynchronous copy global -> shared; ok = false writes a zero.
__device__ __forceinline__ void cp_async_4(float *smem_dst, const float *gmem_src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src), "r"(ok ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

template <int kMode> struct F32Shape {
    static constexpr int BM = kMode == kF32Dot8 ? 64 : 128;   // CTA tile (square)
    static constexpr int TM = BM / 16;                        // outputs per thread per axis
    static constexpr int CH = kMode == kF32Dot8 ? 8 : 1;      // chains per output
    static constexpr int LD = BM + 4;                         // padded stage row
    static constexpr int STAGE_FLOATS = 2 * kF32BK * LD;      // A and B of one stage
    static constexpr int MIN_CTAS = kMode == kF32Dot8 ? 1 : 2;
};

// Dynamic shared memory: two pipeline stages, then (kF32Block with packed
// panels) one folded-panel value per output: fold[e][thread].
template <int kMode>
constexpr uint32_t f32_smem_bytes(bool folds) {
    using S = F32Shape<kMode>;
    return 4u * (2 * S::STAGE_FLOATS + (folds ? S::TM * S::TM * kF32Threads : 0));
}

// One CTA computes a BM x BM block of C; 16 x 16 threads, each TM x TM
// outputs (rows ty*4.. and 64+ty*4.. when TM = 8, columns likewise).  Stages
// of kF32BK k are copied straight into shared memory (k-major: As[k][m],
// Bs[k][n]) by cp.async, double-buffered, so no registers hold prefetched
// operands; each thread then walks the stage's k in order with its A/B
// fragments double-buffered in registers.
template <int kMode>
__global__ void __launch_bounds__(kF32Threads, F32Shape<kMode>::MIN_CTAS)
gemm_f32_kernel(MatmulF32 p) {
    using S = F32Shape<kMode>;
    constexpr int BM = S::BM, TM = S::TM, CH = S::CH, LD = S::LD;
    constexpr int LOADS = BM * kF32BK / kF32Threads;   // elements per operand per thread
    extern __shared__ __align__(16) float f32_smem[];
    float *fold = f32_smem + 2 * S::STAGE_FLOATS;

    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const uint32_t m_base = blockIdx.y * BM, n_base = blockIdx.x * BM;
    auto row_of = [&](int i) -> uint32_t {
        return m_base + (TM == 8 ? (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4) : ty * 4 + i);
    };
    auto col_of = [&](int j) -> uint32_t {
        return n_base + (TM == 8 ? (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4) : tx * 4 + j);
    };

    // Stage loader.  Element q of this thread's share of a stage sits at a
    // fixed offset along one axis and steps along the other, so its global
    // address is base + q * step and only k0 changes between stages.
    // k-contiguous operand (A, or B^T): row = tid / BK + q * (threads / BK),
    // k = tid % BK.  Otherwise: row = tid % BM, k = tid / BM + q * (threads / BM).
    // ("row" is m for A and n for B; shared memory holds [k][row].)
    struct Loader {
        const float *g;      // element q = 0 of stage 0
        uint64_t g_q, g_stage;
        uint32_t s0, s_q;    // shared-memory float offsets
        uint32_t var0, var_q, var_lim;  // the stepping coordinate must stay < var_lim
        uint32_t fix, fix_lim;          // the fixed coordinate must stay < fix_lim
        bool k_steps;        // the stepping coordinate is k (else the row)
    };
    auto make_loader = [&](const float *base, uint32_t ld, bool k_contig, uint32_t row_base,
                           uint32_t rows, uint32_t soff) {
        Loader l;
        if (k_contig) {
            const uint32_t r = tid / kF32BK, k = tid % kF32BK;
            l.g = base + static_cast<uint64_t>(row_base + r) * ld + k;
            l.g_q = static_cast<uint64_t>(kF32Threads / kF32BK) * ld;
            l.g_stage = kF32BK;
            l.s0 = soff + k * LD + r;
            l.s_q = kF32Threads / kF32BK;
            l.var0 = row_base + r;
            l.var_q = kF32Threads / kF32BK;
            l.var_lim = rows;
            l.fix = k;
            l.fix_lim = p.K;
            l.k_steps = false;
        } else {
            const uint32_t r = tid % BM, k = tid / BM;
            l.g = base + static_cast<uint64_t>(k) * ld + row_base + r;
            l.g_q = static_cast<uint64_t>(kF32Threads / BM) * ld;
            l.g_stage = static_cast<uint64_t>(kF32BK) * ld;
            l.s0 = soff + k * LD + r;
            l.s_q = (kF32Threads / BM) * LD;
            l.var0 = k;
            l.var_q = kF32Threads / BM;
            l.var_lim = p.K;
            l.fix = row_base + r;
            l.fix_lim = rows;
            l.k_steps = true;
        }
        return l;
    };
    const Loader la = make_loader(p.A, p.lda, !p.trans_a, m_base, p.M, 0);
    const Loader lb = make_loader(p.B, p.ldb, p.trans_b != 0, n_base, p.N, kF32BK * LD);
    auto issue_operand = [&](const Loader &l, uint32_t t, float *stage, const float *fallback) {
        const uint32_t k0 = t * kF32BK;
        const float *g = l.g + t * l.g_stage;
        // k0 shifts whichever coordinate is k
        const uint32_t var0 = l.var0 + (l.k_steps ? k0 : 0);
        const bool fix_ok = (l.fix + (l.k_steps ? 0 : k0)) < l.fix_lim;
#pragma unroll
        for (int q = 0; q < LOADS; ++q) {
            const bool ok = fix_ok && var0 + q * l.var_q < l.var_lim;
            cp_async_4(stage + l.s0 + q * l.s_q, ok ? g + q * l.g_q : fallback, ok);
        }
    };
    auto issue = [&](uint32_t t, int buf) {
        float *stage = f32_smem + buf * S::STAGE_FLOATS;
        issue_operand(la, t, stage, p.A);
        issue_operand(lb, t, stage, p.B);
        cp_async_commit();
    };

    // Accumulators.  kF32Block keeps them as pairs for fma.rn.f32x2: for
    // even i, j, pair[i/2][j/2][0] holds outputs (i, j) and (i+1, j+1) and
    // pair[i/2][j/2][1] holds (i, j+1) and (i+1, j); output (i, j) is in
    // slot (i % 2 != j % 2), half i % 2.  Every output still gets one fma per
    // k, in k order.  The other modes keep CH floats per output.
    constexpr bool kPaired = kMode == kF32Block;
    float acc[kPaired ? 1 : TM][kPaired ? 1 : TM][CH];
    uint64_t pair[kPaired ? TM / 2 : 1][kPaired ? TM / 2 : 1][2];
#pragma unroll
    for (int i = 0; i < (kPaired ? 1 : TM); ++i)
#pragma unroll
        for (int j = 0; j < (kPaired ? 1 : TM); ++j)
#pragma unroll
            for (int c = 0; c < CH; ++c) acc[i][j][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < (kPaired ? TM / 2 : 1); ++i)
#pragma unroll
        for (int j = 0; j < (kPaired ? TM / 2 : 1); ++j) pair[i][j][0] = pair[i][j][1] = 0ull;
    auto value = [&](int i, int j, int lane) -> float {
        if constexpr (kPaired)
            return half_f32x2(pair[i / 2][j / 2][(i & 1) != (j & 1)], i & 1);
        else
            return acc[i][j][lane];
    };
    auto clear = [&](int i, int j) {
        if constexpr (kPaired) {
            uint64_t &v = pair[i / 2][j / 2][(i & 1) != (j & 1)];
            v = (i & 1) ? pack_f32x2(half_f32x2(v, 0), 0.0f) : pack_f32x2(0.0f, half_f32x2(v, 1));
        } else {
            acc[i][j][0] = 0.0f;
        }
    };

    // Packed-panel outputs (kF32Block only): bit i*TM+j set when the
    // element's chain restarts every 128 k; its folded value lives in
    // fold[(i*TM+j)*threads + tid].
    uint64_t panel_bits = 0;
    if (kMode == kF32Block && p.packed) {
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const uint32_t m = row_of(i);
            if (m >= p.M || !panel_row(p, m)) continue;
#pragma unroll
            for (int j = 0; j < TM; ++j) {
                const uint32_t n = col_of(j);
                if (n < p.N && panel_col(p, n)) panel_bits |= 1ull << (i * TM + j);
            }
        }
    }

    // One k step: fragments from shared memory, then the TM x TM chains.
    auto load_frag = [&](const float *As, const float *Bs, int kk, float *a, float *b) {
#pragma unroll
        for (int h = 0; h < TM / 4; ++h) {
            const float4 va = *reinterpret_cast<const float4 *>(&As[kk * LD + h * 64 + ty * 4]);
            const float4 vb = *reinterpret_cast<const float4 *>(&Bs[kk * LD + h * 64 + tx * 4]);
            a[h * 4 + 0] = va.x; a[h * 4 + 1] = va.y; a[h * 4 + 2] = va.z; a[h * 4 + 3] = va.w;
            b[h * 4 + 0] = vb.x; b[h * 4 + 1] = vb.y; b[h * 4 + 2] = vb.z; b[h * 4 + 3] = vb.w;
        }
    };
    // kF32Block: fragments as 64-bit pairs straight from shared memory.
    auto load_frag2 = [&](const float *As, const float *Bs, int kk, uint64_t *a2, uint64_t *b2) {
#pragma unroll
        for (int h = 0; h < TM / 4; ++h) {
            const ulonglong2 va = *reinterpret_cast<const ulonglong2 *>(&As[kk * LD + h * 64 + ty * 4]);
            const ulonglong2 vb = *reinterpret_cast<const ulonglong2 *>(&Bs[kk * LD + h * 64 + tx * 4]);
            a2[h * 2 + 0] = va.x; a2[h * 2 + 1] = va.y;
            b2[h * 2 + 0] = vb.x; b2[h * 2 + 1] = vb.y;
        }
    };
    auto step2 = [&](const uint64_t *a2, const uint64_t *b2) {
#pragma unroll
        for (int j = 0; j < TM / 2; ++j) {
            const uint64_t bx = swap_f32x2(b2[j]);
#pragma unroll
            for (int i = 0; i < TM / 2; ++i) {
                pair[i][j][0] = fma_f32x2(a2[i], b2[j], pair[i][j][0]);
                pair[i][j][1] = fma_f32x2(a2[i], bx, pair[i][j][1]);
            }
        }
    };
    auto step = [&](const float *a, const float *b, int lane) {
        if constexpr (kPaired) {
            uint64_t a2[TM / 2], b2[TM / 2];
#pragma unroll
            for (int h = 0; h < TM / 2; ++h) {
                a2[h] = pack_f32x2(a[2 * h], a[2 * h + 1]);
                b2[h] = pack_f32x2(b[2 * h], b[2 * h + 1]);
            }
            step2(a2, b2);
        } else {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TM; ++j) {
                    if (kMode == kF32Unfused)
                        acc[i][j][0] = __fadd_rn(acc[i][j][0], __fmul_rn(a[i], b[j]));
                    else
                        acc[i][j][lane] = __fmaf_rn(a[i], b[j], acc[i][j][lane]);
                }
        }
    };

    // kF32Dot8 runs the 8-lane chains over whole groups of 8 k only; the
    // tail k >= K8 is summed after the horizontal add.
    const uint32_t k_main = kMode == kF32Dot8 ? p.K / 8 * 8 : p.K;
    const uint32_t stages = (k_main + kF32BK - 1) / kF32BK;
    if (stages) issue(0, 0);
    for (uint32_t t = 0; t < stages; ++t) {
        if (t + 1 < stages) {
            issue(t + 1, (t + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *As = f32_smem + (t & 1) * S::STAGE_FLOATS;
        const float *Bs = As + kF32BK * LD;
        const uint32_t kcount = min(static_cast<uint32_t>(kF32BK), k_main - t * kF32BK);
        if (kcount == kF32BK) {
            // Two rolled halves of 8 k keep the loop body small enough for
            // the instruction cache; fragments are double-buffered inside.
#pragma unroll 1
            for (int half = 0; half < kF32BK / 8; ++half) {
                if constexpr (kPaired) {
                    uint64_t a2[2][TM / 2], b2[2][TM / 2];
                    load_frag2(As, Bs, half * 8, a2[0], b2[0]);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        if (kk + 1 < 8)
                            load_frag2(As, Bs, half * 8 + kk + 1, a2[(kk + 1) & 1], b2[(kk + 1) & 1]);
                        step2(a2[kk & 1], b2[kk & 1]);
                    }
                } else {
                    float a[2][TM], b[2][TM];
                    load_frag(As, Bs, half * 8, a[0], b[0]);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        if (kk + 1 < 8)
                            load_frag(As, Bs, half * 8 + kk + 1, a[(kk + 1) & 1], b[(kk + 1) & 1]);
                        step(a[kk & 1], b[kk & 1], CH == 8 ? kk : 0);
                    }
                }
            }
        } else {
#pragma unroll
            for (int kk = 0; kk < kF32BK; ++kk) {
                if (kk < static_cast<int>(kcount)) {
                    float a[TM], b[TM];
                    load_frag(As, Bs, kk, a, b);
                    step(a, b, CH == 8 ? kk & 7 : 0);
                }
            }
        }
        if (kMode == kF32Block && panel_bits) {
            const uint32_t k_done = t * kF32BK + kcount;
            if (k_done % kF32Panel == 0 || t + 1 == stages) {
                const bool first = k_done <= static_cast<uint32_t>(kF32Panel);
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TM; ++j) {
                        if (!((panel_bits >> (i * TM + j)) & 1)) continue;
                        float &f = fold[(i * TM + j) * kF32Threads + tid];
                        if (first) {
                            const uint32_t m = row_of(i), n = col_of(j);
                            const float dst = p.beta != 0.0f
                                ? p.C[static_cast<uint64_t>(m) * p.ldc + n] : 0.0f;
                            f = store_panel(value(i, j, 0), p, n, dst);
                        } else {
                            f = __fmaf_rn(p.alpha, value(i, j, 0), f);
                        }
                        clear(i, j);
                    }
            }
        }
        __syncthreads();  // the next issue overwrites this stage's buffer
    }

    // Store.
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const uint32_t m = row_of(i);
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TM; ++j) {
            const uint32_t n = col_of(j);
            if (n >= p.N) continue;
            float *dst = p.C + static_cast<uint64_t>(m) * p.ldc + n;
            const float old = p.beta != 0.0f ? *dst : 0.0f;
            float out;
            if (culled(p, m, n)) {
                out = store_culled(p, n, old);
            } else if (kMode == kF32Unfused) {
                out = store_scalar(value(i, j, 0), p, n, old);
            } else if (kMode == kF32Dot8) {
                const float s0 = __fadd_rn(value(i, j, 0), value(i, j, 4 % CH));
                const float s1 = __fadd_rn(value(i, j, 1 % CH), value(i, j, 5 % CH));
                const float s2 = __fadd_rn(value(i, j, 2 % CH), value(i, j, 6 % CH));
                const float s3 = __fadd_rn(value(i, j, 3 % CH), value(i, j, 7 % CH));
                float dot = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
                uint32_t k = k_main;
                const uint32_t quad_end = k + (p.K - k) / 4 * 4;
                for (; k < quad_end; ++k)
                    dot = __fadd_rn(dot, __fmul_rn(load_a(p, m, k), load_b(p, k, n)));
                for (; k < p.K; ++k) dot = __fmaf_rn(load_a(p, m, k), load_b(p, k, n), dot);
                out = store_panel(dot, p, n, old);
            } else if ((panel_bits >> (i * TM + j)) & 1) {
                out = fold[(i * TM + j) * kF32Threads + tid];
            } else {
                out = store_block(value(i, j, 0), p, n, old);
            }
            *dst = out;
        }
    }
}

template <int kMode>
cudaError_t launch_f32(const LaunchCtx &ctx, const MatmulF32 &p, dim3 grid) {
    const bool folds = kMode == kF32Block && p.packed;
    const uint32_t smem = f32_smem_bytes<kMode>(folds);
    // Opt in to the largest size once per device.
    static std::atomic<uint64_t> opted{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(opted.load() & bit)) {
        e = cudaFuncSetAttribute(gemm_f32_kernel<kMode>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(f32_smem_bytes<kMode>(true)));
        if (e != cudaSuccess) return e;
        opted.fetch_or(bit);
    }
    gemm_f32_kernel<kMode><<<grid, kF32Threads, smem, ctx.stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t matmul_f32(const LaunchCtx &ctx, const MatmulF32 &p) {
    if (!p.M || !p.N || !p.K || !p.tile_m || !p.tile_n) return cudaErrorInvalidValue;
    if (p.mask && (!p.mask_m || !p.mask_n)) return cudaErrorInvalidValue;
    const uint32_t bm = p.mode == kF32Dot8 ? 64 : 128;
    const uint64_t gx = (p.N + bm - 1) / bm, gy = (p.M + bm - 1) / bm;
    if (gx > 0x7fffffffull || gy > 65535ull) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<uint32_t>(gx), static_cast<uint32_t>(gy));
    cudaError_t e;
    switch (p.mode) {
    case kF32Block: e = launch_f32<kF32Block>(ctx, p, grid); break;
    case kF32Unfused: e = launch_f32<kF32Unfused>(ctx, p, grid); break;
    case kF32Dot8: e = launch_f32<kF32Dot8>(ctx, p, grid); break;
    default: return cudaErrorInvalidValue;
    }
    count_launch(ctx);
    return e;
}

}  // namespace vnpu_b200
