// gemv_bulk.cu - MATMUL_I8 for M <= 8 (the decode GEMV) streamed through a
// shared-memory ring.
//
// Bound: HBM.  A decode GEMV reads every weight byte once (K*N int8) and a
// few KB of activations, so its time is the weight stream plus fixed costs:
// the launch, the first DRAM round trip and the wait for the previous
// kernel.  This kernel hides those behind the previous kernel of the stream:
//
//   * one CTA per SM (at most half of the SM's shared memory and registers),
//     so the stream's next kernel fits beside it and starts while it runs
//     (programmatic dependent launch, triggered at entry);
//   * a producer warp copies the CTA's contiguous run of K-major weight
//     columns (Bt[N][k_stride]) into a ring of shared-memory stages with
//     16-byte cp.async before waiting for the previous kernel: the weights
//     do not depend on it, the activations and the output do.  (One TMA
//     cp.async.bulk per stage measured 1.46 TB/s here, whatever the stage
//     and ring sizes: the bulk copies of a CTA did not overlap.);
//   * eight consumer warps split K: warp w, lane l own the 16-byte chunks
//     k = ((j * 8 + w) * 32 + l) * 16 of every column, with the matching
//     activation bytes of all M rows in registers (loaded once, after the
//     wait); __dp4a over int8 -> exact int32 partial sums;
//   * columns are reduced in groups of 8 / M (short unrolled code that the
//     column loop reuses: a straight-line 32-column group stalled on
//     instruction fetch): a butterfly over the warp's lanes (9 shuffles for 8
//     sums) and a sum over the eight warps through shared memory, then one
//     lane per (row, column) applies store_i8_c's
//     dequant epilogue (src/kernels/kernels.cpp:526-535) in the element's
//     reference form, optionally adding a residual row.
//
// int32 accumulation is exact and order-free, so the results are the bits of
// every other MATMUL_I8 kernel here.  Every wait is bounded (a wall-clock
// limit); a CTA that gives up records kErrWaitTimeout, still takes part in
// the consumer barriers, waits for its own copies in flight and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace vnpu_b200 {

namespace {

constexpr uint32_t kBvWarps = 8;                         // consumer warps
constexpr uint32_t kBvThreads = (kBvWarps + 1) * 32;     // + one producer warp
constexpr uint32_t kBvKPerJ = kBvWarps * 32 * 16;        // K bytes one j step covers
constexpr uint32_t kBvStageCap = 16 * 1024;              // bytes of whole columns per stage
constexpr uint32_t kBvRingBytes = 96 * 1024;             // ring; two CTAs fit one SM
constexpr uint32_t kBvMaxStages = 12;
constexpr uint32_t kBvMaxJ = 3;                          // k_stride <= 12288

struct BvParams {
    const int8_t *A;
    uint32_t lda;
    const int8_t *Bt;
    uint32_t k_stride;
    const float *scale_a;
    const float *scale_b;
    const float *bias;
    float *C;
    uint32_t ldc;
    const float *R;      // residual rows (C = R + out) or nullptr
    uint32_t ldr;
    uint32_t M, K, N;
    uint32_t epilogue;
    FormMap fmap;
    uint32_t cps;        // whole columns per stage
    uint32_t stages;     // ring depth
    uint32_t stage_bytes;
    uint32_t *err;
    uint64_t limit_ns;
};

// 16 activation bytes of row m at k (zeros past K; the packed weights are zero there too).
__device__ __forceinline__ int4 act16(const BvParams &p, uint32_t m, uint32_t k) {
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

// Arrive on `bar` once every cp.async this thread has issued so far has
// landed (the barrier's expected count includes this arrival).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kBvWarps * 32) : "memory");
}

// Bounded wait by one lane; the warp follows its verdict.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, const BvParams &p,
                                          volatile int *abort, uint32_t lane) {
    uint32_t ok = 0;
    if (lane == 0) ok = mbar_wait(bar, parity, p.limit_ns, p.err, abort) ? 1u : 0u;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

template <int kM, int kJ>
__global__ void __launch_bounds__(kBvThreads, 2) gemv_i8_bulk_kernel(const BvParams p) {
    static_assert(8 % kM == 0, "rows must divide the 8 reduction slots");
    constexpr int kG = 8 / kM;                           // columns per reduction group
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ __align__(8) uint64_t full_bar[kBvMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kBvMaxStages];
    __shared__ int32_t red[2][kBvWarps][8];
    __shared__ volatile int abort_flag;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t c0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.N / gridDim.x);
    const uint32_t c1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * p.N / gridDim.x);
    const uint32_t ncols = c1 - c0;
    const uint32_t nstages = (ncols + p.cps - 1) / p.cps;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < p.stages; ++s) {
            mbar_init(&full_bar[s], 32);
            mbar_init(&empty_bar[s], kBvWarps);
        }
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // The stream's next kernel may be scheduled now: it fits beside this one.
    pdl_launch_dependents();

    if (warp == kBvWarps) {
        // ---------------------------------------------------------- producer
        // The warp copies each stage in 16-byte cp.async pieces; each lane's
        // pieces arrive on the stage's full barrier (32 arrivals) as they land.
        for (uint32_t s = 0; s < nstages; ++s) {
            const uint32_t slot = s % p.stages;
            if (s >= p.stages &&
                !warp_wait(&empty_bar[slot], ((s / p.stages) - 1u) & 1u, p, &abort_flag, lane))
                break;
            const uint32_t cols = min(p.cps, ncols - s * p.cps);
            const uint32_t pieces = cols * p.k_stride / 16u;
            uint8_t *dst = ring + slot * p.stage_bytes;
            const int8_t *src = p.Bt + static_cast<uint64_t>(c0 + s * p.cps) * p.k_stride;
            for (uint32_t i = lane; i < pieces; i += 32u) cp_async_16(dst + 16u * i, src + 16u * i);
            cp_async_mbar_arrive_noinc(&full_bar[slot]);
        }
        // The CTA may not exit with copies into its shared memory in flight.
        cp_async_wait_all();
        return;
    }

    // -------------------------------------------------------------- consumers
    // Activations and the output may belong to the previous kernel.
    pdl_wait_previous();
    int4 xr[kJ][kM];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
        const uint32_t k = ((j * kBvWarps + warp) * 32u + lane) * 16u;
#pragma unroll
        for (int m = 0; m < kM; ++m)
            xr[j][m] = static_cast<uint32_t>(m) < p.M ? act16(p, m, k) : make_int4(0, 0, 0, 0);
    }
    bool ok = true;
    uint32_t buf = 0;
    for (uint32_t g0 = 0; g0 < ncols; g0 += kG) {
        int32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0;
#pragma unroll
        for (int c = 0; c < kG; ++c) {
            const uint32_t col = g0 + c;
            if (col < ncols) {                            // warp-uniform
                const uint32_t st = col / p.cps, cis = col - st * p.cps;
                const uint32_t slot = st % p.stages;
                if (cis == 0 && ok) ok = warp_wait(&full_bar[slot], (st / p.stages) & 1u, p, &abort_flag, lane);
                if (ok) {
                    const uint8_t *base = ring + slot * p.stage_bytes + cis * p.k_stride;
#pragma unroll
                    for (int j = 0; j < kJ; ++j) {
                        const uint32_t k = ((j * kBvWarps + warp) * 32u + lane) * 16u;
                        if (k < p.k_stride) {
                            const int4 w = *reinterpret_cast<const int4 *>(base + k);
#pragma unroll
                            for (int m = 0; m < kM; ++m) {
                                int s = v[c * kM + m];
                                s = __dp4a(xr[j][m].x, w.x, s);
                                s = __dp4a(xr[j][m].y, w.y, s);
                                s = __dp4a(xr[j][m].z, w.z, s);
                                s = __dp4a(xr[j][m].w, w.w, s);
                                v[c * kM + m] = s;
                            }
                        }
                    }
                }
                if (cis == p.cps - 1u || col == ncols - 1u) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty_bar[slot]);
                }
            }
        }
        // Butterfly over lane bits 2..0: after the step with offset o each lane
        // keeps the half of its sums whose index bit matches its own lane bit,
        // so lane l ends with slot l & 7 summed over its eight-lane group; two
        // more exchanges add the four groups.  Slot = c * kM + m.
#pragma unroll
        for (int off = 4; off >= 1; off >>= 1) {
            const bool upper = (lane & static_cast<uint32_t>(off)) != 0u;
#pragma unroll
            for (int i = 0; i < off; ++i) {
                const int32_t send = upper ? v[i] : v[i + off];
                const int32_t keep = upper ? v[i + off] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 8);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 16);
        if (lane < 8u) red[buf][warp][lane] = v[0];
        consumer_sync();
        if (warp == 0 && lane < 8u) {
            int32_t total = 0;
#pragma unroll
            for (uint32_t w = 0; w < kBvWarps; ++w) total += red[buf][w][lane];
            const uint32_t c = lane / kM, m = lane - c * kM;
            const uint32_t n = c0 + g0 + c;
            if (ok && g0 + c < ncols && m < p.M) {
                const bool has_bias = p.bias != nullptr;
                const float sa = p.scale_a ? __ldg(p.scale_a + m) : 1.0f;
                float out = ref_dequant(total, sa, __ldg(p.scale_b + n), has_bias,
                                        has_bias ? __ldg(p.bias + n) : 0.0f, p.epilogue,
                                        form_at(p.fmap, m, n));
                if (p.R) out = __fadd_rn(p.R[static_cast<uint64_t>(m) * p.ldr + n], out);
                p.C[static_cast<uint64_t>(m) * p.ldc + n] = out;
            }
        }
        buf ^= 1u;
    }
}

template <int kM, int kJ>
cudaError_t launch_bulk(const LaunchCtx &ctx, const BvParams &bp, uint32_t grid) {
    static std::mutex mu;
    static uint32_t opted[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t smem = bp.stages * bp.stage_bytes;
    {
        std::lock_guard<std::mutex> l(mu);
        if (dev < 0 || dev >= 64 || opted[dev] < smem) {
            const cudaError_t e = cudaFuncSetAttribute(gemv_i8_bulk_kernel<kM, kJ>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(kBvRingBytes));
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) opted[dev] = kBvRingBytes;
        }
    }
    return launch_pdl(ctx.stream, gemv_i8_bulk_kernel<kM, kJ>, dim3(grid), dim3(kBvThreads), smem,
                      bp);
}

template <int kM>
cudaError_t launch_bulk_m(const LaunchCtx &ctx, const BvParams &bp, uint32_t grid, uint32_t J) {
    switch (J) {
    case 1: return launch_bulk<kM, 1>(ctx, bp, grid);
    case 2: return launch_bulk<kM, 2>(ctx, bp, grid);
    default: return launch_bulk<kM, 3>(ctx, bp, grid);
    }
}

}  // namespace

// Shapes it takes: the activations of all M rows for a lane's K chunks must
// stay in registers (8 rows: K <= 4096; 3-4 rows: K <= 12288).  Opt-in
// (VNPU_B200_GEMV_BULK=1): at M = 1, K = N = 4096 it measured 11.7 us per
// launch in a graph against 4.0 us for the register-streaming GEMV.
bool gemv_bulk_supported(const MatmulI8 &p) {
    static const bool enabled = std::getenv("VNPU_B200_GEMV_BULK") != nullptr;
    if (!enabled) return false;
    const uint32_t max_k = p.M > 4 ? kBvKPerJ : kBvMaxJ * kBvKPerJ;
    return p.M >= 1 && p.M <= 8 && p.K >= 1 && p.k_stride <= max_k &&
           p.k_stride % 16u == 0u && (reinterpret_cast<uintptr_t>(p.A) % 16u) == 0u &&
           p.lda % 16u == 0u && (reinterpret_cast<uintptr_t>(p.Bt) % 16u) == 0u;
}

cudaError_t matmul_i8_gemv_bulk(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                                uint32_t ldr) {
    if (!gemv_bulk_supported(p)) return cudaErrorInvalidValue;
    BvParams bp;
    bp.A = p.A;
    bp.lda = p.lda;
    bp.Bt = p.Bt;
    bp.k_stride = p.k_stride;
    bp.scale_a = p.scale_a;
    bp.scale_b = p.scale_b;
    bp.bias = p.bias;
    bp.C = p.C;
    bp.ldc = p.ldc;
    bp.R = R;
    bp.ldr = ldr;
    bp.M = p.M;
    bp.K = p.K;
    bp.N = p.N;
    bp.epilogue = p.epilogue;
    bp.fmap = p.fmap;
    // VNPU_B200_BULK_STAGE_KB / _RING_KB / _GRID_PER_SM tune the stage size,
    // the ring size and the CTAs per SM (measurement knobs).
    uint32_t stage_cap = kBvStageCap, ring = kBvRingBytes, per_sm = 1;
    if (const char *e = std::getenv("VNPU_B200_BULK_STAGE_KB")) stage_cap = std::atoi(e) * 1024u;
    if (const char *e = std::getenv("VNPU_B200_BULK_RING_KB"))
        ring = std::min<uint32_t>(std::atoi(e) * 1024u, kBvRingBytes);
    if (const char *e = std::getenv("VNPU_B200_BULK_GRID_PER_SM")) per_sm = std::max(1, std::atoi(e));
    bp.cps = p.k_stride >= stage_cap ? 1u : stage_cap / p.k_stride;
    bp.stage_bytes = bp.cps * p.k_stride;
    bp.stages = ring / bp.stage_bytes;
    if (bp.stages > kBvMaxStages) bp.stages = kBvMaxStages;
    if (bp.stages < 2) return cudaErrorInvalidValue;
    bp.err = ctx.err;
    bp.limit_ns = ctx.wait_limit_ns;
    const uint32_t J = (p.k_stride + kBvKPerJ - 1) / kBvKPerJ;
    uint32_t grid = static_cast<uint32_t>(ctx.num_sms) * per_sm;
    if (grid > p.N) grid = p.N;
    cudaError_t e;
    switch (p.M) {
    case 1: e = launch_bulk_m<1>(ctx, bp, grid, J); break;
    case 2: e = launch_bulk_m<2>(ctx, bp, grid, J); break;
    case 3:
    case 4: e = launch_bulk_m<4>(ctx, bp, grid, J); break;
    default: e = launch_bulk<8, 1>(ctx, bp, grid); break;
    }
    if (ctx.launch_counter) ++*ctx.launch_counter;
    return e;
}

}  // namespace vnpu_b200
