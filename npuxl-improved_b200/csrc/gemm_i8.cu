// gemm_i8.cu - MATMUL_I8 on sm_100a.
//
// C[m][n] = epilogue(dequant(sum_k A[m][k] * B[k][n]))   (int8 x int8 -> int32)
//
// Restates the reference's int8 GEMM (src/kernels/kernels.cpp:526-978,
// dispatch :922-978): int32 accumulation over all of K is exact, so any tiling
// gives the reference's integers; the dequant epilogue (store_i8_c,
// kernels.cpp:526-535) is reproduced operation for operation in
// ref_dequant() (common.cuh).
//
// Three kernels:
//  * tcgen05  - persistent warp-specialised tensor-core GEMM.  One CTA per SM,
//               128x256 output tile, K in 128-byte steps.  Warp 0 issues TMA
//               loads (128B swizzle) into a 4-stage shared-memory ring; warp 1
//               (one elected thread) issues tcgen05.mma kind::i8 into one of
//               two 128x256 int32 accumulators in tensor memory (all 512
//               columns); warps 2-5 drain the other accumulator with
//               tcgen05.ld, apply the dequant epilogue and store f32 C.
//  * gemv     - M <= 8 decode: HBM-bound stream of the K-major weights with
//               16-byte loads, __dp4a, warp-shuffle reduction.
//  * simt     - any stride / alignment the TMA path cannot take: 64x64 tiles
//               through shared memory with __dp4a.  Also the GPU-side
//               cross-check of the other two.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <atomic>
#include <mutex>

#include "gemm_tc.cuh"

namespace vnpu_b200 {
namespace {

// Name of the kernel the most recent MATMUL_I8 launch used.
std::atomic<const char *> g_last_kernel{"none"};

inline void count_launch(const LaunchCtx &ctx) {
    if (ctx.launch_counter) *ctx.launch_counter += 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kStages];
    __shared__ __align__(8) uint64_t empty_bar[kStages];
    __shared__ __align__(8) uint64_t tmem_full_bar[2];
    __shared__ __align__(8) uint64_t tmem_empty_bar[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_slot;
    __shared__ volatile int abort_flag;

    // 1024-byte aligned tile ring (128B swizzle atoms are 1024 bytes).
    // The stream's next kernel may be scheduled now; it waits for this one
    // to finish before it touches memory.
    pdl_launch_dependents();
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t *ring = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t total_tiles = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (uint32_t a = 0; a < 2; ++a) {
            mbar_init(&tmem_full_bar[a], 1);
            mbar_init(&tmem_empty_bar[a], kEpiWarps);
        }
        mbar_init(&drain_bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Set-up above overlapped the previous kernel of the stream; wait for it
    // before the first global-memory access (a no-op without PDL).
    pdl_wait_previous();
    const uint32_t tmem_base = tmem_base_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                uint32_t mb, nb;
                tile_coords(t, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
                for (uint32_t kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.limit_ns, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = ring + s * kStageBytes;
                    uint8_t *sb = sa + kABytes;
                    mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
                    tma_load_2d(sa, &tmap_a, &full_bar[s], static_cast<int32_t>(kb * kBK),
                                static_cast<int32_t>(mb * kBM));
                    tma_load_2d(sb, &tmap_b, &full_bar[s], static_cast<int32_t>(kb * kBK),
                                static_cast<int32_t>(nb * kBN));
                }
            }
            // Never leave with copies in flight: wait for the last loads issued.
            const uint32_t tail = it < kStages ? it : kStages;
            for (uint32_t i = it - tail; i < it; ++i)
                mbar_wait(&full_bar[i % kStages], (i / kStages) & 1u, p.limit_ns, p.err,
                          nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_i8(kBM, kBN);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++tcount) {
                const uint32_t acc = tcount & 1u;
                const uint32_t use = tcount >> 1;
                if (!mbar_wait(&tmem_empty_bar[acc], (use & 1u) ^ 1u, p.limit_ns, p.err,
                               &abort_flag))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kBN;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&full_bar[s], ph, p.limit_ns, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(ring + s * kStageBytes);
                    const uint64_t adesc = umma_desc_k_sw128(sa);
                    const uint64_t bdesc = umma_desc_k_sw128(sa + kABytes);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk) {
                        // +32 bytes of K inside the swizzle atom = +2 in the
                        // 16-byte-granular start address field.
                        umma_i8(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc,
                                (kb | kk) != 0u);
                    }
                    umma_commit(&empty_bar[s]);
                }
                if (!ok) break;
                umma_commit(&tmem_full_bar[acc]);
            }
            // All issued MMAs complete before tensor memory is released.
            umma_commit(&drain_bar);
            mbar_wait(&drain_bar, 0, p.limit_ns, p.err, nullptr);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // Warp w may only touch TMEM lanes 32*(w%4) .. +31.
        const uint32_t lane_base = (warp & 3u) * 32u;
        const uint32_t row = lane_base + lane;
        const bool vec_ok = (p.ldc % 4u == 0u) &&
                            ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0u);
        uint32_t tcount = 0;
        for (uint32_t t = blockIdx.x; t < total_tiles; t += gridDim.x, ++tcount) {
            uint32_t mb, nb;
            tile_coords(t, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
            const uint32_t acc = tcount & 1u;
            const uint32_t use = tcount >> 1;
            // Row scale, column scales and biases of the tile are fetched
            // while the accumulators are still being computed.
            const uint32_t m = mb * kBM + row;
            const bool row_ok = m < p.M;
            const float sa = row_ok ? (p.scale_a ? __ldg(p.scale_a + m) : 1.0f) : 0.0f;
            float sreg[kBN / 32u], breg[kBN / 32u];
#pragma unroll
            for (uint32_t c = 0; c < kBN / 32u; ++c) fetch_col(p, nb * kBN + c * 32u + lane, sreg[c], breg[c]);
            // Lane 0 waits, the warp follows its verdict: the tcgen05.ld below
            // is .sync.aligned and needs all 32 lanes together.
            uint32_t ok = 0;
            if (lane == 0)
                ok = mbar_wait(&tmem_full_bar[acc], use & 1u, p.limit_ns, p.err, &abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            float *crow = p.C + static_cast<uint64_t>(row_ok ? m : 0) * p.ldc;
#pragma unroll
            for (uint32_t c = 0; c < kBN / 32u; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32cols(tmem_base + (lane_base << 16) + acc * kBN + c * 32u, r);
                tmem_wait_ld();
                const uint32_t n0 = nb * kBN + c * 32u;
                if (n0 >= p.N) continue;   // warp-uniform
                float v[32];
                dequant32_shfl_any(p.variant, r, v, sa, sreg[c], breg[c]);
                if (row_ok) store_row32(v, crow, n0, p.N, vec_ok);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty_bar[acc]);
        }
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ===========================================================================
// tcgen05 pair GEMM (cta_group::2): a cluster of two CTAs on two SMs computes
// one 256x256 output tile.  CTA r holds rows [128r, 128r+128) of the A tile
// and columns [128r, 128r+128) of the B tile in its own shared memory; the
// leader (r = 0) issues tcgen05.mma.cta_group::2 with M=256, N=256, which
// reads both halves and writes each CTA's 128 rows of D into that CTA's
// tensor memory.  Per SM that is 32 KiB of operands per 128-deep K step
// instead of 48 KiB for the 128x256 single-CTA tile.
//   barriers: full[s] (leader only) counts both CTAs' TMA bytes;
//             empty[s] (both) is arrived by the leader's commit, multicast;
//             tmem_full[a] (both) likewise; tmem_empty[a] (leader) gets one
//             arrival from each of the 16 epilogue warps of the pair.
// No TMA multicast anywhere: each CTA loads only its own tiles.
// ===========================================================================

template <uint32_t kNEpiWarps, uint32_t kNStages, uint32_t kTN = kPTileN, bool kSwiglu = false,
          uint32_t kVar = kVarRuntime>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads(kNEpiWarps), 1)
    gemm_i8_tcgen05_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                const __grid_constant__ CUtensorMap tmap_b,
                                const __grid_constant__ CUtensorMap tmap_c, const TcParams p) {
    static_assert(kTN % 32u == 0u && kTN >= 64u && kTN <= 256u, "pair tile width");
    constexpr uint32_t kBRows = kTN / 2u;                      // B rows per CTA
    constexpr uint32_t kStageB = pair_stage_bytes(kTN);        // A + B bytes per CTA and stage
    // The tile's 32-column chunks are dealt to kNEpiWarps / 4 column groups of
    // warps, kChunks consecutive chunks each (the last group may get fewer).
    constexpr uint32_t kGroups = kNEpiWarps / 4u;
    constexpr uint32_t kTileChunks = kTN / 32u;
    constexpr uint32_t kChunks = (kTileChunks + kGroups - 1u) / kGroups;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kNStages];
    __shared__ __align__(8) uint64_t empty_bar[kNStages];
    __shared__ __align__(8) uint64_t tmem_full_bar[2];
    __shared__ __align__(8) uint64_t tmem_empty_bar[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ uint32_t tmem_base_slot;
    __shared__ volatile int abort_flag;

    // The stream's next kernel may be scheduled now; it waits for this one
    // to finish before it touches memory.
    pdl_launch_dependents();
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t *ring = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t pair = blockIdx.x >> 1;
    const uint32_t npairs = gridDim.x >> 1;
    const uint32_t total_tiles = p.tiles_m * p.tiles_n * p.splits;   // work units

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kNStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (uint32_t a = 0; a < 2; ++a) {
            mbar_init(&tmem_full_bar[a], 1);
            mbar_init(&tmem_empty_bar[a], 2 * kNEpiWarps);
        }
        mbar_init(&drain_bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        if (p.tma_store) tma_prefetch_desc(&tmap_c);
    }
    if (warp == 1) {
        tmem_alloc_pair(&tmem_base_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();   // both CTAs' barriers initialised, tensor memory allocated
    tc_fence_after();
    // Set-up above overlapped the previous kernel of the stream; wait for it
    // before the first global-memory access (a no-op without PDL).
    pdl_wait_previous();
    const uint32_t tmem_base = tmem_base_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (uint32_t t = pair; t < total_tiles && ok; t += npairs) {
                uint32_t mb, nb;
                const uint32_t tile = t / p.splits, split = t - tile * p.splits;
                tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
                const uint32_t kbps = p.splits > 1 ? p.kb_per_split : p.num_kb;
                const uint32_t kb0 = split * kbps;
                const uint32_t kb1 = min(p.num_kb, kb0 + kbps);
                for (uint32_t kb = kb0; kb < kb1; ++kb, ++it) {
                    const uint32_t s = it % kNStages;
                    const uint32_t ph = (it / kNStages) & 1u;
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.limit_ns, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    // The leader's full barrier counts both CTAs' bytes.
                    if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * kStageB);
                    const uint32_t leader_full = mapa_shared(smem_addr(&full_bar[s]), 0);
                    uint8_t *sa = ring + s * kStageB;
                    uint8_t *sb = sa + kPABytes;
                    tma_load_2d_pair(sa, &tmap_a, leader_full, static_cast<int32_t>(kb * kBK),
                                     static_cast<int32_t>(mb * kPTileM + rank * 128u));
                    // SwiGLU: CTA 0 holds gate rows nb*128.., CTA 1 the up rows
                    // I + nb*128.. (D columns 0-127 gate, 128-255 up).
                    const uint32_t brow = kSwiglu ? (rank ? p.swiglu_i : 0u) + nb * 128u
                                                  : nb * kTN + rank * kBRows;
                    tma_load_2d_pair(sb, &tmap_b, leader_full, static_cast<int32_t>(kb * kBK),
                                     static_cast<int32_t>(brow));
                }
            }
            // The leader never leaves with copies in flight (its full barriers
            // count the peer's bytes too).
            if (rank == 0) {
                const uint32_t tail = it < kNStages ? it : kNStages;
                for (uint32_t i = it - tail; i < it; ++i)
                    mbar_wait(&full_bar[i % kNStages], (i / kNStages) & 1u, p.limit_ns, p.err,
                              nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc = umma_idesc_i8(kPTileM, kTN);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            for (uint32_t t = pair; t < total_tiles && ok; t += npairs, ++tcount) {
                const uint32_t acc = tcount & 1u;
                const uint32_t use = tcount >> 1;
                if (!mbar_wait(&tmem_empty_bar[acc], (use & 1u) ^ 1u, p.limit_ns, p.err,
                               &abort_flag))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kTN;
                const uint32_t split = t % p.splits;
                const uint32_t kbps = p.splits > 1 ? p.kb_per_split : p.num_kb;
                const uint32_t kb0 = split * kbps;
                const uint32_t kb1 = min(p.num_kb, kb0 + kbps);
                for (uint32_t kb = kb0; kb < kb1; ++kb, ++it) {
                    const uint32_t s = it % kNStages;
                    const uint32_t ph = (it / kNStages) & 1u;
                    if (!mbar_wait(&full_bar[s], ph, p.limit_ns, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(ring + s * kStageB);
                    const uint64_t adesc = umma_desc_k_sw128(sa);
                    const uint64_t bdesc = umma_desc_k_sw128(sa + kPABytes);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk)
                        umma_i8_pair(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc,
                                     kb != kb0 || kk != 0u);
                    umma_commit_pair_mc(&empty_bar[s], 0x3);
                }
                if (!ok) break;
                umma_commit_pair_mc(&tmem_full_bar[acc], 0x3);
            }
            umma_commit_pair_mc(&drain_bar, 0x1);
            mbar_wait(&drain_bar, 0, p.limit_ns, p.err, nullptr);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Warp w reads TMEM lanes 32*(w%4)..+31 and takes the kChunks 32-column
        // chunks of column group (w-2)/4 (with 8 warps and kTN = 256: warps 2-5
        // columns 0-127, 6-9 columns 128-255).  Each 32x32 chunk is dequantised in registers, written
        // 128B-swizzled into this warp's 4 KiB staging buffer and stored to C
        // by TMA (rows >= M and columns >= N are clipped by the tensor map);
        // without a C tensor map the rows are stored directly.
        const uint32_t lane_base = (warp & 3u) * 32u;
        const uint32_t chunk0 = ((warp - 2u) >> 2) * kChunks;   // first chunk of the group
        const uint32_t col_base = chunk0 * 32u;
        const uint32_t row = rank * 128u + lane_base + lane;
        const bool vec_ok = (p.ldc % 4u == 0u) &&
                            ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0u);
        uint8_t *stage_out = ring + kNStages * kStageB + (warp - 2u) * kPStageOutBytes;
        float *my_row = reinterpret_cast<float *>(stage_out + lane * 128u);
        const uint32_t leader_empty0 = mapa_shared(smem_addr(&tmem_empty_bar[0]), 0);
        const uint32_t leader_empty1 = mapa_shared(smem_addr(&tmem_empty_bar[1]), 0);
        uint32_t tcount = 0;
        for (uint32_t t = pair; t < total_tiles; t += npairs, ++tcount) {
            uint32_t mb, nb;
            const uint32_t tile = t / p.splits, split = t - tile * p.splits;
            tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
            // split K: raw int32 sums into this split's slice of the workspace
            const uint32_t row_off = p.splits > 1 ? split * p.m_pad : 0u;
            const uint32_t acc = tcount & 1u;
            const uint32_t use = tcount >> 1;
            // Scales and biases for the tile, fetched before the accumulators are ready.
            const uint32_t m_first = mb * kPTileM + rank * 128u + lane_base;  // warp's first row
            const uint32_t m = m_first + lane;
            const bool row_ok = m < p.M;
            const float sa = row_ok ? (p.scale_a ? __ldg(p.scale_a + m) : 1.0f) : 0.0f;
            float sreg[kChunks], breg[kChunks];
            // SwiGLU: the warp's first kChunks / 2 chunks are gate columns
            // sw_col.., the rest the matching up columns (TMEM 128 + sw_col..).
            constexpr uint32_t kHalf = kChunks / 2u;
            const uint32_t sw_col = ((warp - 2u) >> 2) * kHalf * 32u;
#pragma unroll
            for (uint32_t c = 0; c < kChunks; ++c) {
                const uint32_t wcol =
                    kSwiglu ? (c < kHalf ? nb * 128u + sw_col + c * 32u
                                         : p.swiglu_i + nb * 128u + sw_col + (c - kHalf) * 32u)
                            : nb * kTN + col_base + c * 32u;
                fetch_col(p, wcol + lane, sreg[c], breg[c]);
            }
            uint32_t ok = 0;
            if (lane == 0)
                ok = mbar_wait(&tmem_full_bar[acc], use & 1u, p.limit_ns, p.err, &abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            float *crow = p.C + static_cast<uint64_t>(row_off + (row_ok ? m : 0)) * p.ldc;
#pragma unroll
            // All of the warp's accumulator columns in one round of tensor-memory
            // loads (one wait instead of one per chunk); the accumulator is
            // released before any of it is dequantised or stored.
            uint32_t rr[kChunks][32];
            __syncwarp();
#pragma unroll
            for (uint32_t c = 0; c < kChunks; ++c)
                if (chunk0 + c < kTileChunks) {  // warp-uniform
                    const uint32_t tcol = kSwiglu ? (c < kHalf ? sw_col + c * 32u
                                                               : 128u + sw_col + (c - kHalf) * 32u)
                                                  : col_base + c * 32u;
                    tmem_ld_32cols(tmem_base + (lane_base << 16) + acc * kTN + tcol, rr[c]);
                }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_empty1 : leader_empty0);
            if constexpr (kSwiglu) {
                // gate and up dequantised, then SWIGLU_F32's expression
                // (src/kernels/llm.cpp:289-306), stored as kHalf output chunks.
                if (m_first < p.M) {
#pragma unroll
                    for (uint32_t c = 0; c < kChunks; ++c)
                        dequant_chunk<kVar>(p.variant, rr[c], sa, sreg[c], breg[c]);
                }
#pragma unroll
                for (uint32_t k = 0; k < kHalf; ++k) {
                    const uint32_t n0 = nb * 128u + sw_col + k * 32u;
                    if (n0 >= p.swiglu_i || m_first >= p.M) continue;  // warp-uniform
#pragma unroll
                    for (uint32_t j = 0; j < 32u; ++j) {
                        const float g = __uint_as_float(rr[k][j]);
                        const float s = __fdiv_rn(g, __fadd_rn(1.0f, ref_exp256_lane(-g)));
                        rr[k][j] = __float_as_uint(
                            __fmul_rn(__fmul_rn(s, __uint_as_float(rr[k + kHalf][j])), p.swiglu_alpha));
                    }
                    if (p.tma_store) {
                        if (lane == 0) bulk_wait_read0();
                        __syncwarp();
#pragma unroll
                        for (uint32_t j = 0; j < 8u; ++j)
                            *reinterpret_cast<uint4 *>(my_row + 4u * (j ^ (lane & 7u))) =
                                make_uint4(rr[k][4 * j], rr[k][4 * j + 1], rr[k][4 * j + 2],
                                           rr[k][4 * j + 3]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmap_c, stage_out, static_cast<int32_t>(n0),
                                         static_cast<int32_t>(m_first));
                            bulk_commit();
                        }
                    } else if (row_ok) {
                        store_row32(reinterpret_cast<const float(&)[32]>(rr[k]), crow, n0,
                                    p.swiglu_i, vec_ok);
                    }
                }
                continue;
            }
#pragma unroll
            for (uint32_t c = 0; c < kChunks; ++c) {
                const uint32_t col = col_base + c * 32u;
                const uint32_t n0 = nb * kTN + col;
                if (chunk0 + c >= kTileChunks || n0 >= p.N || m_first >= p.M) continue;  // warp-uniform
                if (p.splits == 1) dequant_chunk<kVar>(p.variant, rr[c], sa, sreg[c], breg[c]);
                const float(&v)[32] = reinterpret_cast<const float(&)[32]>(rr[c]);
                if (p.ndst) {
                    // Scatter: the 32x32 chunk is transposed through the staging
                    // buffer so each store instruction writes four whole 128-byte
                    // row segments, then goes to every destination (peers over
                    // NVLink) at column col_off + n.
                    if (lane == 0) bulk_wait_read0();
                    __syncwarp();
#pragma unroll
                    for (uint32_t j = 0; j < 8u; ++j)
                        *reinterpret_cast<uint4 *>(my_row + 4u * (j ^ (lane & 7u))) =
                            make_uint4(rr[c][4 * j], rr[c][4 * j + 1], rr[c][4 * j + 2],
                                       rr[c][4 * j + 3]);
                    __syncwarp();
                    const uint32_t g = lane & 7u;
                    const uint32_t ncol = n0 + 4u * g;
#pragma unroll
                    for (uint32_t i = 0; i < 8u; ++i) {
                        const uint32_t rrow = 4u * i + (lane >> 3);
                        const float4 val = *reinterpret_cast<const float4 *>(
                            stage_out + rrow * 128u + ((g ^ (rrow & 7u)) << 4));
                        const uint32_t mrow = m_first + rrow;
                        if (mrow >= p.M || ncol >= p.N) continue;
                        const uint64_t off = static_cast<uint64_t>(mrow) * p.ldd + p.col_off + ncol;
#pragma unroll
                        for (uint32_t d = 0; d < 8u; ++d) {
                            if (d >= p.ndst) break;
                            float *o = p.dst[d] + off;
                            if (ncol + 4u <= p.N) {
                                *reinterpret_cast<float4 *>(o) = val;
                            } else {
                                o[0] = val.x;
                                if (ncol + 1u < p.N) o[1] = val.y;
                                if (ncol + 2u < p.N) o[2] = val.z;
                            }
                        }
                    }
                    __syncwarp();   // the staging buffer is reused by the next chunk
                } else if (p.tma_store) {
                    if (lane == 0) bulk_wait_read0();  // previous store has read the buffer
                    __syncwarp();
#pragma unroll
                    for (uint32_t j = 0; j < 8u; ++j)
                        *reinterpret_cast<uint4 *>(my_row + 4u * (j ^ (lane & 7u))) =
                            make_uint4(rr[c][4 * j], rr[c][4 * j + 1], rr[c][4 * j + 2],
                                       rr[c][4 * j + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmap_c, stage_out, static_cast<int32_t>(n0),
                                     static_cast<int32_t>(row_off + m_first));
                        bulk_commit();
                    }
                } else if (row_ok) {
                    store_row32(v, crow, n0, p.N, vec_ok);
                }
            }
        }
        // Shared memory must outlive the stores' reads; their global writes
        // complete with the grid like any other store.
        if (lane == 0) bulk_wait_read0();
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // the peer's smem / TMEM are no longer in use by the pair MMA
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// Split-K finish: C[m][n] = dequant(sum over splits of ws[s][m][n]) - the
// int32 sums are exact, so the result is the single-pass GEMM's bit for bit.
// ws rows are s * m_pad + m, N columns; four columns per thread (N % 4 == 0).
// With R (MATMUL_I8_RESIDUAL) C = R + that, ADD_F32's single rounding.
__global__ void __launch_bounds__(256) splitk_finish_kernel(
    const int4 *__restrict__ ws, uint32_t splits, uint32_t m_pad, uint32_t M, uint32_t N,
    const float *__restrict__ scale_a, const float *__restrict__ scale_b,
    const float *__restrict__ bias, float *__restrict__ C, uint32_t ldc, uint32_t epilogue,
    const FormMap fm, const float *__restrict__ R, uint32_t ldr) {
    pdl_enter();
    const uint32_t n4 = N / 4;
    const uint32_t total = M * n4;
    const uint32_t slice4 = m_pad * n4;
    const bool has_bias = bias != nullptr;
    const bool vec = (ldc % 4u == 0u) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0u);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const uint32_t m = i / n4;
        const uint32_t n = (i - m * n4) * 4u;
        int4 a = __ldcs(ws + i);   // m * n4 + n / 4 == i
        for (uint32_t sp = 1; sp < splits; ++sp) {
            const int4 b = __ldcs(ws + sp * slice4 + i);
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        const float sa = scale_a ? __ldg(scale_a + m) : 1.0f;
        const float4 sb = __ldg(reinterpret_cast<const float4 *>(scale_b) + n / 4u);
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (has_bias) {
            bv.x = __ldg(bias + n);
            bv.y = __ldg(bias + n + 1);
            bv.z = __ldg(bias + n + 2);
            bv.w = __ldg(bias + n + 3);
        }
        float4 o = make_float4(
            ref_dequant(a.x, sa, sb.x, has_bias, bv.x, epilogue, form_at(fm, m, n)),
            ref_dequant(a.y, sa, sb.y, has_bias, bv.y, epilogue, form_at(fm, m, n + 1u)),
            ref_dequant(a.z, sa, sb.z, has_bias, bv.z, epilogue, form_at(fm, m, n + 2u)),
            ref_dequant(a.w, sa, sb.w, has_bias, bv.w, epilogue, form_at(fm, m, n + 3u)));
        if (R) {
            const float *r = R + static_cast<uint64_t>(m) * ldr + n;
            o.x = __fadd_rn(__ldg(r), o.x);
            o.y = __fadd_rn(__ldg(r + 1), o.y);
            o.z = __fadd_rn(__ldg(r + 2), o.z);
            o.w = __fadd_rn(__ldg(r + 3), o.w);
        }
        float *c = C + static_cast<uint64_t>(m) * ldc + n;
        if (vec) {
            *reinterpret_cast<float4 *>(c) = o;
        } else {
            c[0] = o.x;
            c[1] = o.y;
            c[2] = o.z;
            c[3] = o.w;
        }
    }
}

// ===========================================================================
// M <= 8 decode on the tensor core ("swap AB"): D[n][m] = sum_k Bt[n][k] A[m][k].
// The packed weights are the 128-row UMMA operand and the (at most 8)
// activation rows the N=8 operand, so the kernel is a pure TMA stream of the
// weight matrix.  One cluster of S CTAs owns 128 weight rows (output
// columns); its CTAs split K, each accumulates its slice in tensor memory,
// and the leader CTA adds the S partial int32 tiles through distributed
// shared memory (exact, fixed order) and applies the dequant epilogue.
// ===========================================================================

constexpr uint32_t kSkWBytes = 128 * kBK;   // 16 KiB of weight rows per stage
constexpr uint32_t kSkXBytes = 8 * kBK;     // 1 KiB of activations per stage
constexpr uint32_t kSkThreads = 128;
constexpr uint32_t kSkMaxCluster = 8;
constexpr uint32_t kSkPartBytes = 128 * 8 * 4;  // one CTA's partial tile [128][8] int32
// Shared memory of a kStages-deep ring with partial tiles for csize ranks.
constexpr uint32_t sk_smem_bytes(uint32_t stages, uint32_t csize) {
    return stages * (kSkWBytes + kSkXBytes) + csize * kSkPartBytes + 1024;
}

struct SkParams {
    const float *scale_a;
    const float *scale_b;
    const float *bias;
    float *C;
    uint32_t ldc;
    uint32_t M, N, K;
    uint32_t num_kb, kb_per_rank;
    uint32_t epilogue;
    FormMap fmap;
    uint32_t *err;
    uint64_t limit_ns;
};

template <uint32_t kSkStages, uint32_t kMinBlocks>
__global__ void __launch_bounds__(kSkThreads, kMinBlocks)
    gemv_i8_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_w,
                           const __grid_constant__ CUtensorMap tmap_x, const SkParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kSkStages];
    __shared__ __align__(8) uint64_t empty_bar[kSkStages];
    __shared__ __align__(8) uint64_t mma_done_bar;
    __shared__ uint32_t tmem_base_slot;
    __shared__ volatile int abort_flag;

    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t *ring = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t *wtiles = ring;                              // [stage][16 KiB]
    uint8_t *xtiles = ring + kSkStages * kSkWBytes;      // [stage][1 KiB]
    // [rank][128 rows][8 m] int32: each CTA of the cluster stores its partial
    // tile into its own slot of the leader's copy.
    int32_t *parts = reinterpret_cast<int32_t *>(xtiles + kSkStages * kSkXBytes);

    // The next kernel of the stream may start its prologue (and its own
    // weight stream) while this one runs.
    pdl_launch_dependents();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t csize = cluster_nctarank();
    const uint32_t n0 = (blockIdx.x / csize) * 128u;
    const uint32_t kb0 = rank * p.kb_per_rank;
    const uint32_t kb1 = min(p.num_kb, kb0 + p.kb_per_rank);
    const uint32_t nkb = kb1 > kb0 ? kb1 - kb0 : 0u;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kSkStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&mma_done_bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_slot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_slot;

    if (warp == 0 && lane == 0) {
        // Weights (resident, written by no earlier kernel) for the first
        // stages go out before waiting on the previous kernel; activations,
        // which the previous kernel may have produced, only after it.
        const uint32_t first = nkb < kSkStages ? nkb : kSkStages;
        for (uint32_t i = 0; i < first; ++i) {
            mbar_arrive_expect_tx(&full_bar[i], kSkWBytes + kSkXBytes);
            tma_load_2d(wtiles + i * kSkWBytes, &tmap_w, &full_bar[i],
                        static_cast<int32_t>((kb0 + i) * kBK), static_cast<int32_t>(n0));
        }
        pdl_wait_previous();
        for (uint32_t i = 0; i < first; ++i)
            tma_load_2d(xtiles + i * kSkXBytes, &tmap_x, &full_bar[i],
                        static_cast<int32_t>((kb0 + i) * kBK), 0);
        uint32_t issued = first;
        for (uint32_t i = first; i < nkb; ++i, ++issued) {
            const uint32_t s = i % kSkStages, ph = (i / kSkStages) & 1u;
            if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.limit_ns, p.err, &abort_flag)) break;
            mbar_arrive_expect_tx(&full_bar[s], kSkWBytes + kSkXBytes);
            const int32_t k = static_cast<int32_t>((kb0 + i) * kBK);
            tma_load_2d(wtiles + s * kSkWBytes, &tmap_w, &full_bar[s], k, static_cast<int32_t>(n0));
            tma_load_2d(xtiles + s * kSkXBytes, &tmap_x, &full_bar[s], k, 0);
        }
        // Never leave with copies in flight.
        const uint32_t tail = issued < kSkStages ? issued : kSkStages;
        for (uint32_t i = issued - tail; i < issued; ++i)
            mbar_wait(&full_bar[i % kSkStages], (i / kSkStages) & 1u, p.limit_ns, p.err, nullptr);
    } else if (warp == 1 && lane == 0 && nkb > 0) {
        constexpr uint32_t idesc = umma_idesc_i8(128, 8);
        for (uint32_t i = 0; i < nkb; ++i) {
            const uint32_t s = i % kSkStages, ph = (i / kSkStages) & 1u;
            if (!mbar_wait(&full_bar[s], ph, p.limit_ns, p.err, &abort_flag)) break;
            tc_fence_after();
            const uint64_t adesc = umma_desc_k_sw128(smem_addr(wtiles + s * kSkWBytes));
            const uint64_t bdesc = umma_desc_k_sw128(smem_addr(xtiles + s * kSkXBytes));
#pragma unroll
            for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk)
                umma_i8(tmem_base, adesc + 2u * kk, bdesc + 2u * kk, idesc, (i | kk) != 0u);
            umma_commit(&empty_bar[s]);
        }
        umma_commit(&mma_done_bar);  // also after an early exit: all issued MMAs done
    }

    // ---- partial sums: TMEM lane = weight row n0 + 32*warp + lane, column = m
    uint32_t ok = 1;
    if (nkb > 0) {
        if (lane == 0) ok = mbar_wait(&mma_done_bar, 0, p.limit_ns, p.err, &abort_flag);
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    __syncwarp();
    uint32_t r[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    if (nkb > 0 && ok) {
        tc_fence_after();
        tmem_ld_8cols(tmem_base + ((warp * 32u) << 16), r);
        tmem_wait_ld();
    }
    const uint32_t row = warp * 32u + lane;
    // Push this CTA's partial row into its slot of the leader's buffer
    // (fire-and-forget stores; the cluster barrier below orders them).
    const uint32_t slot = mapa_shared(smem_addr(parts + (rank * 128u + row) * 8u), 0);
    st_shared_cluster_v4(slot, static_cast<int32_t>(r[0]), static_cast<int32_t>(r[1]),
                         static_cast<int32_t>(r[2]), static_cast<int32_t>(r[3]));
    st_shared_cluster_v4(slot + 16u, static_cast<int32_t>(r[4]), static_cast<int32_t>(r[5]),
                         static_cast<int32_t>(r[6]), static_cast<int32_t>(r[7]));

    tc_fence_before();
    cluster_sync_all();   // all partial tiles have landed in the leader

    if (rank == 0) {
        // C may still be read or written by the previous kernel until it ends.
        pdl_wait_previous();
        const uint32_t n = n0 + row;
        if (n < p.N) {
            const bool has_bias = p.bias != nullptr;
            const float sb = __ldg(p.scale_b + n);
            const float bv = has_bias ? __ldg(p.bias + n) : 0.0f;
            int32_t acc[8];
#pragma unroll
            for (uint32_t m = 0; m < 8; ++m) acc[m] = 0;
            for (uint32_t q = 0; q < csize; ++q) {
                const int4 lo = *reinterpret_cast<const int4 *>(parts + (q * 128u + row) * 8u);
                const int4 hi = *reinterpret_cast<const int4 *>(parts + (q * 128u + row) * 8u + 4u);
                acc[0] += lo.x; acc[1] += lo.y; acc[2] += lo.z; acc[3] += lo.w;
                acc[4] += hi.x; acc[5] += hi.y; acc[6] += hi.z; acc[7] += hi.w;
            }
#pragma unroll
            for (uint32_t m = 0; m < 8; ++m) {
                if (m < p.M) {
                    const float sa = p.scale_a ? __ldg(p.scale_a + m) : 1.0f;
                    p.C[static_cast<uint64_t>(m) * p.ldc + n] =
                        ref_dequant(acc[m], sa, sb, has_bias, bv, p.epilogue, form_at(p.fmap, m, n));
                }
            }
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 32);
    }
}

// ===========================================================================
// M <= 8 decode GEMV
// ===========================================================================


struct GvParams {
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

// 16 bytes of row m of A starting at k (zeros past K; B is zero there too).
template <bool kAligned>
__device__ __forceinline__ int4 load_a16(const GvParams &p, uint32_t m, uint32_t k) {
    const int8_t *row = p.A + static_cast<uint64_t>(m) * p.lda;
    if (kAligned && k + 16u <= p.K) return __ldg(reinterpret_cast<const int4 *>(row + k));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (uint32_t b = 0; b < 16u; ++b)
        if (k + b < p.K)
            w[b >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(row[k + b])) << (8u * (b & 3u));
    return make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]), static_cast<int>(w[2]),
                     static_cast<int>(w[3]));
}

// kCols columns per warp, kUnroll 512-byte K chunks of each in flight per
// lane.  One row fragment of A (16 bytes per row) serves all kCols columns,
// so more columns per warp cut the L1 traffic of A for M > 1.
// Epilogue variants of the streaming GEMV (the extra kernel argument).
struct GvPlain {};
// C = R + out (VNPU_B200_OP_MATMUL_I8_RESIDUAL); *advance_pos += advance
// (when not NULL) once the previous kernels of the stream are complete.
struct GvResidual {
    const float *R;
    uint32_t ldr;
    int32_t *advance_pos;
    int32_t advance;
};
// QKV projection + RoPE + KV-cache append for one token
// (VNPU_B200_OP_QKV_ROPE_APPEND): warp w computes rotation pair w, the
// columns (j, j + D/2) of one head of the Q, K or V part.
constexpr uint32_t kGvMaxPairs = 256;
struct GvQkv {
    float *Q, *Kout, *Vout, *Kc, *Vc, *mask;
    const int32_t *position;
    uint32_t *err;
    uint32_t heads, D, cap, pos0;
    float scaling;
    float inv[kGvMaxPairs];   // 1 / theta^(2j/D), computed on the host like ROPE_F32
};

// The two columns a warp of the QKV variant owns.
__device__ __forceinline__ void qkv_pair_columns(const GvQkv &x, uint32_t pair, uint32_t &sec,
                                                 uint32_t &h, uint32_t &j, uint32_t &n0) {
    const uint32_t half = x.D / 2, per_sec = x.heads * half;
    sec = pair / per_sec;
    const uint32_t r = pair - sec * per_sec;
    h = r / half;
    j = r - h * half;
    n0 = sec * x.heads * x.D + h * x.D + j;
}

template <int kM, bool kAligned, int kCols, int kUnroll, int kThreads, typename Extra>
__global__ void __launch_bounds__(kThreads) gemv_i8_kernel(const GvParams p, const Extra x) {
    constexpr bool kQkv = std::is_same<Extra, GvQkv>::value;
    static_assert(!kQkv || (kM == 1 && kCols == 2), "the QKV epilogue is one token, column pairs");
    constexpr int kGvColsPerWarp = kCols;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_first = blockIdx.x * (kThreads / 32 * kCols) + warp * kGvColsPerWarp;
    // Columns of this warp (QKV: a rotation pair, D/2 apart).
    uint32_t ncol[kGvColsPerWarp];
    uint32_t q_sec = 0, q_h = 0, q_j = 0;
    bool warp_valid = true;
    if constexpr (kQkv) {
        const uint32_t pair = blockIdx.x * (kThreads / 32) + warp;
        warp_valid = pair < 3 * x.heads * (x.D / 2);
        uint32_t n0 = 0;
        if (warp_valid) qkv_pair_columns(x, pair, q_sec, q_h, q_j, n0);
        ncol[0] = n0;
        ncol[1] = n0 + x.D / 2;
    } else {
#pragma unroll
        for (int c = 0; c < kGvColsPerWarp; ++c) ncol[c] = n_first + c;
    }
    int32_t acc[kGvColsPerWarp][kM];
#pragma unroll
    for (int c = 0; c < kGvColsPerWarp; ++c)
#pragma unroll
        for (int m = 0; m < kM; ++m) acc[c][m] = 0;

    const int4 *bcol[kGvColsPerWarp];
#pragma unroll
    for (int c = 0; c < kGvColsPerWarp; ++c) {
        const uint32_t n = min(ncol[c], p.N - 1);
        bcol[c] = reinterpret_cast<const int4 *>(p.Bt + static_cast<uint64_t>(n) * p.k_stride);
    }
    // Each lane owns 16 bytes of every 512-byte K chunk; kUnroll chunks of
    // each column in flight (M = 1: 8 chunks, 4 KiB, so K <= 4096 is one DRAM
    // round trip).
    const uint32_t k_end = p.K;
    pdl_launch_dependents();
    bool waited = false;
    for (uint32_t k0 = lane * 16u; k0 < k_end; k0 += 512u * kUnroll) {
        int4 b[kUnroll][kGvColsPerWarp];
#pragma unroll
        for (uint32_t u = 0; u < kUnroll; ++u) {
            const uint32_t k = k0 + u * 512u;
#pragma unroll
            for (int c = 0; c < kGvColsPerWarp; ++c)
                b[u][c] = k < k_end ? __ldcs(bcol[c] + (k >> 4)) : make_int4(0, 0, 0, 0);
        }
        // Weights are resident; the activations may come from the previous
        // kernel of the stream: wait for it only now.
        if (!waited) {
            pdl_wait_previous();
            waited = true;
        }
#pragma unroll
        for (uint32_t u = 0; u < kUnroll; ++u) {
            const uint32_t k = k0 + u * 512u;
            if (k >= k_end) break;
#pragma unroll
            for (int m = 0; m < kM; ++m) {
                if (m >= static_cast<int>(p.M)) break;
                const int4 a = load_a16<kAligned>(p, m, k);
#pragma unroll
                for (int c = 0; c < kGvColsPerWarp; ++c) {
                    int s = acc[c][m];
                    s = __dp4a(a.x, b[u][c].x, s);
                    s = __dp4a(a.y, b[u][c].y, s);
                    s = __dp4a(a.z, b[u][c].z, s);
                    s = __dp4a(a.w, b[u][c].w, s);
                    acc[c][m] = s;
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < kGvColsPerWarp; ++c)
#pragma unroll
        for (int m = 0; m < kM; ++m)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                acc[c][m] += __shfl_xor_sync(0xffffffffu, acc[c][m], o);

    if (!waited) pdl_wait_previous();
    if constexpr (std::is_same<Extra, GvResidual>::value)
        if (x.advance_pos && blockIdx.x == 0 && threadIdx.x == 0) *x.advance_pos += x.advance;
    const bool has_bias = p.bias != nullptr;
    if constexpr (kQkv) {
        // Lane 0 holds both columns of the pair: dequantize them as MATMUL_I8
        // would, rotate Q/K as ROPE_F32 does, place them as KV_APPEND does.
        if (lane != 0 || !warp_valid) return;
        const float sa = p.scale_a ? __ldg(p.scale_a) : 1.0f;
        float v[2];
#pragma unroll
        for (int c = 0; c < 2; ++c)
            v[c] = ref_dequant(acc[c][0], sa, __ldg(p.scale_b + ncol[c]), has_bias,
                               has_bias ? __ldg(p.bias + ncol[c]) : 0.0f, p.epilogue,
                               form_at(p.fmap, 0u, ncol[c]));
        const int32_t pos = x.position ? *x.position : static_cast<int32_t>(x.pos0);
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
    }
#pragma unroll
    for (int c = 0; c < kGvColsPerWarp; ++c) {
        const uint32_t n = ncol[c];
        if (n >= p.N) continue;
#pragma unroll
        for (int m = 0; m < kM; ++m) {
            if (static_cast<uint32_t>(m) == lane && static_cast<uint32_t>(m) < p.M) {
                const float sa = p.scale_a ? __ldg(p.scale_a + m) : 1.0f;
                float out = ref_dequant(acc[c][m], sa, __ldg(p.scale_b + n), has_bias,
                                        has_bias ? __ldg(p.bias + n) : 0.0f, p.epilogue,
                                        form_at(p.fmap, static_cast<uint32_t>(m), n));
                if constexpr (std::is_same<Extra, GvResidual>::value)
                    out = __fadd_rn(x.R[static_cast<uint64_t>(m) * x.ldr + n], out);
                p.C[static_cast<uint64_t>(m) * p.ldc + n] = out;
            }
        }
    }
}

// ===========================================================================
// SIMT fallback: 64x64 tiles, 256 threads, 4x4 outputs per thread.
// ===========================================================================

__global__ void __launch_bounds__(256) gemm_i8_simt_kernel(const GvParams p) {
    __shared__ int32_t As[64][9];   // 64 rows x 32 K bytes (8 words), padded
    __shared__ int32_t Bs[64][9];   // 64 columns x 32 K bytes
    const uint32_t tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const uint32_t m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    int32_t acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < p.K; k0 += 32) {
        for (uint32_t i = threadIdx.x; i < 64 * 8; i += 256) {
            const uint32_t r = i >> 3, w = i & 7;
            uint32_t av = 0, bv = 0;
            const uint32_t m = m0 + r, n = n0 + r;
#pragma unroll
            for (uint32_t b = 0; b < 4; ++b) {
                const uint32_t k = k0 + w * 4 + b;
                if (m < p.M && k < p.K)
                    av |= static_cast<uint32_t>(static_cast<uint8_t>(
                              p.A[static_cast<uint64_t>(m) * p.lda + k]))
                          << (8 * b);
                if (n < p.N && k < p.K)
                    bv |= static_cast<uint32_t>(static_cast<uint8_t>(
                              p.Bt[static_cast<uint64_t>(n) * p.k_stride + k]))
                          << (8 * b);
            }
            As[r][w] = static_cast<int32_t>(av);
            Bs[r][w] = static_cast<int32_t>(bv);
        }
        __syncthreads();
#pragma unroll
        for (uint32_t w = 0; w < 8; ++w) {
            int32_t a[4], b[4];
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                a[i] = As[ty * 4 + i][w];
                b[i] = Bs[tx * 4 + i][w];
            }
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i)
#pragma unroll
                for (uint32_t j = 0; j < 4; ++j) acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
    const bool has_bias = p.bias != nullptr;
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
        const uint32_t m = m0 + ty * 4 + i;
        if (m >= p.M) continue;
        const float sa = p.scale_a ? p.scale_a[m] : 1.0f;
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t n = n0 + tx * 4 + j;
            if (n >= p.N) continue;
            p.C[static_cast<uint64_t>(m) * p.ldc + n] =
                ref_dequant(acc[i][j], sa, p.scale_b[n], has_bias, has_bias ? p.bias[n] : 0.0f,
                            p.epilogue, form_at(p.fmap, m, n));
        }
    }
}

GvParams gv_params(const MatmulI8 &p) {
    GvParams g;
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

template <int kM, int kCols, int kUnroll, int kThreads, typename Extra>
cudaError_t launch_gemv_cfg(const LaunchCtx &ctx, const GvParams &g, bool aligned, const Extra &x);

template <int kM, typename Extra = GvPlain>
cudaError_t launch_gemv_m(const LaunchCtx &ctx, const GvParams &g, bool aligned,
                          const Extra &x = Extra()) {
    // One column per warp, 8 chunks (4 KiB of it) in flight per lane,
    // 128-thread CTAs.  Measured for M = 1 on 4096x4096 / 4096x22016 /
    // 11008x4096 (graphs over weight copies larger than L2): 4.2 / 5.7 / 4.5
    // TB/s, against 3.9 / 5.1 / 4.3 with two columns per warp and 256
    // threads; for M = 2 / 4 / 8 on 4096x4096: 5.95 / 9.7 / 16.7 us against
    // 6.6 / 10.7 / 19.3 (the tensor-core GEMV, 6.2 / 6.6 / 7.2 us, takes
    // M > 2).  The QKV epilogue needs its two columns per warp.
    if constexpr (kM == 1 && std::is_same<Extra, GvQkv>::value)
        return launch_gemv_cfg<1, 2, 8, 128>(ctx, g, aligned, x);
    else
        return launch_gemv_cfg<kM, 1, 8, 128>(ctx, g, aligned, x);
}

template <int kM, int kCols, int kUnroll, int kThreads, typename Extra>
cudaError_t launch_gemv_cfg(const LaunchCtx &ctx, const GvParams &g, bool aligned, const Extra &x) {
    constexpr int kColsPerCta = kThreads / 32 * kCols;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((g.N + kColsPerCta - 1) / kColsPerCta, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.stream = ctx.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = std::getenv("VNPU_B200_NO_PDL") ? 0 : 1;
    g_last_kernel.store("gemv_i8_kernel", std::memory_order_relaxed);
    if (aligned)
        return cudaLaunchKernelEx(&cfg, gemv_i8_kernel<kM, true, kCols, kUnroll, kThreads, Extra>,
                                  g, x);
    return cudaLaunchKernelEx(&cfg, gemv_i8_kernel<kM, false, kCols, kUnroll, kThreads, Extra>,
                              g, x);
}

// Driver entry point for cuTensorMapEncodeTiled, resolved once.
PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

bool encode_tmap_kmajor_i8(CUtensorMap *map, const void *base, uint64_t k_extent, uint64_t rows,
                           uint64_t row_stride_bytes, uint32_t box_k, uint32_t box_rows) {
    auto fn = tmap_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {k_extent, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_k, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t dim0,
                    uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swizzle) {
    auto fn = tmap_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

MatmulKernel choose_matmul_kernel(uint32_t M, uint32_t K, uint32_t N, uint32_t lda,
                                  const void *A) {
    (void)N;
    // TMA needs a 16-byte aligned base and a row stride that is a multiple of
    // 16 bytes; anything else takes the SIMT kernel (still on the GPU).
    const bool tma_ok = (reinterpret_cast<uintptr_t>(A) % 16u == 0u) && (lda % 16u == 0u) &&
                        K >= 16u;
    // VNPU_B200_FORCE_KERNEL=tcgen05|gemv|simt pins the choice where the kernel
    // can take the shape (tests use it to compare kernels on equal inputs).
    if (const char *f = std::getenv("VNPU_B200_FORCE_KERNEL")) {
        if (!std::strcmp(f, "simt")) return MatmulKernel::kSimt;
        if (!std::strcmp(f, "gemv") && M <= 8) return MatmulKernel::kGemv;
        if (!std::strcmp(f, "tcgen05") && tma_ok) return MatmulKernel::kTcgen05;
    }
    if (M <= 8) return MatmulKernel::kGemv;
    return tma_ok ? MatmulKernel::kTcgen05 : MatmulKernel::kSimt;
}

const char *last_matmul_kernel() { return g_last_kernel.load(std::memory_order_relaxed); }

const char *matmul_kernel_name(MatmulKernel k) {
    switch (k) {
    case MatmulKernel::kTcgen05: return "tcgen05";
    case MatmulKernel::kGemv: return "gemv";
    default: return "simt";
    }
}

namespace {

// Per-device one-time kernel set-up: shared-memory opt-in and the number of
// co-resident CTA pairs.
struct DeviceSetup {
    bool done = false;
    int max_pairs = 0;
    int max_wide_pairs = 0;
};
DeviceSetup g_setup[64];
std::mutex g_setup_mutex;

cudaError_t device_setup(int &max_pairs, int &max_wide_pairs) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return e != cudaSuccess ? e : cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> l(g_setup_mutex);
    DeviceSetup &d = g_setup[dev];
    if (!d.done) {
        if ((e = cudaFuncSetAttribute(gemm_i8_tcgen05_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kSmemBytes))) != cudaSuccess)
            return e;
        if ((e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, 6>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, 6)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<16, 5>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(16, 5)))) != cudaSuccess)
            return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(pair_threads(8), 1, 1);
        cfg.dynamicSmemBytes = pair_smem_bytes(8, 6);
        int clusters = 0;
        if ((e = cudaOccupancyMaxActiveClusters(&clusters, gemm_i8_tcgen05_pair_kernel<8, 6>,
                                                &cfg)) != cudaSuccess)
            return e;
        d.max_pairs = clusters;
        cfg.blockDim = dim3(pair_threads(16), 1, 1);
        cfg.dynamicSmemBytes = pair_smem_bytes(16, 5);
        if ((e = cudaOccupancyMaxActiveClusters(&clusters, gemm_i8_tcgen05_pair_kernel<16, 5>,
                                                &cfg)) != cudaSuccess)
            return e;
        if (clusters < d.max_pairs) d.max_pairs = clusters;
        if ((e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, 6, 224>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, 6, 224)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<16, 5, 224>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(16, 5, 224)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<16, 5, 256, true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(16, 5)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, 6, 256, false, kVarPlain>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, 6)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<16, 5, 256, false, kVarPlain>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(16, 5)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<16, 5, 256, false, kVarSilu>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(16, 5)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, kNarrowStages128, 128>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, kNarrowStages128, 128)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, kNarrowStages128, 128, false, kVarPlain>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, kNarrowStages128, 128)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, kNarrowStages64, 64>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, kNarrowStages64, 64)))) != cudaSuccess ||
            (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_kernel<8, kNarrowStages64, 64, false, kVarPlain>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(pair_smem_bytes(8, kNarrowStages64, 64)))) != cudaSuccess)
            return e;
        if ((e = wide_device_setup(d.max_wide_pairs)) != cudaSuccess) return e;
        d.done = true;
        if (std::getenv("VNPU_DEBUG"))
            std::fprintf(stderr, "[vnpu-b200] device %d: %d co-resident CTA pairs (256x256), %d (256x512)\n",
                         dev, d.max_pairs, d.max_wide_pairs);
    }
    max_pairs = d.max_pairs;
    max_wide_pairs = d.max_wide_pairs;
    return cudaSuccess;
}

}  // namespace

// Raster band height: as many m-tiles as keep the band's A panels (tile_m x
// K int8 each) within kRasterABytes of L2, so B streams from HBM once per band
// while the band's A stays resident.  VNPU_B200_GROUP_M overrides.
constexpr uint64_t kRasterABytes = 32ull << 20;

static uint32_t raster_group(uint32_t tiles_m, uint32_t tile_m, uint32_t K) {
    uint64_t g = kRasterABytes / (static_cast<uint64_t>(tile_m) * (K ? K : 1));
    if (const char *e = std::getenv("VNPU_B200_GROUP_M")) g = std::strtoull(e, nullptr, 10);
    if (g < 1) g = 1;
    if (g > tiles_m) g = tiles_m;
    return static_cast<uint32_t>(g);
}

// Tile shape of the CTA-pair GEMM: 256x256 or 256x224 (pair kernel),
// 256x512 or 256x448 (wide kernel), whichever has the least estimated time:
// waves (tiles over co-resident pairs, rounded up) x tile width / the tile's
// rate per output column relative to the 256x256 tile.  The wide tiles read a
// quarter fewer operand bytes per MAC (about 10% faster per column at
// K >= 8192, 2% at K = 4096, where more of the epilogue shows); 224-column
// tiles read more operand bytes per MAC than the 256-column ones.  Rates
// measured on B200 at M = K = 8192 (GEMM alone, us): N = 3584 pair 185.0,
// pair-224 188.5, wide 186.7, wide-224 179.3; N = 7168 353.1 / 367.7 /
// 339.6 / 322.0; N = 14336 683.8 / 806.8 / 651.2 / 633.7; N = 28672 wide
// 1265-1345, wide-224 1304.  The wide kernel only takes NONE / RELU
// epilogues (SiLU and GELU measured slower on it).
// With allow_narrow, shapes whose 256-column tiles leave pairs idle may take
// 256x128 or 256x64 tiles (pair kernel) when those still fit in one wave:
// the same operand rows spread over more SMs, each with a shorter MMA chain
// and a smaller share of the output to store.
// VNPU_B200_PAIR_WIDE=0|1 and VNPU_B200_PAIR_TN=64|128|224|256 pin the choice.
// Returns the chosen shape's estimated cost (0 when none qualifies);
// wide_only limits the choice to the wide kernel.
// Per-column rate of the narrow pair tiles relative to the 256x256 tile (a
// narrow tile reads more operand bytes per MAC and pays the same fixed cost
// per tile).  Measured on B200 (CUDA graph of 20 launches, us per launch,
// 256 / 128 / 64 columns): 512^3 7.54 / 6.38 / 5.65, 1024^3 8.97 / 7.90 /
// 7.64, 512x2048x2048 11.59 / 10.76 / 10.34, 256x4096x4096 16.87 / 16.36 /
// 15.80, 512x4096x4096 17.20 / 17.07 / 26.7 (two waves at 64).
constexpr double kNarrowRate128 = 0.80;
constexpr double kNarrowRate64 = 0.55;

double pick_pair_tile(uint32_t M, uint32_t N, uint32_t K, uint32_t epilogue, uint32_t pairs,
                      uint32_t wide_pairs, bool have_wide, bool &wide, uint32_t &tn,
                      bool wide_only = false, bool allow_narrow = false) {
    const uint32_t tiles_m = (M + kPTileM - 1) / kPTileM;
    const double wide_rate = K >= 8192u ? 1.10 : 1.02;
    const char *fw = std::getenv("VNPU_B200_PAIR_WIDE");
    const char *ft = std::getenv("VNPU_B200_PAIR_TN");
    double best = 0.0;
    bool first = true;
    for (int w = wide_only ? 1 : 0; w < 2; ++w) {
        if (w && (!have_wide || (epilogue > 1u && !fw))) continue;
        if (fw && (fw[0] == '1') != (w == 1)) continue;
        for (uint32_t t : {256u, 224u, 128u, 64u}) {
            if (ft && static_cast<uint32_t>(std::atoi(ft)) != t) continue;
            const bool narrow = t < 224u;
            if (narrow && (w || !(allow_narrow || ft))) continue;
            const uint32_t cols = w ? 2u * t : t;
            const uint32_t tiles = tiles_m * ((N + cols - 1) / cols);
            const uint32_t cap = w ? wide_pairs : pairs;
            // the wide tile needs a full wave to pay for its idle accumulator set
            if (w && tiles < cap && !fw) continue;
            // a narrow tile only where it still fits in one wave, and with a
            // SiLU / GELU epilogue only for short K (512x4096x4096 SiLU: 25.2 us
            // at 256x128 with 8 epilogue warps, 24.7 us at 256x256 with 16)
            if (narrow && !ft && (tiles > cap || (epilogue >= 2u && K > 1024u))) continue;
            const uint32_t waves = (tiles + cap - 1) / cap;
            const double rate = (w ? wide_rate : 1.0) *
                                (t == 224u ? (w ? 0.94 : 0.88)
                                           : t == 128u ? kNarrowRate128
                                                       : t == 64u ? kNarrowRate64 : 1.0);
            const double cost = waves * static_cast<double>(cols) / rate;
            // a 224-column tile must win clearly (3%): its rates are measured
            // at M = K = 8192 only
            if (first || cost < best * (t == 224u ? 0.97 : 0.995)) {
                best = cost;
                wide = w == 1;
                tn = t;
                first = false;
            }
        }
    }
    if (first) {
        wide = false;
        tn = 256;
        return 0.0;
    }
    return best;
}

cudaError_t matmul_i8_scatter(const LaunchCtx &ctx, const MatmulI8 &p) {
    int max_pairs = 0, max_wide_pairs = 0;
    cudaError_t se = device_setup(max_pairs, max_wide_pairs);
    if (se != cudaSuccess) return se;
    if (!p.tmap_b128 || max_pairs <= 0 || p.fmap.form == kFormMixed) return cudaErrorNotSupported;
    CUtensorMap tmap_a;
    if ((reinterpret_cast<uintptr_t>(p.A) % 16u) || (p.lda % 16u) ||
        !encode_tmap_kmajor_i8(&tmap_a, p.A, p.K, p.M, p.lda, kBK, 128))
        return cudaErrorNotSupported;
    TcParams tp;
    tp.scale_a = p.scale_a;
    tp.scale_b = p.scale_b;
    tp.bias = p.bias;
    tp.C = p.C;
    tp.ldc = p.ldc;
    tp.M = p.M;
    tp.N = p.N;
    tp.K = p.K;
    // The pair kernel's tile width (256 or 224) by the same estimate as
    // MATMUL_I8; the scatter epilogue has no wide-kernel form.
    bool wide = false;
    uint32_t tn = 256;
    pick_pair_tile(p.M, p.N, p.K, p.epilogue, static_cast<uint32_t>(max_pairs), 0, false, wide, tn);
    tp.tiles_m = (p.M + kPTileM - 1) / kPTileM;
    tp.tiles_n = (p.N + tn - 1) / tn;
    tp.num_kb = (p.K + kBK - 1) / kBK;
    tp.group_m = raster_group(tp.tiles_m, kPTileM, p.K);
    tp.epilogue = p.epilogue;
    tp.form = p.fmap.form;
    tp.variant = epi_variant(p.epilogue, p.bias != nullptr, p.fmap.form);
    tp.tma_store = 0;
    tp.err = ctx.err;
    tp.limit_ns = ctx.wait_limit_ns;
    for (uint32_t d = 0; d < p.ndst && d < 8u; ++d) tp.dst[d] = p.dst[d];
    tp.ndst = p.ndst;
    tp.ldd = p.ldd;
    tp.col_off = p.col_offset;
    CUtensorMap tmap_c;
    std::memset(&tmap_c, 0, sizeof(tmap_c));
    const uint32_t tiles = tp.tiles_m * tp.tiles_n;
    const uint32_t cap = static_cast<uint32_t>(max_pairs);
    const uint32_t pairs = tiles < cap ? tiles : cap;
    if (tn == 224u) {
        CUtensorMap tmap_b112;
        if (!encode_tmap_kmajor_i8(&tmap_b112, p.Bt, p.k_stride, p.N, p.k_stride, kBK, 112))
            return cudaErrorInvalidValue;
        VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, 6, 224>, dim3(2 * pairs),
                               dim3(pair_threads(8)), pair_smem_bytes(8, 6, 224), tmap_a, tmap_b112,
                               tmap_c, tp));
    } else {
        VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, 6>, dim3(2 * pairs),
                               dim3(pair_threads(8)), pair_smem_bytes(8, 6), tmap_a, *p.tmap_b128,
                               tmap_c, tp));
    }
    g_last_kernel.store(tn == 224u ? "gemm_i8_tcgen05_pair_kernel<224>" : "gemm_i8_tcgen05_pair_kernel",
                        std::memory_order_relaxed);
    count_launch(ctx);
    return cudaGetLastError();
}

// The CTA-pair GEMM split over K (tp filled for 256x256 tiles, tp.kb_per_split
// set): raw int32 sums of each split into a workspace, then
// splitk_finish_kernel.
cudaError_t matmul_i8_pair_splitk(const LaunchCtx &ctx, const MatmulI8 &p, TcParams tp,
                                  const CUtensorMap &tmap_a, uint32_t splits, uint32_t max_pairs) {
    tp.splits = splits;
    tp.m_pad = tp.tiles_m * kPTileM;
    const uint64_t rows = static_cast<uint64_t>(splits) * tp.m_pad;
    int32_t *ws = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&ws),
                                    rows * p.N * sizeof(int32_t), ctx.stream);
    if (e != cudaSuccess) return e;
    CUtensorMap tmap_w;
    tp.C = reinterpret_cast<float *>(ws);
    tp.ldc = p.N;
    tp.tma_store = encode_tmap_2d(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws, p.N, rows,
                                  static_cast<uint64_t>(p.N) * 4u, 32, 32,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (!tp.tma_store) std::memset(&tmap_w, 0, sizeof(tmap_w));
    const uint32_t units = tp.tiles_m * tp.tiles_n * splits;
    const uint32_t pairs = units < max_pairs ? units : max_pairs;
    e = launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, 6>, dim3(2 * pairs),
                   dim3(pair_threads(8)), pair_smem_bytes(8, 6), tmap_a, *p.tmap_b128, tmap_w, tp);
    count_launch(ctx);
    if (e == cudaSuccess) {
        const uint32_t total = p.M * (p.N / 4u);
        const uint32_t blocks = std::min<uint32_t>((total + 255u) / 256u,
                                                   static_cast<uint32_t>(ctx.num_sms) * 8u);
        e = launch_pdl(ctx.stream, splitk_finish_kernel, dim3(blocks), dim3(256), 0,
                       reinterpret_cast<const int4 *>(ws), splits, tp.m_pad, p.M, p.N, p.scale_a,
                       p.scale_b, p.bias, p.C, p.ldc, p.epilogue, p.fmap, p.R, p.ldr);
        count_launch(ctx);
    }
    cudaFreeAsync(ws, ctx.stream);
    g_last_kernel.store("gemm_i8_tcgen05_pair_kernel+splitk", std::memory_order_relaxed);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t matmul_i8_swiglu(const LaunchCtx &ctx, const MatmulI8 &p, float *Y, uint32_t ldy,
                             float alpha) {
    const uint32_t I = p.N / 2u;
    if ((p.N & 1u) || I == 0 || p.R || p.ndst) return cudaErrorInvalidValue;
    const bool no_epi = std::getenv("VNPU_B200_NO_SWIGLU_EPI") != nullptr;
    // Decode: one warp streams gate column j and up column I + j.
    if (!no_epi && p.M <= 2u) {
        const cudaError_t e = matmul_i8_swiglu_gemv_stream(ctx, p, Y, ldy, I, alpha);
        if (e != cudaErrorInvalidValue) {
            if (e == cudaSuccess) g_last_kernel.store("gemv_i8_stream_kernel+swiglu", std::memory_order_relaxed);
            return e;
        }
    }
    int max_pairs = 0, max_wide_pairs = 0;
    cudaError_t se = device_setup(max_pairs, max_wide_pairs);
    if (se != cudaSuccess) return se;
    // The CTA pair's two B halves are the gate rows and the matching up rows.
    CUtensorMap tmap_a;
    const bool pair_ok = !no_epi && p.M > kBM && p.tmap_b128 && max_pairs > 0 &&
                         p.fmap.form != kFormMixed &&
                         choose_matmul_kernel(p.M, p.K, p.N, p.lda, p.A) == MatmulKernel::kTcgen05 &&
                         encode_tmap_kmajor_i8(&tmap_a, p.A, p.K, p.M, p.lda, kBK, 128);
    if (pair_ok) {
        TcParams tp;
        tp.scale_a = p.scale_a;
        tp.scale_b = p.scale_b;
        tp.bias = p.bias;
        tp.C = Y;
        tp.ldc = ldy;
        tp.M = p.M;
        tp.N = p.N;
        tp.K = p.K;
        tp.tiles_m = (p.M + kPTileM - 1) / kPTileM;
        tp.tiles_n = (I + 127u) / 128u;
        tp.num_kb = (p.K + kBK - 1) / kBK;
        tp.group_m = raster_group(tp.tiles_m, kPTileM, p.K);
        tp.epilogue = p.epilogue;
        tp.form = p.fmap.form;
        tp.variant = epi_variant(p.epilogue, p.bias != nullptr, p.fmap.form);
        tp.err = ctx.err;
        tp.limit_ns = ctx.wait_limit_ns;
        tp.swiglu_i = I;
        tp.swiglu_alpha = alpha;
        CUtensorMap tmap_c;
        tp.tma_store = (reinterpret_cast<uintptr_t>(Y) % 16u == 0u) && (ldy % 4u == 0u) &&
                       encode_tmap_2d(&tmap_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, Y, I, p.M,
                                      static_cast<uint64_t>(ldy) * 4u, 32, 32,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
        if (!tp.tma_store) std::memset(&tmap_c, 0, sizeof(tmap_c));
        const uint32_t tiles = tp.tiles_m * tp.tiles_n;
        const uint32_t pairs = tiles < static_cast<uint32_t>(max_pairs) ? tiles
                                                                        : static_cast<uint32_t>(max_pairs);
        // 16 epilogue warps: the SwiGLU's exp and division per element make
        // the epilogue latency-bound, as with the SiLU / GELU epilogues.
        VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<16, 5, 256, true>,
                               dim3(2 * pairs), dim3(pair_threads(16)), pair_smem_bytes(16, 5),
                               tmap_a, *p.tmap_b128, tmap_c, tp));
        g_last_kernel.store("gemm_i8_tcgen05_pair_kernel+swiglu", std::memory_order_relaxed);
        count_launch(ctx);
        return cudaGetLastError();
    }
    // Elsewhere: the product into stream-ordered scratch, then the halves.
    float *scratch = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&scratch),
                                    static_cast<size_t>(p.M) * p.N * sizeof(float), ctx.stream);
    if (e != cudaSuccess) return e;
    MatmulI8 q = p;
    q.C = scratch;
    q.ldc = p.N;
    e = matmul_i8(ctx, q);
    if (e == cudaSuccess) e = swiglu_rows(ctx, scratch, p.N, Y, ldy, p.M, I, alpha);
    cudaFreeAsync(scratch, ctx.stream);
    return e;
}

cudaError_t matmul_i8_tcgen05(const LaunchCtx &ctx, const MatmulI8 &p) {
    int max_pairs = 0, max_wide_pairs = 0;
    cudaError_t se = device_setup(max_pairs, max_wide_pairs);
    if (se != cudaSuccess) return se;
    if (!p.tmap_b) return cudaErrorInvalidValue;
    // Elements in more than one rounding form: raw int32 sums split over K
    // and the finish kernel's per-element epilogue, or the SIMT kernel.
    const bool mixed = p.fmap.form == kFormMixed;
    // Pairs of CTAs (256x256 tiles) whenever M fills more than one 128-row
    // tile; the single-CTA 128x256 kernel otherwise.
    const bool use_pair = p.M > kBM && p.tmap_b128 && max_pairs > 0 &&
                          std::getenv("VNPU_B200_NO_PAIR") == nullptr;
    if (use_pair) {
        CUtensorMap tmap_a;
        if (!encode_tmap_kmajor_i8(&tmap_a, p.A, p.K, p.M, p.lda, kBK, 128))
            return cudaErrorInvalidValue;
        TcParams tp;
        tp.scale_a = p.scale_a;
        tp.scale_b = p.scale_b;
        tp.bias = p.bias;
        tp.C = p.C;
        tp.ldc = p.ldc;
        tp.M = p.M;
        tp.N = p.N;
        tp.K = p.K;
        // 256x512 tiles when they fill at least one wave of pairs, cost fewer
        // waves than the 256x256 tiles after their per-tile speed-up (measured
        // on B200: ~10% at K >= 8192, ~2% at K = 4096, where the wide tile's
        // half-hidden epilogue weighs more), and the epilogue is light (NONE /
        // RELU: SiLU and GELU epilogues are slower on the wide tile).
        const uint32_t tiles_m = (p.M + kPTileM - 1) / kPTileM;
        const uint32_t tiles_p = tiles_m * ((p.N + kPTileN - 1) / kPTileN);
        const uint32_t wp = static_cast<uint32_t>(max_wide_pairs > 0 ? max_wide_pairs : 1);
        const uint32_t pp = static_cast<uint32_t>(max_pairs > 0 ? max_pairs : 1);
        // Tile shape: the one with the least estimated time, waves x tile
        // width / relative rate per column (pair_tile_cost).
        // (Shapes that split K keep the 256x256 tile: the split rule below.)
        uint32_t tn = 256;
        bool wide = false;
        const bool no_splitk = std::getenv("VNPU_B200_NO_SPLITK") != nullptr;
        const uint32_t kb_total = (p.K + kBK - 1) / kBK;
        // Without a residual a split must keep >= 24 k-blocks (512x4096x4096:
        // 17.3 us unsplit against 18.2 us in two splits of 16); the residual
        // rides on the split-K finish kernel, so it splits from 8.
        uint32_t kb_min = p.R ? 8u : 24u;
        if (const char *e = std::getenv("VNPU_B200_SPLITK_MIN_KB"))   // tests pin it
            kb_min = std::max(1, std::atoi(e));
        const bool splits_k = !no_splitk && p.N % 4u == 0u &&
                              std::min(std::min(pp / tiles_p, 4u), kb_total / kb_min) >= 2u;
        if (!mixed && !splits_k)
            pick_pair_tile(p.M, p.N, p.K, p.epilogue, pp, wp, max_wide_pairs > 0, wide, tn,
                           false, true);
        tp.tiles_m = tiles_m;
        const uint32_t tile_cols = wide ? 2u * tn : tn;
        tp.tiles_n = (p.N + tile_cols - 1) / tile_cols;
        tp.num_kb = (p.K + kBK - 1) / kBK;
        // Split K when the 256x256 tiles leave at least half of the pairs idle
        // and K is long: each split (at least 8 k-blocks) sums its range into
        // a stream-ordered int32 workspace, a second kernel adds the splits
        // (exact) and applies the epilogue.
        tp.group_m = raster_group(tp.tiles_m, kPTileM, p.K);
        tp.epilogue = p.epilogue;
        tp.form = p.fmap.form;
        tp.variant = epi_variant(p.epilogue, p.bias != nullptr, p.fmap.form);
        tp.err = ctx.err;
        tp.limit_ns = ctx.wait_limit_ns;
        uint32_t splits = 1;
        if (!wide && tn == 256u && p.N % 4u == 0u && !no_splitk) {
            uint32_t sk = pp / tiles_p;
            sk = std::min(sk, 4u);
            sk = std::min(sk, tp.num_kb / kb_min);
            if (sk >= 2) {
                tp.kb_per_split = (tp.num_kb + sk - 1) / sk;
                splits = (tp.num_kb + tp.kb_per_split - 1) / tp.kb_per_split;
            }
        }
        if (mixed && splits == 1 && p.N % 4u == 0u && tp.num_kb >= 2u) {
            tp.kb_per_split = (tp.num_kb + 1u) / 2u;
            splits = (tp.num_kb + tp.kb_per_split - 1u) / tp.kb_per_split;
        }
        if (mixed && splits == 1)
            return p.R ? cudaErrorNotSupported : matmul_i8_simt(ctx, p);
        if (splits > 1)   // every other field of tp is set above
            return matmul_i8_pair_splitk(ctx, p, tp, tmap_a, splits, static_cast<uint32_t>(max_pairs));
        if (p.R) return cudaErrorNotSupported;   // the residual rides on the split-K finish only
        CUtensorMap tmap_c;
        tp.tma_store = (reinterpret_cast<uintptr_t>(p.C) % 16u == 0u) && (p.ldc % 4u == 0u) &&
                       encode_tmap_2d(&tmap_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.C, p.N, p.M,
                                      static_cast<uint64_t>(p.ldc) * 4u, 32, 32,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
        if (!tp.tma_store) std::memset(&tmap_c, 0, sizeof(tmap_c));
        const uint32_t tiles = tp.tiles_m * tp.tiles_n;
        const uint32_t cap = static_cast<uint32_t>(wide ? max_wide_pairs : max_pairs);
        const uint32_t pairs = tiles < cap ? tiles : cap;
        // 224-, 128- and 64-column tiles: each CTA loads tn / 2 weight rows
        // per stage (its own box height); the 128-row map serves the
        // 256-column tiles.
        CUtensorMap tmap_bn;
        const CUtensorMap *tmap_b = p.tmap_b128;
        if (tn != 256u) {
            if (!encode_tmap_kmajor_i8(&tmap_bn, p.Bt, p.k_stride, p.N, p.k_stride, kBK, tn / 2u))
                return cudaErrorInvalidValue;
            tmap_b = &tmap_bn;
        }
        // 16 epilogue warps: SiLU / GELU (latency-bound epilogue), or one short
        // tile per pair with the per-launch variant switch (the epilogue is
        // most of the time: 512^3 9.3 -> 8.8 us).  With the NONE/no-bias
        // variant compiled in, 8 warps are faster there too (512^3 7.80 ->
        // 7.55 us, 1024^3 9.34 -> 9.02 us).
        bool epi16 = p.epilogue >= 2 ||
                     (tiles <= cap && tp.num_kb <= 8u && !use_plain_variant(tp.variant));
        if (const char *e = std::getenv("VNPU_B200_EPI_WARPS")) epi16 = std::atoi(e) == 16;
        // Narrow tiles: 8 epilogue warps (at most four 32-column chunks per tile).
        if (tn == 128u && use_plain_variant(tp.variant))
            VNPU_LAUNCH(launch_pdl(ctx.stream,
                                   gemm_i8_tcgen05_pair_kernel<8, kNarrowStages128, 128, false, kVarPlain>,
                                   dim3(2 * pairs), dim3(pair_threads(8)),
                                   pair_smem_bytes(8, kNarrowStages128, 128), tmap_a, *tmap_b, tmap_c, tp));
        else if (tn == 128u)
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, kNarrowStages128, 128>,
                                   dim3(2 * pairs), dim3(pair_threads(8)),
                                   pair_smem_bytes(8, kNarrowStages128, 128), tmap_a, *tmap_b, tmap_c, tp));
        else if (tn == 64u && use_plain_variant(tp.variant))
            VNPU_LAUNCH(launch_pdl(ctx.stream,
                                   gemm_i8_tcgen05_pair_kernel<8, kNarrowStages64, 64, false, kVarPlain>,
                                   dim3(2 * pairs), dim3(pair_threads(8)),
                                   pair_smem_bytes(8, kNarrowStages64, 64), tmap_a, *tmap_b, tmap_c, tp));
        else if (tn == 64u)
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, kNarrowStages64, 64>,
                                   dim3(2 * pairs), dim3(pair_threads(8)),
                                   pair_smem_bytes(8, kNarrowStages64, 64), tmap_a, *tmap_b, tmap_c, tp));
        else if (wide)
            VNPU_LAUNCH(launch_wide_pair(ctx.stream, tn, pairs, tmap_a, *tmap_b, tmap_c, tp));
        else if (epi16 && tn == 224u)
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<16, 5, 224>,
                                   dim3(2 * pairs), dim3(pair_threads(16)),
                                   pair_smem_bytes(16, 5, 224), tmap_a, *tmap_b, tmap_c, tp));
        else if (epi16 && use_compiled_variant(tp.variant, kVarSilu))
            VNPU_LAUNCH(launch_pdl(ctx.stream,
                                   gemm_i8_tcgen05_pair_kernel<16, 5, 256, false, kVarSilu>,
                                   dim3(2 * pairs), dim3(pair_threads(16)), pair_smem_bytes(16, 5),
                                   tmap_a, *tmap_b, tmap_c, tp));
        else if (epi16 && use_plain_variant(tp.variant))
            VNPU_LAUNCH(launch_pdl(ctx.stream,
                                   gemm_i8_tcgen05_pair_kernel<16, 5, 256, false, kVarPlain>,
                                   dim3(2 * pairs), dim3(pair_threads(16)), pair_smem_bytes(16, 5),
                                   tmap_a, *tmap_b, tmap_c, tp));
        else if (epi16)
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<16, 5>, dim3(2 * pairs),
                                   dim3(pair_threads(16)), pair_smem_bytes(16, 5), tmap_a,
                                   *tmap_b, tmap_c, tp));
        else if (tn == 224u)
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, 6, 224>,
                                   dim3(2 * pairs), dim3(pair_threads(8)),
                                   pair_smem_bytes(8, 6, 224), tmap_a, *tmap_b, tmap_c, tp));
        else if (use_plain_variant(tp.variant))
            VNPU_LAUNCH(launch_pdl(ctx.stream,
                                   gemm_i8_tcgen05_pair_kernel<8, 6, 256, false, kVarPlain>,
                                   dim3(2 * pairs), dim3(pair_threads(8)), pair_smem_bytes(8, 6),
                                   tmap_a, *tmap_b, tmap_c, tp));
        else
            VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_pair_kernel<8, 6>, dim3(2 * pairs),
                                   dim3(pair_threads(8)), pair_smem_bytes(8, 6), tmap_a,
                                   *tmap_b, tmap_c, tp));
        g_last_kernel.store(wide ? (tn == 224u ? "gemm_i8_tcgen05_pair_wide_kernel<224>"
                                               : "gemm_i8_tcgen05_pair_wide_kernel")
                                 : tn == 224u ? "gemm_i8_tcgen05_pair_kernel<224>"
                                 : tn == 128u ? "gemm_i8_tcgen05_pair_kernel<128>"
                                 : tn == 64u  ? "gemm_i8_tcgen05_pair_kernel<64>"
                                              : "gemm_i8_tcgen05_pair_kernel",
                            std::memory_order_relaxed);
        count_launch(ctx);
        return cudaGetLastError();
    }
    if (p.R) return cudaErrorNotSupported;
    if (mixed) return matmul_i8_simt(ctx, p);
    CUtensorMap tmap_a;
    if (!encode_tmap_kmajor_i8(&tmap_a, p.A, p.K, p.M, p.lda, kBK, kBM))
        return cudaErrorInvalidValue;
    TcParams tp;
    tp.scale_a = p.scale_a;
    tp.scale_b = p.scale_b;
    tp.bias = p.bias;
    tp.C = p.C;
    tp.ldc = p.ldc;
    tp.M = p.M;
    tp.N = p.N;
    tp.K = p.K;
    tp.tiles_m = (p.M + kBM - 1) / kBM;
    tp.tiles_n = (p.N + kBN - 1) / kBN;
    tp.num_kb = (p.K + kBK - 1) / kBK;
    tp.group_m = raster_group(tp.tiles_m, kBM, p.K);
    tp.epilogue = p.epilogue;
    tp.form = p.fmap.form;
    tp.variant = epi_variant(p.epilogue, p.bias != nullptr, p.fmap.form);
    tp.tma_store = 0;
    tp.err = ctx.err;
    tp.limit_ns = ctx.wait_limit_ns;
    const uint32_t tiles = tp.tiles_m * tp.tiles_n;
    const uint32_t grid = tiles < static_cast<uint32_t>(ctx.num_sms) ? tiles
                                                                     : static_cast<uint32_t>(ctx.num_sms);
    VNPU_LAUNCH(launch_pdl(ctx.stream, gemm_i8_tcgen05_kernel, dim3(grid), dim3(kThreads),
                           kSmemBytes, tmap_a, *p.tmap_b, tp));
    g_last_kernel.store("gemm_i8_tcgen05_kernel", std::memory_order_relaxed);
    count_launch(ctx);
    return cudaGetLastError();
}

namespace {

template <uint32_t kStages, uint32_t kMinBlocks>
cudaError_t gemv_tcgen05_launch(const LaunchCtx &ctx, const MatmulI8 &p, const CUtensorMap &tmap_x,
                                SkParams sp) {
    // Split K over a cluster so that about kMinBlocks CTAs per SM stream weights.
    const uint32_t blocks = (p.N + 127u) / 128u;
    // Clusters of at most 4: measured best on B200 (8-CTA clusters fit the
    // GPCs less evenly).
    uint32_t max_c = 4u;
    if (const char *e = std::getenv("VNPU_B200_DECODE_CLUSTER")) max_c = std::max(1, std::atoi(e));
    if (max_c > kSkMaxCluster) max_c = kSkMaxCluster;
    while (max_c > 1 && sk_smem_bytes(kStages, max_c) > 226u * 1024u) max_c /= 2u;
    uint32_t csize = 1;
    while (csize < max_c &&
           blocks * csize * 2u <= kMinBlocks * static_cast<uint32_t>(ctx.num_sms) &&
           csize * 2u <= sp.num_kb)
        csize *= 2u;
    sp.kb_per_rank = (sp.num_kb + csize - 1) / csize;
    // Opt in to the shared memory this launch needs (per device, grown on demand).
    static uint32_t opted[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t smem = sk_smem_bytes(kStages, csize);
    if (dev < 0 || dev >= 64 || opted[dev] < smem) {
        const cudaError_t e = cudaFuncSetAttribute(gemv_i8_tcgen05_kernel<kStages, kMinBlocks>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) opted[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks * csize, 1, 1);
    cfg.blockDim = dim3(kSkThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx.stream;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = csize;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = std::getenv("VNPU_B200_NO_PDL") ? 1 : 2;
    g_last_kernel.store("gemv_i8_tcgen05_kernel", std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, gemv_i8_tcgen05_kernel<kStages, kMinBlocks>, *p.tmap_b128,
                              tmap_x, sp);
}

cudaError_t gemv_tcgen05(const LaunchCtx &ctx, const MatmulI8 &p) {
    CUtensorMap tmap_x;
    if (!encode_tmap_kmajor_i8(&tmap_x, p.A, p.K, p.M, p.lda, kBK, 8)) return cudaErrorInvalidValue;
    SkParams sp;
    sp.scale_a = p.scale_a;
    sp.scale_b = p.scale_b;
    sp.bias = p.bias;
    sp.C = p.C;
    sp.ldc = p.ldc;
    sp.M = p.M;
    sp.N = p.N;
    sp.K = p.K;
    sp.num_kb = (p.K + kBK - 1) / kBK;
    sp.epilogue = p.epilogue;
    sp.fmap = p.fmap;
    sp.err = ctx.err;
    sp.limit_ns = ctx.wait_limit_ns;
    // Five 17 KiB stages at two CTAs per SM: measured best of 4/5/8/12 on B200
    // (deeper rings at one CTA per SM leave no room for the next launch).
    uint32_t stages = 5;
    if (const char *e = std::getenv("VNPU_B200_GEMV_STAGES")) stages = std::atoi(e);
    switch (stages) {
    case 4: return gemv_tcgen05_launch<4, 2>(ctx, p, tmap_x, sp);
    case 8: return gemv_tcgen05_launch<8, 1>(ctx, p, tmap_x, sp);
    default: return gemv_tcgen05_launch<5, 2>(ctx, p, tmap_x, sp);
    }
}

}  // namespace

cudaError_t matmul_i8_gemv(const LaunchCtx &ctx, const MatmulI8 &p) {
    const GvParams g = gv_params(p);
    const bool aligned = (reinterpret_cast<uintptr_t>(p.A) % 16u == 0u) && (p.lda % 16u == 0u);
    // The mma.sync GEMV (M <= 8) and the one-column-per-warp streaming GEMV
    // (M <= 2) where they take the shape; VNPU_B200_DECODE=mma|stream|tc|simt
    // selects one kernel (tests compare them).
    const char *decode = std::getenv("VNPU_B200_DECODE");
    if (!std::getenv("VNPU_B200_SIMT_GEMV")) {
        const bool mma = decode ? std::strcmp(decode, "mma") == 0 && gemv_mma_supported(p)
                                : gemv_mma_preferred(p);
        if (mma) {
            g_last_kernel.store("gemv_i8_mma_kernel", std::memory_order_relaxed);
            return matmul_i8_gemv_mma(ctx, p, nullptr, 0, 0);
        }
        if ((!decode || std::strcmp(decode, "stream") == 0) && gemv_stream_supported(p, 1)) {
            g_last_kernel.store("gemv_i8_stream_kernel", std::memory_order_relaxed);
            return matmul_i8_gemv_stream(ctx, p);
        }
    }
    bool use_tc = p.M > 2;
    if (decode) use_tc = std::strcmp(decode, "tc") == 0;
    if (std::getenv("VNPU_B200_SIMT_GEMV")) use_tc = false;
    if (use_tc && aligned && p.K >= 16u && p.tmap_b128) {
        const cudaError_t e = gemv_tcgen05(ctx, p);
        count_launch(ctx);
        return e;
    }
    cudaError_t e;
    switch (p.M) {
    case 1: e = launch_gemv_m<1>(ctx, g, aligned); break;
    case 2: e = launch_gemv_m<2>(ctx, g, aligned); break;
    case 3: e = launch_gemv_m<3>(ctx, g, aligned); break;
    case 4: e = launch_gemv_m<4>(ctx, g, aligned); break;
    default: e = launch_gemv_m<8>(ctx, g, aligned); break;
    }
    count_launch(ctx);
    return e;
}

cudaError_t matmul_i8_gemv_residual(const LaunchCtx &ctx, const MatmulI8 &p, const float *R,
                                    uint32_t ldr) {
    if (p.M != 1) return cudaErrorInvalidValue;
    const char *decode = std::getenv("VNPU_B200_DECODE");
    if (!std::getenv("VNPU_B200_SIMT_GEMV")) {
        const bool mma = decode ? std::strcmp(decode, "mma") == 0 && gemv_mma_supported(p)
                                : gemv_mma_preferred(p);
        if (mma) {
            g_last_kernel.store("gemv_i8_mma_kernel", std::memory_order_relaxed);
            return matmul_i8_gemv_mma(ctx, p, R, ldr, 0);
        }
        if ((!decode || std::strcmp(decode, "stream") == 0) && gemv_stream_supported(p, 1)) {
            g_last_kernel.store("gemv_i8_stream_kernel", std::memory_order_relaxed);
            return matmul_i8_gemv_stream(ctx, p, R, ldr);
        }
    }
    const GvParams g = gv_params(p);
    const bool aligned = (reinterpret_cast<uintptr_t>(p.A) % 16u == 0u) && (p.lda % 16u == 0u);
    const cudaError_t e =
        launch_gemv_m<1>(ctx, g, aligned, GvResidual{R, ldr, p.advance_pos, p.advance});
    count_launch(ctx);
    return e;
}

cudaError_t qkv_rope_append_gemv(const LaunchCtx &ctx, const MatmulI8 &p, const QkvRope &q) {
    if (p.M != 1 || q.head_dim == 0 || (q.head_dim & 1u) || q.head_dim / 2 > kGvMaxPairs ||
        p.N != 3u * q.heads * q.head_dim)
        return cudaErrorInvalidValue;
    if (!std::getenv("VNPU_B200_DECODE") && !std::getenv("VNPU_B200_SIMT_GEMV") &&
        gemv_stream_supported(p, 2)) {
        g_last_kernel.store("gemv_i8_stream_kernel", std::memory_order_relaxed);
        return qkv_rope_append_gemv_stream(ctx, p, q);
    }
    const GvParams g = gv_params(p);
    const bool aligned = (reinterpret_cast<uintptr_t>(p.A) % 16u == 0u) && (p.lda % 16u == 0u);
    GvQkv x;
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
    const cudaError_t e = launch_gemv_m<1>(ctx, g, aligned, x);
    count_launch(ctx);
    return e;
}

cudaError_t matmul_i8_simt(const LaunchCtx &ctx, const MatmulI8 &p) {
    const GvParams g = gv_params(p);
    dim3 grid((p.N + 63) / 64, (p.M + 63) / 64);
    gemm_i8_simt_kernel<<<grid, 256, 0, ctx.stream>>>(g);
    g_last_kernel.store("gemm_i8_simt_kernel", std::memory_order_relaxed);
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t matmul_i8_split_residual(const LaunchCtx &ctx, const MatmulI8 &p) {
    if (!p.R || p.ndst != 0 ||
        choose_matmul_kernel(p.M, p.K, p.N, p.lda, p.A) != MatmulKernel::kTcgen05)
        return cudaErrorNotSupported;
    return matmul_i8_tcgen05(ctx, p);
}

cudaError_t matmul_i8(const LaunchCtx &ctx, const MatmulI8 &p) {
    switch (choose_matmul_kernel(p.M, p.K, p.N, p.lda, p.A)) {
    case MatmulKernel::kTcgen05: return matmul_i8_tcgen05(ctx, p);
    case MatmulKernel::kGemv: return matmul_i8_gemv(ctx, p);
    default: return matmul_i8_simt(ctx, p);
    }
}

}  // namespace vnpu_b200
