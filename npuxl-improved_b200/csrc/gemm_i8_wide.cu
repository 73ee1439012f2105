// gemm_i8_wide.cu - the wide tcgen05 CTA-pair GEMM (MATMUL_I8 for large
// shapes), in its own translation unit so it compiles beside gemm_i8.cu.
#include <cudaTypedefs.h>

#include "gemm_tc.cuh"

namespace vnpu_b200 {
namespace {

template <uint32_t kTN = 256, uint32_t kVar = kVarRuntime>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    gemm_i8_tcgen05_pair_wide_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                     const __grid_constant__ CUtensorMap tmap_b,
                                     const __grid_constant__ CUtensorMap tmap_c,
                                     const TcParams p) {
    static_assert(kTN % 32u == 0u && kTN <= 256u, "wide accumulator width");
    constexpr uint32_t kBRows = kTN / 2u;                  // B rows per CTA and accumulator
    constexpr uint32_t kBBytes1 = kBRows * kBK;
    constexpr uint32_t kStageW = wide_stage_bytes(kTN);
    constexpr uint32_t kTileW = 2u * kTN;
    constexpr uint32_t kHalfChunks = kTN / 32u;            // 32-column chunks per accumulator
    constexpr uint32_t kChunks = (kHalfChunks + 1u) / 2u;  // per column group of warps
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kWStages];
    __shared__ __align__(8) uint64_t empty_bar[kWStages];
    __shared__ __align__(8) uint64_t tmem_full_bar;
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
    const uint32_t total_tiles = p.tiles_m * p.tiles_n;   // 256x512 tiles

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kWStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&tmem_full_bar, 1);
        mbar_init(&tmem_empty_bar[0], 2 * kPEpiWarps);
        mbar_init(&tmem_empty_bar[1], 2 * kPEpiWarps);
        mbar_init(&drain_bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        if (p.tma_store) tma_prefetch_desc(&tmap_c);
    }
    if (warp == 1) {
        tmem_alloc_pair(&tmem_base_slot, kWTmemCols);
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
                tile_coords(t, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
                for (uint32_t kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % kWStages;
                    const uint32_t ph = (it / kWStages) & 1u;
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, p.limit_ns, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * kStageW);
                    const uint32_t leader_full = mapa_shared(smem_addr(&full_bar[s]), 0);
                    uint8_t *sa = ring + s * kStageW;
                    const int32_t k0 = static_cast<int32_t>(kb * kBK);
                    const uint32_t n_first = nb * kTileW + rank * kBRows;
                    tma_load_2d_pair(sa, &tmap_a, leader_full, k0,
                                     static_cast<int32_t>(mb * kPTileM + rank * 128u));
                    tma_load_2d_pair(sa + kPABytes, &tmap_b, leader_full, k0,
                                     static_cast<int32_t>(n_first));
                    tma_load_2d_pair(sa + kPABytes + kBBytes1, &tmap_b, leader_full, k0,
                                     static_cast<int32_t>(n_first + kTN));
                }
            }
            if (rank == 0) {
                const uint32_t tail = it < kWStages ? it : kWStages;
                for (uint32_t i = it - tail; i < it; ++i)
                    mbar_wait(&full_bar[i % kWStages], (i / kWStages) & 1u, p.limit_ns, p.err,
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
                const uint32_t empty_par = (tcount & 1u) ^ 1u;
                const uint32_t hold = p.num_kb < kWStages ? p.num_kb : kWStages;
                // D0 over the first `hold` k-blocks (stages held).
                if (!mbar_wait(&tmem_empty_bar[0], empty_par, p.limit_ns, p.err, &abort_flag))
                    break;
                tc_fence_after();
                for (uint32_t kb = 0; kb < hold; ++kb) {
                    const uint32_t i = it + kb;
                    if (!mbar_wait(&full_bar[i % kWStages], (i / kWStages) & 1u, p.limit_ns,
                                   p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(ring + (i % kWStages) * kStageW);
                    const uint64_t adesc = umma_desc_k_sw128(sa);
                    const uint64_t b0 = umma_desc_k_sw128(sa + kPABytes);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk)
                        umma_i8_pair(tmem_base, adesc + 2u * kk, b0 + 2u * kk, idesc,
                                     (kb | kk) != 0u);
                }
                if (!ok) break;
                // D1 over the held k-blocks once the epilogue has read D1.
                if (!mbar_wait(&tmem_empty_bar[1], empty_par, p.limit_ns, p.err, &abort_flag))
                    break;
                tc_fence_after();
                for (uint32_t kb = 0; kb < hold; ++kb) {
                    const uint32_t i = it + kb;
                    const uint32_t sa = smem_addr(ring + (i % kWStages) * kStageW);
                    const uint64_t adesc = umma_desc_k_sw128(sa);
                    const uint64_t b1 = umma_desc_k_sw128(sa + kPABytes + kBBytes1);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk)
                        umma_i8_pair(tmem_base + kTN, adesc + 2u * kk, b1 + 2u * kk, idesc,
                                     (kb | kk) != 0u);
                    umma_commit_pair_mc(&empty_bar[i % kWStages], 0x3);
                }
                it += hold;
                // Remaining k-blocks: D0 and D1 per stage.
                for (uint32_t kb = hold; kb < p.num_kb; ++kb, ++it) {
                    const uint32_t s = it % kWStages;
                    if (!mbar_wait(&full_bar[s], (it / kWStages) & 1u, p.limit_ns, p.err,
                                   &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(ring + s * kStageW);
                    const uint64_t adesc = umma_desc_k_sw128(sa);
                    const uint64_t b0 = umma_desc_k_sw128(sa + kPABytes);
                    const uint64_t b1 = umma_desc_k_sw128(sa + kPABytes + kBBytes1);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / kUmmaK; ++kk) {
                        umma_i8_pair(tmem_base, adesc + 2u * kk, b0 + 2u * kk, idesc, true);
                        umma_i8_pair(tmem_base + kTN, adesc + 2u * kk, b1 + 2u * kk, idesc,
                                     true);
                    }
                    umma_commit_pair_mc(&empty_bar[s], 0x3);
                }
                if (!ok) break;
                umma_commit_pair_mc(&tmem_full_bar, 0x3);
            }
            umma_commit_pair_mc(&drain_bar, 0x1);
            mbar_wait(&drain_bar, 0, p.limit_ns, p.err, nullptr);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Warp w reads TMEM lanes 32*(w%4)..+31.  For half h, warps 2-5 take
        // the first kChunks 32-column chunks of accumulator h (columns
        // kTN*h + 0..127 when kTN = 256) and warps 6-9 the rest, in 32x32
        // chunks: dequantised in registers, written 128B-swizzled into the
        // warp's 4 KiB staging buffer and stored to C by TMA (rows >= M and
        // columns >= N clipped by the tensor map), or stored directly without
        // a C tensor map.
        const uint32_t lane_base = (warp & 3u) * 32u;
        const uint32_t chunk0 = ((warp - 2u) >> 2) * kChunks;
        const uint32_t col_base = chunk0 * 32u;
        const bool vec_ok = (p.ldc % 4u == 0u) &&
                            ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0u);
        uint8_t *stage_out = ring + kWStages * kStageW + (warp - 2u) * kPStageOutBytes;
        float *my_row = reinterpret_cast<float *>(stage_out + lane * 128u);
        const uint32_t leader_empty0 = mapa_shared(smem_addr(&tmem_empty_bar[0]), 0);
        const uint32_t leader_empty1 = mapa_shared(smem_addr(&tmem_empty_bar[1]), 0);
        uint32_t tcount = 0;
        for (uint32_t t = pair; t < total_tiles; t += npairs, ++tcount) {
            uint32_t mb, nb;
            tile_coords(t, p.tiles_m, p.tiles_n, p.group_m, mb, nb);
            // Scales and biases for the tile, fetched before the accumulators are ready.
            const uint32_t m_first = mb * kPTileM + rank * 128u + lane_base;  // warp's first row
            const uint32_t m = m_first + lane;
            const bool row_ok = m < p.M;
            const float sa = row_ok ? (p.scale_a ? __ldg(p.scale_a + m) : 1.0f) : 0.0f;
            float sreg[2 * kChunks], breg[2 * kChunks];
#pragma unroll
            for (uint32_t c = 0; c < 2u * kChunks; ++c)
                fetch_col(p, nb * kTileW + (c / kChunks) * kTN + col_base + (c % kChunks) * 32u + lane,
                          sreg[c], breg[c]);
            uint32_t ok = 0;
            if (lane == 0)
                ok = mbar_wait(&tmem_full_bar, tcount & 1u, p.limit_ns, p.err, &abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            float *crow = p.C + static_cast<uint64_t>(row_ok ? m : 0) * p.ldc;
#pragma unroll
            for (uint32_t h = 0; h < 2u; ++h) {
                // The warp's 128 columns of half h go to registers in one
                // round of loads, and the half is released before any of it
                // is dequantised or stored: the next tile's MMAs into this
                // half wait only for the tensor-memory reads.
                uint32_t r[kChunks][32];
                __syncwarp();
#pragma unroll
                for (uint32_t c = 0; c < kChunks; ++c)
                    if (chunk0 + c < kHalfChunks)   // warp-uniform
                        tmem_ld_32cols(tmem_base + (lane_base << 16) + h * kTN + col_base + c * 32u,
                                       r[c]);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(h ? leader_empty1 : leader_empty0);
#pragma unroll
                for (uint32_t c = 0; c < kChunks; ++c) {
                    const uint32_t col = h * kTN + col_base + c * 32u;
                    const uint32_t n0 = nb * kTileW + col;
                    if (chunk0 + c >= kHalfChunks || n0 >= p.N || m_first >= p.M) continue;  // warp-uniform
                    dequant_chunk<kVar>(p.variant, r[c], sa, sreg[h * kChunks + c],
                                        breg[h * kChunks + c]);
                    const float(&v)[32] = reinterpret_cast<const float(&)[32]>(r[c]);
                    if (p.tma_store) {
                        if (lane == 0) bulk_wait_read0();  // previous store has read the buffer
                        __syncwarp();
#pragma unroll
                        for (uint32_t j = 0; j < 8u; ++j)
                            *reinterpret_cast<uint4 *>(my_row + 4u * (j ^ (lane & 7u))) =
                                make_uint4(r[c][4 * j], r[c][4 * j + 1], r[c][4 * j + 2],
                                           r[c][4 * j + 3]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmap_c, stage_out, static_cast<int32_t>(n0),
                                         static_cast<int32_t>(m_first));
                            bulk_commit();
                        }
                    } else if (row_ok) {
                        store_row32(v, crow, n0, p.N, vec_ok);
                    }
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
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kWTmemCols);
    }
}

}  // namespace

cudaError_t wide_device_setup(int &max_wide_pairs) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_wide_kernel<256>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kWSmemBytes))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_wide_kernel<224>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(wide_smem_bytes(224)))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_wide_kernel<256, kVarPlain>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kWSmemBytes))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(gemm_i8_tcgen05_pair_wide_kernel<224, kVarPlain>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(wide_smem_bytes(224)))) != cudaSuccess)
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kPThreads, 1, 1);
    cfg.dynamicSmemBytes = kWSmemBytes;
    int clusters = 0;
    if ((e = cudaOccupancyMaxActiveClusters(&clusters, gemm_i8_tcgen05_pair_wide_kernel<256>,
                                            &cfg)) != cudaSuccess)
        return e;
    max_wide_pairs = clusters;
    return cudaSuccess;
}

cudaError_t launch_wide_pair(cudaStream_t stream, uint32_t tn, uint32_t pairs,
                             const CUtensorMap &tmap_a, const CUtensorMap &tmap_b,
                             const CUtensorMap &tmap_c, const TcParams &tp) {
    const dim3 grid(2 * pairs), block(kPThreads);
    const bool plain = use_plain_variant(tp.variant);
    if (tn == 224u)
        return plain ? launch_pdl(stream, gemm_i8_tcgen05_pair_wide_kernel<224, kVarPlain>, grid,
                                  block, wide_smem_bytes(224), tmap_a, tmap_b, tmap_c, tp)
                     : launch_pdl(stream, gemm_i8_tcgen05_pair_wide_kernel<224>, grid, block,
                                  wide_smem_bytes(224), tmap_a, tmap_b, tmap_c, tp);
    return plain ? launch_pdl(stream, gemm_i8_tcgen05_pair_wide_kernel<256, kVarPlain>, grid, block,
                              kWSmemBytes, tmap_a, tmap_b, tmap_c, tp)
                 : launch_pdl(stream, gemm_i8_tcgen05_pair_wide_kernel<256>, grid, block,
                              kWSmemBytes, tmap_a, tmap_b, tmap_c, tp);
}

}  // namespace vnpu_b200
