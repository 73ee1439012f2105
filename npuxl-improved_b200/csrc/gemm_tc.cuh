// gemm_tc.cuh - what the tcgen05 GEMM translation units share: tile
// constants, the kernel parameter block, tile order and the dequant epilogue
// helpers.  gemm_i8.cu holds the single-CTA
// and 256x256 CTA-pair kernels and all host dispatch; gemm_i8_wide.cu the
// wide (256x512 / 256x448) CTA-pair kernel, compiled on its own.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "quant_common.cuh"

namespace vnpu_b200 {

struct TcParams {
    const float *scale_a = nullptr;
    const float *scale_b = nullptr;
    const float *bias = nullptr;
    float *C = nullptr;
    uint32_t ldc = 0;
    uint32_t M = 0, N = 0, K = 0;
    uint32_t tiles_m = 0, tiles_n = 0, num_kb = 0;
    uint32_t group_m = 1;  // raster band height in m-tiles
    uint32_t epilogue = 0, form = 0;
    uint32_t variant = 0;  // epi_variant(epilogue, bias != NULL, form)
    uint32_t tma_store = 0;  // 1: C written by TMA from shared memory
    uint32_t *err = nullptr;
    uint64_t limit_ns = 2000000000ull;
    // Scatter epilogue (ndst > 0): the tile goes to dst[0..ndst-1], each a
    // [M][ldd] matrix, at column col_off + n, by plain stores.
    float *dst[8] = {};
    uint32_t ndst = 0;
    uint32_t ldd = 0;
    uint32_t col_off = 0;
    // Split K (pair kernel): work unit u is tile u / splits, k-blocks
    // [s * kb_per_split, ...) of split s = u % splits; with splits > 1 the
    // epilogue stores the raw int32 sums to rows s * m_pad + m of the
    // workspace (C, ldc = N) and splitk_finish_kernel adds and dequantises.
    uint32_t splits = 1;
    uint32_t kb_per_split = 0;
    uint32_t m_pad = 0;
    // SwiGLU epilogue (pair kernel, kSwiglu): B is a [K][2I] gate/up weight
    // (N = 2I); CTA 0 of a pair loads gate rows n, CTA 1 up rows swiglu_i + n,
    // and C (I columns, row stride ldc) receives swiglu(gate, up) * alpha.
    uint32_t swiglu_i = 0;
    float swiglu_alpha = 1.0f;
};

namespace {

// ===========================================================================
// tcgen05 tensor-core GEMM
// ===========================================================================

constexpr uint32_t kBM = 128;                 // rows per tile (UMMA M)
constexpr uint32_t kBN = 256;                 // columns per tile (UMMA N)
constexpr uint32_t kBK = 128;                 // K bytes per stage (one 128B swizzle atom)
constexpr uint32_t kUmmaK = 32;               // K per tcgen05.mma kind::i8
constexpr uint32_t kStages = 4;
constexpr uint32_t kABytes = kBM * kBK;       // 16 KiB
constexpr uint32_t kBBytes = kBN * kBK;       // 32 KiB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 2 * kBN;       // two accumulators
constexpr uint32_t kThreads = 192;            // 6 warps
constexpr uint32_t kEpiWarps = 4;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack


__device__ __forceinline__ void tile_coords(uint32_t t, uint32_t tiles_m, uint32_t tiles_n,
                                            uint32_t group_m, uint32_t &mb, uint32_t &nb) {
    // Grouped raster: bands of group_m m-tiles walk all n-tiles, so a wave of
    // CTAs shares the band's A row-panels and a contiguous run of B panels in
    // L2; B is streamed from HBM once per band.
    const uint32_t per_band = group_m * tiles_n;
    const uint32_t band = t / per_band;
    const uint32_t first_m = band * group_m;
    const uint32_t rows = min(group_m, tiles_m - first_m);
    const uint32_t r = t - band * per_band;
    mb = first_m + r % rows;
    nb = r / rows;
}

// Store 32 finished values of one row (vec: 16-byte aligned row, ldc % 4 == 0).
__device__ __forceinline__ void store_row32(const float (&v)[32], float *crow, uint32_t n0,
                                            uint32_t N, bool vec) {
    if (vec && n0 + 32u <= N) {
#pragma unroll
        for (uint32_t j = 0; j < 32u; j += 4u)
            *reinterpret_cast<float4 *>(crow + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        return;
    }
#pragma unroll
    for (uint32_t j = 0; j < 32u; ++j)
        if (n0 + j < N) crow[n0 + j] = v[j];
}

// The 16 variants epi_variant() can produce.
#define VNPU_B200_EPI_VARIANTS(X)                                                             \
    X(0x10) X(0x11) X(0x12) X(0x13) X(0x14) X(0x15) X(0x16) X(0x17) X(0x18) X(0x19) X(0x1a) \
    X(0x1b) X(0x02) X(0x03) X(0x0a) X(0x0b)

// Dequant of 32 accumulators of one row whose column scales and biases sit one
// per lane (lane j holds column j's): the epilogue fetches them once per tile,
// before the accumulators are ready, instead of per chunk after.  All 32 lanes
// must execute it (warp shuffles).
template <uint32_t V>
__device__ __forceinline__ void dequant32_shfl(const uint32_t (&r)[32], float (&v)[32], float sa,
                                               float s_lane, float b_lane) {
    constexpr uint32_t ACT = V & 3u, BIAS = (V >> 2) & 3u;
    constexpr bool FUSED = ((V >> 4) & 1u) != 0u;
#pragma unroll
    for (uint32_t j = 0; j < 32u; ++j) {
        const float sb = __shfl_sync(0xffffffffu, s_lane, j);
        const float bb = BIAS != 0 ? __shfl_sync(0xffffffffu, b_lane, j) : 0.0f;
        v[j] = ref_dequant_t<ACT, BIAS, FUSED>(static_cast<int32_t>(r[j]), sa, sb, bb);
    }
}

template <uint32_t V>
__device__ __forceinline__ void dequant32_shfl_inplace(uint32_t (&r)[32], float sa, float s_lane,
                                                       float b_lane) {
    constexpr uint32_t ACT = V & 3u, BIAS = (V >> 2) & 3u;
    constexpr bool FUSED = ((V >> 4) & 1u) != 0u;
#pragma unroll
    for (uint32_t j = 0; j < 32u; ++j) {
        const float sb = __shfl_sync(0xffffffffu, s_lane, j);
        const float bb = BIAS != 0 ? __shfl_sync(0xffffffffu, b_lane, j) : 0.0f;
        r[j] = __float_as_uint(ref_dequant_t<ACT, BIAS, FUSED>(static_cast<int32_t>(r[j]), sa, sb, bb));
    }
}

// One launch-constant form per tcgen05 GEMM launch: a command whose elements
// take more than one form (FormMap kFormMixed) never reaches these kernels'
// epilogues (matmul_i8_tcgen05 routes it to raw split-K sums and the finish
// kernel, or to the SIMT kernel).
__device__ __forceinline__ void dequant32_shfl_any(uint32_t variant, const uint32_t (&r)[32],
                                                   float (&v)[32], float sa, float s_lane,
                                                   float b_lane) {
    switch (variant) {
#define VNPU_B200_CASE(V)                                      \
    case V:                                                    \
        dequant32_shfl<V>(r, v, sa, s_lane, b_lane);           \
        break;
        VNPU_B200_EPI_VARIANTS(VNPU_B200_CASE)
#undef VNPU_B200_CASE
    default:
        break;
    }
}

__device__ __forceinline__ void dequant32_shfl_inplace_any(uint32_t variant, uint32_t (&r)[32],
                                                           float sa, float s_lane, float b_lane) {
    switch (variant) {
#define VNPU_B200_CASE(V)                                      \
    case V:                                                    \
        dequant32_shfl_inplace<V>(r, sa, s_lane, b_lane);      \
        break;
        VNPU_B200_EPI_VARIANTS(VNPU_B200_CASE)
#undef VNPU_B200_CASE
    default:
        break;
    }
}

// The dequant epilogue variant fixed at compile time (kVar), or chosen per
// launch through the switch above (kVar == kVarRuntime).  The fixed form has
// no indirect branch and a shorter instruction stream: at 512^3, where a
// launch is mostly fixed cost, the runtime switch's launch stalled mostly on
// instruction fetch (no_instruction 11.2 cycles per issued instruction).
constexpr uint32_t kVarRuntime = 0xFFFFFFFFu;
constexpr uint32_t kVarPlain = epi_variant(0, false, 0);   // NONE, no bias: every form alike

// SiLU without bias in the block or stream form (the FFN GEMM of the
// BASELINE's config 3) on the 16-epilogue-warp pair kernel.
constexpr uint32_t kVarSilu = epi_variant(2, false, 0);

// The launch takes the instance with `variant` compiled in
// (VNPU_B200_EPI_RUNTIME=1 keeps the runtime-switch instance, for
// comparisons).
inline bool use_compiled_variant(uint32_t variant, uint32_t compiled) {
    static const bool forced_runtime = std::getenv("VNPU_B200_EPI_RUNTIME") != nullptr;
    return variant == compiled && !forced_runtime;
}
inline bool use_plain_variant(uint32_t variant) { return use_compiled_variant(variant, kVarPlain); }

template <uint32_t kVar>
__device__ __forceinline__ void dequant_chunk(uint32_t variant, uint32_t (&r)[32], float sa,
                                              float s_lane, float b_lane) {
    if constexpr (kVar == kVarRuntime)
        dequant32_shfl_inplace_any(variant, r, sa, s_lane, b_lane);
    else
        dequant32_shfl_inplace<kVar>(r, sa, s_lane, b_lane);
}

// Column scale and bias of column n for the lane that holds it (n past N: 1, 0).
__device__ __forceinline__ void fetch_col(const TcParams &p, uint32_t n, float &s, float &b) {
    s = n < p.N ? __ldg(p.scale_b + n) : 1.0f;
    b = (p.bias && n < p.N) ? __ldg(p.bias + n) : 0.0f;
}

constexpr uint32_t kPStages = 6;                  // stage count of the wide kernel's sibling (8 warps)
constexpr uint32_t kPTileM = 256;                 // per pair
constexpr uint32_t kPTileN = 256;                 // per pair
constexpr uint32_t kPABytes = 128 * kBK;          // 16 KiB per CTA
constexpr uint32_t kPBBytes = 128 * kBK;          // 16 KiB per CTA
constexpr uint32_t kPStageBytes = kPABytes + kPBBytes;
constexpr uint32_t kPEpiWarps = 8;                // per CTA (wide kernel)
constexpr uint32_t kPThreads = (2 + kPEpiWarps) * 32;
// The 256x256 pair kernel comes in two shapes: 8 epilogue warps and 6 stages
// for NONE / RELU (the MMA issuer keeps its sub-partition), and 16 epilogue
// warps and 5 stages for SiLU / GELU, whose dequant epilogue (polynomial exp,
// IEEE divisions) is latency-bound: four warps per sub-partition hide it
// behind the next tile's MMAs.
// The tile width kTN (columns per pair: 256, or 224 where 224-column tiles
// divide the shard into fuller waves, e.g. 3584 = 16 x 224 on 74 pairs) sets
// each CTA's half of the B tile: kTN / 2 rows of 128 K bytes.
constexpr uint32_t pair_threads(uint32_t epi_warps) { return (2 + epi_warps) * 32; }
constexpr uint32_t pair_stage_bytes(uint32_t tn) { return 128 * kBK + (tn / 2) * kBK; }
constexpr uint32_t pair_smem_bytes(uint32_t epi_warps, uint32_t stages, uint32_t tn = 256) {
    return stages * pair_stage_bytes(tn) + epi_warps * 32 * 32 * 4 + 1024;
}
constexpr uint32_t kPStageOutBytes = 32 * 32 * 4;  // one 32 rows x 32 floats staging buffer
// Ring depth of the narrow pair tiles (8 epilogue warps): as many 24 / 20 KiB
// stages as fit beside the epilogue's staging buffers.  Where few tiles run at
// once the main loop is bound by the copies in flight per SM (256x256 and
// 256x128 tiles with 6 stages both took ~0.4 us per 128-deep k-block at
// 512x4096x4096), so the deeper ring is the narrow tile's speed.
constexpr uint32_t kNarrowStages128 = 8;
constexpr uint32_t kNarrowStages64 = 9;


// ===========================================================================
// Wide tcgen05 pair GEMM: a CTA pair computes a 256x512 output tile as two
// 256x256 accumulators (TMEM columns 0-255 and 256-511 of each CTA: all 512).
// Per 128-deep K step each SM loads 16 KiB of A and 2 x 16 KiB of B for
// 128x512 outputs: a quarter fewer operand bytes per MAC than the 256x256
// pair tile, whose rate is bounded by how fast TMA delivers tiles from L2.
// With both halves of tensor memory in use there is no second accumulator
// set, so the epilogue drains D0 then D1 and releases each half as soon as it
// is read; at the start of a tile the MMA issuer runs D0's MMAs over every
// k-block already staged (holding those stages) while D1 is still being
// drained, then issues D1's MMAs on the held stages and releases them.
//   barriers: full[s] (leader) counts both CTAs' bytes; empty[s] (both) is
//             arrived by the leader's multicast commit; tmem_full (both);
//             tmem_empty[h] (leader) gets 16 arrivals, one per epilogue warp
//             of the pair, when half h has been read.
// No TMA multicast: each CTA loads only its own tiles.
// ===========================================================================

// kTN is the width of each accumulator (256, or 224 for 448-column tiles
// where those fill the waves better); the tile is 256 x 2kTN.
constexpr uint32_t kWStages = 4;
constexpr uint32_t kWTileN = 512;                          // per pair (kTN = 256)
constexpr uint32_t wide_stage_bytes(uint32_t tn) { return kPABytes + 2u * (tn / 2u) * kBK; }
constexpr uint32_t wide_smem_bytes(uint32_t tn) {
    return kWStages * wide_stage_bytes(tn) + kPEpiWarps * kPStageOutBytes + 1024;
}
constexpr uint32_t kWSmemBytes = wide_smem_bytes(256);     // 48 KiB stages
constexpr uint32_t kWTmemCols = 512;
static_assert(kWSmemBytes <= 227u * 1024u, "wide pair tile exceeds shared memory");

}  // namespace

// Shared-memory opt-in for every wide-kernel instance and the number of
// co-resident CTA pairs of the 256x512 tile.
cudaError_t wide_device_setup(int &max_wide_pairs);

// One launch of the wide CTA-pair kernel (programmatic dependent launch):
// accumulator width tn (256 or 224), 2 * pairs CTAs.
// tp.variant == kVarPlain takes the instance with that variant compiled in.
cudaError_t launch_wide_pair(cudaStream_t stream, uint32_t tn, uint32_t pairs,
                             const CUtensorMap &tmap_a, const CUtensorMap &tmap_b,
                             const CUtensorMap &tmap_c, const TcParams &tp);

}  // namespace vnpu_b200
