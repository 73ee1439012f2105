// common.cuh - device helpers shared by the sm_100a kernels.
//
// * the reference's float arithmetic, restated with explicit rounding
//   intrinsics so nvcc's contraction never changes a result: every fused
//   multiply-add is a __fmaf_rn that mirrors a fusion GCC performs in the
//   reference's AVX2 kernels, every other product/sum is __fmul_rn/__fadd_rn;
// * inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor), and the
//   5th-generation tensor core (tcgen05 alloc/mma/commit/ld);
// * bounded waits: every spin on an mbarrier gives up after a wall-clock
//   limit, records an error code in the stream's device error word, and lets
//   the kernel wind down instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <utility>
#include <cuda_runtime.h>

#include "kernels.h"

namespace vnpu_b200 {

// DeviceError and EpiForm come from kernels.h.

// ---------------------------------------------------------------------------
// Reference arithmetic (src/internal.h:87-136, src/kernels/kernels.cpp:526-535)
// ---------------------------------------------------------------------------

// 2^f on [0,1): the reference's degree-5 polynomial (internal.h:97-101).
__device__ __forceinline__ float exp2_poly(float f, bool fused) {
    const float c1 = 0.6931471805599453f, c2 = 0.2402265069591007f,
                c3 = 0.05550410866482158f, c4 = 0.009618129107628477f,
                c5 = 0.0013333558146428443f;
    if (fused) {
        float p = __fmaf_rn(f, c5, c4);
        p = __fmaf_rn(f, p, c3);
        p = __fmaf_rn(f, p, c2);
        p = __fmaf_rn(f, p, c1);
        return __fmaf_rn(f, p, 1.0f);
    }
    float p = __fadd_rn(c4, __fmul_rn(f, c5));
    p = __fadd_rn(c3, __fmul_rn(f, p));
    p = __fadd_rn(c2, __fmul_rn(f, p));
    p = __fadd_rn(c1, __fmul_rn(f, p));
    return __fadd_rn(1.0f, __fmul_rn(f, p));
}

// fast_expf (internal.h:87-108): cut-offs at +-80, z = x*log2e, split into
// floor and fraction, polynomial, exact scaling by 2^floor.
// p * 2^n for n in [-126, 127] and p in [1, 2): one exact multiply (the
// power of two is a normal float, the product neither overflows nor goes
// subnormal), the same value ldexp gives.
__device__ __forceinline__ float scale_pow2(float p, int n) {
    return __fmul_rn(p, __int_as_float((n + 127) << 23));
}

__device__ __forceinline__ float ref_fast_expf(float x, bool fused) {
    if (x < -80.0f) return 0.0f;
    if (x > 80.0f) return __int_as_float(0x7f800000);
    const float z = __fmul_rn(x, 1.4426950408889634f);
    const float zi = floorf(z);  // in [-116, 115] here
    const float f = __fsub_rn(z, zi);
    return scale_pow2(exp2_poly(f, fused), __float2int_rz(zi));
}

// exp256_ps (src/kernels/llm.cpp:32-56): clamps to [-80,80] instead; for the
// clamped range 2^n built from exponent bits equals ldexpf exactly.
__device__ __forceinline__ float ref_exp256_lane(float x) {
    x = fmaxf(-80.0f, fminf(x, 80.0f));
    const float z = __fmul_rn(x, 1.4426950408889634f);
    const float zi = floorf(z);
    const float f = __fsub_rn(z, zi);
    return scale_pow2(exp2_poly(f, true), __float2int_rz(zi));
}

__device__ __forceinline__ float ref_silu(float x, bool fused) {
    return __fdiv_rn(x, __fadd_rn(1.0f, ref_fast_expf(-x, fused)));
}

__device__ __forceinline__ float ref_gelu_tanh(float x, bool fused) {
    const float k0 = 0.7978845608028654f, k1 = 0.035677408136300125f;
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = fused ? __fmul_rn(k0, __fmaf_rn(k1, x3, x))
                              : __fmul_rn(k0, __fadd_rn(x, __fmul_rn(k1, x3)));
    const float e = ref_fast_expf(__fmul_rn(-2.0f, inner), fused);
    const float t = __fsub_rn(__fdiv_rn(2.0f, __fadd_rn(1.0f, e)), 1.0f);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

__device__ __forceinline__ float ref_activation(float v, uint32_t epilogue, bool fused) {
    switch (epilogue) {
    case 1: return v > 0.0f ? v : 0.0f;
    case 2: return ref_silu(v, fused);
    case 3:
    case 4: return ref_gelu_tanh(v, fused);
    default: return v;
    }
}

// ---- branch-free variants, selected once per launch ------------------------
// Same arithmetic as above; out-of-range and NaN inputs handled with selects
// so a warp can interleave independent elements.  fast_expf: NaN propagates
// (as in the reference: z, floor and the polynomial all become NaN).
template <bool FUSED>
__device__ __forceinline__ float ref_fast_expf_sel(float x) {
    const float xc = x < -80.0f ? -80.0f : (x > 80.0f ? 80.0f : x);
    const float z = __fmul_rn(xc, 1.4426950408889634f);
    const float zi = floorf(z);
    const float f = __fsub_rn(z, zi);
    const int n = __float2int_rz(zi);
    const float r = scale_pow2(exp2_poly(f, FUSED), n);
    return x < -80.0f ? 0.0f : (x > 80.0f ? __int_as_float(0x7f800000) : r);
}

// Activation variants: 0 none, 1 relu, 2 silu, 3 gelu (tanh; GELU_ERF aliases it).
template <uint32_t ACT, bool FUSED>
__device__ __forceinline__ float ref_activation_t(float v) {
    if constexpr (ACT == 1) {
        return v > 0.0f ? v : 0.0f;
    } else if constexpr (ACT == 2) {
        return __fdiv_rn(v, __fadd_rn(1.0f, ref_fast_expf_sel<FUSED>(-v)));
    } else if constexpr (ACT == 3) {
        const float k0 = 0.7978845608028654f, k1 = 0.035677408136300125f;
        const float x3 = __fmul_rn(__fmul_rn(v, v), v);
        const float inner = FUSED ? __fmul_rn(k0, __fmaf_rn(k1, x3, v))
                                  : __fmul_rn(k0, __fadd_rn(v, __fmul_rn(k1, x3)));
        const float e = ref_fast_expf_sel<FUSED>(__fmul_rn(-2.0f, inner));
        const float t = __fsub_rn(__fdiv_rn(2.0f, __fadd_rn(1.0f, e)), 1.0f);
        return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, t));
    } else {
        return v;
    }
}

// BIAS: 0 none, 1 fused (fmaf), 2 two roundings.
template <uint32_t ACT, uint32_t BIAS, bool FUSED>
__device__ __forceinline__ float ref_dequant_t(int32_t acc, float sa, float sb, float bias) {
    const float t = __fmul_rn(__int2float_rn(acc), sa);
    float out;
    if constexpr (BIAS == 0) out = __fmul_rn(t, sb);
    else if constexpr (BIAS == 1) out = __fmaf_rn(t, sb, bias);
    else out = __fadd_rn(__fmul_rn(t, sb), bias);
    return ref_activation_t<ACT, FUSED>(out);
}

// Launch-constant epilogue variant: act | bias << 2 | fused << 4, or
// kVariantMixed when the form varies by element (FormMap, form_at).
constexpr uint32_t kVariantMixed = 0x40u;
__host__ __device__ constexpr uint32_t epi_variant(uint32_t epilogue, bool has_bias,
                                                   uint32_t form) {
    if (form == kFormMixed) return kVariantMixed;
    const uint32_t act = epilogue == 1 ? 1u : epilogue == 2 ? 2u : (epilogue == 3 || epilogue == 4) ? 3u : 0u;
    const uint32_t bias = !has_bias ? 0u : (form == kFormBlock ? 1u : 2u);
    const uint32_t fused = (act >= 2 && form == kFormScalar) ? 0u : 1u;
    return act | (bias << 2) | (fused << 4);
}

// store_i8_c (kernels.cpp:526-535) for one accumulator.
__device__ __forceinline__ float ref_dequant(int32_t acc, float sa, float sb, bool has_bias,
                                             float bias, uint32_t epilogue, uint32_t form) {
    const float t = __fmul_rn(__int2float_rn(acc), sa);
    float out;
    if (!has_bias) {
        out = __fmul_rn(t, sb);
    } else if (form == kFormBlock) {
        out = __fmaf_rn(t, sb, bias);
    } else {
        out = __fadd_rn(__fmul_rn(t, sb), bias);
    }
    return ref_activation(out, epilogue, form != kFormScalar);
}

// The form of element (m, n) of a launch (n the launch's own column; fm.col_base
// places it in the whole output whose reference tile grid fm describes).  m is
// below fm.M for every element that is stored.
__device__ __forceinline__ uint32_t form_at(const FormMap &fm, uint32_t m, uint32_t n) {
    if (fm.form != kFormMixed) return fm.form;
    const uint32_t m0 = m / fm.tm * fm.tm;
    const uint32_t left = fm.M - m0;                       // rows from the tile start on
    const uint32_t rows = left < fm.tm ? left : fm.tm;
    const uint32_t rc = (left <= fm.tm ? 2u : 0u) |
                        (((rows & 1u) != 0u && m - m0 == rows - 1u) ? 1u : 0u);
    const uint32_t c = n + fm.col_base;
    const uint32_t n0 = c / fm.tn * fm.tn;
    const uint32_t cleft = fm.N - n0;
    const uint32_t cols = cleft < fm.tn ? cleft : fm.tn;
    const uint32_t cc = (cleft <= fm.tn ? 2u : 0u) | (c - n0 >= (cols & ~31u) ? 1u : 0u);
    return (fm.table >> (2u * (rc * 4u + cc))) & 3u;
}

// ---------------------------------------------------------------------------
// Time and errors
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(uint32_t *err, uint32_t code) {
    if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------------------
// Shared memory, mbarriers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete.  Gives up when the
// wall-clock deadline passes (or when another thread of the CTA has already
// given up, *abort != 0): records kErrWaitTimeout and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                          uint32_t *err, volatile int *abort) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait(a, parity)) return true;
        if ((spin & 63u) == 0) {
            if (abort && *abort) return false;
            if (global_timer_ns() - start > limit_ns) {
                record_error(err, kErrWaitTimeout);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled load into this CTA's shared memory, completing on `bar`.
// x is the innermost (contiguous) coordinate in elements; the caller keeps
// x * elem_bytes a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, uint64_t *bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// 2-D tiled store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *smem_src, int32_t x,
                                             int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tmap)),
        "r"(smem_addr(smem_src)), "r"(x), "r"(y)
        : "memory");
}
// One contiguous global -> shared copy by the TMA unit (no tensor map, no
// multicast): both addresses 16-byte aligned, bytes a multiple of 16; the
// bytes complete on `bar` (expect them with mbar_arrive_expect_tx).
__device__ __forceinline__ void bulk_load_1d(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                             uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Shared-memory sources of committed bulk stores may be reused.
__device__ __forceinline__ void bulk_wait_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// At most one committed bulk store may still be reading shared memory.
__device__ __forceinline__ void bulk_wait_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, tensor memory)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], int8 x int8 -> int32.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_8cols(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row swizzle atoms 1024 bytes
// apart (SBO), leading offset unused for this layout (encoded 1), version 1,
// layout type 2 = SWIZZLE_128B.  The tile base must be 1024-byte aligned;
// stepping K inside the atom adds the byte offset to the start address.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for kind::i8: D s32, A s8, B s8, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_i8(uint32_t m, uint32_t n) {
    return (2u << 4)            // D format: s32
           | (1u << 7)          // A format: signed 8-bit
           | (1u << 10)         // B format: signed 8-bit
           | ((n >> 3) << 17)   // N / 8
           | ((m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------------------
// Clusters and cta_group::2 (a pair of CTAs on two SMs sharing one MMA)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// 32-bit load from another CTA's shared memory (distributed shared memory).
// 16-byte global -> shared copy that does not block the issuing thread
// (completion by cp_async_wait_all).
__device__ __forceinline__ void cp_async_16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// The same copy with zero fill: `valid` false writes 16 zero bytes and reads
// nothing (gmem_src must still be a mapped address).
__device__ __forceinline__ void cp_async_16_zfill(void *smem_dst, const void *gmem_src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src), "r"(valid ? 16u : 0u)
                 : "memory");
}
// sm_100 two-lane FMA: d.lo = fma(a.lo, b.lo, c.lo), d.hi = fma(a.hi, b.hi,
// c.hi), each rounded once like fmaf.  Half the issue slots of two FFMAs.
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float half_f32x2(uint64_t v, int hi) {
    float lo_v, hi_v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo_v), "=f"(hi_v) : "l"(v));
    return hi ? hi_v : lo_v;
}
__device__ __forceinline__ uint64_t swap_f32x2(uint64_t v) {
    return pack_f32x2(half_f32x2(v, 1), half_f32x2(v, 0));
}

// 4-byte form (any 4-aligned addresses, e.g. to transpose while copying).
__device__ __forceinline__ void cp_async_4_zfill(void *smem_dst, const void *gmem_src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src), "r"(valid ? 4u : 0u)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void st_shared_cluster_f32(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}

__device__ __forceinline__ int32_t ld_shared_cluster_s32(uint32_t cluster_addr) {
    int32_t v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
    return v;
}

__device__ __forceinline__ void st_shared_cluster_v4(uint32_t cluster_addr, int32_t a, int32_t b,
                                                     int32_t c, int32_t d) {
    asm volatile("st.shared::cluster.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a),
                 "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel has completed and its memory
// is visible.  Both are no-ops for launches without the PDL attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_previous() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Programmatic dependent launch at kernel entry: let the stream's next kernel
// be scheduled now (its CTAs then wait in their own pdl_enter), and wait
// until the previous kernel has finished and its writes are visible.  Both
// are no-ops for a kernel launched without the PDL attribute.
__device__ __forceinline__ void pdl_enter() {
    pdl_launch_dependents();
    pdl_wait_previous();
}

// Host: launch a kernel that begins with pdl_enter() with programmatic
// dependent launch allowed (VNPU_B200_NO_PDL turns it off), so a chain of
// short dependent kernels hides its launch latency.
inline bool pdl_allowed() {
    static const bool allowed = std::getenv("VNPU_B200_NO_PDL") == nullptr;
    return allowed;
}
#define VNPU_LAUNCH(expr)                                  \
    do {                                                   \
        const cudaError_t vnpu_launch_rc_ = (expr);        \
        if (vnpu_launch_rc_ != cudaSuccess) return vnpu_launch_rc_; \
    } while (0)
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(cudaStream_t stream, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                              size_t smem, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_allowed() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Arrive on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

// All threads of all CTAs of the cluster.  Only used where every thread of
// the pair is guaranteed to arrive (kernel start, and the end after every
// bounded wait has returned).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on the leader CTA's mbarrier (cluster address), for cta_group::2 MMAs.
// No multicast: each CTA loads its own tile.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap,
                                                 uint32_t leader_bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Pair MMA: issued by the leader CTA only; A rows and B columns come half
// from each CTA's shared memory at the same offsets; each CTA's tensor memory
// receives its 128 rows of D.
__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` in every CTA of `cta_mask` when the pair MMAs issued so far
// complete.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_addr(bar)),
        "h"(cta_mask)
        : "memory");
}

}  // namespace vnpu_b200
