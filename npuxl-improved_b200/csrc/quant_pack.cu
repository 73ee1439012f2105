// quant_pack.cu - QUANTIZE_I8 and PACK_WEIGHTS_I8 on sm_100a.
//
// QUANTIZE_I8 restates src/kernels/llm.cpp:387-436 bit for bit:
//   scale = maxabs/127 (IEEE divide; 1.0 when <= 0 or not finite),
//   inv = 1/scale (IEEE divide), q = roundf(x*inv) (half away from zero, as
//   std::round), clamp to [-128, 127].  NaN elements never win the max, as
//   with std::max(maxabs, |x|).
// All of it is HBM-bound byte work: rows are read once (kept in registers
// when they fit), written once.
#include <cstdio>
#include <mutex>

#include "../../include/vnpu_b200.h"
#include "common.cuh"
#include "kernels.h"
#include "quant_common.cuh"

namespace vnpu_b200 {
namespace {

constexpr int kQThreads = 256;
// float4 per thread kept in registers: 8 (rows <= 8192, more CTAs per SM)
// or 12 (rows <= 12288, e.g. the decoder block's 11008-wide SwiGLU output,
// which would otherwise be read twice).
constexpr int kQRegVecNarrow = 8;
constexpr int kQRegVecWide = 12;

// One CTA per row; vector path: cols % 4 == 0 and 16-byte aligned rows.
template <bool kVec, int kQRegVec = kQRegVecNarrow>
__global__ void __launch_bounds__(kQThreads) quantize_rows_kernel(const float *__restrict__ X,
                                                                  int8_t *__restrict__ Y,
                                                                  float *__restrict__ scales,
                                                                  uint64_t cols) {
    pdl_enter();
    __shared__ float red[32];
    const uint64_t r = blockIdx.x;
    const float *x = X + r * cols;
    int8_t *y = Y + r * cols;
    float m = 0.0f;
    if (kVec) {
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        const uint64_t n4 = cols >> 2;
        if (n4 <= static_cast<uint64_t>(kQThreads) * kQRegVec) {
            float4 v[kQRegVec];
#pragma unroll
            for (int i = 0; i < kQRegVec; ++i) {
                const uint64_t j = threadIdx.x + static_cast<uint64_t>(i) * kQThreads;
                v[i] = j < n4 ? __ldg(x4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)),
                                   fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            }
            const float scale = scale_from_absmax(block_max(m, red));
            const float inv = __fdiv_rn(1.0f, scale);
            if (threadIdx.x == 0) scales[r] = scale;
            uint32_t *y4 = reinterpret_cast<uint32_t *>(y);
#pragma unroll
            for (int i = 0; i < kQRegVec; ++i) {
                const uint64_t j = threadIdx.x + static_cast<uint64_t>(i) * kQThreads;
                if (j < n4) y4[j] = pack4(v[i].x, v[i].y, v[i].z, v[i].w, inv);
            }
            return;
        }
        for (uint64_t j = threadIdx.x; j < n4; j += kQThreads) {
            const float4 v = __ldg(x4 + j);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        const float scale = scale_from_absmax(block_max(m, red));
        const float inv = __fdiv_rn(1.0f, scale);
        if (threadIdx.x == 0) scales[r] = scale;
        uint32_t *y4 = reinterpret_cast<uint32_t *>(y);
        for (uint64_t j = threadIdx.x; j < n4; j += kQThreads) {
            const float4 v = __ldg(x4 + j);
            y4[j] = pack4(v.x, v.y, v.z, v.w, inv);
        }
        return;
    }
    for (uint64_t j = threadIdx.x; j < cols; j += kQThreads) m = fmaxf(m, fabsf(x[j]));
    const float scale = scale_from_absmax(block_max(m, red));
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scales[r] = scale;
    for (uint64_t j = threadIdx.x; j < cols; j += kQThreads) y[j] = quantize_value(x[j], inv);
}

// Per-column absmax: CTA = 32 columns x all rows; 8 warps stride the rows.
__global__ void __launch_bounds__(256) column_absmax_kernel(const float *__restrict__ X,
                                                            float *__restrict__ scales,
                                                            uint64_t rows, uint64_t cols) {
    __shared__ float part[8][33];
    const uint64_t c = static_cast<uint64_t>(blockIdx.x) * 32 + (threadIdx.x & 31);
    const int w = threadIdx.x >> 5;
    float m = 0.0f;
    if (c < cols)
        for (uint64_t r = w; r < rows; r += 8) m = fmaxf(m, fabsf(X[r * cols + c]));
    part[w][threadIdx.x & 31] = m;
    __syncthreads();
    if (w == 0) {
        float v = part[0][threadIdx.x];
#pragma unroll
        for (int i = 1; i < 8; ++i) v = fmaxf(v, part[i][threadIdx.x]);
        if (c < cols) scales[c] = scale_from_absmax(v);
    }
}

__global__ void quantize_by_column_kernel(const float *__restrict__ X, int8_t *__restrict__ Y,
                                          const float *__restrict__ scales, uint64_t rows,
                                          uint64_t cols) {
    const uint64_t total = rows * cols;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t c = i % cols;
        Y[i] = quantize_value(X[i], __fdiv_rn(1.0f, scales[c]));
    }
}

__global__ void tensor_absmax_kernel(const float *__restrict__ X, uint64_t n,
                                     uint32_t *__restrict__ out_bits) {
    __shared__ float red[32];
    float m = 0.0f;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        m = fmaxf(m, fabsf(X[i]));
    m = block_max(m, red);
    // absmax >= 0 (or +inf): its IEEE bits order like unsigned integers.
    if (threadIdx.x == 0) atomicMax(out_bits, __float_as_uint(m));
}

__global__ void quantize_tensor_kernel(const float *__restrict__ X, int8_t *__restrict__ Y,
                                       float *__restrict__ scales, uint64_t n,
                                       const uint32_t *__restrict__ absmax_bits) {
    const float scale = scale_from_absmax(__uint_as_float(*absmax_bits));
    // src/kernels/llm.cpp:432: inv = 1/(scales[0] > 0 ? scales[0] : 1).
    const float inv = __fdiv_rn(1.0f, scale > 0.0f ? scale : 1.0f);
    if (blockIdx.x == 0 && threadIdx.x == 0) scales[0] = scale;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        Y[i] = quantize_value(X[i], inv);
}

// ---------------------------------------------------------------------------
// PACK_WEIGHTS_I8: B (K x N, ldb) -> Bt[N][k_stride], zero padded in K, plus
// int32 column sums (src/core/scheduler.cpp:783-805).  64 x 64 byte tiles
// through shared memory; column sums accumulate with integer atomics (exact,
// order-free).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pack_transpose_kernel(const int8_t *__restrict__ B,
                                                             uint32_t K, uint32_t N,
                                                             uint32_t ldb,
                                                             int8_t *__restrict__ Bt,
                                                             uint32_t k_stride,
                                                             int32_t *__restrict__ colsum) {
    __shared__ int8_t tile[64][65];
    __shared__ int32_t sums[64];
    const uint32_t k0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
    if (threadIdx.x < 64) sums[threadIdx.x] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
        const uint32_t kk = i / 64, nn = i % 64;
        const uint32_t k = k0 + kk, n = n0 + nn;
        int8_t v = 0;
        if (k < K && n < N) v = B[static_cast<uint64_t>(k) * ldb + n];
        tile[kk][nn] = v;
        if (v) atomicAdd(&sums[nn], static_cast<int32_t>(v));
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
        const uint32_t nn = i / 64, kk = i % 64;
        const uint32_t k = k0 + kk, n = n0 + nn;
        if (n < N && k < k_stride) Bt[static_cast<uint64_t>(n) * k_stride + k] = tile[kk][nn];
    }
    if (threadIdx.x < 64 && n0 + threadIdx.x < N && sums[threadIdx.x])
        atomicAdd(&colsum[n0 + threadIdx.x], sums[threadIdx.x]);
}

// trans_b = 1: B is N x K (ldb); rows copy straight into the padded layout.
__global__ void pack_rows_kernel(const int8_t *__restrict__ B, uint32_t K, uint32_t N,
                                 uint32_t ldb, int8_t *__restrict__ Bt, uint32_t k_stride,
                                 int32_t *__restrict__ colsum) {
    __shared__ int32_t red[32];
    const uint32_t n = blockIdx.x;
    int32_t s = 0;
    for (uint32_t k = threadIdx.x; k < k_stride; k += blockDim.x) {
        const int8_t v = k < K ? B[static_cast<uint64_t>(n) * ldb + k] : 0;
        Bt[static_cast<uint64_t>(n) * k_stride + k] = v;
        s += v;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t t = 0;
        for (uint32_t w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
        colsum[n] = t;
    }
}

inline void count_launch(const LaunchCtx &ctx, uint64_t n = 1) {
    if (ctx.launch_counter) *ctx.launch_counter += n;
}

}  // namespace

cudaError_t quantize_rows(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                          uint64_t rows, uint64_t cols) {
    if (rows > 0x7fffffffull) return cudaErrorInvalidValue;
    const bool vec = (cols % 4 == 0) && (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(Y) % 4 == 0);
    if (vec && cols > static_cast<uint64_t>(kQThreads) * 4 * kQRegVecNarrow &&
        cols <= static_cast<uint64_t>(kQThreads) * 4 * kQRegVecWide)
        VNPU_LAUNCH(launch_pdl(ctx.stream, quantize_rows_kernel<true, kQRegVecWide>,
                               dim3(static_cast<unsigned>(rows)), dim3(kQThreads), 0, X, Y, scales,
                               cols));
    else if (vec)
        VNPU_LAUNCH(launch_pdl(ctx.stream, quantize_rows_kernel<true>, dim3(static_cast<unsigned>(rows)), dim3(kQThreads), 0, 
            X, Y, scales, cols));
    else
        VNPU_LAUNCH(launch_pdl(ctx.stream, quantize_rows_kernel<false>, dim3(static_cast<unsigned>(rows)), dim3(kQThreads), 0, 
            X, Y, scales, cols));
    count_launch(ctx);
    return cudaGetLastError();
}

cudaError_t quantize_columns(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                             uint64_t rows, uint64_t cols) {
    const uint64_t blocks = (cols + 31) / 32;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidValue;
    column_absmax_kernel<<<static_cast<unsigned>(blocks), 256, 0, ctx.stream>>>(X, scales, rows,
                                                                                cols);
    const unsigned grid = static_cast<unsigned>(ctx.num_sms) * 8;
    quantize_by_column_kernel<<<grid, 256, 0, ctx.stream>>>(X, Y, scales, rows, cols);
    count_launch(ctx, 2);
    return cudaGetLastError();
}

cudaError_t quantize_tensor(const LaunchCtx &ctx, const float *X, int8_t *Y, float *scales,
                            uint64_t rows, uint64_t cols, uint32_t *absmax_scratch) {
    const uint64_t n = rows * cols;
    cudaError_t e = cudaMemsetAsync(absmax_scratch, 0, sizeof(uint32_t), ctx.stream);
    if (e != cudaSuccess) return e;
    const unsigned grid = static_cast<unsigned>(ctx.num_sms) * 8;
    tensor_absmax_kernel<<<grid, 256, 0, ctx.stream>>>(X, n, absmax_scratch);
    quantize_tensor_kernel<<<grid, 256, 0, ctx.stream>>>(X, Y, scales, n, absmax_scratch);
    count_launch(ctx, 2);
    return cudaGetLastError();
}

cudaError_t pack_weights(const LaunchCtx &ctx, const int8_t *B, uint32_t K, uint32_t N,
                         uint32_t ldb, uint32_t trans_b, int8_t *Bt, uint32_t k_stride,
                         int32_t *column_sums) {
    if (trans_b) {
        pack_rows_kernel<<<N, 256, 0, ctx.stream>>>(B, K, N, ldb, Bt, k_stride, column_sums);
        count_launch(ctx);
        return cudaGetLastError();
    }
    cudaError_t e = cudaMemsetAsync(column_sums, 0, sizeof(int32_t) * N, ctx.stream);
    if (e != cudaSuccess) return e;
    dim3 grid((k_stride + 63) / 64, (N + 63) / 64);
    pack_transpose_kernel<<<grid, 256, 0, ctx.stream>>>(B, K, N, ldb, Bt, k_stride,
                                                        column_sums);
    count_launch(ctx);
    return cudaGetLastError();
}

}  // namespace vnpu_b200

// ---------------------------------------------------------------------------
// Per-tensor QUANTIZE_I8 that allocates nothing (vnpu_b200_quantize_i8_tensor_noalloc).
//
// Same bits as quantize_tensor(): the tensor's absmax is an order-free max.
// Its scratch is one file-scope device array per device instead of the vnpu
// stream's scratch word:
//   words [0, kNoAllocMaxChunks)  one partial absmax per CTA of pass 1 (each
//                                 is written before it is read: no clearing)
//   word  kNoAllocCounter         CTAs of pass 1 that have finished; must be
//                                 zero when a call starts.  Zeroed when the
//                                 address is first looked up, and the last CTA
//                                 of every call puts it back to zero.
//   word  kNoAllocResult          the tensor absmax (IEEE bits), pass 2 reads it
// Pass 1 gives each CTA a fixed chunk of kNoAllocChunk elements, so the scratch
// bounds the tensor at kNoAllocChunk * kNoAllocMaxChunks elements (2^28 = 1 GiB
// of f32); larger tensors are rejected before anything is launched.
// ---------------------------------------------------------------------------
namespace vnpu_b200 {
namespace {

constexpr uint64_t kNoAllocChunk = 1ull << 14;
constexpr uint32_t kNoAllocMaxChunks = 1u << 14;
constexpr uint32_t kNoAllocCounter = kNoAllocMaxChunks;       // own 128-byte line
constexpr uint32_t kNoAllocResult = kNoAllocMaxChunks + 32;   // own 128-byte line
constexpr uint32_t kNoAllocWords = kNoAllocMaxChunks + 64;    // 65,792 bytes
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint32_t g_quant_noalloc_scratch[kNoAllocWords];

// Pass 1: CTA c takes elements [c * kNoAllocChunk, (c + 1) * kNoAllocChunk).
// The last CTA to finish (threadfence-reduction pattern) folds the partials.
__global__ void __launch_bounds__(256) tensor_absmax_chunks_kernel(const float *__restrict__ X,
                                                                   uint64_t n,
                                                                   uint32_t *scratch) {
    __shared__ float red[32];
    __shared__ bool last;
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kNoAllocChunk;
    const uint64_t end = base + kNoAllocChunk < n ? base + kNoAllocChunk : n;
    float m = 0.0f;
#pragma unroll 8
    for (uint64_t i = base + threadIdx.x; i < end; i += 256) m = fmaxf(m, fabsf(__ldcs(X + i)));
    m = block_max(m, red);
    if (threadIdx.x == 0) {
        scratch[blockIdx.x] = __float_as_uint(m);
        __threadfence();
        last = atomicAdd(scratch + kNoAllocCounter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    uint32_t bits = 0;  // partials are >= 0 (or +inf): IEEE bits order as unsigned
    for (uint32_t c = threadIdx.x; c < gridDim.x; c += 256) bits = max(bits, __ldcg(scratch + c));
    m = block_max(__uint_as_float(bits), red);
    if (threadIdx.x == 0) {
        scratch[kNoAllocResult] = __float_as_uint(m);
        scratch[kNoAllocCounter] = 0;
    }
}

struct NoAllocDevice {
    uint32_t *scratch = nullptr;
    int num_sms = 0;
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

void noalloc_error(const char *what) {
    std::fprintf(stderr, "[vnpu-b200] vnpu_b200_quantize_i8_tensor_noalloc: %s\n", what);
}

// The scratch address of `device` (the current device), resolved on every
// call (cheap once the module is loaded).  When it differs from the one seen
// before - the first call on the device, or a new context after
// cudaDeviceReset reloaded the module - the counter is zeroed synchronously.
vnpu_status_t noalloc_device(int device, NoAllocDevice *out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice &d = g_noalloc_dev[device];
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_quant_noalloc_scratch) != cudaSuccess) {
        cudaGetLastError();
        noalloc_error("cannot resolve the static scratch on this device");
        return VNPU_ERR_DEVICE_ERROR;
    }
    if (p != d.scratch) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
            cudaMemset(static_cast<uint32_t *>(p) + kNoAllocCounter, 0, sizeof(uint32_t)) !=
                cudaSuccess) {
            cudaGetLastError();
            noalloc_error("cannot initialise the static scratch on this device");
            return VNPU_ERR_DEVICE_ERROR;
        }
        d.scratch = static_cast<uint32_t *>(p);
        d.num_sms = sms;
    }
    *out = d;
    return VNPU_OK;
}

bool on_device(const void *p, int device) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) &&
           a.device == device;
}

vnpu_status_t quantize_tensor_noalloc(int device, cudaStream_t stream, const float *X, int8_t *Y,
                                      float *scale, uint64_t rows, uint64_t cols) {
    if (!X || !Y || !scale || !rows || !cols) {
        noalloc_error("X, Y and scale must be non-null and rows, cols non-zero");
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    if (rows > (kNoAllocChunk * kNoAllocMaxChunks) / cols) {
        char msg[160];
        std::snprintf(msg, sizeof msg,
                      "rows*cols exceeds the static scratch limit of %llu elements",
                      static_cast<unsigned long long>(kNoAllocChunk * kNoAllocMaxChunks));
        noalloc_error(msg);
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    if (!on_device(X, device) || !on_device(Y, device) || !on_device(scale, device)) {
        noalloc_error("X, Y and scale must be device memory of the given device");
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    NoAllocDevice d;
    const vnpu_status_t st = noalloc_device(device, &d);
    if (st != VNPU_OK) return st;
    uint64_t n = rows * cols;
    const unsigned chunks = static_cast<unsigned>((n + kNoAllocChunk - 1) / kNoAllocChunk);
    // Launch errors come back from each launch itself, so an error the caller
    // left pending on the thread is neither reported nor cleared here.  If the
    // second launch fails the first one is already enqueued.
    uint32_t *scratch = d.scratch;
    void *absmax_args[] = {const_cast<float **>(&X), &n, &scratch};
    if (cudaLaunchKernel(reinterpret_cast<const void *>(tensor_absmax_chunks_kernel), dim3(chunks),
                         dim3(256), absmax_args, 0, stream) != cudaSuccess) {
        noalloc_error("kernel launch failed");
        return VNPU_ERR_DEVICE_ERROR;
    }
    uint32_t *result = d.scratch + kNoAllocResult;
    void *quant_args[] = {const_cast<float **>(&X), &Y, &scale, &n, &result};
    if (cudaLaunchKernel(reinterpret_cast<const void *>(quantize_tensor_kernel),
                         dim3(static_cast<unsigned>(d.num_sms) * 8), dim3(256), quant_args, 0,
                         stream) != cudaSuccess) {
        noalloc_error("kernel launch failed after the first of its two kernels was enqueued");
        return VNPU_ERR_DEVICE_ERROR;
    }
    return VNPU_OK;
}

}  // namespace
}  // namespace vnpu_b200

extern "C" VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_quantize_i8_tensor_noalloc(
    int device, void *cuda_stream, const float *X, int8_t *Y, float *scale, uint64_t rows,
    uint64_t cols) {
    int count = 0;
    if (device < 0 || device >= vnpu_b200::kNoAllocMaxDevices ||
        cudaGetDeviceCount(&count) != cudaSuccess || device >= count) {
        cudaGetLastError();
        vnpu_b200::noalloc_error("no such CUDA device");
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        vnpu_b200::noalloc_error("cannot make the device current");
        return VNPU_ERR_DEVICE_ERROR;
    }
    const vnpu_status_t st = vnpu_b200::quantize_tensor_noalloc(
        device, static_cast<cudaStream_t>(cuda_stream), X, Y, scale, rows, cols);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return st;
}
