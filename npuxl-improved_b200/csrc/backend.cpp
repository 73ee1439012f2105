// backend.cpp - the vnpu_get_backend_v1 function table (reference
// src/core/backend.cpp:8-60, layout include/vnpu_backend.h:101-148) and the
// ABI entry points that are outside the B200 int8 path.
//
// The cluster / remote-node / speculative-decoding entry points belong to the
// reference's TCP appliance (src/cluster/*), which this backend does not
// rebuild: they exist so engines keep linking and report
// VNPU_ERR_UNSUPPORTED.  The column-sharded multi-GPU GEMM is driven one
// process per GPU (see bench.py / tests) with NCCL from torch.distributed.
#include <cstring>

#include "../../include/vnpu_backend.h"
#include "runtime.h"

extern "C" {

VNPU_API vnpu_status_t VNPU_CALL vnpu_autotune_gemm(vnpu_device_t *device, uint32_t M,
                                                    uint32_t K, uint32_t N, uint32_t iterations,
                                                    vnpu_dtype_t dtype,
                                                    vnpu_tune_result_t *result) {
    (void)iterations;
    if (!device || !M || !K || !N || !result) return VNPU_ERR_INVALID_ARGUMENT;
    // The GPU kernels use fixed tensor-core tiles chosen at build time; report
    // them (reference src/core/autotune.cpp sweeps CPU tiles instead).
    std::memset(result, 0, sizeof(*result));
    result->tile_m = 128;
    result->tile_k = 128;
    result->tile_n = 256;
    result->unit = VNPU_UNIT_GPU;
    result->threads = device->info.num_threads;
    return dtype == VNPU_DTYPE_I8 ? VNPU_OK : VNPU_ERR_UNSUPPORTED;
}

VNPU_API void VNPU_CALL vnpu_cluster_config_init(vnpu_cluster_config_t *config) {
    if (!config) return;
    std::memset(config, 0, sizeof(*config));
    config->abi_version = VNPU_ABI_VERSION;
    config->num_streams = 1;
    config->request_timeout_ms = 30000;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_create(const vnpu_cluster_config_t *,
                                                     vnpu_cluster_t **out) {
    if (out) *out = nullptr;
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API void VNPU_CALL vnpu_cluster_destroy(vnpu_cluster_t *) {}
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_add_device(vnpu_cluster_t *, vnpu_device_t *,
                                                         uint32_t) {
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_add_remote(vnpu_cluster_t *,
                                                         const vnpu_remote_node_config_t *,
                                                         vnpu_remote_node_t **out) {
    if (out) *out = nullptr;
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_get_stats(const vnpu_cluster_t *,
                                                        vnpu_cluster_stats_t *stats) {
    if (stats) std::memset(stats, 0, sizeof(*stats));
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_cache_weights_f32(vnpu_cluster_t *, const char *,
                                                                const float *, uint32_t,
                                                                uint32_t, uint32_t,
                                                                vnpu_weight_handle_t **out) {
    if (out) *out = nullptr;
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_cluster_matmul_f32(vnpu_cluster_t *, vnpu_weight_handle_t *,
                                                         const float *, float *, uint32_t,
                                                         uint32_t, uint32_t, uint32_t) {
    return VNPU_ERR_UNSUPPORTED;
}

VNPU_API void VNPU_CALL vnpu_node_config_init(vnpu_node_config_t *config) {
    if (!config) return;
    std::memset(config, 0, sizeof(*config));
    config->abi_version = VNPU_ABI_VERSION;
    config->port = 7878;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_node_run(const vnpu_node_config_t *) {
    return VNPU_ERR_UNSUPPORTED;
}
VNPU_API void VNPU_CALL vnpu_node_stop(void) {}

VNPU_API void VNPU_CALL vnpu_speculative_config_init(vnpu_speculative_config_t *config) {
    if (!config) return;
    std::memset(config, 0, sizeof(*config));
    config->abi_version = VNPU_ABI_VERSION;
    config->gamma = 4;
}
VNPU_API vnpu_status_t VNPU_CALL vnpu_speculative_step(vnpu_cluster_t *,
                                                       const vnpu_speculative_config_t *,
                                                       const int32_t *, uint32_t,
                                                       vnpu_logits_fn_t, void *,
                                                       vnpu_logits_fn_t, void *,
                                                       vnpu_speculative_result_t *result) {
    if (result) std::memset(result, 0, sizeof(*result));
    return VNPU_ERR_UNSUPPORTED;
}

// IEEE half / bfloat16 conversions, round to nearest even.
VNPU_API uint16_t VNPU_CALL vnpu_float_to_bf16(float value) {
    uint32_t u;
    std::memcpy(&u, &value, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

VNPU_API float VNPU_CALL vnpu_bf16_to_float(uint16_t value) {
    const uint32_t u = static_cast<uint32_t>(value) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

VNPU_API uint16_t VNPU_CALL vnpu_float_to_f16(float value) {
    uint32_t u;
    std::memcpy(&u, &value, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t absu = u & 0x7fffffffu;
    if (absu > 0x7f800000u) return static_cast<uint16_t>(sign | 0x7e00u);  // NaN
    if (absu >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // overflow -> inf
    if (absu < 0x38800000u) {                                                // subnormal / zero
        if (absu < 0x33000000u) return static_cast<uint16_t>(sign);
        const uint32_t e = absu >> 23;
        const uint32_t m = (absu & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;  // 14..24
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return static_cast<uint16_t>(sign | h);
    }
    uint32_t h = ((absu >> 13) - (112u << 10));
    const uint32_t rem = absu & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return static_cast<uint16_t>(sign | h);
}

VNPU_API float VNPU_CALL vnpu_f16_to_float(uint16_t value) {
    const uint32_t sign = (static_cast<uint32_t>(value) & 0x8000u) << 16;
    uint32_t e = (value >> 10) & 0x1fu;
    uint32_t m = value & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        if (m == 0) {
            u = sign;
        } else {
            e = 113;
            while (!(m & 0x400u)) {
                m <<= 1;
                --e;
            }
            u = sign | (e << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

}  // extern "C"

// ---------------------------------------------------------------- vtable

namespace {

const vnpu_backend_v1_t kBackend = {
    VNPU_ABI_VERSION,
    static_cast<uint32_t>(sizeof(vnpu_backend_v1_t)),
    "vnpu-b200",
    vnpu_device_create,
    vnpu_device_destroy,
    vnpu_device_get_info,
    vnpu_device_get_status,
    vnpu_stream_create,
    vnpu_stream_destroy,
    vnpu_stream_sync,
    vnpu_stream_submit,
    vnpu_event_create,
    vnpu_event_destroy,
    vnpu_event_wait,
    vnpu_buffer_alloc,
    vnpu_buffer_free,
    vnpu_buffer_host_ptr,
    vnpu_matmul_f32,
    vnpu_matmul_i8,
    vnpu_quantize_i8,
    vnpu_pack_weights_i8,
    vnpu_packed_weights_destroy,
    vnpu_rmsnorm_f32,
    vnpu_softmax_f32,
    vnpu_rope_f32,
    vnpu_swiglu_f32,
    vnpu_gelu_f32,
    vnpu_attention_f32,
    vnpu_mtp_head_f32,
    vnpu_trace_enable,
    vnpu_trace_get_summary,
    vnpu_trace_dump,
    vnpu_trace_write_chrome,
    vnpu_autotune_gemm,
    vnpu_cluster_create,
    vnpu_cluster_destroy,
    vnpu_cluster_add_device,
    vnpu_cluster_add_remote,
    vnpu_cluster_cache_weights_f32,
    vnpu_cluster_matmul_f32,
    vnpu_cluster_get_stats,
    vnpu_node_run,
    vnpu_speculative_step,
    vnpu_status_string,
    vnpu_version_string,
    // reserved[]: B200 extensions (vnpu_b200.h), in this order.
    {reinterpret_cast<void *>(&vnpu_b200_stream_handle),
     reinterpret_cast<void *>(&vnpu_b200_device_ordinal),
     reinterpret_cast<void *>(&vnpu_b200_kernel_launches),
     reinterpret_cast<void *>(&vnpu_b200_packed_weights_device),
     reinterpret_cast<void *>(&vnpu_b200_matmul_i8_kernel),
     reinterpret_cast<void *>(&vnpu_b200_selftest_wait_timeout), nullptr, nullptr},
};

}  // namespace

extern "C" VNPU_API const vnpu_backend_v1_t *VNPU_CALL vnpu_get_backend_v1(void) {
    return &kBackend;
}
