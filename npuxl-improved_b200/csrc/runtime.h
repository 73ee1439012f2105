// runtime.h - object model of the B200 backend behind the vnpu v1 ABI.
//
// Reference object model: src/internal.h:618-725 (vnpu_event, vnpu_buffer,
// vnpu_packed_weights, vnpu_stream, vnpu_device).  The B200 versions:
//   device  - one CUDA device (ordinal), its counters, MMIO window, trace;
//   stream  - one CUDA stream + a device-side error word that kernels'
//             bounded waits write into; commands are enqueued directly from
//             the submitting thread (no worker thread: the GPU is the worker);
//   event   - a CUDA event recorded after a submitted batch + batch status;
//   buffer  - an HBM allocation (cudaMalloc, zero-filled);
//   packed  - resident K-major int8 weights in HBM + device scales, with host
//             copies of scales / column sums for vnpu_packed_weights_info.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/vnpu.h"
#include "../../include/vnpu_b200.h"

namespace vnpu_b200 {

uint64_t now_ns();

struct TraceEvent {
    std::string name;
    uint32_t opcode = 0;
    uint32_t unit = 0;
    uint32_t category = 0;  // 0 compute, 1 memory, 2 sync
    uint64_t start_ns = 0;
    uint64_t dur_ns = 0;
    uint64_t bytes_read = 0;
    uint64_t bytes_written = 0;
    uint64_t flops = 0;
};

struct PendingTrace {
    TraceEvent ev;
    cudaEvent_t begin = nullptr;
    cudaEvent_t end = nullptr;
};

// Sherlock-style trace (reference src/internal.h:443-505,
// src/core/runtime.cpp:327-627) with device time: each traced command is
// bracketed by a pair of CUDA events on its stream, resolved at sync.
struct TraceState {
    std::atomic<bool> enabled{false};
    std::mutex mutex;
    std::vector<TraceEvent> events;
    std::string trace_file;
    static constexpr size_t kMaxEvents = 200000;

    void reset();
    void add(const TraceEvent &ev);
    void summary(vnpu_trace_summary_t *out);
    vnpu_status_t dump_text(const char *path);
    vnpu_status_t write_chrome(const char *path);
};

}  // namespace vnpu_b200

struct vnpu_event {
    std::mutex mutex;
    cudaEvent_t ev = nullptr;
    int ev_device = -1;
    bool recorded = false;       // a batch was submitted with this event
    bool host_signaled = false;  // signalled without GPU work (empty submit)
    vnpu_status_t status = VNPU_OK;
    vnpu_stream_t *stream = nullptr;
    uint64_t command_count = 0;
};

struct vnpu_buffer {
    vnpu_device_t *device = nullptr;
    void *ptr = nullptr;
    uint64_t bytes = 0;
    uint64_t handle = 0;
};

struct vnpu_packed_weights {
    vnpu_device_t *device = nullptr;
    int8_t *bt = nullptr;            // [N][k_stride] K-major, zero padded
    float *scales = nullptr;         // device, N
    int32_t *column_sums = nullptr;  // device, N
    std::vector<float> host_scales;
    std::vector<int32_t> host_column_sums;
    uint32_t K = 0, N = 0, k_stride = 0;
    CUtensorMap tmap{};              // box 128 (K) x 256 (N), 128B swizzle
    CUtensorMap tmap128{};           // box 128 (K) x 128 (N), for the CTA-pair kernel
    bool tmap_ok = false;
    bool tmap128_ok = false;
};

struct vnpu_stream {
    vnpu_device_t *device = nullptr;
    int priority = 0;
    cudaStream_t cs = nullptr;
    uint32_t *d_err = nullptr;       // device error word (kernels atomicOr)
    uint32_t *d_scratch = nullptr;   // 4 bytes: per-tensor absmax
    uint32_t *d_flag = nullptr;      // 4 bytes, zero: the wait self-test's flag
    std::mutex mutex;                // one producer per stream, but be safe
    std::atomic<uint32_t> last_error{0};
    std::atomic<uint64_t> pending{0};
    std::vector<vnpu_b200::PendingTrace> traces;
    bool capturing = false;          // inside vnpu_b200_capture_begin/end
    uint64_t captured_launches = 0;  // kernels recorded by the capture
    // Copy engines for host operands: uploads run on `up`, downloads on
    // `down`, each joined to `cs` by events, so a command's download
    // overlaps the next command's upload and kernels.
    cudaStream_t up = nullptr;
    cudaStream_t down = nullptr;
    // Host ranges that downloads not yet joined into `cs` and `up` write.
    std::vector<std::pair<const char *, uint64_t>> pending_down;
    bool cs_wrote_host = false;      // a COPY/MEMSET on `cs` wrote host memory since `up` last waited
};

struct vnpu_b200_graph {
    vnpu_device_t *device = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;  // kernel launches per replay
};

struct vnpu_device {
    int ordinal = 0;
    vnpu_config_t config{};
    vnpu_device_info_t info{};
    int num_sms = 148;
    // MATMUL_I8 epilogue rounding: the reference device's per-element choice
    // (epi_forced false), or one form for every element (VNPU_B200_EPILOGUE).
    uint32_t epi_form = 0;
    bool epi_forced = false;
    uint64_t wait_limit_ns = 2000000000ull;
    cudaStream_t aux = nullptr;  // device-level work (pack) and status reads
    vnpu_b200::TraceState trace;
    std::atomic<uint32_t> regs[VNPU_REG_COUNT];
    std::atomic<uint64_t> commands_submitted{0};
    std::atomic<uint64_t> commands_completed{0};
    std::atomic<uint64_t> kernel_ns{0};
    std::atomic<uint64_t> dispatch_ns{0};
    std::atomic<uint64_t> memory_ns{0};
    std::atomic<uint64_t> sync_ns{0};
    std::atomic<uint64_t> bytes_read{0};
    std::atomic<uint64_t> bytes_written{0};
    std::atomic<uint64_t> flops{0};
    std::atomic<uint64_t> tiles_dispatched{0};
    std::atomic<uint64_t> tiles_culled{0};
    std::atomic<uint64_t> dma_bytes{0};
    std::atomic<uint64_t> interrupts{0};
    std::atomic<uint32_t> busy{0};
    std::atomic<uint32_t> error{0};
    std::atomic<uint32_t> last_opcode{0};
    std::atomic<uint32_t> tile_m{128}, tile_k{128}, tile_n{256};
    // MATMUL_F32 and MATMUL_I8 reproduce the reference device of the same
    // configuration: its worker-thread count, tile defaults, VNPU_PACK, ISA
    // and host L2 size decide which of its kernels, and so which rounding,
    // owns each output element.
    uint32_t f32_threads = 1;
    std::atomic<uint32_t> f32_tile_m{128}, f32_tile_k{128}, f32_tile_n{64};
    bool f32_pack = true;
    bool f32_scalar = false;
    uint64_t host_l2 = 256u * 1024u;   // the host's L2 bytes, as the reference reads it
    std::atomic<uint64_t> launches{0};  // kernels launched by this library
    vnpu_interrupt_cb_t irq_cb = nullptr;
    void *irq_user = nullptr;
    std::mutex irq_mutex;
    std::mutex stream_mutex;
    std::vector<vnpu_stream_t *> streams;
    std::string name;

    void raise_irq(uint32_t bits);
};
