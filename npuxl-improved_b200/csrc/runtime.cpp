// runtime.cpp - the vnpu v1 C ABI on a B200: devices, streams, events,
// buffers, packed weights and the command processor.
//
// Reference behaviour restated here (file:line in the reference):
//   argument checks and error codes ...... src/core/scheduler.cpp:370-608,
//                                           src/core/runtime.cpp:1291-1440
//   sticky stream error .................. src/core/runtime.cpp:1248-1254,1281-1289
//   event wait with timeout .............. src/core/runtime.cpp:1165-1178
//   per-command byte/flop accounting ..... src/core/scheduler.cpp:420-426 etc.
//   MMIO window, IRQ ..................... src/core/runtime.cpp:1102-1148
// What is new: commands are enqueued on the stream's CUDA stream by the
// submitting thread; pointer operands in host memory are staged through HBM
// (stream-ordered allocations) so callers written for the CPU library keep
// working, while device pointers are used in place.  No command ever falls
// back to the CPU: a device without sm_100 refuses to create.
#include "runtime.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>

#include <unistd.h>

#include "kernels.h"

using vnpu_b200::LaunchCtx;

namespace vnpu_b200 {

uint64_t now_ns() {
    return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now().time_since_epoch())
                                     .count());
}

namespace {

void debug_log(const char *fmt, ...) {
    if (!std::getenv("VNPU_DEBUG")) return;
    va_list ap;
    va_start(ap, fmt);
    std::fprintf(stderr, "[vnpu-b200] ");
    std::vfprintf(stderr, fmt, ap);
    std::fputc('\n', stderr);
    va_end(ap);
}

// A command-level failure: becomes the command's status (reference: thrown
// std::runtime_error -> VNPU_ERR_INTERNAL in schedule_command).
struct CommandError : std::runtime_error {
    vnpu_status_t status;
    CommandError(const char *what, vnpu_status_t s = VNPU_ERR_INTERNAL)
        : std::runtime_error(what), status(s) {}
};

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        debug_log("%s: %s", what, cudaGetErrorString(e));
        throw CommandError(what, e == cudaErrorMemoryAllocation ? VNPU_ERR_OUT_OF_MEMORY
                                                                 : VNPU_ERR_DEVICE_ERROR);
    }
}

template <typename F>
vnpu_status_t guard(F &&fn) noexcept {
    try {
        return fn();
    } catch (const CommandError &e) {
        debug_log("error: %s", e.what());
        return e.status;
    } catch (const std::bad_alloc &) {
        return VNPU_ERR_OUT_OF_MEMORY;
    } catch (...) {
        return VNPU_ERR_INTERNAL;
    }
}

// ---------------------------------------------------------------------------
// Pointer staging: device pointers are used in place; host pointers (pinned
// or pageable) are copied into stream-ordered HBM allocations before the
// kernel and back after it.
// ---------------------------------------------------------------------------
enum class Mem { kDevice, kHost, kForeign };

Mem classify(const void *p, int device) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return Mem::kHost;
    }
    switch (a.type) {
    case cudaMemoryTypeDevice:
        return a.device == device ? Mem::kDevice : Mem::kForeign;
    case cudaMemoryTypeManaged:
        return Mem::kDevice;
    default:
        return Mem::kHost;
    }
}

// Order stream `waiter` after everything enqueued on `signaller` so far.
void stream_after(cudaStream_t waiter, cudaStream_t signaller) {
    cudaEvent_t ev = nullptr;
    cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "order event");
    cudaError_t e = cudaEventRecord(ev, signaller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(waiter, ev, 0);
    cudaEventDestroy(ev);
    cuda_check(e, "stream order");
}

// Join every pending download into the compute and upload streams.
void join_downloads(vnpu_stream_t *s) {
    if (s->pending_down.empty()) return;
    stream_after(s->cs, s->down);
    stream_after(s->up, s->down);
    s->pending_down.clear();
}

bool overlaps_download(const vnpu_stream_t *s, const void *p, uint64_t bytes) {
    const char *a = static_cast<const char *>(p);
    for (const auto &r : s->pending_down)
        if (a < r.first + r.second && r.first < a + bytes) return true;
    return false;
}

class Staging {
public:
    // Copies on `s` itself (device-level paths without a vnpu stream).
    Staging(cudaStream_t s, int device, bool capturing = false)
        : s_(s), device_(device), capturing_(capturing) {}
    // Copies on the vnpu stream's copy-engine streams.
    explicit Staging(vnpu_stream_t *vs)
        : s_(vs->cs), device_(vs->device->ordinal), capturing_(vs->capturing), vs_(vs) {}
    ~Staging() {
        for (auto &a : allocs_) cudaFreeAsync(a, s_);
    }
    // Input operand of `bytes` bytes.
    template <typename T>
    const T *in(const T *p, uint64_t bytes) {
        return static_cast<const T *>(stage(const_cast<T *>(p), bytes, true, false));
    }
    // Output operand; `read_too` also copies the current contents in
    // (in-place operands, or outputs with gaps the kernel does not write).
    template <typename T>
    T *out(T *p, uint64_t bytes, bool read_too) {
        return static_cast<T *>(stage(p, bytes, read_too, true));
    }
    // Copy staged outputs back after the command's kernels.
    void finish() {
        if (outs_.empty()) return;
        if (!vs_) {
            for (auto &o : outs_)
                cuda_check(cudaMemcpyAsync(o.host, o.dev, o.bytes, cudaMemcpyDeviceToHost, s_),
                           "copy result to host");
            outs_.clear();
            return;
        }
        stream_after(vs_->down, s_);
        for (auto &o : outs_) {
            cuda_check(cudaMemcpyAsync(o.host, o.dev, o.bytes, cudaMemcpyDeviceToHost, vs_->down),
                       "copy result to host");
            vs_->pending_down.emplace_back(static_cast<const char *>(o.host), o.bytes);
        }
        // Output buffers are released behind their download.
        for (auto &o : outs_) {
            auto it = std::find(allocs_.begin(), allocs_.end(), o.dev);
            if (it != allocs_.end()) {
                allocs_.erase(it);
                cudaFreeAsync(o.dev, vs_->down);
            }
        }
        outs_.clear();
        if (vs_->pending_down.size() > 256) join_downloads(vs_);
    }
    uint64_t staged_bytes() const { return staged_; }

private:
    void *stage(void *p, uint64_t bytes, bool copy_in, bool copy_out) {
        if (!p || !bytes) return p;
        const Mem m = classify(p, device_);
        if (m == Mem::kDevice) return p;
        if (m == Mem::kForeign)
            throw CommandError("operand lives on another GPU", VNPU_ERR_INVALID_ARGUMENT);
        if (capturing_)
            throw CommandError("host operand inside a graph capture", VNPU_ERR_INVALID_ARGUMENT);
        auto it = map_.find(p);
        if (it != map_.end()) {
            if (copy_out) outs_.push_back({p, it->second, bytes});
            return it->second;
        }
        void *d = nullptr;
        if (vs_ && copy_in) {
            // Upload on the copy-engine stream, after any pending download
            // into the same host bytes and any host write made on `cs`.
            if (overlaps_download(vs_, p, bytes)) join_downloads(vs_);
            if (vs_->cs_wrote_host) {
                stream_after(vs_->up, s_);
                vs_->cs_wrote_host = false;
            }
            cuda_check(cudaMallocAsync(&d, bytes, vs_->up), "stage operand");
            allocs_.push_back(d);
            cuda_check(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, vs_->up), "stage in");
            stream_after(s_, vs_->up);
        } else {
            cuda_check(cudaMallocAsync(&d, bytes, s_), "stage operand");
            allocs_.push_back(d);
            if (copy_in)
                cuda_check(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, s_), "stage in");
        }
        map_[p] = d;
        staged_ += bytes;
        if (copy_out) outs_.push_back({p, d, bytes});
        return d;
    }
    struct Out {
        void *host;
        void *dev;
        uint64_t bytes;
    };
    cudaStream_t s_;
    int device_;
    bool capturing_;
    vnpu_stream_t *vs_ = nullptr;
    std::vector<void *> allocs_;
    std::vector<Out> outs_;
    std::unordered_map<void *, void *> map_;
    uint64_t staged_ = 0;
};

// Physical cores of this host: distinct SMT sibling sets in sysfs (the
// reference's default worker count, src/core/runtime.cpp:98-145,858-866).
uint32_t host_physical_cores() {
    const unsigned logical = std::max(1u, std::thread::hardware_concurrency());
    std::set<std::string> cores;
    for (unsigned cpu = 0; cpu < logical; ++cpu) {
        const std::string path = "/sys/devices/system/cpu/cpu" + std::to_string(cpu) +
                                 "/topology/core_cpus_list";
        std::FILE *f = std::fopen(path.c_str(), "r");
        if (!f) break;
        char buf[128] = {};
        const size_t got = std::fread(buf, 1, sizeof(buf) - 1, f);
        std::fclose(f);
        std::string key(buf, got);
        while (!key.empty() && (key.back() == '\n' || key.back() == ' ')) key.pop_back();
        if (!key.empty()) cores.insert(key);
    }
    return cores.empty() ? logical : static_cast<uint32_t>(cores.size());
}

bool env_is(const char *name, const char *value) {
    const char *e = std::getenv(name);
    return e && !std::strcmp(e, value);
}

// VNPU_B200_EPILOGUE=block|stream|scalar rounds every MATMUL_I8 element in
// that one form; unset (or "reference"), each element takes the form the
// reference device gives it (i8_form_map).
bool epi_form_from_env(uint32_t &form) {
    const char *e = std::getenv("VNPU_B200_EPILOGUE");
    if (!e) return false;
    if (!std::strcmp(e, "block")) form = kFormBlock;
    else if (!std::strcmp(e, "stream")) form = kFormStream;
    else if (!std::strcmp(e, "scalar")) form = kFormScalar;
    else return false;
    return true;
}

// Bytes of per-worker scratch the reference kernels stage into
// (VNPU_LOCAL_STORE_BYTES, include/vnpu.h:51).
constexpr uint64_t kRefScratchBytes = 256u * 1024u;

FormMap i8_form_map(const vnpu_device_t *d, uint32_t unit, uint32_t flags, uint32_t M, uint32_t K,
                    uint32_t N, bool has_bias, uint32_t epilogue, uint32_t n_full = 0,
                    uint32_t col_base = 0);

struct Accounting {
    uint64_t bytes_read = 0, bytes_written = 0, flops = 0, tiles = 0, dma = 0;
};

LaunchCtx make_ctx(vnpu_stream_t *s, uint64_t *counter) {
    LaunchCtx c;
    c.stream = s->cs;
    c.err = s->d_err;
    c.num_sms = s->device->num_sms;
    c.wait_limit_ns = s->device->wait_limit_ns;
    c.launch_counter = counter;
    return c;
}

// ---------------------------------------------------------------------------
// Command executors.  Each validates like the reference executor it names,
// stages host operands, enqueues the kernel and fills the accounting.
// ---------------------------------------------------------------------------

// src/core/scheduler.cpp:370-428
void exec_matmul_i8(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                    const LaunchCtx &ctx, Accounting &acc) {
    const auto &in = cmd.args.matmul_i8;
    vnpu_packed_weights_t *w = in.B;
    if (!in.A || !w || !in.C || !in.M || !in.K || !in.N)
        throw CommandError("invalid matmul_i8 arguments");
    if (w->K != in.K || w->N != in.N) throw CommandError("packed weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    const uint32_t lda = in.lda ? in.lda : in.K;
    const uint32_t ldc = in.ldc ? in.ldc : in.N;
    if (lda < in.K || ldc < in.N) throw CommandError("invalid int8 leading dimensions");
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(in.A, static_cast<uint64_t>(in.M - 1) * lda + in.K);
    p.lda = lda;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(in.scale_a, sizeof(float) * in.M);
    p.scale_b = w->scales;
    p.bias = st.in(in.bias, sizeof(float) * in.N);
    const uint64_t c_span = (static_cast<uint64_t>(in.M - 1) * ldc + in.N) * sizeof(float);
    p.C = st.out(in.C, c_span, ldc != in.N);
    p.ldc = ldc;
    p.M = in.M;
    p.K = in.K;
    p.N = in.N;
    p.epilogue = in.epilogue;
    p.fmap = i8_form_map(s->device, in.unit, flags, in.M, in.K, in.N, in.bias != nullptr,
                         in.epilogue);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    cuda_check(matmul_i8(ctx, p), "matmul_i8 launch");
    st.finish();
    const uint64_t a_bytes = static_cast<uint64_t>(in.M) * in.K;
    const uint64_t b_bytes = static_cast<uint64_t>(in.K) * in.N;
    acc.bytes_read = a_bytes + b_bytes + sizeof(float) * (in.N + (in.scale_a ? in.M : 0));
    acc.bytes_written = static_cast<uint64_t>(in.M) * in.N * sizeof(float);
    acc.flops = 2ull * in.M * in.K * in.N;
    acc.tiles = ((in.M + 127) / 128) * ((in.N + 255) / 256);
    acc.dma = st.staged_bytes();
}

static_assert(sizeof(vnpu_b200_matmul_i8_shard_args_t) <= sizeof(vnpu_command_t::args),
              "shard args fit the command");

static_assert(sizeof(vnpu_b200_matmul_i8_swiglu_args_t) <= sizeof(vnpu_command_t::args),
              "matmul + swiglu args fit the command");

static_assert(VNPU_B200_ADVANCE_OFFSET + sizeof(vnpu_b200_advance_t) <=
                  sizeof(vnpu_command_t::args),
              "the position advance fits the command");
static_assert(sizeof(vnpu_b200_matmul_i8_residual_args_t) <= VNPU_B200_ADVANCE_OFFSET,
              "the position advance follows the command's own arguments");

// VNPU_B200_CMD_FLAG_ADVANCE_POSITION (the command's own flag: a batch's
// other commands' flags do not apply): the device position, staged.
struct AdvancePosition {
    int32_t *position = nullptr;
    int32_t step = 0;

    AdvancePosition(const vnpu_command_t &cmd, Staging &st) {
        if (!(cmd.flags & VNPU_B200_CMD_FLAG_ADVANCE_POSITION)) return;
        vnpu_b200_advance_t f;
        std::memcpy(&f, cmd.args.raw + VNPU_B200_ADVANCE_OFFSET, sizeof(f));
        if (!f.position) throw CommandError("ADVANCE_POSITION without a position",
                                            VNPU_ERR_INVALID_ARGUMENT);
        position = st.out(f.position, sizeof(int32_t), true);
        step = f.advance;
    }
};

// MATMUL_I8 of a [K][2I] gate/up weight, then SWIGLU_F32 of its halves: the
// validation of exec_matmul_i8, the rounding forms of the 2I-wide product.
void exec_matmul_i8_swiglu(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                           const LaunchCtx &ctx, Accounting &acc) {
    vnpu_b200_matmul_i8_swiglu_args_t in;
    std::memcpy(&in, cmd.args.raw, sizeof(in));
    vnpu_packed_weights_t *w = in.B;
    if (!in.A || !w || !in.Y || !in.M || !in.K || !in.N || (in.N & 1u))
        throw CommandError("invalid matmul_i8_swiglu arguments", VNPU_ERR_INVALID_ARGUMENT);
    if (w->K != in.K || w->N != in.N) throw CommandError("packed weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    const uint32_t I = in.N / 2u;
    const uint32_t lda = in.lda ? in.lda : in.K;
    const uint32_t ldy = in.ldy ? in.ldy : I;
    if (lda < in.K || ldy < I)
        throw CommandError("invalid leading dimensions", VNPU_ERR_INVALID_ARGUMENT);
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(in.A, static_cast<uint64_t>(in.M - 1) * lda + in.K);
    p.lda = lda;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(in.scale_a, sizeof(float) * in.M);
    p.scale_b = w->scales;
    p.bias = st.in(in.bias, sizeof(float) * in.N);
    const uint64_t y_span = (static_cast<uint64_t>(in.M - 1) * ldy + I) * sizeof(float);
    float *Y = st.out(in.Y, y_span, ldy != I);
    p.C = nullptr;
    p.M = in.M;
    p.K = in.K;
    p.N = in.N;
    p.epilogue = in.epilogue;
    p.fmap = i8_form_map(s->device, VNPU_UNIT_AUTO, flags, in.M, in.K, in.N, in.bias != nullptr,
                         in.epilogue);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    if (cmd.flags & VNPU_B200_CMD_FLAG_ADVANCE_POSITION)
        throw CommandError("ADVANCE_POSITION on MATMUL_I8_SWIGLU", VNPU_ERR_INVALID_ARGUMENT);
    cuda_check(matmul_i8_swiglu(ctx, p, Y, ldy, in.alpha == 0.0f ? 1.0f : in.alpha),
               "matmul_i8_swiglu launch");
    st.finish();
    acc.bytes_read = static_cast<uint64_t>(in.M) * in.K + static_cast<uint64_t>(in.K) * in.N;
    acc.bytes_written = static_cast<uint64_t>(in.M) * I * sizeof(float);
    acc.flops = 2ull * in.M * in.K * in.N + 4ull * in.M * I;
    acc.dma = st.staged_bytes();
}

// MATMUL_I8 of the columns col_base.. of an n_full-wide product: the same
// validation and kernels as exec_matmul_i8, with every element rounded as in
// the whole product.
void exec_matmul_i8_shard(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                          const LaunchCtx &ctx, Accounting &acc) {
    vnpu_b200_matmul_i8_shard_args_t in;
    std::memcpy(&in, cmd.args.raw, sizeof(in));
    vnpu_packed_weights_t *w = in.B;
    const uint32_t n_full = in.n_full ? in.n_full : in.N;
    if (!in.A || !w || !in.C || !in.M || !in.K || !in.N ||
        static_cast<uint64_t>(in.col_base) + in.N > n_full)
        throw CommandError("invalid matmul_i8_shard arguments", VNPU_ERR_INVALID_ARGUMENT);
    if (w->K != in.K || w->N != in.N) throw CommandError("packed weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    const uint32_t lda = in.lda ? in.lda : in.K;
    const uint32_t ldc = in.ldc ? in.ldc : in.N;
    if (lda < in.K || ldc < in.N) throw CommandError("invalid int8 leading dimensions");
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(in.A, static_cast<uint64_t>(in.M - 1) * lda + in.K);
    p.lda = lda;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(in.scale_a, sizeof(float) * in.M);
    p.scale_b = w->scales;
    p.bias = st.in(in.bias, sizeof(float) * in.N);
    const uint64_t c_span = (static_cast<uint64_t>(in.M - 1) * ldc + in.N) * sizeof(float);
    p.C = st.out(in.C, c_span, ldc != in.N);
    p.ldc = ldc;
    p.M = in.M;
    p.K = in.K;
    p.N = in.N;
    p.epilogue = in.epilogue;
    p.fmap = i8_form_map(s->device, VNPU_UNIT_AUTO, flags, in.M, in.K, in.N, in.bias != nullptr,
                         in.epilogue, n_full, in.col_base);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    cuda_check(matmul_i8(ctx, p), "matmul_i8_shard launch");
    st.finish();
    acc.bytes_read = static_cast<uint64_t>(in.M) * in.K + static_cast<uint64_t>(in.K) * in.N;
    acc.bytes_written = static_cast<uint64_t>(in.M) * in.N * sizeof(float);
    acc.flops = 2ull * in.M * in.K * in.N;
    acc.dma = st.staged_bytes();
}

// choose_unit, src/core/scheduler.cpp:43-62 (GPU is this device: the F32
// path then follows the reference's default unit).
uint32_t f32_unit(const vnpu_matmul_f32_args_t &a, uint32_t flags) {
    if (flags & VNPU_CMD_FLAG_CELL_DMA) return VNPU_UNIT_CELL;
    if (flags & VNPU_CMD_FLAG_VOODOO_FIFO) return VNPU_UNIT_VOODOO;
    if (a.unit != VNPU_UNIT_AUTO && a.unit != VNPU_UNIT_GPU) return a.unit;
    if (a.tile_mask || (flags & VNPU_CMD_FLAG_WILDCAT_CULL)) return VNPU_UNIT_WILDCAT;
    return VNPU_UNIT_VOODOO;
}

uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

// Widest int8 decode column tile, src/core/scheduler.cpp:75-93: half of the
// host L2 shared by `rows` int32 staging rows, at most what a worker's 256 KiB
// scratch stages, whole 32-column groups, at least 256.
uint32_t decode_tile_cap(uint64_t l2, uint32_t rows) {
    if (!l2) l2 = 512u * 1024u;
    uint64_t cols = std::min<uint64_t>(l2 / (8ull * rows), kRefScratchBytes / (4ull * rows));
    cols &= ~uint64_t{31};
    return static_cast<uint32_t>(std::min<uint64_t>(std::max<uint64_t>(cols, 256), 0x7fffffffu));
}

// The reference's tile geometry, src/core/scheduler.cpp:95-207.
void ref_tile_geometry(const vnpu_device_t *d, uint32_t unit, uint32_t M, uint32_t N, bool int8,
                       uint32_t &tm, uint32_t &tn) {
    tm = std::max<uint32_t>(1, d->f32_tile_m.load());
    tn = std::max<uint32_t>(1, d->f32_tile_n.load());
    const uint32_t units = std::max<uint32_t>(1, d->f32_threads);
    const bool voodoo = unit == VNPU_UNIT_VOODOO || unit == VNPU_UNIT_AUTO;
    if (M <= 8 && voodoo) {
        tm = M;
        if (int8 && M <= 3 && N / units >= 1024u) {
            // one contiguous column slice per worker, bounded by the staging cap
            uint32_t tiles = std::min<uint32_t>(units, std::max<uint32_t>(1, N / 256u));
            const uint32_t cap = decode_tile_cap(d->host_l2, M);
            if (ceil_div(N, tiles) > cap) tiles = ceil_div(ceil_div(N, cap), units) * units;
            tn = std::min<uint32_t>(N, std::max<uint32_t>(1, (ceil_div(N, tiles) + 31u) & ~31u));
            return;
        }
        tn = std::min<uint32_t>(std::max<uint32_t>(32, tn), 64);  // 32..64 column tiles
        tn = std::min(tn, N);
        return;
    }
    if (d->f32_pack && voodoo && M >= 3 && ceil_div(N, 64) >= 2 * units) {
        tm = M;  // one panel-packed tile spans all rows
        tn = 64;
        return;
    }
    if (unit == VNPU_UNIT_WILDCAT) {
        tm = std::min<uint32_t>(tm, 32);
        tn = std::min<uint32_t>(tn, 64);
    } else if (unit == VNPU_UNIT_CELL) {
        tm = std::min<uint32_t>(tm, 16);
        tn = std::min<uint32_t>(tn, 64);
    }
    const uint64_t target = static_cast<uint64_t>(units) * 64;
    auto count = [&] { return static_cast<uint64_t>(ceil_div(M, tm)) * ceil_div(N, tn); };
    while (count() > target && (tm < M || tn < N)) {
        if (tm < M) tm = std::min(M, tm * 2);
        if (tn < N) tn = std::min(N, tn * 2);
    }
}

// choose_unit for MATMUL_I8 (src/core/scheduler.cpp:43-62, :378-382): the
// GPU unit is this device and follows the default unit.
uint32_t i8_unit(uint32_t unit, uint32_t flags) {
    if (flags & VNPU_CMD_FLAG_CELL_DMA) return VNPU_UNIT_CELL;
    if (flags & VNPU_CMD_FLAG_VOODOO_FIFO) return VNPU_UNIT_VOODOO;
    if (unit != VNPU_UNIT_AUTO && unit != VNPU_UNIT_GPU) return unit;
    if (flags & VNPU_CMD_FLAG_WILDCAT_CULL) return VNPU_UNIT_WILDCAT;
    return VNPU_UNIT_VOODOO;
}

// The form in which the reference's AVX2 kernels round the dequant epilogue
// of an element of a rows x cols tile (gemm_i8_dispatch_tile,
// src/kernels/kernels.cpp:922-978).  `single`: the element's row is the odd
// last row of the tile; `tail`: its column lies past the tile's last whole
// 32 columns.  Which kernel GCC fused where was found element by element
// against the reference build (the oracle's restatement is pinned to it):
//   rank-2/3 staged streams (:581-632)                        stream
//   packed panel or unpacked 2x32 / 1x32 register blocks      block
//   the scalar tile over a row pair's column tail             stream
//   the scalar tile over a single row's column tail           scalar
//   the rank-1 row stream of an unpacked single row (:746-764) stream
uint32_t ref_tile_form(uint32_t rows, uint32_t cols, uint32_t K, bool pack, bool single,
                       bool tail) {
    const uint64_t stride8 = (static_cast<uint64_t>(cols) + 7u) & ~uint64_t{7};
    if (cols >= 1024u && (rows == 2u || rows == 3u) && stride8 * rows * 4u <= kRefScratchBytes)
        return kFormStream;
    if (pack && rows >= 3u && static_cast<uint64_t>(K) * cols <= kRefScratchBytes)
        return tail ? (single ? kFormScalar : kFormStream) : kFormBlock;
    if (!single) return tail ? kFormStream : kFormBlock;
    if (static_cast<uint64_t>(cols) * 4u <= kRefScratchBytes) return kFormStream;
    return tail ? kFormScalar : kFormBlock;   // the 1x32 blocked walk, scalar tail
}

// MATMUL_I8's epilogue rounding, element by element, as the reference device
// this one models computes an M x K x N product (n_full columns in all, this
// launch's column 0 at col_base; n_full 0 = N).  Command flags and
// VNPU_B200_EPILOGUE force one form.  The map collapses to one form when every
// class of element that occurs rounds to the same bits: without a bias the
// block and stream forms agree, with NONE / RELU the stream and scalar ones.
FormMap i8_form_map(const vnpu_device_t *d, uint32_t unit, uint32_t flags, uint32_t M, uint32_t K,
                    uint32_t N, bool has_bias, uint32_t epilogue, uint32_t n_full,
                    uint32_t col_base) {
    FormMap fm;
    if (!n_full) n_full = N;
    const bool act = epilogue >= VNPU_EPILOGUE_SILU && epilogue <= VNPU_EPILOGUE_GELU_ERF;
    auto canon = [&](uint32_t f) -> uint32_t {
        if (!has_bias) return (act && f == kFormScalar) ? kFormScalar : kFormBlock;
        if (!act) return f == kFormBlock ? kFormBlock : kFormStream;
        return f;
    };
    if (flags & VNPU_CMD_FLAG_EPI_SCALAR) fm.form = kFormScalar;
    else if (flags & VNPU_CMD_FLAG_EPI_STREAM) fm.form = kFormStream;
    else if (flags & VNPU_CMD_FLAG_EPI_BLOCK) fm.form = kFormBlock;
    else if (d->epi_forced) fm.form = d->epi_form;
    else {
        unit = i8_unit(unit, flags);
        if (d->f32_scalar || unit == VNPU_UNIT_CELL) {
            fm.form = kFormScalar;   // scalar ISA / Cell tile: nothing fused
        } else {
            uint32_t tm, tn;
            ref_tile_geometry(d, unit, M, n_full, true, tm, tn);
            const uint32_t tiles_m = ceil_div(M, tm), tiles_n = ceil_div(n_full, tn);
            const uint32_t rows_last = M - (tiles_m - 1) * tm;
            const uint32_t cols_last = n_full - (tiles_n - 1) * tn;
            // classes that occur: row (last tile?, odd single row?), column
            // (last tile?, tail?)
            bool row_cls[4] = {}, col_cls[4] = {};
            if (tiles_m > 1) {
                row_cls[0] = tm >= 2;
                row_cls[1] = (tm & 1u) != 0;
            }
            row_cls[2] = rows_last >= 2;
            row_cls[3] = (rows_last & 1u) != 0;
            if (tiles_n > 1) {
                col_cls[0] = tn >= 32;
                col_cls[1] = (tn & 31u) != 0;
            }
            col_cls[2] = cols_last >= 32;
            col_cls[3] = (cols_last & 31u) != 0;
            uint32_t seen = 0;   // canonical forms present, one bit each
            for (uint32_t rc = 0; rc < 4; ++rc)
                for (uint32_t cc = 0; cc < 4; ++cc) {
                    const uint32_t rows = (rc & 2u) ? rows_last : tm;
                    const uint32_t cols = (cc & 2u) ? cols_last : tn;
                    const uint32_t f = ref_tile_form(rows, cols, K, d->f32_pack, rc & 1u, cc & 1u);
                    fm.table |= f << (2u * (rc * 4u + cc));
                    if (row_cls[rc] && col_cls[cc]) seen |= 1u << canon(f);
                }
            if (seen && !(seen & (seen - 1u))) {
                fm.form = static_cast<uint32_t>(__builtin_ctz(seen));
                fm.table = 0;
            } else {
                fm.form = kFormMixed;
                fm.tm = tm;
                fm.tn = tn;
            }
        }
    }
    fm.M = M;
    fm.N = n_full;
    fm.col_base = col_base;
    return fm;
}

// src/core/scheduler.cpp:274-352 (prepare_matmul_f32 + execute_matmul_f32)
void exec_matmul_f32(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                     const LaunchCtx &ctx, Accounting &acc) {
    const auto &in = cmd.args.matmul_f32;
    if (!in.A || !in.B || !in.C || !in.M || !in.K || !in.N)
        throw CommandError("invalid matmul_f32 arguments");
    if (static_cast<uint64_t>(in.M) * in.K > UINT64_MAX / in.N)
        throw CommandError("matmul_f32 size overflow");
    if (in.trans_a > 1 || in.trans_b > 1 || in.epilogue > VNPU_EPILOGUE_GELU_ERF)
        throw CommandError("invalid matmul_f32 arguments");
    const uint32_t lda = in.lda ? in.lda : (in.trans_a ? in.M : in.K);
    const uint32_t ldb = in.ldb ? in.ldb : (in.trans_b ? in.K : in.N);
    const uint32_t ldc = in.ldc ? in.ldc : in.N;
    if (lda < (in.trans_a ? in.M : in.K) || ldb < (in.trans_b ? in.K : in.N) || ldc < in.N)
        throw CommandError("invalid matmul_f32 leading dimensions");
    const vnpu_device_t *d = s->device;
    const uint32_t unit = f32_unit(in, flags);
    const bool scalar_isa = d->f32_scalar || (flags & VNPU_CMD_FLAG_EPI_SCALAR);
    MatmulF32 p;
    ref_tile_geometry(d, unit, in.M, in.N, false, p.tile_m, p.tile_n);
    if (unit == VNPU_UNIT_CELL || scalar_isa || in.trans_a) p.mode = kF32Unfused;
    else if (in.trans_b) p.mode = kF32Dot8;
    else p.mode = kF32Block;
    p.packed = p.mode == kF32Block && d->f32_pack;
    Staging st(s);
    const uint64_t a_span = in.trans_a ? static_cast<uint64_t>(in.K - 1) * lda + in.M
                                       : static_cast<uint64_t>(in.M - 1) * lda + in.K;
    const uint64_t b_span = in.trans_b ? static_cast<uint64_t>(in.N - 1) * ldb + in.K
                                       : static_cast<uint64_t>(in.K - 1) * ldb + in.N;
    p.A = st.in(in.A, a_span * sizeof(float));
    p.B = st.in(in.B, b_span * sizeof(float));
    p.bias = st.in(in.bias, sizeof(float) * in.N);
    const uint64_t c_span = (static_cast<uint64_t>(in.M - 1) * ldc + in.N) * sizeof(float);
    p.C = st.out(in.C, c_span, in.beta != 0.0f || ldc != in.N);
    if (in.tile_mask && in.mask_tile_m && in.mask_tile_n) {
        p.mask = st.in(in.tile_mask, static_cast<uint64_t>(in.mask_tile_m) * in.mask_tile_n);
        p.mask_m = in.mask_tile_m;
        p.mask_n = in.mask_tile_n;
    }
    p.M = in.M;
    p.K = in.K;
    p.N = in.N;
    p.lda = lda;
    p.ldb = ldb;
    p.ldc = ldc;
    p.trans_a = in.trans_a;
    p.trans_b = in.trans_b;
    p.alpha = in.alpha == 0.0f ? 1.0f : in.alpha;
    p.beta = in.beta;
    p.epilogue = in.epilogue;
    cuda_check(matmul_f32(ctx, p), "matmul_f32 launch");
    st.finish();
    const uint64_t a_bytes = static_cast<uint64_t>(in.M) * in.K * sizeof(float);
    const uint64_t b_bytes = static_cast<uint64_t>(in.K) * in.N * sizeof(float);
    const uint64_t c_bytes = static_cast<uint64_t>(in.M) * in.N * sizeof(float);
    acc.bytes_read = a_bytes + b_bytes + (in.bias ? sizeof(float) * in.N : 0) +
                     (in.beta != 0.0f ? c_bytes : 0);
    acc.bytes_written = c_bytes;
    acc.flops = 2ull * in.M * in.K * in.N;
    acc.tiles = static_cast<uint64_t>(ceil_div(in.M, p.tile_m)) * ceil_div(in.N, p.tile_n);
    acc.dma = unit == VNPU_UNIT_CELL ? a_bytes + b_bytes : st.staged_bytes();
}

void exec_matmul_i8_scatter(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                            const LaunchCtx &ctx, Accounting &acc) {
    vnpu_b200_matmul_i8_scatter_args_t in;
    std::memcpy(&in, cmd.args.raw, sizeof(in));
    vnpu_packed_weights_t *w = in.B;
    if (!in.A || !w || !in.M || !in.K || !in.N || !in.ndst || in.ndst > VNPU_B200_SCATTER_MAX ||
        !in.ldd || in.ldd % 4u || in.col_offset % 4u ||
        static_cast<uint64_t>(in.col_offset) + in.N > in.ldd)
        throw CommandError("invalid matmul_i8_scatter arguments", VNPU_ERR_INVALID_ARGUMENT);
    for (uint32_t d = 0; d < in.ndst; ++d)
        if (!in.dst[d] || reinterpret_cast<uintptr_t>(in.dst[d]) % 16u)
            throw CommandError("invalid matmul_i8_scatter destination", VNPU_ERR_INVALID_ARGUMENT);
    if (w->K != in.K || w->N != in.N) throw CommandError("packed weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    const uint32_t lda = in.lda ? in.lda : in.K;
    if (lda < in.K) throw CommandError("invalid int8 leading dimension");
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(in.A, static_cast<uint64_t>(in.M - 1) * lda + in.K);
    p.lda = lda;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(in.scale_a, sizeof(float) * in.M);
    p.scale_b = w->scales;
    p.bias = st.in(in.bias, sizeof(float) * in.N);
    p.C = in.dst[0];
    p.ldc = in.ldd;
    p.M = in.M;
    p.K = in.K;
    p.N = in.N;
    p.epilogue = in.epilogue;
    // the shard's columns round as columns col_offset.. of the whole ldd-wide
    // product the reference device would compute
    p.fmap = i8_form_map(s->device, VNPU_UNIT_AUTO, flags, in.M, in.K, in.N, in.bias != nullptr,
                         in.epilogue, in.ldd, in.col_offset);
    if (p.fmap.form == kFormMixed)
        throw CommandError("matmul_i8_scatter: the reference device rounds this shard's elements "
                           "in more than one form; submit MATMUL_I8 per shard or force one form "
                           "with a VNPU_CMD_FLAG_EPI_* flag", VNPU_ERR_UNSUPPORTED);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    for (uint32_t d = 0; d < in.ndst; ++d) p.dst[d] = in.dst[d];
    p.ndst = in.ndst;
    p.ldd = in.ldd;
    p.col_offset = in.col_offset;
    const cudaError_t e = matmul_i8_scatter(ctx, p);
    if (e == cudaErrorNotSupported)
        throw CommandError("matmul_i8_scatter needs a TMA-aligned A", VNPU_ERR_UNSUPPORTED);
    cuda_check(e, "matmul_i8_scatter launch");
    st.finish();
    acc.bytes_read = static_cast<uint64_t>(in.M) * in.K + static_cast<uint64_t>(in.K) * in.N;
    acc.bytes_written = static_cast<uint64_t>(in.M) * in.N * sizeof(float) * in.ndst;
    acc.flops = 2ull * in.M * in.K * in.N;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:430-473
void exec_quantize_i8(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                      Accounting &acc) {
    const auto &a = cmd.args.quantize_i8;
    if (!a.X || !a.Y || !a.scales || !a.rows || !a.cols || a.axis > VNPU_QUANT_PER_TENSOR)
        throw CommandError("invalid quantize_i8 arguments");
    if (a.cols && a.rows > UINT64_MAX / a.cols) throw CommandError("quantize shape overflow");
    const uint64_t total = a.rows * a.cols;
    if (total > (UINT64_MAX >> 3)) throw CommandError("quantize shape overflow");
    const uint64_t nscales = a.axis == VNPU_QUANT_PER_ROW      ? a.rows
                             : a.axis == VNPU_QUANT_PER_COLUMN ? a.cols
                                                               : 1;
    Staging st(s);
    const float *X = st.in(a.X, total * sizeof(float));
    int8_t *Y = st.out(a.Y, total, false);
    float *sc = st.out(a.scales, nscales * sizeof(float), false);
    cudaError_t e;
    if (a.axis == VNPU_QUANT_PER_ROW)
        e = quantize_rows(ctx, X, Y, sc, a.rows, a.cols);
    else if (a.axis == VNPU_QUANT_PER_COLUMN)
        e = quantize_columns(ctx, X, Y, sc, a.rows, a.cols);
    else
        e = quantize_tensor(ctx, X, Y, sc, a.rows, a.cols, s->d_scratch);
    cuda_check(e, "quantize_i8 launch");
    st.finish();
    acc.bytes_read = total * sizeof(float);
    acc.bytes_written = total;
    acc.flops = total * 3;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:475-490
void exec_rmsnorm(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                  Accounting &acc) {
    const auto &a = cmd.args.rmsnorm;
    if (!a.X || !a.Y || !a.rows || !a.cols) throw CommandError("invalid rmsnorm arguments");
    const uint64_t n = static_cast<uint64_t>(a.rows) * a.cols;
    Staging st(s);
    float *Y = st.out(a.Y, n * sizeof(float), a.Y == a.X);
    const float *X = st.in(a.X, n * sizeof(float));
    const float *W = st.in(a.W, sizeof(float) * a.cols);
    const float eps = a.eps > 0.0f ? a.eps : 1e-5f;
    cuda_check(rmsnorm(ctx, X, W, Y, a.rows, a.cols, eps), "rmsnorm launch");
    st.finish();
    acc.bytes_read = n * sizeof(float) + (a.W ? a.cols * sizeof(float) : 0);
    acc.bytes_written = n * sizeof(float);
    acc.flops = n * 5;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:510-535 + rotate_vector's frequencies (llm.cpp:188-217)
// RoPE inverse frequencies, src/kernels/llm.cpp:188-217: the same float libm
// calls as the reference, evaluated once per pair on the host.
void rope_inv_freq(float theta, uint32_t head_dim, bool interleaved, float *inv) {
    for (uint32_t j = 0; j < head_dim / 2; ++j) {
        const float expo = interleaved
                               ? static_cast<float>(2 * j) / static_cast<float>(head_dim)
                               : 2.0f * static_cast<float>(j) / static_cast<float>(head_dim);
        inv[j] = 1.0f / std::pow(theta, expo);
    }
}

void exec_rope(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
               Accounting &acc) {
    const auto &a = cmd.args.rope;
    if ((!a.Q && !a.K) || !a.batch || !a.heads || !a.head_dim || (!a.q_seq && !a.k_seq) ||
        (a.head_dim & 1u))
        throw CommandError("invalid rope arguments");
    if (a.head_dim > 512) throw CommandError("rope head_dim above 512", VNPU_ERR_UNSUPPORTED);
    const float theta = a.theta_base > 0.0f ? a.theta_base : 10000.0f;
    const float scaling = a.scaling > 0.0f ? a.scaling : 1.0f;
    float inv[256];
    rope_inv_freq(theta, a.head_dim, a.interleaved != 0, inv);
    const uint64_t qn = static_cast<uint64_t>(a.batch) * a.heads * a.q_seq * a.head_dim;
    const uint64_t kn = static_cast<uint64_t>(a.batch) * a.heads * a.k_seq * a.head_dim;
    const uint32_t seq = std::max(a.q_seq, a.k_seq);
    Staging st(s);
    float *Q = st.out(a.Q, qn * sizeof(float), true);
    float *K = st.out(a.K, kn * sizeof(float), true);
    const int32_t *pos = st.in(a.positions, sizeof(int32_t) * seq);
    cuda_check(rope(ctx, a.q_seq ? Q : nullptr, a.k_seq ? K : nullptr, pos, a.batch, a.heads,
                    a.q_seq, a.k_seq, a.head_dim, a.position_offset, a.interleaved, scaling,
                    inv),
               "rope launch");
    st.finish();
    acc.bytes_read = (qn + kn) * sizeof(float);
    acc.bytes_written = (qn + kn) * sizeof(float);
    acc.flops = (qn + kn) * 8;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:537-549
void exec_rmsnorm_quantize(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                           Accounting &acc) {
    vnpu_b200_rmsnorm_quantize_args_t a;
    std::memcpy(&a, cmd.args.raw, sizeof(a));
    if (!a.X || !a.Q || !a.scales || !a.rows || !a.cols)
        throw CommandError("invalid rmsnorm_quantize arguments");
    const uint64_t n = static_cast<uint64_t>(a.rows) * a.cols;
    Staging st(s);
    float *Y = a.Y ? st.out(a.Y, n * sizeof(float), a.Y == a.X) : nullptr;
    const float *X = st.in(a.X, n * sizeof(float));
    const float *W = st.in(a.W, sizeof(float) * a.cols);
    int8_t *Q = st.out(a.Q, n, false);
    float *sc = st.out(a.scales, sizeof(float) * a.rows, false);
    const float eps = a.eps > 0.0f ? a.eps : 1e-5f;
    cuda_check(rmsnorm_quantize(ctx, X, W, Y, Q, sc, a.rows, a.cols, eps), "rmsnorm_quantize launch");
    st.finish();
    acc.bytes_read = n * sizeof(float) + (a.W ? a.cols * sizeof(float) : 0);
    acc.bytes_written = n + (a.Y ? n * sizeof(float) : 0) + a.rows * sizeof(float);
    acc.flops = n * 8;
    acc.dma = st.staged_bytes();
}

void exec_swiglu_quantize(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                          Accounting &acc) {
    vnpu_b200_swiglu_quantize_args_t a;
    std::memcpy(&a, cmd.args.raw, sizeof(a));
    const uint32_t ld = a.ld ? a.ld : a.cols;
    if (!a.gate || !a.up || !a.Q || !a.scales || !a.rows || !a.cols || ld < a.cols)
        throw CommandError("invalid swiglu_quantize arguments");
    const uint64_t n = static_cast<uint64_t>(a.rows) * a.cols;
    const uint64_t span = static_cast<uint64_t>(a.rows - 1) * ld + a.cols;   // gate / up extent
    Staging st(s);
    float *Y = a.Y ? st.out(a.Y, n * sizeof(float), a.Y == a.gate || a.Y == a.up) : nullptr;
    const float *G = st.in(a.gate, span * sizeof(float));
    const float *U = st.in(a.up, span * sizeof(float));
    int8_t *Q = st.out(a.Q, n, false);
    float *sc = st.out(a.scales, sizeof(float) * a.rows, false);
    cuda_check(swiglu_quantize(ctx, G, U, Y, Q, sc, a.rows, a.cols, ld,
                               a.alpha == 0.0f ? 1.0f : a.alpha),
               "swiglu_quantize launch");
    st.finish();
    acc.bytes_read = n * 2 * sizeof(float);
    acc.bytes_written = n + (a.Y ? n * sizeof(float) : 0) + a.rows * sizeof(float);
    acc.flops = n * 11;
    acc.dma = st.staged_bytes();
}

void exec_kv_append(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                    Accounting &acc) {
    vnpu_b200_kv_append_args_t a;
    std::memcpy(&a, cmd.args.raw, sizeof(a));
    if (!a.K || !a.V || !a.K_cache || !a.V_cache || !a.heads || !a.T || !a.head_dim ||
        !a.capacity)
        throw CommandError("invalid kv_append arguments", VNPU_ERR_INVALID_ARGUMENT);
    if (!a.position && static_cast<uint64_t>(a.position_offset) + a.T > a.capacity)
        throw CommandError("kv_append past the cache capacity", VNPU_ERR_INVALID_ARGUMENT);
    const uint64_t n = static_cast<uint64_t>(a.heads) * a.T * a.head_dim;
    const uint64_t cn = static_cast<uint64_t>(a.heads) * a.capacity * a.head_dim;
    Staging st(s);
    const float *K = st.in(a.K, n * sizeof(float));
    const float *V = st.in(a.V, n * sizeof(float));
    float *Kc = st.out(a.K_cache, cn * sizeof(float), true);
    float *Vc = st.out(a.V_cache, cn * sizeof(float), true);
    float *M = a.mask ? st.out(a.mask, sizeof(float) * a.heads * a.capacity, true) : nullptr;
    const int32_t *P = a.position ? st.in(a.position, sizeof(int32_t)) : nullptr;
    cuda_check(kv_append(ctx, K, V, Kc, Vc, M, P, a.heads, a.T, a.head_dim, a.capacity,
                         a.position_offset),
               "kv_append launch");
    st.finish();
    acc.bytes_read = 2 * n * sizeof(float);
    acc.bytes_written = 2 * n * sizeof(float);
    acc.dma = st.staged_bytes();
}

static_assert(sizeof(vnpu_b200_qkv_rope_append_args_t) <= sizeof(vnpu_command_t::args),
              "QKV args fit the command");
static_assert(sizeof(vnpu_b200_matmul_i8_residual_args_t) <= sizeof(vnpu_command_t::args),
              "residual args fit the command");

// MATMUL_I8 (QKV weights) + ROPE_F32 + KV_APPEND in one command.
void exec_qkv_rope_append(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                          const LaunchCtx &ctx, Accounting &acc) {
    vnpu_b200_qkv_rope_append_args_t a;
    std::memcpy(&a, cmd.args.raw, sizeof(a));
    vnpu_packed_weights_t *w = a.B;
    if (!a.A || !w || !a.Q || !a.K_cache || !a.V_cache || !a.T || !a.K || !a.heads ||
        !a.head_dim || (a.head_dim & 1u) || !a.capacity)
        throw CommandError("invalid qkv_rope_append arguments", VNPU_ERR_INVALID_ARGUMENT);
    if (a.head_dim > 512)
        throw CommandError("qkv_rope_append head_dim above 512", VNPU_ERR_UNSUPPORTED);
    const uint64_t N = 3ull * a.heads * a.head_dim;
    if (w->K != a.K || w->N != N) throw CommandError("packed QKV weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    if (!a.position && static_cast<uint64_t>(a.position_offset) + a.T > a.capacity)
        throw CommandError("qkv_rope_append past the cache capacity", VNPU_ERR_INVALID_ARGUMENT);
    const float theta = a.theta_base > 0.0f ? a.theta_base : 10000.0f;
    float inv[256];
    rope_inv_freq(theta, a.head_dim, false, inv);
    const uint64_t n = static_cast<uint64_t>(a.heads) * a.T * a.head_dim;
    const uint64_t cn = static_cast<uint64_t>(a.heads) * a.capacity * a.head_dim;
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(a.A, static_cast<uint64_t>(a.T) * a.K);
    p.lda = a.K;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(a.scale_a, sizeof(float) * a.T);
    p.scale_b = w->scales;
    p.bias = st.in(a.bias, sizeof(float) * N);
    p.M = a.T;
    p.K = a.K;
    p.N = static_cast<uint32_t>(N);
    p.ldc = static_cast<uint32_t>(N);
    p.epilogue = a.epilogue;
    p.fmap = i8_form_map(s->device, VNPU_UNIT_AUTO, flags, a.T, a.K, static_cast<uint32_t>(N),
                         a.bias != nullptr, a.epilogue);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    QkvRope q;
    q.Q = st.out(a.Q, n * sizeof(float), false);
    q.K_out = st.out(a.K_out, n * sizeof(float), false);
    q.V_out = st.out(a.V_out, n * sizeof(float), false);
    q.K_cache = st.out(a.K_cache, cn * sizeof(float), true);
    q.V_cache = st.out(a.V_cache, cn * sizeof(float), true);
    q.mask = a.mask ? st.out(a.mask, sizeof(float) * a.heads * a.capacity, true) : nullptr;
    q.position = a.position ? st.in(a.position, sizeof(int32_t)) : nullptr;
    q.heads = a.heads;
    q.head_dim = a.head_dim;
    q.capacity = a.capacity;
    q.position_offset = a.position_offset;
    q.scaling = a.scaling > 0.0f ? a.scaling : 1.0f;
    q.inv_freq = inv;
    if (a.T == 1) {
        cuda_check(qkv_rope_append_gemv(ctx, p, q), "qkv_rope_append launch");
    } else {
        // MATMUL_I8 into a stream-ordered scratch, then split / rotate / append.
        float *tmp = nullptr;
        cuda_check(cudaMallocAsync(reinterpret_cast<void **>(&tmp), N * a.T * sizeof(float),
                                   ctx.stream),
                   "qkv scratch");
        p.C = tmp;
        cudaError_t e = matmul_i8(ctx, p);
        if (e == cudaSuccess) e = qkv_split_rope_append(ctx, tmp, a.T, q);
        cudaFreeAsync(tmp, ctx.stream);
        cuda_check(e, "qkv_rope_append launch");
    }
    st.finish();
    acc.bytes_read = static_cast<uint64_t>(a.T) * a.K + static_cast<uint64_t>(a.K) * N;
    acc.bytes_written = 4 * n * sizeof(float);
    acc.flops = 2ull * a.T * a.K * N;
    acc.dma = st.staged_bytes();
}

// C = R + MATMUL_I8(A, B): the GEMV epilogue for one row, else MATMUL_I8
// then ADD_F32's addition.
void exec_matmul_i8_residual(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags,
                             const LaunchCtx &ctx, Accounting &acc) {
    vnpu_b200_matmul_i8_residual_args_t a;
    std::memcpy(&a, cmd.args.raw, sizeof(a));
    vnpu_packed_weights_t *w = a.B;
    if (!a.A || !w || !a.R || !a.C || !a.M || !a.K || !a.N)
        throw CommandError("invalid matmul_i8_residual arguments", VNPU_ERR_INVALID_ARGUMENT);
    if (w->K != a.K || w->N != a.N) throw CommandError("packed weight shape mismatch");
    if (w->device != s->device) throw CommandError("packed weights belong to another device");
    const uint32_t lda = a.lda ? a.lda : a.K;
    const uint32_t ldr = a.ldr ? a.ldr : a.N;
    const uint32_t ldc = a.ldc ? a.ldc : a.N;
    if (lda < a.K || ldr < a.N || ldc < a.N)
        throw CommandError("invalid matmul_i8_residual leading dimensions",
                           VNPU_ERR_INVALID_ARGUMENT);
    if (a.M > 1 && (ldr != a.N || ldc != a.N))
        throw CommandError("matmul_i8_residual with M > 1 needs dense R and C",
                           VNPU_ERR_UNSUPPORTED);
    Staging st(s);
    MatmulI8 p;
    p.A = st.in(a.A, static_cast<uint64_t>(a.M - 1) * lda + a.K);
    p.lda = lda;
    p.Bt = w->bt;
    p.k_stride = w->k_stride;
    p.scale_a = st.in(a.scale_a, sizeof(float) * a.M);
    p.scale_b = w->scales;
    p.bias = st.in(a.bias, sizeof(float) * a.N);
    const uint64_t r_span = (static_cast<uint64_t>(a.M - 1) * ldr + a.N) * sizeof(float);
    const uint64_t c_span = (static_cast<uint64_t>(a.M - 1) * ldc + a.N) * sizeof(float);
    const float *R = st.in(a.R, r_span);
    p.C = st.out(a.C, c_span, ldc != a.N);
    p.ldc = ldc;
    p.M = a.M;
    p.K = a.K;
    p.N = a.N;
    p.epilogue = a.epilogue;
    p.fmap = i8_form_map(s->device, VNPU_UNIT_AUTO, flags, a.M, a.K, a.N, a.bias != nullptr,
                         a.epilogue);
    p.tmap_b = w->tmap_ok ? &w->tmap : nullptr;
    p.tmap_b128 = w->tmap128_ok ? &w->tmap128 : nullptr;
    const AdvancePosition adv(cmd, st);
    bool advanced = false;
    if (a.M == 1) {
        // the GEMV advances the position itself
        MatmulI8 f = p;
        f.advance_pos = adv.position;
        f.advance = adv.step;
        cuda_check(matmul_i8_gemv_residual(ctx, f, R, ldr), "matmul_i8_residual launch");
        advanced = true;
    } else {
        const uint64_t count = static_cast<uint64_t>(a.M) * a.N;
        const bool aliased = R < p.C + count && p.C < R + count;
        float *out = p.C;
        float *tmp = nullptr;
        if (aliased) {
            cuda_check(cudaMallocAsync(reinterpret_cast<void **>(&tmp), count * sizeof(float),
                                       ctx.stream),
                       "residual scratch");
            p.C = tmp;
        }
        cudaError_t e = cudaErrorNotSupported;
        if (!aliased) {
            // split-K shapes add R in the finish kernel
            MatmulI8 f = p;
            f.R = R;
            f.ldr = ldr;
            e = matmul_i8_split_residual(ctx, f);
        }
        if (e == cudaErrorNotSupported) {
            e = matmul_i8(ctx, p);
            if (e == cudaSuccess) e = add(ctx, R, p.C, out, count, 1.0f, 1.0f);
        }
        if (tmp) cudaFreeAsync(tmp, ctx.stream);
        cuda_check(e, "matmul_i8_residual launch");
    }
    if (adv.position && !advanced)
        cuda_check(block_position(ctx, adv.position, adv.step, true), "position advance");
    st.finish();
    acc.bytes_read = static_cast<uint64_t>(a.M) * a.K + static_cast<uint64_t>(a.K) * a.N +
                     static_cast<uint64_t>(a.M) * a.N * sizeof(float);
    acc.bytes_written = static_cast<uint64_t>(a.M) * a.N * sizeof(float);
    acc.flops = 2ull * a.M * a.K * a.N;
    acc.dma = st.staged_bytes();
}

void exec_swiglu(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                 Accounting &acc) {
    const auto &a = cmd.args.swiglu;
    if (!a.gate || !a.up || !a.Y || !a.count) throw CommandError("invalid swiglu arguments");
    const uint64_t bytes = a.count * sizeof(float);
    Staging st(s);
    float *Y = st.out(a.Y, bytes, a.Y == a.gate || a.Y == a.up);
    const float *G = st.in(a.gate, bytes);
    const float *U = st.in(a.up, bytes);
    cuda_check(swiglu(ctx, G, U, Y, a.count, a.alpha == 0.0f ? 1.0f : a.alpha), "swiglu launch");
    st.finish();
    acc.bytes_read = a.count * 2 * sizeof(float);
    acc.bytes_written = bytes;
    acc.flops = a.count * 8;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:566-581 (ADD only; MUL is not on the block's path)
void exec_add(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
              Accounting &acc) {
    const auto &a = cmd.args.binary;
    if (!a.A || !a.B || !a.Y || !a.count) throw CommandError("invalid binary arguments");
    const bool dflt = a.alpha == 0.0f && a.beta == 0.0f;
    const uint64_t bytes = a.count * sizeof(float);
    Staging st(s);
    float *Y = st.out(a.Y, bytes, a.Y == a.A || a.Y == a.B);
    const float *A = st.in(a.A, bytes);
    const float *B = st.in(a.B, bytes);
    cuda_check(add(ctx, A, B, Y, a.count, dflt ? 1.0f : a.alpha, dflt ? 1.0f : a.beta),
               "add launch");
    st.finish();
    acc.bytes_read = a.count * 2 * sizeof(float);
    acc.bytes_written = bytes;
    acc.flops = a.count * 3;
    acc.dma = st.staged_bytes();
}

// src/core/scheduler.cpp:583-608
void exec_attention(vnpu_stream_t *s, const vnpu_command_t &cmd, const LaunchCtx &ctx,
                    Accounting &acc) {
    const auto &a = cmd.args.attention;
    if (!a.Q || !a.K || !a.V || !a.O || !a.batch || !a.heads || !a.seq_q || !a.seq_k ||
        !a.head_dim)
        throw CommandError("invalid attention arguments");
    if (a.head_dim > 256)
        throw CommandError("attention head_dim above 256", VNPU_ERR_UNSUPPORTED);
    const uint64_t bh = static_cast<uint64_t>(a.batch) * a.heads;
    const uint64_t qn = bh * a.seq_q * a.head_dim;
    const uint64_t kn = bh * a.seq_k * a.head_dim;
    const uint64_t mn = a.mask ? bh * a.seq_q * a.seq_k : 0;
    const float scale =
        a.scale > 0.0f ? a.scale : 1.0f / std::sqrt(static_cast<float>(a.head_dim));
    Staging st(s);
    float *O = st.out(a.O, qn * sizeof(float), false);
    const float *Q = st.in(a.Q, qn * sizeof(float));
    const float *K = st.in(a.K, kn * sizeof(float));
    const float *V = st.in(a.V, kn * sizeof(float));
    const float *M = st.in(a.mask, mn * sizeof(float));
    cuda_check(attention(ctx, Q, K, V, M, O, a.batch, a.heads, a.seq_q, a.seq_k, a.head_dim,
                         a.causal, scale, (cmd.flags & VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR) != 0u),
               "attention launch");
    st.finish();
    acc.bytes_read = (qn + 2 * kn + mn) * sizeof(float);
    acc.bytes_written = qn * sizeof(float);
    acc.flops = 4ull * bh * a.seq_q * a.seq_k * a.head_dim;
    acc.dma = st.staged_bytes();
}

void exec_copy(vnpu_stream_t *s, const vnpu_command_t &cmd, Accounting &acc) {
    const auto &a = cmd.args.copy;
    if (!a.dst || !a.src || !a.bytes) throw CommandError("invalid copy arguments");
    // Unified addressing tells the two sides apart; `direction` is advisory.
    // Host bytes a pending download writes are read or overwritten in order.
    join_downloads(s);
    cuda_check(cudaMemcpyAsync(a.dst, a.src, a.bytes, cudaMemcpyDefault, s->cs), "copy");
    if (classify(a.dst, s->device->ordinal) == Mem::kHost) s->cs_wrote_host = true;
    acc.bytes_read = a.bytes;
    acc.bytes_written = a.bytes;
    acc.dma = a.bytes;
}

void exec_memset(vnpu_stream_t *s, const vnpu_command_t &cmd, Accounting &acc) {
    const auto &a = cmd.args.memset;
    if (!a.dst || !a.bytes) throw CommandError("invalid memset arguments");
    if (s->capturing && classify(a.dst, s->device->ordinal) != Mem::kDevice)
        throw CommandError("host memset inside a graph capture", VNPU_ERR_INVALID_ARGUMENT);
    if (classify(a.dst, s->device->ordinal) == Mem::kDevice) {
        cuda_check(cudaMemsetAsync(a.dst, static_cast<int>(a.value & 0xffu), a.bytes, s->cs),
                   "memset");
    } else {
        // Host destination: keep stream order, then fill on the host.
        join_downloads(s);
        cuda_check(cudaStreamSynchronize(s->cs), "memset order");
        std::memset(a.dst, static_cast<int>(a.value & 0xffu), a.bytes);
    }
    acc.bytes_written = a.bytes;
    acc.dma = a.bytes;
}

void exec_pack(vnpu_stream_t *s, const vnpu_command_t &cmd, Accounting &acc) {
    const auto &a = cmd.args.pack_weights_i8;
    if (!a.B || !a.out || !a.K || !a.N) throw CommandError("invalid pack_weights arguments");
    if (s->capturing)
        throw CommandError("PACK_WEIGHTS_I8 inside a graph capture", VNPU_ERR_INVALID_ARGUMENT);
    // Stream order: everything before this command must have produced B.
    join_downloads(s);
    cuda_check(cudaStreamSynchronize(s->cs), "pack order");
    vnpu_packed_weights_t *w = nullptr;
    const vnpu_status_t rc =
        vnpu_pack_weights_i8(s->device, a.B, a.scales, a.K, a.N, a.ldb, a.trans_b, &w);
    if (rc != VNPU_OK) throw CommandError("pack_weights failed", rc);
    *a.out = w;
    acc.bytes_read = static_cast<uint64_t>(a.K) * a.N * 2;
    acc.bytes_written = static_cast<uint64_t>(w->k_stride) * a.N;
    acc.dma = static_cast<uint64_t>(a.K) * a.N * 2;
}

const char *opcode_name(uint32_t op);

vnpu_status_t execute_command(vnpu_stream_t *s, const vnpu_command_t &cmd, uint32_t flags) {
    vnpu_device_t *dev = s->device;
    if (cmd.opcode >= VNPU_OP_COUNT && cmd.opcode != VNPU_B200_OP_RMSNORM_QUANTIZE_I8 &&
        cmd.opcode != VNPU_B200_OP_SWIGLU_QUANTIZE_I8 && cmd.opcode != VNPU_B200_OP_KV_APPEND &&
        cmd.opcode != VNPU_B200_OP_MATMUL_I8_SCATTER &&
        cmd.opcode != VNPU_B200_OP_QKV_ROPE_APPEND && cmd.opcode != VNPU_B200_OP_MATMUL_I8_RESIDUAL &&
        cmd.opcode != VNPU_B200_OP_MATMUL_I8_SHARD && cmd.opcode != VNPU_B200_OP_MATMUL_I8_SWIGLU)
        return VNPU_ERR_INVALID_COMMAND;
    dev->last_opcode.store(cmd.opcode);
    const bool tracing = dev->trace.enabled.load();
    PendingTrace pt;
    uint32_t category = 0;
    if (cmd.opcode == VNPU_OP_COPY || cmd.opcode == VNPU_OP_MEMSET ||
        cmd.opcode == VNPU_OP_PACK_WEIGHTS_I8)
        category = 1;
    else if (cmd.opcode == VNPU_OP_BARRIER || cmd.opcode == VNPU_OP_NOP)
        category = 2;
    if (tracing && !s->capturing) {
        pt.ev.name = std::string(opcode_name(cmd.opcode)) + "#" + std::to_string(cmd.id);
        pt.ev.opcode = cmd.opcode;
        pt.ev.unit = cmd.opcode == VNPU_OP_MATMUL_I8 ? VNPU_UNIT_GPU : VNPU_UNIT_GPU;
        pt.ev.category = category;
        pt.ev.start_ns = now_ns();
        cudaEventCreate(&pt.begin);
        cudaEventCreate(&pt.end);
        cudaEventRecord(pt.begin, s->cs);
    }
    const uint64_t t0 = now_ns();
    uint64_t launched = 0;
    const LaunchCtx ctx = make_ctx(s, &launched);
    Accounting acc;
    const vnpu_status_t rc = guard([&]() -> vnpu_status_t {
        switch (cmd.opcode) {
        case VNPU_OP_NOP:
        case VNPU_OP_BARRIER: break;
        case VNPU_OP_MATMUL_I8: exec_matmul_i8(s, cmd, flags, ctx, acc); break;
        case VNPU_OP_MATMUL_F32: exec_matmul_f32(s, cmd, flags, ctx, acc); break;
        case VNPU_OP_QUANTIZE_I8: exec_quantize_i8(s, cmd, ctx, acc); break;
        case VNPU_OP_RMSNORM_F32: exec_rmsnorm(s, cmd, ctx, acc); break;
        case VNPU_OP_ROPE_F32: exec_rope(s, cmd, ctx, acc); break;
        case VNPU_OP_SWIGLU_F32: exec_swiglu(s, cmd, ctx, acc); break;
        case VNPU_OP_ADD_F32: exec_add(s, cmd, ctx, acc); break;
        case VNPU_OP_ATTENTION_F32: exec_attention(s, cmd, ctx, acc); break;
        case VNPU_OP_COPY: exec_copy(s, cmd, acc); break;
        case VNPU_B200_OP_RMSNORM_QUANTIZE_I8: exec_rmsnorm_quantize(s, cmd, ctx, acc); break;
        case VNPU_B200_OP_SWIGLU_QUANTIZE_I8: exec_swiglu_quantize(s, cmd, ctx, acc); break;
        case VNPU_B200_OP_KV_APPEND: exec_kv_append(s, cmd, ctx, acc); break;
        case VNPU_B200_OP_MATMUL_I8_SCATTER: exec_matmul_i8_scatter(s, cmd, flags, ctx, acc); break;
        case VNPU_B200_OP_QKV_ROPE_APPEND: exec_qkv_rope_append(s, cmd, flags, ctx, acc); break;
        case VNPU_B200_OP_MATMUL_I8_RESIDUAL: exec_matmul_i8_residual(s, cmd, flags, ctx, acc); break;
        case VNPU_B200_OP_MATMUL_I8_SHARD: exec_matmul_i8_shard(s, cmd, flags, ctx, acc); break;
        case VNPU_B200_OP_MATMUL_I8_SWIGLU: exec_matmul_i8_swiglu(s, cmd, flags, ctx, acc); break;
        case VNPU_OP_MEMSET: exec_memset(s, cmd, acc); break;
        case VNPU_OP_PACK_WEIGHTS_I8: exec_pack(s, cmd, acc); break;
        default:
            // SOFTMAX, GELU, MUL, MTP_HEAD: outside the int8 hot path this
            // backend implements.
            return VNPU_ERR_UNSUPPORTED;
        }
        return VNPU_OK;
    });
    const uint64_t host_ns = now_ns() - t0;
    if (s->capturing)
        s->captured_launches += launched;  // counted when the graph is replayed
    else
        dev->launches.fetch_add(launched);
    dev->dispatch_ns.fetch_add(host_ns);
    if (category == 1) dev->memory_ns.fetch_add(host_ns);
    dev->bytes_read.fetch_add(acc.bytes_read);
    dev->bytes_written.fetch_add(acc.bytes_written);
    dev->flops.fetch_add(acc.flops);
    dev->tiles_dispatched.fetch_add(acc.tiles);
    dev->dma_bytes.fetch_add(acc.dma);
    if (tracing && !s->capturing) {
        cudaEventRecord(pt.end, s->cs);
        pt.ev.bytes_read = acc.bytes_read;
        pt.ev.bytes_written = acc.bytes_written;
        pt.ev.flops = acc.flops;
        if (rc == VNPU_OK) {
            s->traces.push_back(pt);
        } else {
            cudaEventDestroy(pt.begin);
            cudaEventDestroy(pt.end);
        }
    }
    return rc;
}

// Resolve traced commands of a synchronised stream into trace events.
void drain_traces(vnpu_stream_t *s) {
    for (auto &pt : s->traces) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, pt.begin, pt.end) == cudaSuccess) {
            pt.ev.dur_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1e6);
            s->device->kernel_ns.fetch_add(pt.ev.dur_ns);
            s->device->trace.add(pt.ev);
        }
        cudaEventDestroy(pt.begin);
        cudaEventDestroy(pt.end);
    }
    s->traces.clear();
    cudaGetLastError();
}

// Read (and clear) the stream's device error word.
uint32_t take_device_error(vnpu_stream_t *s) {
    uint32_t h = 0;
    if (cudaMemcpyAsync(&h, s->d_err, sizeof(h), cudaMemcpyDeviceToHost, s->device->aux) !=
            cudaSuccess ||
        cudaStreamSynchronize(s->device->aux) != cudaSuccess) {
        cudaGetLastError();
        return kErrBadConfig;
    }
    if (h) {
        cudaMemsetAsync(s->d_err, 0, sizeof(uint32_t), s->device->aux);
        cudaStreamSynchronize(s->device->aux);
    }
    return h;
}

void record_stream_error(vnpu_stream_t *s, vnpu_status_t rc) {
    const uint32_t code = static_cast<uint32_t>(-static_cast<int32_t>(rc));
    s->last_error.store(code);
    s->device->error.store(code);
    s->device->regs[VNPU_REG_ERROR / 4].store(code);
}

vnpu_status_t stream_sync_impl(vnpu_stream_t *s) {
    const uint64_t t0 = now_ns();
    cudaSetDevice(s->device->ordinal);
    cudaError_t e = cudaStreamSynchronize(s->cs);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->down);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->up);
    s->pending_down.clear();
    s->cs_wrote_host = false;
    if (e != cudaSuccess) {
        debug_log("stream sync: %s", cudaGetErrorString(e));
        record_stream_error(s, VNPU_ERR_DEVICE_ERROR);
    } else if (take_device_error(s)) {
        record_stream_error(s, VNPU_ERR_DEVICE_ERROR);
    }
    drain_traces(s);
    const uint64_t done = s->pending.exchange(0);
    s->device->commands_completed.fetch_add(done);
    s->device->regs[VNPU_REG_CMD_HEAD / 4].store(
        static_cast<uint32_t>(s->device->commands_completed.load()));
    s->device->sync_ns.fetch_add(now_ns() - t0);
    return s->last_error.load() ? VNPU_ERR_DEVICE_ERROR : VNPU_OK;
}

const char *opcode_name(uint32_t op) {
    static const char *names[] = {"NOP",           "MATMUL_F32",   "MATMUL_I8",
                                  "RMSNORM_F32",   "SOFTMAX_F32",  "ROPE_F32",
                                  "SWIGLU_F32",    "GELU_F32",     "ADD_F32",
                                  "MUL_F32",       "ATTENTION_F32", "QUANTIZE_I8",
                                  "PACK_WEIGHTS_I8", "MTP_HEAD_F32", "COPY",
                                  "MEMSET",        "BARRIER"};
    if (op == VNPU_B200_OP_RMSNORM_QUANTIZE_I8) return "RMSNORM_QUANTIZE_I8";
    if (op == VNPU_B200_OP_SWIGLU_QUANTIZE_I8) return "SWIGLU_QUANTIZE_I8";
    if (op == VNPU_B200_OP_KV_APPEND) return "KV_APPEND";
    if (op == VNPU_B200_OP_MATMUL_I8_SCATTER) return "MATMUL_I8_SCATTER";
    if (op == VNPU_B200_OP_QKV_ROPE_APPEND) return "QKV_ROPE_APPEND";
    if (op == VNPU_B200_OP_MATMUL_I8_RESIDUAL) return "MATMUL_I8_RESIDUAL";
    if (op == VNPU_B200_OP_MATMUL_I8_SHARD) return "MATMUL_I8_SHARD";
    if (op == VNPU_B200_OP_MATMUL_I8_SWIGLU) return "MATMUL_I8_SWIGLU";
    return op < sizeof(names) / sizeof(names[0]) ? names[op] : "UNKNOWN";
}

}  // namespace

// ---------------------------------------------------------------------------
// Trace state
// ---------------------------------------------------------------------------
void TraceState::reset() {
    std::lock_guard<std::mutex> l(mutex);
    events.clear();
}

void TraceState::add(const TraceEvent &ev) {
    std::lock_guard<std::mutex> l(mutex);
    if (events.size() < kMaxEvents) events.push_back(ev);
}

void TraceState::summary(vnpu_trace_summary_t *out) {
    std::lock_guard<std::mutex> l(mutex);
    std::memset(out, 0, sizeof(*out));
    uint64_t per_op[VNPU_OP_COUNT] = {};
    for (const auto &e : events) {
        out->events++;
        out->total_time_ns += e.dur_ns;
        if (e.category == 1) out->memory_time_ns += e.dur_ns;
        else if (e.category == 2) out->sync_time_ns += e.dur_ns;
        else out->compute_time_ns += e.dur_ns;
        out->bytes_read += e.bytes_read;
        out->bytes_written += e.bytes_written;
        out->flops += e.flops;
        if (e.opcode < VNPU_OP_COUNT) per_op[e.opcode] += e.dur_ns;
    }
    for (uint32_t o = 0; o < VNPU_OP_COUNT; ++o)
        if (per_op[o] > out->hot_time_ns) {
            out->hot_time_ns = per_op[o];
            out->hot_opcode = o;
        }
    if (out->total_time_ns) {
        const double sec = static_cast<double>(out->total_time_ns) * 1e-9;
        out->achieved_gflops = static_cast<double>(out->flops) / sec * 1e-9;
        out->achieved_gbytes_s =
            static_cast<double>(out->bytes_read + out->bytes_written) / sec * 1e-9;
    }
}

vnpu_status_t TraceState::dump_text(const char *path) {
    vnpu_trace_summary_t s;
    summary(&s);
    FILE *f = path && path[0] ? std::fopen(path, "w") : stderr;
    if (!f) return VNPU_ERR_IO;
    std::fprintf(f, "vnpu-b200 trace: %llu events, %.3f ms device time\n",
                 static_cast<unsigned long long>(s.events), s.total_time_ns * 1e-6);
    std::fprintf(f, "  compute %.3f ms, memory %.3f ms, sync %.3f ms\n",
                 s.compute_time_ns * 1e-6, s.memory_time_ns * 1e-6, s.sync_time_ns * 1e-6);
    std::fprintf(f, "  %.1f GFLOP/s (int8 ops count as flops), %.1f GB/s\n", s.achieved_gflops,
                 s.achieved_gbytes_s);
    std::fprintf(f, "  hot opcode %s: %.3f ms\n", opcode_name(s.hot_opcode), s.hot_time_ns * 1e-6);
    {
        std::lock_guard<std::mutex> l(mutex);
        for (const auto &e : events)
            std::fprintf(f, "  %-24s %10.3f us  %12llu flops  %12llu B\n", e.name.c_str(),
                         e.dur_ns * 1e-3, static_cast<unsigned long long>(e.flops),
                         static_cast<unsigned long long>(e.bytes_read + e.bytes_written));
    }
    if (f != stderr) std::fclose(f);
    return VNPU_OK;
}

vnpu_status_t TraceState::write_chrome(const char *path) {
    FILE *f = std::fopen(path, "w");
    if (!f) return VNPU_ERR_IO;
    std::lock_guard<std::mutex> l(mutex);
    const uint64_t base = events.empty() ? 0 : events.front().start_ns;
    std::fprintf(f, "{\"traceEvents\":[\n");
    for (size_t i = 0; i < events.size(); ++i) {
        const auto &e = events[i];
        std::fprintf(f,
                     "{\"name\":\"%s\",\"cat\":\"%s\",\"ph\":\"X\",\"pid\":0,\"tid\":%u,"
                     "\"ts\":%.3f,\"dur\":%.3f,\"args\":{\"flops\":%llu,\"bytes\":%llu}}%s\n",
                     e.name.c_str(), e.category == 1 ? "memory" : (e.category == 2 ? "sync" : "compute"),
                     e.category, (e.start_ns - base) * 1e-3, e.dur_ns * 1e-3,
                     static_cast<unsigned long long>(e.flops),
                     static_cast<unsigned long long>(e.bytes_read + e.bytes_written),
                     i + 1 < events.size() ? "," : "");
    }
    std::fprintf(f, "]}\n");
    std::fclose(f);
    return VNPU_OK;
}

}  // namespace vnpu_b200

using namespace vnpu_b200;

void vnpu_device::raise_irq(uint32_t bits) {
    regs[VNPU_REG_IRQ_STATUS / 4].fetch_or(bits);
    interrupts.fetch_add(1);
    vnpu_interrupt_cb_t cb;
    void *user;
    {
        std::lock_guard<std::mutex> l(irq_mutex);
        cb = irq_cb;
        user = irq_user;
    }
    if (cb && (regs[VNPU_REG_IRQ_MASK / 4].load() & bits)) cb(this, bits, user);
}

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

VNPU_API void VNPU_CALL vnpu_config_init(vnpu_config_t *config) {
    if (!config) return;
    std::memset(config, 0, sizeof(*config));
    config->abi_version = VNPU_ABI_VERSION;
    if (const char *t = std::getenv("VNPU_THREADS")) config->num_threads = static_cast<uint32_t>(std::atoi(t));
    if (const char *t = std::getenv("VNPU_TRACE"))
        if (std::atoi(t)) config->flags |= VNPU_CONFIG_TRACE;
    if (const char *t = std::getenv("VNPU_TRACE_FILE")) config->trace_file = t;
}

VNPU_API const char *VNPU_CALL vnpu_status_string(vnpu_status_t status) {
    switch (status) {
    case VNPU_OK: return "OK";
    case VNPU_ERR_INVALID_ARGUMENT: return "invalid argument";
    case VNPU_ERR_OUT_OF_MEMORY: return "out of memory";
    case VNPU_ERR_UNSUPPORTED: return "unsupported";
    case VNPU_ERR_INVALID_COMMAND: return "invalid command";
    case VNPU_ERR_DEVICE_BUSY: return "device busy";
    case VNPU_ERR_DEVICE_ERROR: return "device error";
    case VNPU_ERR_TIMEOUT: return "timeout";
    case VNPU_ERR_NETWORK: return "network error";
    case VNPU_ERR_AUTH: return "authentication error";
    case VNPU_ERR_PROTOCOL: return "protocol error";
    case VNPU_ERR_NOT_FOUND: return "not found";
    case VNPU_ERR_IO: return "I/O error";
    default: return "internal error";
    }
}

VNPU_API const char *VNPU_CALL vnpu_version_string(void) { return "vnpu 1.0.0 (b200 sm_100a)"; }
VNPU_API uint32_t VNPU_CALL vnpu_abi_version(void) { return VNPU_ABI_VERSION; }
VNPU_API const char *VNPU_CALL vnpu_opcode_name(uint32_t opcode) { return opcode_name(opcode); }

VNPU_API const char *VNPU_CALL vnpu_unit_name(uint32_t unit) {
    switch (unit) {
    case VNPU_UNIT_AUTO: return "AUTO";
    case VNPU_UNIT_VOODOO: return "VOODOO";
    case VNPU_UNIT_WILDCAT: return "WILDCAT";
    case VNPU_UNIT_CELL: return "CELL";
    case VNPU_UNIT_GPU: return "GPU";
    default: return "UNKNOWN";
    }
}

// ---------------------------------------------------------------- devices
VNPU_API vnpu_status_t VNPU_CALL vnpu_device_create(const vnpu_config_t *config,
                                                    vnpu_device_t **out_device) {
    if (!out_device) return VNPU_ERR_INVALID_ARGUMENT;
    *out_device = nullptr;
    return guard([&]() -> vnpu_status_t {
        vnpu_config_t cfg;
        if (config) cfg = *config;
        else vnpu_config_init(&cfg);
        int ordinal = static_cast<int>(cfg.reserved0);
        if (const char *e = std::getenv("VNPU_CUDA_DEVICE")) ordinal = std::atoi(e);
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
            cudaGetLastError();
            debug_log("no CUDA device: the B200 backend has no CPU path");
            return VNPU_ERR_UNSUPPORTED;
        }
        if (ordinal < 0 || ordinal >= count) return VNPU_ERR_INVALID_ARGUMENT;
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, ordinal) != cudaSuccess) return VNPU_ERR_DEVICE_ERROR;
        if (prop.major != 10 || prop.minor != 0) {
            debug_log("device %d is sm_%d%d; this library is built for sm_100a only", ordinal,
                      prop.major, prop.minor);
            return VNPU_ERR_UNSUPPORTED;
        }
        if (cudaSetDevice(ordinal) != cudaSuccess) return VNPU_ERR_DEVICE_ERROR;
        auto *d = new vnpu_device_t();
        d->ordinal = ordinal;
        d->config = cfg;
        d->num_sms = prop.multiProcessorCount;
        d->epi_forced = epi_form_from_env(d->epi_form);
        // The reference device whose MATMUL_F32 results this one reproduces
        // (src/core/runtime.cpp:858-938).
        const bool ref_mode = env_is("VNPU_MODE", "reference");
        d->f32_scalar = ref_mode || env_is("VNPU_FORCE_ISA", "scalar") ||
                        (d->epi_forced && d->epi_form == kFormScalar);
        d->f32_pack = !ref_mode && !env_is("VNPU_PACK", "0");
        const uint32_t logical = std::max(1u, std::thread::hardware_concurrency());
        d->f32_threads = std::min(cfg.num_threads ? cfg.num_threads : host_physical_cores(),
                                  logical);
        {
            // as the reference reads it (src/core/runtime.cpp:174-179), 256 KiB
            // when unknown (src/internal.h:187)
            const long l2 = sysconf(_SC_LEVEL2_CACHE_SIZE);
            d->host_l2 = l2 > 0 ? static_cast<uint64_t>(l2) : 256u * 1024u;
        }
        if (cfg.tile_m && cfg.tile_k && cfg.tile_n) {
            d->f32_tile_m.store(cfg.tile_m);
            d->f32_tile_k.store(cfg.tile_k);
            d->f32_tile_n.store(cfg.tile_n);
        } else if (d->f32_scalar) {
            d->f32_tile_m.store(32);
            d->f32_tile_k.store(64);
            d->f32_tile_n.store(32);
        }
        if (const char *e = std::getenv("VNPU_B200_WAIT_LIMIT_MS"))
            d->wait_limit_ns = static_cast<uint64_t>(std::atoll(e)) * 1000000ull;
        if (cudaStreamCreateWithFlags(&d->aux, cudaStreamNonBlocking) != cudaSuccess) {
            delete d;
            return VNPU_ERR_DEVICE_ERROR;
        }
        // Keep stream-ordered staging allocations cached in the pool.
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
            uint64_t thr = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        d->name = cfg.node_name ? cfg.node_name : "vnpu0";
        auto &info = d->info;
        std::memset(&info, 0, sizeof(info));
        info.abi_version = VNPU_ABI_VERSION;
        std::snprintf(info.name, sizeof(info.name), "%s", d->name.c_str());
        std::snprintf(info.vendor, sizeof(info.vendor), "NVIDIA %.48s", prop.name);
        std::snprintf(info.cpu_arch, sizeof(info.cpu_arch), "sm_%d%da", prop.major, prop.minor);
        std::snprintf(info.backend, sizeof(info.backend), "CUDA sm_100a (tcgen05 int8)");
        info.simd_bits = 32 * 32;  // a warp of 32-bit lanes
        info.num_threads = static_cast<uint32_t>(prop.multiProcessorCount);
        info.num_compute_units = static_cast<uint32_t>(prop.multiProcessorCount);
        info.local_store_bytes = static_cast<uint32_t>(prop.sharedMemPerBlockOptin);
        info.tile_m = 128;
        info.tile_k = 128;
        info.tile_n = 256;
        info.physical_cores = static_cast<uint32_t>(prop.multiProcessorCount);
        info.features = VNPU_FEATURE_GPU_FUTURE | VNPU_FEATURE_THREADS | VNPU_FEATURE_TRACE;
        info.l1d_bytes = prop.sharedMemPerMultiprocessor;
        info.l2_bytes = static_cast<uint64_t>(prop.l2CacheSize);
        info.l3_bytes = 0;
        info.total_memory_bytes = prop.totalGlobalMem;
        for (auto &r : d->regs) r.store(0);
        d->regs[VNPU_REG_ID / 4].store(VNPU_MAGIC);
        d->regs[VNPU_REG_VERSION / 4].store(VNPU_ABI_VERSION);
        d->regs[VNPU_REG_CONTROL / 4].store(1);
        d->regs[VNPU_REG_STATUS / 4].store(1);
        d->regs[VNPU_REG_ACTIVE_CUS / 4].store(info.num_compute_units);
        d->regs[VNPU_REG_CLOCK_MHZ / 4].store(static_cast<uint32_t>(prop.clockRate / 1000));
        d->regs[VNPU_REG_FEATURE_LO / 4].store(static_cast<uint32_t>(info.features & 0xffffffffu));
        d->regs[VNPU_REG_FEATURE_HI / 4].store(static_cast<uint32_t>(info.features >> 32));
        d->regs[VNPU_REG_IRQ_MASK / 4].store(0xffffffffu);
        d->trace.enabled.store((cfg.flags & VNPU_CONFIG_TRACE) != 0);
        d->trace.trace_file = cfg.trace_file ? cfg.trace_file : "";
        debug_log("created %s on GPU %d (%s, %d SMs)", d->name.c_str(), ordinal, prop.name,
                  prop.multiProcessorCount);
        *out_device = d;
        return VNPU_OK;
    });
}

VNPU_API void VNPU_CALL vnpu_device_destroy(vnpu_device_t *device) {
    if (!device) return;
    std::vector<vnpu_stream_t *> streams;
    {
        std::lock_guard<std::mutex> l(device->stream_mutex);
        streams.swap(device->streams);
    }
    cudaSetDevice(device->ordinal);
    for (auto *s : streams) {
        stream_sync_impl(s);
        cudaStreamDestroy(s->cs);
        cudaStreamDestroy(s->up);
        cudaStreamDestroy(s->down);
        cudaFree(s->d_err);
        delete s;
    }
    if ((device->config.flags & VNPU_CONFIG_TRACE_CHROME) && !device->trace.trace_file.empty())
        device->trace.write_chrome(device->trace.trace_file.c_str());
    cudaStreamDestroy(device->aux);
    delete device;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_device_get_info(const vnpu_device_t *device,
                                                      vnpu_device_info_t *info) {
    if (!device || !info) return VNPU_ERR_INVALID_ARGUMENT;
    *info = device->info;
    info->tile_m = device->tile_m.load();
    info->tile_k = device->tile_k.load();
    info->tile_n = device->tile_n.load();
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_device_get_status(const vnpu_device_t *device,
                                                        vnpu_device_status_t *st) {
    if (!device || !st) return VNPU_ERR_INVALID_ARGUMENT;
    std::memset(st, 0, sizeof(*st));
    st->commands_submitted = device->commands_submitted.load();
    st->commands_completed = device->commands_completed.load();
    st->kernel_time_ns = device->kernel_ns.load();
    st->dispatch_time_ns = device->dispatch_ns.load();
    st->memory_time_ns = device->memory_ns.load();
    st->sync_time_ns = device->sync_ns.load();
    st->bytes_read = device->bytes_read.load();
    st->bytes_written = device->bytes_written.load();
    st->flops = device->flops.load();
    st->tiles_dispatched = device->tiles_dispatched.load();
    st->tiles_culled = device->tiles_culled.load();
    st->dma_bytes = device->dma_bytes.load();
    st->interrupts = device->interrupts.load();
    st->busy = device->busy.load();
    st->error = device->error.load();
    st->last_opcode = device->last_opcode.load();
    st->active_workers = device->busy.load();
    st->reserved[0] = device->launches.load();
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_device_reset(vnpu_device_t *device) {
    if (!device) return VNPU_ERR_INVALID_ARGUMENT;
    if (device->busy.load()) return VNPU_ERR_DEVICE_BUSY;
    device->commands_submitted.store(0);
    device->commands_completed.store(0);
    device->kernel_ns.store(0);
    device->dispatch_ns.store(0);
    device->memory_ns.store(0);
    device->sync_ns.store(0);
    device->bytes_read.store(0);
    device->bytes_written.store(0);
    device->flops.store(0);
    device->tiles_dispatched.store(0);
    device->tiles_culled.store(0);
    device->dma_bytes.store(0);
    device->interrupts.store(0);
    device->error.store(0);
    device->last_opcode.store(0);
    device->regs[VNPU_REG_ERROR / 4].store(0);
    device->regs[VNPU_REG_IRQ_STATUS / 4].store(0);
    device->trace.reset();
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_device_set_tiles(vnpu_device_t *device, uint32_t tile_m,
                                                       uint32_t tile_k, uint32_t tile_n) {
    if (!device || !tile_m || !tile_k || !tile_n) return VNPU_ERR_INVALID_ARGUMENT;
    // Recorded for callers that read them back; the GPU kernels keep their
    // fixed tensor-core tiles.
    device->tile_m.store(tile_m);
    device->tile_k.store(tile_k);
    device->tile_n.store(tile_n);
    device->f32_tile_m.store(tile_m);
    device->f32_tile_k.store(tile_k);
    device->f32_tile_n.store(tile_n);
    return VNPU_OK;
}

VNPU_API uint32_t VNPU_CALL vnpu_mmio_read32(vnpu_device_t *device, uint32_t offset) {
    if (!device || (offset & 3u)) return 0xffffffffu;
    const uint32_t idx = offset / 4;
    if (idx >= VNPU_REG_COUNT) return 0xffffffffu;
    switch (offset) {
    case VNPU_REG_STATUS: return 1u | (device->busy.load() ? 2u : 0u);
    case VNPU_REG_ERROR: return device->regs[idx].load() | (device->error.load() ? 1u : 0u);
    case VNPU_REG_CMD_HEAD: return static_cast<uint32_t>(device->commands_completed.load());
    case VNPU_REG_CMD_TAIL: return static_cast<uint32_t>(device->commands_submitted.load());
    case VNPU_REG_ACTIVE_CUS: return device->regs[idx].load();
    case VNPU_REG_THERMAL: return 0;
    default: return device->regs[idx].load();
    }
}

VNPU_API void VNPU_CALL vnpu_mmio_write32(vnpu_device_t *device, uint32_t offset,
                                          uint32_t value) {
    if (!device || (offset & 3u)) return;
    const uint32_t idx = offset / 4;
    if (idx >= VNPU_REG_COUNT) return;
    device->regs[idx].store(value);
    if (offset == VNPU_REG_DOORBELL && value) device->raise_irq(1u << 0);
    else if (offset == VNPU_REG_CONTROL && (value & 2u)) vnpu_device_reset(device);
    else if (offset == VNPU_REG_IRQ_STATUS) device->regs[idx].store(0);
}

VNPU_API void VNPU_CALL vnpu_device_set_interrupt_callback(vnpu_device_t *device,
                                                           vnpu_interrupt_cb_t cb,
                                                           void *user_data) {
    if (!device) return;
    std::lock_guard<std::mutex> l(device->irq_mutex);
    device->irq_cb = cb;
    device->irq_user = user_data;
}

// ---------------------------------------------------------------- streams
VNPU_API vnpu_status_t VNPU_CALL vnpu_stream_create(vnpu_device_t *device, int priority,
                                                    vnpu_stream_t **out_stream) {
    if (!device || !out_stream) return VNPU_ERR_INVALID_ARGUMENT;
    *out_stream = nullptr;
    return guard([&]() -> vnpu_status_t {
        cudaSetDevice(device->ordinal);
        auto *s = new vnpu_stream_t();
        s->device = device;
        s->priority = priority;
        int lo = 0, hi = 0;
        cudaDeviceGetStreamPriorityRange(&lo, &hi);
        // vnpu: larger priority = more urgent; CUDA: numerically lower.
        const int cuda_prio = priority > 0 ? hi : lo;
        if (cudaStreamCreateWithPriority(&s->cs, cudaStreamNonBlocking, cuda_prio) != cudaSuccess ||
            cudaStreamCreateWithFlags(&s->up, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&s->down, cudaStreamNonBlocking) != cudaSuccess ||
            cudaMalloc(&s->d_err, 3 * sizeof(uint32_t)) != cudaSuccess ||
            cudaMemset(s->d_err, 0, 3 * sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            if (s->cs) cudaStreamDestroy(s->cs);
            if (s->up) cudaStreamDestroy(s->up);
            if (s->down) cudaStreamDestroy(s->down);
            delete s;
            return VNPU_ERR_DEVICE_ERROR;
        }
        s->d_scratch = s->d_err + 1;
        s->d_flag = s->d_err + 2;
        std::lock_guard<std::mutex> l(device->stream_mutex);
        device->streams.push_back(s);
        *out_stream = s;
        return VNPU_OK;
    });
}

VNPU_API void VNPU_CALL vnpu_stream_destroy(vnpu_stream_t *stream) {
    if (!stream) return;
    vnpu_device_t *d = stream->device;
    {
        std::lock_guard<std::mutex> l(d->stream_mutex);
        auto &v = d->streams;
        v.erase(std::remove(v.begin(), v.end(), stream), v.end());
    }
    stream_sync_impl(stream);
    cudaStreamDestroy(stream->cs);
    cudaStreamDestroy(stream->up);
    cudaStreamDestroy(stream->down);
    cudaFree(stream->d_err);
    delete stream;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_stream_sync(vnpu_stream_t *stream) {
    if (!stream) return VNPU_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> l(stream->mutex);
    if (stream->capturing) return VNPU_ERR_DEVICE_BUSY;
    return stream_sync_impl(stream);
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_stream_submit(vnpu_stream_t *stream,
                                                    const vnpu_command_t *commands,
                                                    uint64_t count, vnpu_event_t *event) {
    if (!stream || (!commands && count) || count > (1u << 24)) return VNPU_ERR_INVALID_ARGUMENT;
    if (count == 0) {
        if (event) {
            std::lock_guard<std::mutex> l(event->mutex);
            event->host_signaled = true;
            event->recorded = false;
            event->status = VNPU_OK;
        }
        return VNPU_OK;
    }
    return guard([&]() -> vnpu_status_t {
        std::lock_guard<std::mutex> l(stream->mutex);
        vnpu_device_t *d = stream->device;
        cudaSetDevice(d->ordinal);
        uint32_t flags = 0;
        for (uint64_t i = 0; i < count; ++i) flags |= commands[i].flags;
        d->commands_submitted.fetch_add(count);
        d->regs[VNPU_REG_CMD_TAIL / 4].store(static_cast<uint32_t>(d->commands_submitted.load()));
        stream->pending.fetch_add(count);
        d->busy.fetch_add(1);
        vnpu_status_t batch = VNPU_OK;
        for (uint64_t i = 0; i < count; ++i) {
            const vnpu_status_t rc = execute_command(stream, commands[i], flags);
            if (rc != VNPU_OK) {
                batch = rc == VNPU_ERR_UNSUPPORTED ? rc : VNPU_ERR_INTERNAL;
                record_stream_error(stream, rc);
            }
        }
        d->busy.fetch_sub(1);
        d->raise_irq(1u << 1);
        if (event) {
            std::lock_guard<std::mutex> el(event->mutex);
            if (event->ev && event->ev_device != d->ordinal) {
                cudaEventDestroy(event->ev);
                event->ev = nullptr;
            }
            if (!event->ev) {
                if (cudaEventCreateWithFlags(&event->ev, cudaEventDisableTiming) != cudaSuccess)
                    return VNPU_ERR_DEVICE_ERROR;
                event->ev_device = d->ordinal;
            }
            // The batch is done when its kernels and its downloads are.
            if (!stream->pending_down.empty()) {
                stream_after(stream->down, stream->cs);
                cudaEventRecord(event->ev, stream->down);
            } else {
                cudaEventRecord(event->ev, stream->cs);
            }
            event->recorded = true;
            event->host_signaled = false;
            event->status = batch;
            event->stream = stream;
            event->command_count = count;
        }
        return VNPU_OK;
    });
}

// ---------------------------------------------------------------- events
VNPU_API vnpu_status_t VNPU_CALL vnpu_event_create(vnpu_event_t **out_event) {
    if (!out_event) return VNPU_ERR_INVALID_ARGUMENT;
    *out_event = nullptr;
    try {
        *out_event = new vnpu_event_t();
        return VNPU_OK;
    } catch (...) {
        return VNPU_ERR_OUT_OF_MEMORY;
    }
}

VNPU_API void VNPU_CALL vnpu_event_destroy(vnpu_event_t *event) {
    if (!event) return;
    if (event->ev) cudaEventDestroy(event->ev);
    delete event;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_event_wait(vnpu_event_t *event, uint32_t timeout_ms) {
    if (!event) return VNPU_ERR_INVALID_ARGUMENT;
    const uint64_t deadline = now_ns() + static_cast<uint64_t>(timeout_ms) * 1000000ull;
    for (;;) {
        {
            std::lock_guard<std::mutex> l(event->mutex);
            if (event->host_signaled) return event->status;
            if (event->recorded) {
                const cudaError_t q = cudaEventQuery(event->ev);
                if (q == cudaSuccess) {
                    vnpu_status_t st = event->status;
                    if (st == VNPU_OK && event->stream &&
                        take_device_error(event->stream)) {
                        record_stream_error(event->stream, VNPU_ERR_DEVICE_ERROR);
                        st = VNPU_ERR_DEVICE_ERROR;
                        event->status = st;
                    }
                    return st;
                }
                if (q != cudaErrorNotReady) {
                    cudaGetLastError();
                    return VNPU_ERR_DEVICE_ERROR;
                }
            }
        }
        if (now_ns() >= deadline) return VNPU_ERR_TIMEOUT;
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_event_query(const vnpu_event_t *event) {
    if (!event) return VNPU_ERR_INVALID_ARGUMENT;
    auto *e = const_cast<vnpu_event_t *>(event);
    std::lock_guard<std::mutex> l(e->mutex);
    if (e->host_signaled) return VNPU_OK;
    if (!e->recorded) return VNPU_ERR_DEVICE_BUSY;
    const cudaError_t q = cudaEventQuery(e->ev);
    if (q == cudaSuccess) return VNPU_OK;
    if (q != cudaErrorNotReady) cudaGetLastError();
    return VNPU_ERR_DEVICE_BUSY;
}

// ---------------------------------------------------------------- buffers
VNPU_API vnpu_status_t VNPU_CALL vnpu_buffer_alloc(vnpu_device_t *device, uint64_t bytes,
                                                   vnpu_buffer_t **out_buffer) {
    if (!device || !bytes || !out_buffer) return VNPU_ERR_INVALID_ARGUMENT;
    *out_buffer = nullptr;
    return guard([&]() -> vnpu_status_t {
        cudaSetDevice(device->ordinal);
        void *p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return VNPU_ERR_OUT_OF_MEMORY;
        }
        if (cudaMemset(p, 0, bytes) != cudaSuccess) {
            cudaFree(p);
            return VNPU_ERR_DEVICE_ERROR;
        }
        static std::atomic<uint64_t> next{1};
        auto *b = new vnpu_buffer_t();
        b->device = device;
        b->ptr = p;
        b->bytes = bytes;
        b->handle = next.fetch_add(1);
        *out_buffer = b;
        return VNPU_OK;
    });
}

VNPU_API void VNPU_CALL vnpu_buffer_free(vnpu_buffer_t *buffer) {
    if (!buffer) return;
    cudaSetDevice(buffer->device->ordinal);
    cudaFree(buffer->ptr);
    delete buffer;
}

// The address commands use for this buffer: an HBM address (unified
// addressing), reachable from the host only through COPY commands.
VNPU_API void *VNPU_CALL vnpu_buffer_host_ptr(vnpu_buffer_t *buffer) {
    return buffer ? buffer->ptr : nullptr;
}

VNPU_API uint64_t VNPU_CALL vnpu_buffer_size(const vnpu_buffer_t *buffer) {
    return buffer ? buffer->bytes : 0;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_buffer_copy(vnpu_stream_t *stream, void *dst,
                                                  const void *src, uint64_t bytes,
                                                  uint32_t direction) {
    if (!stream || !dst || !src || !bytes) return VNPU_ERR_INVALID_ARGUMENT;
    vnpu_command_t cmd{};
    cmd.opcode = VNPU_OP_COPY;
    cmd.args.copy.dst = dst;
    cmd.args.copy.src = src;
    cmd.args.copy.bytes = bytes;
    cmd.args.copy.direction = direction;
    const vnpu_status_t rc = vnpu_stream_submit(stream, &cmd, 1, nullptr);
    return rc != VNPU_OK ? rc : vnpu_stream_sync(stream);
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_buffer_memset(vnpu_stream_t *stream, void *dst,
                                                    uint32_t value, uint64_t bytes) {
    if (!stream || !dst || !bytes) return VNPU_ERR_INVALID_ARGUMENT;
    vnpu_command_t cmd{};
    cmd.opcode = VNPU_OP_MEMSET;
    cmd.args.memset.dst = dst;
    cmd.args.memset.value = value;
    cmd.args.memset.bytes = bytes;
    const vnpu_status_t rc = vnpu_stream_submit(stream, &cmd, 1, nullptr);
    return rc != VNPU_OK ? rc : vnpu_stream_sync(stream);
}

// ---------------------------------------------------------------- packed weights
// src/core/scheduler.cpp:763-836.  The K-major copy lives in HBM; scales and
// column sums are kept on both sides (vnpu_packed_weights_info hands out host
// pointers, as the reference does).
VNPU_API vnpu_status_t VNPU_CALL vnpu_pack_weights_i8(vnpu_device_t *device, const int8_t *B,
                                                      const float *scales, uint32_t K,
                                                      uint32_t N, uint32_t ldb,
                                                      uint32_t trans_b,
                                                      vnpu_packed_weights_t **out_weights) {
    if (!device || !B || !out_weights || !K || !N || trans_b > 1)
        return VNPU_ERR_INVALID_ARGUMENT;
    *out_weights = nullptr;
    const uint32_t ldb_eff = ldb ? ldb : (trans_b ? K : N);
    if (ldb_eff < (trans_b ? K : N)) return VNPU_ERR_INVALID_ARGUMENT;
    return guard([&]() -> vnpu_status_t {
        cudaSetDevice(device->ordinal);
        auto w = std::make_unique<vnpu_packed_weights_t>();
        w->device = device;
        w->K = K;
        w->N = N;
        w->k_stride = (K + 127u) & ~127u;
        const uint64_t bt_bytes = static_cast<uint64_t>(N) * w->k_stride;
        auto fail = [&](cudaError_t e) {
            cudaFree(w->bt);
            cudaFree(w->scales);
            cudaFree(w->column_sums);
            w->bt = nullptr;
            w->scales = nullptr;
            w->column_sums = nullptr;
            cudaGetLastError();
            return e == cudaErrorMemoryAllocation ? VNPU_ERR_OUT_OF_MEMORY : VNPU_ERR_DEVICE_ERROR;
        };
        cudaError_t e;
        if ((e = cudaMalloc(&w->bt, bt_bytes)) != cudaSuccess ||
            (e = cudaMalloc(&w->scales, sizeof(float) * ((N + 255u) & ~255u))) != cudaSuccess ||
            (e = cudaMalloc(&w->column_sums, sizeof(int32_t) * N)) != cudaSuccess)
            return fail(e);
        uint64_t launched = 0;
        LaunchCtx ctx;
        ctx.stream = device->aux;
        ctx.num_sms = device->num_sms;
        ctx.launch_counter = &launched;
        {
            Staging st(device->aux, device->ordinal);
            const uint64_t b_span = trans_b ? static_cast<uint64_t>(N - 1) * ldb_eff + K
                                            : static_cast<uint64_t>(K - 1) * ldb_eff + N;
            const int8_t *Bd = st.in(B, b_span);
            if ((e = pack_weights(ctx, Bd, K, N, ldb_eff, trans_b, w->bt, w->k_stride,
                                  w->column_sums)) != cudaSuccess)
                return fail(e);
            w->host_scales.assign(N, 1.0f);
            if (scales) {
                if (classify(scales, device->ordinal) == Mem::kDevice) {
                    e = cudaMemcpyAsync(w->host_scales.data(), scales, sizeof(float) * N,
                                        cudaMemcpyDeviceToHost, device->aux);
                    if (e == cudaSuccess) e = cudaStreamSynchronize(device->aux);
                } else {
                    std::memcpy(w->host_scales.data(), scales, sizeof(float) * N);
                }
                if (e != cudaSuccess) return fail(e);
            }
            // Scales are padded with 1.0 to a multiple of 256 so the epilogue's
            // 16-byte loads of a ragged last tile stay inside the allocation.
            std::vector<float> padded(w->host_scales);
            padded.resize((N + 255u) & ~255u, 1.0f);
            if ((e = cudaMemcpyAsync(w->scales, padded.data(), sizeof(float) * padded.size(),
                                     cudaMemcpyHostToDevice, device->aux)) != cudaSuccess)
                return fail(e);
            if ((e = cudaStreamSynchronize(device->aux)) != cudaSuccess) return fail(e);
            w->host_column_sums.resize(N);
            if ((e = cudaMemcpyAsync(w->host_column_sums.data(), w->column_sums,
                                     sizeof(int32_t) * N, cudaMemcpyDeviceToHost,
                                     device->aux)) != cudaSuccess)
                return fail(e);
        }
        if ((e = cudaStreamSynchronize(device->aux)) != cudaSuccess) return fail(e);
        device->launches.fetch_add(launched);
        w->tmap_ok = encode_tmap_kmajor_i8(&w->tmap, w->bt, w->k_stride, N, w->k_stride, 128, 256);
        w->tmap128_ok =
            encode_tmap_kmajor_i8(&w->tmap128, w->bt, w->k_stride, N, w->k_stride, 128, 128);
        device->dma_bytes.fetch_add(static_cast<uint64_t>(K) * N * 2);
        *out_weights = w.release();
        return VNPU_OK;
    });
}

VNPU_API void VNPU_CALL vnpu_packed_weights_destroy(vnpu_packed_weights_t *w) {
    if (!w) return;
    cudaSetDevice(w->device->ordinal);
    cudaFree(w->bt);
    cudaFree(w->scales);
    cudaFree(w->column_sums);
    delete w;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_packed_weights_info(const vnpu_packed_weights_t *w,
                                                          uint32_t *K, uint32_t *N,
                                                          uint64_t *bytes, const float **scales,
                                                          const int32_t **column_sums) {
    if (!w) return VNPU_ERR_INVALID_ARGUMENT;
    if (K) *K = w->K;
    if (N) *N = w->N;
    if (bytes) *bytes = static_cast<uint64_t>(w->N) * w->k_stride;
    if (scales) *scales = w->host_scales.data();
    if (column_sums) *column_sums = w->host_column_sums.data();
    return VNPU_OK;
}

// ---------------------------------------------------------------- sync wrappers
#define VNPU_B200_SYNC_WRAPPER(fn, op, field, type)                               \
    VNPU_API vnpu_status_t VNPU_CALL fn(vnpu_stream_t *stream, const type *args) { \
        if (!stream || !args) return VNPU_ERR_INVALID_ARGUMENT;                    \
        vnpu_command_t cmd{};                                                      \
        cmd.opcode = op;                                                           \
        cmd.args.field = *args;                                                    \
        const vnpu_status_t rc = vnpu_stream_submit(stream, &cmd, 1, nullptr);     \
        return rc != VNPU_OK ? rc : vnpu_stream_sync(stream);                      \
    }

VNPU_B200_SYNC_WRAPPER(vnpu_matmul_f32, VNPU_OP_MATMUL_F32, matmul_f32, vnpu_matmul_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_matmul_i8, VNPU_OP_MATMUL_I8, matmul_i8, vnpu_matmul_i8_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_quantize_i8, VNPU_OP_QUANTIZE_I8, quantize_i8, vnpu_quantize_i8_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_rmsnorm_f32, VNPU_OP_RMSNORM_F32, rmsnorm, vnpu_rmsnorm_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_softmax_f32, VNPU_OP_SOFTMAX_F32, softmax, vnpu_softmax_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_rope_f32, VNPU_OP_ROPE_F32, rope, vnpu_rope_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_swiglu_f32, VNPU_OP_SWIGLU_F32, swiglu, vnpu_swiglu_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_gelu_f32, VNPU_OP_GELU_F32, unary, vnpu_unary_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_add_f32, VNPU_OP_ADD_F32, binary, vnpu_binary_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_mul_f32, VNPU_OP_MUL_F32, binary, vnpu_binary_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_attention_f32, VNPU_OP_ATTENTION_F32, attention, vnpu_attention_f32_args_t)
VNPU_B200_SYNC_WRAPPER(vnpu_mtp_head_f32, VNPU_OP_MTP_HEAD_F32, mtp_head, vnpu_mtp_head_f32_args_t)

#undef VNPU_B200_SYNC_WRAPPER

// ---------------------------------------------------------------- tracing
VNPU_API vnpu_status_t VNPU_CALL vnpu_trace_enable(vnpu_device_t *device, int enable) {
    if (!device) return VNPU_ERR_INVALID_ARGUMENT;
    device->trace.enabled.store(enable != 0);
    if (enable) device->trace.reset();
    return VNPU_OK;
}

VNPU_API void VNPU_CALL vnpu_trace_reset(vnpu_device_t *device) {
    if (device) device->trace.reset();
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_trace_get_summary(const vnpu_device_t *device,
                                                        vnpu_trace_summary_t *summary) {
    if (!device || !summary) return VNPU_ERR_INVALID_ARGUMENT;
    const_cast<vnpu_device_t *>(device)->trace.summary(summary);
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_trace_dump(const vnpu_device_t *device, const char *path) {
    if (!device) return VNPU_ERR_INVALID_ARGUMENT;
    return const_cast<vnpu_device_t *>(device)->trace.dump_text(path);
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_trace_write_chrome(const vnpu_device_t *device,
                                                         const char *path) {
    if (!device || !path) return VNPU_ERR_INVALID_ARGUMENT;
    return const_cast<vnpu_device_t *>(device)->trace.write_chrome(path);
}

// ---------------------------------------------------------------- B200 extensions
VNPU_API void *VNPU_CALL vnpu_b200_stream_handle(vnpu_stream_t *stream) {
    return stream ? static_cast<void *>(stream->cs) : nullptr;
}

VNPU_API int VNPU_CALL vnpu_b200_device_ordinal(const vnpu_device_t *device) {
    return device ? device->ordinal : -1;
}

VNPU_API uint64_t VNPU_CALL vnpu_b200_kernel_launches(const vnpu_device_t *device) {
    return device ? device->launches.load() : 0;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_reference_model(const vnpu_device_t *device,
                                                          vnpu_b200_reference_model_t *out) {
    if (!device || !out) return VNPU_ERR_INVALID_ARGUMENT;
    std::memset(out, 0, sizeof(*out));
    out->num_threads = device->f32_threads;
    out->tile_m = device->f32_tile_m.load();
    out->tile_k = device->f32_tile_k.load();
    out->tile_n = device->f32_tile_n.load();
    out->pack_b = device->f32_pack ? 1u : 0u;
    out->scalar_isa = device->f32_scalar ? 1u : 0u;
    out->l2_bytes = device->host_l2;
    out->epilogue_forced = device->epi_forced ? 1u : 0u;
    out->epilogue_form = device->epi_form;
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_packed_weights_device(
    const vnpu_packed_weights_t *w, const int8_t **bt, uint32_t *k_stride,
    const float **scales) {
    if (!w) return VNPU_ERR_INVALID_ARGUMENT;
    if (bt) *bt = w->bt;
    if (k_stride) *k_stride = w->k_stride;
    if (scales) *scales = w->scales;
    return VNPU_OK;
}

VNPU_API const char *VNPU_CALL vnpu_b200_matmul_i8_kernel(uint32_t M, uint32_t K, uint32_t N,
                                                         uint32_t lda, const void *A) {
    return matmul_kernel_name(choose_matmul_kernel(M, K, N, lda ? lda : K, A));
}

VNPU_API const char *VNPU_CALL vnpu_b200_last_matmul_kernel(void) { return last_matmul_kernel(); }

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_get_handle(const void *device_ptr,
                                                         uint8_t handle[64]) {
    if (!device_ptr || !handle) return VNPU_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void *>(device_ptr)) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    std::memcpy(handle, &h, sizeof(h));
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_open(int device, const uint8_t handle[64],
                                                   void **out_ptr) {
    if (!handle || !out_ptr) return VNPU_ERR_INVALID_ARGUMENT;
    *out_ptr = nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *out_ptr = nullptr;
        return VNPU_ERR_DEVICE_ERROR;
    }
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_ipc_close(void *ptr) {
    if (!ptr) return VNPU_ERR_INVALID_ARGUMENT;
    if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_DEVICE_ERROR;
    }
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_selftest_wait_timeout(vnpu_stream_t *stream,
                                                                uint32_t timeout_us) {
    if (!stream || !timeout_us || timeout_us > 10000000u) return VNPU_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> l(stream->mutex);
    cudaSetDevice(stream->device->ordinal);
    vnpu_status_t rc = stream_sync_impl(stream);
    if (rc != VNPU_OK) return rc;
    uint64_t launched = 0;
    const LaunchCtx ctx = make_ctx(stream, &launched);
    if (wait_timeout_probe(ctx, stream->d_flag, static_cast<uint64_t>(timeout_us) * 1000ull) !=
        cudaSuccess)
        return VNPU_ERR_DEVICE_ERROR;
    stream->device->launches.fetch_add(launched);
    if (cudaStreamSynchronize(stream->cs) != cudaSuccess) return VNPU_ERR_DEVICE_ERROR;
    const uint32_t err = take_device_error(stream);
    return (err & kErrWaitTimeout) ? VNPU_ERR_TIMEOUT : (err ? VNPU_ERR_DEVICE_ERROR : VNPU_OK);
}

// ---------------------------------------------------------------- graph capture
VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_capture_begin(vnpu_stream_t *stream) {
    if (!stream) return VNPU_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> l(stream->mutex);
    if (stream->capturing) return VNPU_ERR_DEVICE_BUSY;
    cudaSetDevice(stream->device->ordinal);
    // Work already queued must not be captured: let it finish first.
    const vnpu_status_t rc = stream_sync_impl(stream);
    if (rc != VNPU_OK) return rc;
    if (cudaStreamBeginCapture(stream->cs, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_DEVICE_ERROR;
    }
    stream->capturing = true;
    stream->captured_launches = 0;
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_capture_end(vnpu_stream_t *stream,
                                                      vnpu_b200_graph_t **out_graph) {
    if (!stream || !out_graph) return VNPU_ERR_INVALID_ARGUMENT;
    *out_graph = nullptr;
    std::lock_guard<std::mutex> l(stream->mutex);
    if (!stream->capturing) return VNPU_ERR_INVALID_ARGUMENT;
    cudaSetDevice(stream->device->ordinal);
    stream->capturing = false;
    cudaGraph_t g = nullptr;
    if (cudaStreamEndCapture(stream->cs, &g) != cudaSuccess || !g) {
        cudaGetLastError();
        return VNPU_ERR_DEVICE_ERROR;
    }
    // Commands that failed validation while capturing left a sticky error.
    if (stream->last_error.load()) {
        cudaGraphDestroy(g);
        return VNPU_ERR_DEVICE_ERROR;
    }
    cudaGraphExec_t exec = nullptr;
    if (cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
        cudaGetLastError();
        cudaGraphDestroy(g);
        return VNPU_ERR_DEVICE_ERROR;
    }
    auto *graph = new vnpu_b200_graph_t();
    graph->device = stream->device;
    graph->graph = g;
    graph->exec = exec;
    graph->kernels = stream->captured_launches;
    *out_graph = graph;
    return VNPU_OK;
}

VNPU_API vnpu_status_t VNPU_CALL vnpu_b200_graph_launch(vnpu_b200_graph_t *graph,
                                                       vnpu_stream_t *stream) {
    if (!graph || !stream || graph->device != stream->device) return VNPU_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> l(stream->mutex);
    if (stream->capturing) return VNPU_ERR_DEVICE_BUSY;
    cudaSetDevice(stream->device->ordinal);
    if (cudaGraphLaunch(graph->exec, stream->cs) != cudaSuccess) {
        cudaGetLastError();
        return VNPU_ERR_DEVICE_ERROR;
    }
    stream->device->launches.fetch_add(graph->kernels);
    return VNPU_OK;
}

VNPU_API void VNPU_CALL vnpu_b200_graph_destroy(vnpu_b200_graph_t *graph) {
    if (!graph) return;
    cudaSetDevice(graph->device->ordinal);
    cudaGraphExecDestroy(graph->exec);
    cudaGraphDestroy(graph->graph);
    delete graph;
}

}  // extern "C"
