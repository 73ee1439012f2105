// compat.cpp - the legacy virtual_npu_* / vgpu_npu_* / sherlock_* API
// (include/vnpu_compat.h) on the B200 library.
//
// Behaviour restated from the reference's src/compat/compat.cpp:
//   VRAM, teams/threads, areas + page bitmap ..... :195-321
//   status accumulators, dump ..................... :323-365
//   virtual_npu_compute / process + culls ......... :367-493
//   Sherlock global trace ......................... :495-597
//   vgpu_npu register window and FIFO ............. :603-809
//   unit-1 ALU stream, FIFO execution ............. :35-47, :811-949
// The VRAM stays host memory the caller reads and writes through the
// returned pointer.  Every GEMM command becomes one MATMUL_F32 on this
// library's GPU device (operands staged from the VRAM through HBM), so a
// legacy matmul gets the GPU kernel and the reference's exact bits.  The
// graphics commands keep the reference's counter-only behaviour; the fill,
// blit, texture and unit-1 ALU commands are byte work on that host VRAM.
#include "../../include/vnpu_compat.h"

#include <sys/mman.h>

#include <algorithm>
#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

namespace {

constexpr size_t kPageBytes = 4096;

uint64_t wall_ns() {
    return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now().time_since_epoch())
                                     .count());
}

// Zero-filled, lazily committed host VRAM.
uint8_t *map_vram(size_t bytes) {
    void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE,
                   MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    return p == MAP_FAILED ? nullptr : static_cast<uint8_t *>(p);
}

void unmap_vram(uint8_t *p, size_t bytes) {
    if (p) munmap(p, bytes);
}

uint32_t get32(const uint8_t *p) {
    uint32_t v;
    std::memcpy(&v, p, sizeof v);
    return v;
}

void put32(uint8_t *p, uint32_t v) { std::memcpy(p, &v, sizeof v); }

// a * b * c overflows size_t.
bool size_product_overflows(size_t a, size_t b, size_t c) {
    const size_t max = std::numeric_limits<size_t>::max();
    if (a && b > max / a) return true;
    return c && a * b > max / c;
}

// Unit-1 ALU op on the operand pair (a, b); the low byte selects it.  The
// four "mux" codes reduce to picking one operand: (a&b)|(~a&b) is b and
// (a&b)|(a&~b) is a.
uint32_t unit1_alu(uint32_t a, uint32_t b, uint32_t op) {
    switch (op & 0xffu) {
    case 0x01: return a + b;
    case 0x02: return a * b;
    case 0x03: return a ^ b;
    case 0x04:
    case 0x06: return b;
    default: return a;  // 0x05, 0x07 and unknown codes
    }
}

// Legacy engine -> vnpu compute unit.
uint32_t unit_for_op_kind(uint32_t op_kind) {
    switch (op_kind) {
    case NPU_OP_VOODOO:
    case NPU_OP_MERGED: return VNPU_UNIT_VOODOO;
    case NPU_OP_WILDCAT:
    case NPU_OP_SHADER_GEMM:
    case NPU_OP_SHADER_MATMUL: return VNPU_UNIT_WILDCAT;
    case NPU_OP_FUSED_GEMM:
    case NPU_OP_TENSOR_CORE: return VNPU_UNIT_CELL;
    default: return VNPU_UNIT_AUTO;
    }
}

// A vnpu device + stream on this library, named for the legacy object.
struct Engine {
    vnpu_device_t *device = nullptr;
    vnpu_stream_t *stream = nullptr;

    bool open(const char *name) {
        vnpu_config_t cfg;
        vnpu_config_init(&cfg);
        cfg.node_name = name;
        if (vnpu_device_create(&cfg, &device) != VNPU_OK) return false;
        if (vnpu_stream_create(device, 0, &stream) != VNPU_OK) {
            vnpu_device_destroy(device);
            device = nullptr;
            return false;
        }
        return true;
    }
    void close() {
        if (stream) vnpu_stream_destroy(stream);
        if (device) vnpu_device_destroy(device);
        stream = nullptr;
        device = nullptr;
    }
    // C = A . B, f32 row-major, alpha 1, beta 0, on this device's GPU.
    bool gemm(uint8_t *vram, size_t a, size_t b, size_t c, uint32_t M, uint32_t K, uint32_t N,
              uint32_t unit) {
        vnpu_matmul_f32_args_t args{};
        args.A = reinterpret_cast<const float *>(vram + a);
        args.B = reinterpret_cast<const float *>(vram + b);
        args.C = reinterpret_cast<float *>(vram + c);
        args.M = M;
        args.K = K;
        args.N = N;
        args.alpha = 1.0f;
        args.beta = 0.0f;
        args.unit = unit;
        return vnpu_matmul_f32(stream, &args) == VNPU_OK;
    }
};

// ---- Sherlock global trace ----------------------------------------------------
struct SherlockState {
    std::mutex mutex;
    int enabled = 1;
    double dispatch = 0, memory = 0, compute = 0, sync = 0;
    uint64_t bytes_read = 0, bytes_written = 0, cache_misses = 0, ops = 0;
    uint64_t origin_ns = wall_ns();

    void clear_locked() {
        dispatch = memory = compute = sync = 0;
        bytes_read = bytes_written = cache_misses = ops = 0;
        origin_ns = wall_ns();
    }
};

SherlockState &sherlock() {
    static SherlockState s;
    return s;
}

thread_local uint64_t t_trap_start[SHERLOCK_TRAP_COUNT] = {};

// ---- queued commands ---------------------------------------------------------
struct GemmCommand {
    size_t a, b, c, ctl;
    size_t M, K, N;
    size_t tile_m, tile_n;
    uint32_t op_kind;
    uint32_t cull_threshold;
};

struct Area {
    void *addr;
    size_t bytes;
    int lock;
};

enum FifoOp : uint32_t { kFill = 1, kBlit, kTexture, kTriangle, kSwap, kUnit1, kMatmul };

struct FifoCommand {
    uint32_t op = 0;
    uint32_t w[8] = {};          // operands, per op
    std::vector<uint8_t> bytes;  // texture payload
};

struct TmuBinding {
    uint32_t base = 0;
    int format = 0, w = 0, h = 0, tmudiv = 0;
};

}  // namespace

struct virtual_npu {
    Engine engine;
    uint8_t *vram = nullptr;
    size_t vram_size = 0;
    std::vector<GemmCommand> queue;
    virtual_npu_status_t acc{};
    std::vector<uint64_t> page_bits;
    size_t pages = 0;
    int bitmap_enabled = 1;
    std::vector<Area> areas;
    std::vector<std::pair<int, std::string>> teams;   // (id, name)
    std::vector<std::pair<int, int>> threads;          // (id, team); priority kept below
    std::vector<int> thread_priority;
    size_t heap_next = 0x100000;  // areas are carved upward from 1 MiB
    int next_team = 1;
    int next_thread = 1;
    std::mutex mutex;

    void mark_pages(size_t first, size_t count, bool on) {
        for (size_t p = first; p < first + count && p < pages; ++p) {
            if (on) page_bits[p / 64] |= 1ull << (p % 64);
            else page_bits[p / 64] &= ~(1ull << (p % 64));
        }
    }
};

struct vgpu_npu {
    Engine engine;
    uint8_t *vram = nullptr;
    size_t vram_size = 0;
    std::vector<FifoCommand> fifo;
    uint64_t results[9] = {};
    uint64_t unit1_results[9] = {};
    TmuBinding tmu[4];
    uint32_t prog_base = 0, prog_size = 0;
    uint32_t hier_z_addr = 0, hier_z_scale = 0;
    int busy = 1;
    int error = 0;
    int unit = 1;
    std::mutex mutex;

    bool in_vram(size_t off, size_t bytes) const {
        return off <= vram_size && bytes <= vram_size - off;
    }
    void push(FifoCommand c) {
        std::lock_guard<std::mutex> g(mutex);
        fifo.push_back(std::move(c));
    }
};

namespace {

void zero_culled_elements(uint8_t *vram, const GemmCommand &c, uint64_t &culled) {
    uint8_t *C = vram + c.c;
    const uint8_t *ctl = vram + c.ctl;
    for (size_t i = 0; i < c.M * c.N; ++i) {
        if (get32(ctl + 4 * i) >= c.cull_threshold) continue;
        put32(C + 4 * i, 0);
        ++culled;
    }
}

// One control word per output tile (read at the tile's top-left element).
void zero_culled_tiles(uint8_t *vram, const GemmCommand &c, uint64_t &culled) {
    uint8_t *C = vram + c.c;
    const uint8_t *ctl = vram + c.ctl;
    const size_t tm = std::max<size_t>(1, c.tile_m), tn = std::max<size_t>(1, c.tile_n);
    for (size_t m0 = 0; m0 < c.M; m0 += tm) {
        const size_t rows = std::min(tm, c.M - m0);
        for (size_t n0 = 0; n0 < c.N; n0 += tn) {
            const size_t cols = std::min(tn, c.N - n0);
            const size_t top_left = m0 * c.N + n0;
            if (get32(ctl + 4 * top_left) >= c.cull_threshold) continue;
            for (size_t r = 0; r < rows; ++r)
                std::memset(C + 4 * ((m0 + r) * c.N + n0), 0, 4 * cols);
            culled += rows * cols;
        }
    }
}

void run_unit1(vgpu_npu *n, const FifoCommand &c) {
    const uint32_t src = c.w[0], dst = c.w[1], count = c.w[2], cull_addr = c.w[3];
    const uint32_t op = c.w[4], threshold = c.w[5];
    uint64_t processed = 0, culled = 0;
    for (size_t head = 0; head < count; head += 64) {
        const size_t len = std::min<size_t>(64, count - head);
        if (cull_addr && threshold) {
            // One control word per 64-element block; out-of-VRAM reads as 0.
            const size_t at = static_cast<size_t>(cull_addr) + head * 4;
            const uint32_t ctrl = n->in_vram(at, 4) ? get32(n->vram + at) : 0;
            if (ctrl < threshold) {
                culled += len;
                continue;
            }
        }
        for (size_t i = 0; i < len; ++i) {
            const size_t s = static_cast<size_t>(src) + (head + i) * 4;
            const size_t d = static_cast<size_t>(dst) + (head + i) * 4;
            if (!n->in_vram(s, 4) || !n->in_vram(d, 4)) break;
            const uint32_t a = get32(n->vram + s);
            const uint32_t out = unit1_alu(a, a, op);
            put32(n->vram + d, out);
            if (op & 0x100u) n->unit1_results[NPU_RESULT_ALU_OPS] += out;
            ++processed;
        }
    }
    n->results[NPU_RESULT_PIXELS] += count;
    n->results[NPU_RESULT_PROCESSED] += processed;
    n->results[NPU_RESULT_CULLED] += culled;
    n->results[NPU_RESULT_ALU_OPS] += processed;
    n->unit1_results[NPU_RESULT_PROCESSED] += processed;
    n->unit1_results[NPU_RESULT_CULLED] += culled;
    n->unit1_results[NPU_RESULT_ALU_OPS] += processed;
}

void run_matmul(vgpu_npu *n, const FifoCommand &c) {
    const uint32_t a = c.w[0], b = c.w[1], out = c.w[2], M = c.w[3], K = c.w[4], N = c.w[5];
    if (!n->in_vram(a, 4ull * M * K) || !n->in_vram(b, 4ull * K * N) ||
        !n->in_vram(out, 4ull * M * N)) {
        n->error = 1;
        return;
    }
    if (!n->engine.gemm(n->vram, a, b, out, M, K, N, c.w[6])) {
        n->error = 1;
        return;
    }
    n->results[NPU_RESULT_ALU_OPS] += 2ull * M * K * N;
    n->results[NPU_RESULT_PROCESSED] += static_cast<uint64_t>(M) * N;
}

}  // namespace

extern "C" {

// ---- virtual_npu ----------------------------------------------------------------
VNPU_API virtual_npu_t *virtual_npu_create(size_t vram_bytes) {
    if (!vram_bytes) vram_bytes = 256ull << 20;
    auto *n = new (std::nothrow) virtual_npu();
    if (!n) return nullptr;
    n->vram = map_vram(vram_bytes);
    if (!n->vram || !n->engine.open("virtual_npu_compat")) {
        unmap_vram(n->vram, vram_bytes);
        delete n;
        return nullptr;
    }
    n->vram_size = vram_bytes;
    n->pages = (vram_bytes + kPageBytes - 1) / kPageBytes;
    n->page_bits.assign((n->pages + 63) / 64, 0);
    n->teams.emplace_back(1, "npu_init");
    n->threads.emplace_back(1, 1);
    n->thread_priority.push_back(10);
    n->acc.busy = 1;
    return n;
}

VNPU_API void virtual_npu_destroy(virtual_npu_t *n) {
    if (!n) return;
    n->engine.close();
    unmap_vram(n->vram, n->vram_size);
    delete n;
}

VNPU_API uint8_t *virtual_npu_memory(virtual_npu_t *n) { return n ? n->vram : nullptr; }
VNPU_API size_t virtual_npu_memory_size(virtual_npu_t *n) { return n ? n->vram_size : 0; }

VNPU_API void virtual_npu_set_memory_bitmap(virtual_npu_t *n, int enable) {
    if (n) n->bitmap_enabled = enable != 0;
}

VNPU_API uint64_t virtual_npu_get_bitmap_mask(virtual_npu_t *n, size_t page) {
    if (!n || !n->bitmap_enabled || page >= n->pages) return 0;
    return (n->page_bits[page / 64] >> (page % 64)) & 1ull;
}

VNPU_API int virtual_npu_create_team(virtual_npu_t *n, const char *name) {
    if (!n) return -1;
    std::lock_guard<std::mutex> g(n->mutex);
    const int id = n->next_team++;
    n->teams.emplace_back(id, name ? name : "team");
    n->threads.emplace_back(n->next_thread++, id);  // each team starts with one thread
    n->thread_priority.push_back(10);
    return id;
}

VNPU_API int virtual_npu_create_thread(virtual_npu_t *n, int team, int priority) {
    if (!n) return -1;
    std::lock_guard<std::mutex> g(n->mutex);
    const int id = n->next_thread++;
    n->threads.emplace_back(id, team);
    n->thread_priority.push_back(priority > 0 && priority <= 100 ? priority : 10);
    return id;
}

VNPU_API void virtual_npu_reschedule(virtual_npu_t *) {}

VNPU_API void *virtual_npu_create_area(virtual_npu_t *n, const char *, size_t size, int lock) {
    if (!n || !size) return nullptr;
    std::lock_guard<std::mutex> g(n->mutex);
    const size_t bytes = (size + kPageBytes - 1) / kPageBytes * kPageBytes;
    if (bytes < size || n->heap_next > n->vram_size || bytes > n->vram_size - n->heap_next)
        return nullptr;
    void *addr = n->vram + n->heap_next;
    n->areas.push_back({addr, bytes, lock});
    n->mark_pages(n->heap_next / kPageBytes, bytes / kPageBytes, true);
    n->heap_next += bytes;
    return addr;
}

VNPU_API int virtual_npu_delete_area(virtual_npu_t *n, void *addr) {
    if (!n || !addr) return -1;
    std::lock_guard<std::mutex> g(n->mutex);
    auto it = std::find_if(n->areas.begin(), n->areas.end(),
                           [&](const Area &a) { return a.addr == addr; });
    if (it == n->areas.end()) return -1;
    const size_t first = static_cast<size_t>(static_cast<uint8_t *>(addr) - n->vram) / kPageBytes;
    n->mark_pages(first, it->bytes / kPageBytes, false);
    n->areas.erase(it);
    return 0;
}

VNPU_API void virtual_npu_read_status(virtual_npu_t *n, virtual_npu_status_t *s) {
    if (n && s) *s = n->acc;
}

VNPU_API void virtual_npu_reset_acc(virtual_npu_t *n) {
    if (!n) return;
    n->acc.ops = n->acc.processed = n->acc.culled = 0;
    n->acc.dispatches = n->acc.batches = 0;
}

VNPU_API void virtual_npu_invalidate(virtual_npu_t *n) {
    if (!n) return;
    n->queue.clear();
    n->acc = virtual_npu_status_t{};
    n->acc.busy = 1;
}

VNPU_API void virtual_npu_reset(virtual_npu_t *n) { virtual_npu_invalidate(n); }

VNPU_API void virtual_npu_dump(virtual_npu_t *n) {
    if (!n) return;
    std::fprintf(stderr,
                 "[virtual_npu] vram=%zu cmds=%zu busy=%d error=%d ops=%" PRIu64
                 " proc=%" PRIu64 " cull=%" PRIu64 " disp=%" PRIu64 " batch=%" PRIu64 "\n",
                 n->vram_size, n->queue.size(), n->acc.busy, n->acc.error, n->acc.ops,
                 n->acc.processed, n->acc.culled, n->acc.dispatches, n->acc.batches);
}

VNPU_API void virtual_npu_compute(virtual_npu_t *n, size_t a_addr, size_t b_addr, size_t c_addr,
                                  size_t ctl_addr, size_t M, size_t K, size_t N, size_t tile_m,
                                  size_t tile_k, size_t tile_n, uint32_t op_kind,
                                  uint32_t op_code, uint32_t cull_threshold) {
    (void)tile_k;
    (void)op_code;
    if (!n || !M || !K || !N) return;
    const size_t u32max = std::numeric_limits<uint32_t>::max();
    if (size_product_overflows(M, K, 4) || size_product_overflows(K, N, 4) ||
        size_product_overflows(M, N, 4) || M > u32max || K > u32max || N > u32max)
        return;
    auto fits = [&](size_t off, size_t bytes) {
        return off <= n->vram_size && bytes <= n->vram_size - off;
    };
    if (!fits(a_addr, M * K * 4) || !fits(b_addr, K * N * 4) || !fits(c_addr, M * N * 4) ||
        (cull_threshold && ctl_addr && !fits(ctl_addr, M * N * 4))) {
        n->acc.error = 1;
        return;
    }
    n->queue.push_back(GemmCommand{a_addr, b_addr, c_addr, ctl_addr, M, K, N,
                                   tile_m ? tile_m : 32, tile_n ? tile_n : 32, op_kind,
                                   cull_threshold});
}

VNPU_API void virtual_npu_process(virtual_npu_t *n) {
    if (!n) return;
    n->acc.busy = 1;
    n->acc.error = 0;
    for (const GemmCommand &c : n->queue) {
        if (!n->engine.gemm(n->vram, c.a, c.b, c.c, static_cast<uint32_t>(c.M),
                            static_cast<uint32_t>(c.K), static_cast<uint32_t>(c.N),
                            unit_for_op_kind(c.op_kind))) {
            n->acc.error = 1;
            continue;
        }
        uint64_t culled = 0;
        if (c.cull_threshold && c.ctl) {
            if (c.op_kind == NPU_OP_WILDCAT || c.op_kind == NPU_OP_MERGED)
                zero_culled_tiles(n->vram, c, culled);
            else
                zero_culled_elements(n->vram, c, culled);
        }
        const uint64_t outputs = static_cast<uint64_t>(c.M) * c.N;
        n->acc.ops += 2ull * c.M * c.K * c.N;
        n->acc.processed += outputs - std::min(outputs, culled);
        n->acc.culled += culled;
        n->acc.dispatches++;
        n->acc.batches++;
    }
    n->queue.clear();
    n->acc.busy = 0;
}

// ---- Sherlock -------------------------------------------------------------------
// Enabling resets the counters under the same lock (the reference's enable
// re-enters its non-recursive mutex through sherlock_reset_trace).
VNPU_API void sherlock_enable_tracing(int enable) {
    SherlockState &s = sherlock();
    std::lock_guard<std::mutex> g(s.mutex);
    s.enabled = enable != 0;
    if (enable) s.clear_locked();
}

VNPU_API void sherlock_reset_trace(void) {
    SherlockState &s = sherlock();
    std::lock_guard<std::mutex> g(s.mutex);
    s.clear_locked();
}

VNPU_API void sherlock_get_trace(sherlock_trace_t *t) {
    if (!t) return;
    SherlockState &s = sherlock();
    std::lock_guard<std::mutex> g(s.mutex);
    t->dispatch_time = s.dispatch;
    t->memory_time = s.memory;
    t->compute_time = s.compute;
    t->sync_time = s.sync;
    t->total_time = static_cast<double>(wall_ns() - s.origin_ns) / 1e9;
    t->bytes_read = s.bytes_read;
    t->bytes_written = s.bytes_written;
    t->cache_misses = s.cache_misses;
    t->ops_count = s.ops;
    t->traps_enabled = s.enabled;
}

VNPU_API void sherlock_dump_trace(const char *label) {
    sherlock_trace_t t;
    sherlock_get_trace(&t);
    if (!t.traps_enabled) return;
    const double total = t.total_time > 0.0 ? t.total_time : 1.0;
    auto line = [&](const char *what, double sec) {
        std::printf("%-15s %.6f ms (%.1f%%)\n", what, sec * 1e3, 100.0 * sec / total);
    };
    std::printf("\n=== SHERLOCK TRACE [%s] ===\n", label ? label : "UNKNOWN");
    std::printf("Total time:     %.6f ms\n", t.total_time * 1e3);
    line("Dispatch:", t.dispatch_time);
    line("Memory:", t.memory_time);
    line("Compute:", t.compute_time);
    line("Sync:", t.sync_time);
    std::printf("Ops:            %" PRIu64 "\n", t.ops_count);
    std::printf("Bytes read:     %" PRIu64 "\n", t.bytes_read);
    std::printf("Bytes written:  %" PRIu64 "\n", t.bytes_written);
    std::printf("=============================\n\n");
}

VNPU_API void sherlock_trace_start(virtual_npu_t *, int trap, const char *) {
    if (trap >= 0 && trap < SHERLOCK_TRAP_COUNT) t_trap_start[trap] = wall_ns();
}

VNPU_API void sherlock_trace_end(virtual_npu_t *, int trap, uint64_t ops, uint64_t bytes) {
    if (trap < 0 || trap >= SHERLOCK_TRAP_COUNT) return;
    const uint64_t start = t_trap_start[trap];
    const double elapsed = start ? static_cast<double>(wall_ns() - start) / 1e9 : 0.0;
    SherlockState &s = sherlock();
    std::lock_guard<std::mutex> g(s.mutex);
    if (!s.enabled) return;
    switch (trap) {
    case SHERLOCK_TRAP_MEMORY:
    case SHERLOCK_TRAP_ALLOC:
    case SHERLOCK_TRAP_TRANSFER: s.memory += elapsed; break;
    case SHERLOCK_TRAP_DISPATCH: s.dispatch += elapsed; break;
    case SHERLOCK_TRAP_SYNC:
    case SHERLOCK_TRAP_DEPENDENCY: s.sync += elapsed; break;
    default: s.compute += elapsed; break;  // COMPUTE, INSTRUCTION, ACCURACY
    }
    s.ops += ops;
    s.bytes_read += bytes / 2;  // the legacy trace splits traffic evenly
    s.bytes_written += bytes / 2;
    t_trap_start[trap] = 0;
}

// ---- vgpu_npu -------------------------------------------------------------------
VNPU_API vgpu_npu_t *vgpu_npu_create_ex(size_t vram_bytes) {
    if (!vram_bytes) vram_bytes = 2ull << 30;
    auto *n = new (std::nothrow) vgpu_npu();
    if (!n) return nullptr;
    n->vram = map_vram(vram_bytes);
    if (!n->vram || !n->engine.open("vgpu_npu_compat")) {
        unmap_vram(n->vram, vram_bytes);
        delete n;
        return nullptr;
    }
    n->vram_size = vram_bytes;
    return n;
}

VNPU_API vgpu_npu_t *vgpu_npu_create(void) { return vgpu_npu_create_ex(2ull << 30); }

VNPU_API void vgpu_npu_destroy(vgpu_npu_t *n) {
    if (!n) return;
    n->engine.close();
    unmap_vram(n->vram, n->vram_size);
    delete n;
}

VNPU_API uint8_t *vgpu_npu_vram_ptr(vgpu_npu_t *n) { return n ? n->vram : nullptr; }
VNPU_API size_t vgpu_npu_vram_size(vgpu_npu_t *n) { return n ? n->vram_size : 0; }

VNPU_API uint32_t vgpu_npu_readl(vgpu_npu_t *n, uint32_t addr) {
    return n && n->in_vram(addr, 4) ? get32(n->vram + addr) : 0;
}

VNPU_API void vgpu_npu_writel(vgpu_npu_t *n, uint32_t addr, uint32_t val) {
    if (n && n->in_vram(addr, 4)) put32(n->vram + addr, val);
}

VNPU_API void vgpu_npu_read_status(vgpu_npu_t *n, vgpu_npu_status_t *s) {
    if (!n || !s) return;
    s->busy = n->busy;
    s->error = n->error;
    s->unit = n->unit;
    std::memcpy(s->results, n->results, sizeof s->results);
}

VNPU_API void vgpu_npu_clear_npu(vgpu_npu_t *n, uint32_t addr, uint32_t count, uint32_t value) {
    if (!n) return;
    FifoCommand c;
    c.op = kFill;
    c.w[0] = addr;
    c.w[1] = count;
    c.w[2] = value;
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_fill_npu(vgpu_npu_t *n, uint32_t addr, uint32_t count, uint32_t value) {
    vgpu_npu_clear_npu(n, addr, count, value);
}

VNPU_API void vgpu_npu_blit_npu(vgpu_npu_t *n, uint32_t src, uint32_t dst, uint32_t count,
                                uint32_t) {
    if (!n) return;
    FifoCommand c;
    c.op = kBlit;
    c.w[0] = src;
    c.w[1] = dst;
    c.w[2] = count;
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_texture_upload_npu(vgpu_npu_t *n, int tmu, uint32_t base,
                                          const uint8_t *src, int w, int h, size_t stride,
                                          int format) {
    if (!n || !src || w <= 0 || h <= 0 || tmu < 0 || tmu >= 4) return;
    if (!stride) stride = static_cast<size_t>(w) * 4;
    FifoCommand c;
    c.op = kTexture;
    c.w[0] = base;
    c.w[1] = static_cast<uint32_t>(w);
    c.w[2] = static_cast<uint32_t>(h);
    c.w[3] = static_cast<uint32_t>(stride);
    c.w[4] = static_cast<uint32_t>(format);
    c.w[5] = static_cast<uint32_t>(tmu);
    c.bytes.assign(src, src + static_cast<size_t>(h) * stride);  // copied at call time
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_bind_tmu_npu(vgpu_npu_t *n, int tmu, uint32_t base, int format, int w,
                                    int h, int tmudiv) {
    if (!n || tmu < 0 || tmu >= 4) return;
    n->tmu[tmu] = TmuBinding{base, format, w, h, tmudiv};
}

VNPU_API void vgpu_npu_draw_triangle_npu(vgpu_npu_t *n, int32_t, int32_t, int32_t, int32_t,
                                         int32_t, int32_t, uint32_t, uint32_t, uint32_t,
                                         uint32_t, uint32_t, int) {
    if (!n) return;
    FifoCommand c;
    c.op = kTriangle;  // counted, not rasterised
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_swapbuffers_npu(vgpu_npu_t *n) {
    if (!n) return;
    FifoCommand c;
    c.op = kSwap;
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_unit1_shader_load(vgpu_npu_t *n, uint32_t prog_base, uint32_t prog_size) {
    if (!n) return;
    n->prog_base = prog_base;
    n->prog_size = prog_size;
}

VNPU_API void vgpu_npu_unit1_compute_npu(vgpu_npu_t *n, uint32_t src, uint32_t dst,
                                         uint32_t count, uint32_t op, uint32_t cull_addr,
                                         uint32_t cull_threshold) {
    if (!n) return;
    FifoCommand c;
    c.op = kUnit1;
    c.w[0] = src;
    c.w[1] = dst;
    c.w[2] = count;
    c.w[3] = cull_addr;
    c.w[4] = op;
    c.w[5] = cull_threshold;
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_matmul_npu(vgpu_npu_t *n, uint32_t a, uint32_t b, uint32_t out,
                                  uint32_t M, uint32_t K, uint32_t N, uint32_t unit) {
    if (!n || !M || !K || !N) return;
    FifoCommand c;
    c.op = kMatmul;
    c.w[0] = a;
    c.w[1] = b;
    c.w[2] = out;
    c.w[3] = M;
    c.w[4] = K;
    c.w[5] = N;
    c.w[6] = unit;
    n->push(std::move(c));
}

VNPU_API void vgpu_npu_unit1_hierarchical_z_load(vgpu_npu_t *n, uint32_t cull_addr,
                                                 uint32_t cull_scale) {
    if (!n) return;
    n->hier_z_addr = cull_addr;
    n->hier_z_scale = cull_scale;
    n->unit1_results[NPU_RESULT_CULLED] = cull_scale;
}

VNPU_API uint64_t vgpu_npu_unit1_read_result(vgpu_npu_t *n, int index) {
    return n && index >= 0 && index < 9 ? n->unit1_results[index] : 0;
}

VNPU_API void vgpu_npu_unit1_reset_results(vgpu_npu_t *n) {
    if (n) std::fill(std::begin(n->unit1_results), std::end(n->unit1_results), 0);
}

VNPU_API void vgpu_npu_process(vgpu_npu_t *n) {
    if (!n) return;
    n->busy = 1;
    n->error = 0;
    std::vector<FifoCommand> work;
    {
        std::lock_guard<std::mutex> g(n->mutex);
        work.swap(n->fifo);
    }
    for (const FifoCommand &c : work) {
        switch (c.op) {
        case kFill: {
            size_t at = c.w[0];
            for (uint32_t i = 0; i < c.w[1] && n->in_vram(at, 4); ++i, at += 4)
                put32(n->vram + at, c.w[2]);
            n->results[NPU_RESULT_FILLS] += c.w[1];
            n->results[NPU_RESULT_PIXELS] += c.w[1];
            break;
        }
        case kBlit: {
            size_t s = c.w[0], d = c.w[1];
            for (uint32_t i = 0; i < c.w[2] && n->in_vram(s, 4) && n->in_vram(d, 4);
                 ++i, s += 4, d += 4)
                put32(n->vram + d, get32(n->vram + s));
            n->results[NPU_RESULT_BLITS] += c.w[2];
            break;
        }
        case kTexture: {
            const size_t bytes = static_cast<size_t>(c.w[2]) * c.w[3];
            if (n->in_vram(c.w[0], bytes) && c.bytes.size() >= bytes)
                std::memcpy(n->vram + c.w[0], c.bytes.data(), bytes);
            n->results[NPU_RESULT_TEXELS] += static_cast<uint64_t>(c.w[1]) * c.w[2];
            n->results[NPU_RESULT_TEX_UPLOAD_BYTES] += bytes;
            break;
        }
        case kTriangle: n->results[NPU_RESULT_TRIS]++; break;
        case kSwap: n->busy = 0; break;
        case kUnit1: run_unit1(n, c); break;
        case kMatmul: run_matmul(n, c); break;
        default: n->error = 1; break;
        }
    }
    n->busy = 0;
}

}  // extern "C"
