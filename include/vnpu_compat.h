/*
 * vnpu_compat.h - the legacy virtual_npu_* / vgpu_npu_* / sherlock_* C API,
 * exported by the B200 library so programs written against the original NPU
 * experiments still compile and link.
 *
 * Replaces the reference's include/vnpu_compat.h:1-193 (implementation
 * src/compat/compat.cpp:1-951) declaration for declaration: same names,
 * argument lists, struct layouts and enum values.  What changed is the
 * backing: the flat "VRAM" stays host memory the caller reads and writes
 * directly, matmul commands run as MATMUL_F32 on the GPU (bit-exact with the
 * reference's CPU kernels), and the graphics calls keep the reference's
 * counter-only behaviour.  Unlike the reference's shared library, these
 * symbols have default visibility, so linking against libvnpu.so works (the
 * reference exposes them only through its static archive).
 */
#ifndef VNPU_COMPAT_H
#define VNPU_COMPAT_H

#include <stddef.h>
#include <stdint.h>

#include "vnpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- virtual_npu: flat VRAM, queued GEMM commands -------------------------- */
typedef struct virtual_npu virtual_npu_t;

VNPU_API virtual_npu_t *virtual_npu_create(size_t vram_bytes);   /* 0 = 256 MiB */
VNPU_API void virtual_npu_destroy(virtual_npu_t *n);

VNPU_API uint8_t *virtual_npu_memory(virtual_npu_t *n);
VNPU_API size_t virtual_npu_memory_size(virtual_npu_t *n);
VNPU_API void virtual_npu_set_memory_bitmap(virtual_npu_t *n, int enable);
VNPU_API uint64_t virtual_npu_get_bitmap_mask(virtual_npu_t *n, size_t page);

VNPU_API int virtual_npu_create_team(virtual_npu_t *n, const char *name);
VNPU_API int virtual_npu_create_thread(virtual_npu_t *n, int team, int priority);
VNPU_API void virtual_npu_reschedule(virtual_npu_t *n);
VNPU_API void *virtual_npu_create_area(virtual_npu_t *n, const char *name, size_t size,
                                       int lock);
VNPU_API int virtual_npu_delete_area(virtual_npu_t *n, void *addr);

typedef struct virtual_npu_status {
    int busy;
    int error;
    uint64_t ops;
    uint64_t processed;
    uint64_t culled;
    uint64_t dispatches;
    uint64_t batches;
} virtual_npu_status_t;

VNPU_API void virtual_npu_read_status(virtual_npu_t *n, virtual_npu_status_t *s);
VNPU_API void virtual_npu_reset_acc(virtual_npu_t *n);
VNPU_API void virtual_npu_invalidate(virtual_npu_t *n);
VNPU_API void virtual_npu_reset(virtual_npu_t *n);
VNPU_API void virtual_npu_dump(virtual_npu_t *n);

/* op_kind of virtual_npu_compute: the legacy engine it names maps onto a
 * vnpu compute unit (VOODOO / WILDCAT / CELL / AUTO). */
enum {
    NPU_OP_CPU = 0,
    NPU_OP_VOODOO = 1,
    NPU_OP_WILDCAT = 2,
    NPU_OP_MERGED = 3,
    NPU_OP_SHADER_GEMM = 4,
    NPU_OP_SHADER_MATMUL = 5,
    NPU_OP_FUSED_GEMM = 6,
    NPU_OP_TENSOR_CORE = 7,
    NPU_OP_VNPU_AUTO = 8
};

/* Queues C[MxN] = A[MxK] . B[KxN] (f32, row-major, byte offsets into the
 * VRAM).  With cull_threshold and ctl_addr, outputs (or output tiles, for
 * WILDCAT / MERGED) whose u32 control word is below the threshold are zeroed
 * after the product. */
VNPU_API void virtual_npu_compute(virtual_npu_t *n, size_t a_addr, size_t b_addr, size_t c_addr,
                                  size_t ctl_addr, size_t M, size_t K, size_t N, size_t tile_m,
                                  size_t tile_k, size_t tile_n, uint32_t op_kind,
                                  uint32_t op_code, uint32_t cull_threshold);
VNPU_API void virtual_npu_process(virtual_npu_t *n);

/* ---- Sherlock tracing (wall-clock timers) ---------------------------------- */
enum {
    SHERLOCK_TRAP_DISPATCH = 0,
    SHERLOCK_TRAP_MEMORY = 1,
    SHERLOCK_TRAP_INSTRUCTION = 2,
    SHERLOCK_TRAP_SYNC = 3,
    SHERLOCK_TRAP_ALLOC = 4,
    SHERLOCK_TRAP_TRANSFER = 5,
    SHERLOCK_TRAP_DEPENDENCY = 6,
    SHERLOCK_TRAP_ACCURACY = 7,
    SHERLOCK_TRAP_COMPUTE = 8,
    SHERLOCK_TRAP_COUNT = 9
};

typedef struct sherlock_trace {
    double dispatch_time;
    double memory_time;
    double compute_time;
    double sync_time;
    double total_time;
    uint64_t bytes_read;
    uint64_t bytes_written;
    uint64_t cache_misses;
    uint64_t ops_count;
    int traps_enabled;
} sherlock_trace_t;

VNPU_API void sherlock_enable_tracing(int enable);
VNPU_API void sherlock_reset_trace(void);
VNPU_API void sherlock_dump_trace(const char *label);
VNPU_API void sherlock_get_trace(sherlock_trace_t *trace);
VNPU_API void sherlock_trace_start(virtual_npu_t *n, int trap_type, const char *name);
VNPU_API void sherlock_trace_end(virtual_npu_t *n, int trap_type, uint64_t ops,
                                 uint64_t bytes);

/* ---- vgpu_npu: register-window device with a command FIFO ------------------ */
typedef struct vgpu_npu vgpu_npu_t;

VNPU_API vgpu_npu_t *vgpu_npu_create(void);                    /* 2 GiB VRAM */
VNPU_API vgpu_npu_t *vgpu_npu_create_ex(size_t vram_bytes);   /* 0 = 2 GiB */
VNPU_API void vgpu_npu_destroy(vgpu_npu_t *npu);

VNPU_API uint8_t *vgpu_npu_vram_ptr(vgpu_npu_t *npu);
VNPU_API size_t vgpu_npu_vram_size(vgpu_npu_t *npu);
VNPU_API uint32_t vgpu_npu_readl(vgpu_npu_t *npu, uint32_t addr);
VNPU_API void vgpu_npu_writel(vgpu_npu_t *npu, uint32_t addr, uint32_t val);

typedef struct vgpu_npu_status {
    int busy;
    int error;
    int unit;
    uint64_t results[9];
} vgpu_npu_status_t;

VNPU_API void vgpu_npu_read_status(vgpu_npu_t *npu, vgpu_npu_status_t *s);

/* Indices of vgpu_npu_status_t.results and vgpu_npu_unit1_read_result. */
enum {
    NPU_RESULT_PIXELS = 0,
    NPU_RESULT_TEXELS = 1,
    NPU_RESULT_TRIS = 2,
    NPU_RESULT_FILLS = 3,
    NPU_RESULT_BLITS = 4,
    NPU_RESULT_TEX_UPLOAD_BYTES = 5,
    NPU_RESULT_ALU_OPS = 6,
    NPU_RESULT_CULLED = 7,
    NPU_RESULT_PROCESSED = 8
};

VNPU_API void vgpu_npu_clear_npu(vgpu_npu_t *npu, uint32_t addr, uint32_t count,
                                 uint32_t value);
VNPU_API void vgpu_npu_fill_npu(vgpu_npu_t *npu, uint32_t addr, uint32_t count,
                                uint32_t value);
VNPU_API void vgpu_npu_blit_npu(vgpu_npu_t *npu, uint32_t src_addr, uint32_t dst_addr,
                                uint32_t count, uint32_t ctrl);
VNPU_API void vgpu_npu_texture_upload_npu(vgpu_npu_t *npu, int tmu, uint32_t base,
                                          const uint8_t *src, int w, int h, size_t stride,
                                          int format);
VNPU_API void vgpu_npu_bind_tmu_npu(vgpu_npu_t *npu, int tmu, uint32_t base, int format,
                                    int w, int h, int tmudiv);
VNPU_API void vgpu_npu_draw_triangle_npu(vgpu_npu_t *npu, int32_t ax, int32_t ay, int32_t bx,
                                         int32_t by, int32_t cx, int32_t cy, uint32_t color0,
                                         uint32_t color1, uint32_t fbzMode,
                                         uint32_t textureMode0, uint32_t textureMode1,
                                         int bilinear);
VNPU_API void vgpu_npu_swapbuffers_npu(vgpu_npu_t *npu);
VNPU_API void vgpu_npu_unit1_shader_load(vgpu_npu_t *npu, uint32_t prog_base,
                                         uint32_t prog_size);
VNPU_API void vgpu_npu_unit1_compute_npu(vgpu_npu_t *npu, uint32_t src_addr, uint32_t dst_addr,
                                         uint32_t count, uint32_t op, uint32_t cull_addr,
                                         uint32_t cull_threshold);
VNPU_API void vgpu_npu_unit1_hierarchical_z_load(vgpu_npu_t *npu, uint32_t cull_addr,
                                                 uint32_t cull_scale);
VNPU_API uint64_t vgpu_npu_unit1_read_result(vgpu_npu_t *npu, int index);
VNPU_API void vgpu_npu_unit1_reset_results(vgpu_npu_t *npu);
VNPU_API void vgpu_npu_process(vgpu_npu_t *npu);

/* Queues C[MxN] = A[MxK] . B[KxN] on VRAM byte offsets, run as MATMUL_F32
 * with the given vnpu compute unit. */
VNPU_API void vgpu_npu_matmul_npu(vgpu_npu_t *npu, uint32_t a_addr, uint32_t b_addr,
                                  uint32_t c_addr, uint32_t M, uint32_t K, uint32_t N,
                                  uint32_t unit);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VNPU_COMPAT_H */
