/*
 * legacy_scenario.c - a program written against the legacy virtual_npu_* /
 * vgpu_npu_* / sherlock_* API (include/vnpu_compat.h and its old include
 * names), used to compare the B200 library with the reference's compat layer
 * (src/compat/compat.cpp) on the same calls.
 *
 *   legacy_scenario <out.bin>
 *
 * Every observable result (return values, status counters, VRAM contents
 * after the commands, GEMM outputs) is appended to out.bin as tagged
 * records, so two runs compare byte for byte.  Wall-clock times are not
 * recorded.  Exit status 3: the library refused to create a device (no GPU).
 * The worker-thread count that decides the reference's GEMM tiling comes
 * from VNPU_THREADS, which both libraries read.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "virtual_npu.h"
#include "vgpu_npu.h"
#include "includes/private/video/vgpu_npu.h"

static FILE *g_out;

static void emit(const char *tag, const void *data, size_t bytes)
{
    uint32_t len = (uint32_t)strlen(tag);
    uint64_t n = bytes;
    fwrite(&len, sizeof len, 1, g_out);
    fwrite(tag, 1, len, g_out);
    fwrite(&n, sizeof n, 1, g_out);
    if (bytes) fwrite(data, 1, bytes, g_out);
}

static void emit_u64(const char *tag, uint64_t v) { emit(tag, &v, sizeof v); }

static uint64_t g_rng = 0x243F6A8885A308D3ull;

/* Exact floats in [-1, 1): 24 random bits scaled by 2^-23. */
static float next_float(void)
{
    g_rng = g_rng * 6364136223846793005ull + 1442695040888963407ull;
    return (float)((g_rng >> 40) & 0xFFFFFFu) / 8388608.0f - 1.0f;
}

static void fill_floats(uint8_t *vram, size_t off, size_t count)
{
    float *p = (float *)(vram + off);
    for (size_t i = 0; i < count; ++i) p[i] = next_float();
}

static int run_virtual_npu(void)
{
    virtual_npu_t *n = virtual_npu_create(64u << 20);
    if (!n) return 3;
    uint8_t *vram = virtual_npu_memory(n);
    emit_u64("vn.size", virtual_npu_memory_size(n));

    /* areas and the page bitmap */
    uint8_t *a1 = virtual_npu_create_area(n, "weights", 10000, 0);
    uint8_t *a2 = virtual_npu_create_area(n, "scratch", 4096, 1);
    uint8_t *a3 = virtual_npu_create_area(n, "flag", 1, 0);
    emit_u64("vn.area1", (uint64_t)(a1 - vram));
    emit_u64("vn.area2", (uint64_t)(a2 - vram));
    emit_u64("vn.area3", (uint64_t)(a3 - vram));
    emit_u64("vn.area_huge", virtual_npu_create_area(n, "huge", 1u << 30, 0) == NULL);
    emit_u64("vn.delete", (uint64_t)(int64_t)virtual_npu_delete_area(n, a2));
    emit_u64("vn.delete_again", (uint64_t)(int64_t)virtual_npu_delete_area(n, a2));
    for (size_t page = 254; page < 264; ++page) emit_u64("vn.page", virtual_npu_get_bitmap_mask(n, page));
    virtual_npu_set_memory_bitmap(n, 0);
    emit_u64("vn.page_off", virtual_npu_get_bitmap_mask(n, 256));
    virtual_npu_set_memory_bitmap(n, 1);
    emit_u64("vn.page_past_end", virtual_npu_get_bitmap_mask(n, 1u << 30));

    /* teams and threads */
    int t1 = virtual_npu_create_team(n, "decoder");
    int t2 = virtual_npu_create_team(n, NULL);
    int th1 = virtual_npu_create_thread(n, t1, 50);
    int th2 = virtual_npu_create_thread(n, t2, 500);
    virtual_npu_reschedule(n);
    emit_u64("vn.team1", (uint64_t)(int64_t)t1);
    emit_u64("vn.team2", (uint64_t)(int64_t)t2);
    emit_u64("vn.thread1", (uint64_t)(int64_t)th1);
    emit_u64("vn.thread2", (uint64_t)(int64_t)th2);

    /* GEMM commands */
    const size_t M = 70, K = 300, N = 90, A = 2u << 20, B = 6u << 20, CTL = 20u << 20;
    const size_t C[5] = {10u << 20, 11u << 20, 12u << 20, 13u << 20, 14u << 20};
    fill_floats(vram, A, M * K);
    fill_floats(vram, B, K * N);
    for (size_t i = 0; i < M * N; ++i) {
        uint32_t v = (uint32_t)((i * 2654435761u) % 100u);
        memcpy(vram + CTL + 4 * i, &v, 4);
    }
    virtual_npu_compute(n, A, B, C[0], 0, M, K, N, 0, 0, 0, NPU_OP_VOODOO, 0, 0);
    virtual_npu_compute(n, A, B, C[1], CTL, M, K, N, 16, 0, 16, NPU_OP_WILDCAT, 0, 50);
    virtual_npu_compute(n, A, B, C[2], CTL, M, K, N, 0, 0, 0, NPU_OP_CPU, 0, 30);
    virtual_npu_compute(n, A, B, C[3], 0, M, K, N, 0, 0, 0, NPU_OP_TENSOR_CORE, 0, 0);
    virtual_npu_compute(n, A, B, C[4], CTL, 5, K, N, 0, 0, 0, NPU_OP_MERGED, 0, 40);
    virtual_npu_compute(n, A, B, (64u << 20) - 100, 0, M, K, N, 0, 0, 0, NPU_OP_VOODOO, 0, 0);
    virtual_npu_compute(n, A, B, C[0], 0, 0, K, N, 0, 0, 0, NPU_OP_VOODOO, 0, 0);

    virtual_npu_status_t st;
    memset(&st, 0, sizeof st); /* padding bytes are recorded too */
    virtual_npu_read_status(n, &st);
    emit("vn.status_queued", &st, sizeof st);
    virtual_npu_process(n);
    virtual_npu_read_status(n, &st);
    emit("vn.status_done", &st, sizeof st);
    for (int i = 0; i < 5; ++i) emit("vn.C", vram + C[i], 4 * (i == 4 ? 5 : M) * N);
    virtual_npu_process(n); /* empty queue */
    virtual_npu_read_status(n, &st);
    emit("vn.status_empty", &st, sizeof st);
    virtual_npu_reset_acc(n);
    virtual_npu_read_status(n, &st);
    emit("vn.status_reset", &st, sizeof st);
    virtual_npu_compute(n, A, B, C[0], 0, M, K, N, 0, 0, 0, NPU_OP_VOODOO, 0, 0);
    virtual_npu_invalidate(n);
    virtual_npu_process(n);
    virtual_npu_read_status(n, &st);
    emit("vn.status_invalidated", &st, sizeof st);

    /* Sherlock: counters only (times are wall clock) */
    sherlock_trace_start(n, SHERLOCK_TRAP_COMPUTE, "gemm");
    sherlock_trace_end(n, SHERLOCK_TRAP_COMPUTE, 1000, 4096);
    sherlock_trace_end(n, SHERLOCK_TRAP_TRANSFER, 7, 101);
    sherlock_trace_end(n, 42, 1, 1);
    sherlock_trace_t tr;
    sherlock_get_trace(&tr);
    emit_u64("sh.ops", tr.ops_count);
    emit_u64("sh.read", tr.bytes_read);
    emit_u64("sh.written", tr.bytes_written);
    emit_u64("sh.misses", tr.cache_misses);
    emit_u64("sh.enabled", (uint64_t)tr.traps_enabled);
    sherlock_enable_tracing(0);
    sherlock_trace_end(n, SHERLOCK_TRAP_MEMORY, 5, 10);
    sherlock_get_trace(&tr);
    emit_u64("sh.ops_disabled", tr.ops_count);
    emit_u64("sh.enabled_after", (uint64_t)tr.traps_enabled);
    sherlock_reset_trace();
    sherlock_get_trace(&tr);
    emit_u64("sh.ops_reset", tr.ops_count);

    virtual_npu_destroy(n);
    return 0;
}

static int run_vgpu_npu(void)
{
    vgpu_npu_t *g = vgpu_npu_create_ex(16u << 20);
    if (!g) return 3;
    uint8_t *vram = vgpu_npu_vram_ptr(g);
    const size_t size = vgpu_npu_vram_size(g);
    emit_u64("vg.size", size);

    vgpu_npu_writel(g, 100, 0xdeadbeefu);
    vgpu_npu_writel(g, (uint32_t)size, 1u);
    emit_u64("vg.readl", vgpu_npu_readl(g, 100));
    emit_u64("vg.readl_edge", vgpu_npu_readl(g, (uint32_t)size - 2));

    vgpu_npu_fill_npu(g, 4096, 1000, 0x01020304u);
    vgpu_npu_clear_npu(g, (uint32_t)size - 8, 10, 7u);
    vgpu_npu_blit_npu(g, 4096, 8192, 500, 0);

    uint8_t tex[16 * 8 * 4];
    for (size_t i = 0; i < sizeof tex; ++i) tex[i] = (uint8_t)(i * 7 + 3);
    vgpu_npu_texture_upload_npu(g, 1, 65536, tex, 16, 8, 0, 2);
    vgpu_npu_texture_upload_npu(g, 5, 70000, tex, 16, 8, 0, 2);   /* bad TMU: ignored */
    vgpu_npu_bind_tmu_npu(g, 0, 65536, 1, 16, 8, 0);
    for (int i = 0; i < 3; ++i)
        vgpu_npu_draw_triangle_npu(g, 0, 0, 10, 0, 0, 10, 0xffu, 0xff00u, 0, 0, 0, 1);
    vgpu_npu_swapbuffers_npu(g);

    const uint32_t SRC = 131072, CULL = 196608;
    for (uint32_t i = 0; i < 300; ++i) vgpu_npu_writel(g, SRC + 4 * i, i * 2654435761u);
    const uint32_t ctrl[5] = {10, 0, 99, 5, 77};
    for (uint32_t b = 0; b < 5; ++b) vgpu_npu_writel(g, CULL + 256 * b, ctrl[b]);
    vgpu_npu_unit1_shader_load(g, 0x1000, 64);
    vgpu_npu_unit1_hierarchical_z_load(g, CULL, 77);
    vgpu_npu_unit1_compute_npu(g, SRC, 262144, 300, 0x101, CULL, 20);
    vgpu_npu_unit1_compute_npu(g, SRC, 266240, 100, 0x02, 0, 0);
    vgpu_npu_unit1_compute_npu(g, SRC, 270336, 64, 0x03, 0, 0);
    vgpu_npu_unit1_compute_npu(g, SRC, 274432, 64, 0x05, 0, 0);

    const uint32_t M = 33, K = 140, N = 50, A = 1u << 20, B = 2u << 20;
    fill_floats(vram, A, (size_t)M * K);
    fill_floats(vram, B, (size_t)K * N);
    vgpu_npu_matmul_npu(g, A, B, 3u << 20, M, K, N, 1);
    vgpu_npu_matmul_npu(g, A, B, 4u << 20, M, K, N, 3);
    vgpu_npu_matmul_npu(g, A, B, (uint32_t)size - 16, M, K, N, 1);   /* out of VRAM */
    vgpu_npu_matmul_npu(g, A, B, 5u << 20, 0, K, N, 1);              /* ignored */

    vgpu_npu_status_t st;
    memset(&st, 0, sizeof st); /* the 4 bytes after `unit` are padding */
    vgpu_npu_read_status(g, &st);
    emit("vg.status_queued", &st, sizeof st);
    vgpu_npu_process(g);
    vgpu_npu_read_status(g, &st);
    emit("vg.status_done", &st, sizeof st);
    for (int i = -1; i <= 9; ++i) emit_u64("vg.unit1", vgpu_npu_unit1_read_result(g, i));
    emit("vg.fill", vram + 4096, 4 * 1000);
    emit("vg.blit", vram + 8192, 4 * 600);
    emit("vg.edge", vram + size - 16, 16);
    emit("vg.tex", vram + 65536, 1024);
    emit("vg.unit1_out", vram + 262144, 4 * 300);
    emit("vg.unit1_mul", vram + 266240, 4 * 100);
    emit("vg.unit1_xor", vram + 270336, 4 * 64);
    emit("vg.unit1_mux", vram + 274432, 4 * 64);
    emit("vg.C_voodoo", vram + (3u << 20), 4 * M * N);
    emit("vg.C_cell", vram + (4u << 20), 4 * M * N);
    vgpu_npu_unit1_reset_results(g);
    emit_u64("vg.unit1_reset", vgpu_npu_unit1_read_result(g, NPU_RESULT_ALU_OPS));
    vgpu_npu_destroy(g);

    g = vgpu_npu_create();
    if (!g) return 3;
    emit_u64("vg.default_size", vgpu_npu_vram_size(g));
    vgpu_npu_destroy(g);
    return 0;
}

int main(int argc, char **argv)
{
    if (argc != 2) {
        fprintf(stderr, "usage: %s <out.bin>\n", argv[0]);
        return 2;
    }
    g_out = fopen(argv[1], "wb");
    if (!g_out) return 2;
    int rc = run_virtual_npu();
    if (!rc) rc = run_vgpu_npu();
    fclose(g_out);
    printf("legacy scenario: %s\n", rc == 3 ? "no device" : "done");
    return rc;
}
