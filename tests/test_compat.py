"""The legacy virtual_npu_* / vgpu_npu_* / sherlock_* API (include/vnpu_compat.h),
checked without a GPU.

* libvnpu.so exports every function the header declares, and the header
  declares exactly the reference's legacy surface (include/vnpu_compat.h of
  the reference), with the same struct layouts;
* a legacy program (tests/compat/legacy_scenario.c) that includes the old
  header names compiles and links against libvnpu.so; without a GPU the
  library refuses the device and the program says so;
* the committed golden run of that program against the reference's compat
  layer agrees with the oracle: its GEMM records are the reference's
  MATMUL_F32 bits (unit mapping, Wildcat tile culls, element culls), so the
  B200 run on a GPU (tests/test_gpu_compat.py) is held to the reference.
"""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

import vnpu
from conftest import ROOT, bits_equal, build_legacy_scenario, read_records, reference_dir

INCLUDE = os.path.join(ROOT, "include")
REF_DIR = reference_dir()
GOLDEN = os.path.join(ROOT, "tests", "golden", "legacy_scenario.bin")
LIB_DIR = os.path.dirname(vnpu.LIB_PATH)


def compat_functions(text: str):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b((?:virtual_npu|vgpu_npu|sherlock)_\w+)\s*\(", text))


def test_library_exports_the_legacy_surface(b200_lib):
    names = compat_functions(open(os.path.join(INCLUDE, "vnpu_compat.h")).read())
    assert len(names) >= 45
    assert not [n for n in names if not hasattr(b200_lib.h, n)]


def test_same_surface_as_reference_header():
    ref = os.path.join(REF_DIR, "include", "vnpu_compat.h")
    if not os.path.exists(ref):
        pytest.skip("reference checkout not present")
    ours = compat_functions(open(os.path.join(INCLUDE, "vnpu_compat.h")).read())
    assert ours == compat_functions(open(ref).read())


def _layout_probe(tmp_path, include_dir, tag):
    src = tmp_path / f"probe_{tag}.c"
    src.write_text(r'''
#include <stddef.h>
#include <stdio.h>
#include "vnpu_compat.h"
#define F(s, f) printf(#s "." #f " %zu\n", offsetof(s, f))
int main(void) {
    printf("virtual_npu_status_t %zu\n", sizeof(virtual_npu_status_t));
    F(virtual_npu_status_t, error); F(virtual_npu_status_t, ops); F(virtual_npu_status_t, batches);
    printf("sherlock_trace_t %zu\n", sizeof(sherlock_trace_t));
    F(sherlock_trace_t, total_time); F(sherlock_trace_t, bytes_read); F(sherlock_trace_t, traps_enabled);
    printf("vgpu_npu_status_t %zu\n", sizeof(vgpu_npu_status_t));
    F(vgpu_npu_status_t, unit); F(vgpu_npu_status_t, results);
    printf("enums %d %d %d %d\n", NPU_OP_VNPU_AUTO, SHERLOCK_TRAP_COUNT, NPU_RESULT_PROCESSED,
           NPU_OP_TENSOR_CORE);
    return 0;
}''')
    exe = tmp_path / f"probe_{tag}"
    subprocess.run(["gcc", "-I", include_dir, str(src), "-o", str(exe)], check=True)
    return subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout


def test_struct_layouts(tmp_path):
    ours = _layout_probe(tmp_path, INCLUDE, "b200")
    assert "virtual_npu_status_t 48" in ours and "vgpu_npu_status_t 88" in ours
    ref_include = os.path.join(REF_DIR, "include")
    if os.path.exists(os.path.join(ref_include, "vnpu_compat.h")):
        assert ours == _layout_probe(tmp_path, ref_include, "ref")


def test_legacy_program_links_and_reports_no_device(tmp_path):
    exe = build_legacy_scenario(str(tmp_path), INCLUDE,
                                ["-L", LIB_DIR, "-lvnpu", f"-Wl,-rpath,{LIB_DIR}"])
    r = subprocess.run([exe, str(tmp_path / "out.bin")], capture_output=True, text=True,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""}, timeout=120)
    assert r.returncode == 3 and "no device" in r.stdout


class _Lcg:
    """The scenario's generator: exact floats in [-1, 1)."""

    def __init__(self):
        self.s = 0x243F6A8885A308D3

    def floats(self, n):
        out = np.empty(n, np.float32)
        s = self.s
        for i in range(n):
            s = (s * 6364136223846793005 + 1442695040888963407) & (2 ** 64 - 1)
            out[i] = ((s >> 40) & 0xFFFFFF) / 8388608.0 - 1.0
        self.s = s
        return out


def _tile_cull(C, ctl, thr, tm, tn):
    C = C.copy()
    M, N = C.shape
    for m0 in range(0, M, tm):
        for n0 in range(0, N, tn):
            if ctl[m0 * N + n0] < thr:
                C[m0:m0 + tm, n0:n0 + tn] = 0
    return C


def test_golden_gemm_records_match_oracle(oracle):
    """The reference's legacy GEMMs (compat.cpp:450-488, :858-884) are
    MATMUL_F32 with its unit mapping, then host culls."""
    rec = read_records(GOLDEN)
    Cs = [np.frombuffer(b, np.float32) for t, b in rec if t == "vn.C"]
    rng = _Lcg()
    M, K, N = 70, 300, 90
    A = rng.floats(M * K).reshape(M, K)
    B = rng.floats(K * N).reshape(K, N)
    ctl = (np.arange(M * N, dtype=np.uint64) * 2654435761 % 100).astype(np.uint32)

    def f32(unit, m=M):
        return oracle.matmul_f32(A[:m], B, m, K, N, unit=unit, threads=4)

    assert bits_equal(Cs[0].reshape(M, N), f32(1))
    assert bits_equal(Cs[1].reshape(M, N), _tile_cull(f32(2), ctl, 50, 16, 16))
    elem = f32(1)
    elem.reshape(-1)[ctl < 30] = 0
    assert bits_equal(Cs[2].reshape(M, N), elem)
    assert bits_equal(Cs[3].reshape(M, N), f32(3))
    assert bits_equal(Cs[4].reshape(5, N), _tile_cull(f32(1, 5), ctl[:5 * N], 40, 32, 32))
    status = np.frombuffer(dict(rec)["vn.status_done"], np.uint64)
    # busy/error in the first word, then ops, processed, culled, dispatches,
    # batches; the out-of-VRAM and M = 0 commands never queued
    culled = int((_tile_cull(f32(2), ctl, 50, 16, 16) == 0).sum() - (f32(2) == 0).sum()
                 + (ctl < 30).sum()
                 + (_tile_cull(f32(1, 5), ctl[:5 * N], 40, 32, 32) == 0).sum()
                 - (f32(1, 5) == 0).sum())
    assert status[1] == 2 * (4 * M + 5) * K * N
    assert status[3] == culled and status[2] == (4 * M + 5) * N - culled
    assert status[4] == 5 and status[5] == 5

    Mg, Kg, Ng = 33, 140, 50
    Ag = rng.floats(Mg * Kg).reshape(Mg, Kg)
    Bg = rng.floats(Kg * Ng).reshape(Kg, Ng)
    d = dict(rec)
    assert bits_equal(np.frombuffer(d["vg.C_voodoo"], np.float32).reshape(Mg, Ng),
                      oracle.matmul_f32(Ag, Bg, Mg, Kg, Ng, unit=1, threads=4))
    assert bits_equal(np.frombuffer(d["vg.C_cell"], np.float32).reshape(Mg, Ng),
                      oracle.matmul_f32(Ag, Bg, Mg, Kg, Ng, unit=3, threads=4))


def test_golden_is_the_reference_run(tmp_path):
    """Re-running the scenario against the reference archive reproduces the
    committed fixture (when the reference is built here)."""
    archive = os.path.join(ROOT, "oracle", "_ref", "libvnpu_ref.a")
    if not (os.path.exists(archive) and os.path.exists(os.path.join(REF_DIR, "include"))):
        pytest.skip("reference archive not built here")
    exe = build_legacy_scenario(str(tmp_path), os.path.join(REF_DIR, "include"),
                                [archive, "-lstdc++", "-lpthread", "-lm"])
    out = tmp_path / "ref.bin"
    subprocess.run([exe, str(out)], check=True, timeout=300,
                   env={**os.environ, "VNPU_THREADS": "4", "VNPU_FORCE_ISA": "avx2"})
    assert out.read_bytes() == open(GOLDEN, "rb").read()
