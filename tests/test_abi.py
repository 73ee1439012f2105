"""The drop-in boundary, checked without a GPU.

* libvnpu.so loads and exports every function include/*.h declares;
* every struct of the ABI has the reference's size and field offsets
  (a C probe compiled once against include/ here and once against the
  reference's own headers, when the reference checkout is present);
* the ctypes mirror (vnpu.py) agrees with the C layout.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import pytest

import vnpu
from conftest import ROOT, reference_dir

INCLUDE = os.path.join(ROOT, "include")
REFERENCE_INCLUDE = os.path.join(reference_dir(), "include") if reference_dir() else ""
HEADERS = ["vnpu.h", "vnpu_backend.h", "vnpu_b200.h"]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(os.path.join(INCLUDE, h)).read()
        names += re.findall(r"VNPU_API\s+[^;]*?VNPU_CALL\s+(\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_the_reference_surface():
    names = declared_functions()
    assert len(names) >= 70
    for must in ("vnpu_matmul_i8", "vnpu_quantize_i8", "vnpu_pack_weights_i8",
                 "vnpu_stream_submit", "vnpu_get_backend_v1", "vnpu_b200_stream_handle"):
        assert must in names


def test_library_exports_every_declared_function(b200_lib):
    missing = [n for n in declared_functions() if not hasattr(b200_lib.h, n)]
    assert not missing, missing


def test_exported_surface_matches_reference_library(b200_lib, ref_lib):
    """Every function the reference exports from vnpu.h / vnpu_backend.h exists here."""
    if not os.path.isdir(REFERENCE_INCLUDE):
        pytest.skip("reference checkout not present")
    ref_text = "".join(open(os.path.join(REFERENCE_INCLUDE, h)).read()
                       for h in ("vnpu.h", "vnpu_backend.h"))
    ref_names = set(re.findall(r"VNPU_API\s+[^;]*?VNPU_CALL\s+(\w+)\s*\(", ref_text))
    assert ref_names
    assert not [n for n in ref_names if not hasattr(b200_lib.h, n)]


def _structs(header_text):
    out = {}
    for name, body in re.findall(r"typedef struct (\w+) \{(.*?)\n\} \1;", header_text, re.S):
        fields = []
        depth = 0
        for line in body.splitlines():
            line = line.split("/*")[0].strip()
            if line.startswith("union"):
                depth += 1
                continue
            if line.startswith("}"):
                depth -= 1
                m = re.match(r"\}\s*(\w+);", line)
                if m:
                    fields.append(m.group(1))
                continue
            if depth or not line.endswith(";"):
                continue
            m = re.search(r"(\w+)\s*(\[[^\]]*\])?;$", line)
            if m:
                fields.append(m.group(1))
        out[name] = fields
    return out


def _probe_source():
    text = "".join(open(os.path.join(INCLUDE, h)).read() for h in ("vnpu.h", "vnpu_backend.h"))
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "vnpu_backend.h"', "int main(void){"]
    for s, fields in sorted(_structs(text).items()):
        lines.append(f'printf("{s} %zu\\n", sizeof({s}));')
        for f in fields:
            lines.append(f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));')
    lines.append("return 0;}")
    return "\n".join(lines)


def _run_probe(tmp_path, include_dir, tag):
    src = tmp_path / f"probe_{tag}.c"
    exe = tmp_path / f"probe_{tag}"
    src.write_text(_probe_source())
    subprocess.run(["gcc", "-std=c11", "-I", include_dir, str(src), "-o", str(exe)], check=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout


def test_struct_layouts(tmp_path):
    ours = _run_probe(tmp_path, INCLUDE, "ours")
    table = dict(line.rsplit(" ", 1) for line in ours.strip().splitlines())
    assert table["vnpu_command_t"] == "208"
    assert table["vnpu_command_t.args"] == "16"
    assert int(table["vnpu_backend_v1_t"]) == C.sizeof(C.c_void_p) * (1 + 42 + 8) + 8
    assert C.sizeof(vnpu.Command) == int(table["vnpu_command_t"])
    assert C.sizeof(vnpu.MatmulI8Args) == int(table["vnpu_matmul_i8_args_t"])
    assert C.sizeof(vnpu.DeviceInfo) == int(table["vnpu_device_info_t"])
    assert C.sizeof(vnpu.DeviceStatus) == int(table["vnpu_device_status_t"])
    assert C.sizeof(vnpu.AttentionArgs) == int(table["vnpu_attention_f32_args_t"])
    if not os.path.isdir(REFERENCE_INCLUDE):
        pytest.skip("reference headers not present: layout compared to the ctypes mirror only")
    theirs = _run_probe(tmp_path, REFERENCE_INCLUDE, "ref")
    assert ours == theirs


def test_vtable(b200_lib):
    class Table(C.Structure):
        _fields_ = [("abi_version", C.c_uint32), ("table_size", C.c_uint32),
                    ("backend_name", C.c_char_p)] + \
                   [(f"fn{i}", C.c_void_p) for i in range(42)] + [("reserved", C.c_void_p * 8)]
    p = b200_lib.get_backend_v1()
    t = C.cast(p, C.POINTER(Table)).contents
    assert t.abi_version == 1
    assert t.table_size == C.sizeof(Table)
    assert t.backend_name == b"vnpu-b200"
    assert all(getattr(t, f"fn{i}") for i in range(42))
    # slot 15 is matmul_i8 (include/vnpu_backend.h field order)
    assert t.fn15 == C.cast(b200_lib.h.vnpu_matmul_i8, C.c_void_p).value
    assert all(t.reserved[i] for i in range(8))
    assert t.reserved[0] == C.cast(b200_lib.h.vnpu_b200_stream_handle, C.c_void_p).value
    assert t.reserved[6] == C.cast(b200_lib.h.vnpu_cluster_cache_weights_i8, C.c_void_p).value
    assert t.reserved[7] == C.cast(b200_lib.h.vnpu_cluster_matmul_i8, C.c_void_p).value


def test_dynamic_load_example_links(tmp_path, b200_lib):
    """A dlopen consumer in the style of the reference's examples/dynamic_load.c
    finds the table and calls through it (no GPU: device_create is refused)."""
    src = tmp_path / "dl.c"
    src.write_text(r'''
#include <dlfcn.h>
#include <stdio.h>
#include "vnpu_backend.h"
int main(int argc, char **argv) {
    void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    if (!h) { printf("dlopen failed\n"); return 2; }
    const vnpu_backend_v1_t *(*get)(void) = (const vnpu_backend_v1_t *(*)(void))dlsym(h, "vnpu_get_backend_v1");
    const vnpu_backend_v1_t *t = get();
    vnpu_device_t *d = 0;
    vnpu_status_t rc = t->device_create(0, &d);
    printf("%s %u %d %s\n", t->backend_name, t->abi_version, (int)rc, t->status_string(rc));
    return 0;
}''')
    exe = tmp_path / "dl"
    subprocess.run(["gcc", "-I", INCLUDE, str(src), "-o", str(exe), "-ldl"], check=True)
    out = subprocess.run([str(exe), vnpu.LIB_PATH], capture_output=True, text=True, check=True,
                         env={**os.environ, "CUDA_VISIBLE_DEVICES": ""}).stdout
    name, abi, rc, _ = out.split(" ", 3)
    assert (name, abi) == ("vnpu-b200", "1")
    assert int(rc) in (vnpu.ERR_UNSUPPORTED, vnpu.OK)


def test_b200_extension_structs(tmp_path):
    """The fused-prologue argument structs (include/vnpu_b200.h) match the
    ctypes mirror and fit in vnpu_command_t.args.raw."""
    src = tmp_path / "ext.c"
    src.write_text(r'''
#include <stddef.h>
#include <stdio.h>
#include "vnpu_b200.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f))
int main(void) {
    printf("rq %zu\nsq %zu\nraw %zu\n", sizeof(vnpu_b200_rmsnorm_quantize_args_t),
           sizeof(vnpu_b200_swiglu_quantize_args_t), sizeof(((vnpu_command_t *)0)->args.raw));
    F(vnpu_b200_rmsnorm_quantize_args_t, Q); F(vnpu_b200_rmsnorm_quantize_args_t, eps);
    F(vnpu_b200_swiglu_quantize_args_t, scales); F(vnpu_b200_swiglu_quantize_args_t, alpha);
    printf("sc %zu\n", sizeof(vnpu_b200_matmul_i8_scatter_args_t));
    F(vnpu_b200_matmul_i8_scatter_args_t, dst); F(vnpu_b200_matmul_i8_scatter_args_t, ndst);
    printf("qkv %zu\n", sizeof(vnpu_b200_qkv_rope_append_args_t));
    F(vnpu_b200_qkv_rope_append_args_t, position); F(vnpu_b200_qkv_rope_append_args_t, T);
    F(vnpu_b200_qkv_rope_append_args_t, theta_base); F(vnpu_b200_qkv_rope_append_args_t, epilogue);
    printf("res %zu\n", sizeof(vnpu_b200_matmul_i8_residual_args_t));
    F(vnpu_b200_matmul_i8_residual_args_t, R); F(vnpu_b200_matmul_i8_residual_args_t, ldr);
    F(vnpu_b200_matmul_i8_residual_args_t, epilogue);
    printf("adv %zu\noff %u\nflags %u\n", sizeof(vnpu_b200_advance_t),
           VNPU_B200_ADVANCE_OFFSET, VNPU_B200_CMD_FLAG_ADVANCE_POSITION);
    F(vnpu_b200_advance_t, position); F(vnpu_b200_advance_t, advance);
    printf("ops %u %u %u %u\n", VNPU_B200_OP_RMSNORM_QUANTIZE_I8, VNPU_B200_OP_SWIGLU_QUANTIZE_I8,
           VNPU_B200_OP_QKV_ROPE_APPEND, VNPU_B200_OP_MATMUL_I8_RESIDUAL);
    return 0;
}''')
    exe = tmp_path / "ext"
    subprocess.run(["gcc", "-std=c11", "-I", INCLUDE, str(src), "-o", str(exe)], check=True)
    out = dict(l.rsplit(" ", 1) if not l.startswith("ops") else ("ops", l[4:])
               for l in subprocess.run([str(exe)], check=True, capture_output=True,
                                       text=True).stdout.strip().splitlines())
    assert int(out["rq"]) == C.sizeof(vnpu.RmsnormQuantizeArgs) <= int(out["raw"])
    assert int(out["sq"]) == C.sizeof(vnpu.SwigluQuantizeArgs) <= int(out["raw"])
    assert int(out["vnpu_b200_rmsnorm_quantize_args_t.Q"]) == vnpu.RmsnormQuantizeArgs.Q.offset
    assert int(out["vnpu_b200_rmsnorm_quantize_args_t.eps"]) == vnpu.RmsnormQuantizeArgs.eps.offset
    assert int(out["vnpu_b200_swiglu_quantize_args_t.scales"]) == vnpu.SwigluQuantizeArgs.scales.offset
    assert int(out["vnpu_b200_swiglu_quantize_args_t.alpha"]) == vnpu.SwigluQuantizeArgs.alpha.offset
    assert int(out["sc"]) == C.sizeof(vnpu.MatmulI8ScatterArgs) <= int(out["raw"])
    assert int(out["vnpu_b200_matmul_i8_scatter_args_t.dst"]) == vnpu.MatmulI8ScatterArgs.dst.offset
    assert int(out["vnpu_b200_matmul_i8_scatter_args_t.ndst"]) == vnpu.MatmulI8ScatterArgs.ndst.offset
    assert int(out["qkv"]) == C.sizeof(vnpu.QkvRopeAppendArgs) <= int(out["raw"])
    for f in ("position", "T", "theta_base", "epilogue"):
        assert int(out[f"vnpu_b200_qkv_rope_append_args_t.{f}"]) == \
            getattr(vnpu.QkvRopeAppendArgs, f).offset
    assert int(out["res"]) == C.sizeof(vnpu.MatmulI8ResidualArgs) <= int(out["raw"])
    for f in ("R", "ldr", "epilogue"):
        assert int(out[f"vnpu_b200_matmul_i8_residual_args_t.{f}"]) == \
            getattr(vnpu.MatmulI8ResidualArgs, f).offset
    assert int(out["adv"]) == C.sizeof(vnpu.AdvanceArgs)
    assert int(out["off"]) == vnpu.ADVANCE_OFFSET
    assert int(out["off"]) + int(out["adv"]) <= int(out["raw"])
    assert int(out["res"]) <= vnpu.ADVANCE_OFFSET
    assert int(out["flags"]) == vnpu.CMD_FLAG_ADVANCE_POSITION
    for f in ("position", "advance"):
        assert int(out[f"vnpu_b200_advance_t.{f}"]) == getattr(vnpu.AdvanceArgs, f).offset
    assert out["ops"].split() == [str(vnpu.OP_B200_RMSNORM_QUANTIZE_I8),
                                  str(vnpu.OP_B200_SWIGLU_QUANTIZE_I8),
                                  str(vnpu.OP_B200_QKV_ROPE_APPEND),
                                  str(vnpu.OP_B200_MATMUL_I8_RESIDUAL)]
