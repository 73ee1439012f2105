"""Host-side behaviour of the B200 library that needs no GPU.

Argument checks, status codes, names, conversion helpers and the rule that
there is no CPU path: without a B200 the device refuses to exist.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import vnpu


def _create(lib, env=None):
    cfg = vnpu.Config()
    lib.config_init(C.byref(cfg))
    dev = vnpu.vp()
    return lib.device_create(C.byref(cfg), C.byref(dev)), dev


def test_no_cpu_fallback_without_gpu(b200_lib, monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    rc, dev = _create(b200_lib)
    # Either a B200 is visible (GPU box, env ignored after init) or creation is
    # refused; never a device that would compute on the host.
    if rc == vnpu.OK:
        info = vnpu.DeviceInfo()
        b200_lib.device_get_info(dev, C.byref(info))
        assert info.cpu_arch.startswith(b"sm_100")
        b200_lib.device_destroy(dev)
    else:
        assert rc == vnpu.ERR_UNSUPPORTED
        assert not dev.value


def test_status_and_names_match_reference(b200_lib):
    expect = {0: b"OK", -1: b"invalid argument", -2: b"out of memory", -3: b"unsupported",
              -4: b"invalid command", -5: b"device busy", -6: b"device error", -7: b"timeout",
              -8: b"network error", -9: b"authentication error", -10: b"protocol error",
              -11: b"not found", -12: b"I/O error", -100: b"internal error"}
    for code, text in expect.items():
        assert b200_lib.status_string(code) == text
    b200_lib.h.vnpu_opcode_name.restype = C.c_char_p
    b200_lib.h.vnpu_unit_name.restype = C.c_char_p
    assert b200_lib.h.vnpu_opcode_name(2) == b"MATMUL_I8"
    assert b200_lib.h.vnpu_opcode_name(16) == b"BARRIER"
    assert b200_lib.h.vnpu_opcode_name(99) == b"UNKNOWN"
    assert b200_lib.h.vnpu_unit_name(16) == b"GPU"


def test_names_identical_to_reference_library(b200_lib, ref_lib):
    for lib in (b200_lib, ref_lib):
        lib.h.vnpu_opcode_name.restype = C.c_char_p
        lib.h.vnpu_unit_name.restype = C.c_char_p
    for op in range(18):
        assert b200_lib.h.vnpu_opcode_name(op) == ref_lib.h.vnpu_opcode_name(op)
    for u in (0, 1, 2, 3, 16, 7):
        assert b200_lib.h.vnpu_unit_name(u) == ref_lib.h.vnpu_unit_name(u)
    for code in list(range(-12, 1)) + [-100, -55]:
        assert b200_lib.status_string(code) == ref_lib.status_string(code)


def test_config_init_reads_environment(b200_lib, monkeypatch):
    monkeypatch.setenv("VNPU_THREADS", "7")
    monkeypatch.setenv("VNPU_TRACE", "1")
    cfg = vnpu.Config()
    b200_lib.config_init(C.byref(cfg))
    assert cfg.abi_version == 1 and cfg.num_threads == 7 and cfg.flags & 1


def test_null_arguments(b200_lib):
    h = b200_lib.h
    assert b200_lib.stream_submit(None, None, 0, None) == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.stream_sync(None) == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.event_wait(None, 0) == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.buffer_alloc(None, 16, C.byref(vnpu.vp())) == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.pack_weights_i8(None, None, None, 4, 4, 0, 0, C.byref(vnpu.vp())) \
        == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.packed_weights_info(None, None, None, None, None, None) \
        == vnpu.ERR_INVALID_ARGUMENT
    assert b200_lib.matmul_i8(None, None) == vnpu.ERR_INVALID_ARGUMENT
    h.vnpu_node_run.restype = C.c_int
    assert h.vnpu_node_run(None) == vnpu.ERR_UNSUPPORTED


def test_cluster_without_devices(b200_lib):
    """The local cluster's host logic (src/cluster/cluster.cpp:243-546): a
    cluster with no worker refuses a GEMM with DEVICE_ERROR, remote nodes are
    unsupported, weights are cached, stats start at zero."""
    lib = b200_lib
    cl = vnpu.vp()
    assert lib.cluster_create(None, C.byref(cl)) == vnpu.OK and cl.value
    try:
        B = np.arange(12, dtype=np.float32).reshape(3, 4)
        h = vnpu.vp()
        assert lib.cluster_cache_weights_f32(cl, b"w", B.ctypes.data, 3, 4, 0, C.byref(h)) == vnpu.OK
        assert lib.cluster_cache_weights_f32(cl, b"w", B.ctypes.data, 3, 4, 2,
                                             C.byref(vnpu.vp())) == vnpu.ERR_INVALID_ARGUMENT
        A = np.ones((2, 3), np.float32)
        Cm = np.zeros((2, 4), np.float32)
        assert lib.cluster_matmul_f32(cl, h, A.ctypes.data, Cm.ctypes.data, 2, 3, 4, 0) \
            == vnpu.ERR_DEVICE_ERROR
        assert lib.cluster_matmul_f32(cl, h, A.ctypes.data, Cm.ctypes.data, 2, 5, 4, 0) \
            == vnpu.ERR_INVALID_ARGUMENT
        assert lib.cluster_add_remote(cl, None, C.byref(vnpu.vp())) == vnpu.ERR_UNSUPPORTED
        st = vnpu.ClusterStats()
        assert lib.cluster_get_stats(cl, C.byref(st)) == vnpu.OK
        assert st.total_jobs == 0 and st.local_jobs == 0
        assert lib.cluster_add_device(cl, None, 1) == vnpu.ERR_INVALID_ARGUMENT
        # the int8 column-sharded entries: no device to hold a shard, an f32
        # handle is not an int8 one, shapes are checked
        B8 = np.ones((3, 4), np.int8)
        assert lib.cluster_cache_weights_i8(cl, b"q", B8.ctypes.data, None, 3, 4, 0,
                                            C.byref(vnpu.vp())) == vnpu.ERR_DEVICE_ERROR
        assert lib.cluster_cache_weights_i8(cl, b"q", B8.ctypes.data, None, 3, 4, 2,
                                            C.byref(vnpu.vp())) == vnpu.ERR_INVALID_ARGUMENT
        A8 = np.ones((2, 3), np.int8)
        assert lib.cluster_matmul_i8(cl, h, A8.ctypes.data, None, None, Cm.ctypes.data,
                                     2, 3, 4, 0, 0) == vnpu.ERR_INVALID_ARGUMENT
    finally:
        lib.cluster_destroy(cl)


def test_events_without_work(b200_lib):
    ev = vnpu.vp()
    assert b200_lib.event_create(C.byref(ev)) == vnpu.OK
    assert b200_lib.event_query(ev) == vnpu.ERR_DEVICE_BUSY     # never submitted
    assert b200_lib.event_wait(ev, 0) == vnpu.ERR_TIMEOUT
    assert b200_lib.event_wait(ev, 5) == vnpu.ERR_TIMEOUT
    b200_lib.event_destroy(ev)


def test_half_and_bfloat_conversions(b200_lib):
    h = b200_lib.h
    h.vnpu_float_to_f16.restype = C.c_uint16
    h.vnpu_float_to_f16.argtypes = [C.c_float]
    h.vnpu_f16_to_float.restype = C.c_float
    h.vnpu_f16_to_float.argtypes = [C.c_uint16]
    h.vnpu_float_to_bf16.restype = C.c_uint16
    h.vnpu_float_to_bf16.argtypes = [C.c_float]
    h.vnpu_bf16_to_float.restype = C.c_float
    h.vnpu_bf16_to_float.argtypes = [C.c_uint16]
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e4, 500),
                           rng.normal(0, 1e-6, 500),
                           [0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 6e-8, 3e-8, 2.98e-8,
                            np.inf, -np.inf]]).astype(np.float32)
    for v in vals:
        assert h.vnpu_float_to_f16(float(v)) == int(np.float32(v).astype(np.float16).view(np.uint16)), v
    for bits in range(0, 65536, 7):
        f16 = np.uint16(bits).view(np.float16)
        got = h.vnpu_f16_to_float(bits)
        if np.isnan(f16):
            assert np.isnan(got)
        else:
            assert np.float32(got) == np.float32(f16)
    # bfloat16: round to nearest even of the top 16 bits
    for v in vals:
        u = int(np.float32(v).view(np.uint32))
        expect = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 if not np.isnan(v) else None
        got = h.vnpu_float_to_bf16(float(v))
        if expect is not None:
            assert got == expect & 0xFFFF
        back = h.vnpu_bf16_to_float(got)
        assert np.float32(back).view(np.uint32) == np.uint32(got << 16)
