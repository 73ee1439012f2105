"""Runtime semantics of the B200 backend on a GPU, through the C ABI.

Mirrors the reference's selftest/conformance expectations
(tools/selftest.cpp:246-280 concurrent streams, :450-567 events/trace;
src/core/runtime.cpp:1248-1289 sticky stream errors).  Failure paths are made
on the host (bad arguments) or with the bounded device-wait self-test; nothing
here faults or hangs a GPU.
"""
from __future__ import annotations

import ctypes as C
import json
import threading

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu


def test_device_info(gpu, b200_lib):
    info = gpu.info()
    assert info.features & vnpu.FEATURE_GPU_FUTURE
    assert info.cpu_arch.startswith(b"sm_100")
    assert info.num_compute_units >= 100
    assert info.total_memory_bytes > 100 * 2 ** 30
    assert b200_lib.version_string().startswith(b"vnpu 1.0.0")


def test_event_batch_and_status(gpu, b200_lib, oracle):
    rng = np.random.default_rng(1)
    X = rng.normal(0, 1, (64, 512)).astype(np.float32)
    Y = np.empty((64, 512), np.int8)
    s = np.empty(64, np.float32)
    ev = vnpu.vp()
    assert b200_lib.event_create(C.byref(ev)) == vnpu.OK
    cmd = vnpu.Command()
    cmd.opcode = vnpu.OP_QUANTIZE_I8
    cmd.args.quantize_i8 = vnpu.QuantizeI8Args(X.ctypes.data, Y.ctypes.data, s.ctypes.data,
                                               64, 512, 0, 0)
    nop = vnpu.Command()
    nop.opcode = vnpu.OP_BARRIER
    arr = (vnpu.Command * 2)(cmd, nop)
    assert b200_lib.stream_submit(gpu.stream, arr, 2, ev) == vnpu.OK
    assert b200_lib.event_wait(ev, 10000) == vnpu.OK
    assert b200_lib.event_query(ev) == vnpu.OK
    Yo, so = oracle.quantize(X, 0)
    assert bits_equal(Y, Yo) and bits_equal(s, so)
    # empty submit signals at once
    assert b200_lib.stream_submit(gpu.stream, None, 0, ev) == vnpu.OK
    assert b200_lib.event_query(ev) == vnpu.OK
    b200_lib.event_destroy(ev)


def test_sticky_error_after_bad_command(b200_lib):
    """A failing command: submit still returns OK, the event reports
    INTERNAL, and every later sync of that stream reports DEVICE_ERROR
    (reference src/core/runtime.cpp:1248-1254,1281-1289).  Other streams are
    unaffected."""
    with vnpu.Device(b200_lib) as dev:
        w = dev.pack(np.ones((64, 32), np.int8), None, 64, 32)
        bad = vnpu.Command()
        bad.opcode = vnpu.OP_MATMUL_I8
        A = np.ones((4, 48), np.int8)
        Cm = np.empty((4, 32), np.float32)
        bad.args.matmul_i8 = vnpu.MatmulI8Args(A.ctypes.data, w, None, None, Cm.ctypes.data,
                                               4, 48, 32, 0, 0, 0, 0)  # K mismatch
        ev = vnpu.vp()
        b200_lib.event_create(C.byref(ev))
        assert b200_lib.stream_submit(dev.stream, C.byref(bad), 1, ev) == vnpu.OK
        assert b200_lib.event_wait(ev, 1000) == vnpu.ERR_INTERNAL
        assert dev.sync() == vnpu.ERR_DEVICE_ERROR
        assert dev.sync() == vnpu.ERR_DEVICE_ERROR
        st = dev.status()
        assert st.error != 0
        other = vnpu.vp()
        assert b200_lib.stream_create(dev.dev, 0, C.byref(other)) == vnpu.OK
        assert b200_lib.stream_sync(other) == vnpu.OK
        b200_lib.event_destroy(ev)
        dev.unpack(w)


def test_invalid_arguments_rejected(gpu, b200_lib):
    w = gpu.pack(np.ones((16, 16), np.int8), None, 16, 16)
    A = np.ones((2, 16), np.int8)
    Cm = np.empty((2, 16), np.float32)
    with vnpu.Device(b200_lib) as dev2:
        # lda < K
        rc = dev2.matmul_i8(A, w, None, None, Cm, 2, 16, 16, lda=8, check=False)
        assert rc == vnpu.ERR_DEVICE_ERROR
    gpu.unpack(w)
    bad = vnpu.vp()
    assert b200_lib.pack_weights_i8(gpu.dev, A.ctypes.data, None, 16, 16, 4, 0, C.byref(bad)) \
        == vnpu.ERR_INVALID_ARGUMENT  # ldb < N
    assert b200_lib.pack_weights_i8(gpu.dev, A.ctypes.data, None, 16, 16, 0, 2, C.byref(bad)) \
        == vnpu.ERR_INVALID_ARGUMENT  # trans_b > 1


def test_unsupported_opcode(b200_lib):
    with vnpu.Device(b200_lib) as dev:
        cmd = vnpu.Command()
        cmd.opcode = vnpu.OP_SOFTMAX_F32
        ev = vnpu.vp()
        b200_lib.event_create(C.byref(ev))
        assert b200_lib.stream_submit(dev.stream, C.byref(cmd), 1, ev) == vnpu.OK
        assert b200_lib.event_wait(ev, 1000) == vnpu.ERR_UNSUPPORTED
        b200_lib.event_destroy(ev)


def test_device_wait_timeout_is_reported(b200_lib, oracle):
    """The bounded device-side wait gives up, reports TIMEOUT, and the
    context stays usable (a quantize afterwards is still bit-exact)."""
    with vnpu.Device(b200_lib) as dev:
        assert b200_lib.b200_selftest_wait(dev.stream, 2000) == vnpu.ERR_TIMEOUT
        X = np.random.default_rng(0).normal(0, 1, (8, 100)).astype(np.float32)
        Y = np.empty((8, 100), np.int8)
        s = np.empty(8, np.float32)
        dev.quantize_i8(X, Y, s, 8, 100, 0)
        assert bits_equal(Y, oracle.quantize(X, 0)[0])


def test_buffers_copy_memset(gpu, b200_lib):
    buf = vnpu.vp()
    assert b200_lib.buffer_alloc(gpu.dev, 1 << 20, C.byref(buf)) == vnpu.OK
    d = b200_lib.buffer_host_ptr(buf)
    assert d and b200_lib.buffer_size(buf) == 1 << 20
    src = np.arange(1 << 18, dtype=np.uint32)
    out = np.zeros_like(src)
    assert b200_lib.buffer_copy(gpu.stream, d, src.ctypes.data, src.nbytes, vnpu.COPY_H2D) == vnpu.OK
    assert b200_lib.buffer_copy(gpu.stream, out.ctypes.data, d, src.nbytes, vnpu.COPY_D2H) == vnpu.OK
    assert np.array_equal(out, src)
    assert b200_lib.buffer_memset(gpu.stream, d, 0xAB, 4096) == vnpu.OK
    assert b200_lib.buffer_copy(gpu.stream, out.ctypes.data, d, 4096, vnpu.COPY_D2H) == vnpu.OK
    assert np.all(out[:1024] == 0xABABABAB) and out[1024] == 1024
    b200_lib.buffer_free(buf)


def test_fresh_buffer_is_zeroed(gpu, b200_lib):
    buf = vnpu.vp()
    assert b200_lib.buffer_alloc(gpu.dev, 4096, C.byref(buf)) == vnpu.OK
    out = np.ones(1024, np.uint32)
    b200_lib.buffer_copy(gpu.stream, out.ctypes.data, b200_lib.buffer_host_ptr(buf), 4096, 2)
    assert not out.any()
    b200_lib.buffer_free(buf)


def test_packed_weights_info(gpu, oracle):
    rng = np.random.default_rng(8)
    K, N = 300, 77
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    sb = rng.uniform(0.1, 1, N).astype(np.float32)
    sums, _ = oracle.column_sums(B)
    for trans, src in ((0, B), (1, np.ascontiguousarray(B.T))):
        w = gpu.pack(src, sb, K, N, trans_b=trans)
        Kr, Nr, nbytes, sc, cs = gpu.packed_info(w)
        assert (Kr, Nr) == (K, N) and nbytes >= K * N
        got_cs = np.ctypeslib.as_array(C.cast(cs, C.POINTER(C.c_int32)), (N,))
        got_sc = np.ctypeslib.as_array(C.cast(sc, C.POINTER(C.c_float)), (N,))
        assert np.array_equal(got_cs, sums) and bits_equal(got_sc.copy(), sb)
        gpu.unpack(w)


def test_trans_b_same_result(gpu, oracle):
    rng = np.random.default_rng(12)
    M, K, N = 40, 200, 96
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    sb = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    outs = []
    for trans, src in ((0, B), (1, np.ascontiguousarray(B.T))):
        w = gpu.pack(src, sb, K, N, trans_b=trans)
        Cm = np.empty((M, N), np.float32)
        gpu.matmul_i8(A, w, None, None, Cm, M, K, N)
        gpu.unpack(w)
        outs.append(Cm)
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(outs[0], oracle.matmul_i8(A, B, None, sb, None, 0, 0))


def test_all_units_bit_identical(gpu, oracle):
    """conformance.cpp:251-345: every unit gives the same bits."""
    rng = np.random.default_rng(2)
    M, K, N = 19, 47, 31
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    w = gpu.pack(B, sb, K, N)
    ref = oracle.matmul_i8(A, B, sa, sb, None, 0, 0)
    for unit in (vnpu.UNIT_AUTO, vnpu.UNIT_VOODOO, vnpu.UNIT_WILDCAT, vnpu.UNIT_CELL,
                 vnpu.UNIT_GPU):
        Cm = np.empty((M, N), np.float32)
        gpu.matmul_i8(A, w, sa, None, Cm, M, K, N, unit=unit)
        assert bits_equal(Cm, ref)
    gpu.unpack(w)


def test_concurrent_streams(b200_lib, oracle):
    """Several threads, one stream each, one device (selftest.cpp:246-280)."""
    rng = np.random.default_rng(3)
    M, K, N = 64, 256, 128
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    ref = oracle.matmul_i8(A, B, sa, sb, None, 0, 0)
    with vnpu.Device(b200_lib) as dev:
        w = dev.pack(B, sb, K, N)
        errors = []

        def worker():
            st = vnpu.vp()
            if b200_lib.stream_create(dev.dev, 0, C.byref(st)) != vnpu.OK:
                errors.append("create")
                return
            for _ in range(20):
                Cm = np.empty((M, N), np.float32)
                a = vnpu.MatmulI8Args(A.ctypes.data, w, sa.ctypes.data, None, Cm.ctypes.data,
                                      M, K, N, 0, 0, 0, 0)
                if b200_lib.matmul_i8(st, C.byref(a)) != vnpu.OK or not bits_equal(Cm, ref):
                    errors.append("mismatch")
            b200_lib.stream_destroy(st)

        ts = [threading.Thread(target=worker) for _ in range(4)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        dev.unpack(w)
    assert not errors


def test_trace_and_counters(b200_lib, tmp_path):
    with vnpu.Device(b200_lib) as dev:
        h = b200_lib.h
        h.vnpu_trace_enable.restype = C.c_int
        assert h.vnpu_trace_enable(dev.dev, 1) == vnpu.OK
        launches0 = b200_lib.b200_kernel_launches(dev.dev)
        M, K, N = 256, 512, 512
        A = np.ones((M, K), np.int8)
        w = dev.pack(np.ones((K, N), np.int8), None, K, N)
        Cm = np.empty((M, N), np.float32)
        dev.matmul_i8(A, w, None, None, Cm, M, K, N)
        assert np.all(Cm == K)
        dev.unpack(w)
        assert b200_lib.b200_kernel_launches(dev.dev) > launches0
        s = vnpu.TraceSummary()
        h.vnpu_trace_get_summary.restype = C.c_int
        assert h.vnpu_trace_get_summary(dev.dev, C.byref(s)) == vnpu.OK
        assert s.events >= 1 and s.flops == 2 * M * K * N and s.total_time_ns > 0
        assert s.hot_opcode == vnpu.OP_MATMUL_I8
        path = str(tmp_path / "trace.json")
        h.vnpu_trace_write_chrome.restype = C.c_int
        assert h.vnpu_trace_write_chrome(dev.dev, path.encode()) == vnpu.OK
        events = json.load(open(path))["traceEvents"]
        assert events and events[0]["name"].startswith("MATMUL_I8")
        st = dev.status()
        assert st.commands_submitted == st.commands_completed >= 1
        assert st.flops >= 2 * M * K * N


def test_mmio_window(gpu, b200_lib):
    h = b200_lib.h
    h.vnpu_mmio_read32.restype = C.c_uint32
    h.vnpu_mmio_read32.argtypes = [C.c_void_p, C.c_uint32]
    assert h.vnpu_mmio_read32(gpu.dev, 0x00) == 0x56504E55
    assert h.vnpu_mmio_read32(gpu.dev, 0x04) == 1
    assert h.vnpu_mmio_read32(gpu.dev, 0x03) == 0xFFFFFFFF


def test_graph_capture_replay(gpu, b200_lib, oracle):
    """Commands captured into a CUDA graph replay to the same bits; host
    operands and syncs are refused while capturing."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(21)
    M, K, N = 300, 512, 384
    Xf = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    A, sa = oracle.quantize(Xf, 0)
    ref = oracle.matmul_i8(A, B, sa, sb, None, 2, 0)
    dX = torch.from_numpy(Xf).cuda()
    dA = torch.empty((M, K), dtype=torch.int8, device="cuda")
    dsa = torch.empty(M, device="cuda")
    dC = torch.zeros((M, N), device="cuda")
    torch.cuda.synchronize()
    w = gpu.pack(B, sb, K, N)
    q = vnpu.Command()
    q.opcode = vnpu.OP_QUANTIZE_I8
    q.args.quantize_i8 = vnpu.QuantizeI8Args(dX.data_ptr(), dA.data_ptr(), dsa.data_ptr(), M, K, 0, 0)
    mm = vnpu.Command()
    mm.opcode = vnpu.OP_MATMUL_I8
    mm.args.matmul_i8 = vnpu.MatmulI8Args(dA.data_ptr(), w, dsa.data_ptr(), None, dC.data_ptr(),
                                          M, K, N, 0, 0, 2, 0)
    launches0 = b200_lib.b200_kernel_launches(gpu.dev)
    g = gpu.capture([q, mm])
    assert b200_lib.b200_kernel_launches(gpu.dev) == launches0  # recorded, not run
    assert not dC.any().item()
    for _ in range(3):
        gpu.replay(g)
    assert gpu.sync() == vnpu.OK
    assert b200_lib.b200_kernel_launches(gpu.dev) >= launches0 + 6
    assert bits_equal(dC.cpu().numpy(), ref)
    b200_lib.b200_graph_destroy(g)
    # host operand while capturing -> refused; sync while capturing -> busy
    with vnpu.Device(b200_lib) as dev2:
        assert b200_lib.b200_capture_begin(dev2.stream) == vnpu.OK
        assert dev2.sync() == vnpu.ERR_DEVICE_BUSY
        hq = vnpu.Command()
        hq.opcode = vnpu.OP_QUANTIZE_I8
        hq.args.quantize_i8 = vnpu.QuantizeI8Args(Xf.ctypes.data, dA.data_ptr(), dsa.data_ptr(),
                                                  M, K, 0, 0)
        assert dev2.submit([hq]) == vnpu.OK
        out = vnpu.vp()
        assert b200_lib.b200_capture_end(dev2.stream, C.byref(out)) == vnpu.ERR_DEVICE_ERROR
        assert not out.value
    gpu.unpack(w)


# ----------------------------------------------------------------- host operands
# Host inputs are uploaded and host outputs downloaded on two copy-engine
# streams joined to the kernel stream by events.  These cases chain commands
# through host memory inside one batch, so a missing join shows as a wrong
# result.
def _q_cmd(X, Y, s, rows, cols, axis=0):
    c = vnpu.Command()
    c.opcode = vnpu.OP_QUANTIZE_I8
    c.args.quantize_i8 = vnpu.QuantizeI8Args(vnpu.ptr(X), vnpu.ptr(Y), vnpu.ptr(s), rows, cols,
                                             axis, 0)
    return c


def _mm_cmd(A, w, sa, bias, Cout, M, K, N, epi=0):
    c = vnpu.Command()
    c.opcode = vnpu.OP_MATMUL_I8
    c.args.matmul_i8 = vnpu.MatmulI8Args(vnpu.ptr(A), w, vnpu.ptr(sa), vnpu.ptr(bias),
                                         vnpu.ptr(Cout), M, K, N, 0, 0, epi, vnpu.UNIT_GPU)
    return c


def _copy_cmd(dst, src, nbytes):
    c = vnpu.Command()
    c.opcode = vnpu.OP_COPY
    c.args.copy = vnpu.CopyArgs(vnpu.ptr(dst), vnpu.ptr(src), nbytes, 0)
    return c


def test_host_output_feeds_next_command(gpu, oracle):
    """QUANTIZE_I8 writes host A/sa (download), MATMUL_I8 of the same batch
    reads them (upload): the upload waits for the download."""
    rng = np.random.default_rng(21)
    M, K, N = 300, 1024, 768
    X = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    w = gpu.pack(B, sb, K, N)
    try:
        for rep in range(3):
            A = np.zeros((M, K), np.int8)
            sa = np.zeros(M, np.float32)
            Cout = np.full((M, N), np.nan, np.float32)
            X2 = X * (rep + 1)
            assert gpu.submit([_q_cmd(X2, A, sa, M, K), _mm_cmd(A, w, sa, None, Cout, M, K, N)]) \
                == vnpu.OK
            assert gpu.sync() == vnpu.OK
            Ao, sao = oracle.quantize(X2, 0)
            assert bits_equal(A, Ao) and bits_equal(sa, sao)
            assert bits_equal(Cout, oracle.matmul_i8(Ao, B, sao, sb, None, 0, 0))
    finally:
        gpu.unpack(w)


def test_copy_reads_pending_download_and_upload_reads_copy(gpu, b200_lib, oracle):
    """Download -> COPY host->device -> COPY device->host -> upload, one batch."""
    rng = np.random.default_rng(22)
    rows, cols = 256, 2048
    X = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    Y = np.zeros((rows, cols), np.int8)          # host output of cmd 0
    s = np.zeros(rows, np.float32)
    dbuf = vnpu.vp()
    assert b200_lib.buffer_alloc(gpu.dev, rows * cols, C.byref(dbuf)) == vnpu.OK
    dev_ptr = b200_lib.buffer_host_ptr(dbuf)
    Z = np.zeros((rows, cols), np.int8)          # host, written by a COPY on the kernel stream
    X2 = np.zeros((rows, cols), np.float32)      # host input of the last command
    Y2 = np.zeros((rows, cols), np.int8)
    s2 = np.zeros(rows, np.float32)
    try:
        cmds = [_q_cmd(X, Y, s, rows, cols),
                _copy_cmd(dev_ptr, Y, rows * cols),      # reads the pending download
                _copy_cmd(Z, dev_ptr, rows * cols),      # writes host memory on the kernel stream
                _copy_cmd(X2, X, X.nbytes),              # host -> host
                _q_cmd(X2, Y2, s2, rows, cols)]          # uploads what the COPY wrote
        assert gpu.submit(cmds) == vnpu.OK
        assert gpu.sync() == vnpu.OK
        Yo, so = oracle.quantize(X, 0)
        assert bits_equal(Y, Yo) and np.array_equal(Z, Yo)
        assert bits_equal(Y2, Yo) and bits_equal(s2, so)
    finally:
        b200_lib.buffer_free(dbuf)


def test_event_covers_downloads(gpu, b200_lib, oracle):
    rng = np.random.default_rng(23)
    M, K, N = 512, 2048, 4096
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    w = gpu.pack(B, sb, K, N)
    ev = vnpu.vp()
    assert b200_lib.event_create(C.byref(ev)) == vnpu.OK
    try:
        Cout = np.full((M, N), np.nan, np.float32)
        assert gpu.submit([_mm_cmd(A, w, sa, None, Cout, M, K, N)], ev) == vnpu.OK
        assert b200_lib.event_wait(ev, 10000) == vnpu.OK
        # no stream sync: the event alone guarantees the host copy
        assert bits_equal(Cout, oracle.matmul_i8(A, B, sa, sb, None, 0, 0))
    finally:
        b200_lib.event_destroy(ev)
        gpu.unpack(w)


def test_pipelined_steps_with_host_buffers(gpu, oracle):
    """Many QUANTIZE_I8 + MATMUL_I8 steps, each with its own host X and C,
    submitted back to back and synchronised once (uploads of step i+1 overlap
    the download of step i)."""
    rng = np.random.default_rng(24)
    M, K, N, steps = 256, 1024, 1024, 6
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    w = gpu.pack(B, sb, K, N)
    A8 = np.zeros((M, K), np.int8)   # host, reused by every step (WAR/RAW through host)
    sa = np.zeros(M, np.float32)
    Xs = [rng.uniform(-1, 1, (M, K)).astype(np.float32) * (i + 1) for i in range(steps)]
    Cs = [np.full((M, N), np.nan, np.float32) for _ in range(steps)]
    try:
        for i in range(steps):
            assert gpu.submit([_q_cmd(Xs[i], A8, sa, M, K),
                               _mm_cmd(A8, w, sa, None, Cs[i], M, K, N)]) == vnpu.OK
        assert gpu.sync() == vnpu.OK
        for i in range(steps):
            Ao, sao = oracle.quantize(Xs[i], 0)
            assert bits_equal(Cs[i], oracle.matmul_i8(Ao, B, sao, sb, None, 0, 0)), i
    finally:
        gpu.unpack(w)


# ----------------------------------------------------------------- KV_APPEND
def _kv_cmd(K, V, Kc, Vc, mask, position, heads, T, D, cap, pos0):
    return vnpu.b200_command(vnpu.OP_B200_KV_APPEND, vnpu.KvAppendArgs(
        vnpu.ptr(K), vnpu.ptr(V), vnpu.ptr(Kc), vnpu.ptr(Vc), vnpu.ptr(mask), vnpu.ptr(position),
        heads, T, D, cap, pos0, 0))


@pytest.mark.parametrize("T,D,use_pos,with_mask", [(1, 128, True, True), (5, 128, False, True),
                                                   (3, 6, True, False), (1, 13, False, True)])
def test_kv_append(gpu, T, D, use_pos, with_mask):
    """Head-major K/V land in slots pos..pos+T-1 of every head; the mask's
    slots become 0; nothing else changes.  pos from a device int32 or the
    offset field."""
    torch = pytest.importorskip("torch")
    H, cap, pos = 4, 40, 17
    rng = np.random.default_rng(T * 100 + D)
    K = torch.from_numpy(rng.normal(0, 1, (H, T, D)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.normal(0, 1, (H, T, D)).astype(np.float32)).cuda()
    Kc = torch.full((H, cap, D), 7.0, device="cuda")
    Vc = torch.full((H, cap, D), -7.0, device="cuda")
    mask = torch.full((H, cap), float("-inf"), device="cuda") if with_mask else None
    P = torch.tensor([pos], dtype=torch.int32, device="cuda") if use_pos else None
    torch.cuda.synchronize()
    assert gpu.submit([_kv_cmd(K, V, Kc, Vc, mask, P, H, T, D, cap, 0 if use_pos else pos)]) == vnpu.OK
    assert gpu.sync() == vnpu.OK
    Ke = torch.full((H, cap, D), 7.0); Ke[:, pos:pos + T] = K.cpu()
    Ve = torch.full((H, cap, D), -7.0); Ve[:, pos:pos + T] = V.cpu()
    assert torch.equal(Kc.cpu(), Ke) and torch.equal(Vc.cpu(), Ve)
    if with_mask:
        Me = torch.full((H, cap), float("-inf")); Me[:, pos:pos + T] = 0.0
        assert torch.equal(mask.cpu(), Me)


def test_kv_append_past_capacity(b200_lib):
    """A host-known slot past the capacity is refused before launch; a device
    position past it writes nothing and reports a device error (no fault)."""
    torch = pytest.importorskip("torch")
    dev = vnpu.Device(b200_lib)
    try:
        H, T, D, cap = 2, 3, 8, 10
        K = torch.ones((H, T, D), device="cuda")
        Kc = torch.zeros((H, cap, D), device="cuda")
        Vc = torch.zeros((H, cap, D), device="cuda")
        torch.cuda.synchronize()
        assert dev.submit([_kv_cmd(K, K, Kc, Vc, None, None, H, T, D, cap, 8)]) == vnpu.OK
        assert dev.sync() == vnpu.ERR_DEVICE_ERROR          # sticky, as for any failed command
    finally:
        dev.close()
    dev = vnpu.Device(b200_lib)
    try:
        P = torch.tensor([9], dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        assert dev.submit([_kv_cmd(K, K, Kc, Vc, None, P, H, T, D, cap, 0)]) == vnpu.OK
        assert dev.sync() == vnpu.ERR_DEVICE_ERROR
        # slot 9 (in range) was written for t = 0; slots 10, 11 were not
        assert torch.equal(Kc[:, 9].cpu(), torch.ones((H, D))) and Kc[:, :9].abs().sum().item() == 0
    finally:
        dev.close()
