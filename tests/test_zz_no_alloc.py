"""vnpu_b200_quantize_i8_tensor_noalloc: per-tensor QUANTIZE_I8 with its
scratch in a static device array (include/vnpu_b200.h).

Compared bit for bit with the library's vnpu_quantize_i8 (axis PER_TENSOR) on
the same device tensors, on calls made back to back, so a scratch word left
over from one call would show in the next.  The file sorts last so it also
runs after every other GPU test in the same process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu

CHUNK = 1 << 14          # elements per CTA of the absmax pass
LIMIT = CHUNK * (1 << 14)  # 2^28 elements: what the static scratch can hold


@pytest.fixture(scope="module")
def torch():
    return pytest.importorskip("torch")


@pytest.fixture(scope="module")
def noalloc(b200_lib):
    f = b200_lib.h.vnpu_b200_quantize_i8_tensor_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64,
                  C.c_uint64]
    return f


def _noalloc(f, torch, X, rows, cols, Xptr=None):
    Y = torch.empty(rows * cols, dtype=torch.int8, device="cuda")
    s = torch.full((1,), -1.0, device="cuda")
    rc = f(0, torch.cuda.current_stream().cuda_stream,
           Xptr if Xptr is not None else X.data_ptr(), Y.data_ptr(), s.data_ptr(), rows, cols)
    return rc, Y, s


def _existing(gpu, torch, X, rows, cols):
    Y = torch.empty(rows * cols, dtype=torch.int8, device="cuda")
    s = torch.full((1,), -2.0, device="cuda")
    torch.cuda.synchronize()
    gpu.quantize_i8(X, Y, s, rows, cols, vnpu.QUANT_PER_TENSOR)
    assert gpu.sync() == vnpu.OK
    return Y, s


def _check(gpu, torch, f, X, rows, cols):
    rc, Y, s = _noalloc(f, torch, X, rows, cols)
    assert rc == vnpu.OK
    torch.cuda.synchronize()
    Ye, se = _existing(gpu, torch, X, rows, cols)
    assert torch.equal(Y, Ye), (rows, cols)
    assert bits_equal(s.cpu().numpy(), se.cpu().numpy()), (rows, cols, float(s), float(se))
    return Y, s


def test_two_calls_in_a_row_match_existing_entry_point(gpu, torch, noalloc):
    g = torch.Generator(device="cuda").manual_seed(1)
    # First call: large values over 3 chunks + 5, the max in the last chunk.
    r1, c1 = 7, 3 * CHUNK // 7 + 1
    X1 = torch.empty(r1 * c1, device="cuda").normal_(0, 10, generator=g)
    X1[-1] = 900.0
    # Second call right after, on the same stream: smaller magnitudes, so a
    # stale absmax (or completion counter) from the first call would change it.
    r2, c2 = 1000, 333
    X2 = torch.empty(r2 * c2, device="cuda").uniform_(-1, 1, generator=g)
    rc1, Y1, s1 = _noalloc(noalloc, torch, X1, r1, c1)
    rc2, Y2, s2 = _noalloc(noalloc, torch, X2, r2, c2)
    assert rc1 == vnpu.OK and rc2 == vnpu.OK
    torch.cuda.synchronize()
    for X, r, c, Y, s in ((X1, r1, c1, Y1, s1), (X2, r2, c2, Y2, s2)):
        Ye, se = _existing(gpu, torch, X, r, c)
        assert torch.equal(Y, Ye)
        assert bits_equal(s.cpu().numpy(), se.cpu().numpy())
    assert float(s1) == np.float32(900.0) / np.float32(127.0)
    assert float(s2) < 1.0


def test_edge_shapes_and_values(gpu, torch, noalloc, oracle):
    rng = np.random.default_rng(7)
    for rows, cols in ((1, 1), (1, CHUNK), (1, CHUNK + 1), (3, 5), (CHUNK, 2), (129, 257)):
        x = rng.normal(0, 2, rows * cols).astype(np.float32)
        if x.size >= 5:
            # a tie each way, a NaN (never the max), a negative zero, +inf
            x[:5] = [2.5, -2.5, np.nan, -0.0, np.inf]
        X = torch.from_numpy(x).cuda()
        Y, s = _check(gpu, torch, noalloc, X, rows, cols)
        if rows * cols <= 1 << 16:
            Yo, so = oracle.quantize(x.reshape(rows, cols), 2)
            assert np.array_equal(Y.cpu().numpy().reshape(rows, cols), Yo)
            assert bits_equal(s.cpu().numpy(), so)
    # All zeros: scale 1.0 (src/kernels/llm.cpp:421-436 guard).
    Z = torch.zeros(5 * CHUNK, device="cuda")
    Y, s = _check(gpu, torch, noalloc, Z, 5, CHUNK)
    assert float(s) == 1.0 and not Y.any()


def test_unaligned_input(gpu, torch, noalloc):
    g = torch.Generator(device="cuda").manual_seed(3)
    buf = torch.empty(2 * CHUNK + 1, device="cuda").normal_(0, 1, generator=g)
    X = buf[1:]  # 4-byte aligned only
    _check(gpu, torch, noalloc, X, 2, CHUNK)


def test_maximum_size(gpu, torch, noalloc):
    """Exactly the limit (2^28 elements, 1 GiB of f32), the max in the last chunk."""
    rows, cols = 1 << 14, 1 << 14
    g = torch.Generator(device="cuda").manual_seed(4)
    X = torch.empty(rows * cols, device="cuda").uniform_(-3, 3, generator=g)
    X[-7] = -41.0
    Y, s = _check(gpu, torch, noalloc, X, rows, cols)
    assert float(s) == np.float32(41.0) / np.float32(127.0)
    del X, Y
    torch.cuda.empty_cache()


def test_rejections(torch, noalloc):
    X = torch.zeros(16, device="cuda")
    Y = torch.zeros(16, dtype=torch.int8, device="cuda")
    s = torch.zeros(1, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    ok = (X.data_ptr(), Y.data_ptr(), s.data_ptr())
    # Beyond the static scratch: rejected before anything is enqueued.
    assert noalloc(0, st, *ok, LIMIT // 4 + 1, 4) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(0, st, *ok, 1, LIMIT + 1) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(0, st, *ok, 1 << 40, 1 << 40) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(0, st, *ok, 0, 4) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(0, st, None, ok[1], ok[2], 1, 4) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(-1, st, *ok, 1, 4) == vnpu.ERR_INVALID_ARGUMENT
    assert noalloc(4096, st, *ok, 1, 4) == vnpu.ERR_INVALID_ARGUMENT
    host = np.zeros(16, np.float32)
    assert noalloc(0, st, host.ctypes.data, *ok[1:], 1, 16) == vnpu.ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert float(s) == 0.0 and not Y.any()


def test_allocates_no_device_memory(gpu, torch, noalloc):
    """Device memory in use (the driver's count, which a cudaMalloc or a pool
    growth of any library would change) and torch's allocator are the same
    before and after calls made once the scratch is set up on the device."""
    g = torch.Generator(device="cuda").manual_seed(9)
    rows, cols = 300, 7 * CHUNK // 300 + 11
    X = torch.empty(rows * cols, device="cuda").normal_(0, 3, generator=g)
    Y = torch.empty(rows * cols, dtype=torch.int8, device="cuda")
    s = torch.empty(1, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert noalloc(0, st, X.data_ptr(), Y.data_ptr(), s.data_ptr(), rows, cols) == vnpu.OK
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_allocated()
    for _ in range(3):
        assert noalloc(0, st, X.data_ptr(), Y.data_ptr(), s.data_ptr(), rows, cols) == vnpu.OK
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == torch0
    Ye, se = _existing(gpu, torch, X, rows, cols)
    assert torch.equal(Y, Ye) and bits_equal(s.cpu().numpy(), se.cpu().numpy())
