"""MATMUL_F32 on the B200 (CUDA-core kernels) against the reference's bits.

The reference's F32 GEMM rounds each output the way the CPU kernel owning
its tile does (src/kernels/kernels.cpp:19-352,480-520), and the tile map
depends on the device configuration (thread count, tile defaults, VNPU_PACK,
ISA; src/core/scheduler.cpp:95-207).  Each test configures the B200 device
like the reference device it compares with and asserts bit equality: against
the committed golden outputs of the reference itself, then against the
oracle restatement on seeded shapes, host and device operands.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu


def b200_device(lib, threads, tiles=None, pack=1, scalar=False):
    saved = {k: os.environ.pop(k, None) for k in ("VNPU_PACK", "VNPU_FORCE_ISA")}
    os.environ["VNPU_PACK"] = str(pack)
    if scalar:
        os.environ["VNPU_FORCE_ISA"] = "scalar"
    try:
        return vnpu.Device(lib, num_threads=threads, tiles=tiles)
    finally:
        for k, v in saved.items():
            os.environ.pop(k, None)
            if v is not None:
                os.environ[k] = v


@pytest.mark.parametrize("i", range(8))
def test_golden(b200_lib, golden, i):
    M, K, N, avx2, thr, pack, unit, ta, tb, epi, tm, tk, tn, mm, mn = (
        int(v) for v in golden["f32_cases"][i])
    alpha, beta = (float(v) for v in golden[f"f32_{i}_ab"])
    with b200_device(b200_lib, thr, (tm, tk, tn), pack, scalar=not avx2) as d:
        C = golden[f"f32_{i}_C0"].copy()
        d.matmul_f32(golden[f"f32_{i}_A"], golden[f"f32_{i}_B"], C, M, K, N,
                     bias=golden.get(f"f32_{i}_bias"), trans_a=ta, trans_b=tb, alpha=alpha,
                     beta=beta, epilogue=epi, unit=unit, tile_mask=golden.get(f"f32_{i}_mask"),
                     mask_tile_m=mm, mask_tile_n=mn)
    assert bits_equal(C, golden[f"f32_{i}_C"])


def _case(rng, M, K, N, ta=0, tb=0, pads=(0, 0, 0)):
    A = rng.normal(0, 1, (K, M + pads[0]) if ta else (M, K + pads[0])).astype(np.float32)
    B = rng.normal(0, 1, (N, K + pads[1]) if tb else (K, N + pads[1])).astype(np.float32)
    C0 = rng.normal(0, 1, (M, N + pads[2])).astype(np.float32)
    ld = dict(lda=A.shape[1] if pads[0] else 0, ldb=B.shape[1] if pads[1] else 0,
              ldc=C0.shape[1] if pads[2] else 0)
    return A, B, C0, ld


def test_seeded_sweep_host_operands(b200_lib, oracle):
    """Every form, unit, transpose, stride, mask and epilogue; operands in
    host memory (staged through HBM by the stream)."""
    rng = np.random.default_rng(21)
    for _ in range(40):
        M = int(rng.choice([1, 3, 5, 8, 9, 31, 64, 130, 257]))
        K = int(rng.integers(1, 400))
        N = int(rng.choice([1, 7, 33, 64, 65, 128, 200, 300]))
        scalar = rng.random() < 0.15
        threads, pack = int(rng.integers(1, 9)), int(rng.random() < 0.7)
        unit = int(rng.choice([0, 1, 2, 3]))
        ta, tb = int(rng.random() < 0.2), int(rng.random() < 0.25)
        beta = float(rng.choice([0.0, 0.7, -1.3]))
        alpha = float(rng.choice([0.0, 1.0, -2.1]))
        epi = int(rng.integers(0, 5))
        pads = tuple(int(rng.choice([0, 3])) for _ in range(3))
        mask, mtm, mtn = None, 0, 0
        if rng.random() < 0.2:
            mtm, mtn = int(rng.integers(1, 4)), int(rng.integers(1, 4))
            mask = (rng.random(mtm * mtn) < 0.6).astype(np.uint8)
        A, B, C0, ld = _case(rng, M, K, N, ta, tb, pads)
        bias = rng.normal(0, 1, N).astype(np.float32) if rng.random() < 0.5 else None
        tiles = (32, 64, 32) if scalar else (128, 128, 64)
        with b200_device(b200_lib, threads, tiles, pack, scalar) as d:
            C = C0.copy()
            d.matmul_f32(A, B, C, M, K, N, bias=bias, trans_a=ta, trans_b=tb, alpha=alpha,
                         beta=beta, epilogue=epi, unit=unit, tile_mask=mask, mask_tile_m=mtm,
                         mask_tile_n=mtn, **ld)
        resolved = unit if unit else (2 if mask is not None else 1)
        Co = oracle.matmul_f32(A, B, M, K, N, bias=bias, C=C0, trans_a=ta, trans_b=tb,
                               alpha=alpha, beta=beta, epilogue=epi, unit=resolved,
                               tile_mask=mask, mask_tile_m=mtm, mask_tile_n=mtn,
                               threads=threads, tiles=tiles, pack_b=pack, avx2=int(not scalar),
                               **ld)
        assert bits_equal(C, Co), (M, K, N, scalar, threads, pack, unit, ta, tb, alpha, beta, epi)


@pytest.mark.parametrize("M,K,N,ta,tb,threads", [
    (1024, 1000, 768, 0, 0, 8),     # packed panels, 8 panel folds
    (600, 777, 520, 0, 0, 16),      # register-block map (few tiles per thread)
    (700, 300, 333, 0, 1, 8),       # B^T dots, K % 8 = 4
    (333, 515, 640, 1, 0, 8),       # A^T: unfused chains
])
def test_large_device_operands(gpu, b200_lib, oracle, M, K, N, ta, tb, threads):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(M + K + N)
    A, B, C0, _ = _case(rng, M, K, N, ta, tb)
    bias = rng.normal(0, 1, N).astype(np.float32)
    dA, dB, dC, dbias = (torch.from_numpy(x).cuda() for x in (A, B, C0, bias))
    with b200_device(b200_lib, threads) as d:
        d.matmul_f32(dA, dB, dC, M, K, N, bias=dbias, trans_a=ta, trans_b=tb, alpha=0.5,
                     beta=0.25, epilogue=vnpu.EPI_SILU)
    Co = oracle.matmul_f32(A, B, M, K, N, bias=bias, C=C0, trans_a=ta, trans_b=tb, alpha=0.5,
                           beta=0.25, epilogue=vnpu.EPI_SILU, threads=threads)
    assert bits_equal(dC.cpu().numpy(), Co)


def test_rejections(b200_lib):
    """Invalid arguments fail the command like the reference's
    prepare_matmul_f32 (src/core/scheduler.cpp:280-299)."""
    A = np.zeros((4, 4), np.float32)
    C = np.zeros((4, 4), np.float32)
    for kw in (dict(lda=2), dict(ldc=3), dict(trans_a=2), dict(epilogue=9)):
        with vnpu.Device(b200_lib) as d:
            assert d.matmul_f32(A, A, C, 4, 4, 4, check=False, **kw) != vnpu.OK, kw
    with vnpu.Device(b200_lib) as d:
        assert d.matmul_f32(A, None, C, 4, 4, 4, check=False) != vnpu.OK
    with vnpu.Device(b200_lib) as d:
        assert d.matmul_f32(A, A, C, 0, 4, 4, check=False) != vnpu.OK
