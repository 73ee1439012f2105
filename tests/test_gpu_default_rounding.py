"""MATMUL_I8 with no command flags gives the reference's bits.

The reference device rounds the dequant epilogue (bias add, SiLU / GELU
polynomial) of each output element in the form of the CPU kernel that owns
the element's tile (src/kernels/kernels.cpp:922-978), and its tile grid
follows from M, N, its worker-thread count, its tile defaults and VNPU_PACK
(src/core/scheduler.cpp:75-207).  A B200 device models the reference device
of the same configuration (vnpu_b200_reference_model) and every int8 GEMM
kernel rounds each element in that element's form.

Each case runs the B200 library with no flags and compares the bits with
  * the reference library built from its own sources (oracle/_ref), run with
    the same configuration on the same inputs, where the shape is small
    enough for the host CPU, and
  * the oracle's restatement of the reference device (pinned to the
    reference by tests/test_oracle.py), on row samples at full size.
Tolerance: 0 ulp (bit-exact) throughout.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import vnpu
from conftest import REF_LIB, bits_equal, ulp_diff

pytestmark = pytest.mark.gpu


def _device(b200_lib, threads=0, tiles=None, pack=None):
    if pack is not None:
        os.environ["VNPU_PACK"] = str(pack)
    try:
        return vnpu.Device(b200_lib, num_threads=threads, ordinal=0, tiles=tiles)
    finally:
        os.environ.pop("VNPU_PACK", None)


def _reference_run(model, A, B, sa, sb, bias, epi, unit=0, lda=0):
    """The reference library with the configuration `model` describes, or
    None when it is not built here."""
    if not os.path.exists(REF_LIB):
        return None
    lib = vnpu.Lib(REF_LIB)
    os.environ["VNPU_FORCE_ISA"] = "scalar" if model.scalar_isa else "avx2"
    os.environ["VNPU_PACK"] = str(model.pack_b)
    try:
        d = vnpu.Device(lib, num_threads=model.num_threads,
                        tiles=(model.tile_m, model.tile_k, model.tile_n))
    finally:
        os.environ.pop("VNPU_FORCE_ISA", None)
        os.environ.pop("VNPU_PACK", None)
    M = A.shape[0]
    K, N = B.shape
    with d:
        assert d.info().num_threads == model.num_threads
        w = d.pack(B, sb, K, N)
        C = np.empty((M, N), np.float32)
        d.matmul_i8(A, w, sa, bias, C, M, K, N, lda=lda, epilogue=epi, unit=unit)
        d.unpack(w)
    return C


def _b200_run(dev, A, B, sa, sb, bias, epi, unit=0, lda=0, M=None):
    M = M if M is not None else A.shape[0]
    K, N = B.shape
    w = dev.pack(B, sb, K, N)
    try:
        C = np.full((M, N), np.nan, np.float32)
        dev.matmul_i8(A, w, sa, bias, C, M, K, N, lda=lda, epilogue=epi, unit=unit)
        kernel = dev.lib.b200_last_matmul_kernel().decode()
    finally:
        dev.unpack(w)
    return C, kernel


def _check(dev, oracle, A, B, sa, sb, bias, epi, unit=0, with_reference=True):
    C, kernel = _b200_run(dev, A, B, sa, sb, bias, epi, unit)
    model = dev.reference_model()
    want = oracle.matmul_i8_model(model, A, B, sa, sb, bias, epi, unit=unit)
    assert bits_equal(C, want), f"{kernel}: max ulp {ulp_diff(C, want)}"
    if with_reference:
        ref = _reference_run(model, A, B, sa, sb, bias, epi, unit)
        if ref is not None:
            assert bits_equal(C, ref), f"{kernel} vs reference: max ulp {ulp_diff(C, ref)}"
    return kernel


# ----------------------------------------------------------------- BASELINE configurations
def test_config1_512_cube(b200_lib, oracle):
    """512^3, A U[-1,1] seed 0 quantized per row, B N(0,0.02)
    seed 1 quantized per column, no bias, epilogue NONE; and the same
    operands with a bias and SiLU, where the forms differ."""
    A, sa = oracle.quantize(np.random.default_rng(0).uniform(-1, 1, (512, 512)).astype(np.float32), 0)
    B, sb = oracle.quantize(np.random.default_rng(1).normal(0, 0.02, (512, 512)).astype(np.float32), 1)
    bias = np.random.default_rng(2).normal(0, 0.01, 512).astype(np.float32)
    with _device(b200_lib) as dev:
        _check(dev, oracle, A, B, sa, sb, None, vnpu.EPI_NONE)
        _check(dev, oracle, A, B, sa, sb, bias, vnpu.EPI_SILU)


@pytest.mark.parametrize("M", [1, 4, 8])
def test_config2_decode(b200_lib, oracle, M):
    """M in {1,4,8}, K = N = 4096, A U[-1,1], B N(0,0.02), bias
    N(0,0.01): M = 1 is the reference's rank-1 stream, M = 4 / 8 its packed
    64-column tiles."""
    rng = np.random.default_rng(40 + M)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, 4096)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (4096, 4096)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, 4096).astype(np.float32)
    with _device(b200_lib) as dev:
        _check(dev, oracle, A, B, sa, sb, bias, vnpu.EPI_NONE)
        _check(dev, oracle, A, B, sa, sb, bias, vnpu.EPI_SILU)


def test_config3_ffn_rows(b200_lib, oracle):
    """4096 x 4096 x 14336, A N(0,1), B N(0,0.02), SiLU; row
    samples against the model of the whole product."""
    rng = np.random.default_rng(3)
    M, K, N = 4096, 4096, 14336
    A, sa = oracle.quantize(rng.normal(0, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    rows = np.arange(5, M, 331)
    with _device(b200_lib) as dev:
        for bias in (None, rng.normal(0, 0.01, N).astype(np.float32)):
            C, kernel = _b200_run(dev, A, B, sa, sb, bias, vnpu.EPI_SILU)
            want = oracle.matmul_i8_model(dev.reference_model(), A, B, sa, sb, bias,
                                          vnpu.EPI_SILU, rows=rows)
            assert bits_equal(C[rows], want), f"{kernel}: max ulp {ulp_diff(C[rows], want)}"


def test_config5_shard_widths(b200_lib, oracle, monkeypatch):
    """8192 x 8192 x N for the whole weight (N = 28672) and the
    shard each of 2 / 4 / 8 GPUs holds (14336 / 7168 / 3584 columns), A
    U[-1,1], B N(0,0.02); row samples of every shard, through the kernel the
    dispatcher picks and through the other tcgen05 pair kernel."""
    rng = np.random.default_rng(5)
    M = K = 8192
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    Bfull, sbfull = oracle.quantize(rng.normal(0, 0.02, (K, 28672)).astype(np.float32), 1)
    rows = np.arange(3, M, 1021)
    kernels = set()
    with _device(b200_lib) as dev:
        for N in (28672, 14336, 7168, 3584):
            B = np.ascontiguousarray(Bfull[:, :N])
            sb = np.ascontiguousarray(sbfull[:N])
            want = oracle.matmul_i8(A[rows], B, sa[rows], sb, None, 0, 0)
            for wide in (None, "1", "0"):
                if wide is None:
                    monkeypatch.delenv("VNPU_B200_PAIR_WIDE", raising=False)
                else:
                    monkeypatch.setenv("VNPU_B200_PAIR_WIDE", wide)
                C, kernel = _b200_run(dev, A, B, sa, sb, None, vnpu.EPI_NONE)
                kernels.add(kernel)
                assert bits_equal(C[rows], want), (N, wide, kernel)
    monkeypatch.delenv("VNPU_B200_PAIR_WIDE", raising=False)
    assert {"gemm_i8_tcgen05_pair_wide_kernel", "gemm_i8_tcgen05_pair_kernel"} <= kernels


# ----------------------------------------------------------------- mixed forms, every kernel
@pytest.mark.parametrize("M,K,N,threads,tiles,pack,unit,epi", [
    (2, 64, 3100, 3, None, 1, 0, 2),        # rank-2 slices beside a narrow last slice (GEMV)
    (2, 300, 2000, 2, None, 1, 0, 3),       # narrow tiles: row-pair blocks, a 16-column tail
    (3, 8192, 40, 1, None, 1, 0, 2),        # unpacked: the odd row streams (tensor-core GEMV)
    (5, 64, 100, 1, None, 1, 0, 2),         # packed: stream / scalar column tails
    (7, 4096, 70, 2, None, 1, 1, 3),        # packed 64-column tiles, odd row, 6-column tail
    (37, 8192, 300, 4, None, 1, 0, 2),      # single-CTA tcgen05: odd rows unpacked, tails
    (301, 4100, 700, 16, None, 1, 0, 2),    # pair kernel: 45-row last tile, tails
    (257, 8192, 700, 16, None, 1, 0, 3),    # split K: one-row last tile, tails
    (64, 256, 500, 2, (128, 128, 100), 0, 0, 2),   # 100-column tiles: a tail in every tile
    (100, 256, 300, 2, None, 1, 2, 2),      # WILDCAT tiles
    (100, 256, 300, 2, None, 1, 3, 2),      # CELL: scalar throughout
])
def test_mixed_forms(b200_lib, oracle, M, K, N, threads, tiles, pack, unit, epi):
    rng = np.random.default_rng(M * 31 + N + K)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    with _device(b200_lib, threads, tiles, pack) as dev:
        model = dev.reference_model()
        assert model.num_threads == threads and model.pack_b == pack
        if unit != 3:
            F = oracle.i8_forms(M, K, N, unit or 1, threads,
                                (model.tile_m, model.tile_k, model.tile_n), pack)
            assert len(np.unique(F)) > 1, "case does not mix forms"
        _check(dev, oracle, A, B, sa, sb, bias, epi, unit)


def test_mixed_forms_unaligned_rows(b200_lib, oracle):
    """Rows of A at a stride that is not a multiple of 16 take the SIMT
    kernel; its epilogue follows the same map."""
    rng = np.random.default_rng(77)
    M, K, N, lda = 150, 320, 300, 325
    Abuf = rng.integers(-128, 128, (M, lda), dtype=np.int8)
    A = np.ascontiguousarray(Abuf[:, :K])
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    with _device(b200_lib, 2) as dev:
        w = dev.pack(B, sb, K, N)
        try:
            C = np.full((M, N), np.nan, np.float32)
            dev.matmul_i8(Abuf, w, sa, bias, C, M, K, N, lda=lda, epilogue=vnpu.EPI_SILU)
            assert dev.lib.b200_last_matmul_kernel().decode() == "gemm_i8_simt_kernel"
        finally:
            dev.unpack(w)
        want = oracle.matmul_i8_model(dev.reference_model(), A, B, sa, sb, bias, vnpu.EPI_SILU)
        assert bits_equal(C, want)
        ref = _reference_run(dev.reference_model(), Abuf, B, sa, sb, bias, vnpu.EPI_SILU, lda=lda)
        if ref is not None:
            assert bits_equal(C, ref)


def test_forced_forms_override(b200_lib, oracle):
    """The command flags still force one form for every element."""
    rng = np.random.default_rng(9)
    M, K, N = 5, 64, 100
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    with _device(b200_lib, 1) as dev:
        w = dev.pack(B, sb, K, N)
        try:
            for form, flag in vnpu.FORM_FLAGS.items():
                C = np.full((M, N), np.nan, np.float32)
                dev.matmul_i8(A, w, sa, bias, C, M, K, N, epilogue=vnpu.EPI_SILU, flags=flag)
                assert bits_equal(C, oracle.matmul_i8(A, B, sa, sb, bias, vnpu.EPI_SILU, form))
        finally:
            dev.unpack(w)
