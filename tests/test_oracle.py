"""The C restatement (oracle/) pinned to the reference.

1. Against the committed golden vectors, which the reference library itself
   produced (tests/golden/make_golden.py): every value bit-exact.
2. Against the reference library built from its own sources, when it is
   present (oracle/_ref): fresh seeded inputs, every value bit-exact, for
   both of the reference's ISAs (VNPU_FORCE_ISA=avx2 and scalar) and the
   kernels each shape selects.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import vnpu
from conftest import bits_equal


# ---------------------------------------------------------------- golden vectors
@pytest.mark.parametrize("name,axis", [("row", 0), ("col", 1), ("tensor", 2)])
def test_quantize_golden(oracle, golden, name, axis):
    Y, s = oracle.quantize(golden[f"quant_{name}_X"], axis)
    assert bits_equal(Y, golden[f"quant_{name}_Y"])
    assert bits_equal(s, golden[f"quant_{name}_s"])


def test_quantize_golden_has_ties(golden):
    """The fixture exercises round-half-away-from-zero: 2.5 -> 3, -2.5 -> -3."""
    Y = golden["quant_row_Y"]
    assert Y[0, 3] == 3 and Y[0, 4] == -3 and Y[0, 1] == 1 and Y[0, 2] == -1


@pytest.mark.parametrize("i", range(11))
def test_matmul_golden(oracle, golden, i):
    M, K, N, has_bias, epi = (int(v) for v in golden["mm_cases"][i])
    bias = golden.get(f"mm{i}_bias")
    C = oracle.matmul_i8(golden[f"mm{i}_A"], golden[f"mm{i}_B"], golden[f"mm{i}_sa"],
                         golden[f"mm{i}_sb"], bias, epi, int(golden["mm_forms"][i]))
    assert bits_equal(C, golden[f"mm{i}_C"])


def test_matmul_golden_forms_cover_reference_paths(golden):
    """Bias cases exist for all three forms the reference produces."""
    forms = {int(f) for f, c in zip(golden["mm_forms"], golden["mm_cases"]) if c[3]}
    assert forms == {0, 1, 2}


def test_block_ops_golden(oracle, golden):
    assert bits_equal(oracle.rmsnorm(golden["rms_X"], golden["rms_W"], 1e-6, 0), golden["rms_Y"])
    assert bits_equal(oracle.rmsnorm(golden["rms2_X"], None, 0.0, 0), golden["rms2_Y"])
    Q, K = golden["rope_Q"], golden["rope_K"]
    _, H, T, D = Q.shape
    Qr, Kr = oracle.rope(Q, K, None, 1, H, T, T, D, position_offset=5)
    assert bits_equal(Qr, golden["rope_Qr"]) and bits_equal(Kr, golden["rope_Kr"])
    Qi, _ = oracle.rope(golden["ropei_Q"], None, golden["ropei_pos"], 1, 2, 9, 0, 64,
                        interleaved=1, theta=500000.0, scaling=0.5)
    assert bits_equal(Qi, golden["ropei_Qr"])
    assert bits_equal(oracle.swiglu(golden["swiglu_g"], golden["swiglu_u"], 0.0, 0),
                      golden["swiglu_Y"])
    assert bits_equal(oracle.add(golden["add_A"], golden["add_B"], 0.7, 1.3, 0), golden["add_Y"])


@pytest.mark.parametrize("name", ["attn", "attnd", "attnm"])
def test_attention_golden(oracle, golden, name):
    h, sq, sk, d, causal = (int(v) for v in golden[f"{name}_shape"])
    O = oracle.attention(golden[f"{name}_Q"], golden[f"{name}_K"], golden[f"{name}_V"],
                         golden.get(f"{name}_M"), 1, h, sq, sk, d, causal, 0.0)
    assert bits_equal(O, golden[f"{name}_O"])


def test_fast_expf_properties(oracle):
    """fast_expf (src/internal.h:87-108): cut-offs and 2^n scaling exact."""
    assert oracle.fast_expf(-80.5, 0) == 0.0
    assert oracle.fast_expf(80.5, 0) == float("inf")
    for n in range(-10, 11):
        assert oracle.fast_expf(n * 0.6931471805599453, 0) == pytest.approx(2.0 ** n, rel=2e-4)


def _f32_golden_case(golden, i):
    M, K, N, avx2, thr, pack, unit, ta, tb, epi, tm, tk, tn, mm, mn = (
        int(v) for v in golden["f32_cases"][i])
    alpha, beta = (float(v) for v in golden[f"f32_{i}_ab"])
    return dict(M=M, K=K, N=N, bias=golden.get(f"f32_{i}_bias"), C=golden[f"f32_{i}_C0"],
                trans_a=ta, trans_b=tb, alpha=alpha, beta=beta, epilogue=epi, unit=unit,
                tile_mask=golden.get(f"f32_{i}_mask"), mask_tile_m=mm, mask_tile_n=mn,
                threads=thr, tiles=(tm, tk, tn), pack_b=pack, avx2=avx2)


@pytest.mark.parametrize("i", range(8))
def test_matmul_f32_golden(oracle, golden, i):
    kw = _f32_golden_case(golden, i)
    C = oracle.matmul_f32(golden[f"f32_{i}_A"], golden[f"f32_{i}_B"], **kw)
    assert bits_equal(C, golden[f"f32_{i}_C"])


def test_matmul_f32_golden_needs_the_kernel_map(oracle, golden):
    """The fixtures tell the kernels apart: computing a case as if every
    element took another kernel's rounding changes bits."""
    kw = _f32_golden_case(golden, 0)          # packed panels, K = 260 > 128
    C = oracle.matmul_f32(golden["f32_0_A"], golden["f32_0_B"], **dict(kw, pack_b=0))
    assert not bits_equal(C, golden["f32_0_C"])
    kw = _f32_golden_case(golden, 3)          # B^T dots
    C = oracle.matmul_f32(golden["f32_3_A"], golden["f32_3_B"], **dict(kw, avx2=0))
    assert not bits_equal(C, golden["f32_3_C"])


# ---------------------------------------------------------------- live reference
def _ref_device(ref_lib, isa, threads):
    os.environ["VNPU_FORCE_ISA"] = isa
    try:
        return vnpu.Device(ref_lib, num_threads=threads)
    finally:
        os.environ.pop("VNPU_FORCE_ISA", None)


@pytest.mark.parametrize("isa", ["avx2", "scalar"])
def test_quantize_vs_reference(ref_lib, oracle, isa):
    rng = np.random.default_rng(17)
    with _ref_device(ref_lib, isa, 4) as d:
        for rows, cols in ((1, 1), (5, 333), (64, 4096), (300, 17)):
            X = rng.normal(0, 2, (rows, cols)).astype(np.float32)
            X.flat[: min(4, X.size)] = [0.5, -1.5, np.nan, -0.0][: min(4, X.size)]
            for axis in (0, 1, 2):
                Yo, so = oracle.quantize(X, axis)
                Y = np.empty_like(Yo)
                s = np.empty_like(so)
                d.quantize_i8(X, Y, s, rows, cols, axis)
                assert bits_equal(Y, Yo) and bits_equal(s, so), (rows, cols, axis)


@pytest.mark.parametrize("isa,threads,M,K,N,epi,form", [
    ("avx2", 8, 64, 512, 512, 2, 0),     # packed panel, 2x32 blocks: block form
    ("avx2", 8, 4, 1024, 256, 3, 0),     # decode 64-column packed tiles
    ("avx2", 8, 1, 1024, 512, 2, 2),     # rank-1 stream
    ("avx2", 1, 2, 256, 2048, 1, 2),     # rank-2 stream (column slice >= 1024)
    ("scalar", 4, 37, 129, 70, 2, 1),
    ("scalar", 4, 3, 64, 2048, 4, 1),
])
def test_matmul_vs_reference(ref_lib, oracle, isa, threads, M, K, N, epi, form):
    rng = np.random.default_rng(M * 7 + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    with _ref_device(ref_lib, isa, threads) as d:
        w = d.pack(B, sb, K, N)
        C = np.empty((M, N), np.float32)
        d.matmul_i8(A, w, sa, bias, C, M, K, N, epilogue=epi, unit=vnpu.UNIT_VOODOO)
        d.unpack(w)
    assert bits_equal(C, oracle.matmul_i8(A, B, sa, sb, bias, epi, form))


def test_no_bias_is_form_free(ref_lib, oracle):
    """Without bias and with NONE/RELU every reference path gives one answer."""
    rng = np.random.default_rng(99)
    M, K, N = 19, 47, 31
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    ref = oracle.matmul_i8(A, B, sa, sb, None, 0, 0)
    for form in (1, 2):
        assert bits_equal(oracle.matmul_i8(A, B, sa, sb, None, 0, form), ref)
    for isa in ("avx2", "scalar"):
        for threads in (1, 2):
            with _ref_device(ref_lib, isa, threads) as d:
                w = d.pack(B, sb, K, N)
                for unit in (vnpu.UNIT_AUTO, vnpu.UNIT_VOODOO, vnpu.UNIT_WILDCAT, vnpu.UNIT_CELL):
                    C = np.empty((M, N), np.float32)
                    d.matmul_i8(A, w, sa, None, C, M, K, N, unit=unit)
                    assert bits_equal(C, ref), (isa, threads, unit)
                d.unpack(w)


def test_column_sums_vs_reference(ref_lib, oracle):
    rng = np.random.default_rng(4)
    K, N = 77, 45
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    sums, _ = oracle.column_sums(B)
    with _ref_device(ref_lib, "avx2", 2) as d:
        w = d.pack(B, None, K, N)
        Kr, Nr, _, sc_ptr, cs_ptr = d.packed_info(w)
        import ctypes as C
        cs = np.ctypeslib.as_array(C.cast(cs_ptr, C.POINTER(C.c_int32)), (N,)).copy()
        sc = np.ctypeslib.as_array(C.cast(sc_ptr, C.POINTER(C.c_float)), (N,)).copy()
        d.unpack(w)
    assert (Kr, Nr) == (K, N)
    assert np.array_equal(cs, sums)
    assert np.all(sc == 1.0)  # scales NULL -> 1.0 (src/core/scheduler.cpp:795)


@pytest.mark.parametrize("H,sq,sk,D", [(2, 40, 40, 128), (4, 1, 200, 64), (1, 33, 70, 24)])
def test_block_ops_vs_reference(ref_lib, oracle, H, sq, sk, D):
    rng = np.random.default_rng(H * 1000 + sq + sk)
    with _ref_device(ref_lib, "avx2", 4) as d:
        Q = rng.normal(0, 1, (1, H, sq, D)).astype(np.float32)
        K = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
        V = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
        O = np.empty((1, H, sq, D), np.float32)
        d.attention(Q, K, V, None, O, 1, H, sq, sk, D, 1, 0.0)
        assert bits_equal(O, oracle.attention(Q, K, V, None, 1, H, sq, sk, D, 1, 0.0))
        X = rng.normal(0, 1, (sq, D * 8 + 3)).astype(np.float32)
        Y = np.empty_like(X)
        d.rmsnorm(X, None, Y, X.shape[0], X.shape[1], 1e-6)
        assert bits_equal(Y, oracle.rmsnorm(X, None, 1e-6, 0))


def test_block_driver_host_matches_reference(ref_lib, oracle):
    """The decoder-block driver on host arrays: the oracle restatement and the
    reference library give the same bits for prefill and KV-cached decode."""
    from llm_block import BlockConfig, HostBlock
    cfg = BlockConfig(d=128, heads=4, inter=352, cap=40)
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (9, cfg.d)).astype(np.float32)
    os.environ["VNPU_FORCE_ISA"] = "avx2"
    try:
        ref = HostBlock(cfg, lib=ref_lib, threads=4)
    finally:
        os.environ.pop("VNPU_FORCE_ISA", None)
    orc = HostBlock(cfg, oracle=oracle)
    try:
        assert bits_equal(ref.forward(x, 0), orc.forward(x, 0))
        for p in range(9, 13):
            t = rng.normal(0, 1, (1, cfg.d)).astype(np.float32)
            assert bits_equal(ref.forward(t, p), orc.forward(t, p)), p
    finally:
        ref.close()
        orc.close()


def test_matmul_f32_vs_reference(ref_lib, oracle):
    """Seeded random MATMUL_F32 configurations: every kernel, unit, ISA,
    VNPU_PACK setting, transpose, stride, culling mask and epilogue."""
    rng = np.random.default_rng(5)
    for _ in range(60):
        M = int(rng.choice([1, 3, 5, 8, 9, 31, 64, 97]))
        K = int(rng.integers(1, 300))
        N = int(rng.choice([1, 7, 33, 64, 65, 128, 200]))
        isa = "avx2" if rng.random() < 0.85 else "scalar"
        threads, pack = int(rng.integers(1, 9)), int(rng.random() < 0.7)
        unit = int(rng.choice([0, 1, 2, 3]))
        ta, tb = int(rng.random() < 0.2), int(rng.random() < 0.25)
        beta = float(rng.choice([0.0, 0.7, -1.3]))
        alpha = float(rng.choice([0.0, 1.0, -2.1]))
        epi = int(rng.integers(0, 5))
        pads = [int(rng.choice([0, 3])) for _ in range(3)]
        mask, mtm, mtn = None, 0, 0
        if rng.random() < 0.2:
            mtm, mtn = int(rng.integers(1, 4)), int(rng.integers(1, 4))
            mask = (rng.random(mtm * mtn) < 0.6).astype(np.uint8)
        A = rng.normal(0, 1, (K, M + pads[0]) if ta else (M, K + pads[0])).astype(np.float32)
        B = rng.normal(0, 1, (N, K + pads[1]) if tb else (K, N + pads[1])).astype(np.float32)
        C0 = rng.normal(0, 1, (M, N + pads[2])).astype(np.float32)
        bias = rng.normal(0, 1, N).astype(np.float32) if rng.random() < 0.5 else None
        ld = dict(lda=A.shape[1] if pads[0] else 0, ldb=B.shape[1] if pads[1] else 0,
                  ldc=C0.shape[1] if pads[2] else 0)
        os.environ["VNPU_PACK"] = str(pack)
        try:
            d = _ref_device(ref_lib, isa, threads)
        finally:
            os.environ.pop("VNPU_PACK", None)
        with d:
            info = d.info()
            Cr = C0.copy()
            d.matmul_f32(A, B, Cr, M, K, N, bias=bias, trans_a=ta, trans_b=tb, alpha=alpha,
                         beta=beta, epilogue=epi, unit=unit, tile_mask=mask, mask_tile_m=mtm,
                         mask_tile_n=mtn, **ld)
        resolved = unit if unit else (2 if mask is not None else 1)
        Co = oracle.matmul_f32(A, B, M, K, N, bias=bias, C=C0, trans_a=ta, trans_b=tb, alpha=alpha,
                               beta=beta, epilogue=epi, unit=resolved, tile_mask=mask,
                               mask_tile_m=mtm, mask_tile_n=mtn, threads=info.num_threads,
                               tiles=(info.tile_m, info.tile_k, info.tile_n), pack_b=pack,
                               avx2=int(isa == "avx2"), **ld)
        assert bits_equal(Cr, Co), (M, K, N, isa, threads, pack, unit, ta, tb, alpha, beta, epi)


# ---------------------------------------------------------------- MATMUL_I8 default rounding
def _ref_device_cfg(ref_lib, isa, threads, pack, tiles=None):
    os.environ["VNPU_FORCE_ISA"] = isa
    os.environ["VNPU_PACK"] = str(pack)
    try:
        return vnpu.Device(ref_lib, num_threads=threads, tiles=tiles)
    finally:
        os.environ.pop("VNPU_FORCE_ISA", None)
        os.environ.pop("VNPU_PACK", None)


def test_matmul_i8_device_model_vs_reference(ref_lib, oracle):
    """MATMUL_I8 with no command flags: the reference rounds each output in
    the form of the kernel that owns its tile (block / stream / scalar), which
    its tile geometry picks from M, N, the thread count, the tile defaults and
    VNPU_PACK.  oracle_matmul_i8_device restates that choice element by
    element; seeded shapes cover the rank-1/2/3 streams, packed panels, the
    unpacked 2x32 blocks, column tails, leftover rows, wide decode slices
    whose last slice is narrower than 1024 columns, WILDCAT/CELL units and
    the scalar ISA."""
    rng = np.random.default_rng(11)
    for _ in range(70):
        M = int(rng.choice([1, 2, 3, 4, 5, 7, 8, 9, 11, 16, 31, 33, 64, 130]))
        K = int(rng.choice([16, 64, 200, 4100, 5000]))
        N = int(rng.choice([20, 45, 64, 70, 100, 300, 1030, 2100, 3100]))
        threads = int(rng.integers(1, 5))
        pack = int(rng.random() < 0.75)
        unit = int(rng.choice([0, 1, 1, 1, 2, 3]))
        isa = "avx2" if rng.random() < 0.9 else "scalar"
        tiles = None
        if rng.random() < 0.3:
            tiles = (int(rng.choice([8, 32, 128])), 128, int(rng.choice([16, 40, 64, 100, 2048])))
        epi = int(rng.choice([0, 2, 3]))
        A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
        B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
        bias = rng.normal(0, 0.5, N).astype(np.float32)
        with _ref_device_cfg(ref_lib, isa, threads, pack, tiles) as d:
            info = d.info()
            w = d.pack(B, sb, K, N)
            C = np.empty((M, N), np.float32)
            d.matmul_i8(A, w, sa, bias, C, M, K, N, epilogue=epi, unit=unit)
            d.unpack(w)
        Co = oracle.matmul_i8_device(A, B, sa, sb, bias, epi, unit, info.num_threads,
                                     (info.tile_m, info.tile_k, info.tile_n), pack,
                                     int(isa == "avx2"), info.l2_bytes)
        assert bits_equal(C, Co), (M, K, N, threads, pack, unit, isa, tiles, epi)


def test_matmul_i8_device_model_needs_every_form(oracle):
    """The forms the model assigns differ where the reference's kernels do:
    rank-1 stream for one row, packed blocks with stream / scalar column
    tails, rank-2 stream slices next to a narrow last slice."""
    F = oracle.i8_forms(1, 64, 100, threads=1)
    assert np.all(F == oracle.FORM_STREAM)
    F = oracle.i8_forms(5, 64, 100, threads=1)          # packed, 64-column tiles
    assert F[0, 0] == oracle.FORM_AVX2 and F[0, 97] == oracle.FORM_STREAM
    assert F[4, 97] == oracle.FORM_SCALAR and F[4, 10] == oracle.FORM_AVX2
    F = oracle.i8_forms(2, 64, 3100, threads=3)         # slices 1056, 1056, 988
    assert np.all(F[:, :2112] == oracle.FORM_STREAM)
    assert F[0, 2112] == oracle.FORM_AVX2 and F[1, 3099] == oracle.FORM_STREAM
    F = oracle.i8_forms(3, 5000, 40, threads=1)         # packed (K x 40 fits the scratch)
    assert F[2, 0] == oracle.FORM_AVX2 and F[2, 39] == oracle.FORM_SCALAR
    F = oracle.i8_forms(3, 8192, 40, threads=1)         # unpacked: the odd row streams
    assert np.all(F[2] == oracle.FORM_STREAM) and F[0, 0] == oracle.FORM_AVX2


@pytest.mark.parametrize("M", [1, 4, 8])
def test_matmul_i8_decode_config_vs_reference(ref_lib, oracle, M):
    """The decode GEMV configuration (M in {1,4,8}, K = N = 4096, bias
    N(0, 0.01)) through the reference with no flags, against the model."""
    rng = np.random.default_rng(100 + M)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, 4096)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (4096, 4096)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, 4096).astype(np.float32)
    for threads in (4, 16):
        with _ref_device_cfg(ref_lib, "avx2", threads, 1) as d:
            info = d.info()
            w = d.pack(B, sb, 4096, 4096)
            C = np.empty((M, 4096), np.float32)
            d.matmul_i8(A, w, sa, bias, C, M, 4096, 4096)
            d.unpack(w)
        Co = oracle.matmul_i8_device(A, B, sa, sb, bias, 0, 0, info.num_threads,
                                     (info.tile_m, info.tile_k, info.tile_n), 1, 1, info.l2_bytes)
        assert bits_equal(C, Co), (M, threads)
