"""Generate tests/golden/golden.npz from the reference library itself.

Runs the reference implementation built from its own sources
(``make -C oracle ref REF=<reference checkout>`` -> oracle/_ref/libvnpu_ref.so)
through its public C ABI on seeded inputs and stores inputs and outputs.
The fixtures pin both the CPU restatement (oracle/oracle.c) and the B200
kernels to the reference's actual behaviour; the tests never need the
reference itself at run time.

For MATMUL_I8 with a bias or an activation, the reference's last bits depend
on which of its kernels ran (see vnpu_b200.h: block / stream / scalar forms);
each such case records the form it was produced with, established here by
comparing against the three restated forms.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "npuxl-improved_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import vnpu  # noqa: E402

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libvnpu_ref.so")
ORACLE_LIB = os.path.join(ROOT, "oracle", "liboracle.so")
FORMS = {"block": 0, "scalar": 1, "stream": 2}


def ref_device(lib, isa: str, threads: int):
    os.environ["VNPU_FORCE_ISA"] = isa
    return vnpu.Device(lib, num_threads=threads)


def which_form(orc, out, A, B, sa, sb, bias, epi):
    hits = []
    for name, form in FORMS.items():
        o = orc.matmul_i8(A, B, sa, sb, bias, epi, form)
        if np.array_equal(o.view(np.uint32), out.view(np.uint32)):
            hits.append(name)
    return hits


def main():
    lib = vnpu.Lib(REF_LIB)
    from vnpu_oracle import Oracle
    orc = Oracle(ORACLE_LIB)
    rng = np.random.default_rng(20261201)
    g = {}

    # ---- QUANTIZE_I8 -----------------------------------------------------
    d = ref_device(lib, "avx2", 4)
    for name, (r, c, axis) in {"row": (37, 300, 0), "col": (64, 48, 1), "tensor": (19, 47, 2)}.items():
        X = rng.uniform(-1, 1, (r, c)).astype(np.float32)
        # exact .5 ties after scaling: round half away from zero must show
        X[0, :6] = [1.0, 0.5 / 127, -0.5 / 127, 2.5 / 127, -2.5 / 127, 0.0]
        X[1, :3] = [np.float32(3.0), np.float32(-3.0), np.float32(1.5)]
        Y = np.empty((r, c), np.int8)
        n = r if axis == 0 else (c if axis == 1 else 1)
        s = np.empty(n, np.float32)
        d.quantize_i8(X, Y, s, r, c, axis)
        g[f"quant_{name}_X"], g[f"quant_{name}_Y"], g[f"quant_{name}_s"] = X, Y, s
    d.close()

    # ---- MATMUL_I8 ---------------------------------------------------------
    # (M, K, N, isa, threads, with_bias, epilogue)
    cases = [
        (19, 47, 31, "avx2", 2, False, 0),     # conformance shape
        (64, 256, 128, "avx2", 2, False, 0),   # conformance shape
        (1, 160, 1376, "avx2", 2, False, 0),   # conformance N, shorter K
        (130, 200, 300, "avx2", 8, False, 1),  # ragged, RELU
        (64, 256, 256, "avx2", 8, True, 0),    # register-block kernels: block form
        (64, 256, 256, "avx2", 8, True, 2),    # ... with SiLU
        (1, 512, 256, "avx2", 8, True, 0),     # decode rank-1 stream: stream form
        (8, 256, 256, "avx2", 8, True, 3),     # decode packed tile, GELU
        (3, 128, 1024, "avx2", 1, True, 2),    # rank-3 stream
        (40, 96, 72, "scalar", 2, True, 2),    # VNPU_FORCE_ISA=scalar
        (5, 300, 200, "scalar", 2, True, 4),   # GELU_ERF aliases tanh
    ]
    g["mm_cases"] = np.array([[M, K, N, int(b), e] for (M, K, N, _, _, b, e) in cases], np.int64)
    forms = []
    for i, (M, K, N, isa, th, with_bias, epi) in enumerate(cases):
        Af = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        Bf = rng.normal(0, 0.02, (K, N)).astype(np.float32)
        A, sa = orc.quantize(Af, 0)
        B, sb = orc.quantize(Bf, 1)
        bias = rng.normal(0, 0.01, N).astype(np.float32) if with_bias else None
        d = ref_device(lib, isa, th)
        w = d.pack(B, sb, K, N)
        C = np.empty((M, N), np.float32)
        d.matmul_i8(A, w, sa, bias, C, M, K, N, epilogue=epi, unit=vnpu.UNIT_VOODOO)
        d.unpack(w)
        d.close()
        hits = which_form(orc, C, A, B, sa, sb, bias, epi)
        if not hits:
            raise SystemExit(f"case {i}: reference output matches no restated form")
        forms.append(FORMS[hits[0]])
        g[f"mm{i}_A"], g[f"mm{i}_B"], g[f"mm{i}_sa"], g[f"mm{i}_sb"] = A, B, sa, sb
        if bias is not None:
            g[f"mm{i}_bias"] = bias
        g[f"mm{i}_C"] = C
        print(f"matmul case {i} {M}x{K}x{N} {isa}/t{th} bias={with_bias} epi={epi}: forms {hits}")
    g["mm_forms"] = np.array(forms, np.int64)

    # ---- block ops (AVX2 build) ----------------------------------------------
    d = ref_device(lib, "avx2", 4)
    X = rng.normal(0, 1, (3, 4096)).astype(np.float32)
    W = rng.normal(1, 0.1, 4096).astype(np.float32)
    Y = np.empty_like(X)
    d.rmsnorm(X, W, Y, 3, 4096, 1e-6)
    g["rms_X"], g["rms_W"], g["rms_Y"] = X, W, Y
    X2 = rng.normal(0, 1, (2, 1003)).astype(np.float32)  # ragged tail, no weight
    Y2 = np.empty_like(X2)
    d.rmsnorm(X2, None, Y2, 2, 1003, 0.0)
    g["rms2_X"], g["rms2_Y"] = X2, Y2

    H, T, D = 2, 21, 128
    Q = rng.normal(0, 1, (1, H, T, D)).astype(np.float32)
    K = rng.normal(0, 1, (1, H, T, D)).astype(np.float32)
    Qr, Kr = Q.copy(), K.copy()
    d.rope(Qr, Kr, None, 1, H, T, T, D, position_offset=5)
    g["rope_Q"], g["rope_K"], g["rope_Qr"], g["rope_Kr"] = Q, K, Qr, Kr
    pos = (np.arange(9, dtype=np.int32) * 7 + 500).astype(np.int32)
    Qi = rng.normal(0, 1, (1, 2, 9, 64)).astype(np.float32)
    Qir = Qi.copy()
    d.rope(Qir, None, pos, 1, 2, 9, 0, 64, interleaved=1, theta=500000.0, scaling=0.5)
    g["ropei_Q"], g["ropei_pos"], g["ropei_Qr"] = Qi, pos, Qir

    gate = rng.normal(0, 3, 11008 + 5).astype(np.float32)
    gate[:4] = [-90.0, 90.0, -85.0, 85.0]
    up = rng.normal(0, 1, gate.size).astype(np.float32)
    Ys = np.empty_like(gate)
    d.swiglu(gate, up, Ys, gate.size, 0.0)
    g["swiglu_g"], g["swiglu_u"], g["swiglu_Y"] = gate, up, Ys

    a = rng.normal(0, 1, 4099).astype(np.float32)
    b = rng.normal(0, 1, 4099).astype(np.float32)
    Ya = np.empty_like(a)
    d.add(a, b, Ya, a.size, 0.7, 1.3)
    g["add_A"], g["add_B"], g["add_Y"] = a, b, Ya

    for name, (h, sq, sk, dd, causal, masked) in {
        "attn": (2, 37, 42, 128, 1, False),
        "attnd": (2, 1, 100, 128, 1, False),      # decode: one query, long cache
        "attnm": (2, 20, 20, 48, 0, True),        # additive mask, head_dim % 8 != 0 tail free
    }.items():
        Qa = rng.normal(0, 1, (1, h, sq, dd)).astype(np.float32)
        Ka = rng.normal(0, 1, (1, h, sk, dd)).astype(np.float32)
        Va = rng.normal(0, 1, (1, h, sk, dd)).astype(np.float32)
        Ma = rng.normal(0, 1, (1, h, sq, sk)).astype(np.float32) if masked else None
        Oa = np.empty((1, h, sq, dd), np.float32)
        d.attention(Qa, Ka, Va, Ma, Oa, 1, h, sq, sk, dd, causal, 0.0)
        g[f"{name}_Q"], g[f"{name}_K"], g[f"{name}_V"], g[f"{name}_O"] = Qa, Ka, Va, Oa
        if Ma is not None:
            g[f"{name}_M"] = Ma
        g[f"{name}_shape"] = np.array([h, sq, sk, dd, causal], np.int64)
    d.close()

    # ---- MATMUL_F32 (the GEMM behind the legacy virtual_npu/vgpu_npu shims)
    # Which reference kernel owns an element depends on the device's thread
    # count, tile defaults, VNPU_PACK, the unit and the transposes; the cases
    # cover every kernel (packed panels, register blocks + row stream, B^T
    # dots with ragged tails, scalar A^T, Cell, scalar ISA, Wildcat culling).
    frng = np.random.default_rng(20261202)
    f32_cases = [
        # M, K, N, isa, threads, pack, unit, ta, tb, bias, alpha, beta, epi, mask
        (48, 260, 256, "avx2", 2, 1, 1, 0, 0, 1, 1.0, 0.0, 0, None),
        (40, 200, 130, "avx2", 8, 0, 1, 0, 0, 1, 1.5, 0.7, 2, None),
        (5, 257, 100, "avx2", 8, 1, 1, 0, 0, 0, 1.0, 0.0, 0, None),
        (37, 131, 70, "avx2", 3, 1, 1, 0, 1, 1, 1.3, 0.7, 3, None),
        (33, 90, 50, "avx2", 4, 1, 1, 1, 0, 1, 1.0, -1.3, 1, None),
        (30, 100, 90, "avx2", 4, 1, 3, 0, 0, 1, 0.75, 0.7, 2, None),
        (31, 77, 45, "scalar", 4, 1, 1, 0, 0, 1, 1.0, 0.7, 2, None),
        (100, 64, 200, "avx2", 2, 1, 2, 0, 0, 1, 1.0, 0.5, 0, (3, 2)),
    ]
    rows = []
    for i, (M, K, N, isa, thr, pack, unit, ta, tb, has_bias, alpha, beta, epi,
            mask) in enumerate(f32_cases):
        A = frng.normal(0, 1, (K, M) if ta else (M, K)).astype(np.float32)
        B = frng.normal(0, 1, (N, K) if tb else (K, N)).astype(np.float32)
        bias = frng.normal(0, 1, N).astype(np.float32) if has_bias else None
        C0 = frng.normal(0, 1, (M, N)).astype(np.float32)
        tm = frng.integers(0, 2, mask[0] * mask[1]).astype(np.uint8) if mask else None
        os.environ["VNPU_PACK"] = str(pack)
        d = ref_device(lib, isa, thr)
        os.environ.pop("VNPU_PACK")
        info = d.info()
        Cr = C0.copy()
        d.matmul_f32(A, B, Cr, M, K, N, bias=bias, trans_a=ta, trans_b=tb, alpha=alpha, beta=beta,
                     epilogue=epi, unit=unit, tile_mask=tm, mask_tile_m=mask[0] if mask else 0,
                     mask_tile_n=mask[1] if mask else 0)
        d.close()
        g[f"f32_{i}_A"], g[f"f32_{i}_B"], g[f"f32_{i}_C0"], g[f"f32_{i}_C"] = A, B, C0, Cr
        if bias is not None:
            g[f"f32_{i}_bias"] = bias
        if tm is not None:
            g[f"f32_{i}_mask"] = tm
        rows.append([M, K, N, int(isa == "avx2"), info.num_threads, pack, unit, ta, tb, epi,
                     info.tile_m, info.tile_k, info.tile_n, mask[0] if mask else 0,
                     mask[1] if mask else 0])
        g[f"f32_{i}_ab"] = np.array([alpha, beta], np.float32)
    g["f32_cases"] = np.array(rows, np.int64)

    out = os.path.join(HERE, "golden.npz")
    np.savez_compressed(out, **g)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
