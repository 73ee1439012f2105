"""Parity of the B200 kernels with the reference, through the C ABI.

Bar (north star): int32 accumulators and QUANTIZE_I8 codes bit-exact; the
dequantised f32 GEMM output bit-exact for the same epilogue form (tolerance
0 ulp, which is inside the stated 1 ulp); f32 block ops within 1e-4 relative /
1e-5 absolute (the kernels restate the reference's operation order, so most
are checked at 0 ulp, RoPE within 4 ulp because it uses the device sinf/cosf).

Checked against the committed golden vectors (produced by the reference
library itself) and against the C restatement in oracle/ on fresh seeded
inputs, including ragged shapes, strides and the three GEMM kernels.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import vnpu
from conftest import bits_equal, ulp_diff

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5


@pytest.fixture
def force_kernel():
    """Pin the MATMUL_I8 kernel choice for one test."""
    def _set(name):
        if name:
            os.environ["VNPU_B200_FORCE_KERNEL"] = name
        else:
            os.environ.pop("VNPU_B200_FORCE_KERNEL", None)
    yield _set
    os.environ.pop("VNPU_B200_FORCE_KERNEL", None)


def run_matmul(dev, A, B, sa, sb, bias, epi, form=0, lda=0, ldc=0, Cbuf=None, M=None, K=None,
               N=None):
    K = K if K is not None else B.shape[0]
    N = N if N is not None else B.shape[1]
    M = M if M is not None else A.shape[0]
    w = dev.pack(B, sb, K, N)
    try:
        C = Cbuf if Cbuf is not None else np.full((M, N), np.nan, np.float32)
        dev.matmul_i8(A, w, sa, bias, C, M, K, N, lda=lda, ldc=ldc, epilogue=epi,
                      flags=vnpu.FORM_FLAGS[form])
    finally:
        dev.unpack(w)
    return C


# --------------------------------------------------------------------------- QUANTIZE_I8
@pytest.mark.parametrize("name,axis", [("row", 0), ("col", 1), ("tensor", 2)])
def test_quantize_golden(gpu, golden, name, axis):
    X = golden[f"quant_{name}_X"]
    r, c = X.shape
    Y = np.empty((r, c), np.int8)
    s = np.empty(golden[f"quant_{name}_s"].shape, np.float32)
    gpu.quantize_i8(X, Y, s, r, c, axis)
    assert bits_equal(Y, golden[f"quant_{name}_Y"])
    assert bits_equal(s, golden[f"quant_{name}_s"])


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 4097), (64, 4096), (7, 12000), (512, 4096),
                                       (33, 8192)])
@pytest.mark.parametrize("axis", [0, 1, 2])
def test_quantize_vs_oracle(gpu, oracle, rows, cols, axis):
    rng = np.random.default_rng(rows * 7919 + cols + axis)
    X = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    if rows > 1 and cols > 8:
        X[0, :4] = [np.nan, np.inf if axis != 0 else 2.0, -0.0, 1e-30]
        X[-1, :] = 0.0  # all-zero row: scale 1.0
    Yo, so = oracle.quantize(X, axis)
    Y = np.empty_like(Yo)
    s = np.empty_like(so)
    gpu.quantize_i8(X, Y, s, rows, cols, axis)
    assert bits_equal(Y, Yo)
    assert bits_equal(s, so)


def test_quantize_device_pointers(gpu, oracle):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    X = rng.normal(0, 1, (256, 4096)).astype(np.float32)
    Yo, so = oracle.quantize(X, 0)
    dX = torch.from_numpy(X).cuda()
    dY = torch.empty((256, 4096), dtype=torch.int8, device="cuda")
    ds = torch.empty(256, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu.quantize_i8(dX.data_ptr(), dY.data_ptr(), ds.data_ptr(), 256, 4096, 0)
    assert bits_equal(dY.cpu().numpy(), Yo)
    assert bits_equal(ds.cpu().numpy(), so)


# --------------------------------------------------------------------------- MATMUL_I8
def _golden_case(golden, i):
    M, K, N, has_bias, epi = (int(v) for v in golden["mm_cases"][i])
    A, B = golden[f"mm{i}_A"], golden[f"mm{i}_B"]
    sa, sb = golden[f"mm{i}_sa"], golden[f"mm{i}_sb"]
    bias = golden.get(f"mm{i}_bias")
    return M, K, N, epi, A, B, sa, sb, bias, golden[f"mm{i}_C"], int(golden["mm_forms"][i])


@pytest.mark.parametrize("i", range(11))
@pytest.mark.parametrize("kernel", [None, "simt"])
def test_matmul_golden(gpu, golden, force_kernel, i, kernel):
    M, K, N, epi, A, B, sa, sb, bias, Cref, form = _golden_case(golden, i)
    force_kernel(kernel)
    C = run_matmul(gpu, A, B, sa, sb, bias, epi, form)
    assert bits_equal(C, Cref), f"case {i}: max ulp {ulp_diff(C, Cref)}"


@pytest.mark.parametrize("kernel", ["tcgen05", "gemv", "simt"])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (4, 4096, 512), (8, 4096, 384),
                                   (9, 1000, 257), (128, 128, 256), (200, 1024, 1000),
                                   (257, 777, 513), (512, 512, 512)])
def test_matmul_int32_exact(gpu, oracle, force_kernel, kernel, M, K, N):
    """scale 1, no bias, |acc| < 2^24: C == float(acc) exactly."""
    if kernel == "gemv" and M > 8:
        pytest.skip("gemv takes M <= 8")
    rng = np.random.default_rng(M * 131 + K * 7 + N)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    acc = oracle.gemm_acc(A, B)
    assert np.abs(acc).max() < 2 ** 24
    force_kernel(kernel)
    C = run_matmul(gpu, A, B, None, None, None, 0)
    assert bits_equal(C, acc.astype(np.float32))


@pytest.mark.parametrize("form", [0, 1, 2])
@pytest.mark.parametrize("epi", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("M,K,N", [(1, 300, 200), (6, 129, 77), (130, 200, 300),
                                   (256, 1024, 512)])
def test_matmul_epilogue_forms(gpu, oracle, form, epi, M, K, N):
    rng = np.random.default_rng(epi * 1000 + form * 100 + M)
    Af = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    Bf = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    A, sa = oracle.quantize(Af, 0)
    B, sb = oracle.quantize(Bf, 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    Co = oracle.matmul_i8(A, B, sa, sb, bias, epi, form)
    C = run_matmul(gpu, A, B, sa, sb, bias, epi, form)
    assert bits_equal(C, Co), f"max ulp {ulp_diff(C, Co)}"


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 17, 127, 128, 129, 255, 257])
@pytest.mark.parametrize("N", [1, 7, 255, 256, 257])
@pytest.mark.parametrize("K", [1, 15, 16, 17, 127, 128, 129, 1000])
def test_matmul_ragged_shapes(gpu, oracle, M, N, K):
    rng = np.random.default_rng(M * 100003 + N * 101 + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    sb = rng.uniform(1e-4, 2e-3, N).astype(np.float32)
    bias = rng.normal(0, 0.1, N).astype(np.float32)
    Co = oracle.matmul_i8(A, B, sa, sb, bias, 2, 0)
    C = run_matmul(gpu, A, B, sa, sb, bias, 2, 0)
    assert bits_equal(C, Co), f"max ulp {ulp_diff(C, Co)}"


@pytest.mark.parametrize("lda_pad,ldc_pad", [(0, 0), (16, 0), (5, 3), (48, 64)])
def test_matmul_strides(gpu, oracle, lda_pad, ldc_pad):
    """lda > K (aligned and not), ldc > N: gaps in C must be left untouched."""
    M, K, N = 150, 320, 300
    lda, ldc = K + lda_pad, N + ldc_pad
    rng = np.random.default_rng(lda * 3 + ldc)
    Abuf = rng.integers(-128, 128, (M, lda), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    sa = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    sb = rng.uniform(1e-4, 2e-3, N).astype(np.float32)
    Co = oracle.matmul_i8(Abuf[:, :K], B, sa, sb, None, 0, 0)
    Cbuf = np.full((M, ldc), 7.25, np.float32)
    run_matmul(gpu, Abuf, B, sa, sb, None, 0, 0, lda=lda, ldc=ldc, Cbuf=Cbuf, M=M, K=K, N=N)
    assert bits_equal(Cbuf[:, :N], Co)
    assert np.all(Cbuf[:, N:] == 7.25)


def test_matmul_device_pointers_and_kernels_agree(gpu, oracle, force_kernel):
    """Device-resident operands; tcgen05 and simt give the same bits."""
    torch = pytest.importorskip("torch")
    M, K, N = 1024, 2048, 1536
    rng = np.random.default_rng(11)
    Af = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    Bf = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    A, sa = oracle.quantize(Af, 0)
    B, sb = oracle.quantize(Bf, 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    dA = torch.from_numpy(A).cuda()
    dsa = torch.from_numpy(sa).cuda()
    dbias = torch.from_numpy(bias).cuda()
    w = gpu.pack(torch.from_numpy(B).cuda().data_ptr(), torch.from_numpy(sb).cuda().data_ptr(),
                 K, N)
    outs = {}
    try:
        for kern in ("tcgen05", "simt"):
            force_kernel(kern)
            dC = torch.full((M, N), float("nan"), device="cuda")
            torch.cuda.synchronize()
            gpu.matmul_i8(dA.data_ptr(), w, dsa.data_ptr(), dbias.data_ptr(), dC.data_ptr(),
                          M, K, N, epilogue=2)
            outs[kern] = dC.cpu().numpy()
    finally:
        gpu.unpack(w)
    assert bits_equal(outs["tcgen05"], outs["simt"])
    rows = np.arange(0, M, 37)
    Co = oracle.matmul_i8_model(gpu.reference_model(), A, B, sa, sb, bias, 2, rows=rows)
    assert bits_equal(outs["tcgen05"][rows], Co)


@pytest.mark.parametrize("M,K,N", [(8192, 8192, 8192), (4096, 4096, 14336)])
def test_matmul_full_size_sampled(gpu, oracle, M, K, N):
    """Headline sizes: every 97th row against the oracle, plus a row-sum
    checksum of all rows against the oracle's int32 arithmetic."""
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cuda").manual_seed(M + N)
    dA = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    dB = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    ones_a = torch.ones(M, device="cuda")
    ones_b = torch.ones(N, device="cuda")
    w = gpu.pack(dB.data_ptr(), ones_b.data_ptr(), K, N)
    try:
        dC = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        gpu.matmul_i8(dA.data_ptr(), w, ones_a.data_ptr(), None, dC.data_ptr(), M, K, N)
        torch.cuda.synchronize()
    finally:
        gpu.unpack(w)
    A = dA.cpu().numpy()
    B = dB.cpu().numpy()
    rows = np.arange(0, M, 97)
    acc = oracle.gemm_acc(A[rows], B)
    C_rows = dC[torch.from_numpy(rows).cuda()].cpu().numpy()
    # |acc| may exceed 2^24 at K=8192: compare with float(acc), the exact
    # int32->f32 rounding the epilogue performs (scale 1.0).
    assert bits_equal(C_rows, acc.astype(np.float32))
    # every row: sum over n of float(acc) in float64 equals A . (B summed over n)
    colsum = B.astype(np.int64).sum(axis=1)
    exact = A.astype(np.int64) @ colsum
    got = dC.double().sum(dim=1).cpu().numpy()
    # float(acc) rounds each |acc| <= 2^14 * K by at most 2^-24 relative
    bound = N * (128.0 * 128.0 * K) * 2.0 ** -24 + 1.0
    assert np.abs(got - exact).max() <= bound


# --------------------------------------------------------------------------- block ops
def test_rmsnorm_golden(gpu, golden):
    X, W = golden["rms_X"], golden["rms_W"]
    Y = np.empty_like(X)
    gpu.rmsnorm(X, W, Y, X.shape[0], X.shape[1], 1e-6)
    assert bits_equal(Y, golden["rms_Y"])
    X2 = golden["rms2_X"]
    Y2 = np.empty_like(X2)
    gpu.rmsnorm(X2, None, Y2, X2.shape[0], X2.shape[1], 0.0)
    assert bits_equal(Y2, golden["rms2_Y"])


@pytest.mark.parametrize("kernel", ["row", "warp"])
def test_rmsnorm_block_sizes(gpu, oracle, monkeypatch, kernel):
    """The row-staged kernel (default up to 48K columns) and the warp-per-row
    kernel both equal the oracle: vector/tail splits, no weights, wide rows."""
    if kernel == "warp":
        monkeypatch.setenv("VNPU_B200_RMSNORM_WARP", "1")
    rng = np.random.default_rng(3)
    for rows, cols, weighted in ((512, 4096, True), (1, 4096, True), (7, 11008, True),
                                 (3, 13, True), (2, 4100, False), (1, 20000, True),
                                 (2, 49153, True), (5, 7, False)):
        X = rng.normal(0, 1, (rows, cols)).astype(np.float32)
        W = rng.normal(1, 0.1, cols).astype(np.float32) if weighted else None
        Y = np.empty_like(X)
        gpu.rmsnorm(X, W, Y, rows, cols, 1e-6)
        assert bits_equal(Y, oracle.rmsnorm(X, W, 1e-6, 0)), (rows, cols)
    monkeypatch.delenv("VNPU_B200_RMSNORM_WARP", raising=False)


@pytest.mark.parametrize("rows,cols,weighted,want_y", [
    (1, 4096, True, False), (512, 4096, True, True), (7, 11008, False, True),
    (3, 13, True, True), (2, 4100, True, False), (1, 30000, True, False)])
def test_rmsnorm_quantize_fused_equals_two_commands(gpu, oracle, rows, cols, weighted, want_y):
    """VNPU_B200_OP_RMSNORM_QUANTIZE_I8 gives the bits of RMSNORM_F32 then
    QUANTIZE_I8 per row (both on the GPU and in the oracle)."""
    rng = np.random.default_rng(rows * 7 + cols)
    X = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    X[0, :2] = [0.0, 3.5]
    W = rng.normal(1, 0.1, cols).astype(np.float32) if weighted else None
    Y = np.full((rows, cols), np.nan, np.float32) if want_y else None
    Q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    gpu.rmsnorm_quantize(X, W, Y, Q, s, rows, cols, 1e-6)
    Y2 = np.empty((rows, cols), np.float32)
    gpu.rmsnorm(X, W, Y2, rows, cols, 1e-6)
    Q2 = np.empty_like(Q)
    s2 = np.empty_like(s)
    gpu.quantize_i8(Y2, Q2, s2, rows, cols, vnpu.QUANT_PER_ROW)
    assert np.array_equal(Q, Q2) and bits_equal(s, s2)
    if want_y:
        assert bits_equal(Y, Y2)
    Yo = oracle.rmsnorm(X, W, 1e-6, 0)
    Qo, so = oracle.quantize(Yo, 0)
    assert np.array_equal(Q, Qo) and bits_equal(s, so)


@pytest.mark.parametrize("rows,cols,want_y,alpha", [
    (1, 11008, False, 0.0), (512, 11008, True, 0.0), (3, 13, True, 1.7), (2, 4098, False, 0.0)])
def test_swiglu_quantize_fused_equals_two_commands(gpu, oracle, rows, cols, want_y, alpha):
    rng = np.random.default_rng(rows * 11 + cols)
    G = rng.normal(0, 2, (rows, cols)).astype(np.float32)
    U = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    Y = np.full((rows, cols), np.nan, np.float32) if want_y else None
    Q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    gpu.swiglu_quantize(G, U, Y, Q, s, rows, cols, alpha)
    Y2 = np.empty((rows, cols), np.float32)
    gpu.swiglu(G, U, Y2, rows * cols, alpha)
    Q2 = np.empty_like(Q)
    s2 = np.empty_like(s)
    gpu.quantize_i8(Y2, Q2, s2, rows, cols, vnpu.QUANT_PER_ROW)
    assert np.array_equal(Q, Q2) and bits_equal(s, s2)
    if want_y:
        assert bits_equal(Y, Y2)
    Yo = oracle.swiglu(G, U, alpha, 0)
    Qo, so = oracle.quantize(Yo.reshape(rows, cols), 0)
    assert np.array_equal(Q, Qo) and bits_equal(s, so)
    # gate and up as the two halves of one [rows][2*cols] GEMM output (ld)
    GU = np.concatenate([G, U], axis=1)
    Yl = np.full((rows, cols), np.nan, np.float32) if want_y else None
    Ql = np.zeros((rows, cols), np.int8)
    sl = np.zeros(rows, np.float32)
    gpu.swiglu_quantize(GU[:, :cols], GU[:, cols:], Yl, Ql, sl, rows, cols, alpha, ld=2 * cols)
    assert np.array_equal(Ql, Q) and bits_equal(sl, s)
    if want_y:
        assert bits_equal(Yl, Y)


def test_rope_golden(gpu, golden):
    Q, K = golden["rope_Q"].copy(), golden["rope_K"].copy()
    _, H, T, D = Q.shape
    gpu.rope(Q, K, None, 1, H, T, T, D, position_offset=5)
    for got, ref in ((Q, golden["rope_Qr"]), (K, golden["rope_Kr"])):
        np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
        assert ulp_diff(got, ref) <= 4 or np.abs(got - ref).max() <= ATOL
    Qi = golden["ropei_Q"].copy()
    gpu.rope(Qi, None, golden["ropei_pos"], 1, 2, 9, 0, 64, interleaved=1, theta=500000.0,
             scaling=0.5)
    np.testing.assert_allclose(Qi, golden["ropei_Qr"], rtol=RTOL, atol=ATOL)


def test_rope_decode_positions(gpu, oracle):
    rng = np.random.default_rng(9)
    for pos in (0, 511, 639):
        Q = rng.normal(0, 1, (1, 32, 1, 128)).astype(np.float32)
        K = rng.normal(0, 1, (1, 32, 1, 128)).astype(np.float32)
        Qg, Kg = Q.copy(), K.copy()
        gpu.rope(Qg, Kg, None, 1, 32, 1, 1, 128, position_offset=pos)
        Qo, Ko = oracle.rope(Q, K, None, 1, 32, 1, 1, 128, position_offset=pos)
        np.testing.assert_allclose(Qg, Qo, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(Kg, Ko, rtol=RTOL, atol=ATOL)


def test_swiglu_add_golden(gpu, golden):
    g, u = golden["swiglu_g"], golden["swiglu_u"]
    Y = np.empty_like(g)
    gpu.swiglu(g, u, Y, g.size, 0.0)
    assert bits_equal(Y, golden["swiglu_Y"])
    a, b = golden["add_A"], golden["add_B"]
    Y = np.empty_like(a)
    gpu.add(a, b, Y, a.size, 0.7, 1.3)
    assert bits_equal(Y, golden["add_Y"])


@pytest.mark.parametrize("name", ["attn", "attnd", "attnm"])
def test_attention_golden(gpu, golden, name):
    h, sq, sk, d, causal = (int(v) for v in golden[f"{name}_shape"])
    O = np.empty((1, h, sq, d), np.float32)
    gpu.attention(golden[f"{name}_Q"], golden[f"{name}_K"], golden[f"{name}_V"],
                  golden.get(f"{name}_M"), O, 1, h, sq, sk, d, causal, 0.0)
    assert bits_equal(O, golden[f"{name}_O"]), f"max ulp {ulp_diff(O, golden[f'{name}_O'])}"


@pytest.mark.parametrize("sq,sk,causal,masked", [
    (512, 512, 1, False), (16, 16, 1, False), (17, 100, 1, True), (33, 33, 0, False),
    (100, 300, 1, False), (64, 63, 0, True), (2, 2, 1, False), (129, 130, 0, True),
    (65, 65, 1, False), (200, 456, 1, True), (640, 640, 1, False)])
def test_prefill_attention_tiled_vs_general(gpu, oracle, monkeypatch, sq, sk, causal, masked):
    """head_dim 128: the register-tiled prefill kernel and the general kernel
    both equal the reference restatement bit for bit (ragged query and key
    blocks, causal offsets with seq_k > seq_q, additive masks with -inf)."""
    H, D = 4, 128
    rng = np.random.default_rng(sq * 7 + sk * 3 + causal)
    Q = rng.normal(0, 1, (1, H, sq, D)).astype(np.float32)
    K = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    V = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    M = None
    if masked:
        M = rng.normal(0, 1, (1, H, sq, sk)).astype(np.float32)
        M[..., sk // 3:sk // 2] = -np.inf
        M[:, :, 0, :] = -np.inf            # a query with every key masked
    ref = oracle.attention(Q, K, V, M, 1, H, sq, sk, D, causal, 0.0)
    for mode in ("tiled", "general"):
        if mode == "general":
            monkeypatch.setenv("VNPU_B200_ATTN", "general")
        O = np.full((1, H, sq, D), np.nan, np.float32)
        gpu.attention(Q, K, V, M, O, 1, H, sq, sk, D, causal, 0.0)
        assert bits_equal(O, ref), f"{mode}: max ulp {ulp_diff(O, ref)}"
    monkeypatch.delenv("VNPU_B200_ATTN", raising=False)


@pytest.mark.parametrize("sq,sk,causal,masked", [(512, 512, 1, False), (130, 200, 0, True),
                                                 (77, 77, 1, True)])
def test_prefill_attention_zero_probabilities(gpu, oracle, sq, sk, causal, masked):
    """Scores spread over hundreds: probabilities underflow to zero in the
    middle of key blocks, so the value phase takes its per-key test (the
    reference skips p == 0) instead of the prefix fast path; bit-exact."""
    H, D = 4, 128
    rng = np.random.default_rng(sq + 31 * sk)
    Q = (rng.normal(0, 1, (1, H, sq, D)) * 25.0).astype(np.float32)
    K = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    V = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    M = None
    if masked:
        M = rng.normal(0, 1, (1, H, sq, sk)).astype(np.float32)
        M[..., 5:9] = -np.inf
    ref = oracle.attention(Q, K, V, M, 1, H, sq, sk, D, causal, 0.0)
    O = np.full((1, H, sq, D), np.nan, np.float32)
    gpu.attention(Q, K, V, M, O, 1, H, sq, sk, D, causal, 0.0)
    assert bits_equal(O, ref), f"max ulp {ulp_diff(O, ref)}"


@pytest.mark.parametrize("B,H,sq,sk,D,causal,masked", [
    (1, 4, 512, 512, 128, 1, False),    # 64-query prefill kernel
    (2, 3, 100, 300, 128, 1, True),     # batch 2, ragged query block, causal offset
    (1, 4, 33, 33, 64, 0, False),       # general kernel (head_dim 64)
    (2, 2, 20, 45, 40, 1, True),        # general kernel, head_dim 40
    (1, 32, 1, 640, 128, 0, True),      # decode: both layouts are the same addresses
])
def test_attention_token_major_output(gpu, B, H, sq, sk, D, causal, masked):
    """VNPU_CMD_FLAG_ATTN_TOKEN_MAJOR writes the same bits as the reference
    layout, at [batch][seq_q][heads][D] instead of [batch][heads][seq_q][D]."""
    rng = np.random.default_rng(B * 100 + sq + sk + D)
    Q = rng.normal(0, 1, (B, H, sq, D)).astype(np.float32)
    K = rng.normal(0, 1, (B, H, sk, D)).astype(np.float32)
    V = rng.normal(0, 1, (B, H, sk, D)).astype(np.float32)
    M = rng.normal(0, 1, (B, H, sq, sk)).astype(np.float32) if masked else None
    O = np.full((B, H, sq, D), np.nan, np.float32)
    gpu.attention(Q, K, V, M, O, B, H, sq, sk, D, causal, 0.0)
    Ot = np.full((B, sq, H, D), np.nan, np.float32)
    gpu.attention(Q, K, V, M, Ot, B, H, sq, sk, D, causal, 0.0,
                  flags=vnpu.CMD_FLAG_ATTN_TOKEN_MAJOR)
    assert bits_equal(Ot, np.ascontiguousarray(O.transpose(0, 2, 1, 3)))


@pytest.mark.parametrize("sq,sk", [(512, 512), (1, 513), (1, 640), (16, 16), (17, 100)])
def test_attention_block_shapes(gpu, oracle, sq, sk):
    H, D = 32 if sq <= 16 else 8, 128
    rng = np.random.default_rng(sq * 1000 + sk)
    Q = rng.normal(0, 1, (1, H, sq, D)).astype(np.float32)
    K = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    V = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    O = np.empty((1, H, sq, D), np.float32)
    gpu.attention(Q, K, V, None, O, 1, H, sq, sk, D, 1, 0.0)
    Oo = oracle.attention(Q, K, V, None, 1, H, sq, sk, D, 1, 0.0)
    assert bits_equal(O, Oo), f"max ulp {ulp_diff(O, Oo)}"


@pytest.mark.parametrize("M,K,N", [(129, 256, 256), (300, 1000, 700), (1024, 2048, 1536),
                                   (2000, 640, 2056)])
def test_pair_and_single_cta_kernels_agree(gpu, oracle, monkeypatch, M, K, N):
    """The CTA-pair (256x256) and single-CTA (128x256) tcgen05 kernels give
    the same bits, equal to the oracle on sampled rows."""
    rng = np.random.default_rng(M + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    monkeypatch.setenv("VNPU_B200_NO_SPLITK", "1")
    monkeypatch.setenv("VNPU_B200_PAIR_TN", "256")
    outs = []
    for no_pair in (False, True):
        if no_pair:
            monkeypatch.setenv("VNPU_B200_NO_PAIR", "1")
        outs.append(run_matmul(gpu, A, B, sa, sb, bias, 3, 0))
        # Rows of A that are not 16-byte aligned (K % 16) cannot be TMA
        # sources: both runs then take the SIMT kernel.
        assert gpu.lib.b200_last_matmul_kernel().decode() == (
            "gemm_i8_simt_kernel" if K % 16 else
            "gemm_i8_tcgen05_kernel" if no_pair else "gemm_i8_tcgen05_pair_kernel")
    monkeypatch.delenv("VNPU_B200_NO_PAIR", raising=False)
    assert bits_equal(outs[0], outs[1])
    rows = np.arange(0, M, 13)
    assert bits_equal(outs[0][rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, 3, 0))


@pytest.mark.parametrize("M,K,N,epi,form,pad,bias_on", [
    (512, 4096, 4096, 0, 0, 0, False),   # the decoder block's O projection: 2 splits
    (512, 11008, 4096, 0, 0, 0, True),   # its down projection: 2 splits of 43 k-blocks
    (300, 2048, 1000, 2, 0, 0, True),    # ragged M and N, SiLU
    (129, 4096, 512, 1, 1, 0, True),     # two tiles: 4 splits, stream form
    (256, 3008, 256, 4, 2, 0, True),     # ragged K: 3 splits of 8 k-blocks, scalar form
    (300, 2048, 1000, 0, 0, 3, True),    # ldc % 4 != 0: scalar stores in the finish kernel
])
def test_splitk_pair_kernel_agrees(gpu, oracle, monkeypatch, M, K, N, epi, form, pad, bias_on):
    """The CTA-pair GEMM split over K (raw int32 sums of each split in a
    workspace, added exactly and dequantised by a second kernel) gives the
    same bits as the single pass and the oracle."""
    rng = np.random.default_rng(M * 5 + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32) if bias_on else None
    ldc = N + pad if pad else 0
    monkeypatch.setenv("VNPU_B200_PAIR_TN", "256")
    outs = []
    # splits of >= 8 k-blocks (the rule for MATMUL_I8_RESIDUAL; plain
    # MATMUL_I8 splits only from 24)
    monkeypatch.setenv("VNPU_B200_SPLITK_MIN_KB", "8")
    for split in (True, False):
        if split:
            monkeypatch.delenv("VNPU_B200_NO_SPLITK", raising=False)
        else:
            monkeypatch.setenv("VNPU_B200_NO_SPLITK", "1")
        Cbuf = np.full((M, ldc), np.nan, np.float32) if pad else None
        C = run_matmul(gpu, A, B, sa, sb, bias, epi, form, ldc=ldc, Cbuf=Cbuf)
        assert gpu.lib.b200_last_matmul_kernel().decode() == (
            "gemm_i8_tcgen05_pair_kernel+splitk" if split else "gemm_i8_tcgen05_pair_kernel")
        outs.append(C[:, :N].copy())
        if pad:
            assert np.isnan(C[:, N:]).all()
    monkeypatch.delenv("VNPU_B200_NO_SPLITK", raising=False)
    assert bits_equal(outs[0], outs[1])
    rows = np.unique(np.r_[np.arange(0, M, 37), M - 1])
    assert bits_equal(outs[0][rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, epi, form))


def test_splitk_in_cuda_graph(gpu, oracle, monkeypatch):
    """A split-K GEMM (stream-ordered workspace allocated and freed inside the
    command) recorded as a CUDA graph and replayed twice gives the eager bits,
    with and without the residual folded into its finish kernel."""
    import torch
    monkeypatch.setenv("VNPU_B200_SPLITK_MIN_KB", "8")   # split the plain product too
    M, K, N = 512, 4096, 4096
    rng = np.random.default_rng(4242)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    w = gpu.pack(B, sb, K, N)
    try:
        Ad, sad = torch.from_numpy(A).cuda(), torch.from_numpy(sa).cuda()
        R = torch.from_numpy(rng.normal(0, 1, (M, N)).astype(np.float32)).cuda()
        C1 = torch.full((M, N), float("nan"), device="cuda")
        C2 = torch.full((M, N), float("nan"), device="cuda")
        mm = vnpu.Command()
        mm.opcode = vnpu.OP_MATMUL_I8
        mm.args.matmul_i8 = vnpu.MatmulI8Args(Ad.data_ptr(), w, sad.data_ptr(), None,
                                              C1.data_ptr(), M, K, N, 0, 0, 0, vnpu.UNIT_AUTO)
        res = vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, vnpu.MatmulI8ResidualArgs(
            Ad.data_ptr(), w, sad.data_ptr(), None, R.data_ptr(), C2.data_ptr(), M, K, N, 0, 0, 0,
            0, 0))
        torch.cuda.synchronize()
        assert gpu.submit([mm, res]) == vnpu.OK and gpu.sync() == vnpu.OK
        assert gpu.lib.b200_last_matmul_kernel().decode() == "gemm_i8_tcgen05_pair_kernel+splitk"
        eager1, eager2 = C1.cpu().numpy(), C2.cpu().numpy()
        rows = np.arange(0, M, 61)
        assert bits_equal(eager1[rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, None, 0, 0))
        assert bits_equal(eager2, oracle.add(R.cpu().numpy(), eager1, 1.0, 1.0, 0))
        g = gpu.capture([mm, res])
        try:
            for _ in range(2):
                C1.fill_(float("nan"))
                C2.fill_(float("nan"))
                torch.cuda.synchronize()
                gpu.replay(g)
                assert gpu.sync() == vnpu.OK
                assert bits_equal(C1.cpu().numpy(), eager1)
                assert bits_equal(C2.cpu().numpy(), eager2)
        finally:
            gpu.lib.b200_graph_destroy(g)
    finally:
        gpu.unpack(w)


@pytest.mark.parametrize("M,K,N,epi,form,pad", [
    (129, 256, 256, 3, 0, 0),      # one partial 256x512 tile
    (300, 1008, 700, 2, 0, 0),     # ragged K (8 k-blocks), ragged N
    (257, 128, 513, 1, 1, 0),      # one k-block: the held-stage prologue is the whole tile
    (512, 384, 1024, 2, 2, 0),     # three k-blocks < four stages
    (1024, 2048, 1536, 4, 0, 0),
    (2000, 640, 2056, 2, 0, 3),    # ldc % 4 != 0: direct stores instead of TMA
    (4096, 4096, 4096, 0, 0, 0),   # 128 tiles: more than one wave of pairs
])
def test_wide_pair_kernel_agrees(gpu, oracle, monkeypatch, M, K, N, epi, form, pad):
    """The 256x512 CTA-pair kernel (two accumulators in all 512 TMEM columns,
    D1 deferred at each tile start) gives the same bits as the 256x256 pair
    kernel and the oracle."""
    rng = np.random.default_rng(M * 3 + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    ldc = N + pad if pad else 0
    monkeypatch.setenv("VNPU_B200_NO_SPLITK", "1")
    monkeypatch.setenv("VNPU_B200_PAIR_TN", "256")
    outs = []
    for wide in ("1", "0"):
        monkeypatch.setenv("VNPU_B200_PAIR_WIDE", wide)
        Cbuf = np.full((M, ldc), np.nan, np.float32) if pad else None
        C = run_matmul(gpu, A, B, sa, sb, bias, epi, form, ldc=ldc, Cbuf=Cbuf)
        assert gpu.lib.b200_last_matmul_kernel().decode() == (
            "gemm_i8_tcgen05_pair_wide_kernel" if wide == "1" else "gemm_i8_tcgen05_pair_kernel")
        outs.append(C[:, :N].copy())
        if pad:
            assert np.isnan(C[:, N:]).all()   # nothing written past N
    monkeypatch.delenv("VNPU_B200_PAIR_WIDE", raising=False)
    assert bits_equal(outs[0], outs[1])
    rows = np.unique(np.r_[np.arange(0, M, 17), M - 1])
    assert bits_equal(outs[0][rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, epi, form))


@pytest.mark.parametrize("M,K,N,epi,form,pad", [
    (129, 256, 224, 3, 0, 0),      # one partial tile, exactly one 224-column tile
    (300, 1008, 700, 2, 0, 0),     # ragged K and N
    (257, 128, 449, 1, 1, 0),      # one k-block; N one past two 224-column tiles
    (512, 384, 1024, 2, 2, 0),     # three k-blocks
    (2000, 640, 2056, 2, 0, 3),    # ldc % 4 != 0: direct stores
    (1024, 2048, 3584, 0, 0, 0),   # the 8-way shard width of 28672 (16 x 224)
    (4096, 1024, 7168, 0, 0, 0),   # the 4-way shard width (16 x 448): several waves
])
def test_224_column_tiles_agree(gpu, oracle, monkeypatch, M, K, N, epi, form, pad):
    """The 224-column tiles (256x224 pair kernel, 256x448 wide kernel: each
    CTA loads 112 weight rows per stage) give the same bits as the 256x256
    pair kernel and the oracle."""
    rng = np.random.default_rng(M * 5 + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    ldc = N + pad if pad else 0
    monkeypatch.setenv("VNPU_B200_NO_SPLITK", "1")
    outs = []
    for wide, tn, name in (("0", "256", "gemm_i8_tcgen05_pair_kernel"),
                           ("0", "224", "gemm_i8_tcgen05_pair_kernel<224>"),
                           ("1", "224", "gemm_i8_tcgen05_pair_wide_kernel<224>")):
        monkeypatch.setenv("VNPU_B200_PAIR_WIDE", wide)
        monkeypatch.setenv("VNPU_B200_PAIR_TN", tn)
        Cbuf = np.full((M, ldc), np.nan, np.float32) if pad else None
        C = run_matmul(gpu, A, B, sa, sb, bias, epi, form, ldc=ldc, Cbuf=Cbuf)
        assert gpu.lib.b200_last_matmul_kernel().decode() == name
        outs.append(C[:, :N].copy())
        if pad:
            assert np.isnan(C[:, N:]).all()   # nothing written past N
    monkeypatch.delenv("VNPU_B200_PAIR_WIDE", raising=False)
    monkeypatch.delenv("VNPU_B200_PAIR_TN", raising=False)
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(outs[0], outs[2])
    rows = np.unique(np.r_[np.arange(0, M, 17), M - 1])
    assert bits_equal(outs[1][rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, epi, form))


@pytest.mark.parametrize("M,K,N,epi,form,pad", [
    (512, 512, 512, 0, 0, 0),      # configs[0]'s shape: 16 tiles of 256x64
    (257, 128, 449, 1, 1, 0),      # one k-block; ragged M and N
    (300, 640, 1000, 2, 2, 3),     # SiLU, stream form, ldc % 4 != 0: direct stores
    (512, 4096, 4096, 0, 0, 0),    # the prefill projection shape
    (600, 896, 200, 3, 0, 0),      # GELU, N below one 256-column tile
])
def test_narrow_column_tiles_agree(gpu, oracle, monkeypatch, M, K, N, epi, form, pad):
    """The 128- and 64-column pair tiles (each CTA loads 64 or 32 weight rows
    per stage) give the same bits as the 256x256 pair kernel and the oracle."""
    rng = np.random.default_rng(M * 7 + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    ldc = N + pad if pad else 0
    monkeypatch.setenv("VNPU_B200_NO_SPLITK", "1")
    monkeypatch.setenv("VNPU_B200_PAIR_WIDE", "0")
    outs = []
    for tn, name in (("256", "gemm_i8_tcgen05_pair_kernel"),
                     ("128", "gemm_i8_tcgen05_pair_kernel<128>"),
                     ("64", "gemm_i8_tcgen05_pair_kernel<64>")):
        monkeypatch.setenv("VNPU_B200_PAIR_TN", tn)
        Cbuf = np.full((M, ldc), np.nan, np.float32) if pad else None
        C = run_matmul(gpu, A, B, sa, sb, bias, epi, form, ldc=ldc, Cbuf=Cbuf)
        assert gpu.lib.b200_last_matmul_kernel().decode() == name
        outs.append(C[:, :N].copy())
        if pad:
            assert np.isnan(C[:, N:]).all()   # nothing written past N
    monkeypatch.delenv("VNPU_B200_PAIR_WIDE", raising=False)
    monkeypatch.delenv("VNPU_B200_PAIR_TN", raising=False)
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(outs[0], outs[2])
    rows = np.unique(np.r_[np.arange(0, M, 17), M - 1])
    assert bits_equal(outs[2][rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, epi, form))


def test_narrow_tiles_chosen_for_underfilled_shapes(gpu, oracle, monkeypatch):
    """Shapes whose 256-column tiles fill few CTA pairs take the narrow tiles
    by default (512^3: 16 pairs of 256x64 instead of 4 of 256x256), and the
    result is the oracle's."""
    for var in ("VNPU_B200_PAIR_TN", "VNPU_B200_PAIR_WIDE", "VNPU_B200_NO_SPLITK"):
        monkeypatch.delenv(var, raising=False)
    rng = np.random.default_rng(5)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (512, 512)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (512, 512)).astype(np.float32), 1)
    C = run_matmul(gpu, A, B, sa, sb, None, 0, 0)
    assert gpu.lib.b200_last_matmul_kernel().decode().startswith("gemm_i8_tcgen05_pair_kernel<")
    assert bits_equal(C, oracle.matmul_i8(A, B, sa, sb, None, 0, 0))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (4096, 11008), (100, 300),
                                 (16, 128), (1000, 1000), (130, 12288)])
def test_decode_tensor_core_vs_simt(gpu, oracle, monkeypatch, M, K, N):
    """The M<=8 decode kernel on the tensor core (cluster split-K, partials
    summed through distributed shared memory) equals the SIMT GEMV and the
    oracle bit for bit, with bias (the decode shape of configs[1])."""
    rng = np.random.default_rng(M * 1000 + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    outs = []
    for simt in (False, True):
        if simt:
            monkeypatch.delenv("VNPU_B200_DECODE", raising=False)
            monkeypatch.setenv("VNPU_B200_SIMT_GEMV", "1")
        else:
            monkeypatch.setenv("VNPU_B200_DECODE", "tc")   # the tensor core for every M
        outs.append(run_matmul(gpu, A, B, sa, sb, bias, 0, 2))
    monkeypatch.delenv("VNPU_B200_SIMT_GEMV", raising=False)
    assert bits_equal(outs[0], outs[1])
    assert bits_equal(outs[0], oracle.matmul_i8(A, B, sa, sb, bias, 0, 2))


@pytest.mark.parametrize("sk,causal,masked,D,H", [(1, 1, False, 128, 4), (3, 0, False, 16, 4),
                                                  (64, 1, False, 128, 4), (65, 0, True, 128, 4),
                                                  (513, 1, False, 128, 4), (640, 0, True, 128, 32),
                                                  (300, 1, False, 40, 4), (1000, 1, True, 256, 4),
                                                  (700, 0, True, 256, 2), (1400, 1, False, 128, 3),
                                                  (77, 0, False, 12, 4)])
def test_decode_attention_matches_oracle(gpu, oracle, monkeypatch, sk, causal, masked, D, H):
    """One query per head (decode): the cluster kernel (D % 16 == 0 and the V
    slices fit in shared memory), the single-CTA decode kernel and the general
    kernel all equal the reference restatement bit for bit, masks included."""
    rng = np.random.default_rng(sk * 10 + D)
    Q = rng.normal(0, 1, (1, H, 1, D)).astype(np.float32)
    K = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    V = rng.normal(0, 1, (1, H, sk, D)).astype(np.float32)
    M = None
    if masked:
        M = np.zeros((1, H, 1, sk), np.float32)
        M[..., sk // 2:] = -np.inf          # e.g. KV-cache slots not yet filled
        M[..., :3] += rng.normal(0, 1, 3).astype(np.float32)
    ref = oracle.attention(Q, K, V, M, 1, H, 1, sk, D, causal, 0.0)
    for mode in ("cluster", "decode", "general"):
        monkeypatch.setenv("VNPU_B200_ATTN", mode)
        O = np.empty((1, H, 1, D), np.float32)
        gpu.attention(Q, K, V, M, O, 1, H, 1, sk, D, causal, 0.0)
        assert bits_equal(O, ref), f"{mode}: max ulp {ulp_diff(O, ref)}"
    monkeypatch.delenv("VNPU_B200_ATTN", raising=False)


@pytest.mark.parametrize("csize", ["1", "2", "4", "8"])
def test_fused_prologues_any_cluster_size(gpu, oracle, monkeypatch, csize):
    """The fused prologues split a row over 1-8 CTAs; every split gives the
    stand-alone bits (ragged slices, a row narrower than the split)."""
    monkeypatch.setenv("VNPU_B200_FUSED_CLUSTER", csize)
    rng = np.random.default_rng(int(csize))
    for rows, cols in ((1, 4096), (3, 11008), (2, 100), (1, 7)):
        X = rng.normal(0, 1, (rows, cols)).astype(np.float32)
        W = rng.normal(1, 0.1, cols).astype(np.float32)
        Q = np.zeros((rows, cols), np.int8)
        s = np.zeros(rows, np.float32)
        Y = np.full((rows, cols), np.nan, np.float32)
        gpu.rmsnorm_quantize(X, W, Y, Q, s, rows, cols, 1e-6)
        Yo = oracle.rmsnorm(X, W, 1e-6, 0)
        Qo, so = oracle.quantize(Yo, 0)
        assert bits_equal(Y, Yo) and np.array_equal(Q, Qo) and bits_equal(s, so), (rows, cols)
        U = rng.normal(0, 1, (rows, cols)).astype(np.float32)
        gpu.swiglu_quantize(X, U, Y, Q, s, rows, cols, 0.0)
        Yo = oracle.swiglu(X, U, 0.0, 0).reshape(rows, cols)
        Qo, so = oracle.quantize(Yo, 0)
        assert bits_equal(Y, Yo) and np.array_equal(Q, Qo) and bits_equal(s, so), (rows, cols)
    monkeypatch.delenv("VNPU_B200_FUSED_CLUSTER", raising=False)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("K,N", [(4096, 4096), (11008, 4096), (4096, 11008), (100, 300),
                                 (16, 128), (1000, 1000), (130, 12288), (12288, 130), (20, 5),
                                 (8192, 300), (4096, 147), (30000, 64)])
def test_decode_stream_kernel_agrees(gpu, oracle, monkeypatch, M, K, N):
    """The decode GEMVs that land their weights in shared memory before the
    programmatic wait - the mma.sync kernel (M <= 8) and the one-column-per-
    warp kernel (M <= 2) - give the bits of the tensor-core GEMV, the
    register-streaming GEMV and the oracle, with bias, for K / N shapes with
    ragged tails, fewer columns than a CTA covers and K too long for their
    shared memory (which takes the other kernels)."""
    rng = np.random.default_rng(M * 7919 + K * 13 + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32)
    k_stride = -(-K // 128) * 128
    mma_ok = K % 16 == 0 and k_stride <= 8192
    stream_ok = M <= 2 and mma_ok
    preferred = mma_ok and (M >= 2 or (N <= 32 * 148 and k_stride <= 4096))
    outs = {}
    for mode in ("default", "mma", "stream", "tc", "simt"):
        monkeypatch.delenv("VNPU_B200_DECODE", raising=False)
        monkeypatch.delenv("VNPU_B200_SIMT_GEMV", raising=False)
        if mode in ("tc", "mma", "stream"):
            monkeypatch.setenv("VNPU_B200_DECODE", mode)
        elif mode == "simt":
            monkeypatch.setenv("VNPU_B200_SIMT_GEMV", "1")
        outs[mode] = run_matmul(gpu, A, B, sa, sb, bias, 2, 2)
        kernel = gpu.lib.b200_last_matmul_kernel().decode()
        if mode == "default":
            want_kernel = ("gemv_i8_mma_kernel" if preferred else
                           "gemv_i8_stream_kernel" if stream_ok else None)
            if want_kernel:
                assert kernel == want_kernel, kernel
            else:
                assert kernel not in ("gemv_i8_mma_kernel", "gemv_i8_stream_kernel"), kernel
        elif mode == "mma":
            assert (kernel == "gemv_i8_mma_kernel") == mma_ok, kernel
        elif mode == "stream":
            assert (kernel == "gemv_i8_stream_kernel") == stream_ok, kernel
    monkeypatch.delenv("VNPU_B200_DECODE", raising=False)
    monkeypatch.delenv("VNPU_B200_SIMT_GEMV", raising=False)
    want = oracle.matmul_i8(A, B, sa, sb, bias, 2, 2)
    for mode, C in outs.items():
        assert bits_equal(C, want), (mode, ulp_diff(C, want))


def test_decode_stream_kernel_residual(gpu, oracle, monkeypatch):
    """MATMUL_I8_RESIDUAL at M = 1 on the shared-memory GEMVs (the mma.sync
    kernel at 4096 x 4096 and 3000 x 1000, the one-column kernel at 4096 x
    12288): C = R + out with ADD_F32's single rounding, equal to the
    register-streaming GEMV's."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    for K, N in ((4096, 4096), (11008, 4096), (3008, 1000), (4096, 12288)):
        A, sa = oracle.quantize(rng.uniform(-1, 1, (1, K)).astype(np.float32), 0)
        B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
        R = rng.normal(0, 1, (1, N)).astype(np.float32)
        w = gpu.pack(B, sb, K, N)
        try:
            dA = torch.from_numpy(A).cuda()
            dsa = torch.from_numpy(sa).cuda()
            dR = torch.from_numpy(R).cuda()
            res = {}
            for simt in (False, True):
                if simt:
                    monkeypatch.setenv("VNPU_B200_SIMT_GEMV", "1")
                dC = torch.full((1, N), float("nan"), device="cuda")
                torch.cuda.synchronize()
                args = vnpu.MatmulI8ResidualArgs(dA.data_ptr(), w, dsa.data_ptr(), None,
                                                 dR.data_ptr(), dC.data_ptr(), 1, K, N, 0, 0, 0, 0)
                assert gpu.submit([vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, args)]) == 0
                assert gpu.sync() == 0
                res[simt] = dC.cpu().numpy()
            monkeypatch.delenv("VNPU_B200_SIMT_GEMV", raising=False)
        finally:
            gpu.unpack(w)
        want = R + oracle.matmul_i8(A, B, sa, sb, None, 0, 0)
        assert bits_equal(res[False], res[True]) and bits_equal(res[False], want.astype(np.float32))
