"""The fused decoder-block opcodes against the command sequences they replace.

* VNPU_B200_OP_QKV_ROPE_APPEND == MATMUL_I8 (QKV weights) -> head-major split
  -> ROPE_F32 -> KV_APPEND, bit for bit: the one-token GEMV epilogue and the
  T > 1 path (MATMUL_I8 + split / rotate / append kernel), device and host
  operands, device-side position.
* VNPU_B200_OP_MATMUL_I8_RESIDUAL == MATMUL_I8 then ADD_F32 (alpha = beta =
  1), bit for bit: GEMV epilogue (M = 1), tensor-core GEMV and tcgen05 GEMM
  followed by the addition, in place (R = C) and not.
Failure paths are made on the host (a position past the capacity): the
kernel skips the writes and reports through the stream's error word.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return pytest.importorskip("torch")


def _weights(gpu, oracle, rng, K, N):
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    return gpu.pack(B, sb, K, N)


def _submit(gpu, cmds):
    arr = (vnpu.Command * len(cmds))(*cmds)
    assert gpu.lib.stream_submit(gpu.stream, arr, len(cmds), None) == vnpu.OK
    return gpu.sync()


def _matmul_cmd(A, w, sa, bias, Cp, M, K, N, epilogue=0):
    c = vnpu.Command()
    c.opcode = vnpu.OP_MATMUL_I8
    c.args.matmul_i8 = vnpu.MatmulI8Args(A, w, sa, bias, Cp, M, K, N, 0, 0, epilogue,
                                         vnpu.UNIT_GPU)
    return c


def _qkv_reference(gpu, torch, A8, w, sa, bias, T, K, H, D, cap, pos, use_ptr, theta):
    """MATMUL_I8 -> split -> ROPE_F32 -> KV_APPEND on fresh caches."""
    N = 3 * H * D
    C_ = torch.empty((T, N), device="cuda")
    kc = torch.zeros((H, cap, D), device="cuda")
    vc = torch.zeros((H, cap, D), device="cuda")
    mask = torch.full((H, cap), float("-inf"), device="cuda")
    posbuf = torch.tensor([pos], dtype=torch.int32, device="cuda")
    assert _submit(gpu, [_matmul_cmd(A8.data_ptr(), w, sa.data_ptr(),
                                     bias.data_ptr() if bias is not None else None,
                                     C_.data_ptr(), T, K, N)]) == vnpu.OK
    d = H * D
    Q = C_[:, :d].reshape(T, H, D).transpose(0, 1).contiguous()
    Kh = C_[:, d:2 * d].reshape(T, H, D).transpose(0, 1).contiguous()
    Vh = C_[:, 2 * d:].reshape(T, H, D).transpose(0, 1).contiguous()
    torch.cuda.synchronize()
    if use_ptr:   # decode form: positions[t] = pos (T = 1)
        rope = vnpu.RopeArgs(Q.data_ptr(), Kh.data_ptr(), posbuf.data_ptr(), 1, H, T, T, D, 0, 0,
                             theta, 1.0)
    else:
        rope = vnpu.RopeArgs(Q.data_ptr(), Kh.data_ptr(), None, 1, H, T, T, D, pos, 0, theta, 1.0)
    c = vnpu.Command()
    c.opcode = vnpu.OP_ROPE_F32
    c.args.rope = rope
    app = vnpu.b200_command(vnpu.OP_B200_KV_APPEND, vnpu.KvAppendArgs(
        Kh.data_ptr(), Vh.data_ptr(), kc.data_ptr(), vc.data_ptr(), mask.data_ptr(),
        posbuf.data_ptr() if use_ptr else None, H, T, D, cap, 0 if use_ptr else pos, 0))
    assert _submit(gpu, [c, app]) == vnpu.OK
    return [x.cpu().numpy() for x in (Q, Kh, Vh, kc, vc, mask)]


def _qkv_fused(gpu, torch, A8, w, sa, bias, T, K, H, D, cap, pos, use_ptr, theta, outs=True):
    kc = torch.zeros((H, cap, D), device="cuda")
    vc = torch.zeros((H, cap, D), device="cuda")
    mask = torch.full((H, cap), float("-inf"), device="cuda")
    Q = torch.full((H, T, D), float("nan"), device="cuda")
    Ko = torch.full((H, T, D), float("nan"), device="cuda")
    Vo = torch.full((H, T, D), float("nan"), device="cuda")
    posbuf = torch.tensor([pos], dtype=torch.int32, device="cuda")
    args = vnpu.QkvRopeAppendArgs(
        A8.data_ptr(), w, sa.data_ptr(), bias.data_ptr() if bias is not None else None,
        Q.data_ptr(), Ko.data_ptr() if outs else None, Vo.data_ptr() if outs else None,
        kc.data_ptr(), vc.data_ptr(), mask.data_ptr(), posbuf.data_ptr() if use_ptr else None,
        T, K, H, D, cap, 0 if use_ptr else pos, theta, 1.0, 0, 0)
    torch.cuda.synchronize()
    rc = _submit(gpu, [vnpu.b200_command(vnpu.OP_B200_QKV_ROPE_APPEND, args)])
    return rc, [x.cpu().numpy() for x in (Q, Ko, Vo, kc, vc, mask)]


@pytest.mark.parametrize("T,K,H,D,pos,use_ptr,with_bias", [
    (1, 512, 4, 128, 37, True, False),     # decode: GEMV epilogue, device position
    (1, 4096, 32, 128, 600, True, True),   # the decoder block's shape
    (1, 300, 2, 64, 5, False, True),       # K % 16 != 0 (unaligned GEMV loads)
    (1, 256, 3, 40, 0, False, False),
    (7, 512, 4, 128, 3, False, True),      # T > 1: MATMUL_I8 + split kernel
    (130, 256, 2, 64, 10, False, False),   # tcgen05 GEMM + split kernel
])
def test_qkv_rope_append_equals_sequence(gpu, oracle, torch, T, K, H, D, pos, use_ptr,
                                         with_bias):
    rng = np.random.default_rng(T * 1000 + K + D)
    N = 3 * H * D
    cap = pos + T + 4
    w = _weights(gpu, oracle, rng, K, N)
    A8h, sah = oracle.quantize(rng.uniform(-1, 1, (T, K)).astype(np.float32), 0)
    A8, sa = torch.from_numpy(A8h).cuda(), torch.from_numpy(sah).cuda()
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda() if with_bias else None
    try:
        ref = _qkv_reference(gpu, torch, A8, w, sa, bias, T, K, H, D, cap, pos, use_ptr, 10000.0)
        rc, got = _qkv_fused(gpu, torch, A8, w, sa, bias, T, K, H, D, cap, pos, use_ptr, 10000.0)
        assert rc == vnpu.OK
        for name, a, b in zip(("Q", "K", "V", "K_cache", "V_cache", "mask"), got, ref):
            assert bits_equal(a, b), name
    finally:
        gpu.unpack(w)


def test_qkv_rope_append_host_operands_no_outputs(gpu, oracle, torch):
    """Host activations and caches (staged), K_out/V_out omitted."""
    rng = np.random.default_rng(3)
    T, K, H, D, pos, cap = 1, 256, 2, 64, 9, 16
    N = 3 * H * D
    w = _weights(gpu, oracle, rng, K, N)
    A8h, sah = oracle.quantize(rng.uniform(-1, 1, (T, K)).astype(np.float32), 0)
    try:
        ref = _qkv_reference(gpu, torch, torch.from_numpy(A8h).cuda(), w,
                             torch.from_numpy(sah).cuda(), None, T, K, H, D, cap, pos, False,
                             500000.0)
        Q = np.full((H, T, D), np.nan, np.float32)
        kc = np.zeros((H, cap, D), np.float32)
        vc = np.zeros((H, cap, D), np.float32)
        mask = np.full((H, cap), -np.inf, np.float32)
        args = vnpu.QkvRopeAppendArgs(A8h.ctypes.data, w, sah.ctypes.data, None, Q.ctypes.data,
                                      None, None, kc.ctypes.data, vc.ctypes.data,
                                      mask.ctypes.data, None, T, K, H, D, cap, pos, 500000.0,
                                      1.0, 0, 0)
        assert _submit(gpu, [vnpu.b200_command(vnpu.OP_B200_QKV_ROPE_APPEND, args)]) == vnpu.OK
        for name, a, b in zip(("Q", "K_cache", "V_cache", "mask"), (Q, kc, vc, mask),
                              (ref[0], ref[3], ref[4], ref[5])):
            assert bits_equal(a, b), name
    finally:
        gpu.unpack(w)


def test_qkv_rope_append_position_past_capacity(b200_lib, oracle, torch):
    """A device position outside the cache: nothing is written to the cache,
    the stream reports the device error."""
    with vnpu.Device(b200_lib) as d:
        rng = np.random.default_rng(4)
        T, K, H, D, cap = 1, 128, 2, 64, 8
        w = _weights(d, oracle, rng, K, 3 * H * D)
        A8h, sah = oracle.quantize(rng.uniform(-1, 1, (T, K)).astype(np.float32), 0)
        A8, sa = torch.from_numpy(A8h).cuda(), torch.from_numpy(sah).cuda()
        rc, got = _qkv_fused(d, torch, A8, w, sa, None, T, K, H, D, cap, cap + 3, True, 10000.0)
        assert rc == vnpu.ERR_DEVICE_ERROR
        assert not got[3].any() and not got[4].any() and np.isneginf(got[5]).all()
        d.unpack(w)


@pytest.mark.parametrize("M,K,N,inplace,epi", [
    (1, 4096, 4096, False, 0), (1, 1000, 333, True, 0), (4, 512, 1024, False, 0),
    (300, 256, 512, True, 0), (300, 256, 512, False, 0), (512, 4096, 4096, False, 0),
    (777, 1000, 1000, False, 1), (260, 4096, 11008, False, 0), (300, 256, 512, False, 2),
    (300, 2048, 1000, False, 1), (512, 11008, 4096, False, 0), (512, 4096, 4096, True, 0)])
def test_residual_equals_matmul_then_add(gpu, oracle, torch, M, K, N, inplace, epi):
    """MATMUL_I8_RESIDUAL equals MATMUL_I8 then ADD_F32 bit for bit: the GEMV
    epilogue (M = 1), the add in the split-K finish kernel (M = 300, 512 with
    long K), and the two-pass form otherwise (R aliasing C, ragged N,
    epilogues)."""
    rng = np.random.default_rng(M + K + N)
    w = _weights(gpu, oracle, rng, K, N)
    A8h, sah = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    A8, sa = torch.from_numpy(A8h).cuda(), torch.from_numpy(sah).cuda()
    R = torch.from_numpy(rng.normal(0, 1, (M, N)).astype(np.float32)).cuda()
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    try:
        P = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        assert _submit(gpu, [_matmul_cmd(A8.data_ptr(), w, sa.data_ptr(), bias.data_ptr(),
                                         P.data_ptr(), M, K, N, epi)]) == vnpu.OK
        ref = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        gpu.add(R.data_ptr(), P.data_ptr(), ref.data_ptr(), M * N, 1.0, 1.0)
        out = R.clone() if inplace else torch.full((M, N), float("nan"), device="cuda")
        Rp = out if inplace else R
        torch.cuda.synchronize()
        args = vnpu.MatmulI8ResidualArgs(A8.data_ptr(), w, sa.data_ptr(), bias.data_ptr(),
                                         Rp.data_ptr(), out.data_ptr(), M, K, N, 0, 0, 0, epi, 0)
        assert _submit(gpu, [vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, args)]) == vnpu.OK
        assert bits_equal(out.cpu().numpy(), ref.cpu().numpy())
    finally:
        gpu.unpack(w)


def test_residual_host_operands(gpu, oracle):
    rng = np.random.default_rng(8)
    M, K, N = 1, 384, 200
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    A8, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    R = rng.normal(0, 1, (M, N)).astype(np.float32)
    w = gpu.pack(B, sb, K, N)
    try:
        out = np.full((M, N), np.nan, np.float32)
        args = vnpu.MatmulI8ResidualArgs(A8.ctypes.data, w, sa.ctypes.data, None, R.ctypes.data,
                                         out.ctypes.data, M, K, N, 0, 0, 0, 0, 0)
        assert _submit(gpu, [vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, args)]) == vnpu.OK
        prod = oracle.matmul_i8(A8, B, sa, sb, None, 0, 0)
        assert bits_equal(out, oracle.add(R, prod, 1.0, 1.0, 0))
    finally:
        gpu.unpack(w)


@pytest.mark.parametrize("M,K,N,kernels", [
    (1, 4096, 4096, 1),     # the decode O projection: mma GEMV
    (1, 1024, 6000, 1),     # N past the mma GEMV's shapes: streaming GEMV
    (1, 11008, 4096, 1),    # the decode down projection: register-streaming GEMV
    (1, 1000, 333, 1),      # lda % 16 != 0
    (3, 512, 1024, None),   # several rows: a one-thread kernel after the product
])
def test_residual_advances_position(gpu, oracle, torch, M, K, N, kernels):
    """MATMUL_I8_RESIDUAL with ADVANCE_POSITION gives the residual command's
    bits and adds to the device position; for one row the GEMV itself does it
    (no further launch), also in a batch beside commands without the flag."""
    rng = np.random.default_rng(M * 3 + K + N)
    w = _weights(gpu, oracle, rng, K, N)
    A8h, sah = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    A8, sa = torch.from_numpy(A8h).cuda(), torch.from_numpy(sah).cuda()
    R = torch.from_numpy(rng.normal(0, 1, (M, N)).astype(np.float32)).cuda()
    try:
        ref = torch.full((M, N), float("nan"), device="cuda")
        out = torch.full((M, N), float("nan"), device="cuda")
        pos = torch.tensor([5], dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        plain = vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, vnpu.MatmulI8ResidualArgs(
            A8.data_ptr(), w, sa.data_ptr(), None, R.data_ptr(), ref.data_ptr(), M, K, N, 0, 0, 0,
            0, 0))
        assert _submit(gpu, [plain]) == vnpu.OK
        adv = vnpu.with_advance_position(vnpu.b200_command(
            vnpu.OP_B200_MATMUL_I8_RESIDUAL, vnpu.MatmulI8ResidualArgs(
                A8.data_ptr(), w, sa.data_ptr(), None, R.data_ptr(), out.data_ptr(), M, K, N, 0,
                0, 0, 0, 0)), pos, 3)
        launches0 = gpu.lib.b200_kernel_launches(gpu.dev)
        assert _submit(gpu, [adv]) == vnpu.OK
        launched = gpu.lib.b200_kernel_launches(gpu.dev) - launches0
        assert bits_equal(out.cpu().numpy(), ref.cpu().numpy())
        assert int(pos.item()) == 8
        if kernels is not None:
            assert launched == kernels, launched
        # in one batch after a command without the flag: only the flagged one advances
        assert _submit(gpu, [plain, adv]) == vnpu.OK
        assert int(pos.item()) == 11
        assert bits_equal(out.cpu().numpy(), ref.cpu().numpy())
    finally:
        gpu.unpack(w)


def test_advance_position_rejects_bad_fields(b200_lib, oracle, torch):
    """ADVANCE_POSITION without a position, or on MATMUL_I8_SWIGLU, fails the
    command (the stream's error at the next sync) and moves nothing."""
    rng = np.random.default_rng(2)
    A8h, sah = oracle.quantize(rng.uniform(-1, 1, (1, 128)).astype(np.float32), 0)
    A8, sa = torch.from_numpy(A8h).cuda(), torch.from_numpy(sah).cuda()
    R = torch.zeros((1, 64), device="cuda")
    out = torch.zeros((1, 64), device="cuda")
    Y = torch.zeros((1, 32), device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    for case in ("no_position", "swiglu"):
        with vnpu.Device(b200_lib) as d:
            w = _weights(d, oracle, rng, 128, 64)
            if case == "swiglu":
                a = vnpu.MatmulI8SwigluArgs(A8.data_ptr(), w, sa.data_ptr(), None, Y.data_ptr(), 1,
                                            128, 64, 0, 0, 0, 1.0, 0)
                cmd = vnpu.with_advance_position(
                    vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_SWIGLU, a), pos, 1)
            else:
                args = vnpu.MatmulI8ResidualArgs(A8.data_ptr(), w, sa.data_ptr(), None,
                                                 R.data_ptr(), out.data_ptr(), 1, 128, 64, 0, 0,
                                                 0, 0, 0)
                cmd = vnpu.with_advance_position(
                    vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, args), None, 1)
            assert d.submit([cmd]) == vnpu.OK
            assert d.sync() == vnpu.ERR_DEVICE_ERROR, case
            assert int(pos.item()) == 0
            d.unpack(w)


# ------------------------------------------------------------------ MATMUL_I8_SWIGLU
@pytest.mark.parametrize("M,K,I,bias_on,ldy_pad,alpha,kernel", [
    (1, 4096, 1024, False, 0, 1.0, "gemv_i8_stream_kernel+swiglu"),   # decode token
    (1, 4096, 1000, True, 3, 0.5, "gemv_i8_stream_kernel+swiglu"),    # bias: the 2I-wide forms
    (2, 1024, 520, False, 0, 1.0, "gemv_i8_stream_kernel+swiglu"),
    (5, 1024, 700, True, 0, 1.0, None),                                # product, then the halves
    (300, 512, 1000, False, 0, 1.0, "gemm_i8_tcgen05_pair_kernel+swiglu"),  # ragged I
    (257, 128, 256, False, 1, 2.0, "gemm_i8_tcgen05_pair_kernel+swiglu"),   # direct stores
    (512, 4096, 11008, False, 0, 1.0, "gemm_i8_tcgen05_pair_kernel+swiglu"),  # block prefill
])
def test_matmul_swiglu_equals_matmul_then_swiglu(gpu, oracle, torch, M, K, I, bias_on, ldy_pad,
                                                 alpha, kernel):
    """VNPU_B200_OP_MATMUL_I8_SWIGLU gives the bits of MATMUL_I8 on the
    [K][2I] gate/up weight followed by SWIGLU_F32 of the output's halves (the
    reference block, tools/llm_bench.cpp:298-311), unflagged: each element in
    the rounding form it has in the 2I-wide product."""
    rng = np.random.default_rng(M * 3 + K + I)
    N = 2 * I
    w = _weights(gpu, oracle, rng, K, N)
    try:
        A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
        A_d = torch.from_numpy(A).cuda()
        sa_d = torch.from_numpy(sa).cuda()
        bias = (torch.from_numpy(rng.normal(0, 0.01, N).astype(np.float32)).cuda()
                if bias_on else None)
        C = torch.full((M, N), float("nan"), device="cuda")
        assert _submit(gpu, [_matmul_cmd(A_d.data_ptr(), w, sa_d.data_ptr(),
                                         bias.data_ptr() if bias is not None else None,
                                         C.data_ptr(), M, K, N)]) == vnpu.OK
        g = C[:, :I].contiguous()
        u = C[:, I:].contiguous()
        want = torch.empty((M, I), device="cuda")
        gpu.swiglu(g.data_ptr(), u.data_ptr(), want.data_ptr(), M * I, alpha)
        ldy = I + ldy_pad
        Y = torch.full((M, ldy), float("nan"), device="cuda")
        assert gpu.matmul_i8_swiglu(A_d, w, sa_d, bias, Y, M, K, N, ldy=ldy, alpha=alpha) == vnpu.OK
        if kernel:
            assert gpu.lib.b200_last_matmul_kernel().decode() == kernel
        assert bits_equal(Y[:, :I].cpu().numpy(), want.cpu().numpy())
        if ldy_pad:
            assert torch.isnan(Y[:, I:]).all()   # nothing written past I
        # and against the oracle on a few rows (block form: no bias here)
        if not bias_on and M <= 512:
            B, sb = oracle.quantize(np.random.default_rng(M * 3 + K + I).normal(0, 0.02, (K, N))
                                    .astype(np.float32), 1)
            rows = np.unique(np.r_[0, M // 2, M - 1])
            Co = oracle.matmul_i8(A[rows], B, sa[rows], sb, None, 0, 0)
            Yo = oracle.swiglu(Co[:, :I].copy(), Co[:, I:].copy(), alpha)
            assert bits_equal(Y[rows, :I].cpu().numpy(), Yo)
    finally:
        gpu.unpack(w)


def test_matmul_swiglu_host_operands(gpu, oracle):
    """Host A / scales in and host Y out, staged through HBM."""
    M, K, I = 384, 1024, 640
    rng = np.random.default_rng(5)
    w = _weights(gpu, oracle, rng, K, 2 * I)
    try:
        A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
        Y = np.full((M, I), np.nan, np.float32)
        assert gpu.matmul_i8_swiglu(A, w, sa, None, Y, M, K, 2 * I) == vnpu.OK
        B, sb = oracle.quantize(np.random.default_rng(5).normal(0, 0.02, (K, 2 * I))
                                .astype(np.float32), 1)
        rows = np.arange(0, M, 41)
        Co = oracle.matmul_i8(A[rows], B, sa[rows], sb, None, 0, 0)
        assert bits_equal(Y[rows], oracle.swiglu(Co[:, :I].copy(), Co[:, I:].copy(), 1.0))
    finally:
        gpu.unpack(w)
