"""ctypes binding of liboracle.so, the CPU restatement of the reference's
arithmetic (oracle.c / oracle.h).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py load it, as the checker.  The B200 library and
its Python binding (npuxl-improved_b200/vnpu.py) never import it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from vnpu import QUANT_PER_COLUMN, QUANT_PER_ROW, UNIT_VOODOO, _sig, f32, ptr, u32, u64, vp

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")


class Oracle:
    FORM_AVX2 = 0
    FORM_SCALAR = 1
    FORM_STREAM = 2

    def __init__(self, path: str = ORACLE_LIB):
        self.h = C.CDLL(path)
        h = self.h
        i8p = C.c_void_p
        self._matmul = _sig(h, "oracle_matmul_i8", None, i8p, u32, i8p, vp, vp, vp, vp, u32, u32,
                            u32, u32, u32, C.c_int)
        self._acc = _sig(h, "oracle_gemm_i8_acc", None, i8p, u32, i8p, u32, vp, u32, u32, u32)
        self._quant = _sig(h, "oracle_quantize_i8", C.c_int, vp, vp, vp, u64, u64, u32)
        self._colsums = _sig(h, "oracle_column_sums", None, vp, u32, u32, u32, u32, vp, vp)
        self._rms = _sig(h, "oracle_rmsnorm", None, vp, vp, vp, u32, u32, f32, C.c_int)
        self._rope = _sig(h, "oracle_rope", None, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32,
                          f32, f32)
        self._swiglu = _sig(h, "oracle_swiglu", None, vp, vp, vp, u64, f32, C.c_int)
        self._add = _sig(h, "oracle_add", None, vp, vp, vp, u64, f32, f32, C.c_int)
        self._attn = _sig(h, "oracle_attention", None, vp, vp, vp, vp, vp, u32, u32, u32, u32,
                          u32, u32, f32)
        self._mm_f32 = _sig(h, "oracle_matmul_f32", None, vp, vp, vp, vp, u32, u32, u32, u32, u32,
                            u32, u32, u32, f32, f32, u32, u32, vp, u32, u32, u32, u32, u32, u32,
                            C.c_int, C.c_int)
        self._f32_geom = _sig(h, "oracle_f32_tile_geometry", None, u32, u32, u32, u32, u32, u32,
                              u32, C.c_int, C.POINTER(u32), C.POINTER(u32), C.POINTER(u32))
        self._mm_dev = _sig(h, "oracle_matmul_i8_device", None, i8p, u32, i8p, vp, vp, vp, vp, u32,
                            u32, u32, u32, u32, u32, u32, u32, u32, C.c_int, C.c_int, u64)
        self._i8_geom = _sig(h, "oracle_i8_tile_geometry", None, u32, u32, u32, u32, u32, u32,
                             C.c_int, u64, C.POINTER(u32), C.POINTER(u32))
        self._i8_map = _sig(h, "oracle_i8_form_map", None, u32, u32, u32, u32, u32, u32, u32,
                            C.c_int, C.c_int, u64, vp)
        self._i8_form = _sig(h, "oracle_i8_element_form", C.c_int, u32, C.c_int, C.c_int, u32, u32,
                             u32, u32, u32, u32, u32)
        self.fast_expf = _sig(h, "oracle_fast_expf", f32, f32, C.c_int)
        self.dequant = _sig(h, "oracle_dequant", f32, C.c_int32, f32, f32, C.POINTER(f32), u32,
                            C.c_int)

    def quantize(self, X: np.ndarray, axis: int = QUANT_PER_ROW):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        Y = np.empty((rows, cols), np.int8)
        n = rows if axis == QUANT_PER_ROW else (cols if axis == QUANT_PER_COLUMN else 1)
        s = np.empty(n, np.float32)
        rc = self._quant(ptr(X), ptr(Y), ptr(s), rows, cols, axis)
        assert rc == 0
        return Y, s

    def gemm_acc(self, A: np.ndarray, B: np.ndarray) -> np.ndarray:
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        acc = np.empty((M, N), np.int32)
        self._acc(ptr(A), K, ptr(B), N, ptr(acc), M, K, N)
        return acc

    def matmul_i8(self, A, B, scale_a, scale_b, bias=None, epilogue=0, form=0) -> np.ndarray:
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        Cm = np.empty((M, N), np.float32)
        self._matmul(ptr(A), K, ptr(B), ptr(scale_a), ptr(scale_b), ptr(bias), ptr(Cm), N, M, K,
                     N, epilogue, form)
        return Cm

    def matmul_i8_device(self, A, B, scale_a, scale_b, bias=None, epilogue=0, unit=UNIT_VOODOO,
                         threads=8, tiles=(128, 128, 64), pack_b=1, avx2=1, l2_bytes=0):
        """MATMUL_I8 as a reference device with `threads` workers, tile
        defaults `tiles`, VNPU_PACK=`pack_b`, the AVX2 (or scalar) ISA and
        an L2 of `l2_bytes` computes it with no command flags: every element
        in the rounding form of the kernel that owns it."""
        A = np.ascontiguousarray(A, np.int8)
        B = np.ascontiguousarray(B, np.int8)
        M, K = A.shape
        N = B.shape[1]
        Cm = np.empty((M, N), np.float32)
        self._mm_dev(ptr(A), K, ptr(B), ptr(scale_a), ptr(scale_b), ptr(bias), ptr(Cm), N, M, K, N,
                     epilogue, unit, threads, tiles[0], tiles[2], pack_b, avx2, l2_bytes)
        return Cm

    def i8_tile_geometry(self, unit, M, N, threads=8, tiles=(128, 128, 64), pack_b=1, l2_bytes=0):
        tm, tn = u32(), u32()
        self._i8_geom(unit, M, N, threads, tiles[0], tiles[2], pack_b, l2_bytes, C.byref(tm),
                      C.byref(tn))
        return tm.value, tn.value

    def i8_forms(self, M, K, N, unit=UNIT_VOODOO, threads=8, tiles=(128, 128, 64), pack_b=1,
                 avx2=1, l2_bytes=0) -> np.ndarray:
        """ORACLE form of every element of an M x K x N MATMUL_I8."""
        F = np.empty((M, N), np.int32)
        self._i8_map(unit, M, K, N, threads, tiles[0], tiles[2], pack_b, avx2, l2_bytes, ptr(F))
        return F

    def matmul_i8_model(self, model, A, B, scale_a, scale_b, bias=None, epilogue=0, rows=None,
                        n_full=0, col_base=0, unit=0) -> np.ndarray:
        """Rows `rows` (all if None) of MATMUL_I8 as the reference device
        `model` (a B200 device's vnpu_b200_reference_model_t) rounds them, for
        a product whose output has n_full columns (0: B's) of which B holds
        columns col_base.. ; the tile map is that of all M rows of A."""
        M, K = A.shape
        N = B.shape[1]
        n_full = n_full or N
        if model.epilogue_forced:
            F = np.full((M, N), {0: 0, 1: 2, 2: 1}[model.epilogue_form], np.int32)
        else:
            F = self.i8_forms(M, K, n_full, unit, model.num_threads,
                              (model.tile_m, model.tile_k, model.tile_n), model.pack_b,
                              0 if model.scalar_isa else 1, model.l2_bytes)[:, col_base:col_base + N]
        rows = np.arange(M) if rows is None else np.asarray(rows)
        outs = [self.matmul_i8(A[rows], B, scale_a[rows] if scale_a is not None else None,
                               scale_b, bias, epilogue, f).view(np.int32) for f in (0, 1, 2)]
        return np.choose(F[rows], outs).view(np.float32)

    def matmul_f32(self, A, B, M, K, N, bias=None, C=None, lda=0, ldb=0, ldc=0, trans_a=0,
                   trans_b=0, alpha=1.0, beta=0.0, epilogue=0, unit=UNIT_VOODOO, tile_mask=None,
                   mask_tile_m=0, mask_tile_n=0, threads=8, tiles=(128, 128, 64), pack_b=1,
                   avx2=1) -> np.ndarray:
        """MATMUL_F32 as a reference device with `threads` threads, tile
        defaults `tiles`, VNPU_PACK=`pack_b` and the AVX2 (or scalar) ISA
        computes it.  C (optional) holds the prior contents beta reads."""
        ldc_ = ldc or N
        out = np.zeros((M, ldc_), np.float32) if C is None else np.array(C, np.float32, copy=True)
        self._mm_f32(ptr(A), ptr(B), ptr(bias), ptr(out), M, K, N, lda, ldb, ldc, trans_a, trans_b,
                     alpha, beta, epilogue, unit, ptr(tile_mask), mask_tile_m, mask_tile_n,
                     threads, tiles[0], tiles[1], tiles[2], pack_b, avx2)
        return out

    def f32_tile_geometry(self, unit, M, N, threads=8, tiles=(128, 128, 64), pack_b=1):
        tm, tk, tn = u32(), u32(), u32()
        self._f32_geom(unit, M, N, threads, tiles[0], tiles[1], tiles[2], pack_b, C.byref(tm),
                       C.byref(tk), C.byref(tn))
        return tm.value, tk.value, tn.value

    def column_sums(self, B: np.ndarray, trans_b: int = 0):
        B = np.ascontiguousarray(B, np.int8)
        K, N = (B.shape[1], B.shape[0]) if trans_b else B.shape
        sums = np.empty(N, np.int32)
        canon = np.empty((K, N), np.int8)
        self._colsums(ptr(B), K, N, 0, trans_b, ptr(sums), ptr(canon))
        return sums, canon

    def rmsnorm(self, X, W, eps, form=0):
        X = np.ascontiguousarray(X, np.float32)
        Y = np.empty_like(X)
        self._rms(ptr(X), ptr(W), ptr(Y), X.shape[0], X.shape[1], eps, form)
        return Y

    def rope(self, Q, K, positions, batch, heads, q_seq, k_seq, head_dim, position_offset=0,
             interleaved=0, theta=10000.0, scaling=1.0):
        Q = None if Q is None else np.array(Q, np.float32, copy=True)
        K = None if K is None else np.array(K, np.float32, copy=True)
        self._rope(ptr(Q), ptr(K), ptr(positions), batch, heads, q_seq, k_seq, head_dim,
                   position_offset, interleaved, theta, scaling)
        return Q, K

    def swiglu(self, g, u, alpha=1.0, form=0):
        Y = np.empty_like(g)
        self._swiglu(ptr(g), ptr(u), ptr(Y), g.size, alpha, form)
        return Y

    def add(self, A, B, alpha=1.0, beta=1.0, form=0):
        Y = np.empty_like(A)
        self._add(ptr(A), ptr(B), ptr(Y), A.size, alpha, beta, form)
        return Y

    def attention(self, Q, K, V, mask, batch, heads, seq_q, seq_k, head_dim, causal=1, scale=0.0):
        O = np.empty((batch, heads, seq_q, head_dim), np.float32)
        self._attn(ptr(Q), ptr(K), ptr(V), ptr(mask), ptr(O), batch, heads, seq_q, seq_k,
                   head_dim, causal, scale)
        return O
