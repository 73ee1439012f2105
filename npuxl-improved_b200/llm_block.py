"""Synthetic LLM decoder block through the vnpu ABI.

The op sequence is the reference's block driver (tools/llm_bench.cpp:213-326):
RMSNorm -> QUANTIZE_I8 -> MATMUL_I8 (fused QKV weight, d x 3d) -> split and
head-major transpose -> RoPE on Q, K -> causal ATTENTION -> back to token-major
-> QUANTIZE_I8 -> MATMUL_I8 (O) -> ADD residual -> RMSNorm -> QUANTIZE_I8 ->
MATMUL_I8 (fused gate/up, d x 2I) -> split -> SwiGLU -> QUANTIZE_I8 ->
MATMUL_I8 (down) -> ADD residual.  The reference has no KV cache (its
"decode" re-runs the block, llm_bench.cpp:453-455); this driver adds one:
K/V per head in a [heads][cap][head_dim] f32 cache, zero-initialised, and
decode attention over the cache with an additive mask of -inf on the slots
not yet written (fully masked 64-key blocks are skipped, so the result equals
attention over the filled prefix).

Two backends share the code:
* ``B200Block``: every tensor in HBM (torch allocations), vnpu commands on the
  library's stream, layout glue (split / transpose / cache append) as torch
  ops on the same stream; one decode step is captured as a CUDA graph and
  replayed (positions, cache slot and mask advance on the device).
* ``HostBlock``: numpy arrays handed to a vnpu library by host pointer - the
  reference library built from source, or (in tests) any vnpu library - with
  numpy glue, or the oracle restatement in place of a library.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

import vnpu


@dataclass
class BlockConfig:
    d: int = 4096
    heads: int = 32
    inter: int = 11008
    cap: int = 640
    eps: float = 1e-6
    theta: float = 10000.0
    seed: int = 0

    @property
    def head_dim(self) -> int:
        return self.d // self.heads


def make_weights(cfg: BlockConfig):
    """f32 weights N(0, 0.02) (K x N row-major) and unit RMSNorm weights."""
    rng = np.random.default_rng(cfg.seed + 1)
    d, i = cfg.d, cfg.inter
    w = {
        "qkv": rng.normal(0, 0.02, (d, 3 * d)).astype(np.float32),
        "o": rng.normal(0, 0.02, (d, d)).astype(np.float32),
        "gate_up": rng.normal(0, 0.02, (d, 2 * i)).astype(np.float32),
        "down": rng.normal(0, 0.02, (i, d)).astype(np.float32),
    }
    norms = (np.ones(d, np.float32), np.ones(d, np.float32))
    return w, norms


def weight_bytes(cfg: BlockConfig) -> int:
    d, i = cfg.d, cfg.inter
    return d * 3 * d + d * d + d * 2 * i + i * d


# ---------------------------------------------------------------------------
# Host backend (reference library / oracle)
# ---------------------------------------------------------------------------
class HostBlock:
    """The block on host arrays through a vnpu library (or the oracle)."""

    def __init__(self, cfg: BlockConfig, lib=None, oracle=None, threads: int = 0):
        self.cfg = cfg
        self.orc = oracle
        self.dev = vnpu.Device(lib, num_threads=threads) if lib is not None else None
        w, (self.n1, self.n2) = make_weights(cfg)
        self.w = {}
        for name, f in w.items():
            K, N = f.shape
            if self.dev is not None:
                B8 = np.empty((K, N), np.int8)
                sb = np.empty(N, np.float32)
                self.dev.quantize_i8(f, B8, sb, K, N, vnpu.QUANT_PER_COLUMN)
                self.w[name] = (self.dev.pack(B8, sb, K, N), B8, sb, K, N)
            else:
                B8, sb = self.orc.quantize(f, vnpu.QUANT_PER_COLUMN)
                self.w[name] = (None, B8, sb, K, N)
        hd = cfg.head_dim
        self.kc = np.zeros((cfg.heads, cfg.cap, hd), np.float32)
        self.vc = np.zeros((cfg.heads, cfg.cap, hd), np.float32)

    def close(self):
        if self.dev is not None:
            for (w, *_rest) in self.w.values():
                self.dev.unpack(w)
            self.dev.close()
            self.dev = None

    # --- ops ---------------------------------------------------------------
    def _rms(self, x, wn):
        if self.dev is None:
            return self.orc.rmsnorm(x, wn, self.cfg.eps, 0)
        y = np.empty_like(x)
        self.dev.rmsnorm(x, wn, y, x.shape[0], x.shape[1], self.cfg.eps)
        return y

    def _gemm(self, x, name):
        w, B8, sb, K, N = self.w[name]
        M = x.shape[0]
        if self.dev is None:
            A8, sa = self.orc.quantize(x, 0)
            return self.orc.matmul_i8(A8, B8, sa, sb, None, 0, 0)
        A8 = np.empty((M, K), np.int8)
        sa = np.empty(M, np.float32)
        self.dev.quantize_i8(x, A8, sa, M, K, 0)
        Cm = np.empty((M, N), np.float32)
        self.dev.matmul_i8(A8, w, sa, None, Cm, M, K, N)
        return Cm

    def _rope(self, Q, K, T, offset):
        cfg = self.cfg
        if self.dev is None:
            return self.orc.rope(Q, K, None, 1, cfg.heads, T, T, cfg.head_dim,
                                 position_offset=offset, theta=cfg.theta)
        Q = np.ascontiguousarray(Q)
        K = np.ascontiguousarray(K)
        self.dev.rope(Q, K, None, 1, cfg.heads, T, T, cfg.head_dim, position_offset=offset,
                      theta=cfg.theta)
        return Q, K

    def _attn(self, Q, K, V, sq, sk, causal, mask=None):
        cfg = self.cfg
        if self.dev is None:
            return self.orc.attention(Q, K, V, mask, 1, cfg.heads, sq, sk, cfg.head_dim, causal, 0.0)
        O = np.empty((1, cfg.heads, sq, cfg.head_dim), np.float32)
        self.dev.attention(Q, K, V, mask, O, 1, cfg.heads, sq, sk, cfg.head_dim, causal, 0.0)
        return O

    def _swiglu(self, g, u):
        if self.dev is None:
            return self.orc.swiglu(g, u, 1.0, 0)
        y = np.empty_like(g)
        self.dev.swiglu(g, u, y, g.size, 1.0)
        return y

    def _add(self, a, b):
        if self.dev is None:
            return self.orc.add(a, b, 1.0, 1.0, 0)
        y = np.empty_like(a)
        self.dev.add(a, b, y, a.size, 1.0, 1.0)
        return y

    # --- block -------------------------------------------------------------
    def forward(self, x: np.ndarray, pos0: int) -> np.ndarray:
        """Tokens x [T][d] at positions pos0.. ; prefill when pos0 == 0 and
        T > 1 (causal attention over the prompt), decode otherwise (attention
        over the cache with the unwritten slots masked)."""
        cfg = self.cfg
        T, d, H, hd = x.shape[0], cfg.d, cfg.heads, cfg.head_dim
        xn = self._rms(x, self.n1)
        qkv = self._gemm(xn, "qkv")
        heads = lambda a: np.ascontiguousarray(a.reshape(T, H, hd).transpose(1, 0, 2))[None]
        Q, K, V = heads(qkv[:, :d]), heads(qkv[:, d:2 * d]), heads(qkv[:, 2 * d:])
        Q, K = self._rope(Q, K, T, pos0)
        self.kc[:, pos0:pos0 + T] = K[0]
        self.vc[:, pos0:pos0 + T] = V[0]
        if T > 1:
            O = self._attn(Q, K, V, T, T, 1)
        else:
            mask = np.zeros((1, H, 1, cfg.cap), np.float32)
            mask[..., pos0 + 1:] = -np.inf
            O = self._attn(Q, self.kc[None], self.vc[None], 1, cfg.cap, 0, mask)
        attn = np.ascontiguousarray(O[0].transpose(1, 0, 2).reshape(T, d))
        x1 = self._add(x, self._gemm(attn, "o"))
        gu = self._gemm(self._rms(x1, self.n2), "gate_up")
        ff = self._swiglu(np.ascontiguousarray(gu[:, :cfg.inter]),
                          np.ascontiguousarray(gu[:, cfg.inter:]))
        return self._add(x1, self._gemm(ff, "down"))


# ---------------------------------------------------------------------------
# B200 backend
# ---------------------------------------------------------------------------
def _cmd(op, field, args):
    c = vnpu.Command()
    c.opcode = op
    setattr(c.args, field, args)
    return c


class B200Block:
    """The block with every tensor resident in HBM."""

    def __init__(self, cfg: BlockConfig, lib, dev, torch, fused: bool = True,
                 swiglu_epilogue: bool = True):
        self.cfg, self.lib, self.dev, self.t = cfg, lib, dev, torch
        # B200 opcodes: fused RMSNorm/SwiGLU -> QUANTIZE_I8 prologues, the QKV
        # projection with RoPE + cache append, projections with the residual add
        self.fused = fused
        # with fused: the gate/up projection with the SwiGLU in its epilogue
        # (VNPU_B200_OP_MATMUL_I8_SWIGLU) instead of the SwiGLU -> QUANTIZE_I8
        # prologue of the down projection
        self.swiglu_epilogue = fused and swiglu_epilogue
        self.stream = torch.cuda.ExternalStream(lib.b200_stream_handle(dev.stream))
        w, (n1, n2) = make_weights(cfg)
        self.n1 = torch.from_numpy(n1).cuda()
        self.n2 = torch.from_numpy(n2).cuda()
        self.w = {}
        for name, f in w.items():
            K, N = f.shape
            fd = torch.from_numpy(f).cuda()
            B8 = torch.empty((K, N), dtype=torch.int8, device="cuda")
            sb = torch.empty(N, device="cuda")
            torch.cuda.synchronize()
            dev.quantize_i8(fd.data_ptr(), B8.data_ptr(), sb.data_ptr(), K, N, vnpu.QUANT_PER_COLUMN)
            self.w[name] = (dev.pack(B8.data_ptr(), sb.data_ptr(), K, N), K, N)
            del fd, B8
        H, hd = cfg.heads, cfg.head_dim
        self.kc = torch.zeros((1, H, cfg.cap, hd), device="cuda")
        self.vc = torch.zeros((1, H, cfg.cap, hd), device="cuda")
        self.mask = torch.full((1, H, 1, cfg.cap), float("-inf"), device="cuda")
        self.pos = torch.zeros(1, dtype=torch.int32, device="cuda")   # decode position
        self.graph = None
        self.bufs = {}

    def close(self):
        self.graph = None
        for (w, _, _) in self.w.values():
            self.dev.unpack(w)

    def _buf(self, name, shape, dtype=None):
        t = self.t
        key = (name, tuple(shape))
        if key not in self.bufs:
            self.bufs[key] = t.empty(shape, dtype=dtype or t.float32, device="cuda")
        return self.bufs[key]

    def _submit(self, cmds):
        arr = (vnpu.Command * len(cmds))(*cmds)
        rc = self.lib.stream_submit(self.dev.stream, arr, len(cmds), None)
        if rc != vnpu.OK:
            raise RuntimeError(f"submit failed: {rc}")

    def _act_bufs(self, name, M):
        K = self.w[name][1]
        return (self._buf("a8_" + name, (M, K), self.t.int8), self._buf("sa_" + name, (M,)))

    def _mm_cmd(self, name, M, out_name, residual=None):
        """MATMUL_I8 of the already quantized activations of GEMM `name`;
        with `residual`, out = residual + product in one command
        (VNPU_B200_OP_MATMUL_I8_RESIDUAL, the bits of MATMUL_I8 then ADD_F32)."""
        w, K, N = self.w[name]
        a8, sa = self._act_bufs(name, M)
        out = self._buf(out_name, (M, N))
        if residual is not None:
            return vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_RESIDUAL, vnpu.MatmulI8ResidualArgs(
                a8.data_ptr(), w, sa.data_ptr(), None, residual.data_ptr(), out.data_ptr(), M, K,
                N, 0, 0, 0, 0, 0)), out
        return _cmd(vnpu.OP_MATMUL_I8, "matmul_i8",
                    vnpu.MatmulI8Args(a8.data_ptr(), w, sa.data_ptr(), None, out.data_ptr(), M, K,
                                      N, 0, 0, 0, vnpu.UNIT_GPU)), out

    def _gemm_cmds(self, x, name, out_name, residual=None):
        M, K = x.shape[0], self.w[name][1]
        a8, sa = self._act_bufs(name, M)
        q = _cmd(vnpu.OP_QUANTIZE_I8, "quantize_i8",
                 vnpu.QuantizeI8Args(x.data_ptr(), a8.data_ptr(), sa.data_ptr(), M, K, 0, 0))
        mm, out = self._mm_cmd(name, M, out_name, residual)
        return [q, mm], out

    def _norm_gemm_cmds(self, x, wn, name, out_name):
        """RMSNorm -> QUANTIZE_I8 -> MATMUL_I8: one fused prologue command
        (VNPU_B200_OP_RMSNORM_QUANTIZE_I8) when enabled, else the three ops."""
        if not self.fused:
            c, xn = self._rms_cmd(x, wn, out_name + "_n")
            cmds, out = self._gemm_cmds(xn, name, out_name)
            return [c] + cmds, out
        M, K = x.shape
        a8, sa = self._act_bufs(name, M)
        pro = vnpu.b200_command(vnpu.OP_B200_RMSNORM_QUANTIZE_I8, vnpu.RmsnormQuantizeArgs(
            x.data_ptr(), wn.data_ptr(), None, a8.data_ptr(), sa.data_ptr(), M, K, self.cfg.eps, 0))
        mm, out = self._mm_cmd(name, M, out_name)
        return [pro, mm], out

    def _swiglu_gemm_cmds(self, g, u, name, out_name, residual=None):
        """SwiGLU -> QUANTIZE_I8 -> MATMUL_I8 (fused prologue when enabled)."""
        T, inter = g.shape
        if not self.fused:
            ff = self._buf(f"ff{T}", (T, inter))
            sw = _cmd(vnpu.OP_SWIGLU_F32, "swiglu",
                      vnpu.SwigluArgs(g.data_ptr(), u.data_ptr(), ff.data_ptr(), T * inter,
                                      1.0, 0, 0))
            cmds, out = self._gemm_cmds(ff, name, out_name, residual)
            return [sw] + cmds, out
        a8, sa = self._act_bufs(name, T)
        pro = vnpu.b200_command(vnpu.OP_B200_SWIGLU_QUANTIZE_I8, vnpu.SwigluQuantizeArgs(
            g.data_ptr(), u.data_ptr(), None, a8.data_ptr(), sa.data_ptr(), T, inter, 1.0,
            g.stride(0)))
        mm, out = self._mm_cmd(name, T, out_name, residual)
        return [pro, mm], out

    def _rms_cmd(self, x, wn, out_name):
        y = self._buf(out_name, tuple(x.shape))
        return _cmd(vnpu.OP_RMSNORM_F32, "rmsnorm",
                    vnpu.RmsnormArgs(x.data_ptr(), wn.data_ptr(), y.data_ptr(), x.shape[0],
                                     x.shape[1], self.cfg.eps, 0)), y

    def _add_cmd(self, a, b, out_name):
        y = self._buf(out_name, tuple(a.shape))
        return _cmd(vnpu.OP_ADD_F32, "binary",
                    vnpu.BinaryArgs(a.data_ptr(), b.data_ptr(), y.data_ptr(), a.numel(), 1.0, 1.0,
                                    0, 0)), y

    def forward(self, x, pos0: int, positions=None):
        """x [T][d] on the device.  Prefill (T > 1, pos0 == 0) or one decode
        token; `positions` (device int32[1]) replaces pos0 for graph replay."""
        t, cfg = self.t, self.cfg
        T, d, H, hd = x.shape[0], cfg.d, cfg.heads, cfg.head_dim
        with t.cuda.stream(self.stream):
            if self.fused:
                # RMSNorm -> QUANTIZE_I8, then the QKV projection with RoPE and
                # the cache append in its epilogue (VNPU_B200_OP_QKV_ROPE_APPEND).
                w, K_in, _ = self.w["qkv"]
                a8, sa = self._act_bufs("qkv", T)
                pro = vnpu.b200_command(vnpu.OP_B200_RMSNORM_QUANTIZE_I8, vnpu.RmsnormQuantizeArgs(
                    x.data_ptr(), self.n1.data_ptr(), None, a8.data_ptr(), sa.data_ptr(), T, d,
                    cfg.eps, 0))
                Q = self._buf(f"Q{T}", (1, H, T, hd))
                K = self._buf(f"K{T}", (1, H, T, hd)) if T > 1 else None
                V = self._buf(f"V{T}", (1, H, T, hd)) if T > 1 else None
                qkv = vnpu.b200_command(vnpu.OP_B200_QKV_ROPE_APPEND, vnpu.QkvRopeAppendArgs(
                    a8.data_ptr(), w, sa.data_ptr(), None, Q.data_ptr(),
                    K.data_ptr() if K is not None else None,
                    V.data_ptr() if V is not None else None, self.kc.data_ptr(),
                    self.vc.data_ptr(), self.mask.data_ptr(),
                    positions.data_ptr() if positions is not None else None, T, K_in, H, hd,
                    cfg.cap, pos0, cfg.theta, 1.0, 0, 0))
                self._submit([pro, qkv])
            else:
                cmds, qkv = self._norm_gemm_cmds(x, self.n1, "qkv", f"qkv{T}")
                self._submit(cmds)
                Q = qkv[:, :d].reshape(T, H, hd).transpose(0, 1).contiguous()[None]
                K = qkv[:, d:2 * d].reshape(T, H, hd).transpose(0, 1).contiguous()[None]
                V = qkv[:, 2 * d:].reshape(T, H, hd).transpose(0, 1).contiguous()[None]
                rope = vnpu.RopeArgs(Q.data_ptr(), K.data_ptr(),
                                     positions.data_ptr() if positions is not None else None,
                                     1, H, T, T, hd, pos0, 0, cfg.theta, 1.0)
                self._submit([_cmd(vnpu.OP_ROPE_F32, "rope", rope)])
            # fused prefill: the attention writes token-major rows, the O
            # projection's input, so no transpose copy follows
            tok_major = self.fused and T > 1
            O = self._buf(f"O{T}", (T, d) if tok_major else (1, H, T, hd))
            if T > 1:
                if not self.fused:
                    self.kc[:, :, pos0:pos0 + T].copy_(K)
                    self.vc[:, :, pos0:pos0 + T].copy_(V)
                    self.mask[..., pos0:pos0 + T] = 0.0
                att = vnpu.AttentionArgs(Q.data_ptr(), K.data_ptr(), V.data_ptr(), None,
                                         O.data_ptr(), None, 0, 1, H, T, T, hd, 1, 0.0, 0)
            else:
                if not self.fused:
                    idx = positions.long() if positions is not None else t.tensor([pos0], device="cuda")
                    self.kc.index_copy_(2, idx, K)
                    self.vc.index_copy_(2, idx, V)
                    self.mask.index_fill_(3, idx, 0.0)
                att = vnpu.AttentionArgs(Q.data_ptr(), self.kc.data_ptr(), self.vc.data_ptr(),
                                         self.mask.data_ptr(), O.data_ptr(), None, 0, 1, H, 1,
                                         cfg.cap, hd, 0, 0.0, 0)
            acmd = _cmd(vnpu.OP_ATTENTION_F32, "attention", att)
            if tok_major:
                acmd.flags = vnpu.CMD_FLAG_ATTN_TOKEN_MAJOR
            self._submit([acmd])
            attn = O if tok_major else O[0].transpose(0, 1).reshape(T, d).contiguous()
            if self.swiglu_epilogue:
                # O projection + residual; RMSNorm -> QUANTIZE_I8; the gate/up
                # projection writes swiglu(gate, up) (MATMUL_I8_SWIGLU); the
                # down projection quantizes it and adds the residual.
                cmds, x1 = self._gemm_cmds(attn, "o", f"x1{T}", residual=x)
                w, K_in, N_gu = self.w["gate_up"]
                a8, sa = self._act_bufs("gate_up", T)
                pro = vnpu.b200_command(vnpu.OP_B200_RMSNORM_QUANTIZE_I8, vnpu.RmsnormQuantizeArgs(
                    x1.data_ptr(), self.n2.data_ptr(), None, a8.data_ptr(), sa.data_ptr(), T, d,
                    cfg.eps, 0))
                ff = self._buf(f"ff{T}", (T, cfg.inter))
                sw = vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_SWIGLU, vnpu.MatmulI8SwigluArgs(
                    a8.data_ptr(), w, sa.data_ptr(), None, ff.data_ptr(), T, K_in, N_gu, 0, 0, 0,
                    1.0, 0))
                cmds3, y = self._gemm_cmds(ff, "down", f"y{T}", residual=x1)
                self._submit(cmds + [pro, sw] + cmds3)
                self._keep = (Q, K, V, attn, ff)
                return y
            if self.fused:
                # the residual adds ride on the O and down projections
                # (VNPU_B200_OP_MATMUL_I8_RESIDUAL)
                cmds, x1 = self._gemm_cmds(attn, "o", f"x1{T}", residual=x)
                cmds2, gu = self._norm_gemm_cmds(x1, self.n2, "gate_up", f"gu{T}")
                self._submit(cmds + cmds2)
            else:
                cmds, proj = self._gemm_cmds(attn, "o", f"proj{T}")
                a, x1 = self._add_cmd(x, proj, f"x1{T}")
                cmds2, gu = self._norm_gemm_cmds(x1, self.n2, "gate_up", f"gu{T}")
                self._submit(cmds + [a] + cmds2)
            if self.fused:
                # SWIGLU_QUANTIZE_I8 reads the two halves of gu in place (ld)
                g, u = gu[:, :cfg.inter], gu[:, cfg.inter:]
            else:
                g = gu[:, :cfg.inter].contiguous()
                u = gu[:, cfg.inter:].contiguous()
            if self.fused:
                cmds3, y = self._swiglu_gemm_cmds(g, u, "down", f"y{T}", residual=x1)
                self._submit(cmds3)
            else:
                cmds3, down = self._swiglu_gemm_cmds(g, u, "down", f"down{T}")
                a2, y = self._add_cmd(x1, down, f"y{T}")
                self._submit(cmds3 + [a2])
            # keep the temporaries alive until the stream has used them
            self._keep = (Q, K, V, attn, g, u)
        return y

    def capture_decode(self, x):
        """Record one decode step (token x [1][d] at device position self.pos)
        as a CUDA graph that also advances self.pos; returns the output buffer."""
        t = self.t
        self.dev.sync()
        t.cuda.synchronize()
        g = t.cuda.CUDAGraph()
        with t.cuda.graph(g, stream=self.stream, capture_error_mode="relaxed"):
            y = self.forward(x, 0, positions=self.pos)
            self.pos.add_(1)
        self.graph = g
        return y

    def replay_decode(self):
        """One decode step: the graph replays on the library stream, ordered
        with everything else this block submits there."""
        with self.t.cuda.stream(self.stream):
            self.graph.replay()
