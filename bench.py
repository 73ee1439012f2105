"""Benchmark of the B200 MATMUL_I8 hot path (one JSON line on rank 0).

Workload: column-sharded MATMUL_I8, M=8192, K=8192,
N=28672, split evenly over the N GPUs (strong scaling); activations f32
U[-1,1] quantized per row by QUANTIZE_I8 every step, weights f32 N(0,0.02)
quantized per column and packed once (resident).  One step = QUANTIZE_I8 of
A + MATMUL_I8 on this rank's column shard.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

value   - whole-job int8 TOPS with inputs resident in HBM, device-timed with
          CUDA events on the library's stream, max over ranks.
e2e     - the same step through the C ABI with HOST buffers: A f32 from pinned
          host memory in, C f32 shard to pinned host memory out, copies inside
          the timed region.
roofline- the tcgen05 GEMM kernel alone, algorithmic int8 ops / event time,
          against 2x the measured dense bf16 rate (int8 runs at twice bf16 on
          B200; nominal 4.5 POPS).
--impl reference times the reference's own CPU implementation (built from
its sources into oracle/_ref) on this host's cores, on a row sample of the
same workload, through the same ABI calls.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "npuxl-improved_b200"))

import numpy as np  # noqa: E402

import vnpu  # noqa: E402
from shard import column_shard  # noqa: E402

M_TOTAL, K_TOTAL, N_TOTAL = 8192, 8192, 28672
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libvnpu_ref.so")
ORACLE_LIB = os.path.join(ROOT, "oracle", "liboracle.so")
WORKLOAD = ("MATMUL_I8 column-sharded M=8192 K=8192 N=28672 (QUANTIZE_I8 per row of A "
            "each step; weights per-column quantized, packed, resident)")
METRIC = "int8 GEMM TOPS (MATMUL_I8 8192x8192x28672 column-sharded)"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "bf16": p["bf16_tflops"],
                "bf16_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def profile_traffic(key: str):
    """DRAM bytes per launch recorded from an ncu capture (profiles/*.md)."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for f in sorted(os.listdir(pdir)):
        if not f.endswith(".md"):
            continue
        for line in open(os.path.join(pdir, f)):
            if line.startswith(f"dram_bytes_per_launch[{key}]:"):
                try:
                    return int(line.split("]:", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """NVML SM clock / throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None
        self.names = {
            0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap", 0x2: "applications_clocks_setting",
            0x100: "sync_boost",
        }

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                r = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.names.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nvml:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.nvml:
            self.t.join()

    def report(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ===========================================================================
# CPU reference arm / baseline
# ===========================================================================
def reference_sample(rows: int, steps: int, warmup: int, threads: int, A=None, B8=None, sb=None):
    """Time QUANTIZE_I8 and MATMUL_I8 (each separately) of `rows` rows of the
    workload on the reference's CPU implementation (host buffers, its own
    thread pool).  A (rows x K f32) and the weights B8 (K x N int8, per-column
    scales sb) may be given (the GPU arm passes its own, to check its rows);
    otherwise they are drawn with the workload's distributions.  Returns the
    timings and the sample's output rows."""
    if os.path.exists(REF_LIB):
        lib, kind = vnpu.Lib(REF_LIB), "reference"
        os.environ.setdefault("VNPU_FORCE_ISA", "avx2")
    else:
        lib, kind = None, "port"
    rng = np.random.default_rng(1)
    n = N_TOTAL
    if A is None:
        A = rng.uniform(-1, 1, (rows, K_TOTAL)).astype(np.float32)
    if lib is None:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from vnpu_oracle import Oracle
        orc = Oracle(ORACLE_LIB)
        if B8 is None:
            B8, sb = orc.quantize(rng.normal(0, 0.02, (K_TOTAL, n)).astype(np.float32), 1)
        tq, tm = [], []
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            A8, sa = orc.quantize(A, 0)
            t1 = time.perf_counter()
            Cout = orc.matmul_i8(A8, B8, sa, sb, None, 0, 0)
            t2 = time.perf_counter()
            if i >= warmup:
                tq.append(t1 - t0)
                tm.append(t2 - t1)
        cores = 1
    else:
        dev = vnpu.Device(lib, num_threads=threads)
        if B8 is None:
            Bf = rng.normal(0, 0.02, (K_TOTAL, n)).astype(np.float32)
            B8 = np.empty((K_TOTAL, n), np.int8)
            sb = np.empty(n, np.float32)
            dev.quantize_i8(Bf, B8, sb, K_TOTAL, n, vnpu.QUANT_PER_COLUMN)
            del Bf
        w = dev.pack(B8, sb, K_TOTAL, n)
        A8 = np.empty((rows, K_TOTAL), np.int8)
        sa = np.empty(rows, np.float32)
        Cout = np.empty((rows, n), np.float32)
        tq, tm = [], []
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            dev.quantize_i8(A, A8, sa, rows, K_TOTAL, vnpu.QUANT_PER_ROW)
            t1 = time.perf_counter()
            dev.matmul_i8(A8, w, sa, None, Cout, rows, K_TOTAL, n, unit=vnpu.UNIT_VOODOO)
            t2 = time.perf_counter()
            if i >= warmup:
                tq.append(t1 - t0)
                tm.append(t2 - t1)
        cores = dev.info().num_threads
        dev.unpack(w)
        dev.close()
    q, m = statistics.median(tq), statistics.median(tm)
    t = q + m
    ops = 2.0 * rows * K_TOTAL * n
    return {"value": ops / t / 1e12, "unit": "TOPS", "cores": cores, "kind": kind,
            "sample": f"{rows} rows of A ({rows}x{K_TOTAL}x{n}, quantize+matmul, host buffers), "
                      f"median of {len(tq)} steps, {t:.3f} s/step",
            "seconds_per_step": t,
            "quantize_i8": {"seconds": q, "gbs": 5.0 * rows * K_TOTAL / q / 1e9,
                            "bytes": 5 * rows * K_TOTAL},
            "matmul_i8": {"seconds": m, "tops": ops / m / 1e12},
            "C": Cout}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # about 1 s of work per step on a many-core host
    rows = int(os.environ.get("VNPU_BENCH_REF_ROWS", "32"))
    r = reference_sample(rows, max(1, args.steps), max(0, min(args.warmup, 2)), threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "TOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["seconds_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_rows": rows, "M": M_TOTAL, "K": K_TOTAL,
                   "N": N_TOTAL, "isa": os.environ.get("VNPU_FORCE_ISA", "port")},
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample",
                                           "quantize_i8", "matmul_i8")},
        "e2e": {"value": r["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ===========================================================================
# B200 arm
# ===========================================================================
class Stream:
    """The library's CUDA stream seen from torch, for events."""

    def __init__(self, lib, dev):
        import torch
        self.torch = torch
        self.cs = torch.cuda.ExternalStream(lib.b200_stream_handle(dev.stream))

    def event(self):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record(self.cs)
        return e


def cmd_quantize(X, Y, s, rows, cols):
    c = vnpu.Command()
    c.opcode = vnpu.OP_QUANTIZE_I8
    c.args.quantize_i8 = vnpu.QuantizeI8Args(X, Y, s, rows, cols, vnpu.QUANT_PER_ROW, 0)
    return c


def cmd_matmul(A, w, sa, bias, Cp, M, K, N, epi=0, ldc=0):
    c = vnpu.Command()
    c.opcode = vnpu.OP_MATMUL_I8
    c.args.matmul_i8 = vnpu.MatmulI8Args(A, w, sa, bias, Cp, M, K, N, 0, ldc, epi,
                                         vnpu.UNIT_GPU)
    return c


def _copy_cmd(dst, src, nbytes):
    c = vnpu.Command()
    c.opcode = vnpu.OP_COPY
    c.args.copy = vnpu.CopyArgs(dst, src, nbytes, 0)
    return c


def submit(lib, dev, cmds):
    arr = (vnpu.Command * len(cmds))(*cmds)
    rc = lib.stream_submit(dev.stream, arr, len(cmds), None)
    if rc != vnpu.OK:
        raise RuntimeError(f"submit failed: {rc}")


def time_loop(lib, dev, st, cmds, iters):
    """Average ms of one iteration of `cmds`, device-timed on the library stream."""
    arr = (vnpu.Command * len(cmds))(*cmds)
    n = len(cmds)
    e0 = st.event()
    for _ in range(iters):
        if lib.stream_submit(dev.stream, arr, n, None) != vnpu.OK:
            raise RuntimeError("submit failed")
    e1 = st.event()
    if dev.sync() != vnpu.OK:
        raise RuntimeError("stream error")
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def make_weights(lib, dev, torch, K, N, seed, shard=None, keep_int8=False):
    """f32 N(0,0.02) weights -> QUANTIZE_I8 per column on the GPU -> pack.
    keep_int8: also return the K x N int8 matrix (a 4th value)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    n0, n1 = shard if shard else (0, N)
    Bf = torch.empty((K, N), device="cuda").normal_(0, 0.02, generator=g)[:, n0:n1].contiguous()
    n = n1 - n0
    B8 = torch.empty((K, n), dtype=torch.int8, device="cuda")
    sb = torch.empty(n, device="cuda")
    torch.cuda.synchronize()
    dev.quantize_i8(Bf.data_ptr(), B8.data_ptr(), sb.data_ptr(), K, n, vnpu.QUANT_PER_COLUMN)
    w = dev.pack(B8.data_ptr(), sb.data_ptr(), K, n)
    del Bf
    if keep_int8:
        return w, sb, n, B8
    del B8
    return w, sb, n


def gemm_secondary(lib, dev, st, torch, M, K, N, epi, with_bias, iters=20):
    g = torch.Generator(device="cuda").manual_seed(M + N)
    Af = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
    A8 = torch.empty((M, K), dtype=torch.int8, device="cuda")
    sa = torch.empty(M, device="cuda")
    w, sb, n = make_weights(lib, dev, torch, K, N, seed=7)
    bias = torch.empty(N, device="cuda").normal_(0, 0.01, generator=g) if with_bias else None
    Cm = torch.empty((M, N), device="cuda")
    torch.cuda.synchronize()
    q = cmd_quantize(Af.data_ptr(), A8.data_ptr(), sa.data_ptr(), M, K)
    mm = cmd_matmul(A8.data_ptr(), w, sa.data_ptr(), bias.data_ptr() if bias is not None else None,
                    Cm.data_ptr(), M, K, N, epi)
    time_loop(lib, dev, st, [q, mm], 3)
    ms = time_loop(lib, dev, st, [mm], iters)
    kernel = lib.b200_last_matmul_kernel().decode()
    out = {"shape": f"{M}x{K}x{N}", "epilogue": ["none", "relu", "silu", "gelu"][epi],
           "bias": with_bias, "ms": ms, "tops": 2.0 * M * K * N / ms / 1e9, "kernel": kernel}
    if ms < 0.05:
        # Launch-bound shape: also the device time per launch in a CUDA graph
        # (the submit loop above includes the host's per-command cost).
        graph = dev.capture([mm] * 20)
        dev.replay(graph)
        dev.sync()
        e0 = st.event()
        for _ in range(10):
            dev.replay(graph)
        e1 = st.event()
        dev.sync()
        e1.synchronize()
        ms_g = e0.elapsed_time(e1) / 200
        lib.b200_graph_destroy(graph)
        out.update({"ms_graph": ms_g, "tops_graph": 2.0 * M * K * N / ms_g / 1e9})
        # Library comparator at the same launch-bound size: cuBLAS int8
        # (torch._int_mm) in a CUDA graph of 20 launches.
        try:
            A_ = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda")
            B_ = torch.randint(-128, 128, (N, K), dtype=torch.int8, device="cuda").t()
            torch._int_mm(A_, B_)
            torch.cuda.synchronize()
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_):
                for _ in range(20):
                    torch._int_mm(A_, B_)
            g_.replay()
            torch.cuda.synchronize()
            c0 = torch.cuda.Event(enable_timing=True)
            c1 = torch.cuda.Event(enable_timing=True)
            c0.record()
            for _ in range(10):
                g_.replay()
            c1.record()
            torch.cuda.synchronize()
            out["cublas_int8_ms_graph"] = c0.elapsed_time(c1) / 200
            del g_, A_, B_
        except Exception as exc:  # library comparator only
            out["cublas_int8_ms_graph"] = f"unavailable: {exc}"
    dev.unpack(w)
    return out


def cmd_matmul_f32(A, B, Cp, M, K, N, trans_b=0):
    c = vnpu.Command()
    c.opcode = vnpu.OP_MATMUL_F32
    c.args.matmul_f32 = vnpu.MatmulF32Args(A, B, None, Cp, M, K, N, 0, 0, 0, 0, trans_b, 1.0,
                                           0.0, 0, vnpu.UNIT_AUTO, 0, None, 0, 0)
    return c


def f32_secondary(lib, dev, st, torch, M, K, N, trans_b=0, iters=5, ref_rows=64):
    """MATMUL_F32 (the legacy shims' GEMM): CUDA-core kernels that reproduce
    the reference's per-tile rounding; inputs larger than L2.  The reference
    is timed on `ref_rows` rows of the same GEMM on the host cores."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    A = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
    B = torch.empty((N, K) if trans_b else (K, N), device="cuda").uniform_(-1, 1, generator=g)
    Cm = torch.empty((M, N), device="cuda")
    torch.cuda.synchronize()
    mm = cmd_matmul_f32(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, K, N, trans_b)
    time_loop(lib, dev, st, [mm], 2)
    ms = time_loop(lib, dev, st, [mm], iters)
    out = {"shape": f"{M}x{K}x{N}", "trans_b": trans_b, "ms": ms,
           "tflops": 2.0 * M * K * N / ms / 1e9,
           "kernel": "gemm_f32_kernel<%s>" % ("kF32Dot8" if trans_b else "kF32Block")}
    # Library comparator: cuBLAS FP32 SGEMM (TF32 off) on the same shape; it
    # sums in its own order, so its bits differ from the reference's.
    try:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        Bm = B.t() if trans_b else B
        torch.mm(A, Bm)
        torch.cuda.synchronize()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(iters):
            torch.mm(A, Bm)
        c1.record()
        torch.cuda.synchronize()
        out["cublas_sgemm_tflops"] = 2.0 * M * K * N / (c0.elapsed_time(c1) / iters) / 1e9
        torch.backends.cuda.matmul.allow_tf32 = prev
    except Exception as exc:  # library comparator only
        out["cublas_sgemm_tflops"] = f"unavailable: {exc}"
    if os.path.exists(REF_LIB):
        os.environ.setdefault("VNPU_FORCE_ISA", "avx2")
        rlib = vnpu.Lib(REF_LIB)
        with vnpu.Device(rlib, num_threads=os.cpu_count() or 1) as rd:
            Ah = A[:ref_rows].cpu().numpy()
            Bh = B.cpu().numpy()
            Ch = np.empty((ref_rows, N), np.float32)
            rd.matmul_f32(Ah, Bh, Ch, ref_rows, K, N, trans_b=trans_b)
            t0 = time.perf_counter()
            rd.matmul_f32(Ah, Bh, Ch, ref_rows, K, N, trans_b=trans_b)
            t = time.perf_counter() - t0
            out["reference_cpu"] = {"tflops": 2.0 * ref_rows * K * N / t / 1e12,
                                    "cores": rd.info().num_threads,
                                    "sample": f"{ref_rows} rows ({ref_rows}x{K}x{N}), host buffers"}
    return out


def gemv_secondary(lib, dev, st, torch, M, K=4096, N=4096, copies=32, rounds=8):
    """Decode GEMV with bias; rotates `copies` weight sets (> 4x L2) so the
    16 MiB matrix is read from HBM each launch."""
    g = torch.Generator(device="cuda").manual_seed(M)
    Af = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
    A8 = torch.empty((M, K), dtype=torch.int8, device="cuda")
    sa = torch.empty(M, device="cuda")
    bias = torch.empty(N, device="cuda").normal_(0, 0.01, generator=g)
    Cm = torch.empty((M, N), device="cuda")
    torch.cuda.synchronize()
    dev.quantize_i8(Af.data_ptr(), A8.data_ptr(), sa.data_ptr(), M, K, vnpu.QUANT_PER_ROW)
    ws = [make_weights(lib, dev, torch, K, N, seed=100 + i)[0] for i in range(copies)]
    cmds = [cmd_matmul(A8.data_ptr(), w, sa.data_ptr(), bias.data_ptr(), Cm.data_ptr(), M, K, N)
            for w in ws]
    time_loop(lib, dev, st, cmds, 2)
    # One CUDA graph of all copies: kernel time without host launch gaps.
    graph = dev.capture(cmds)
    dev.replay(graph)
    dev.sync()
    e0 = st.event()
    for _ in range(rounds):
        dev.replay(graph)
    e1 = st.event()
    dev.sync()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / rounds / copies
    ms_submit = time_loop(lib, dev, st, cmds, 2) / copies
    lib.b200_graph_destroy(graph)
    for w in ws:
        dev.unpack(w)
    nbytes = K * N + K * M + 4 * M + 4 * N + 4 * N + 4 * M * N
    return {"M": M, "K": K, "N": N, "us": ms * 1e3, "gbs": nbytes / ms / 1e6,
            "us_per_submit_ungraphed": ms_submit * 1e3,
            "bytes_per_launch": nbytes,
            "weight_copies": copies, "kernel": lib.b200_matmul_kernel(M, K, N, 0, A8.data_ptr()).decode()}


def llm_block_secondary(lib, dev, torch, prefill=512, decode=128, with_reference=True):
    """d=4096, 32 heads, I=11008, prefill `prefill` tokens then
    `decode` KV-cached steps (one CUDA graph per step, replayed)."""
    from llm_block import B200Block, BlockConfig, HostBlock, weight_bytes
    cfg = BlockConfig(cap=prefill + decode)
    st = Stream(lib, dev)

    def run(swiglu_epilogue):
        blk = B200Block(cfg, lib, dev, torch, swiglu_epilogue=swiglu_epilogue)
        g = torch.Generator(device="cuda").manual_seed(11)
        x = torch.empty((prefill, cfg.d), device="cuda").normal_(0, 1, generator=g)
        for _ in range(3):                        # warm-up: first passes pay one-off costs
            blk.forward(x, 0)
        dev.sync()
        blk.kc.zero_()
        blk.vc.zero_()
        blk.mask.fill_(float("-inf"))
        e0 = st.event()
        blk.forward(x, 0)
        e1 = st.event()
        dev.sync()
        e1.synchronize()
        ms_prefill = e0.elapsed_time(e1)
        xin = blk._buf("decode_in", (1, cfg.d))
        xin.normal_(0, 1, generator=g)
        blk.pos.fill_(prefill)
        torch.cuda.synchronize()
        blk.capture_decode(xin)
        blk.pos.fill_(prefill)
        torch.cuda.synchronize()
        e0 = st.event()
        for _ in range(decode):
            blk.replay_decode()
        e1 = st.event()
        e1.synchronize()
        ms_decode = e0.elapsed_time(e1)
        blk.close()
        return ms_prefill, ms_decode

    def run_capi():
        """The same block driven inside the library (vnpu_b200_block_*)."""
        from llm_block import make_weights
        w, (n1, n2) = make_weights(cfg)
        c = vnpu.BlockConfigArgs(cfg.d, cfg.heads, cfg.inter, cfg.cap, cfg.eps, cfg.theta, 0, 0)
        blk = vnpu.vp()
        lib.check(lib.b200_block_create(dev.stream, C.byref(c), vnpu.ptr(w["qkv"]),
                                        vnpu.ptr(w["o"]), vnpu.ptr(w["gate_up"]),
                                        vnpu.ptr(w["down"]), vnpu.ptr(n1), vnpu.ptr(n2),
                                        C.byref(blk)), "block_create")
        del w
        g = torch.Generator(device="cuda").manual_seed(11)
        x = torch.empty((prefill, cfg.d), device="cuda").normal_(0, 1, generator=g)
        y = torch.empty_like(x)
        for _ in range(3):
            lib.check(lib.b200_block_forward(blk, x.data_ptr(), prefill, 0, y.data_ptr()), "fwd")
        dev.sync()
        lib.check(lib.b200_block_reset(blk), "reset")
        e0 = st.event()
        lib.check(lib.b200_block_forward(blk, x.data_ptr(), prefill, 0, y.data_ptr()), "fwd")
        e1 = st.event()
        dev.sync()
        e1.synchronize()
        ms_pre = e0.elapsed_time(e1)
        xin = torch.empty((1, cfg.d), device="cuda").normal_(0, 1, generator=g)
        yout = torch.empty_like(xin)
        lib.check(lib.b200_block_decode(blk, xin.data_ptr(), yout.data_ptr()), "decode")
        dev.sync()
        lib.check(lib.b200_block_forward(blk, x.data_ptr(), prefill, 0, y.data_ptr()), "fwd")
        dev.sync()
        e0 = st.event()
        for _ in range(decode):
            lib.check(lib.b200_block_decode(blk, xin.data_ptr(), yout.data_ptr()), "decode")
        e1 = st.event()
        dev.sync()
        e1.synchronize()
        ms_dec = e0.elapsed_time(e1)
        lib.b200_block_destroy(blk)
        return ms_pre, ms_dec

    ms_prefill, ms_decode = run(True)
    pro_prefill, pro_decode = run(False)
    capi_prefill, capi_decode = run_capi()
    out = {"config": f"d={cfg.d} heads={cfg.heads} I={cfg.inter} prefill {prefill} + {decode} decode",
           "prefill_ms": ms_prefill, "prefill_tok_s": prefill / ms_prefill * 1e3,
           "decode_ms_per_token": ms_decode / decode, "decode_tok_s": decode / ms_decode * 1e3,
           "decode_weight_gbs": weight_bytes(cfg) / (ms_decode / decode) / 1e6,
           "decode": "one CUDA graph per token step (vnpu commands + torch layout glue)",
           "gate_up": "MATMUL_I8_SWIGLU (SwiGLU in the gate/up GEMM's epilogue) -> QUANTIZE_I8",
           "swiglu_prologue": {"gate_up": "MATMUL_I8 (2I columns) -> SWIGLU_QUANTIZE_I8",
                               "prefill_ms": pro_prefill,
                               "decode_ms_per_token": pro_decode / decode},
           "library_driver": {"api": "vnpu_b200_block_forward (prefill) / vnpu_b200_block_decode "
                                     "(one CUDA-graph launch per token, position advanced on the "
                                     "device)",
                              "prefill_ms": capi_prefill,
                              "decode_ms_per_token": capi_decode / decode}}
    if with_reference and os.path.exists(REF_LIB):
        import time as _time
        os.environ.setdefault("VNPU_FORCE_ISA", "avx2")
        ref = HostBlock(cfg, lib=vnpu.Lib(REF_LIB), threads=os.cpu_count() or 1)
        xh = np.random.default_rng(11).normal(0, 1, (prefill, cfg.d)).astype(np.float32)
        t0 = _time.perf_counter()
        ref.forward(xh, 0)
        t_pre = _time.perf_counter() - t0
        steps = 8
        t0 = _time.perf_counter()
        for i in range(steps):
            ref.forward(np.random.default_rng(i).normal(0, 1, (1, cfg.d)).astype(np.float32),
                        prefill + i)
        t_dec = (_time.perf_counter() - t0) / steps
        ref.close()
        out["reference_cpu"] = {"prefill_tok_s": prefill / t_pre, "decode_tok_s": 1.0 / t_dec,
                                "cores": os.cpu_count(), "decode_sample_steps": steps,
                                "kind": "reference", "isa": "avx2"}
    return out


def run_b200(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from shard import VNPU_OK, join_group
        if join_group("nccl", rank, world, 300.0, device_id=torch.device("cuda", local)) != VNPU_OK:
            raise SystemExit(f"rank {rank}: not every rank joined within 300 s")
    lib = vnpu.Lib(vnpu.LIB_PATH)
    dev = vnpu.Device(lib, ordinal=local)
    st = Stream(lib, dev)
    pk = peaks()

    M, K = M_TOTAL, K_TOTAL
    n0, n1 = column_shard(N_TOTAL, world, rank)
    w, sb, n, *kept = make_weights(lib, dev, torch, K, N_TOTAL, seed=1, shard=(n0, n1),
                                   keep_int8=world == 1)
    B8_dev = kept[0] if kept else None
    g = torch.Generator(device="cuda").manual_seed(0)
    Af = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
    A8 = torch.empty((M, K), dtype=torch.int8, device="cuda")
    sa = torch.empty(M, device="cuda")
    Cm = torch.empty((M, n), device="cuda")
    # A second int8 A / scale buffer and a second vnpu stream: step i + 1's
    # QUANTIZE_I8 runs on that stream while step i's MATMUL_I8 runs (below).
    A8b = torch.empty((M, K), dtype=torch.int8, device="cuda")
    sab = torch.empty(M, device="cuda")
    torch.cuda.synchronize()
    q = cmd_quantize(Af.data_ptr(), A8.data_ptr(), sa.data_ptr(), M, K)
    mm = cmd_matmul(A8.data_ptr(), w, sa.data_ptr(), None, Cm.data_ptr(), M, K, n)
    qb = cmd_quantize(Af.data_ptr(), A8b.data_ptr(), sab.data_ptr(), M, K)
    mmb = cmd_matmul(A8b.data_ptr(), w, sab.data_ptr(), None, Cm.data_ptr(), M, K, n)
    qstream = vnpu.vp()
    lib.check(lib.stream_create(dev.dev, 0, C.byref(qstream)), "stream_create")
    qcs = torch.cuda.ExternalStream(lib.b200_stream_handle(qstream))
    pq_arr = [(vnpu.Command * 1)(q), (vnpu.Command * 1)(qb)]
    pm_arr = [(vnpu.Command * 1)(mm), (vnpu.Command * 1)(mmb)]
    read_done = [torch.cuda.Event(), torch.cuda.Event()]   # GEMM that last read buffer b
    quant_done = [torch.cuda.Event(), torch.cuda.Event()]

    def pipelined_steps(count):
        """`count` steps; step i quantizes into buffer i % 2 on the second
        stream once the GEMM that last read that buffer is done, and its GEMM
        (library stream) waits for that quantize.  The quantize kernel's CTAs
        do not fit on an SM beside a GEMM CTA, so step i + 1's quantize runs on
        the SMs step i's last, partly empty wave of tiles leaves idle."""
        for i in range(count):
            b = i % 2
            qcs.wait_event(read_done[b])
            if lib.stream_submit(qstream, pq_arr[b], 1, None) != vnpu.OK:
                raise RuntimeError("submit failed")
            quant_done[b].record(qcs)
            st.cs.wait_event(quant_done[b])
            if lib.stream_submit(dev.stream, pm_arr[b], 1, None) != vnpu.OK:
                raise RuntimeError("submit failed")
            read_done[b].record(st.cs)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up, then the timed steps (device-resident inputs)
    for b in range(2):
        read_done[b].record(st.cs)
    pipelined_steps(args.warmup)
    torch.cuda.synchronize()
    barrier()
    launches0 = lib.b200_kernel_launches(dev.dev)
    clocks = ClockSampler(local)
    with clocks:
        e0 = st.event()
        for b in range(2):               # the first quantize starts with the clock
            read_done[b].record(st.cs)
        pipelined_steps(args.steps)
        e1 = st.event()
        rc = dev.sync()
        rcq = lib.stream_sync(qstream)
        e1.synchronize()
        launches = lib.b200_kernel_launches(dev.dev) - launches0
        if rc != vnpu.OK or rcq != vnpu.OK:
            raise RuntimeError(f"stream error {rc} / {rcq}")
        ms_step = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        barrier()
        # ---- the same steps one after the other on one stream (for reference)
        ms_serial = max_over_ranks(time_loop(lib, dev, st, [q, mm], max(3, args.steps)))
        barrier()
        # ---- the GEMM kernel alone (roofline), still under the clock sampler
        ms_gemm = max_over_ranks(time_loop(lib, dev, st, [mm], max(3, args.steps)))
        gemm_kernel = lib.b200_last_matmul_kernel().decode()
    lib.stream_destroy(qstream)
    ops_rank = 2.0 * M * K * n
    int8_peak = 2.0 * pk["bf16"]
    achieved = ops_rank / ms_gemm / 1e9
    traffic = profile_traffic(f"{gemm_kernel}:{M}x{K}x{n}")

    # ---- e2e through the C ABI with host buffers (pinned).  With N > 1 each
    # rank uploads and quantizes only its M/N rows of X (QUANTIZE_I8 is per
    # row, so the codes are those of the whole matrix) and the int8 rows and
    # scales are all-gathered over NVLink (NCCL) before MATMUL_I8: a quarter
    # of the bytes, and no PCIe traffic for the replication.
    rows = M // world
    hA = torch.empty((rows, K), dtype=torch.float32).uniform_(-1, 1).pin_memory()
    hC = torch.empty((M, n), dtype=torch.float32).pin_memory()
    r0 = rank * rows
    qe = cmd_quantize(hA.data_ptr(), A8[r0:r0 + rows].data_ptr(), sa[r0:r0 + rows].data_ptr(),
                      rows, K)
    me = cmd_matmul(A8.data_ptr(), w, sa.data_ptr(), None, hC.data_ptr(), M, K, n)
    e_steps = max(2, min(args.steps, 5))
    q_arr = (vnpu.Command * 1)(qe)
    m_arr = (vnpu.Command * 1)(me)
    qa_parts = [A8[i * rows:(i + 1) * rows] for i in range(world)]
    qs_parts = [sa[i * rows:(i + 1) * rows] for i in range(world)]

    def e2e_step():
        if lib.stream_submit(dev.stream, q_arr, 1, None) != vnpu.OK:
            raise RuntimeError("submit failed")
        if world > 1:
            # NCCL on the library's stream, ordered after the quantize and
            # before the GEMM
            with torch.cuda.stream(st.cs):
                dist.all_gather(qa_parts, qa_parts[rank].clone())
                dist.all_gather(qs_parts, qs_parts[rank].clone())
        if lib.stream_submit(dev.stream, m_arr, 1, None) != vnpu.OK:
            raise RuntimeError("submit failed")

    # Warm-up: the same back-to-back loop as the timed one, so the staging
    # allocations reach their steady-state pool size before the clock starts.
    for _ in range(max(args.warmup, 1)):
        for _ in range(e_steps):
            e2e_step()
        dev.sync()
    barrier()
    # Host-perceived time of e_steps back-to-back steps, each uploading its X
    # rows and downloading its C (downloads run on the stream's copy-engine
    # stream, so the clock stops at vnpu_stream_sync).
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    if dev.sync() != vnpu.OK:
        raise RuntimeError("stream error")
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks((time.perf_counter() - t0) * 1e3 / e_steps)

    # ---- all-gather of the shards over NCCL (config 5's collective)
    allgather = None
    if world > 1:
        # shard-major [P][M][width]: width = the widest shard (all shards are
        # equal when N / P is a multiple of 256, as here: no padding)
        width = max(b - a for a, b in (column_shard(N_TOTAL, world, r) for r in range(world)))
        shard_pad = torch.zeros((M, width), device="cuda")
        shard_pad[:, :n] = Cm
        gathered = torch.empty((world, M, width), device="cuda")
        dist.all_gather_into_tensor(gathered, shard_pad)
        torch.cuda.synchronize()
        barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        reps = 3
        for _ in range(reps):
            dist.all_gather_into_tensor(gathered, shard_pad)
        a1.record()
        torch.cuda.synchronize()
        ms_ag = max_over_ranks(a0.elapsed_time(a1) / reps)
        recv = (world - 1) * M * width * 4
        allgather = {"ms": ms_ag, "bytes_received_per_rank": recv,
                     "gbs_per_rank": recv / ms_ag / 1e6, "layout": "shard-major [P][M][N/P]",
                     "ms_step_plus_gather": ms_step + ms_ag}
        # ---- the same gather fused into the GEMM: MATMUL_I8_SCATTER writes the
        # rank's shard into every rank's full [M][N] output (CUDA IPC, NVLink
        # stores from the epilogue); a one-element NCCL all-reduce is the
        # barrier after which every full output is complete.
        buf = vnpu.vp()
        lib.check(lib.buffer_alloc(dev.dev, M * N_TOTAL * 4, vnpu.C.byref(buf)), "buffer_alloc")
        full = lib.buffer_host_ptr(buf)
        handles = [None] * world
        dist.all_gather_object(handles, dev.ipc_handle(full))
        peers = [full if r == rank else dev.ipc_open(handles[r], local) for r in range(world)]
        flag = torch.zeros(1, device="cuda")
        sc_args = vnpu.MatmulI8ScatterArgs(
            A8.data_ptr(), w, sa.data_ptr(), None,
            (vnpu.vp * vnpu.B200_SCATTER_MAX)(*(peers + [None] * (vnpu.B200_SCATTER_MAX - world))),
            M, K, n, 0, N_TOTAL, n0, world, 0)
        sc_arr = (vnpu.Command * 1)(vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_SCATTER, sc_args))

        def fused_step():
            if lib.stream_submit(dev.stream, sc_arr, 1, None) != vnpu.OK:
                raise RuntimeError("submit failed")
            with torch.cuda.stream(st.cs):
                dist.all_reduce(flag)

        for _ in range(max(args.warmup, 1)):
            fused_step()
        dev.sync()
        torch.cuda.synchronize()
        # the fused result equals the NCCL-gathered one (shard-major -> row-major),
        # both from the activations now in A8
        lib.check(dev.submit([cmd_matmul(A8.data_ptr(), w, sa.data_ptr(), None, Cm.data_ptr(),
                                         M, K, n)]), "submit")
        lib.check(dev.sync(), "matmul")
        shard_pad[:, :n] = Cm
        gathered = torch.empty((world, M, width), device="cuda")
        dist.all_gather_into_tensor(gathered, shard_pad)
        full_t = torch.empty((M, N_TOTAL), device="cuda")
        lib.check(dev.submit([_copy_cmd(full_t.data_ptr(), full, M * N_TOTAL * 4)]), "copy")
        lib.check(dev.sync(), "copy")
        torch.cuda.synchronize()
        same = True
        for r in range(world):
            r0_, r1_ = column_shard(N_TOTAL, world, r)
            same &= bool(torch.equal(full_t[:, r0_:r1_], gathered[r, :, :r1_ - r0_]))
        del gathered, full_t
        barrier()
        f0 = st.event()
        for _ in range(reps):
            fused_step()
        f1 = st.event()
        dev.sync()
        f1.synchronize()
        ms_fused = max_over_ranks(f0.elapsed_time(f1) / reps)
        allgather["fused"] = {
            "ms_gemm_plus_gather": ms_fused, "ms_separate": ms_gemm + ms_ag,
            "tops_whole_job": 2.0 * M * K * N_TOTAL / ms_fused / 1e9,
            "bound": ("NVLink: every rank receives (P-1)/P of the f32 output, "
                      f"{(world - 1) * M * N_TOTAL * 4 / world / 1e6:.0f} MB, "
                      f"{(world - 1) * M * N_TOTAL * 4 / world / 770e9 * 1e3:.3f} ms at the measured "
                      "770 GB/s per direction, against the GEMM's "
                      f"{ms_gemm:.3f} ms"),
            "speedup_vs_separate": (ms_gemm + ms_ag) / ms_fused, "bit_identical_to_nccl": same,
            "path": "VNPU_B200_OP_MATMUL_I8_SCATTER into every rank's full output over CUDA IPC, "
                    "then a one-element NCCL all-reduce as the barrier"}
        barrier()
        for r in range(world):
            if r != rank:
                lib.b200_ipc_close(peers[r])
        barrier()
        lib.buffer_free(buf)
        del shard_pad

    out = None
    if rank == 0:
        secondary = {}
        cpu = None
        if world == 1 and not args.no_secondary:
            secondary["gemm_8192_cube"] = gemm_secondary(lib, dev, st, torch, 8192, 8192, 8192, 0, False)
            secondary["ffn_4096x4096x14336_silu"] = gemm_secondary(lib, dev, st, torch, 4096, 4096,
                                                                   14336, 2, False)
            secondary["gemm_512_cube"] = gemm_secondary(lib, dev, st, torch, 512, 512, 512, 0, False,
                                                        iters=200)
            secondary["gemm_1024_cube"] = gemm_secondary(lib, dev, st, torch, 1024, 1024, 1024, 0,
                                                         False, iters=200)
            secondary["gemm_512x4096x4096"] = gemm_secondary(lib, dev, st, torch, 512, 4096, 4096,
                                                             0, False, iters=100)
            for m in (1, 4, 8):
                gv = gemv_secondary(lib, dev, st, torch, m)
                gv["frac_of_hbm"] = gv["gbs"] / pk["hbm_gbs"]
                secondary[f"gemv_m{m}"] = gv
            secondary["matmul_f32_4096_cube"] = f32_secondary(lib, dev, st, torch, 4096, 4096,
                                                              4096)
            if not args.no_block:
                secondary["llm_block"] = llm_block_secondary(
                    lib, dev, torch, with_reference=not args.no_cpu_baseline)
            try:
                A_ = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda")
                B_ = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda").t()
                torch._int_mm(A_, B_)
                torch.cuda.synchronize()
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                c0.record()
                for _ in range(10):
                    torch._int_mm(A_, B_)
                c1.record()
                torch.cuda.synchronize()
                secondary["cublas_int8_8192_cube_tops"] = 2.0 * 8192 ** 3 / (c0.elapsed_time(c1) / 10) / 1e9
                del A_, B_
            except Exception as exc:  # library comparator only
                secondary["cublas_int8_8192_cube_tops"] = f"unavailable: {exc}"
        if world == 1 and not args.no_cpu_baseline:
            # The CPU implementation on the first rows of the very inputs the
            # timed steps used (A f32, the int8 weights and scales): its rows
            # must be the GPU's C bit for bit.
            rows = int(os.environ.get("VNPU_BENCH_REF_ROWS", "32"))
            r = reference_sample(rows, 3, 1, os.cpu_count() or 1, A=Af[:rows].cpu().numpy(),
                                 B8=B8_dev.cpu().numpy(), sb=sb.cpu().numpy())
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "quantize_i8",
                                     "matmul_i8")}
            gpu_rows = Cm[:rows].cpu().numpy()
            cpu["check"] = {"rows": rows, "bit_exact_vs_gpu_C": bool(np.array_equal(
                gpu_rows.view(np.uint32), r["C"].view(np.uint32)))}
        total_ops = 2.0 * M * K * N_TOTAL
        out = {
            "metric": METRIC, "value": total_ops / ms_step / 1e9, "unit": "TOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N_TOTAL, "n_per_gpu": n,
                       "epilogue": "none", "bias": False, "parallelism": f"column shard x{world}",
                       "l2": "inputs larger than L2 (A f32 256 MiB, B int8 224 MiB/P, C f32 896 MiB/P)",
                       "step": "QUANTIZE_I8(A) + MATMUL_I8; step i+1's QUANTIZE_I8 runs on a second "
                               "vnpu stream beside step i's MATMUL_I8 (two int8 A buffers, CUDA "
                               "events order each quantize after the GEMM that last read its buffer)",
                       "ms_per_step_serial": ms_serial},
            "roofline": {"bound": "tensor",
                         "kernel": gemm_kernel,
                         "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                         "frac": achieved / int8_peak, "traffic": traffic,
                         "peak_source": f"2 x {pk['source']} bf16 dense ({pk['bf16']} TFLOP/s); "
                                        f"nominal int8 dense 4500 TOPS",
                         "frac_of_nominal": achieved / 4500.0, "ms_per_launch": ms_gemm,
                         "work": "2*M*K*N/P int8 ops per launch"},
            "e2e": {"value": total_ops / ms_e2e / 1e9, "unit": "TOPS",
                    "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": M * N_TOTAL * 4,
                    "ms_per_step": ms_e2e,
                    "path": ("vnpu_stream_submit(QUANTIZE_I8, MATMUL_I8), host X and C"
                             if world == 1 else
                             "per rank: vnpu_stream_submit(QUANTIZE_I8) of its M/N host rows of X, "
                             "NCCL all-gather of the int8 rows and scales, "
                             "vnpu_stream_submit(MATMUL_I8) into its host C shard; "
                             "bytes are totals over the ranks")},
            "gpu_launches": int(launches),
            "clocks": clocks.report(),
            "cpu_baseline": cpu,
            "secondary": secondary,
        }
        if allgather:
            out["allgather"] = allgather
    dev.unpack(w)
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)
    return 0


def run_kernel_case(spec: str):
    """One small case of one kernel, launched twice (for ncu captures):
    gemm:MxKxN[:silu], gemv:MxKxN, f32:MxKxN[:nt], quantize:RxC, attention:HxSQxSKxD,
    llm_lib:STEPS (the block inside the library: prefill 512, STEPS decode tokens),
    llm_prefill:T (the decoder block's prefill of T tokens, twice) or llm_decode:STEPS (the
    decoder block's graph-captured decode step)."""
    import torch

    lib = vnpu.Lib(vnpu.LIB_PATH)
    dev = vnpu.Device(lib, ordinal=0)
    kind, dims = spec.split(":", 1)
    parts = dims.split(":")
    shape = [int(x) for x in parts[0].split("x")]
    g = torch.Generator(device="cuda").manual_seed(0)
    if kind in ("gemm", "gemv"):
        M, K, N = shape
        epi = 2 if len(parts) > 1 and parts[1] == "silu" else 0
        Af = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
        A8 = torch.empty((M, K), dtype=torch.int8, device="cuda")
        sa = torch.empty(M, device="cuda")
        Cm = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        dev.quantize_i8(Af.data_ptr(), A8.data_ptr(), sa.data_ptr(), M, K, vnpu.QUANT_PER_ROW)
        w, sb, n = make_weights(lib, dev, torch, K, N, seed=3)
        for _ in range(2):
            dev.matmul_i8(A8.data_ptr(), w, sa.data_ptr(), None, Cm.data_ptr(), M, K, N,
                          epilogue=epi)
        dev.unpack(w)
    elif kind == "f32":
        M, K, N = shape
        trans_b = 1 if len(parts) > 1 and parts[1] == "nt" else 0
        A = torch.empty((M, K), device="cuda").uniform_(-1, 1, generator=g)
        B = torch.empty((N, K) if trans_b else (K, N), device="cuda").uniform_(-1, 1, generator=g)
        Cm = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        for _ in range(2):
            dev.matmul_f32(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, K, N, trans_b=trans_b)
    elif kind == "quantize":
        R, Cc = shape
        X = torch.empty((R, Cc), device="cuda").uniform_(-1, 1, generator=g)
        Y = torch.empty((R, Cc), dtype=torch.int8, device="cuda")
        s = torch.empty(R, device="cuda")
        torch.cuda.synchronize()
        for _ in range(2):
            dev.quantize_i8(X.data_ptr(), Y.data_ptr(), s.data_ptr(), R, Cc, vnpu.QUANT_PER_ROW)
    elif kind == "attention":
        H, SQ, SK, D = shape
        Q = torch.randn((1, H, SQ, D), device="cuda", generator=g)
        Kt = torch.randn((1, H, SK, D), device="cuda", generator=g)
        V = torch.randn((1, H, SK, D), device="cuda", generator=g)
        O = torch.empty((1, H, SQ, D), device="cuda")
        torch.cuda.synchronize()
        for _ in range(2):
            dev.attention(Q.data_ptr(), Kt.data_ptr(), V.data_ptr(), None, O.data_ptr(), 1, H,
                          SQ, SK, D, 1, 0.0)
    elif kind == "llm_prefill":
        # configs[3] decoder block: prefill T tokens twice (positions 0 and T).
        from llm_block import B200Block, BlockConfig
        T = shape[0]
        cfg = BlockConfig(cap=2 * T)
        blk = B200Block(cfg, lib, dev, torch)
        x = torch.empty((T, cfg.d), device="cuda").normal_(0, 1, generator=g)
        torch.cuda.synchronize()
        blk.forward(x, 0)
        blk.forward(x, T)
        dev.sync()
        blk.close()
    elif kind == "llm_decode":
        # configs[3] decoder block: prefill 512 tokens, capture one decode step
        # as a CUDA graph, replay it `steps` times.
        from llm_block import B200Block, BlockConfig
        steps = shape[0]
        cfg = BlockConfig(cap=640)
        blk = B200Block(cfg, lib, dev, torch)
        x = torch.empty((512, cfg.d), device="cuda").normal_(0, 1, generator=g)
        blk.forward(x, 0)
        dev.sync()
        xin = blk._buf("decode_in", (1, cfg.d))
        xin.normal_(0, 1, generator=g)
        blk.pos.fill_(512)
        torch.cuda.synchronize()
        blk.capture_decode(xin)
        blk.pos.fill_(512)
        torch.cuda.synchronize()
        for _ in range(steps):
            blk.replay_decode()
        torch.cuda.synchronize()
        blk.close()
    elif kind == "llm_lib":
        # the same block driven inside the library (vnpu_b200_block_*): prefill
        # 512 tokens, then `steps` decode tokens (one graph launch each)
        from llm_block import BlockConfig, make_weights
        steps = shape[0]
        cfg = BlockConfig(cap=640)
        w, (n1, n2) = make_weights(cfg)
        c = vnpu.BlockConfigArgs(cfg.d, cfg.heads, cfg.inter, cfg.cap, cfg.eps, cfg.theta, 0, 0)
        blk = vnpu.vp()
        lib.check(lib.b200_block_create(dev.stream, C.byref(c), vnpu.ptr(w["qkv"]),
                                        vnpu.ptr(w["o"]), vnpu.ptr(w["gate_up"]),
                                        vnpu.ptr(w["down"]), vnpu.ptr(n1), vnpu.ptr(n2),
                                        C.byref(blk)), "block_create")
        del w
        x = torch.empty((512, cfg.d), device="cuda").normal_(0, 1, generator=g)
        y = torch.empty_like(x)
        lib.check(lib.b200_block_forward(blk, x.data_ptr(), 512, 0, y.data_ptr()), "forward")
        xin = torch.empty((1, cfg.d), device="cuda").normal_(0, 1, generator=g)
        yout = torch.empty_like(xin)
        for _ in range(steps):
            lib.check(lib.b200_block_decode(blk, xin.data_ptr(), yout.data_ptr()), "decode")
        dev.sync()
        lib.b200_block_destroy(blk)
    else:
        raise SystemExit(f"unknown kernel case {spec}")
    rc = dev.sync()
    dev.close()
    print(f"kernel case {spec}: rc={rc}")
    return 0 if rc == vnpu.OK else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-block", action="store_true", help="skip the decoder-block secondary")
    ap.add_argument("--kernel-case", default=None,
                    help="run one small kernel case twice and exit (ncu captures)")
    args = ap.parse_args()
    if args.kernel_case:
        return run_kernel_case(args.kernel_case)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
