"""ctypes binding of the vnpu v1 C ABI.

The same binding drives both libraries that export this ABI:

* ``libvnpu.so`` built from ``csrc/`` - the B200 backend (device memory,
  CUDA streams, sm_100a kernels);
* the reference library built from its own sources into ``oracle/_ref`` -
  used only by tests and by ``bench.py``'s reference arm.

The struct layouts follow the reference header ``include/vnpu.h:186-468``
field for field; ``include/vnpu.h`` in this repository is the C statement of
the same ABI.  Pointer arguments are plain integers: a numpy array's
``ctypes.data`` (host memory) or a device address (``torch.Tensor.data_ptr()``).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libvnpu.so")

# Status codes (include/vnpu.h:103-118)
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_OUT_OF_MEMORY = -2
ERR_UNSUPPORTED = -3
ERR_INVALID_COMMAND = -4
ERR_DEVICE_BUSY = -5
ERR_DEVICE_ERROR = -6
ERR_TIMEOUT = -7
ERR_INTERNAL = -100

# Opcodes (include/vnpu.h:165-184)
OP_NOP, OP_MATMUL_F32, OP_MATMUL_I8, OP_RMSNORM_F32, OP_SOFTMAX_F32 = 0, 1, 2, 3, 4
OP_ROPE_F32, OP_SWIGLU_F32, OP_GELU_F32, OP_ADD_F32, OP_MUL_F32 = 5, 6, 7, 8, 9
OP_ATTENTION_F32, OP_QUANTIZE_I8, OP_PACK_WEIGHTS_I8, OP_MTP_HEAD_F32 = 10, 11, 12, 13
OP_COPY, OP_MEMSET, OP_BARRIER = 14, 15, 16

UNIT_AUTO, UNIT_VOODOO, UNIT_WILDCAT, UNIT_CELL, UNIT_GPU = 0, 1, 2, 3, 16
EPI_NONE, EPI_RELU, EPI_SILU, EPI_GELU_TANH, EPI_GELU_ERF = 0, 1, 2, 3, 4
QUANT_PER_ROW, QUANT_PER_COLUMN, QUANT_PER_TENSOR = 0, 1, 2
COPY_H2H, COPY_H2D, COPY_D2H, COPY_D2D = 0, 1, 2, 3

FEATURE_GPU_FUTURE = 1 << 31

# B200 extensions (include/vnpu_b200.h)
CMD_FLAG_EPI_STREAM = 1 << 8
CMD_FLAG_EPI_SCALAR = 1 << 9
CMD_FLAG_ATTN_TOKEN_MAJOR = 1 << 10   # ATTENTION_F32 writes O as [batch][seq_q][heads][D]
CMD_FLAG_EPI_BLOCK = 1 << 11
# oracle form index (oracle/oracle.h) -> command flags of the B200 library
FORM_FLAGS = {0: CMD_FLAG_EPI_BLOCK, 1: CMD_FLAG_EPI_SCALAR, 2: CMD_FLAG_EPI_STREAM}

vp = C.c_void_p
u32 = C.c_uint32
u64 = C.c_uint64
f32 = C.c_float


class Config(C.Structure):
    _fields_ = [("abi_version", u32), ("num_threads", u32), ("num_compute_units", u32),
                ("tile_m", u32), ("tile_k", u32), ("tile_n", u32), ("flags", u32),
                ("reserved0", u32), ("trace_file", C.c_char_p), ("node_name", C.c_char_p)]


class DeviceInfo(C.Structure):
    _fields_ = [("abi_version", u32), ("name", C.c_char * 64), ("vendor", C.c_char * 64),
                ("cpu_arch", C.c_char * 32), ("backend", C.c_char * 64), ("simd_bits", u32),
                ("num_threads", u32), ("num_compute_units", u32), ("local_store_bytes", u32),
                ("tile_m", u32), ("tile_k", u32), ("tile_n", u32), ("physical_cores", u32),
                ("features", u64), ("l1d_bytes", u64), ("l2_bytes", u64), ("l3_bytes", u64),
                ("total_memory_bytes", u64)]


class DeviceStatus(C.Structure):
    _fields_ = [(n, u64) for n in ("commands_submitted", "commands_completed", "kernel_time_ns",
                                   "dispatch_time_ns", "memory_time_ns", "sync_time_ns",
                                   "bytes_read", "bytes_written", "flops", "tiles_dispatched",
                                   "tiles_culled", "dma_bytes", "interrupts")] + \
              [("busy", u32), ("error", u32), ("last_opcode", u32), ("active_workers", u32),
               ("reserved", u64 * 4)]


class TraceSummary(C.Structure):
    _fields_ = [(n, u64) for n in ("events", "total_time_ns", "dispatch_time_ns", "memory_time_ns",
                                   "compute_time_ns", "sync_time_ns", "bytes_read",
                                   "bytes_written", "flops")] + \
              [("achieved_gflops", C.c_double), ("achieved_gbytes_s", C.c_double),
               ("hot_opcode", u32), ("hot_time_ns", u64), ("trace_overhead_ns", C.c_double)]


class ReferenceModel(C.Structure):
    """vnpu_b200_reference_model_t (include/vnpu_b200.h)."""
    _fields_ = [("num_threads", u32), ("tile_m", u32), ("tile_k", u32), ("tile_n", u32),
                ("pack_b", u32), ("scalar_isa", u32), ("l2_bytes", u64),
                ("epilogue_forced", u32), ("epilogue_form", u32)]


class BlockConfigArgs(C.Structure):
    """vnpu_b200_block_config_t (include/vnpu_b200.h)."""
    _fields_ = [("d_model", u32), ("heads", u32), ("inter", u32), ("capacity", u32),
                ("eps", C.c_float), ("theta_base", C.c_float), ("flags", u32), ("reserved0", u32)]


B200_BLOCK_SWIGLU_PROLOGUE = 1 << 0


class ClusterConfig(C.Structure):
    _fields_ = [("abi_version", u32), ("num_streams", u32), ("flags", u32),
                ("request_timeout_ms", u32), ("auth_token", C.c_char_p),
                ("cluster_name", C.c_char_p)]


class ClusterStats(C.Structure):
    _fields_ = [(n, u64) for n in ("local_jobs", "remote_jobs", "total_jobs",
                                   "network_bytes_sent", "network_bytes_received", "failed_jobs",
                                   "culled_tiles")] + \
              [("local_time_ns", C.c_double), ("remote_time_ns", C.c_double),
               ("speedup_estimate", C.c_double)]


class MatmulF32Args(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("bias", vp), ("C", vp), ("M", u32), ("K", u32), ("N", u32),
                ("lda", u32), ("ldb", u32), ("ldc", u32), ("trans_a", u32), ("trans_b", u32),
                ("alpha", f32), ("beta", f32), ("epilogue", u32), ("unit", u32),
                ("reserved0", u32), ("tile_mask", vp), ("mask_tile_m", u32), ("mask_tile_n", u32)]


class MatmulI8Args(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp), ("C", vp),
                ("M", u32), ("K", u32), ("N", u32), ("lda", u32), ("ldc", u32),
                ("epilogue", u32), ("unit", u32)]


class RmsnormArgs(C.Structure):
    _fields_ = [("X", vp), ("W", vp), ("Y", vp), ("rows", u32), ("cols", u32), ("eps", f32),
                ("unit", u32)]


class SoftmaxArgs(C.Structure):
    _fields_ = [("X", vp), ("Y", vp), ("rows", u32), ("cols", u32), ("temperature", f32),
                ("unit", u32)]


class RopeArgs(C.Structure):
    _fields_ = [("Q", vp), ("K", vp), ("positions", vp), ("batch", u32), ("heads", u32),
                ("q_seq", u32), ("k_seq", u32), ("head_dim", u32), ("position_offset", u32),
                ("interleaved", u32), ("theta_base", f32), ("scaling", f32)]


class BinaryArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("Y", vp), ("count", u64), ("alpha", f32), ("beta", f32),
                ("unit", u32), ("reserved0", u32)]


class UnaryArgs(C.Structure):
    _fields_ = [("X", vp), ("Y", vp), ("count", u64), ("param", f32), ("unit", u32),
                ("reserved0", u32)]


class SwigluArgs(C.Structure):
    _fields_ = [("gate", vp), ("up", vp), ("Y", vp), ("count", u64), ("alpha", f32),
                ("unit", u32), ("reserved0", u32)]


class AttentionArgs(C.Structure):
    _fields_ = [("Q", vp), ("K", vp), ("V", vp), ("mask", vp), ("O", vp), ("workspace", vp),
                ("workspace_bytes", u64), ("batch", u32), ("heads", u32), ("seq_q", u32),
                ("seq_k", u32), ("head_dim", u32), ("causal", u32), ("scale", f32),
                ("unit", u32)]


class QuantizeI8Args(C.Structure):
    _fields_ = [("X", vp), ("Y", vp), ("scales", vp), ("rows", u64), ("cols", u64),
                ("axis", u32), ("unit", u32)]


class PackWeightsI8Args(C.Structure):
    _fields_ = [("B", vp), ("scales", vp), ("out", vp), ("K", u32), ("N", u32), ("ldb", u32),
                ("trans_b", u32), ("unit", u32), ("reserved0", u32)]


class MtpHeadArgs(C.Structure):
    _fields_ = [("hidden", vp), ("W", vp), ("bias", vp), ("logits", vp), ("gamma", u32),
                ("hidden_dim", u32), ("vocab", u32), ("trans_w", u32), ("unit", u32),
                ("reserved0", u32)]


# B200 extensions (include/vnpu_b200.h): fused row prologues, args in Command.args.raw
OP_B200_RMSNORM_QUANTIZE_I8 = 0x100
OP_B200_SWIGLU_QUANTIZE_I8 = 0x101


class RmsnormQuantizeArgs(C.Structure):
    _fields_ = [("X", vp), ("W", vp), ("Y", vp), ("Q", vp), ("scales", vp), ("rows", u32),
                ("cols", u32), ("eps", C.c_float), ("reserved0", u32)]


class SwigluQuantizeArgs(C.Structure):
    _fields_ = [("gate", vp), ("up", vp), ("Y", vp), ("Q", vp), ("scales", vp), ("rows", u32),
                ("cols", u32), ("alpha", C.c_float), ("ld", u32)]


OP_B200_KV_APPEND = 0x102


class KvAppendArgs(C.Structure):
    _fields_ = [("K", vp), ("V", vp), ("K_cache", vp), ("V_cache", vp), ("mask", vp),
                ("position", vp), ("heads", u32), ("T", u32), ("head_dim", u32),
                ("capacity", u32), ("position_offset", u32), ("reserved0", u32)]


OP_B200_MATMUL_I8_SCATTER = 0x103
B200_SCATTER_MAX = 8


class MatmulI8ScatterArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp),
                ("dst", vp * B200_SCATTER_MAX), ("M", u32), ("K", u32), ("N", u32), ("lda", u32),
                ("ldd", u32), ("col_offset", u32), ("ndst", u32), ("epilogue", u32)]


OP_B200_QKV_ROPE_APPEND = 0x104


class QkvRopeAppendArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp), ("Q", vp), ("K_out", vp),
                ("V_out", vp), ("K_cache", vp), ("V_cache", vp), ("mask", vp), ("position", vp),
                ("T", u32), ("K", u32), ("heads", u32), ("head_dim", u32), ("capacity", u32),
                ("position_offset", u32), ("theta_base", C.c_float), ("scaling", C.c_float),
                ("epilogue", u32), ("reserved0", u32)]


OP_B200_MATMUL_I8_RESIDUAL = 0x105


class MatmulI8ResidualArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp), ("R", vp), ("C", vp),
                ("M", u32), ("K", u32), ("N", u32), ("lda", u32), ("ldr", u32), ("ldc", u32),
                ("epilogue", u32), ("reserved0", u32)]


# MATMUL_I8_RESIDUAL that also advances a device int32 position: the fields
# sit at byte ADVANCE_OFFSET of the command's argument bytes.
CMD_FLAG_ADVANCE_POSITION = 1 << 14
ADVANCE_OFFSET = 128


class AdvanceArgs(C.Structure):
    _fields_ = [("position", vp), ("advance", C.c_int32), ("reserved", u32)]


def with_advance_position(cmd: "Command", position, advance: int) -> "Command":
    """Ask a MATMUL_I8_RESIDUAL command to add `advance` to the device int32
    at `position` once the stream's earlier commands are complete."""
    cmd.flags |= CMD_FLAG_ADVANCE_POSITION
    o = AdvanceArgs(ptr(position), advance, 0)
    C.memmove(C.addressof(cmd.args) + ADVANCE_OFFSET, C.addressof(o), C.sizeof(o))
    return cmd


OP_B200_MATMUL_I8_SHARD = 0x106


class MatmulI8ShardArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp), ("C", vp),
                ("M", u32), ("K", u32), ("N", u32), ("lda", u32), ("ldc", u32),
                ("epilogue", u32), ("n_full", u32), ("col_base", u32)]


OP_B200_MATMUL_I8_SWIGLU = 0x108


class MatmulI8SwigluArgs(C.Structure):
    _fields_ = [("A", vp), ("B", vp), ("scale_a", vp), ("bias", vp), ("Y", vp),
                ("M", u32), ("K", u32), ("N", u32), ("lda", u32), ("ldy", u32), ("epilogue", u32),
                ("alpha", C.c_float), ("reserved0", u32)]


def b200_command(opcode: int, args: C.Structure) -> "Command":
    """A command whose arguments are a B200 extension struct (copied into args.raw)."""
    c = Command()
    c.opcode = opcode
    C.memmove(C.addressof(c.args), C.addressof(args), C.sizeof(args))
    return c


class CopyArgs(C.Structure):
    _fields_ = [("dst", vp), ("src", vp), ("bytes", u64), ("direction", u32), ("reserved0", u32)]


class MemsetArgs(C.Structure):
    _fields_ = [("dst", vp), ("bytes", u64), ("value", u32), ("reserved0", u32)]


class CommandArgs(C.Union):
    _fields_ = [("matmul_f32", MatmulF32Args), ("matmul_i8", MatmulI8Args),
                ("rmsnorm", RmsnormArgs), ("softmax", SoftmaxArgs), ("rope", RopeArgs),
                ("binary", BinaryArgs), ("unary", UnaryArgs), ("swiglu", SwigluArgs),
                ("attention", AttentionArgs), ("quantize_i8", QuantizeI8Args),
                ("pack_weights_i8", PackWeightsI8Args), ("mtp_head", MtpHeadArgs),
                ("copy", CopyArgs), ("memset", MemsetArgs), ("raw", C.c_uint8 * 192)]


class Command(C.Structure):
    _fields_ = [("opcode", u32), ("flags", u32), ("id", u64), ("args", CommandArgs)]


assert C.sizeof(Command) == 208, C.sizeof(Command)

_ST = C.c_int  # vnpu_status_t


def _sig(lib, name, res, *args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


class VnpuError(RuntimeError):
    def __init__(self, what: str, status: int):
        super().__init__(f"{what}: status {status}")
        self.status = status


def ptr(x) -> Optional[int]:
    """Address of a numpy array / torch tensor / int (None stays None)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    raise TypeError(type(x))


class Lib:
    """One loaded vnpu ABI library (the B200 backend or the reference)."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (run __graft_entry__.build())")
        self.path = path
        self.h = C.CDLL(path)
        h = self.h
        self.config_init = _sig(h, "vnpu_config_init", None, C.POINTER(Config))
        self.status_string = _sig(h, "vnpu_status_string", C.c_char_p, _ST)
        self.version_string = _sig(h, "vnpu_version_string", C.c_char_p)
        self.device_create = _sig(h, "vnpu_device_create", _ST, C.POINTER(Config), C.POINTER(vp))
        self.device_destroy = _sig(h, "vnpu_device_destroy", None, vp)
        self.device_get_info = _sig(h, "vnpu_device_get_info", _ST, vp, C.POINTER(DeviceInfo))
        self.device_get_status = _sig(h, "vnpu_device_get_status", _ST, vp, C.POINTER(DeviceStatus))
        self.stream_create = _sig(h, "vnpu_stream_create", _ST, vp, C.c_int, C.POINTER(vp))
        self.stream_destroy = _sig(h, "vnpu_stream_destroy", None, vp)
        self.stream_sync = _sig(h, "vnpu_stream_sync", _ST, vp)
        self.stream_submit = _sig(h, "vnpu_stream_submit", _ST, vp, C.POINTER(Command), u64, vp)
        self.event_create = _sig(h, "vnpu_event_create", _ST, C.POINTER(vp))
        self.event_destroy = _sig(h, "vnpu_event_destroy", None, vp)
        self.event_wait = _sig(h, "vnpu_event_wait", _ST, vp, u32)
        self.event_query = _sig(h, "vnpu_event_query", _ST, vp)
        self.buffer_alloc = _sig(h, "vnpu_buffer_alloc", _ST, vp, u64, C.POINTER(vp))
        self.buffer_free = _sig(h, "vnpu_buffer_free", None, vp)
        self.buffer_host_ptr = _sig(h, "vnpu_buffer_host_ptr", vp, vp)
        self.buffer_size = _sig(h, "vnpu_buffer_size", u64, vp)
        self.buffer_copy = _sig(h, "vnpu_buffer_copy", _ST, vp, vp, vp, u64, u32)
        self.buffer_memset = _sig(h, "vnpu_buffer_memset", _ST, vp, vp, u32, u64)
        self.pack_weights_i8 = _sig(h, "vnpu_pack_weights_i8", _ST, vp, vp, vp, u32, u32, u32,
                                    u32, C.POINTER(vp))
        self.packed_weights_destroy = _sig(h, "vnpu_packed_weights_destroy", None, vp)
        self.packed_weights_info = _sig(h, "vnpu_packed_weights_info", _ST, vp, C.POINTER(u32),
                                        C.POINTER(u32), C.POINTER(u64), C.POINTER(vp),
                                        C.POINTER(vp))
        self.matmul_i8 = _sig(h, "vnpu_matmul_i8", _ST, vp, C.POINTER(MatmulI8Args))
        self.matmul_f32 = _sig(h, "vnpu_matmul_f32", _ST, vp, C.POINTER(MatmulF32Args))
        self.quantize_i8 = _sig(h, "vnpu_quantize_i8", _ST, vp, C.POINTER(QuantizeI8Args))
        self.rmsnorm_f32 = _sig(h, "vnpu_rmsnorm_f32", _ST, vp, C.POINTER(RmsnormArgs))
        self.rope_f32 = _sig(h, "vnpu_rope_f32", _ST, vp, C.POINTER(RopeArgs))
        self.swiglu_f32 = _sig(h, "vnpu_swiglu_f32", _ST, vp, C.POINTER(SwigluArgs))
        self.add_f32 = _sig(h, "vnpu_add_f32", _ST, vp, C.POINTER(BinaryArgs))
        self.attention_f32 = _sig(h, "vnpu_attention_f32", _ST, vp, C.POINTER(AttentionArgs))
        self.get_backend_v1 = _sig(h, "vnpu_get_backend_v1", vp)
        self.cluster_config_init = _sig(h, "vnpu_cluster_config_init", None,
                                        C.POINTER(ClusterConfig))
        self.cluster_create = _sig(h, "vnpu_cluster_create", _ST, C.POINTER(ClusterConfig),
                                   C.POINTER(vp))
        self.cluster_destroy = _sig(h, "vnpu_cluster_destroy", None, vp)
        self.cluster_add_device = _sig(h, "vnpu_cluster_add_device", _ST, vp, vp, u32)
        self.cluster_add_remote = _sig(h, "vnpu_cluster_add_remote", _ST, vp, vp, C.POINTER(vp))
        self.cluster_get_stats = _sig(h, "vnpu_cluster_get_stats", _ST, vp,
                                      C.POINTER(ClusterStats))
        self.cluster_cache_weights_f32 = _sig(h, "vnpu_cluster_cache_weights_f32", _ST, vp,
                                              C.c_char_p, vp, u32, u32, u32, C.POINTER(vp))
        self.cluster_matmul_f32 = _sig(h, "vnpu_cluster_matmul_f32", _ST, vp, vp, vp, vp, u32,
                                       u32, u32, u32)
        if hasattr(h, "vnpu_cluster_matmul_i8"):
            self.cluster_cache_weights_i8 = _sig(h, "vnpu_cluster_cache_weights_i8", _ST, vp,
                                                 C.c_char_p, vp, vp, u32, u32, u32,
                                                 C.POINTER(vp))
            self.cluster_matmul_i8 = _sig(h, "vnpu_cluster_matmul_i8", _ST, vp, vp, vp, vp, vp,
                                          vp, u32, u32, u32, u32, u32)
        self.is_b200 = hasattr(h, "vnpu_b200_stream_handle")
        if self.is_b200:
            self.b200_stream_handle = _sig(h, "vnpu_b200_stream_handle", vp, vp)
            self.b200_kernel_launches = _sig(h, "vnpu_b200_kernel_launches", u64, vp)
            self.b200_reference_model = _sig(h, "vnpu_b200_reference_model", _ST, vp,
                                             C.POINTER(ReferenceModel))
            self.b200_matmul_kernel = _sig(h, "vnpu_b200_matmul_i8_kernel", C.c_char_p, u32, u32,
                                           u32, u32, vp)
            self.b200_last_matmul_kernel = _sig(h, "vnpu_b200_last_matmul_kernel", C.c_char_p)
            self.b200_ipc_get_handle = _sig(h, "vnpu_b200_ipc_get_handle", _ST, vp,
                                            C.POINTER(C.c_uint8))
            self.b200_ipc_open = _sig(h, "vnpu_b200_ipc_open", _ST, C.c_int,
                                      C.POINTER(C.c_uint8), C.POINTER(vp))
            self.b200_ipc_close = _sig(h, "vnpu_b200_ipc_close", _ST, vp)
            self.b200_selftest_wait = _sig(h, "vnpu_b200_selftest_wait_timeout", _ST, vp, u32)
            self.b200_packed_device = _sig(h, "vnpu_b200_packed_weights_device", _ST, vp,
                                           C.POINTER(vp), C.POINTER(u32), C.POINTER(vp))
            self.b200_capture_begin = _sig(h, "vnpu_b200_capture_begin", _ST, vp)
            self.b200_capture_end = _sig(h, "vnpu_b200_capture_end", _ST, vp, C.POINTER(vp))
            self.b200_graph_launch = _sig(h, "vnpu_b200_graph_launch", _ST, vp, vp)
            self.b200_graph_destroy = _sig(h, "vnpu_b200_graph_destroy", None, vp)
            self.b200_block_create = _sig(h, "vnpu_b200_block_create", _ST, vp,
                                          C.POINTER(BlockConfigArgs), vp, vp, vp, vp, vp, vp,
                                          C.POINTER(vp))
            self.b200_block_forward = _sig(h, "vnpu_b200_block_forward", _ST, vp, vp, u32, u32, vp)
            self.b200_block_decode = _sig(h, "vnpu_b200_block_decode", _ST, vp, vp, vp)
            self.b200_block_reset = _sig(h, "vnpu_b200_block_reset", _ST, vp)
            self.b200_block_destroy = _sig(h, "vnpu_b200_block_destroy", None, vp)

    def check(self, rc: int, what: str):
        if rc != OK:
            msg = self.status_string(rc)
            raise VnpuError(f"{what} failed ({msg.decode() if msg else rc})", rc)


class Device:
    """A vnpu device plus one stream: the unit the tests and the bench drive."""

    def __init__(self, lib: Lib, num_threads: int = 0, ordinal: int = 0, tiles=None):
        self.lib = lib
        cfg = Config()
        lib.config_init(C.byref(cfg))
        if num_threads:
            cfg.num_threads = num_threads
        if tiles:
            cfg.tile_m, cfg.tile_k, cfg.tile_n = tiles
        cfg.reserved0 = ordinal
        dev = vp()
        lib.check(lib.device_create(C.byref(cfg), C.byref(dev)), "device_create")
        self.dev = dev
        st = vp()
        lib.check(lib.stream_create(dev, 0, C.byref(st)), "stream_create")
        self.stream = st

    def close(self):
        if self.dev:
            self.lib.device_destroy(self.dev)
            self.dev = None
            self.stream = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def info(self) -> DeviceInfo:
        inf = DeviceInfo()
        self.lib.check(self.lib.device_get_info(self.dev, C.byref(inf)), "device_get_info")
        return inf

    def reference_model(self) -> ReferenceModel:
        """The reference device configuration whose rounding this B200 device
        reproduces (B200 library only)."""
        rm = ReferenceModel()
        self.lib.check(self.lib.b200_reference_model(self.dev, C.byref(rm)), "reference_model")
        return rm

    def status(self) -> DeviceStatus:
        s = DeviceStatus()
        self.lib.check(self.lib.device_get_status(self.dev, C.byref(s)), "device_get_status")
        return s

    def sync(self) -> int:
        return self.lib.stream_sync(self.stream)

    # -- packed weights ------------------------------------------------------
    def pack(self, B, scales, K: int, N: int, ldb: int = 0, trans_b: int = 0) -> int:
        w = vp()
        self.lib.check(self.lib.pack_weights_i8(self.dev, ptr(B), ptr(scales), K, N, ldb, trans_b,
                                                C.byref(w)), "pack_weights_i8")
        return w.value

    def packed_info(self, w: int):
        K, N, nbytes = u32(), u32(), u64()
        sc, cs = vp(), vp()
        self.lib.check(self.lib.packed_weights_info(w, C.byref(K), C.byref(N), C.byref(nbytes),
                                                    C.byref(sc), C.byref(cs)),
                       "packed_weights_info")
        return K.value, N.value, nbytes.value, sc.value, cs.value

    def unpack(self, w: int):
        self.lib.packed_weights_destroy(w)

    # -- synchronous ops -----------------------------------------------------
    def matmul_i8(self, A, w, scale_a, bias, Cout, M, K, N, lda=0, ldc=0, epilogue=0,
                  unit=UNIT_AUTO, flags=0, check=True) -> int:
        a = MatmulI8Args(ptr(A), w, ptr(scale_a), ptr(bias), ptr(Cout), M, K, N, lda, ldc,
                         epilogue, unit)
        if flags:
            cmd = Command()
            cmd.opcode = OP_MATMUL_I8
            cmd.flags = flags
            cmd.args.matmul_i8 = a
            rc = self.lib.stream_submit(self.stream, C.byref(cmd), 1, None)
            if rc == OK:
                rc = self.lib.stream_sync(self.stream)
        else:
            rc = self.lib.matmul_i8(self.stream, C.byref(a))
        if check:
            self.lib.check(rc, "matmul_i8")
        return rc

    def matmul_f32(self, A, B, Cout, M, K, N, bias=None, lda=0, ldb=0, ldc=0, trans_a=0, trans_b=0,
                   alpha=1.0, beta=0.0, epilogue=0, unit=UNIT_AUTO, tile_mask=None,
                   mask_tile_m=0, mask_tile_n=0, flags=0, check=True) -> int:
        a = MatmulF32Args(ptr(A), ptr(B), ptr(bias), ptr(Cout), M, K, N, lda, ldb, ldc, trans_a,
                          trans_b, alpha, beta, epilogue, unit, 0, ptr(tile_mask), mask_tile_m,
                          mask_tile_n)
        if flags:
            cmd = Command()
            cmd.opcode = OP_MATMUL_F32
            cmd.flags = flags
            cmd.args.matmul_f32 = a
            rc = self.lib.stream_submit(self.stream, C.byref(cmd), 1, None)
            if rc == OK:
                rc = self.lib.stream_sync(self.stream)
        else:
            rc = self.lib.matmul_f32(self.stream, C.byref(a))
        if check:
            self.lib.check(rc, "matmul_f32")
        return rc

    def quantize_i8(self, X, Y, scales, rows, cols, axis=QUANT_PER_ROW, check=True) -> int:
        a = QuantizeI8Args(ptr(X), ptr(Y), ptr(scales), rows, cols, axis, 0)
        rc = self.lib.quantize_i8(self.stream, C.byref(a))
        if check:
            self.lib.check(rc, "quantize_i8")
        return rc

    def matmul_i8_swiglu(self, A, w, scale_a, bias, Y, M, K, N, lda=0, ldy=0, epilogue=EPI_NONE,
                         alpha=1.0, flags=0, sync=True) -> int:
        """MATMUL_I8 of the [K][N = 2I] gate/up weight and SWIGLU_F32 of its
        halves into Y (M x I), as one VNPU_B200_OP_MATMUL_I8_SWIGLU command."""
        a = MatmulI8SwigluArgs(ptr(A), w, ptr(scale_a), ptr(bias), ptr(Y), M, K, N, lda, ldy,
                               epilogue, alpha, 0)
        cmd = b200_command(OP_B200_MATMUL_I8_SWIGLU, a)
        cmd.flags = flags
        rc = self.submit([cmd])
        if rc != OK or not sync:
            return rc
        return self.sync()

    def matmul_i8_scatter(self, A, w, scale_a, bias, dsts, M, K, N, ldd, col_offset,
                          epilogue=EPI_NONE, lda=0, sync=True, flags=0) -> int:
        """MATMUL_I8 of a column shard written into every destination in dsts
        (device pointers, [M][ldd] f32 each) at columns col_offset.."""
        d = (vp * B200_SCATTER_MAX)(*([ptr(x) for x in dsts] + [None] * (B200_SCATTER_MAX - len(dsts))))
        a = MatmulI8ScatterArgs(ptr(A), w, ptr(scale_a), ptr(bias), d, M, K, N, lda, ldd,
                                col_offset, len(dsts), epilogue)
        cmd = b200_command(OP_B200_MATMUL_I8_SCATTER, a)
        cmd.flags = flags
        rc = self.submit([cmd])
        if rc != OK or not sync:
            return rc
        return self.sync()

    def ipc_handle(self, device_ptr) -> bytes:
        h = (C.c_uint8 * 64)()
        self.lib.check(self.lib.b200_ipc_get_handle(ptr(device_ptr), h), "ipc_get_handle")
        return bytes(h)

    def ipc_open(self, handle: bytes, device: int) -> int:
        h = (C.c_uint8 * 64).from_buffer_copy(handle)
        out = vp()
        self.lib.check(self.lib.b200_ipc_open(device, h, C.byref(out)), "ipc_open")
        return out.value

    def rmsnorm_quantize(self, X, W, Y, Q, scales, rows, cols, eps) -> None:
        a = RmsnormQuantizeArgs(ptr(X), ptr(W), ptr(Y), ptr(Q), ptr(scales), rows, cols, eps, 0)
        self.lib.check(self.submit([b200_command(OP_B200_RMSNORM_QUANTIZE_I8, a)]), "submit")
        self.lib.check(self.sync(), "rmsnorm_quantize")

    def swiglu_quantize(self, G, U, Y, Q, scales, rows, cols, alpha=0.0, ld=0) -> None:
        a = SwigluQuantizeArgs(ptr(G), ptr(U), ptr(Y), ptr(Q), ptr(scales), rows, cols, alpha, ld)
        self.lib.check(self.submit([b200_command(OP_B200_SWIGLU_QUANTIZE_I8, a)]), "submit")
        self.lib.check(self.sync(), "swiglu_quantize")

    def rmsnorm(self, X, W, Y, rows, cols, eps) -> None:
        a = RmsnormArgs(ptr(X), ptr(W), ptr(Y), rows, cols, eps, 0)
        self.lib.check(self.lib.rmsnorm_f32(self.stream, C.byref(a)), "rmsnorm_f32")

    def rope(self, Q, K, positions, batch, heads, q_seq, k_seq, head_dim, position_offset=0,
             interleaved=0, theta=10000.0, scaling=1.0) -> None:
        a = RopeArgs(ptr(Q), ptr(K), ptr(positions), batch, heads, q_seq, k_seq, head_dim,
                     position_offset, interleaved, theta, scaling)
        self.lib.check(self.lib.rope_f32(self.stream, C.byref(a)), "rope_f32")

    def swiglu(self, g, u, Y, count, alpha=1.0) -> None:
        a = SwigluArgs(ptr(g), ptr(u), ptr(Y), count, alpha, 0, 0)
        self.lib.check(self.lib.swiglu_f32(self.stream, C.byref(a)), "swiglu_f32")

    def add(self, A, B, Y, count, alpha=1.0, beta=1.0) -> None:
        a = BinaryArgs(ptr(A), ptr(B), ptr(Y), count, alpha, beta, 0, 0)
        self.lib.check(self.lib.add_f32(self.stream, C.byref(a)), "add_f32")

    def attention(self, Q, K, V, mask, O, batch, heads, seq_q, seq_k, head_dim, causal=1,
                  scale=0.0, flags=0) -> None:
        a = AttentionArgs(ptr(Q), ptr(K), ptr(V), ptr(mask), ptr(O), None, 0, batch, heads, seq_q,
                          seq_k, head_dim, causal, scale, 0)
        if flags:
            cmd = Command()
            cmd.opcode = OP_ATTENTION_F32
            cmd.flags = flags
            cmd.args.attention = a
            rc = self.lib.stream_submit(self.stream, C.byref(cmd), 1, None)
            if rc == OK:
                rc = self.lib.stream_sync(self.stream)
            self.lib.check(rc, "attention_f32")
        else:
            self.lib.check(self.lib.attention_f32(self.stream, C.byref(a)), "attention_f32")

    def submit(self, cmds, event=None) -> int:
        arr = (Command * len(cmds))(*cmds)
        return self.lib.stream_submit(self.stream, arr, len(cmds), event)

    def capture(self, cmds) -> int:
        """Record `cmds` (device operands only) as a CUDA graph; returns the handle."""
        self.lib.check(self.lib.b200_capture_begin(self.stream), "capture_begin")
        rc = self.submit(cmds)
        g = vp()
        rc2 = self.lib.b200_capture_end(self.stream, C.byref(g))
        self.lib.check(rc, "submit while capturing")
        self.lib.check(rc2, "capture_end")
        return g.value

    def replay(self, graph: int) -> None:
        self.lib.check(self.lib.b200_graph_launch(graph, self.stream), "graph_launch")
