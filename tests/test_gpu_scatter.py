"""MATMUL_I8_SCATTER: the column-sharded GEMM fused with the all-gather of its
output (include/vnpu_b200.h).

* One GPU, two local destinations: the scattered shard equals MATMUL_I8 of
  the same shard bit for bit, lands at the right columns of every
  destination, and nothing else is written.
* Two GPUs (skipped with fewer): two processes each scatter their shard into
  their own full output and the peer's (CUDA IPC, NVLink stores); after a
  barrier both full outputs equal the oracle's full GEMM.  Hosts the IPC
  entry points too.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return pytest.importorskip("torch")


@pytest.mark.parametrize("M,K,N,ldd,col,epi,with_bias", [
    (300, 1024, 700, 2048, 256, 2, True),
    (512, 2048, 512, 1024, 512, 0, False),
    (77, 256, 1000, 1024, 0, 3, True),
    (1024, 4096, 2048, 4096, 2048, 0, False)])
def test_scatter_matches_matmul(gpu, oracle, torch, M, K, N, ldd, col, epi, with_bias):
    rng = np.random.default_rng(M + N + col)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.01, N).astype(np.float32) if with_bias else None
    w = gpu.pack(B, sb, K, N)
    try:
        Ad = torch.from_numpy(A).cuda()
        sad = torch.from_numpy(sa).cuda()
        bd = torch.from_numpy(bias).cuda() if with_bias else None
        rows = np.arange(0, M, 7)
        # one form forced for both: the scatter equals MATMUL_I8 of the shard
        flags = vnpu.CMD_FLAG_EPI_BLOCK
        dsts = [torch.full((M, ldd), float("nan"), device="cuda") for _ in range(2)]
        torch.cuda.synchronize()
        assert gpu.matmul_i8_scatter(Ad, w, sad, bd, dsts, M, K, N, ldd, col, epi,
                                     flags=flags) == vnpu.OK
        Cref = torch.full((M, N), float("nan"), device="cuda")
        torch.cuda.synchronize()
        gpu.matmul_i8(Ad, w, sad, bd, Cref, M, K, N, epilogue=epi, flags=flags)
        ref = Cref.cpu().numpy()
        for d in dsts:
            h = d.cpu().numpy()
            assert bits_equal(h[:, col:col + N], ref)
            assert np.isnan(h[:, :col]).all() and np.isnan(h[:, col + N:]).all()
        assert bits_equal(ref[rows], oracle.matmul_i8(A[rows], B, sa[rows], sb, bias, epi, 0))
        # no flags: the shard rounds as columns col.. of the ldd-wide product
        assert gpu.matmul_i8_scatter(Ad, w, sad, bd, dsts[:1], M, K, N, ldd, col, epi) == vnpu.OK
        got = dsts[0].cpu().numpy()[:, col:col + N]
        want = oracle.matmul_i8_model(gpu.reference_model(), A, B, sa, sb, bias, epi, rows=rows,
                                      n_full=ldd, col_base=col)
        assert bits_equal(got[rows], want)
    finally:
        gpu.unpack(w)


def test_scatter_rejects_bad_layout(b200_lib, torch):
    dev = vnpu.Device(b200_lib)
    try:
        A = torch.zeros((4, 256), dtype=torch.int8, device="cuda")
        D = torch.zeros((4, 1024), device="cuda")
        B = np.zeros((256, 512), np.int8)
        w = dev.pack(B, None, 256, 512)
        torch.cuda.synchronize()
        # the shard does not fit at column 768 of a 1024-wide output
        assert dev.matmul_i8_scatter(A, w, None, None, [D], 4, 256, 512, 1024, 768) == \
            vnpu.ERR_DEVICE_ERROR
        dev.unpack(w)
    finally:
        dev.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, port, M, K, N_total, seed, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.cuda.set_device(rank)
    lib = vnpu.Lib(vnpu.LIB_PATH)
    dev = vnpu.Device(lib, ordinal=rank)
    rng = np.random.default_rng(seed)   # same inputs on both ranks
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    sa = rng.uniform(0.5, 1.5, M).astype(np.float32)
    B = rng.integers(-128, 128, (K, N_total), dtype=np.int8)
    sb = rng.uniform(0.001, 0.01, N_total).astype(np.float32)
    n = N_total // 2
    col = rank * n
    w = dev.pack(np.ascontiguousarray(B[:, col:col + n]), np.ascontiguousarray(sb[col:col + n]), K, n)
    # full output in library-allocated memory (a cudaMalloc base: exportable)
    buf = vnpu.vp()
    lib.check(lib.buffer_alloc(dev.dev, M * N_total * 4, vnpu.C.byref(buf)), "buffer_alloc")
    mine = lib.buffer_host_ptr(buf)
    handles = [None, None]
    dist.all_gather_object(handles, dev.ipc_handle(mine))
    peer = dev.ipc_open(handles[1 - rank], rank)
    Ad = torch.from_numpy(A).cuda()
    sad = torch.from_numpy(sa).cuda()
    torch.cuda.synchronize()
    rc = dev.matmul_i8_scatter(Ad, w, sad, None, [mine, peer], M, K, n, N_total, col)
    dist.barrier()   # both ranks' scatters have completed
    out = np.empty((M, N_total), np.float32)
    cp = vnpu.Command()
    cp.opcode = vnpu.OP_COPY
    cp.args.copy = vnpu.CopyArgs(out.ctypes.data, mine, out.nbytes, 0)
    lib.check(dev.submit([cp]), "submit copy")
    lib.check(dev.sync(), "copy")
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), out)
    np.save(os.path.join(out_dir, f"rc{rank}.npy"), np.array([rc]))
    dist.barrier()
    lib.b200_ipc_close(peer)
    lib.buffer_free(buf)
    dev.unpack(w)
    dev.close()
    dist.destroy_process_group()


def test_scatter_two_gpus(oracle, torch, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    M, K, N_total, seed = 300, 512, 1024, 5
    mp.spawn(_two_gpu_worker, args=(_free_port(), M, K, N_total, seed, str(tmp_path)), nprocs=2,
             join=True)
    rng = np.random.default_rng(seed)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    sa = rng.uniform(0.5, 1.5, M).astype(np.float32)
    B = rng.integers(-128, 128, (K, N_total), dtype=np.int8)
    sb = rng.uniform(0.001, 0.01, N_total).astype(np.float32)
    ref = oracle.matmul_i8(A, B, sa, sb, None, 0, 0)
    for r in range(2):
        assert int(np.load(tmp_path / f"rc{r}.npy")[0]) == vnpu.OK
        assert bits_equal(np.load(tmp_path / f"rank{r}.npy"), ref), r
