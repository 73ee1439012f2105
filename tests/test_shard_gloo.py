"""Host logic of the column-sharded multi-GPU GEMM, on CPU ranks (gloo).

Each of 2 ranks computes its column shard with the oracle, the shards are
all-gathered shard-major (as NCCL does on the GPU path) and reassembled; the
result must equal the single-rank product bit for bit, since columns never
mix (reference src/kernels/kernels.cpp:526-535).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from shard import column_shard, gathered_to_row_major


@pytest.mark.parametrize("n,world", [(28672, 8), (28672, 3), (1000, 4), (255, 2), (7, 4),
                                     (4096, 1)])
def test_shards_cover_columns(n, world):
    ranges = [column_shard(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 <= a1
    assert all(r0 % 256 == 0 or r0 == n for r0, _ in ranges)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch.distributed as dist

    import vnpu
    from conftest import ORACLE_LIB

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        from vnpu_oracle import Oracle
        orc = Oracle(ORACLE_LIB)
        rng = np.random.default_rng(0)
        M, K, N = 24, 96, 700
        A, sa = orc.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
        B, sb = orc.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
        bias = rng.normal(0, 0.01, N).astype(np.float32)
        n0, n1 = column_shard(N, world, rank)
        width = max(b - a for a, b in (column_shard(N, world, r) for r in range(world)))
        mine = np.zeros((M, width), np.float32)
        mine[:, : n1 - n0] = orc.matmul_i8(A, np.ascontiguousarray(B[:, n0:n1]), sa, sb[n0:n1],
                                           bias[n0:n1], 2, 0)
        gathered = [torch.zeros((M, width)) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(mine))
        shards = [g.numpy()[:, : (lambda r: column_shard(N, world, r)[1] - column_shard(N, world, r)[0])(r)]
                  for r, g in enumerate(gathered)]
        full = gathered_to_row_major(shards, M)
        ref = orc.matmul_i8(A, B, sa, sb, bias, 2, 0)
        q.put((rank, bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


def test_two_rank_column_shard_gather():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def _row_slice_main(rank, world, port, q):
    """End-to-end input path at N > 1 (bench.py): each rank quantizes its M/N
    rows of X per row and the int8 rows and scales are all-gathered; every
    rank then holds the whole matrix's QUANTIZE_I8 result.  Then each rank
    writes its GEMM column shard into a full output at its column offset (the
    MATMUL_I8_SCATTER layout); the assembled output equals the whole GEMM."""
    import torch
    import torch.distributed as dist

    import vnpu
    from conftest import ORACLE_LIB

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vnpu_oracle import Oracle
        orc = Oracle(ORACLE_LIB)
        rng = np.random.default_rng(1)
        M, K, N = 32, 80, 600
        X = rng.normal(0, 1, (M, K)).astype(np.float32)
        X[3, :5] = [2.5, -2.5, 0.0, np.nan, -0.0]
        rows = M // world
        A_mine, s_mine = orc.quantize(np.ascontiguousarray(X[rank * rows:(rank + 1) * rows]), 0)
        a_parts = [torch.zeros((rows, K), dtype=torch.int8) for _ in range(world)]
        s_parts = [torch.zeros(rows) for _ in range(world)]
        dist.all_gather(a_parts, torch.from_numpy(A_mine))
        dist.all_gather(s_parts, torch.from_numpy(s_mine))
        A = torch.cat(a_parts).numpy()
        sa = torch.cat(s_parts).numpy()
        A_ref, s_ref = orc.quantize(X, 0)
        ok = bool(np.array_equal(A, A_ref) and np.array_equal(sa.view(np.uint32), s_ref.view(np.uint32)))
        # scatter layout: shard r lands at its column offset in every full output
        B, sb = orc.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
        full = np.full((M, N), np.nan, np.float32)
        for r in range(world):
            r0, r1 = column_shard(N, world, r)
            full[:, r0:r1] = orc.matmul_i8(A, np.ascontiguousarray(B[:, r0:r1]), sa, sb[r0:r1],
                                           None, 0, 0)
        ref = orc.matmul_i8(A_ref, B, s_ref, sb, None, 0, 0)
        ok &= bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32)))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_rank_row_slice_quantize_and_scatter_layout():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_slice_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def _join_main(rank, world, port, q, timeout_s):
    import time

    from shard import join_group

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == world - 1:
        time.sleep(3600)          # this rank never joins; the test kills it
        return
    t0 = time.monotonic()
    rc = join_group("gloo", rank, world, timeout_s)
    q.put((rank, rc, time.monotonic() - t0))


def test_rank_that_never_joins_times_out():
    """Failure detection on CPU ranks: one of three ranks never joins
    the group.  The others get VNPU_ERR_TIMEOUT once the deadline passes
    instead of blocking; no GPU is involved."""
    import multiprocessing as mp

    from shard import VNPU_ERR_TIMEOUT

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world, timeout_s = 3, 4.0
    procs = [ctx.Process(target=_join_main, args=(r, world, port, q, timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=120) for _ in range(world - 1)]
    finally:
        procs[-1].kill()
        for p in procs:
            p.join(timeout=30)
    for rank, rc, elapsed in results:
        assert rc == VNPU_ERR_TIMEOUT, (rank, rc)
        assert elapsed < timeout_s * 10, (rank, elapsed)


def test_all_ranks_join():
    import multiprocessing as mp

    from shard import VNPU_OK

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()

    procs = [ctx.Process(target=_join_ok_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
    assert all(rc == VNPU_OK for _, rc in results)


def _join_ok_main(rank, world, port, q):
    import torch.distributed as dist

    from shard import join_group

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    rc = join_group("gloo", rank, world, 30.0)
    q.put((rank, rc))
    if dist.is_initialized():
        dist.destroy_process_group()
