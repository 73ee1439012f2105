"""Column (N) sharding of MATMUL_I8 across GPUs.

Each output column depends only on its weight column, scale and bias
(reference src/kernels/kernels.cpp:526-535), so splitting N across ranks needs
no reduction and every rank's columns are bit-identical to a single-GPU run.
The reference's own multi-device split is by rows, F32 only
(src/cluster/cluster.cpp:453-470); the B200 build splits weights by columns so
each GPU keeps 1/P of them resident.

Shards are multiples of ``align`` columns (the tensor-core tile width) except
the last, so only one rank sees a ragged tile.
"""
from __future__ import annotations


def column_shard(n_total: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """Half-open column range [n0, n1) of ``rank`` out of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    blocks = -(-n_total // align)
    base, extra = divmod(blocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(b0 * align, n_total), min(b1 * align, n_total)


def gathered_to_row_major(shards, m: int) -> "list":
    """Reassemble shard-major blocks [(m, n_r) per rank] into row-major rows.

    NCCL all-gathers contiguous buffers, so the gathered output is shard-major
    [P][M][N_r]; a consumer that needs row-major [M][N] concatenates along
    columns (numpy / torch ``cat(dim=1)``).
    """
    import numpy as np

    return np.concatenate([np.asarray(s).reshape(m, -1) for s in shards], axis=1)


# Status codes of include/vnpu.h returned by join_group.
VNPU_OK = 0
VNPU_ERR_TIMEOUT = -7


def join_group(backend: str, rank: int, world: int, timeout_s: float,
               device_id=None) -> int:
    """Join the process group of the column-sharded GEMM within a deadline.

    A rank that never joins (a crashed or hung peer) would otherwise leave the
    others blocked in the rendezvous or in their first collective.  The join
    and a first barrier must both finish within ``timeout_s`` seconds (the
    process group's own timeout, which also bounds every later collective);
    otherwise the group is torn down and ``VNPU_ERR_TIMEOUT`` is returned, as
    the reference reports a wait that ran out (include/vnpu.h, vnpu_event_wait).
    Returns ``VNPU_OK`` when every rank has joined.
    """
    from datetime import timedelta

    import torch.distributed as dist

    kwargs = {"timeout": timedelta(seconds=timeout_s)}
    if device_id is not None:
        kwargs["device_id"] = device_id
    try:
        dist.init_process_group(backend, rank=rank, world_size=world, **kwargs)
        dist.barrier()
        return VNPU_OK
    except (RuntimeError, TimeoutError, ValueError) as exc:   # rendezvous or barrier ran out
        if "timeout" not in str(exc).lower() and "timed out" not in str(exc).lower() \
                and not isinstance(exc, TimeoutError):
            raise
        if dist.is_initialized():
            dist.destroy_process_group()
        return VNPU_ERR_TIMEOUT
