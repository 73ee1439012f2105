"""The int8 column-sharded local cluster (vnpu_cluster_cache_weights_i8 /
vnpu_cluster_matmul_i8, VNPU_B200_OP_MATMUL_I8_SHARD).

The reference's cluster splits only MATMUL_F32, by rows
(src/cluster/cluster.cpp:437-546).  The B200 cluster splits int8 weights by
columns: every output column depends only on its own weight column, scale and
bias (src/kernels/kernels.cpp:526-535), and each shard's epilogue rounds an
element in the form the reference device gives the element of the whole
product (src/kernels/kernels.cpp:922-978 over the tile grid of
src/core/scheduler.cpp:75-207).  So the cluster's C is bit-identical to one
MATMUL_I8 of the whole weight on one device, which is itself the reference
device's output.  Workers are devices on GPU 0 (and GPU 1 when visible).
Tolerance: 0 ulp.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import vnpu
from conftest import bits_equal, ulp_diff

pytestmark = pytest.mark.gpu


def _cluster(lib, devices, weights):
    cfg = vnpu.ClusterConfig()
    lib.cluster_config_init(C.byref(cfg))
    cl = vnpu.vp()
    assert lib.cluster_create(C.byref(cfg), C.byref(cl)) == vnpu.OK
    for d, w in zip(devices, weights):
        assert lib.cluster_add_device(cl, d.dev, w) == vnpu.OK
    return cl


def _single(dev, A, B, sa, sb, bias, epi):
    M, (K, N) = A.shape[0], B.shape
    w = dev.pack(B, sb, K, N)
    try:
        C_ = np.full((M, N), np.nan, np.float32)
        dev.matmul_i8(A, w, sa, bias, C_, M, K, N, epilogue=epi)
    finally:
        dev.unpack(w)
    return C_


@pytest.mark.parametrize("M,K,N,weights,epi,with_bias", [
    (64, 4096, 4096, (1, 1), vnpu.EPI_NONE, False),     # two 2048-column shards
    (1, 4096, 11008, (1, 3), vnpu.EPI_SILU, True),      # decode row, uneven weights
    (37, 1000, 3000, (2, 1), vnpu.EPI_SILU, True),      # ragged shard, odd rows
    (301, 4100, 700, (1, 1), vnpu.EPI_GELU_TANH, True), # mixed forms across the cut
    (8, 512, 200, (1, 1), vnpu.EPI_NONE, True),         # one shard only (N < 256)
])
def test_cluster_matmul_i8_matches_one_device(b200_lib, oracle, M, K, N, weights, epi,
                                              with_bias):
    torch = pytest.importorskip("torch")
    ordinals = [0, 1 if torch.cuda.device_count() > 1 else 0]
    rng = np.random.default_rng(M + K + N)
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32) if with_bias else None
    devs = [vnpu.Device(b200_lib, ordinal=o) for o in ordinals]
    cl = _cluster(b200_lib, devs, weights)
    try:
        h = vnpu.vp()
        assert b200_lib.cluster_cache_weights_i8(cl, b"w8", B.ctypes.data, sb.ctypes.data,
                                                 K, N, 0, C.byref(h)) == vnpu.OK
        ldc = N + 3
        got = np.full((M, ldc), np.nan, np.float32)
        assert b200_lib.cluster_matmul_i8(cl, h, A.ctypes.data, sa.ctypes.data,
                                          bias.ctypes.data if bias is not None else None,
                                          got.ctypes.data, M, K, N, ldc, epi) == vnpu.OK
        assert np.isnan(got[:, N:]).all()       # the row padding is untouched
        got = got[:, :N]
        st = vnpu.ClusterStats()
        assert b200_lib.cluster_get_stats(cl, C.byref(st)) == vnpu.OK
        shards = 1 if N <= 256 else 2
        assert st.total_jobs == 1 and st.local_jobs == shards and st.failed_jobs == 0
        # a wrong shape is refused before any device work
        assert b200_lib.cluster_matmul_i8(cl, h, A.ctypes.data, sa.ctypes.data, None,
                                          got.ctypes.data, M, K + 1, N, 0, epi) \
            == vnpu.ERR_INVALID_ARGUMENT
        want = _single(devs[0], A, B, sa, sb, bias, epi)
        model = devs[0].reference_model()
    finally:
        b200_lib.cluster_destroy(cl)
        for d in devs:
            d.close()
    assert bits_equal(got, want), f"max ulp {ulp_diff(got, want)}"
    rows = np.unique(np.r_[0, M // 2, M - 1])
    ref = oracle.matmul_i8_model(model, A, B, sa, sb, bias, epi, rows=rows)
    assert bits_equal(got[rows], ref), f"vs model: max ulp {ulp_diff(got[rows], ref)}"


def test_shard_opcode_matches_scatter_columns(b200_lib, oracle):
    """VNPU_B200_OP_MATMUL_I8_SHARD on one device: a shard of columns
    [col_base, col_base + width) of a K x n_full product, packed alone, gives
    those columns of the whole product's bits (forms of the whole grid)."""
    rng = np.random.default_rng(11)
    M, K, N = 5, 640, 1500
    A, sa = oracle.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32), 0)
    B, sb = oracle.quantize(rng.uniform(-1, 1, (K, N)).astype(np.float32), 1)
    bias = rng.normal(0, 0.5, N).astype(np.float32)
    with vnpu.Device(b200_lib, num_threads=3) as dev:
        whole = _single(dev, A, B, sa, sb, bias, vnpu.EPI_SILU)
        for n0, n1 in ((0, 512), (512, 1024), (1024, 1500)):
            Bs = np.ascontiguousarray(B[:, n0:n1])
            w = dev.pack(Bs, np.ascontiguousarray(sb[n0:n1]), K, n1 - n0)
            out = np.full((M, n1 - n0), np.nan, np.float32)
            bs = np.ascontiguousarray(bias[n0:n1])
            a = vnpu.MatmulI8ShardArgs(A.ctypes.data, w, sa.ctypes.data, bs.ctypes.data,
                                       out.ctypes.data, M, K, n1 - n0, 0, 0, vnpu.EPI_SILU,
                                       N, n0)
            try:
                dev.lib.check(dev.submit([vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_SHARD, a)]),
                              "submit")
                dev.lib.check(dev.sync(), "sync")
            finally:
                dev.unpack(w)
            assert bits_equal(out, whole[:, n0:n1]), (n0, ulp_diff(out, whole[:, n0:n1]))
        # a shard wider than the whole product is refused
        w = dev.pack(B[:, :100].copy(), sb[:100].copy(), K, 100)
        try:
            bad = vnpu.MatmulI8ShardArgs(A.ctypes.data, w, sa.ctypes.data, None,
                                         out.ctypes.data, M, K, 100, 0, 0, 0, 50, 0)
            rc = dev.submit([vnpu.b200_command(vnpu.OP_B200_MATMUL_I8_SHARD, bad)])
            if rc == vnpu.OK:
                rc = dev.sync()
            # refused at submit (validation) or reported by the stream's sticky error
            assert rc in (vnpu.ERR_INVALID_ARGUMENT, vnpu.ERR_DEVICE_ERROR)
        finally:
            dev.unpack(w)
