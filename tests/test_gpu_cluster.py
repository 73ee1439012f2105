"""The local cluster API (vnpu_cluster_*) over B200 devices.

The reference splits MATMUL_F32 rows across its local devices by weight
(src/cluster/cluster.cpp:437-546); each worker's rows are then a MATMUL_F32 of
their own, rounded by that worker's tile geometry.  The B200 cluster, built
from devices configured like the reference's (same thread count), must give
the reference cluster's bits: checked against the reference library built
from source when it is present, and against the oracle per worker always.
Workers are two streams' worth of devices on GPU 0 (and GPU 1 when visible).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import vnpu
from conftest import REF_LIB, bits_equal

pytestmark = pytest.mark.gpu


def _cluster(lib, devices, weights):
    cfg = vnpu.ClusterConfig()
    lib.cluster_config_init(C.byref(cfg))
    cl = vnpu.vp()
    assert lib.cluster_create(C.byref(cfg), C.byref(cl)) == vnpu.OK
    for d, w in zip(devices, weights):
        assert lib.cluster_add_device(cl, d.dev, w) == vnpu.OK
    return cl


def _run(lib, cl, A, B, M, K, N, trans_b):
    h = vnpu.vp()
    assert lib.cluster_cache_weights_f32(cl, b"w", B.ctypes.data, K, N, trans_b,
                                         C.byref(h)) == vnpu.OK
    Cm = np.full((M, N), np.nan, np.float32)
    assert lib.cluster_matmul_f32(cl, h, A.ctypes.data, Cm.ctypes.data, M, K, N,
                                  vnpu.UNIT_AUTO) == vnpu.OK
    return Cm


@pytest.mark.parametrize("M,K,N,trans_b,weights", [(100, 300, 200, 0, (1, 3)),
                                                   (37, 129, 70, 1, (2, 2)),
                                                   (9, 1000, 640, 0, (1, 1))])
def test_cluster_matmul_matches_reference(b200_lib, oracle, M, K, N, trans_b, weights):
    torch = pytest.importorskip("torch")
    ordinals = [0, 1 if torch.cuda.device_count() > 1 else 0]
    threads = 4
    rng = np.random.default_rng(M + K + N)
    A = rng.normal(0, 1, (M, K)).astype(np.float32)
    B = rng.normal(0, 1, (N, K) if trans_b else (K, N)).astype(np.float32)
    devs = [vnpu.Device(b200_lib, num_threads=threads, ordinal=o) for o in ordinals]
    cl = _cluster(b200_lib, devs, weights)
    try:
        got = _run(b200_lib, cl, A, B, M, K, N, trans_b)
        st = vnpu.ClusterStats()
        assert b200_lib.cluster_get_stats(cl, C.byref(st)) == vnpu.OK
        assert st.total_jobs == 1 and st.local_jobs == 2 and st.failed_jobs == 0
        node = vnpu.vp()
        assert b200_lib.cluster_add_remote(cl, None, C.byref(node)) == vnpu.ERR_UNSUPPORTED
    finally:
        b200_lib.cluster_destroy(cl)
        for d in devs:
            d.close()
    # per-worker oracle: rows split by weight, the cached weights canonical K x N
    Bc = np.ascontiguousarray(B.T) if trans_b else B
    total, start = sum(weights), 0
    for i, w in enumerate(weights):
        rows = M - start if i == len(weights) - 1 else M * w // total
        if rows:
            ref = oracle.matmul_f32(A[start:start + rows], Bc, rows, K, N, threads=threads)
            assert bits_equal(got[start:start + rows], ref), i
        start += rows
    if os.path.exists(REF_LIB):
        os.environ["VNPU_FORCE_ISA"] = "avx2"
        try:
            rlib = vnpu.Lib(REF_LIB)
            rdevs = [vnpu.Device(rlib, num_threads=threads) for _ in ordinals]
        finally:
            os.environ.pop("VNPU_FORCE_ISA", None)
        rcl = _cluster(rlib, rdevs, weights)
        try:
            assert bits_equal(got, _run(rlib, rcl, A, B, M, K, N, trans_b))
        finally:
            rlib.cluster_destroy(rcl)
            for d in rdevs:
                d.close()
