"""The decoder block driven inside the library (vnpu_b200_block_* in
include/vnpu_b200.h) against the Python drivers of npuxl-improved_b200/llm_block.py:
the same bits for a prefill and KV-cached decode tokens, eager forward calls
and the replayed decode graph, with the SwiGLU in the gate/up epilogue or in
the down projection's prologue."""
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


def _create(lib, dev, cfg, flags=0):
    from llm_block import make_weights
    w, (n1, n2) = make_weights(cfg)
    c = vnpu.BlockConfigArgs(cfg.d, cfg.heads, cfg.inter, cfg.cap, cfg.eps, cfg.theta, flags, 0)
    blk = vnpu.vp()
    lib.check(lib.b200_block_create(dev.stream, C.byref(c), vnpu.ptr(w["qkv"]), vnpu.ptr(w["o"]),
                                    vnpu.ptr(w["gate_up"]), vnpu.ptr(w["down"]), vnpu.ptr(n1),
                                    vnpu.ptr(n2), C.byref(blk)), "block_create")
    return blk


@pytest.mark.parametrize("flags,graph", [(0, True), (0, False),
                                         (vnpu.B200_BLOCK_SWIGLU_PROLOGUE, True)])
def test_block_capi_equals_host_driver(b200_lib, torch, flags, graph):
    from llm_block import BlockConfig, HostBlock
    cfg = BlockConfig(d=256, heads=4, inter=704, cap=48)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (20, cfg.d)).astype(np.float32)
    toks = [rng.normal(0, 1, (1, cfg.d)).astype(np.float32) for _ in range(5)]
    dev = vnpu.Device(b200_lib)
    blk = _create(b200_lib, dev, cfg, flags)
    try:
        xd = torch.from_numpy(x).cuda()
        y = torch.full((20, cfg.d), float("nan"), device="cuda")
        b200_lib.check(b200_lib.b200_block_forward(blk, xd.data_ptr(), 20, 0, y.data_ptr()),
                       "block_forward")
        assert dev.sync() == vnpu.OK
        outs = [y.cpu().numpy().copy()]
        xin = torch.empty((1, cfg.d), device="cuda")
        yout = torch.empty((1, cfg.d), device="cuda")
        for i, t in enumerate(toks):
            xin.copy_(torch.from_numpy(t).cuda())
            torch.cuda.synchronize()
            if graph:
                b200_lib.check(b200_lib.b200_block_decode(blk, xin.data_ptr(), yout.data_ptr()),
                               "block_decode")
            else:
                b200_lib.check(b200_lib.b200_block_forward(blk, xin.data_ptr(), 1, 20 + i,
                                                           yout.data_ptr()), "block_forward")
            assert dev.sync() == vnpu.OK
            outs.append(yout.cpu().numpy().copy())
    finally:
        b200_lib.b200_block_destroy(blk)
        dev.close()
    host = HostBlock(cfg, lib=b200_lib)
    want = [host.forward(x, 0)] + [host.forward(t, 20 + i) for i, t in enumerate(toks)]
    host.close()
    for i, (a, b) in enumerate(zip(outs, want)):
        assert bits_equal(a, b), f"step {i}: max abs {np.abs(a - b).max()}"


def test_block_capi_reset_and_errors(b200_lib, torch):
    """reset() empties the cache (the same prefill gives the same bits);
    invalid calls are rejected before anything is enqueued."""
    from llm_block import BlockConfig
    cfg = BlockConfig(d=256, heads=4, inter=704, cap=48)
    dev = vnpu.Device(b200_lib)
    blk = _create(b200_lib, dev, cfg)
    try:
        x = torch.randn((8, cfg.d), device="cuda")
        y1 = torch.empty_like(x)
        y2 = torch.empty_like(x)
        b200_lib.check(b200_lib.b200_block_forward(blk, x.data_ptr(), 8, 0, y1.data_ptr()), "fwd")
        b200_lib.check(b200_lib.b200_block_reset(blk), "reset")
        b200_lib.check(b200_lib.b200_block_forward(blk, x.data_ptr(), 8, 0, y2.data_ptr()), "fwd")
        assert dev.sync() == vnpu.OK
        assert torch.equal(y1, y2)
        E = vnpu.ERR_INVALID_ARGUMENT
        assert b200_lib.b200_block_forward(blk, x.data_ptr(), 8, 3, y1.data_ptr()) == E  # prefill at pos > 0
        assert b200_lib.b200_block_forward(blk, x.data_ptr(), 49, 0, y1.data_ptr()) == E  # past capacity
        assert b200_lib.b200_block_forward(blk, x.data_ptr(), 1, 48, y1.data_ptr()) == E  # slot 48
        assert b200_lib.b200_block_forward(blk, x.data_ptr(), 8, 0, x.data_ptr()) == E  # y aliases x
        assert dev.sync() == vnpu.OK
    finally:
        b200_lib.b200_block_destroy(blk)
        dev.close()
