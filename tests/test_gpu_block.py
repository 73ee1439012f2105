"""The decoder block (configs[3] structure) on the B200, end to end.

* Device-resident driver (torch buffers, CUDA-graph decode; with and without
  the fused RMSNorm/SwiGLU -> QUANTIZE_I8 prologues) vs the same driver on
  host arrays through the B200 library with the reference's op sequence:
  identical bits, which pins the layout glue (QKV split, head-major
  transposes, KV-cache append, mask) and the fused opcodes.
* vs the oracle restatement of the reference: within tolerance (RoPE uses the
  device sinf/cosf, a few ulp from glibc; everything else is bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest

import vnpu
from conftest import bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    return pytest.importorskip("torch")


def _run_device(b200_lib, torch, cfg, x, toks, graph, fused=True, swiglu_epilogue=True):
    from llm_block import B200Block
    dev = vnpu.Device(b200_lib)
    blk = B200Block(cfg, b200_lib, dev, torch, fused=fused, swiglu_epilogue=swiglu_epilogue)
    outs = [blk.forward(torch.from_numpy(x).cuda(), 0).cpu().numpy()]
    first = True
    for i, t in enumerate(toks):
        p = x.shape[0] + i
        if graph:
            xin = blk._buf("decode_in", (1, cfg.d))
            xin.copy_(torch.from_numpy(t).cuda())
            if first:
                blk.pos.fill_(p)
                torch.cuda.synchronize()
                y = blk.capture_decode(xin)
                blk.pos.fill_(p)
                first = False
            blk.replay_decode()
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy().copy())
        else:
            outs.append(blk.forward(torch.from_numpy(t).cuda(), p).cpu().numpy())
    assert dev.sync() == vnpu.OK
    blk.close()
    dev.close()
    return outs


@pytest.mark.parametrize("graph,fused,swiglu_epilogue", [
    (False, False, False), (False, True, True), (True, True, True),
    (True, True, False),   # the SwiGLU -> QUANTIZE_I8 prologue instead of the epilogue
])
def test_block_device_equals_host_driver(b200_lib, torch, graph, fused, swiglu_epilogue):
    from llm_block import BlockConfig, HostBlock
    cfg = BlockConfig(d=256, heads=4, inter=704, cap=48)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (20, cfg.d)).astype(np.float32)
    toks = [rng.normal(0, 1, (1, cfg.d)).astype(np.float32) for _ in range(5)]
    dev_outs = _run_device(b200_lib, torch, cfg, x, toks, graph, fused, swiglu_epilogue)
    host = HostBlock(cfg, lib=b200_lib)
    host_outs = [host.forward(x, 0)] + [host.forward(t, x.shape[0] + i) for i, t in enumerate(toks)]
    host.close()
    for i, (a, b) in enumerate(zip(dev_outs, host_outs)):
        assert bits_equal(a, b), f"step {i}: max abs {np.abs(a - b).max()}"


def test_block_vs_oracle(b200_lib, torch, oracle):
    from llm_block import BlockConfig, HostBlock
    cfg = BlockConfig(d=256, heads=4, inter=704, cap=48)
    rng = np.random.default_rng(6)
    x = rng.normal(0, 1, (20, cfg.d)).astype(np.float32)
    toks = [rng.normal(0, 1, (1, cfg.d)).astype(np.float32) for _ in range(4)]
    dev_outs = _run_device(b200_lib, torch, cfg, x, toks, graph=True)
    orc = HostBlock(cfg, oracle=oracle)
    ref_outs = [orc.forward(x, 0)] + [orc.forward(t, x.shape[0] + i) for i, t in enumerate(toks)]
    for a, b in zip(dev_outs, ref_outs):
        # RoPE's few-ulp differences can move an activation across an int8
        # rounding boundary; the block output stays within 1e-3 of its norm.
        assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(b)
