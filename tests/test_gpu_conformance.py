"""The reference's own conformance programs, compiled from its sources
against its own headers and linked against the B200 library
(oracle/Makefile, target `tools`):

* tools/conformance.cpp - int8 and f32 bit-identity across units, threads,
  packing and streams (:251-345 the int8 checks);
* tests/fuzz_shapes.cpp - random shapes, every unit, against a host
  reference (:117-169 the int8 iterations);
* tools/selftest.cpp (+ selftest_main.cpp) - the reference's self test;
* examples/dynamic_load.c - dlopen + vnpu_get_backend_v1 only.

selftest cases that need an opcode outside the int8 path (SOFTMAX_F32,
GELU_F32, MTP_HEAD_F32) or the TCP appliance (speculative decoding) fail by
design with VNPU_ERR_UNSUPPORTED; every other case must pass.
"""
from __future__ import annotations

import os
import re
import subprocess

import pytest

import vnpu
from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "oracle", "_ref", "bin")
OUTSIDE_THE_PATH = {"rmsnorm_softmax_swiglu_gelu", "mtp_head", "speculative_step"}


def _run(args, timeout=900, env=None):
    exe = os.path.join(BIN, args[0])
    if not os.path.exists(exe):
        pytest.skip(f"{args[0]} not built (make -C oracle tools REF=<reference checkout>)")
    p = subprocess.run([exe] + args[1:], capture_output=True, text=True, timeout=timeout,
                       env={**os.environ, **(env or {})}, cwd=BIN)
    return p.returncode, p.stdout + p.stderr


def test_conformance():
    rc, out = _run(["vnpu-conformance", "--verbose"])
    assert rc == 0, out[-3000:]
    m = re.search(r"(\d+) checks, (\d+) failures", out)
    assert m and int(m.group(1)) >= 10 and m.group(2) == "0", out[-3000:]


def test_fuzz_shapes():
    rc, out = _run(["vnpu-fuzz", "200"])
    assert rc == 0, out[-3000:]
    assert re.search(r"fuzz: 200 iterations, 0 failures", out), out[-3000:]


def test_dynamic_load():
    rc, out = _run(["dynamic_load"], env={"VNPU_LIBRARY": vnpu.LIB_PATH})
    assert rc == 0, out[-3000:]


def test_selftest():
    rc, out = _run(["vnpu-selftest"])
    results = dict((name, status) for status, name in re.findall(r"\[(PASS|FAIL)\] (\S+)", out))
    assert len(results) >= 17, out[-3000:]
    failed = {n for n, s in results.items() if s == "FAIL"}
    assert failed <= OUTSIDE_THE_PATH, (failed - OUTSIDE_THE_PATH, out[-3000:])
    for must in ("gemm_i8_vs_f32", "concurrent_streams_same_device", "attention_small",
                 "rope_inplace", "local_cluster", "backend_vtable", "autotune_small"):
        assert results.get(must) == "PASS", (must, out[-3000:])
