"""Shared fixtures.

Markers: ``gpu`` tests need a B200 and run the B200 library's kernels through
its C ABI; everything else runs on the CPU (oracle vs golden vectors, ABI
surface, host logic, gloo multi-process logic).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "npuxl-improved_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import vnpu  # noqa: E402
from vnpu_oracle import Oracle  # noqa: E402

ORACLE_LIB = os.path.join(ROOT, "oracle", "liboracle.so")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libvnpu_ref.so")
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def reference_dir() -> str:
    """The reference checkout: VNPU_REFERENCE_DIR, else the directory
    oracle/_ref was built from (oracle/Makefile records it); "" if neither."""
    env = os.environ.get("VNPU_REFERENCE_DIR")
    if env:
        return env
    try:
        with open(os.path.join(ROOT, "oracle", "_ref", "REFERENCE_DIR")) as f:
            return f.read().strip()
    except OSError:
        return ""


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


def _ensure_oracle():
    if not os.path.exists(ORACLE_LIB):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def oracle():
    _ensure_oracle()
    return Oracle(ORACLE_LIB)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def b200_lib():
    """The B200 library.  Missing = a build failure, never a skip."""
    return vnpu.Lib(vnpu.LIB_PATH)


@pytest.fixture(scope="session")
def ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference library not built here (oracle/_ref)")
    return vnpu.Lib(REF_LIB)


@pytest.fixture(scope="module")
def gpu(b200_lib):
    """A B200 device + stream; fails loudly if the GPU path cannot start."""
    dev = vnpu.Device(b200_lib, ordinal=0)
    info = dev.info()
    assert info.features & vnpu.FEATURE_GPU_FUTURE, "B200 backend did not report the GPU unit"
    yield dev
    dev.close()


def ulp_diff(a: np.ndarray, b: np.ndarray) -> int:
    """Largest distance in units in the last place between two f32 arrays."""
    ai = a.astype(np.float32).view(np.int32).astype(np.int64)
    bi = b.astype(np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return int(np.abs(ai - bi).max()) if a.size else 0


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def read_records(path: str):
    """Tagged records written by tests/compat/legacy_scenario.c."""
    import struct
    data = open(path, "rb").read()
    out, i = [], 0
    while i < len(data):
        (ln,) = struct.unpack_from("<I", data, i)
        tag = data[i + 4:i + 4 + ln].decode()
        (n,) = struct.unpack_from("<Q", data, i + 4 + ln)
        start = i + 12 + ln
        out.append((tag, data[start:start + n]))
        i = start + n
    return out


def build_legacy_scenario(out_dir: str, include_dir: str, link_args: list) -> str:
    """Compile tests/compat/legacy_scenario.c against a header tree and a
    library; returns the executable's path."""
    exe = os.path.join(out_dir, "legacy_scenario")
    subprocess.run(["gcc", "-O1", "-I", include_dir,
                    os.path.join(ROOT, "tests", "compat", "legacy_scenario.c")] + link_args +
                   ["-o", exe], check=True)
    return exe
