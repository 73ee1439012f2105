"""The legacy API on a GPU: tests/compat/legacy_scenario.c, linked against
libvnpu.so, must write exactly the bytes the reference's compat layer wrote
for the same calls (tests/golden/legacy_scenario.bin): every return value,
counter, VRAM byte and GEMM output (MATMUL_F32 on the B200)."""
from __future__ import annotations

import os
import subprocess

import pytest

import vnpu
from conftest import ROOT, build_legacy_scenario, read_records

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(ROOT, "tests", "golden", "legacy_scenario.bin")


def test_legacy_scenario_matches_reference(tmp_path):
    lib_dir = os.path.dirname(vnpu.LIB_PATH)
    exe = build_legacy_scenario(str(tmp_path), os.path.join(ROOT, "include"),
                                ["-L", lib_dir, "-lvnpu", f"-Wl,-rpath,{lib_dir}"])
    out = tmp_path / "b200.bin"
    env = {k: v for k, v in os.environ.items() if k not in ("VNPU_FORCE_ISA", "VNPU_PACK",
                                                            "VNPU_MODE", "VNPU_B200_EPILOGUE")}
    env["VNPU_THREADS"] = "4"
    r = subprocess.run([exe, str(out)], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    ours, ref = read_records(str(out)), read_records(GOLDEN)
    assert [t for t, _ in ours] == [t for t, _ in ref]
    bad = [t for (t, a), (_, b) in zip(ours, ref) if a != b]
    assert not bad, bad
