"""Generate tests/golden/legacy_scenario.bin from the reference's own compat
layer (src/compat/compat.cpp).

The reference hides its legacy virtual_npu_* / vgpu_npu_* / sherlock_*
symbols in its shared library, so tests/compat/legacy_scenario.c is linked
against its static archive (``make -C oracle ref REF=<reference checkout>``
-> oracle/_ref/libvnpu_ref.a) and compiled against the reference's headers.
VNPU_THREADS=4 and VNPU_FORCE_ISA=avx2 fix the reference device whose GEMM
rounding the B200 library reproduces.

    python tests/golden/make_legacy_golden.py
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_ARCHIVE = os.path.join(ROOT, "oracle", "_ref", "libvnpu_ref.a")
SCENARIO = os.path.join(ROOT, "tests", "compat", "legacy_scenario.c")
ENV = {"VNPU_THREADS": "4", "VNPU_FORCE_ISA": "avx2"}


def run_reference(out_path: str, reference_dir: str) -> None:
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "legacy_ref")
        subprocess.run(["gcc", "-O1", "-I", os.path.join(reference_dir, "include"), SCENARIO,
                        REF_ARCHIVE, "-lstdc++", "-lpthread", "-lm", "-o", exe], check=True)
        subprocess.run([exe, out_path], check=True, env={**os.environ, **ENV}, timeout=300)


def main():
    ref = os.environ.get("VNPU_REFERENCE_DIR", "")
    if not ref:
        sys.exit("set VNPU_REFERENCE_DIR to the reference checkout")
    if not os.path.exists(REF_ARCHIVE):
        sys.exit("build the reference first: make -C oracle ref REF=" + ref)
    out = os.path.join(HERE, "legacy_scenario.bin")
    run_reference(out, ref)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
