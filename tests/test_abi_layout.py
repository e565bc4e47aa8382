"""The restated ABI header must match the engine's structure layouts byte for
byte (golden dump produced from backend/include/compute_backend.h and
backend/core/llm_internal.h by oracle/abi_offsets.c)."""
import os
import subprocess
import tempfile

from tests.conftest import ROOT


def test_abi_offsets_match_engine():
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "abi")
        subprocess.run(["gcc", "-std=c17", "-DFYB_MIRROR", "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "oracle", "abi_offsets.c"), "-o", exe], check=True)
        mine = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    golden = open(os.path.join(ROOT, "tests", "golden", "abi_offsets_ref.txt")).read()
    assert mine == golden
