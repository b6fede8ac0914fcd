"""The reference's own harness, run on the GPU with this library registered.

``scripts/run_baseline.py --impl b200_geqrf --stress`` (reference
``scripts/run_baseline.py:66-114``) draws the reference's 27 stress cases
(n in {32, 176, 512} x 9 structures, ``src/qrbench/inputs.py:84-135``) and its
7 ranked GPUMODE shapes (``src/qrbench/inputs.py:20-28``) on the device,
gates every result with the reference checker and exits 2 on any failure. The
reference tree comes from ``$QRBENCH_REFERENCE`` or the git-ignored
``baseline/_ref/gpumode_qr`` copy; without one (or without Triton, which the
reference's registry module imports) the test is skipped.
"""

from __future__ import annotations

import importlib.util
import subprocess
import sys

import pytest
from conftest import REPO, reference_checkout

pytestmark = pytest.mark.gpu
REF = reference_checkout()


@pytest.mark.skipif(REF is None, reason="reference checkout absent")
@pytest.mark.skipif(importlib.util.find_spec("triton") is None, reason="triton absent")
def test_reference_harness_stress_and_shapes_pass():
    cmd = [sys.executable, "-m", "gpumode_qr_b200.harness", "--reference", str(REF),
           "--impl", "b200_geqrf", "--stress", "--no-write", "--warmup", "3", "--iters", "5"]
    out = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stdout[-4000:] + out.stderr[-4000:]
    lines = out.stdout.splitlines()
    stress = [ln for ln in lines if ln.startswith("[stress]")]
    bench = [ln for ln in lines if ln.startswith("[bench]") and "geomean" not in ln]
    assert len(stress) == 27 and all(" PASS " in ln for ln in stress), "\n".join(stress)
    assert len(bench) == 7 and all(" PASS " in ln for ln in bench), "\n".join(bench)
    print("\n".join(bench + [ln for ln in lines if "geomean" in ln]))
