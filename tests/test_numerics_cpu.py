"""CPU proofs of numerical shortcuts the kernels take (exhaustive over their domains)."""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_block_scale_division_by_small_integers_is_exact(tmp_path):
    # gq_device.cuh divides f16-derived block scales by integer scale factors 1..16 with a
    # reciprocal and one fma correction; this checks it equals IEEE division everywhere.
    exe = tmp_path / "div_check"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", str(exe),
                    str(HERE / "numerics" / "div_by_small_int.c"), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    assert "mismatches 0" in out.stdout
