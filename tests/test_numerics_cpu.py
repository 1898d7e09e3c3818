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


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_f16_quotient_is_exact(tmp_path):
    # gq_device.cuh divides the f16-valued block constants (r = M / S) with a reciprocal
    # approximation, its exact residual and one fma; this checks every finite f16 pair for
    # every reciprocal within 2 ulp.
    exe = tmp_path / "f16_quotient"
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-o", str(exe), str(HERE / "numerics" / "f16_quotient.c"), "-lm"]
    if subprocess.run(["gcc", "-fopenmp", "-x", "c", "-", "-o", str(tmp_path / "omp")], input="int main(){return 0;}",
                      capture_output=True, text=True).returncode == 0:
        cmd.insert(1, "-fopenmp")
    subprocess.run(cmd, check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    assert "mismatches 0" in out.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_invariant_divisor_parameters(tmp_path):
    # the q/k head permutation divides unit and row indices by multiply-high and shifts
    exe = tmp_path / "fast_div"
    root = HERE.parent
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(root / "llima_b200" / "csrc"), "-o", str(exe),
                    str(HERE / "numerics" / "fast_div.cpp")], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    assert "mismatches 0" in out.stdout


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_scale_factor_quotient_keeps_floor_and_threshold(tmp_path):
    # gq_device.cuh's requant_fast finds sf0 = min(16, -128/lo, 127/hi) by Markstein's
    # division from a reciprocal approximation; this checks, for every denominator the fast
    # path can reach and every reciprocal within 2 ulp, that its floor and its comparison
    # with 0.98 equal the IEEE quotient's (the rare path recomputes the quotient itself).
    exe = tmp_path / "scale_factor_quotient"
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-o", str(exe),
           str(HERE / "numerics" / "scale_factor_quotient.c"), "-lm"]
    if subprocess.run(["gcc", "-fopenmp", "-x", "c", "-", "-o", str(tmp_path / "omp")], input="int main(){return 0;}",
                      capture_output=True, text=True).returncode == 0:
        cmd.insert(1, "-fopenmp")
    subprocess.run(cmd, check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    assert out.stdout.count("violations 0") == 2


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_packed_lane_requantization_is_exact(tmp_path):
    # gq_kernels.cu (process_k45) computes Q4_K / Q5_K codes with an integer scale factor as
    # q * sfi + rm in 16-bit lanes of the unshifted code words, the odd bytes by multiply-high,
    # gathered by a byte permute; this checks every scale factor, offset and pair of codes
    # sharing an operation against int8(q * sfi + rm), and the Q5_K code bytes (fifth bits
    # merged by multiply-add) against nibble | bit << 4 for every qs / qh byte pair.
    exe = tmp_path / "lane_requant"
    subprocess.run(["gcc", "-O2", "-o", str(exe), str(HERE / "numerics" / "lane_requant.c")], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    assert "mismatches 0" in out.stdout
