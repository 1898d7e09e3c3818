"""The C ABI from C: tests/c/abi_smoke.c is compiled with gcc as C99 against
include/gguf_b200.h, linked to libgguf_b200.so and run.  It calls only entry points that
need no GPU (sizes, status codes, argument checks), so it runs on CPU-only hosts."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_c_program_builds_and_runs_against_the_header(tmp_path):
    gcc = shutil.which("gcc")
    lib = ROOT / "llima_b200" / "lib" / "libgguf_b200.so"
    if gcc is None or not lib.exists():
        pytest.skip("gcc or the built library is missing")
    exe = tmp_path / "abi_smoke"
    cmd = [gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "c" / "abi_smoke.c"),
           f"-L{lib.parent}", "-lgguf_b200", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "abi_smoke: ok" in r.stdout
