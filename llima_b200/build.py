"""Build libgguf_b200.so in-tree with nvcc for sm_100a.

    python -m llima_b200.build            # or: python llima_b200/build.py

The library is compiled without --use_fast_math and with -fmad=false: the conversion
must reproduce numpy's separately rounded f32 operations bit for bit.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libgguf_b200.so"
SOURCES = ["gq_kernels.cu", "gq_embed.cu", "gq_layout.cu", "gq_fields.cu", "gq_api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgguf_b200.so")
    return cand


def flags(verbose_ptxas: bool = False) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "--expt-relaxed-constexpr",
                "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-cudart", "static",
                f"-I{PKG.parent / 'include'}"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [PKG.parent / "include" / "gguf_b200.h"]
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if LIB.stat().st_mtime >= newest:
            return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *flags(verbose_ptxas), "-shared", "-o", str(tmp), *map(str, srcs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
