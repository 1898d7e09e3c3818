"""The conversion kernels' waits on their tile copies end.

Every tile copy is waited for on an mbarrier with a limit of about a second of global
time; past it the kernel records GQ_KERNEL_WAIT_TIMEOUT and stops instead of spinning.  A
copy that never completes cannot be made on purpose, so the wait itself is tested: a test
kernel (tests/cuda/wait_timeout.cu, built here with nvcc from the library's own device
header) waits on a phase that nothing completes and must come back false after the limit.
"""
import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

from llima_b200 import _native as N
from llima_b200.build import ARCH, CSRC

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def test_wait_on_a_copy_that_never_completes_gives_up(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    so = tmp_path / "libwait.so"
    cmd = [nvcc, *ARCH, "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", f"-I{CSRC}",
           f"-I{ROOT / 'include'}", "-o", str(so), str(ROOT / "tests" / "cuda" / "wait_timeout.cu")]
    subprocess.run(cmd, check=True, capture_output=True)
    lib = ctypes.CDLL(str(so))
    status, waited = ctypes.c_int(-1), ctypes.c_ulonglong(0)
    assert lib.run_wait_never(ctypes.byref(status), ctypes.byref(waited)) == 0
    assert status.value == 0                        # the wait gave up
    assert 0.9e9 <= waited.value <= 5e9             # after about its one-second limit


def test_kernel_error_flags_stay_clear_after_conversions():
    import torch
    from llima_b200.device import DeviceTensor, alloc_outputs, convert
    from llima_b200.synth import gen_tensor_bytes
    for fmt in ("Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0"):
        raw = gen_tensor_bytes(fmt, 64 * 1024, 11)
        t = DeviceTensor(fmt, 64, 1024, torch.from_numpy(raw.copy()).cuda())
        convert(alloc_outputs(t, N.OUT_CODES), N.OUT_CODES)
    torch.cuda.synchronize()
    flags = ctypes.c_uint32(7)
    N.check(N.lib().gq_kernel_errors(0, 1, ctypes.byref(flags)), "gq_kernel_errors")
    assert flags.value == 0
