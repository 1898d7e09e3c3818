"""The allocation-free host conversion, gq_convert_host_noalloc.

Callers that must not allocate device memory while they prepare weights (their device
memory already belongs to another allocator, where cudaMalloc can fail or stall the device)
use gq_convert_host_noalloc, which stages everything in a fixed array inside the library.
These tests call it through the C ABI and compare its results bit for bit with the
session-based gq_convert_host, on two calls in a row with different inputs, so that
anything the shared array keeps from the first call would show up in the second.

This file is collected last on purpose: a run that stops at the first failure has then
already run every other test.  It also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from llima_b200 import _native as N
from llima_b200.formats import FORMATS
from llima_b200.synth import gen_tensor_bytes

pytestmark = pytest.mark.gpu

# (format, rows, cols, heads): the Q4_K 4096x4096 tensors need more staging than the
# fixed array has, so they are converted in pieces (the permuted one in whole heads)
SPECS = [("Q4_K", 4096, 4096, 0), ("Q4_K", 4096, 4096, 32), ("Q4_K", 1024, 4096, 8),
         ("Q6_K", 1024, 4096, 0), ("Q5_K", 256, 2048, 0), ("Q8_0", 512, 4096, 0),
         ("Q4_0", 256, 1024, 0), ("F32", 4096, 1, 0), ("F32", 1024, 1, 8)]


class HostSet:
    """Host buffers and C records of one set of tensors."""

    def __init__(self, seed: int, out_mask: int):
        self.arrays = []
        self.records = (N.Tensor * len(SPECS))()
        for i, (fmt, rows, cols, heads) in enumerate(SPECS):
            f = FORMATS[fmt]
            src = gen_tensor_bytes(fmt, rows * cols, seed * 100 + i, "bias")
            r = N.Tensor()
            r.type, r.perm_heads, r.rows, r.cols = f.type_id, heads, rows, cols
            r.src, r.src_bytes = src.ctypes.data, src.size
            bufs = {"src": src}
            if f.block_values == 0:
                bufs["values"] = np.empty(rows * cols, dtype=np.float32)
            else:
                if out_mask & N.OUT_CODES:
                    bufs["codes"] = np.empty(rows * cols, dtype=np.int8)
                    bufs["scales"] = np.empty(rows * cols // f.block_values, dtype=np.float32)
                if out_mask & N.OUT_F32:
                    bufs["values"] = np.empty(rows * cols, dtype=np.float32)
            for name in ("codes", "scales", "values"):
                if name in bufs:
                    setattr(r, name, bufs[name].ctypes.data)
            self.records[i] = r
            self.arrays.append(bufs)
        self.diags = (N.Diag * len(SPECS))()

    def outputs(self):
        out = []
        for bufs in self.arrays:
            out.append({k: v.copy() for k, v in bufs.items() if k != "src"})
        return out, [(d.round_err_bits, d.clip_err) for d in self.diags]


def _session_result(seed: int, out_mask: int):
    lib = N.lib()
    hs = HostSet(seed, out_mask)
    sess = ctypes.c_void_p()
    N.check(lib.gq_session_create(0, 256 << 20, ctypes.byref(sess)), "gq_session_create")
    try:
        N.check(lib.gq_convert_host(sess, hs.records, len(SPECS), out_mask, hs.diags), "gq_convert_host")
    finally:
        lib.gq_session_destroy(sess)
    return hs.outputs()


def _noalloc_result(seed: int, out_mask: int):
    hs = HostSet(seed, out_mask)
    N.check(N.lib().gq_convert_host_noalloc(0, hs.records, len(SPECS), out_mask, hs.diags, None),
            "gq_convert_host_noalloc")
    return hs.outputs()


@pytest.mark.parametrize("out_mask", [N.OUT_CODES, N.OUT_CODES | N.OUT_F32])
def test_noalloc_matches_session_on_two_calls(out_mask):
    want = {seed: _session_result(seed, out_mask) for seed in (1, 2)}
    for seed in (1, 2):   # two calls in a row, different inputs
        got = _noalloc_result(seed, out_mask)
        (w_out, w_diag), (g_out, g_diag) = want[seed], got
        assert g_diag == w_diag
        for spec, a, b in zip(SPECS, w_out, g_out):
            assert a.keys() == b.keys()
            for name in a:
                assert np.array_equal(a[name].view(np.uint8), b[name].view(np.uint8)), (seed, spec, name)


def test_noalloc_rejects_requests_beyond_its_array():
    lib = N.lib()
    # more tensors than the diagnostics area holds
    many = (N.Tensor * 8193)()
    diags = (N.Diag * 8193)()
    assert lib.gq_convert_host_noalloc(0, many, 8193, N.OUT_CODES, diags, None) == -2
    # a permuted tensor whose single head (128 rows of 1024 super-blocks) exceeds the array
    rows, cols = 128, 1024 * 256
    src = np.zeros(rows * cols // 256 * 144, dtype=np.uint8)
    codes = np.zeros(rows * cols, dtype=np.int8)
    scales = np.zeros(rows * cols // 32, dtype=np.float32)
    t = N.Tensor()
    t.type, t.perm_heads, t.rows, t.cols = 12, 1, rows, cols
    t.src, t.src_bytes = src.ctypes.data, src.size
    t.codes, t.scales = codes.ctypes.data, scales.ctypes.data
    assert lib.gq_convert_host_noalloc(0, ctypes.byref(t), 1, N.OUT_CODES, None, None) == -2
    # the same tensor unpermuted is split into pieces and converts
    t.perm_heads = 0
    assert lib.gq_convert_host_noalloc(0, ctypes.byref(t), 1, N.OUT_CODES, None, None) == 0
    assert not codes.any() and not scales.any()


def test_noalloc_warm_up_call_and_a_user_stream():
    import torch
    lib = N.lib()
    # a call with no tensors loads the library's device code and reserves the array, and
    # converts nothing (the warm-up a caller makes before handing memory to another allocator)
    assert lib.gq_convert_host_noalloc(0, None, 0, N.OUT_CODES, None, None) == 0
    want = _session_result(3, N.OUT_CODES)
    dev_before = torch.cuda.current_device()
    stream = torch.cuda.Stream(device=0)
    for _ in range(2):
        hs = HostSet(3, N.OUT_CODES)
        N.check(lib.gq_convert_host_noalloc(0, hs.records, len(SPECS), N.OUT_CODES, hs.diags,
                                            ctypes.c_void_p(stream.cuda_stream)), "gq_convert_host_noalloc")
        got = hs.outputs()
        assert got[1] == want[1]
        for spec, a, b in zip(SPECS, want[0], got[0]):
            for name in a:
                assert np.array_equal(a[name].view(np.uint8), b[name].view(np.uint8)), (spec, name)
    # the call leaves the caller's current device as it found it
    assert torch.cuda.current_device() == dev_before
