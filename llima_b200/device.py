"""Device-resident API: convert GGUF tensors that already sit in GPU memory.

PyTorch provides the device memory and the stream; the conversion itself is the
libgguf_b200.so kernels reached through the C ABI (``include/gguf_b200.h``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _native as N
from .formats import FORMATS

__all__ = ["DeviceTensor", "DeviceBatch", "alloc_outputs", "convert", "diag_values"]


@dataclass
class DeviceTensor:
    """One tensor's device buffers.  ``src`` holds the GGUF bytes (uint8, 16-byte aligned);
    the outputs are allocated by ``alloc_outputs`` for the requested modes."""
    fmt: str
    rows: int
    cols: int
    src: torch.Tensor
    perm_heads: int = 0
    codes: torch.Tensor | None = None    # (rows, cols) int8 (uint8 storage of int4 for Q4_0)
    scales: torch.Tensor | None = None   # (n_blocks, 1) float32
    values: torch.Tensor | None = None   # (rows, cols) float32 (or the float type itself)
    name: str = ""
    diag: torch.Tensor | None = None     # (2,) int32 diagnostics record after ``convert``

    @property
    def n_values(self) -> int:
        return self.rows * self.cols

    @property
    def src_bytes(self) -> int:
        f = FORMATS[self.fmt]
        return self.n_values // f.unit_values * f.unit_bytes

    @property
    def out_bytes(self) -> int:
        n = 0
        for t in (self.codes, self.scales, self.values):
            if t is not None:
                n += t.numel() * t.element_size()
        return n


def alloc_outputs(t: DeviceTensor, out_mask: int = N.OUT_CODES) -> DeviceTensor:
    f = FORMATS[t.fmt]
    dev = t.src.device
    if f.block_values == 0:
        dtype = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}[t.fmt]
        t.values = torch.empty((t.rows, t.cols), dtype=dtype, device=dev)
        return t
    if out_mask & N.OUT_CODES:
        t.codes = torch.empty((t.rows, t.cols), dtype=torch.int8, device=dev)
        t.scales = torch.empty((t.n_values // f.block_values, 1), dtype=torch.float32, device=dev)
    if out_mask & N.OUT_F32:
        t.values = torch.empty((t.rows, t.cols), dtype=torch.float32, device=dev)
    return t


def _ptr(x):
    return None if x is None else x.data_ptr()


def _record(t: DeviceTensor, diag_ptr) -> N.Tensor:
    f = FORMATS[t.fmt]
    if t.src.dtype != torch.uint8 or not t.src.is_cuda:
        raise TypeError("src must be a CUDA uint8 tensor of GGUF bytes")
    if t.src.numel() < t.src_bytes:
        raise ValueError(f"{t.name or t.fmt}: src holds {t.src.numel()} bytes, needs {t.src_bytes}")
    r = N.Tensor()
    r.type = f.type_id
    r.perm_heads = t.perm_heads
    r.rows = t.rows
    r.cols = t.cols
    r.src = t.src.data_ptr()
    r.src_bytes = t.src.numel()
    r.codes = _ptr(t.codes)
    r.scales = _ptr(t.scales)
    r.values = _ptr(t.values)
    r.diag = diag_ptr
    return r


@dataclass
class DeviceBatch:
    """A fixed list of device tensors converted with one C call (one kernel launch per
    GGML type present).  The ctypes records are built once, so repeated ``run`` calls
    cost only the launches."""
    tensors: list[DeviceTensor]
    out_mask: int = N.OUT_CODES
    diags: torch.Tensor = field(init=False)
    _records: ctypes.Array = field(init=False)

    def __post_init__(self):
        dev = self.tensors[0].src.device if self.tensors else torch.device("cuda")
        self.diags = torch.zeros((max(1, len(self.tensors)), 2), dtype=torch.int32, device=dev)
        arr = (N.Tensor * max(1, len(self.tensors)))()
        stride = self.diags.stride(0) * self.diags.element_size()
        for i, t in enumerate(self.tensors):
            arr[i] = _record(t, self.diags.data_ptr() + i * stride)
        self._records = arr

    def run(self, stream: torch.cuda.Stream | None = None, reset_diag: bool = True) -> None:
        lib = N.lib()
        s = (stream or torch.cuda.current_stream()).cuda_stream
        if reset_diag:
            N.check(lib.gq_diag_reset(self.diags.data_ptr(), len(self.tensors), s), "gq_diag_reset")
        N.check(lib.gq_convert_batch(self._records, len(self.tensors), self.out_mask, s), "gq_convert_batch")


def convert(t: DeviceTensor, out_mask: int = N.OUT_CODES, stream=None) -> DeviceTensor:
    """Convert one device tensor (allocating its outputs when missing)."""
    if t.codes is None and t.values is None:
        alloc_outputs(t, out_mask)
    b = DeviceBatch([t], out_mask)
    b.run(stream)
    t.diag = b.diags[0]
    return t


def diag_values(row: torch.Tensor) -> tuple[np.float32, np.int16]:
    """(round_error, clip_error) of one diagnostics record, as the reference computes them."""
    v = np.ascontiguousarray(row.detach().cpu().numpy().astype(np.int32))
    return v[0:1].view(np.float32)[0], np.int16(v[1])
