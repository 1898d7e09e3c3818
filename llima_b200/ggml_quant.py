"""The call surface of ``sima_lmm.gguf.ggml_quant`` on B200.

Same function names, arguments, return shapes and dtypes, assertions and warning text as
``sima_lmm/gguf/ggml_quant.py`` (sima-neat/llima 0.6.2); every decode, fold and
requantization runs in libgguf_b200.so on the current CUDA device, bit for bit equal to
the reference's numpy:

========================================  ==============================================
reference (``ggml_quant.py``)             kernel (``include/gguf_b200.h``)
========================================  ==============================================
``unpack_q8_0`` (:136-158)                ``gq_convert`` Q8_0, codes
``unpack_dequantize_q8_0`` (:161-171)     ``gq_convert`` Q8_0, f32 (d * q is exact)
``unpack_q4`` (:174-210)                  SYMMETRIC: ``gq_convert`` Q4_0; else
                                          ``gq_unpack_fields`` Q4_1
``unpack_dequantize_q4`` (:213-227)       ``gq_convert`` Q4_0 / Q4_1, f32
``unpack_q5`` (:230-271)                  SYMMETRIC: ``gq_convert`` Q5_0; else
                                          ``gq_unpack_fields`` Q5_1
``unpack_base_quant`` (:706-736)          the above (float types are copied as bytes)
``unpack_k_quant`` (:567-694)             ``gq_unpack_fields``
``remove_superblocks`` (:739-782)         ``gq_remove_superblocks``
``convert_to_simple_block_quant``         ``gq_remove_superblocks`` then
(:697-703)                                ``gq_requantize_symmetric``, on the device
``requantize_symmetric`` (:785-886)       ``gq_requantize_symmetric``
========================================  ==============================================

Inputs the kernels do not take raise instead of falling back to the CPU: in
``requantize_symmetric`` codes outside int8 or of a dtype whose product with f32 is not
f32, and ``output_bits`` outside 2..8; in ``remove_superblocks`` block constants wider
than int16 and super constants other than f16 / f32.  The reference's own pipeline
(``unpack_gguf_tensor``) stays inside these limits.
"""
from __future__ import annotations

from enum import IntEnum

import numpy as np
import torch
from ml_dtypes import bfloat16, int4, uint4

from . import _native as N
from .device import DeviceTensor, alloc_outputs
from .device import convert as _convert_device
from .gguf_conversion import requant_warning

__all__ = ["QuantizationMode", "QuantizationSymmetry", "DEFAULT_GGML_BLK_SIZE", "GGML_SUPER_SIZE",
           "unpack_q8_0", "unpack_dequantize_q8_0", "unpack_q4", "unpack_dequantize_q4", "unpack_q5",
           "unpack_base_quant", "unpack_k_quant", "remove_superblocks", "convert_to_simple_block_quant",
           "requantize_symmetric"]


class QuantizationMode(IntEnum):
    """GGML type numbers (``ggml_quant.py:9-26``)."""
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    BF16 = 30


class QuantizationSymmetry(IntEnum):
    UNQUANTIZED = -1
    SYMMETRIC = 0
    ASYMMETRIC = 1


DEFAULT_GGML_BLK_SIZE: int = 32
GGML_SUPER_SIZE: int = 256

# The names of the reference's format table (ggml_quant.py:104-131); other names raise
# the KeyError its dictionary lookup raises.
_SUPPORTED = ("F32", "F16", "BF16", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "Q4_K", "Q5_K",
              "Q6_K")
# stored unit bytes, blocks per super-block and constants per block of the K-quants
_K_GEOMETRY = {"Q2_K": (84, 16, 2), "Q3_K": (110, 16, 1), "Q4_K": (144, 8, 2), "Q5_K": (176, 8, 2),
               "Q6_K": (210, 16, 1)}
_TYPE_ID = {"Q8_0": 8, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12,
            "Q5_K": 13, "Q6_K": 14}


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise N.NativeLibraryError("the B200 ggml_quant path needs a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _raw(data, unit_bytes: int) -> tuple[np.ndarray, int]:
    """The bytes of ``data`` and the number of whole units; like the reference's
    ``np.frombuffer(...).reshape(n, unit)``, a length that is not a whole number of units
    raises ValueError."""
    raw = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    if raw.size % unit_bytes:
        raise ValueError(f"cannot reshape array of size {raw.size} into shape "
                         f"({raw.size // unit_bytes},{unit_bytes})")
    return raw, raw.size // unit_bytes


def _upload(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).copy()).to(_device())


def _convert(fmt: str, data, unit_bytes: int, mask: int):
    """Whole-tensor conversion of ``data`` as (blocks, 32): (scales, codes) or f32."""
    raw, nb = _raw(data, unit_bytes)
    t = DeviceTensor(fmt, nb, DEFAULT_GGML_BLK_SIZE, _upload(raw))
    alloc_outputs(t, mask)
    _convert_device(t, mask)
    if mask == N.OUT_F32:
        return t.values.cpu().numpy()
    return t.scales.cpu().numpy(), t.codes.cpu().numpy()


def _fields(fmt: str, data, unit_bytes: int):
    """``gq_unpack_fields``: (super / block constants f32, block constants int8 | None,
    values int8) of ``data``."""
    raw, n = _raw(data, unit_bytes)
    dev = _device()
    kq = fmt in _K_GEOMETRY
    if kq:
        _, nb, k = _K_GEOMETRY[fmt]
        sup = torch.empty((n, k), dtype=torch.float32, device=dev)
        blk = torch.empty((n, nb, k), dtype=torch.int8, device=dev)
        vals = torch.empty((n, nb, GGML_SUPER_SIZE // nb), dtype=torch.int8, device=dev)
    else:
        sup = torch.empty((n, 2), dtype=torch.float32, device=dev)
        blk = None
        vals = torch.empty((n, DEFAULT_GGML_BLK_SIZE), dtype=torch.int8, device=dev)
    if n:
        src = _upload(raw)
        N.check(N.lib().gq_unpack_fields(_TYPE_ID[fmt], src.data_ptr(), src.numel(), n, sup.data_ptr(),
                                         None if blk is None else blk.data_ptr(), vals.data_ptr(), _stream()),
                "gq_unpack_fields")
    return sup.cpu().numpy(), None if blk is None else blk.cpu().numpy(), vals.cpu().numpy()


def unpack_q8_0(data: bytes) -> tuple[np.ndarray, np.ndarray]:
    """Q8_0 -> scales f32 (nblocks, 1), codes int8 (nblocks, 32) (``ggml_quant.py:136-158``)."""
    return _convert("Q8_0", data, 34, N.OUT_CODES)


def unpack_dequantize_q8_0(data: bytes) -> np.ndarray:
    """Q8_0 -> f32 (nblocks, 32) = scale * code (``ggml_quant.py:161-171``)."""
    return _convert("Q8_0", data, 34, N.OUT_F32)


def unpack_q4(data: bytes, symmetry: QuantizationSymmetry) -> tuple[np.ndarray, np.ndarray]:
    """Q4 blocks (``ggml_quant.py:174-210``).  SYMMETRIC (Q4_0): scales f32 (nblocks, 1) and
    int4 codes n - 8; otherwise (Q4_1): constants f32 (nblocks, 2) [d, m] and uint4 codes."""
    if symmetry == QuantizationSymmetry.SYMMETRIC:
        s, w = _convert("Q4_0", data, 18, N.OUT_CODES)
        return s, w.view(np.uint8).view(int4)
    c, _, v = _fields("Q4_1", data, 20)
    return c, v.view(np.uint8).view(uint4)


def unpack_dequantize_q4(data: bytes, symmetry: QuantizationSymmetry) -> np.ndarray:
    """Q4 -> f32 (nblocks, 32): d * q, or d * q + m (``ggml_quant.py:213-227``)."""
    if symmetry == QuantizationSymmetry.SYMMETRIC:
        return _convert("Q4_0", data, 18, N.OUT_F32)
    return _convert("Q4_1", data, 20, N.OUT_F32)


def unpack_q5(data: bytes, symmetry: QuantizationSymmetry) -> tuple[np.ndarray, np.ndarray]:
    """Q5 blocks (``ggml_quant.py:230-271``).  SYMMETRIC (Q5_0): scales f32 (nblocks, 1) and
    int8 codes q - 16; otherwise (Q5_1): constants f32 (nblocks, 2) and int8 codes 0..31."""
    if symmetry == QuantizationSymmetry.SYMMETRIC:
        return _convert("Q5_0", data, 22, N.OUT_CODES)
    c, _, v = _fields("Q5_1", data, 24)
    return c, v


def unpack_base_quant(data: bytes, ggml_name: str) -> tuple[np.ndarray | None, np.ndarray]:
    """Float and base quantization types (``ggml_quant.py:706-736``)."""
    if ggml_name not in _SUPPORTED:
        raise KeyError(ggml_name)
    if ggml_name in ("F32", "F16", "BF16"):
        # float tensors are returned as a copy of their bytes, no conversion
        dtype = {"F32": np.float32, "F16": np.float16, "BF16": bfloat16}[ggml_name]
        return None, np.copy(np.frombuffer(data, dtype=dtype))
    if ggml_name == "Q8_0":
        return unpack_q8_0(data)
    if ggml_name in ("Q4_0", "Q4_1"):
        sym = QuantizationSymmetry.SYMMETRIC if ggml_name == "Q4_0" else QuantizationSymmetry.ASYMMETRIC
        return unpack_q4(data, sym)
    if ggml_name in ("Q5_0", "Q5_1"):
        sym = QuantizationSymmetry.SYMMETRIC if ggml_name == "Q5_0" else QuantizationSymmetry.ASYMMETRIC
        return unpack_q5(data, sym)
    raise ValueError(f"Quantization {ggml_name} not implemented yet.")


def unpack_k_quant(data: bytes, ggml_name: str) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """K-quant super-blocks -> (super constants f32 (N, 1|2), block constants int8
    (N, B, 1|2), values int8 (N, B, C)) with no numeric conversion (``ggml_quant.py:567-694``)."""
    assert "_K" in ggml_name
    if ggml_name not in _SUPPORTED:
        raise KeyError(ggml_name)
    if ggml_name not in _K_GEOMETRY:
        raise ValueError(f"K-quant {ggml_name} not implemented yet.")
    sup, blk, vals = _fields(ggml_name, data, _K_GEOMETRY[ggml_name][0])
    return sup, blk, vals


def _fold_inputs(superblock_constants: np.ndarray, block_constants: np.ndarray, quantized: np.ndarray):
    """The reference's checks of ``remove_superblocks`` (``ggml_quant.py:763-769``) and the
    dtypes the kernel takes."""
    assert len(superblock_constants.shape) == 2
    assert len(block_constants.shape) == 3
    assert len(quantized.shape) == 3
    assert superblock_constants.shape[0] == block_constants.shape[0] == quantized.shape[0]
    assert superblock_constants.shape[1] == block_constants.shape[2]
    assert block_constants.shape[1] == quantized.shape[1]
    assert np.issubdtype(block_constants.dtype, np.signedinteger)
    if block_constants.dtype not in (np.int8, np.int16):
        raise TypeError("remove_superblocks on the B200 path takes int8 or int16 block constants, "
                        f"not {block_constants.dtype}")
    if superblock_constants.dtype not in (np.float32, np.float16):
        raise TypeError("remove_superblocks on the B200 path takes f16 or f32 super-block constants, "
                        f"not {superblock_constants.dtype}")
    n, nb, k = block_constants.shape
    if k not in (1, 2):
        raise ValueError("block constants must have 1 or 2 columns (scale, min)")
    # an f16 super constant widens to f32 exactly; the product of an int8 / int16 with it
    # is then what numpy's own promotion computes (int8 * f16 is exact before the f16
    # rounding, int16 * f16 promotes to f32)
    return (np.ascontiguousarray(superblock_constants, dtype=np.float32),
            np.ascontiguousarray(block_constants), n, nb, k)


def _fold_device(sup: np.ndarray, blk: np.ndarray, n: int, nb: int, k: int, want_f16: bool, want_f32: bool):
    dev = _device()
    out16 = torch.empty((n * nb, k), dtype=torch.int16, device=dev) if want_f16 else None
    out32 = torch.empty((n * nb, k), dtype=torch.float32, device=dev) if want_f32 else None
    if n * nb:
        d_sup = _upload(sup)
        d_blk = _upload(blk)
        N.check(N.lib().gq_remove_superblocks(d_sup.data_ptr(), d_blk.data_ptr(), blk.dtype.itemsize, n, nb, k,
                                              None if out16 is None else out16.data_ptr(),
                                              None if out32 is None else out32.data_ptr(), _stream()),
                "gq_remove_superblocks")
    return out16, out32


def remove_superblocks(superblock_constants: np.ndarray, block_constants: np.ndarray,
                       quantized: np.ndarray) -> np.ndarray:
    """Fold super-block constants into block constants (``ggml_quant.py:739-782``): returns
    (f16 (N*M, 1|2), quantized reshaped to (N*M, B))."""
    sup, blk, n, nb, k = _fold_inputs(superblock_constants, block_constants, quantized)
    out16, _ = _fold_device(sup, blk, n, nb, k, True, False)
    block_count = n * nb
    return (out16.cpu().numpy().view(np.float16).reshape(block_count, k),
            np.reshape(quantized, (block_count, quantized.shape[2])))


def convert_to_simple_block_quant(super_constants: np.ndarray, blocks: np.ndarray,
                                  elements: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``remove_superblocks``, then for two-constant types ``requantize_symmetric(..., 8,
    int8)`` (``ggml_quant.py:697-703``); the f16 block constants stay on the device."""
    sup, blk, n, nb, k = _fold_inputs(super_constants, blocks, elements)
    _, bc = _fold_device(sup, blk, n, nb, k, False, True)
    q = np.reshape(elements, (n * nb, elements.shape[2]))
    if k == 2:
        return _requantize_device(bc, q, 8, np.int8)
    return bc.cpu().numpy(), q


def _codes_int8(quantized: np.ndarray) -> np.ndarray:
    """The codes as int8, when numpy's product with f32 stays f32 and every code fits."""
    if np.result_type(quantized.dtype, np.float32) != np.float32:
        raise TypeError(f"requantize_symmetric on the B200 path takes codes whose product with f32 is f32, "
                        f"not {quantized.dtype}")
    if quantized.dtype == np.int8:
        return quantized
    wide = quantized.astype(np.int32)
    if wide.size and (int(wide.min()) < -128 or int(wide.max()) > 127):
        raise TypeError("requantize_symmetric on the B200 path takes codes that fit in int8")
    return wide.astype(np.int8)


def _empty_error(n: int, block: int) -> ValueError:
    """The error numpy raises in the reference for an empty requantization: the block
    minimum over zero columns, or the global maximum over zero blocks."""
    which = "minimum" if block == 0 else "maximum"
    return ValueError(f"zero-size array to reduction operation {which} which has no identity")


def _requantize_device(bc: torch.Tensor, quantized: np.ndarray, output_bits: int, new_dtype):
    """requantize_symmetric on block constants already on the device."""
    n, block = quantized.shape
    if n == 0 or block == 0:
        raise _empty_error(n, block)
    if not 2 <= output_bits <= 8:
        raise ValueError(f"requantize_symmetric on the B200 path takes output_bits 2..8, not {output_bits}")
    q8 = _codes_int8(quantized)
    dev = _device()
    d_q = _upload(q8)
    out_s = torch.empty((n, 1), dtype=torch.float32, device=dev)
    out_q = torch.empty((n, block), dtype=torch.int8, device=dev)
    diag = torch.zeros(2, dtype=torch.int32, device=dev)
    N.check(N.lib().gq_requantize_symmetric(bc.data_ptr(), d_q.data_ptr(), n, block, output_bits, out_s.data_ptr(),
                                            out_q.data_ptr(), diag.data_ptr(), _stream()),
            "gq_requantize_symmetric")
    d = diag.cpu().numpy()
    requant_warning(d[0:1].view(np.float32)[0], np.int16(d[1]))
    return out_s.cpu().numpy(), out_q.cpu().numpy().astype(new_dtype, copy=False)


def requantize_symmetric(block_constants: np.ndarray, quantized: np.ndarray, output_bits: int,
                         new_dtype: np.dtype) -> tuple[np.ndarray, np.ndarray]:
    """Asymmetric (scale, min) blocks -> symmetric scale and signed codes
    (``ggml_quant.py:785-886``); logs the reference's distortion warning."""
    assert block_constants.ndim == 2
    assert block_constants.dtype == np.float32
    assert quantized.ndim == 2
    assert block_constants.shape[0] == quantized.shape[0]
    assert block_constants.shape[1] == 2
    assert np.issubdtype(new_dtype, np.signedinteger)
    if quantized.shape[0] == 0 or quantized.shape[1] == 0:
        raise _empty_error(*quantized.shape)
    return _requantize_device(_upload(block_constants), quantized, output_bits, new_dtype)

