"""Modalix weight layout on the GPU (``ModelGraph._build_conv``, model_graph.py:1012-1079).

After ``load_np_param`` returns (scales (O*I/B, 1), codes (O, I)), ``_build_conv`` reshapes
the scales to (O, I/B) and transposes them to (I/B, O), lays the codes out oi -> oihw ->
hwigo, i.e. (1, 1, I, 1, O), whose memory order is the (I, O) transpose, and, for int4
weights of a padded projection, pads the output channels to a uniform 32-way split with
zero weights and unit scales.  ``modalix_layout_device`` does this with one kernel pass on
device-resident outputs; ``modalix_layout`` is the numpy-in, numpy-out form.
``convert_modalix_device`` / ``modalix_from_gguf`` fuse it with the GGUF conversion itself
(``gq_convert_modalix``): the GGUF bytes go in, the HWIGO codes and transposed scales come
out, and the row-major codes never reach memory.

Bundled projections (Phi-3.5 style ``qkv_proj`` / ``gate_up_proj``): ``_build_conv`` looks up
the bundled tensor when a ``q_proj``/``k_proj``/``v_proj``/``gate_proj``/``up_proj`` weight is
missing and keeps a range of its output rows (model_graph.py:990-998, 1168-1248).
``alternate_weight`` and ``array_partition`` give that name and row range, and
``gguf_conversion.load_partition`` decodes only those rows.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
from ml_dtypes import int4

from . import _native as N

__all__ = ["padded_output_channels", "modalix_layout_device", "modalix_layout", "convert_modalix_device",
           "modalix_from_gguf", "array_partition", "alternate_weight"]

MLA_ROW_SIZE = 16   # sima_lmm/utils.py:4


def padded_output_channels(out_channels: int, is_int4: bool, pad_output: bool = True,
                           relocatable: bool = False, quantizable: bool = False) -> int:
    """Output channel count ``_build_conv`` pads to (model_graph.py:1057-1069)."""
    split_width = ((-(-out_channels // MLA_ROW_SIZE) + 31) // 32) * MLA_ROW_SIZE
    if (pad_output and not relocatable and not quantizable and is_int4 and out_channels > 512
            and out_channels % MLA_ROW_SIZE == 0 and out_channels - 31 * split_width <= 0):
        return 32 * split_width
    return out_channels


def modalix_layout_device(scales: torch.Tensor, codes: torch.Tensor, padded: int | None = None):
    """Device tensors scales (O*I/B, 1) f32 and codes (O, I) int8/uint8 -> scales (I/B, O')
    and codes (I, O') (the HWIGO weight without its unit dimensions)."""
    out_ch, in_ch = codes.shape
    padded = out_ch if padded is None else padded
    nb = scales.numel() // out_ch
    block = in_ch // nb
    out_codes = torch.empty((in_ch, padded), dtype=codes.dtype, device=codes.device)
    out_scales = torch.empty((nb, padded), dtype=torch.float32, device=codes.device)
    N.check(N.lib().gq_modalix_layout(codes.data_ptr(), scales.data_ptr(), out_ch, in_ch, block, padded,
                                      out_codes.data_ptr(), out_scales.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream), "gq_modalix_layout")
    return out_scales, out_codes


def modalix_layout(scales: np.ndarray, codes: np.ndarray, pad_output: bool = False):
    """numpy in, numpy out: (scales (I/B, O'), weight (1, 1, I, 1, O')) as ``_build_conv``
    builds them for ``create_conv_node`` (default reshape, no process functions)."""
    is_int4 = codes.dtype == int4
    out_ch = codes.shape[0]
    padded = padded_output_channels(out_ch, is_int4, pad_output)
    c = torch.from_numpy(np.ascontiguousarray(codes).view(np.uint8 if is_int4 else np.int8)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(scales, dtype=np.float32)).cuda()
    out_s, out_c = modalix_layout_device(s, c, padded)
    w = out_c.cpu().numpy()
    w = w.view(int4) if is_int4 else w
    return out_s.cpu().numpy(), w.reshape(1, 1, codes.shape[1], 1, padded)


def convert_modalix_device(fmt: str, src: torch.Tensor, rows: int, cols: int, heads: int = 0,
                           padded: int | None = None):
    """GGUF bytes on the GPU -> (scales (cols/B, O') f32, codes (cols, O') int8 or int4 bytes,
    diagnostics (2,) int32) in the Modalix layout, O' = ``padded`` (default ``rows``),
    with the llama q/k permutation of ``heads`` heads when ``heads > 0``.

    One pass (``gq_convert_modalix``) when the shape allows it (cols a multiple of 256,
    rows of whole 16-byte chunks); otherwise the conversion and ``gq_modalix_layout`` run
    one after the other on the GPU, with the same result."""
    from .formats import FORMATS
    f = FORMATS[fmt]
    if f.block_values == 0:
        raise TypeError("the Modalix layout writer takes quantized GGUF types")
    dev = src.device
    padded = rows if padded is None else padded
    out_codes = torch.empty((cols, padded), dtype=torch.int8, device=dev)
    out_scales = torch.empty((cols // f.block_values, padded), dtype=torch.float32, device=dev)
    diag = torch.zeros(2, dtype=torch.int32, device=dev)
    rec = N.Tensor()
    rec.type, rec.perm_heads, rec.rows, rec.cols = f.type_id, heads, rows, cols
    rec.src, rec.src_bytes = src.data_ptr(), src.numel()
    rec.codes, rec.scales, rec.diag = out_codes.data_ptr(), out_scales.data_ptr(), diag.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    st = N.lib().gq_convert_modalix(ctypes.byref(rec), padded, stream)
    if st == -2:
        # a shape the fused writer does not take (or a bad size, which the conversion then
        # reports): convert, then lay out
        from .device import DeviceTensor, alloc_outputs, convert
        t = alloc_outputs(DeviceTensor(fmt, rows, cols, src, heads), N.OUT_CODES)
        convert(t, N.OUT_CODES)
        s, c = modalix_layout_device(t.scales, t.codes, padded)
        return s, c, t.diag
    N.check(st, "gq_convert_modalix")
    return out_scales, out_codes, diag


def modalix_from_gguf(gguf_tensor, heads: int = 0, pad_output: bool = False):
    """A GGUF reader tensor -> (scales (I/B, O'), weight (1, 1, I, 1, O')) as
    ``_build_conv`` hands them to ``create_conv_node`` (default reshape, no process
    functions), O' the int4 32-way padding when ``pad_output``; the requantization warning
    is logged as the conversion logs it."""
    from .gguf_conversion import _type_name, requant_warning
    fmt = _type_name(gguf_tensor.tensor_type)
    rows, cols = (int(x) for x in gguf_tensor.shape[::-1])
    is_int4 = fmt == "Q4_0"
    padded = padded_output_channels(rows, is_int4, pad_output)
    src = torch.from_numpy(np.ascontiguousarray(gguf_tensor.data).reshape(-1).view(np.uint8)).cuda()
    s, c, d = convert_modalix_device(fmt, src, rows, cols, heads, padded)
    w = c.cpu().numpy()
    w = w.view(np.uint8).view(int4) if is_int4 else w
    from .formats import FORMATS
    if FORMATS[fmt].asymmetric:
        dv = d.cpu().numpy()
        requant_warning(dv[0:1].view(np.float32)[0], np.int16(dv[1]))
    return s.cpu().numpy(), w.reshape(1, 1, cols, 1, padded)


def array_partition(rows: int, count: int, index: int, span: int) -> tuple[int, int]:
    """Rows [r0, r1) of an array with `rows` rows along axis 0 that
    ``ModelGraph._get_array_partition(count, index, span)`` keeps (model_graph.py:1168-1195):
    the rows split into `count` equal parts (AssertionError otherwise) and `span` parts
    from part `index` are kept, with numpy's slice clamping."""
    assert rows % count == 0
    element = rows // count
    r0 = min(element * index, rows)
    return r0, min(element * index + element * span, rows)


def alternate_weight(weight_name: str, q_size: int | None, kv_size: int | None) -> tuple[str, int, int, int]:
    """``ModelGraph._find_alternate_weight`` (model_graph.py:1197-1248) as data: the bundled
    tensor name and the (count, index, span) of the partition that selects `weight_name`."""
    proj = weight_name.replace(".weight", "").split(".")[-1]
    if proj in ("q_proj", "k_proj", "v_proj"):
        assert q_size is not None
        assert kv_size is not None
        fused = weight_name.replace(proj, "qkv_proj")
    elif proj in ("gate_proj", "up_proj"):
        fused = weight_name.replace(proj, "gate_up_proj")
    else:
        raise NotImplementedError(f"{proj} not found in weight map.")
    if proj == "q_proj":
        part = (q_size + 2 * kv_size, 0, q_size)
    elif proj == "k_proj":
        part = (q_size + 2 * kv_size, q_size, kv_size)
    elif proj == "v_proj":
        part = (q_size + 2 * kv_size, q_size + kv_size, kv_size)
    elif proj == "gate_proj":
        part = (2, 0, 1)
    else:
        part = (2, 1, 1)
    return (fused, *part)
