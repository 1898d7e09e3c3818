"""Modalix weight layout on the GPU (``ModelGraph._build_conv``, model_graph.py:1012-1079).

After ``load_np_param`` returns (scales (O*I/B, 1), codes (O, I)), ``_build_conv`` reshapes
the scales to (O, I/B) and transposes them to (I/B, O), lays the codes out oi -> oihw ->
hwigo, i.e. (1, 1, I, 1, O), whose memory order is the (I, O) transpose, and, for int4
weights of a padded projection, pads the output channels to a uniform 32-way split with
zero weights and unit scales.  ``modalix_layout_device`` does this with one kernel pass on
device-resident outputs; ``modalix_layout`` is the numpy-in, numpy-out form.

Bundled projections (Phi-3.5 style ``qkv_proj`` / ``gate_up_proj``): ``_build_conv`` looks up
the bundled tensor when a ``q_proj``/``k_proj``/``v_proj``/``gate_proj``/``up_proj`` weight is
missing and keeps a range of its output rows (model_graph.py:990-998, 1168-1248).
``alternate_weight`` and ``array_partition`` give that name and row range, and
``gguf_conversion.load_partition`` decodes only those rows.
"""
from __future__ import annotations

import numpy as np
import torch
from ml_dtypes import int4

from . import _native as N

__all__ = ["padded_output_channels", "modalix_layout_device", "modalix_layout", "array_partition",
           "alternate_weight"]

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
