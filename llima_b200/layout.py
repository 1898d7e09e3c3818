"""Modalix weight layout on the GPU (``ModelGraph._build_conv``, model_graph.py:1012-1079).

After ``load_np_param`` returns (scales (O*I/B, 1), codes (O, I)), ``_build_conv`` reshapes
the scales to (O, I/B) and transposes them to (I/B, O), lays the codes out oi -> oihw ->
hwigo, i.e. (1, 1, I, 1, O), whose memory order is the (I, O) transpose, and, for int4
weights of a padded projection, pads the output channels to a uniform 32-way split with
zero weights and unit scales.  ``modalix_layout_device`` does this with one kernel pass on
device-resident outputs; ``modalix_layout`` is the numpy-in, numpy-out form.
"""
from __future__ import annotations

import numpy as np
import torch
from ml_dtypes import int4

from . import _native as N

__all__ = ["padded_output_channels", "modalix_layout_device", "modalix_layout"]

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
