"""Token embeddings for the runtime: GGUF rows -> (int8 codes, bf16 row scales) on B200.

Mirrors, on the GPU:

* ``quantize_embedding_rows(embeddings)`` (``sima_lmm/model/language_model.py:38-54``):
  f32 (vocab, hidden) -> int8 (vocab, hidden) and bf16 (vocab, 1) absmax row scales;
* the GGUF branch of ``LanguageModel.get_embeddings_tensor`` (``language_model.py:578-611``):
  force_float dequantize, ``* embed_scale``, bf16 round, then the row quantization (or,
  without quantization, the bf16-rounded f32 values), fused in one kernel so the f32
  embedding never reaches HBM.

The reference delegates the row rule to ``afe.ir.quantization_conv.
block_quantize_weight_tensor`` (SiMa Palette SDK), which is not available; the kernel
follows the restated rule step = absmax/127, q = clip(rint(x/step), -127, 127), which the
reference's own contract test (``test_embedding_quantization.py:142-150``) accepts.
"""
from __future__ import annotations

import numpy as np
import torch
from ml_dtypes import bfloat16

from . import _native as N
from .formats import FORMATS

__all__ = ["quantize_embedding_rows", "embedding_rows_device", "embeddings_from_gguf"]


def _stream():
    return torch.cuda.current_stream().cuda_stream


def embedding_rows_device(fmt: str, src: torch.Tensor, rows: int, cols: int, embed_scale: float = 1.0,
                          quantize: bool = True):
    """GGUF bytes already on the GPU -> (codes int8, scales bf16 as uint16) or f32 values."""
    f = FORMATS[fmt]
    dev = src.device
    if quantize:
        codes = torch.empty((rows, cols), dtype=torch.int8, device=dev)
        scales = torch.empty((rows, 1), dtype=torch.uint16, device=dev)
        N.check(N.lib().gq_embedding_rows(f.type_id, src.data_ptr(), src.numel(), rows, cols, float(embed_scale),
                                          1, codes.data_ptr(), scales.data_ptr(), None, _stream()),
                "gq_embedding_rows")
        return codes, scales
    values = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    N.check(N.lib().gq_embedding_rows(f.type_id, src.data_ptr(), src.numel(), rows, cols, float(embed_scale),
                                      0, None, None, values.data_ptr(), _stream()), "gq_embedding_rows")
    return values


def quantize_embedding_rows(embeddings: np.ndarray):
    """Same inputs and outputs as ``sima_lmm.model.language_model.quantize_embedding_rows``."""
    assert embeddings.ndim == 2
    x = torch.from_numpy(np.ascontiguousarray(embeddings, dtype=np.float32)).cuda()
    rows, cols = x.shape
    codes = torch.empty((rows, cols), dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, 1), dtype=torch.uint16, device=x.device)
    N.check(N.lib().gq_quantize_rows(x.data_ptr(), rows, cols, codes.data_ptr(), scales.data_ptr(), _stream()),
            "gq_quantize_rows")
    return codes.cpu().numpy(), scales.cpu().numpy().view(bfloat16)


def embeddings_from_gguf(gguf_tensor, embed_scale: float = 1.0, quantize: bool = True):
    """``get_embeddings_tensor``'s GGUF branch for one reader tensor: (codes, bf16 scales)
    when quantizing, else (bf16-rounded f32 values, None)."""
    from .gguf_conversion import _type_name
    fmt = _type_name(gguf_tensor.tensor_type)
    rows, cols = (int(x) for x in gguf_tensor.shape[::-1])
    src = torch.from_numpy(np.ascontiguousarray(gguf_tensor.data).reshape(-1).view(np.uint8)).cuda()
    out = embedding_rows_device(fmt, src, rows, cols, embed_scale, quantize)
    if quantize:
        codes, scales = out
        return codes.cpu().numpy(), scales.cpu().numpy().view(bfloat16)
    return out.cpu().numpy(), None
