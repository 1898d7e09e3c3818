"""GGML formats handled by the B200 path and their block geometry.

Mirrors the format table of ``sima_lmm/gguf/ggml_quant.py:104-131`` for the types on
the path, with the GGML type numbers of ``QuantizationMode`` (``ggml_quant.py:9-26``),
which are also the type ids the C ABI takes (``include/gguf_b200.h``).
"""
from __future__ import annotations

from dataclasses import dataclass

__all__ = ["Format", "FORMATS", "FORMAT_BY_ID", "output_layout"]


@dataclass(frozen=True)
class Format:
    name: str
    type_id: int        # GGML type number
    unit_values: int    # values per stored block / super-block
    unit_bytes: int     # bytes per stored block / super-block
    block_values: int   # values per output scale (0 for float types)
    asymmetric: bool    # converted through requantize_symmetric


FORMATS: dict[str, Format] = {
    "F32": Format("F32", 0, 1, 4, 0, False),
    "F16": Format("F16", 1, 1, 2, 0, False),
    "BF16": Format("BF16", 30, 1, 2, 0, False),
    "Q4_0": Format("Q4_0", 2, 32, 18, 32, False),
    "Q8_0": Format("Q8_0", 8, 32, 34, 32, False),
    "Q4_K": Format("Q4_K", 12, 256, 144, 32, True),
    "Q5_K": Format("Q5_K", 13, 256, 176, 32, True),
    "Q6_K": Format("Q6_K", 14, 256, 210, 16, False),
    "Q4_1": Format("Q4_1", 3, 32, 20, 32, True),
    "Q5_0": Format("Q5_0", 6, 32, 22, 32, False),
    "Q5_1": Format("Q5_1", 7, 32, 24, 32, True),
    "Q2_K": Format("Q2_K", 10, 256, 84, 16, True),
    "Q3_K": Format("Q3_K", 11, 256, 110, 16, False),
}
FORMAT_BY_ID = {f.type_id: f for f in FORMATS.values()}


def output_layout(fmt: str, n_values: int) -> dict:
    """Bytes the conversion writes for one tensor: codes (1 B/value), scales (f32 per
    block) and, in float mode, 4 B/value.  Float types pass through unchanged."""
    f = FORMATS[fmt]
    if f.block_values == 0:
        return {"codes": 0, "scales": 0, "values": n_values * f.unit_bytes}
    return {"codes": n_values, "scales": 4 * (n_values // f.block_values), "values": 4 * n_values}
