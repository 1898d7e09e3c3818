"""numpy restatement of LLiMa's GGUF block decode and requantization.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): this is the checker the CUDA
kernels are compared against, never the thing measured or shipped.

Every function restates one piece of the reference (sima-neat/llima 0.6.2) and cites
the file:line it follows.  The arithmetic is kept in the same precision and order as
the reference so that results are bit-identical:

* block constants of K-quants are ``f16(f32(int) * f32(f16))`` (one f32 product, then
  round-to-nearest-even to f16), ``sima_lmm/gguf/ggml_quant.py:771-777``;
* ``requantize_symmetric`` works in f32 throughout, ``ggml_quant.py:785-886``;
* float -> int16 casts are numpy's own, as in the reference (on x86-64 through int32;
  NaN and out-of-range values become 0), which matters only for non-finite values.

Pinning: ``tests/golden/make_golden.py`` runs the reference functions themselves on
seeded inputs and commits their outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against those files and against
the reference's own known-answer tests (``tests/compilation/unit/test_quantization.py``
and ``test_ggml_kquant_equivalence.py`` in the reference).

The force_float path of the reference calls gguf-py's ``dequantize``
(``sima_lmm/gguf/gguf_conversion.py:171-172``).  gguf-py is a third-party dependency
(pinned 0.17.1 in ``pyproject_metadata.py:146``; 0.19.0 is the version present in
this image) whose source is not part of the reference tree.  ``gguf_dequantize``
below restates its published per-format formulas (gguf-py ``quants.py``:
``Q8_0.dequantize_blocks``, ``Q4_0.dequantize_blocks``, ``Q4_K.dequantize_blocks``,
``Q5_K.dequantize_blocks``, ``Q6_K.dequantize_blocks``) and is pinned against the
installed gguf-py by the golden files.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass

import numpy as np
from ml_dtypes import bfloat16, int4

# Logger name of the reference module, so the warning text lands where the reference's does.
_log = logging.getLogger("sima_lmm.gguf.ggml_quant")

QK_K = 256


@dataclass(frozen=True)
class Format:
    """Block geometry of one GGML type (``ggml_quant.py:104-131``)."""
    name: str
    type_id: int          # GGML type number (``ggml_quant.py:9-26``)
    unit_values: int      # values per stored unit (block or super-block)
    unit_bytes: int       # bytes per stored unit
    block_values: int     # values per output scale after conversion (0: float type)
    n_constants: int      # 1 = symmetric, 2 = asymmetric (scale, min)


FORMATS: dict[str, Format] = {
    "F32": Format("F32", 0, 1, 4, 0, 0),
    "F16": Format("F16", 1, 1, 2, 0, 0),
    "BF16": Format("BF16", 30, 1, 2, 0, 0),
    "Q8_0": Format("Q8_0", 8, 32, 34, 32, 1),
    "Q4_0": Format("Q4_0", 2, 32, 18, 32, 1),
    "Q4_K": Format("Q4_K", 12, 256, 144, 32, 2),
    "Q5_K": Format("Q5_K", 13, 256, 176, 32, 2),
    "Q6_K": Format("Q6_K", 14, 256, 210, 16, 1),
    "Q4_1": Format("Q4_1", 3, 32, 20, 32, 2),
    "Q5_0": Format("Q5_0", 6, 32, 22, 32, 1),
    "Q5_1": Format("Q5_1", 7, 32, 24, 32, 2),
    "Q2_K": Format("Q2_K", 10, 256, 84, 16, 2),
    "Q3_K": Format("Q3_K", 11, 256, 110, 16, 1),
}
FORMAT_BY_ID = {f.type_id: f for f in FORMATS.values()}


def _units(data, fmt: Format) -> np.ndarray:
    """View raw tensor bytes as (n_units, unit_bytes) uint8."""
    raw = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8) if not isinstance(data, np.ndarray) \
        else np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    n = raw.size // fmt.unit_bytes
    return raw[: n * fmt.unit_bytes].reshape(n, fmt.unit_bytes)


def _f16_field(units: np.ndarray, offset: int) -> np.ndarray:
    """f16 stored little-endian at byte ``offset`` of each unit, widened to f32 (exact)."""
    if offset % 2 == 0 and units.shape[1] % 2 == 0 and units.flags.c_contiguous:
        return units.view(np.float16)[:, offset // 2].astype(np.float32)
    return np.ascontiguousarray(units[:, offset:offset + 2]).view(np.float16)[:, 0].astype(np.float32)


# ---------------------------------------------------------------------------
# Simple block formats
# ---------------------------------------------------------------------------

def unpack_q8_0(data) -> tuple[np.ndarray, np.ndarray]:
    """Q8_0: scale = f32(d); codes = the 32 int8 bytes.  ``ggml_quant.py:136-158``."""
    u = _units(data, FORMATS["Q8_0"])
    scales = _f16_field(u, 0).reshape(-1, 1)
    codes = np.ascontiguousarray(u[:, 2:34]).view(np.int8)
    return scales, codes


def unpack_q4_0(data) -> tuple[np.ndarray, np.ndarray]:
    """Q4_0 symmetric: value j = low nibble of byte j minus 8, value 16+j = high nibble
    minus 8, returned as ml_dtypes int4.  ``ggml_quant.py:174-210`` (SYMMETRIC branch)."""
    u = _units(data, FORMATS["Q4_0"])
    scales = _f16_field(u, 0).reshape(-1, 1)
    body = u[:, 2:18]
    vals = np.empty((u.shape[0], 32), dtype=np.int8)
    vals[:, :16] = (body & 0x0F).astype(np.int8) - 8
    vals[:, 16:] = (body >> 4).astype(np.int8) - 8
    return scales, vals.astype(int4)


def _q5_values(u: np.ndarray, qh_off: int) -> np.ndarray:
    """Q5_0/Q5_1 values 0..31: value j takes the low (j < 16) or high (j >= 16) nibble of
    byte j % 16 and bit j of the little-endian uint32 at qh_off.  ``ggml_quant.py:230-271``."""
    qh = np.ascontiguousarray(u[:, qh_off:qh_off + 4]).view(np.uint32)[:, 0]
    body = u[:, qh_off + 4:qh_off + 20]
    nib = np.concatenate([body & 0x0F, body >> 4], axis=1).astype(np.uint8)
    bits = ((qh[:, None] >> np.arange(32, dtype=np.uint32)[None, :]) & 1).astype(np.uint8)
    return (nib | (bits << 4)).astype(np.int8)


def unpack_q5_0(data) -> tuple[np.ndarray, np.ndarray]:
    """Q5_0 symmetric: scale f32(d), codes q - 16 as int8.  ``ggml_quant.py:230-271`` via
    ``gguf_conversion.py:149-153``."""
    u = _units(data, FORMATS["Q5_0"])
    return _f16_field(u, 0).reshape(-1, 1), _q5_values(u, 2) - np.int8(16)


def unpack_asym_base(data, name: str):
    """Q4_1 / Q5_1: constants [d, m] f32 (not negated) and unsigned codes, as
    ``unpack_base_quant`` returns them (``ggml_quant.py:706-736``)."""
    u = _units(data, FORMATS[name])
    consts = np.stack([_f16_field(u, 0), _f16_field(u, 2)], axis=1)
    if name == "Q4_1":
        body = u[:, 4:20]
        q = np.concatenate([body & 0x0F, body >> 4], axis=1).astype(np.int8)
    else:
        q = _q5_values(u, 4)
    return consts, q


# ---------------------------------------------------------------------------
# K-quant super-blocks
# ---------------------------------------------------------------------------

def unpack_6bit_scale_min(packed: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """12 packed bytes -> 8 (scale, min) 6-bit pairs.  ``ggml_quant.py:352-375``.

    Pairs 0-3 sit in the low 6 bits of bytes 0-3 (scales) and 4-7 (mins); pairs 4-7
    take their low 4 bits from the nibbles of bytes 8-11 and their top 2 bits from the
    top 2 bits of bytes 0-3 (scales) and 4-7 (mins)."""
    p = packed.astype(np.uint8)
    sc = np.empty((p.shape[0], 8), dtype=np.int8)
    mn = np.empty((p.shape[0], 8), dtype=np.int8)
    sc[:, :4] = p[:, 0:4] & 0x3F
    mn[:, :4] = p[:, 4:8] & 0x3F
    sc[:, 4:] = (p[:, 8:12] & 0x0F) | ((p[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (p[:, 8:12] >> 4) | ((p[:, 4:8] >> 6) << 4)
    return sc, mn


def pack_6bit_scale_min(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of ``unpack_6bit_scale_min`` (used to build synthetic inputs)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, :4] & 0x3F) | ((sc[:, 4:] >> 4) << 6)
    out[:, 4:8] = (mn[:, :4] & 0x3F) | ((mn[:, 4:] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:] & 0x0F) | ((mn[:, 4:] & 0x0F) << 4)
    return out


def _q4_k_values(qs: np.ndarray) -> np.ndarray:
    """(N,128) nibble bytes -> (N,8,32): sub-block 2g = low nibbles of bytes 32g..32g+31,
    sub-block 2g+1 = their high nibbles.  ``ggml_quant.py:378-395``."""
    g = qs.reshape(-1, 4, 32)
    out = np.empty((qs.shape[0], 4, 2, 32), dtype=np.int8)
    out[:, :, 0, :] = g & 0x0F
    out[:, :, 1, :] = g >> 4
    return out.reshape(-1, 8, 32)


def _q5_k_values(qh: np.ndarray, qs: np.ndarray) -> np.ndarray:
    """Q4_K nibbles plus a fifth bit: sub-block k takes bit k of qh[j] for value j.
    ``ggml_quant.py:311-349`` (bit 2n for low nibbles, 2n+1 for high nibbles of group n)."""
    fifth = ((qh[:, None, :] >> np.arange(8, dtype=np.uint8)[None, :, None]) & 1) << 4
    return (_q4_k_values(qs).view(np.uint8) | fifth).view(np.int8)


def _q6_k_values(ql: np.ndarray, qh: np.ndarray, chunk: int = 4096) -> np.ndarray:
    """Q6_K: value 128h + 32g + j of a super-block is (nibble | 2 high bits << 4) - 32,
    where the nibble is the low (g<2) or high (g>=2) nibble of ql[64h + 32(g&1) + j] and
    the high bits are bits 2g..2g+1 of qh[32h + j].  ``ggml_quant.py:274-308``.  Built
    `chunk` super-blocks at a time, so the temporaries stay in cache."""
    n = ql.shape[0]
    out = np.empty((n, 2, 4, 32), dtype=np.uint8)
    shifts = np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 1, 4, 1)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        q = ql[a:b].reshape(b - a, 2, 2, 32)                     # [h, g & 1, j]
        hb = ((qh[a:b].reshape(b - a, 2, 1, 32) >> shifts) & 3) << 4
        o = out[a:b]
        np.bitwise_or(q & 0x0F, hb[:, :, 0:2], out=o[:, :, 0:2])
        np.bitwise_or(q >> 4, hb[:, :, 2:4], out=o[:, :, 2:4])
    v = out.view(np.int8)
    v -= np.int8(32)
    return v.reshape(n, 16, 16)


def _q2_k_values(qs: np.ndarray) -> np.ndarray:
    """Q2_K: bit pair j of byte b of half h is value 128h + 32j + b.  ``ggml_quant.py:479-498``."""
    halves = qs.reshape(-1, 2, 1, 32)
    out = (halves >> np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 1, 4, 1)) & 3
    return out.astype(np.int8).reshape(-1, 16, 16)


def _q3_k_values(hmask: np.ndarray, qs: np.ndarray) -> np.ndarray:
    """Q3_K: low 2 bits as Q2_K, third bit = bit 4h + j of hmask[b], minus 4.
    ``ggml_quant.py:428-463``."""
    low = (qs.reshape(-1, 2, 1, 32) >> np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 1, 4, 1)) & 3
    hb = (hmask.reshape(-1, 1, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 2, 4, 1)) & 1
    return ((low | (hb << 2)).astype(np.int8) - np.int8(4)).reshape(-1, 16, 16)


def _q3_k_scales(b: np.ndarray) -> np.ndarray:
    """Q3_K: 16 six-bit scales minus 32.  Scale i: low 4 bits from byte i (i < 8, low
    nibble) or byte i - 8 (high nibble), top 2 bits = bits 2(i//4)..+1 of byte 8 + i % 4.
    ``ggml_quant.py:398-425``."""
    b = b.astype(np.uint8)
    i = np.arange(16)
    low = np.where(i < 8, b[:, i % 8] & 0x0F, b[:, i % 8] >> 4)
    top = (b[:, 8 + i % 4] >> (2 * (i // 4)).astype(np.uint8)) & 3
    return ((low | (top << 4)).astype(np.int8) - np.int8(32)).reshape(-1, 16, 1)


def unpack_k_quant(data, name: str) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Split K-quant super-blocks into (super constants f32 (N,k), block constants
    int8 (N,B,k), values int8 (N,B,C)).  ``ggml_quant.py:567-694``; field order per
    format at ``:624-679``."""
    fmt = FORMATS[name]
    u = _units(data, fmt)
    if name == "Q4_K":      # d, dmin | scales[12] | qs[128]
        sup = np.stack([_f16_field(u, 0), _f16_field(u, 2)], axis=1)
        sc, mn = unpack_6bit_scale_min(u[:, 4:16])
        blk = np.stack([sc, mn], axis=2)
        vals = _q4_k_values(u[:, 16:144])
    elif name == "Q5_K":    # d, dmin | scales[12] | qh[32] | qs[128]
        sup = np.stack([_f16_field(u, 0), _f16_field(u, 2)], axis=1)
        sc, mn = unpack_6bit_scale_min(u[:, 4:16])
        blk = np.stack([sc, mn], axis=2)
        vals = _q5_k_values(u[:, 16:48], u[:, 48:176])
    elif name == "Q2_K":    # scales[16] (4-bit scale | 4-bit min << 4) | qs[64] | d, dmin
        sup = np.stack([_f16_field(u, 80), _f16_field(u, 82)], axis=1)
        blk = np.stack([(u[:, 0:16] & 0x0F).astype(np.int8), (u[:, 0:16] >> 4).astype(np.int8)], axis=2)
        vals = _q2_k_values(u[:, 16:80])
    elif name == "Q3_K":    # hmask[32] | qs[64] | scales[12] | d
        sup = _f16_field(u, 108).reshape(-1, 1)
        blk = _q3_k_scales(u[:, 96:108])
        vals = _q3_k_values(u[:, 0:32], u[:, 32:96])
    elif name == "Q6_K":    # ql[128] | qh[64] | scales int8[16] | d
        sup = _f16_field(u, 208).reshape(-1, 1)
        blk = np.ascontiguousarray(u[:, 192:208]).view(np.int8).reshape(-1, 16, 1)
        vals = _q6_k_values(u[:, 0:128], u[:, 128:192])
    else:
        raise ValueError(f"K-quant {name} not implemented yet.")
    return sup, blk, vals


def remove_superblocks(sup: np.ndarray, blk: np.ndarray, vals: np.ndarray):
    """Fold super-block constants into block constants.  ``ggml_quant.py:739-782``:
    f32 product of int8 block constant and f32 super constant, rounded to f16, with
    the min column negated (in f16); then flatten to (N*B, k) and (N*B, C)."""
    prod = blk.astype(np.float32) * sup[:, None, :]
    bc = prod.astype(np.float16)
    if bc.shape[2] == 2:
        bc[..., 1] = -bc[..., 1]
    n_blocks = bc.shape[0] * bc.shape[1]
    return bc.reshape(n_blocks, bc.shape[2]), vals.reshape(n_blocks, vals.shape[2])


@dataclass
class RequantDiag:
    round_error: np.float32
    clip_error: np.int16


SCALE_EPSILON = np.float32(np.float16(1e-4))   # ``ggml_quant.py:836``, widened exactly


def requantize_symmetric(bc: np.ndarray, q: np.ndarray, output_bits: int = 8,
                         new_dtype=np.int8, log: bool = True):
    """Asymmetric (S, M) blocks with unsigned codes -> symmetric scale + signed codes.
    ``ggml_quant.py:785-886``.  Returns (scales (N,1) f32, codes (N,B), RequantDiag).

    Per block, all in f32: S' = S, or M / eps when S == 0 (``:836-838``); r = M / S'
    (``:841``); lo/hi = min/max code + r (``:842-843``); sf = min(16, -2^(b-1)/lo if lo<0,
    (2^(b-1)-1)/hi if hi>0) (``:846-856``); integer sf when sf > 0.98 (``:859-863``);
    rm = int16(rint(r*sf)); q' = clip(int16(rint(q*sf)) + rm) (``:866-875``);
    scale = S / sf with the original S (``:882``)."""
    assert bc.ndim == 2 and bc.shape[1] == 2 and bc.dtype == np.float32
    assert q.ndim == 2 and q.shape[0] == bc.shape[0]
    lo_out = -(1 << (output_bits - 1))
    hi_out = (1 << (output_bits - 1)) - 1
    S = bc[:, 0]
    M = bc[:, 1]
    S_eff = np.where(S == 0, np.where(np.abs(M) > SCALE_EPSILON, M, SCALE_EPSILON), S).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        r = M / S_eff
        lo = q.min(axis=1) + r
        hi = q.max(axis=1) + r
        sf = np.minimum(np.float32(16), np.where(lo < 0, np.float32(lo_out) / lo, np.float32(16)))
        np.minimum(sf, np.where(hi > 0, np.float32(hi_out) / hi, np.float32(16)), out=sf)
        sf = np.where(sf > np.float32(0.98), np.maximum(np.floor(sf), np.float32(1)), sf)
        rmv = r * sf
        # float32 -> int16 by numpy's own cast, as the reference does it (on x86-64 through
        # int32: NaN and out-of-range values give INT32_MIN, whose low 16 bits are 0)
        rm = np.rint(rmv).astype(np.int16)
        round_error = np.max(np.abs(rm - rmv))
        unclipped = np.rint(q * sf[:, None]).astype(np.int16)
        unclipped += rm[:, None]
        clipped = np.clip(unclipped, lo_out, hi_out)
        clip_error = np.max(np.abs(clipped - unclipped))
        scales = (S / sf).reshape(-1, 1)
    assert scales.dtype == np.float32 and sf.dtype == np.float32
    if log and (clip_error > 0 or round_error > 0.5):
        _log.warning(f"Distortion from requantization: rounding {round_error}, clipping {clip_error}")
    return scales, clipped.astype(new_dtype), RequantDiag(np.float32(round_error), np.int16(clip_error))


def convert_k_quant(data, name: str, log: bool = True):
    """``unpack_k_quant`` + ``convert_to_simple_block_quant`` (``ggml_quant.py:697-703``).
    Returns (scales (N*B,1) f32, codes (N*B,C) int8, RequantDiag | None)."""
    sup, blk, vals = unpack_k_quant(data, name)
    bc, q = remove_superblocks(sup, blk, vals)
    bc = bc.astype(np.float32)
    if bc.shape[1] == 2:
        return requantize_symmetric(bc, q, 8, np.int8, log=log)
    return bc, q, None


# ---------------------------------------------------------------------------
# gguf-py dequantize (force_float path), restated
# ---------------------------------------------------------------------------

def gguf_dequantize(data, name: str) -> np.ndarray:
    """f32 values exactly as gguf-py computes them (flat, n_values)."""
    fmt = FORMATS[name]
    if name == "F32":
        return np.frombuffer(bytes(data), dtype=np.float32).copy()
    if name == "F16":
        return np.frombuffer(bytes(data), dtype=np.float16).astype(np.float32)
    if name == "BF16":
        return np.frombuffer(bytes(data), dtype=bfloat16).astype(np.float32)
    u = _units(data, fmt)
    if name == "Q8_0":      # x * d
        d = _f16_field(u, 0)[:, None]
        return (np.ascontiguousarray(u[:, 2:]).view(np.int8).astype(np.float32) * d).reshape(-1)
    if name == "Q4_0":      # d * (nibble - 8), low nibbles first
        d = _f16_field(u, 0)[:, None]
        b = u[:, 2:18]
        q = np.concatenate([b & 0x0F, b >> 4], axis=1).astype(np.int8) - np.int8(8)
        return (d * q.astype(np.float32)).reshape(-1)
    if name in ("Q4_K", "Q5_K"):   # (d*sc)*q - (dmin*m), each product rounded, no fma
        d = _f16_field(u, 0)
        dmin = _f16_field(u, 2)
        sc, mn = unpack_6bit_scale_min(u[:, 4:16])
        ds = (d[:, None] * sc.astype(np.float32))[:, :, None]
        dm = (dmin[:, None] * mn.astype(np.float32))[:, :, None]
        if name == "Q4_K":
            q = _q4_k_values(u[:, 16:144])
        else:
            q = _q5_k_values(u[:, 16:48], u[:, 48:176])
        return (ds * q.astype(np.float32) - dm).reshape(-1)
    if name == "Q4_1":      # (d * q) + m
        consts, q = unpack_asym_base(data, name)
        return (consts[:, :1] * q.astype(np.float32) + consts[:, 1:2]).reshape(-1)
    if name == "Q5_1":      # (d * q) + m
        consts, q = unpack_asym_base(data, name)
        return (consts[:, :1] * q.astype(np.float32) + consts[:, 1:2]).reshape(-1)
    if name == "Q5_0":      # d * (q - 16)
        d = _f16_field(u, 0)[:, None]
        return (d * (_q5_values(u, 2) - np.int8(16)).astype(np.float32)).reshape(-1)
    if name == "Q2_K":      # (d*sc)*q - dmin*m
        d = _f16_field(u, 80)[:, None]
        dmin = _f16_field(u, 82)[:, None]
        dl = (d * (u[:, 0:16] & 0x0F).astype(np.float32))[:, :, None]
        ml = (dmin * (u[:, 0:16] >> 4).astype(np.float32))[:, :, None]
        return (dl * _q2_k_values(u[:, 16:80]).astype(np.float32) - ml).reshape(-1)
    if name == "Q3_K":      # (d*sc) * q
        d = _f16_field(u, 108)[:, None]
        dl = (d * _q3_k_scales(u[:, 96:108])[:, :, 0].astype(np.float32))[:, :, None]
        return (dl * _q3_k_values(u[:, 0:32], u[:, 32:96]).astype(np.float32)).reshape(-1)
    if name == "Q6_K":      # (d*sc) * q
        d = _f16_field(u, 208)
        sc = np.ascontiguousarray(u[:, 192:208]).view(np.int8).astype(np.float32)
        dd = (d[:, None] * sc)[:, :, None]
        q = _q6_k_values(u[:, 0:128], u[:, 128:192]).astype(np.float32)
        return (dd * q).reshape(-1)
    raise NotImplementedError(f"Dequantization for {name} is not yet implemented")


# ---------------------------------------------------------------------------
# Tensor-level dispatch and the q/k head permutation
# ---------------------------------------------------------------------------

def permute_qk(scales, weights: np.ndarray, n_heads: int):
    """Llama/Mistral q/k row order: rows (H, D/2, 2) -> (H, 2, D/2), scales alike.
    ``gguf_conversion.py:314-332``."""
    def perm(a: np.ndarray) -> np.ndarray:
        rows = a.shape[0]
        return a.reshape(n_heads, rows // n_heads // 2, 2, *a.shape[1:]).swapaxes(1, 2).reshape(a.shape)
    if scales is not None:
        s2 = scales.reshape(weights.shape[0], -1)
        scales = perm(s2).reshape(scales.shape)
    return scales, perm(weights)


def unpack_tensor(name: str, data, shape_rows_cols: tuple[int, ...], force_float: bool = False,
                  log: bool = True):
    """``unpack_gguf_tensor`` (``gguf_conversion.py:102-176``) for the formats on the path.
    Returns (scales | None, weights reshaped to (rows, cols), RequantDiag | None)."""
    diag = None
    if name == "F32":
        w = np.frombuffer(bytes(data), dtype=np.float32).copy()
        s = None
    elif name == "F16":
        w = np.frombuffer(bytes(data), dtype=np.float16).copy()
        s = None
    elif name == "BF16":
        w = np.frombuffer(bytes(data), dtype=bfloat16).copy()
        s = None
    elif force_float:
        s, w = None, gguf_dequantize(data, name)
    elif name == "Q8_0":
        s, w = unpack_q8_0(data)
    elif name == "Q4_0":
        s, w = unpack_q4_0(data)
    elif name == "Q5_0":
        s, w = unpack_q5_0(data)
    elif name in ("Q4_1", "Q5_1"):
        consts, q = unpack_asym_base(data, name)
        s, w, diag = requantize_symmetric(consts, q, 8, np.int8, log=log)
    elif name in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"):
        s, w, diag = convert_k_quant(data, name, log=log)
    else:
        raise NotImplementedError(name)
    return s, w.reshape(shape_rows_cols), diag


# ---------------------------------------------------------------------------
# Embedding rows (afe block_quantize_weight_tensor is absent: parity unpinned)
# ---------------------------------------------------------------------------

def quantize_embedding_rows(emb: np.ndarray):
    """Per-row int8 quantization, ``sima_lmm/model/language_model.py:38-54``.

    PARITY UNPINNED: the reference calls ``afe.ir.quantization_conv.
    block_quantize_weight_tensor`` from the SiMa Palette SDK, which is not available.
    Restated assumption: step = absmax/127 (f32), q = clip(rint(x / step), -127, 127);
    the returned scale is step * 127 (the reference's ``* 127.0``, ``:51-52``), zero
    rows get scale 0 (``:53``), stored as bfloat16 (``:54``)."""
    assert emb.ndim == 2
    x = emb.astype(np.float32)
    absmax = np.max(np.abs(x), axis=1)
    step = (absmax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(step[:, None] > 0, np.rint(x / step[:, None]), 0)
    q = np.clip(q, -127, 127).astype(np.int8)
    scales = (step * np.float32(127.0)).astype(np.float32)
    scales[np.count_nonzero(x, axis=1) == 0] = 0.0
    return q, scales.reshape(-1, 1).astype(bfloat16)


# ---------------------------------------------------------------------------
# Modalix weight layout (ModelGraph._build_conv)
# ---------------------------------------------------------------------------

MLA_ROW_SIZE = 16   # sima_lmm/utils.py:4


def padded_output_channels(out_channels: int, is_int4: bool, pad_output: bool = True) -> int:
    """Output channels after the int4 32-way padding of ``model_graph.py:1057-1069`` (for a
    non-relocatable, non-quantizable graph with scales)."""
    split_width = ((-(-out_channels // MLA_ROW_SIZE) + 31) // 32) * MLA_ROW_SIZE
    if (pad_output and is_int4 and out_channels > 512 and out_channels % MLA_ROW_SIZE == 0
            and out_channels - 31 * split_width <= 0):
        return 32 * split_width
    return out_channels


def modalix_layout(scales: np.ndarray, codes: np.ndarray, padded: int):
    """``model_graph.py:1012-1079`` with the default oi->oihw reshape and no process
    functions: scales (O*I/B, 1) -> (I/B, O'), codes (O, I) -> HWIGO (1, 1, I, 1, O'),
    padded with zero codes and unit scales to O' output channels."""
    out_ch = codes.shape[0]
    s = np.transpose(np.reshape(scales, (out_ch, -1)), (1, 0))
    # _layout_array(w, "oi", "oihw") then (w, "oihw", "hwigo") (model_graph.py:1271-1304)
    w = np.transpose(np.expand_dims(codes.reshape(out_ch, -1, 1, 1), 0), (3, 4, 2, 0, 1))
    extra = padded - out_ch
    if extra:
        w = np.pad(w, ((0, 0),) * 4 + ((0, extra),))
        s = np.pad(s, ((0, 0), (0, extra)), constant_values=1)
    return s, w
