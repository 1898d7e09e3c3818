"""Embedding-row kernels (gq_embedding_rows, gq_quantize_rows) against the CPU oracle.

The reference's row quantizer (afe) is not available, so the oracle restates its rule
(oracle/ggml_oracle.py: quantize_embedding_rows); parity with it is bit for bit, and the
reference's own contract (test_embedding_quantization.py:142-150) is checked as well.
"""
import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from llima_b200.embedding import embedding_rows_device, quantize_embedding_rows
from llima_b200.synth import gen_tensor_bytes
from oracle import ggml_oracle as O

pytestmark = pytest.mark.gpu


def _oracle_fused(fmt, raw, rows, cols, embed_scale, quantize):
    with np.errstate(all="ignore"):
        x = O.gguf_dequantize(raw.tobytes(), fmt).reshape(rows, cols).astype(np.float32)
        x *= np.float32(embed_scale)
        x = x.astype(bfloat16).astype(np.float32)
        if not quantize:
            return x
        return O.quantize_embedding_rows(x)


def _raw(fmt, rows, cols, seed):
    if fmt in ("F16", "BF16"):
        v = np.random.default_rng(seed).normal(0, 0.05, rows * cols).astype(np.float32)
        return v.astype(np.float16 if fmt == "F16" else bfloat16).view(np.uint8)
    return gen_tensor_bytes(fmt, rows * cols, seed, "bias")


@pytest.mark.parametrize("fmt,rows,cols", [("Q6_K", 1000, 4096), ("Q8_0", 777, 3584), ("Q4_K", 513, 2048),
                                           ("Q5_K", 300, 2048), ("Q4_0", 257, 1024), ("F16", 100, 640),
                                           ("BF16", 90, 512), ("F32", 64, 256)])
@pytest.mark.parametrize("embed_scale", [1.0, 45.254833995939045])
def test_fused_embedding_rows_match_oracle(fmt, rows, cols, embed_scale):
    raw = _raw(fmt, rows, cols, rows)
    src = torch.from_numpy(raw.copy()).cuda()
    codes, scales = embedding_rows_device(fmt, src, rows, cols, embed_scale, True)
    values = embedding_rows_device(fmt, src, rows, cols, embed_scale, False)
    torch.cuda.synchronize()
    q, s = _oracle_fused(fmt, raw, rows, cols, embed_scale, True)
    v = _oracle_fused(fmt, raw, rows, cols, embed_scale, False)
    assert np.array_equal(codes.cpu().numpy(), q)
    assert np.array_equal(scales.cpu().numpy(), s.view(np.uint16))
    assert np.array_equal(values.cpu().numpy().view(np.uint32), v.view(np.uint32))


@pytest.mark.parametrize("fmt,rows,cols", [("Q6_K", 200, 2048), ("Q4_K", 150, 1024), ("Q5_K", 100, 1024),
                                           ("Q8_0", 300, 512), ("Q4_0", 300, 512)])
@pytest.mark.parametrize("embed_scale", [1.0, 3.0e38, float("inf")])
def test_fused_embedding_rows_nonfinite_and_extreme(fmt, rows, cols, embed_scale):
    """Uniform random bytes (NaN, inf and huge f16 constants in some blocks), a scale that
    overflows, and an infinite scale: every row quantizes as the oracle does (rows whose
    absmax is not finite get zero codes and a non-finite scale)."""
    from llima_b200.formats import FORMATS
    f = FORMATS[fmt]
    n_units = rows * cols // f.unit_values
    raw = np.frombuffer(np.random.default_rng(rows + cols).bytes(n_units * f.unit_bytes), dtype=np.uint8).copy()
    src = torch.from_numpy(raw.copy()).cuda()
    codes, scales = embedding_rows_device(fmt, src, rows, cols, embed_scale, True)
    torch.cuda.synchronize()
    q, s = _oracle_fused(fmt, raw, rows, cols, embed_scale, True)
    assert np.array_equal(codes.cpu().numpy(), q)
    got, want = scales.cpu().numpy(), s.view(np.uint16)
    nan = np.isnan(got.view(bfloat16).astype(np.float32)) & np.isnan(want.view(bfloat16).astype(np.float32))
    assert np.all(nan | (got == want))


@pytest.mark.parametrize("fmt", ["Q6_K", "Q4_K", "Q8_0"])
def test_fused_embedding_rows_half_integer_quotients(fmt):
    """Rows where many y / step land exactly on half-integers (y = absmax * k / 254 in
    bf16), so rint's ties are decided by the exactly divided quotient."""
    rows, cols = 64, 1024
    raw = _raw(fmt, rows, cols, 7)
    src = torch.from_numpy(raw.copy()).cuda()
    codes, scales = embedding_rows_device(fmt, src, rows, cols, 2.0, True)
    torch.cuda.synchronize()
    q, s = _oracle_fused(fmt, raw, rows, cols, 2.0, True)
    assert np.array_equal(codes.cpu().numpy(), q) and np.array_equal(scales.cpu().numpy(), s.view(np.uint16))


def test_quantize_rows_match_oracle_with_zero_rows():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 0.1, (300, 1024)).astype(np.float32).astype(bfloat16).astype(np.float32)
    x[7] = 0.0
    x[100] = -0.0
    q, s = quantize_embedding_rows(x)
    q2, s2 = O.quantize_embedding_rows(x)
    assert q.dtype == np.int8 and s.dtype == bfloat16 and s.shape == (300, 1)
    assert np.array_equal(q, q2) and np.array_equal(s.view(np.uint16), s2.view(np.uint16))
    assert float(s[7, 0]) == 0.0 and float(s[100, 0]) == 0.0


def test_reference_contract_on_its_fixed_matrix():
    # test_embedding_quantization.py:118-150: quantize_embedding_rows(weights * embed_scale)
    weights = np.array([[-1.0, -0.5, 0.0, 0.5], [0.25, 0.75, 1.0, -0.25],
                        [0.125, -0.75, 0.625, -0.375]], dtype=np.float32)
    embed_scale = 8.0 ** 0.5
    x = (weights * np.float32(embed_scale)).astype(bfloat16).astype(np.float32)
    q, s = quantize_embedding_rows(x)
    assert q.dtype == np.int8 and q.shape == weights.shape and s.shape == (3, 1)
    np.testing.assert_allclose(q.astype(np.float32) * s.astype(np.float32) / 127.0, weights * embed_scale,
                               atol=float(np.max(s.astype(np.float32))) / 127.0)
