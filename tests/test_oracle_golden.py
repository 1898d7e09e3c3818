"""Pin the CPU oracle (oracle/ggml_oracle.py) before trusting it.

* every golden case produced by running the reference (tests/golden/make_golden.py);
* the reference's own known-answer tests for this path
  (tests/compilation/unit/test_quantization.py:115-154 and the N=1 / 37-super-block
  cases of test_ggml_kquant_equivalence.py in the reference).
"""
import logging

import ml_dtypes
import numpy as np
import pytest

from oracle import ggml_oracle as O
from tests.golden_cases import case_names, load_case, same_bits

CASES = case_names()


def test_golden_cases_present():
    assert len(CASES) >= 40


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_golden(case, caplog):
    g = load_case(case)
    fmt, rows, cols = g["fmt"], g["rows"], g["cols"]
    with caplog.at_level(logging.WARNING, logger="sima_lmm.gguf.ggml_quant"):
        with np.errstate(all="ignore"):
            s, w, diag = O.unpack_tensor(fmt, g["raw"].tobytes(), (rows, cols))
    codes = w.view(np.uint8) if w.dtype == ml_dtypes.int4 else w
    assert str(w.dtype) == g["codes_dtype"]
    assert same_bits(codes, g["codes"]), case
    if "scales" in g:
        assert s is not None and s.shape == g["scales"].shape
        assert same_bits(s, g["scales"]), case
    else:
        assert s is None
    # identical warning text (or none) as the reference logged
    msgs = [r.getMessage() for r in caplog.records if r.name == "sima_lmm.gguf.ggml_quant"]
    assert "\n".join(msgs) == g["warning"]
    with np.errstate(all="ignore"):
        f32 = O.gguf_dequantize(g["raw"].tobytes(), fmt).reshape(rows, cols)
    assert same_bits(f32, g["f32"]), case
    if "perm_heads" in g:
        ps, pw = O.permute_qk(s, w, g["perm_heads"])
        pcodes = pw.view(np.uint8) if pw.dtype == ml_dtypes.int4 else pw
        assert same_bits(pcodes, g["perm_codes"])
        if "perm_scales" in g:
            assert same_bits(ps, g["perm_scales"])


def test_known_answer_q4_k_nibbles():
    # reference test_quantization.py:128-140: byte 0xA3 -> 3 (low) and 10 (high)
    vals = O._q4_k_values(np.full((1, 128), 0xA3, dtype=np.uint8)).reshape(1, 256)
    for off in range(0, 256, 64):
        assert np.all(vals[0, off:off + 32] == 3)
        assert np.all(vals[0, off + 32:off + 64] == 10)


def test_known_answer_requantize_symmetric():
    # reference test_quantization.py:143-154
    consts = np.array([[0.5, -2.0]], dtype=np.float32)
    q = np.array([[0, 1, 2, 3, 4, 5]], dtype=np.uint8)
    expected = consts[:, :1] * q + consts[:, 1:2]
    s, rq, _ = O.requantize_symmetric(consts, q, 8, np.int8)
    assert s.dtype == np.float32 and rq.dtype == np.int8
    np.testing.assert_allclose(s * rq, expected, atol=float(s[0, 0]) / 2)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_k_value_unpackers_match_loop_definition(seed):
    # the per-super-block loop definitions of test_ggml_kquant_equivalence.py:25-77,
    # restated, on 37 super-blocks of random bytes
    rng = np.random.default_rng(seed)
    buf = rng.integers(0, 256, size=(37, 128 + 64), dtype=np.uint8)
    lo, hi = buf[:, :128], buf[:, 128:]
    got6 = O._q6_k_values(lo, hi).reshape(37, 256)
    for b in range(37):
        for h in range(2):
            e1, e2, hb = lo[b, 64 * h:64 * h + 32], lo[b, 64 * h + 32:64 * h + 64], hi[b, 32 * h:32 * h + 32]
            want = [(e1 & 15) | ((hb & 3) << 4), (e2 & 15) | (((hb >> 2) & 3) << 4),
                    (e1 >> 4) | (((hb >> 4) & 3) << 4), (e2 >> 4) | (((hb >> 6) & 3) << 4)]
            for g in range(4):
                assert np.array_equal(got6[b, 128 * h + 32 * g:128 * h + 32 * g + 32],
                                      want[g].astype(np.int8) - 32)
    got5 = O._q5_k_values(hi[:, :32], lo).reshape(37, 256)
    for b in range(37):
        for n in range(4):
            lo_n = lo[b, 32 * n:32 * n + 32]
            assert np.array_equal(got5[b, 64 * n:64 * n + 32], (lo_n & 15) + np.where(hi[b, :32] & (1 << 2 * n), 16, 0))
            assert np.array_equal(got5[b, 64 * n + 32:64 * n + 64], (lo_n >> 4) + np.where(hi[b, :32] & (2 << 2 * n), 16, 0))


def test_scale_pack_roundtrip():
    rng = np.random.default_rng(3)
    sc = rng.integers(0, 64, size=(50, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(50, 8), dtype=np.uint8)
    s2, m2 = O.unpack_6bit_scale_min(O.pack_6bit_scale_min(sc, mn))
    assert np.array_equal(s2, sc.astype(np.int8)) and np.array_equal(m2, mn.astype(np.int8))


def test_numpy_i16_cast_is_the_rule_the_kernels_follow():
    """numpy's float32 -> int16 cast (which the reference and the oracle use) is, on this
    platform, truncation through int32 with NaN and out-of-range values giving INT32_MIN,
    low 16 bits kept: the rule of the kernels' f32_to_i16_x86."""
    x = np.array([np.nan, np.inf, -np.inf, 1e10, -1e10, 40000.0, -40000.0, 32767.6, -2.5, 496.0],
                 dtype=np.float32)
    x = np.concatenate([x, np.random.default_rng(5).standard_normal(4096).astype(np.float32) * 1e5])
    with np.errstate(all="ignore"):
        got = x.astype(np.int16)
        ok = np.abs(x) < np.float32(2147483648.0)
        rule = np.where(ok, np.trunc(np.where(ok, x, 0)), -2147483648.0).astype(np.int64)
    assert np.array_equal(got, (rule & 0xFFFF).astype(np.uint16).view(np.int16))


def test_layout_restatement_matches_reference_layout_array():
    from tests.golden_cases import GOLDEN, layout_cases
    cases = layout_cases()
    assert cases
    for name in cases:
        with np.load(GOLDEN / f"{name}.npz") as z:
            s, w = O.modalix_layout(z["scales"], z["codes"], z["codes"].shape[0])
            assert s.shape == z["out_scales"].shape and np.array_equal(s, z["out_scales"])
            assert w.shape == z["out_weight"].shape and np.array_equal(w, z["out_weight"])
