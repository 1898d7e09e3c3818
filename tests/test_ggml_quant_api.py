"""The function-level ggml_quant API: oracle pinned on the CPU, GPU mirror checked on a B200.

tests/golden/ggml_quant/*.npz hold what the reference's own functions returned
(``unpack_q8_0``, ``unpack_dequantize_q8_0``, ``unpack_q4``, ``unpack_dequantize_q4``,
``unpack_q5``, ``unpack_base_quant``, ``unpack_k_quant``, ``remove_superblocks``,
``convert_to_simple_block_quant``, ``requantize_symmetric``; sima_lmm/gguf/ggml_quant.py
0.6.2) on seeded and uniform-random bytes, written by ``make_golden.py --only ggml_quant``.

* CPU: the oracle reproduces every one of them bit for bit, and the mirror module
  ``llima_b200.ggml_quant`` raises the reference's errors for bad arguments before it
  touches the GPU.
* GPU (``-m gpu``): ``llima_b200.ggml_quant`` returns the same arrays, dtypes and warning
  text as the reference on every case, and matches the oracle on BASELINE-sized tensors.
"""
import json
import logging

import ml_dtypes
import numpy as np
import pytest

from oracle import ggml_oracle as O
from tests.golden_cases import GOLDEN, same_bits

GQ_DIR = GOLDEN / "ggml_quant"
CASES = json.loads((GQ_DIR / "versions.json").read_text())["cases"]
LOGGER = "sima_lmm.gguf.ggml_quant"


def _load(case: str) -> dict:
    with np.load(GQ_DIR / f"{case}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def _calls(g: dict) -> dict[str, dict]:
    """{call: {"outs": [arrays], "dtypes": [names], "warning": text}} of a golden case."""
    calls: dict[str, dict] = {}
    for k in g:
        if "__" not in k:
            continue
        name, rest = k.split("__", 1)
        c = calls.setdefault(name, {"outs": {}, "dtypes": {}, "warning": ""})
        if rest == "warning":
            c["warning"] = str(g[k])
        elif rest.endswith("__dtype"):
            c["dtypes"][int(rest.split("__")[0])] = str(g[k])
        else:
            c["outs"][int(rest)] = g[k]
    return calls


def _as_u8(a: np.ndarray) -> np.ndarray:
    return a.view(np.uint8) if a.dtype in (ml_dtypes.int4, ml_dtypes.uint4) else a


def _check(got, want: dict, what: str):
    got = got if isinstance(got, tuple) else (got,)
    got = [g for g in got if g is not None]
    assert len(got) == len(want["outs"]), what
    for i, g in enumerate(got):
        assert str(g.dtype) == want["dtypes"][i], (what, i, g.dtype)
        w = want["outs"][i]
        assert g.shape == w.shape, (what, i, g.shape, w.shape)
        assert same_bits(_as_u8(g), w), (what, i)


def test_cases_present():
    assert len(CASES) == 30


# ---------------------------------------------------------------------------------------
# CPU: the oracle against the reference's outputs
# ---------------------------------------------------------------------------------------

def _oracle_call(name: str, fmt: str, raw: np.ndarray, g: dict):
    data = raw.tobytes()
    calls = _calls(g)
    if name == "unpack_q8_0":
        return O.unpack_q8_0(data)
    if name == "unpack_dequantize_q8_0":
        s, w = O.unpack_q8_0(data)
        return s * w
    if name == "unpack_q4":
        if fmt == "Q4_0":
            return O.unpack_q4_0(data)
        c, q = O.unpack_asym_base(data, "Q4_1")
        return c, q.view(np.uint8).view(ml_dtypes.uint4)
    if name == "unpack_dequantize_q4":
        return O.gguf_dequantize(data, fmt).reshape(-1, 32)
    if name == "unpack_q5":
        return O.unpack_q5_0(data) if fmt == "Q5_0" else O.unpack_asym_base(data, "Q5_1")
    if name == "unpack_base_quant":
        if fmt == "Q8_0":
            return O.unpack_q8_0(data)
        if fmt in ("Q4_0", "Q4_1"):
            return _oracle_call("unpack_q4", fmt, raw, g)
        return _oracle_call("unpack_q5", fmt, raw, g)
    if name == "unpack_k_quant":
        return O.unpack_k_quant(data, fmt)
    sup, blk, vals = (calls["unpack_k_quant"]["outs"][i] for i in range(3)) if "unpack_k_quant" in calls else \
        (None, None, None)
    if name == "remove_superblocks":
        return O.remove_superblocks(sup, blk, vals)
    if name == "remove_superblocks_f16_i16":
        return O.remove_superblocks(sup.astype(np.float16), blk.astype(np.int16), vals)
    if name == "convert_to_simple_block_quant":
        s, w, _ = O.convert_k_quant(data, fmt, log=True)
        return s, w
    if name.startswith("requantize_symmetric_"):
        bits = int(name.rsplit("_", 1)[1])
        want_dtype = np.dtype(calls[name]["dtypes"][1])
        if fmt in ("Q4_1", "Q5_1"):
            c, q = calls["unpack_q4" if fmt == "Q4_1" else "unpack_q5"]["outs"][0], \
                calls["unpack_q4" if fmt == "Q4_1" else "unpack_q5"]["outs"][1]
        else:
            bc, q = calls["remove_superblocks"]["outs"][0], calls["remove_superblocks"]["outs"][1]
            c = bc.astype(np.float32)
        s, w, _ = O.requantize_symmetric(c, q, bits, want_dtype, log=True)
        return s, w
    raise AssertionError(name)


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_functions(case, caplog):
    g = _load(case)
    fmt = str(g["fmt"])
    for name, want in _calls(g).items():
        caplog.clear()
        with caplog.at_level(logging.WARNING, logger=LOGGER):
            with np.errstate(all="ignore"):
                got = _oracle_call(name, fmt, g["raw"], g)
        got = tuple(got) if isinstance(got, tuple) else got
        # the oracle returns Q4_1 / Q5_1 / requant codes in the dtype asked; compare bits
        gl = got if isinstance(got, tuple) else (got,)
        for i, a in enumerate(gl):
            w = want["outs"][i]
            assert a.shape == w.shape, (case, name, i)
            assert same_bits(_as_u8(np.asarray(a)), w), (case, name, i)
        msgs = "\n".join(r.getMessage() for r in caplog.records if r.name == LOGGER)
        assert msgs == want["warning"], (case, name)


# ---------------------------------------------------------------------------------------
# CPU: argument checks of the mirror (raised before any device work)
# ---------------------------------------------------------------------------------------

def test_mirror_argument_errors():
    from llima_b200 import ggml_quant as M
    with pytest.raises(AssertionError):
        M.unpack_k_quant(b"", "Q4_0")
    with pytest.raises(KeyError):
        M.unpack_k_quant(b"", "Q8_K")
    with pytest.raises(KeyError):
        M.unpack_base_quant(b"", "Q8_1")
    with pytest.raises(ValueError, match="not implemented yet"):
        M.unpack_base_quant(b"", "Q4_K")
    sup = np.ones((2, 2), np.float32)
    blk = np.ones((2, 8, 2), np.int8)
    vals = np.zeros((2, 8, 32), np.int8)
    with pytest.raises(AssertionError):
        M.remove_superblocks(sup, blk.astype(np.uint8), vals)           # unsigned block constants
    with pytest.raises(AssertionError):
        M.remove_superblocks(sup[:1], blk, vals)                         # super-block counts differ
    with pytest.raises(TypeError):
        M.remove_superblocks(sup, blk.astype(np.int32), vals)           # wider than int16
    with pytest.raises(TypeError):
        M.remove_superblocks(sup.astype(np.float64), blk, vals)
    bc = np.ones((4, 2), np.float32)
    q = np.zeros((4, 32), np.int8)
    with pytest.raises(AssertionError):
        M.requantize_symmetric(bc.astype(np.float16), q, 8, np.int8)     # reference asserts f32
    with pytest.raises(AssertionError):
        M.requantize_symmetric(bc, q, 8, np.uint8)                       # unsigned output dtype
    with pytest.raises(ValueError, match="maximum"):
        M.requantize_symmetric(bc[:0], q[:0], 8, np.int8)
    with pytest.raises(ValueError, match="minimum"):
        M.requantize_symmetric(bc, q[:, :0], 8, np.int8)


def test_mirror_signatures_match_reference_names():
    import inspect

    from llima_b200 import ggml_quant as M
    # parameter names of the reference functions (ggml_quant.py:136-886)
    want = {"unpack_q8_0": ["data"], "unpack_dequantize_q8_0": ["data"], "unpack_q4": ["data", "symmetry"],
            "unpack_dequantize_q4": ["data", "symmetry"], "unpack_q5": ["data", "symmetry"],
            "unpack_base_quant": ["data", "ggml_name"], "unpack_k_quant": ["data", "ggml_name"],
            "remove_superblocks": ["superblock_constants", "block_constants", "quantized"],
            "convert_to_simple_block_quant": ["super_constants", "blocks", "elements"],
            "requantize_symmetric": ["block_constants", "quantized", "output_bits", "new_dtype"]}
    for name, params in want.items():
        assert list(inspect.signature(getattr(M, name)).parameters) == params, name
    assert int(M.QuantizationMode.Q6_K) == 14 and int(M.QuantizationSymmetry.ASYMMETRIC) == 1


# ---------------------------------------------------------------------------------------
# GPU: the mirror against the reference's outputs and the oracle
# ---------------------------------------------------------------------------------------

def _mirror_call(M, name: str, fmt: str, data: bytes, calls: dict):
    sym = M.QuantizationSymmetry.SYMMETRIC if fmt in ("Q4_0", "Q5_0") else M.QuantizationSymmetry.ASYMMETRIC
    if name == "unpack_q8_0":
        return M.unpack_q8_0(data)
    if name == "unpack_dequantize_q8_0":
        return M.unpack_dequantize_q8_0(data)
    if name == "unpack_q4":
        return M.unpack_q4(data, sym)
    if name == "unpack_dequantize_q4":
        return M.unpack_dequantize_q4(data, sym)
    if name == "unpack_q5":
        return M.unpack_q5(data, sym)
    if name == "unpack_base_quant":
        return M.unpack_base_quant(data, fmt)
    if name == "unpack_k_quant":
        return M.unpack_k_quant(data, fmt)
    sup, blk, vals = M.unpack_k_quant(data, fmt) if fmt.endswith("_K") else (None, None, None)
    if name == "remove_superblocks":
        return M.remove_superblocks(sup, blk, vals)
    if name == "remove_superblocks_f16_i16":
        return M.remove_superblocks(sup.astype(np.float16), blk.astype(np.int16), vals)
    if name == "convert_to_simple_block_quant":
        return M.convert_to_simple_block_quant(sup, blk, vals)
    if name.startswith("requantize_symmetric_"):
        bits = int(name.rsplit("_", 1)[1])
        dtype = np.dtype(calls[name]["dtypes"][1])
        if fmt == "Q4_1":
            c, q = M.unpack_q4(data, sym)
        elif fmt == "Q5_1":
            c, q = M.unpack_q5(data, sym)
        else:
            bc, q = M.remove_superblocks(sup, blk, vals)
            c = bc.astype(np.float32)
        return M.requantize_symmetric(c, q, bits, dtype)
    raise AssertionError(name)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_mirror_matches_reference_functions(case, caplog):
    from llima_b200 import ggml_quant as M
    g = _load(case)
    fmt = str(g["fmt"])
    data = g["raw"].tobytes()
    calls = _calls(g)
    for name, want in calls.items():
        caplog.clear()
        with caplog.at_level(logging.WARNING, logger=LOGGER):
            got = _mirror_call(M, name, fmt, data, calls)
        _check(got, want, f"{case}:{name}")
        msgs = "\n".join(r.getMessage() for r in caplog.records if r.name == LOGGER)
        assert msgs == want["warning"], (case, name)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["Q4_K", "Q5_K", "Q6_K", "Q2_K", "Q3_K"])
def test_mirror_k_quant_baseline_size(fmt):
    """unpack_k_quant + convert_to_simple_block_quant at the BASELINE config-2 shape
    (11008 x 4096), against the oracle."""
    from llima_b200 import ggml_quant as M
    from llima_b200.synth import gen_tensor_bytes
    data = gen_tensor_bytes(fmt, 11008 * 4096, 4242).tobytes()
    sup, blk, vals = M.unpack_k_quant(data, fmt)
    osup, oblk, ovals = O.unpack_k_quant(data, fmt)
    assert same_bits(sup, osup) and same_bits(blk, oblk) and same_bits(vals, ovals)
    with np.errstate(all="ignore"):
        s, w = M.convert_to_simple_block_quant(sup, blk, vals)
        os_, ow, _ = O.convert_k_quant(data, fmt, log=False)
    assert same_bits(s, os_) and same_bits(w, ow)


@pytest.mark.gpu
def test_mirror_odd_sizes_and_empty():
    """One unit, a tile and one, a ragged last warp tile, and empty input."""
    from llima_b200 import ggml_quant as M
    from llima_b200.synth import gen_tensor_bytes
    for fmt, ub in (("Q4_K", 144), ("Q6_K", 210), ("Q3_K", 110), ("Q2_K", 84), ("Q5_K", 176)):
        for n in (1, 9, 8 * 8 * 3 + 5):
            data = gen_tensor_bytes(fmt, n * 256, n).tobytes()
            for a, b in zip(M.unpack_k_quant(data, fmt), O.unpack_k_quant(data, fmt)):
                assert same_bits(a, b), (fmt, n)
        sup, blk, vals = M.unpack_k_quant(b"", fmt)
        assert sup.shape[0] == blk.shape[0] == vals.shape[0] == 0
    for fmt, ub in (("Q4_1", 20), ("Q5_1", 24)):
        for n in (1, 33, 32 * 8 * 2 + 7):
            data = gen_tensor_bytes(fmt, n * 32, n).tobytes()
            c, q = (M.unpack_q4 if fmt == "Q4_1" else M.unpack_q5)(data, M.QuantizationSymmetry.ASYMMETRIC)
            oc, oq = O.unpack_asym_base(data, fmt)
            assert same_bits(c, oc) and same_bits(_as_u8(q).view(np.int8), oq), (fmt, n)
