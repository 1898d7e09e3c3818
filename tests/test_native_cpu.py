"""CPU checks of the C ABI library and the host logic (no compute calls, no GPU)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from llima_b200 import _native as N
from llima_b200.formats import FORMATS, output_layout
from llima_b200.shard import piece_cost, plan_shards
from llima_b200.synth import gen_tensor_bytes, head_count_for, model_specs
from oracle import ggml_oracle as O

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol():
    header = (ROOT / "include" / "gguf_b200.h").read_text()
    declared = set(re.findall(r"GQ_API\s+[\w\s\*]+?\b(gq_\w+)\s*\(", header))
    assert declared == set(N.EXPORTS)
    lib = N.lib()
    for name in declared:
        assert hasattr(lib, name)
    assert lib.gq_version() == 2


def test_strerror_and_query():
    lib = N.lib()
    assert lib.gq_strerror(0) == b"success"
    assert b"aligned" in lib.gq_strerror(-3)
    for fmt, f in FORMATS.items():
        lay = N.query(f.type_id, 64, 512)
        assert lay.n_values == 64 * 512
        assert lay.src_bytes == 64 * 512 // f.unit_values * f.unit_bytes
        ol = output_layout(fmt, 64 * 512)
        assert lay.codes_bytes == ol["codes"] and lay.scales_count * 4 == ol["scales"]
    with pytest.raises(N.GqError):
        N.query(12, 3, 100)          # cols not a multiple of 256
    with pytest.raises(N.GqError):
        N.query(99, 1, 32)           # unknown type


def test_validation_errors_before_any_cuda_call():
    lib = N.lib()
    t = N.Tensor()
    t.type, t.rows, t.cols = 99, 1, 32
    assert lib.gq_convert(ctypes.byref(t), 1, None) == -1
    t.type, t.cols = 12, 100
    assert lib.gq_convert(ctypes.byref(t), 1, None) == -2
    t.cols = 256
    t.src_bytes = 144
    assert lib.gq_convert(ctypes.byref(t), 1, None) == -4      # NULL src
    t.src = 0x1001
    assert lib.gq_convert(ctypes.byref(t), 1, None) == -3      # misaligned
    assert lib.gq_convert_batch(None, 1, 1, None) == -4
    assert lib.gq_convert_batch(None, 0, 1, None) == 0
    assert lib.gq_requantize_symmetric(None, None, 1, 0, 8, None, None, None, None) == -5
    assert lib.gq_requantize_symmetric(None, None, 1, 32, 9, None, None, None, None) == -5
    # field unpack: types off its list, sizes, NULL / misaligned pointers, no CUDA call
    assert lib.gq_unpack_fields(8, None, 0, 1, None, None, None, None) == -1         # Q8_0
    assert lib.gq_unpack_fields(12, None, 143, 1, None, None, None, None) == -2      # too few bytes
    assert lib.gq_unpack_fields(12, None, 0, 0, None, None, None, None) == 0         # empty
    assert lib.gq_unpack_fields(12, None, 144, 1, None, None, None, None) == -4
    assert lib.gq_unpack_fields(12, 0x1000, 144, 1, 0x2000, None, 0x3000, None) == -4   # K needs blk
    assert lib.gq_unpack_fields(3, 0x1000, 20, 1, 0x2000, 0x4000, 0x3000, None) == -5   # Q4_1 has none
    assert lib.gq_unpack_fields(12, 0x1008, 144, 1, 0x2000, 0x4000, 0x3000, None) == -3
    assert lib.gq_remove_superblocks(None, None, 4, 1, 8, 2, None, None, None) == -5
    assert lib.gq_remove_superblocks(None, None, 1, 1, 8, 3, None, None, None) == -5
    assert lib.gq_remove_superblocks(None, None, 1, 0, 8, 2, None, None, None) == 0
    assert lib.gq_remove_superblocks(0x1000, 0x2000, 1, 1, 8, 2, None, None, None) == -4
    assert lib.gq_remove_superblocks(0x1002, 0x2000, 1, 1, 8, 2, 0x3000, None, None) == -3


def test_format_table_matches_oracle():
    for name, f in FORMATS.items():
        o = O.FORMATS[name]
        assert (f.type_id, f.unit_values, f.unit_bytes) == (o.type_id, o.unit_values, o.unit_bytes)
        assert f.block_values == o.block_values


def test_model_sets_match_baseline_totals():
    # the Llama-3-8B, Qwen2.5-7B and Llama-3-70B benchmark sets: 291 / 339 / 723 tensors,
    # 5.308 / 5.646 / 45.25 GB of GGUF bytes
    want = {"llama3-8b": (291, 5_307_858_944), "qwen2.5-7b": (339, 5_645_588_480),
            "llama3-70b": (723, 45_250_183_168)}
    for m, (n, nb) in want.items():
        sp = model_specs(m)
        assert len(sp) == n
        assert sum(s.nbytes for s in sp) == nb
    assert head_count_for("llama3-8b", "blk.3.attn_q.weight") == 32
    assert head_count_for("llama3-8b", "blk.3.attn_k.weight") == 8
    assert head_count_for("qwen2.5-7b", "blk.3.attn_q.weight") == 0


def test_synthetic_distributions():
    u = gen_tensor_bytes("Q4_K", 256 * 2000, 1).reshape(-1, 144)
    d = np.ascontiguousarray(u[:, :2]).view(np.float16).astype(np.float32)
    assert d.min() >= 9e-5 and d.max() <= 1.01e-2
    sc, mn = O.unpack_6bit_scale_min(u[:, 4:16])
    assert sc.min() == 0 and sc.max() == 63 and mn.max() == 63
    u6 = gen_tensor_bytes("Q6_K", 256 * 2000, 1).reshape(-1, 210)
    s6 = u6[:, 192:208].view(np.int8)
    assert s6.min() == -64 and s6.max() == 63
    q8 = gen_tensor_bytes("Q8_0", 32 * 4000, 1).reshape(-1, 34)[:, 2:].view(np.int8)
    assert q8.min() == -127 and q8.max() == 127


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_covers_every_row_once_and_balances(world):
    specs = model_specs("llama3-8b")
    items = [(s.fmt, s.rows, s.cols, head_count_for("llama3-8b", s.name) > 0) for s in specs]
    plan = plan_shards(items, world)
    assert len(plan) == world
    seen = {}
    for pieces in plan:
        for p in pieces:
            seen.setdefault(p.index, []).append((p.row0, p.row1))
    for i, (fmt, rows, cols, permuted) in enumerate(items):
        ranges = sorted(seen[i])
        assert ranges[0][0] == 0 and ranges[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        if permuted:
            assert len(ranges) == 1
    loads = [sum(piece_cost(items[p.index][0], p.rows, items[p.index][2]) for p in pieces) for pieces in plan]
    assert max(loads) <= 1.05 * (sum(loads) / world)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "_lib", None)
    monkeypatch.setenv("LLIMA_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(N.NativeLibraryError):
        N.lib()
