"""Bundled-projection selection (ModelGraph._find_alternate_weight / _get_array_partition,
model_graph.py:1168-1248) against the reference's own methods (tests/golden/partition.json)."""
import json
from pathlib import Path

import numpy as np
import pytest

from llima_b200.layout import alternate_weight, array_partition

GOLDEN = Path(__file__).resolve().parent / "golden" / "partition.json"


def test_partition_matches_reference_methods():
    cases = json.loads(GOLDEN.read_text())
    assert len(cases) == 8
    for c in cases:
        fused, count, index, span = alternate_weight(c["weight"], c["q_size"], c["kv_size"])
        assert fused == c["fused"]
        assert array_partition(c["rows"], count, index, span) == (c["r0"], c["r1"])


def test_partition_edge_cases():
    with pytest.raises(NotImplementedError):
        alternate_weight("model.layers.0.self_attn.o_proj.weight", 8, 8)
    with pytest.raises(AssertionError):
        alternate_weight("model.layers.0.self_attn.q_proj.weight", None, 8)
    with pytest.raises(AssertionError):
        array_partition(10, 3, 0, 1)
    # numpy slice clamping: a span past the end keeps what exists
    a = np.arange(12)
    r0, r1 = array_partition(12, 4, 3, 2)
    assert (r0, r1) == (9, 12) and np.array_equal(a[r0:r1], a[9:9 + 6])
