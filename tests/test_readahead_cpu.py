"""Host logic of ``GgufReaderProxy``'s read-ahead (CPU: the conversion is replaced by a stand-in
that records each batch, so no GPU is needed; the GPU tests load real files through the same
proxy).

* a call converts the requested tensor and the quantized tensors after it in file order, up
  to ``LLIMA_B200_READAHEAD_MB``, in one batch, and the later calls hand those results out
  without converting;
* each call logs the requantization warning of its own tensor, as the reference logs it;
* ``attn_q`` / ``attn_k`` are read ahead only with the head count ``perm_heads_of`` gives,
  and a call with another head count or output mode converts afresh;
* results waiting beyond four budgets are dropped oldest first and converted again later;
* a batch that fails (a tensor read ahead that cannot be converted) falls back to the
  requested tensor alone, so a call raises only what its own tensor raises;
* ``LLIMA_B200_READAHEAD_MB=0`` converts one tensor per call.
"""
import logging

import numpy as np
import pytest

from llima_b200 import gguf_conversion as G
from llima_b200.synth import gen_tensor_bytes

# name -> (format, rows, cols), in file order; every quantized tensor is 128 KiB of values
LAYOUT = [
    ("blk.0.attn_norm.weight", "F32", 256, 1),
    ("blk.0.attn_q.weight", "Q8_0", 512, 256),
    ("blk.0.attn_k.weight", "Q8_0", 512, 256),
    ("blk.0.attn_v.weight", "Q4_K", 512, 256),
    ("blk.0.ffn_up.weight", "Q4_K", 512, 256),
    ("blk.1.attn_q.weight", "Q8_0", 512, 256),
    ("blk.1.ffn_up.weight", "Q4_K", 512, 256),
    ("blk.1.ffn_down.weight", "Q6_K", 512, 256),
]


@pytest.fixture()
def gguf_file(tmp_path):
    gguf = pytest.importorskip("gguf")
    path = tmp_path / "ra.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    for i, (name, fmt, rows, cols) in enumerate(LAYOUT):
        if fmt == "F32":
            w.add_tensor(name, np.ones(rows, dtype=np.float32))
            continue
        raw = gen_tensor_bytes(fmt, rows * cols, 50 + i)
        w.add_tensor(name, raw.reshape(rows, -1), raw_shape=(rows, raw.size // rows),
                     raw_dtype=getattr(gguf.GGMLQuantizationType, fmt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


class FakeConvert:
    """Stand-in for convert_tensors: weights filled with the tensor's position in the file
    and its head count, one warning-sized distortion per tensor; records every batch."""

    def __init__(self):
        self.batches = []

    def __call__(self, jobs, force_float=False, device=None):
        self.batches.append([(t.name, heads, force_float) for t, _, heads in jobs])
        out = []
        for t, _, heads in jobs:
            pos = [n for n, *_ in LAYOUT].index(t.name)
            shape = tuple(int(x) for x in t.shape[::-1])
            w = np.full(shape, pos * 10 + heads, dtype=np.float32 if force_float else np.int8)
            out.append((None if force_float else np.full((w.size // 32, 1), pos, np.float32), w,
                        None if force_float else (np.float32(0.75), np.int16(0))))
        return out


def _proxy(path, monkeypatch, mb, heads_of=None):
    fake = FakeConvert()
    monkeypatch.setattr(G, "convert_tensors", fake)
    monkeypatch.setenv("LLIMA_B200_READAHEAD_MB", str(mb))
    return G.GgufReaderProxy(path, perm_heads_of=heads_of), fake


def test_calls_after_the_first_are_served_from_the_read_ahead(gguf_file, monkeypatch, caplog):
    heads = {"blk.0.attn_q.weight": 4, "blk.0.attn_k.weight": 2, "blk.1.attn_q.weight": 4}
    proxy, fake = _proxy(gguf_file, monkeypatch, 1, lambda n: heads.get(n, 0))
    caplog.set_level(logging.WARNING, logger="sima_lmm.gguf.ggml_quant")
    quant = [n for n, fmt, *_ in LAYOUT if fmt != "F32"]
    for n in quant:
        s, w = proxy.load_tensor(n, False, heads.get(n, 0))
        pos = [x for x, *_ in LAYOUT].index(n)
        assert int(w.flat[0]) == pos * 10 + heads.get(n, 0) and float(s[0, 0]) == pos
    # one batch: the first tensor and everything after it within the 1 MiB budget
    assert len(fake.batches) == 1 and [b[0] for b in fake.batches[0]] == quant
    assert [b[1] for b in fake.batches[0]] == [heads.get(n, 0) for n in quant]
    assert sum("Distortion from requantization" in r.message for r in caplog.records) == len(quant)
    assert proxy._ahead_bytes == 0 and not proxy._ahead


def test_budget_bounds_each_batch(gguf_file, monkeypatch):
    # a budget smaller than two tensors: each batch stops once it holds the budget
    proxy, fake = _proxy(gguf_file, monkeypatch, 0, None)
    monkeypatch.setattr(G, "_readahead_bytes", lambda: 100_000)
    proxy.load_tensor("blk.0.attn_v.weight", False)
    proxy.load_tensor("blk.0.ffn_up.weight", False)
    proxy.load_tensor("blk.1.ffn_up.weight", False)
    assert [[b[0] for b in batch] for batch in fake.batches] == [
        ["blk.0.attn_v.weight", "blk.0.ffn_up.weight"], ["blk.1.ffn_up.weight", "blk.1.ffn_down.weight"]]


def test_qk_tensors_need_their_head_count(gguf_file, monkeypatch):
    proxy, fake = _proxy(gguf_file, monkeypatch, 1, None)
    proxy.load_tensor("blk.0.attn_norm.weight", False)       # float: no conversion at all
    assert fake.batches == []
    proxy.load_tensor("blk.0.attn_q.weight", False, 4)
    assert [b[0] for b in fake.batches[0]] == ["blk.0.attn_q.weight", "blk.0.attn_v.weight",
                                               "blk.0.ffn_up.weight", "blk.1.ffn_up.weight",
                                               "blk.1.ffn_down.weight"]
    # attn_k was not read ahead (no head count known): converted by its own call
    s, w = proxy.load_tensor("blk.0.attn_k.weight", False, 2)
    assert int(w.flat[0]) == 2 * 10 + 2 and len(fake.batches) == 2
    # a read-ahead result is only handed out for the same head count and output mode
    _, w = proxy.load_tensor("blk.0.attn_v.weight", True)
    assert w.dtype == np.float32 and len(fake.batches) == 3 and fake.batches[2][0] == ("blk.0.attn_v.weight", 0, True)
    _, w = proxy.load_tensor("blk.0.attn_v.weight", False)
    assert w.dtype == np.int8 and len(fake.batches) == 3


def test_waiting_results_are_bounded(gguf_file, monkeypatch):
    heads = {"blk.0.attn_q.weight": 4, "blk.0.attn_k.weight": 2, "blk.1.attn_q.weight": 4}
    proxy, fake = _proxy(gguf_file, monkeypatch, 1, lambda n: heads.get(n, 0))
    proxy.load_tensor("blk.0.attn_q.weight", False, 4)     # reads ahead the six others
    assert len(proxy._ahead) == 6
    # with a smaller budget, the next batch (a head count nothing was read ahead with)
    # leaves at most four budgets of results waiting: the oldest go first and are converted
    # again when asked for
    monkeypatch.setattr(G, "_readahead_bytes", lambda: 100_000)
    proxy.load_tensor("blk.0.attn_v.weight", False, 2)
    assert proxy._ahead_bytes <= 4 * 100_000
    assert ("blk.0.attn_k.weight", False, 2) not in proxy._ahead
    assert ("blk.1.ffn_down.weight", False, 0) in proxy._ahead
    n = len(fake.batches)
    _, w = proxy.load_tensor("blk.0.attn_k.weight", False, 2)
    assert int(w.flat[0]) == 22 and len(fake.batches) == n + 1
    proxy.load_tensor("blk.1.ffn_down.weight", False)
    assert len(fake.batches) == n + 1


def test_read_ahead_off(gguf_file, monkeypatch):
    calls = []

    def one(t, force_float, heads=0):
        calls.append(t.name)
        return None, np.zeros(1)

    proxy, fake = _proxy(gguf_file, monkeypatch, 0, None)
    monkeypatch.setattr(G, "load_tensor", one)
    for n, fmt, *_ in LAYOUT:
        proxy.load_tensor(n, False)
    assert fake.batches == [] and calls == [n for n, *_ in LAYOUT]


def test_a_tensor_read_ahead_that_fails_does_not_fail_the_call(gguf_file, monkeypatch):
    proxy, fake = _proxy(gguf_file, monkeypatch, 1, None)

    def fussy(jobs, force_float=False, device=None):
        if any(t.name == "blk.1.ffn_down.weight" for t, _, _ in jobs):
            raise RuntimeError("gq_convert_host: size not supported")
        return fake(jobs, force_float, device)

    monkeypatch.setattr(G, "convert_tensors", fussy)
    _, w = proxy.load_tensor("blk.0.attn_v.weight", False)
    assert int(w.flat[0]) == 30
    # the batch with the failing tensor was dropped; the requested tensor went alone
    assert [[b[0] for b in batch] for batch in fake.batches] == [["blk.0.attn_v.weight"]]
    with pytest.raises(RuntimeError):
        proxy.load_tensor("blk.1.ffn_down.weight", False)
