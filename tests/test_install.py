"""``gguf_conversion.install``: the switch that routes the reference's ``GgufModel`` through
the B200 path, in the calling process and in the reference's spawned compile workers
(``sima_lmm/model/base.py:665-709`` submits ``model.gen_files`` to a
``ProcessPoolExecutor`` with the ``spawn`` start method, so every worker unpickles the
model into a fresh, unpatched import of the reference module).

* CPU, with the reference checkout present: a real ``GgufModel`` built on a small GGUF
  file, pickled after ``install``, comes back in a spawned process with the B200 reader
  and ``load_weight``.
* CPU, with the reference checkout present: the installed ``load_weight`` of a real
  ``GgufModel`` reads ahead through the proxy with the model's q/k head counts (the
  conversion replaced by a recorder).
* GPU: a stand-in module shaped like the reference's (same attribute names and pickling
  hooks) gets the patched ``load_weight``: q/k tensors come back permuted as
  ``_permute_qk_proj`` does it (``gguf_conversion.py:314-332``), equal to the oracle, in
  the calling process and in a spawned worker.
"""
import multiprocessing as mp
import os
import pickle
import sys
import types
from pathlib import Path

import numpy as np
import pytest

from llima_b200.synth import gen_tensor_bytes
from oracle import ggml_oracle as O

# the reference checkout (the directory holding sima_lmm/), named by LLIMA_REFERENCE; the
# tests that import it skip when the variable is unset
REFERENCE = Path(os.environ["LLIMA_REFERENCE"]) if os.environ.get("LLIMA_REFERENCE") else None

# name -> (format, rows, cols): a one-layer llama file, 4 heads of 64, 2 kv heads
TENSORS = {
    "token_embd.weight": ("Q8_0", 64, 256),
    "blk.0.attn_q.weight": ("Q4_K", 256, 256),
    "blk.0.attn_k.weight": ("Q6_K", 128, 256),
    "blk.0.attn_output.weight": ("Q4_K", 256, 256),
}


def _write_gguf(path: Path):
    gguf = pytest.importorskip("gguf")
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(1)
    w.add_embedding_length(256)
    w.add_feed_forward_length(512)
    w.add_head_count(4)
    w.add_head_count_kv(2)
    w.add_context_length(128)
    raws = {}
    for i, (name, (fmt, rows, cols)) in enumerate(TENSORS.items()):
        raw = gen_tensor_bytes(fmt, rows * cols, 300 + i)
        w.add_tensor(name, raw.reshape(rows, -1), raw_shape=(rows, raw.size // rows),
                     raw_dtype=getattr(gguf.GGMLQuantizationType, fmt))
        raws[name] = raw
    w.add_tensor("blk.0.attn_norm.weight", np.ones(256, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return raws


def _import_reference():
    if REFERENCE is None or not (REFERENCE / "sima_lmm" / "gguf" / "gguf_conversion.py").exists():
        pytest.skip("reference checkout not available (set LLIMA_REFERENCE)")
    if str(REFERENCE) not in sys.path:
        sys.path.append(str(REFERENCE))   # after this repository: its `tests` must win
    sys.modules.setdefault("llama_cpp", types.SimpleNamespace(Llama=object))
    import sima_lmm.gguf.gguf_conversion as gc
    return gc


def _run_child(target, args, timeout=300):
    """Run target(*args, queue) in a spawned process; its one queue item, or a failure
    with the child's exit code as soon as it dies without one."""
    import queue as _queue
    import time
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=target, args=(*args, q))
    p.start()
    t0 = time.time()
    while True:
        try:
            item = q.get(timeout=1.0)
            break
        except _queue.Empty:
            if not p.is_alive() or time.time() - t0 > timeout:
                p.join(timeout=5)
                raise AssertionError(f"child process ended without a result (exit code {p.exitcode})")
    p.join(timeout=60)
    assert p.exitcode == 0
    return item


def _child_report(data: bytes, ref: str, queue):
    sys.path.append(ref)
    sys.modules.setdefault("llama_cpp", types.SimpleNamespace(Llama=object))
    obj = pickle.loads(data)
    import sima_lmm.gguf.gguf_conversion as gc
    queue.put({"proxy": type(obj.gguf_proxy).__module__,
               "load_weight": type(obj).load_weight.__module__,
               "unpack": gc.unpack_gguf_tensor.__module__,
               "vocab": obj.model_config["vocab_size"]})


def test_install_follows_the_model_into_spawned_workers(tmp_path):
    gc = _import_reference()
    path = tmp_path / "tiny.gguf"
    _write_gguf(path)
    model = gc.GgufModel(path)          # the reference's own path (nothing installed yet)
    assert model._need_permute_qk_proj
    from llima_b200.gguf_conversion import install
    saved = (gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight,
             gc.GgufModel.__dict__.get("__reduce_ex__"), gc.GgufModel.__dict__["model_config"])
    try:
        install(gc)
        data = pickle.dumps(model)
        rep = _run_child(_child_report, (data, str(REFERENCE)))
        assert rep == {"proxy": "llima_b200.gguf_conversion", "load_weight": "llima_b200.gguf_conversion",
                       "unpack": "llima_b200.gguf_conversion", "vocab": 64}
    finally:
        gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight = saved[:3]
        if saved[3] is None:
            del gc.GgufModel.__reduce_ex__
        else:
            gc.GgufModel.__reduce_ex__ = saved[3]
        gc.GgufModel.model_config = saved[4]


def test_installed_model_config_skips_the_embedding_decode(tmp_path, monkeypatch):
    """After install, building a GgufModel reads the vocabulary size from the token
    embedding's header: the config equals the reference's, and no tensor is converted
    (the conversion is made to fail to prove it)."""
    gc = _import_reference()
    path = tmp_path / "tiny.gguf"
    _write_gguf(path)
    want = gc.GgufModel(path).model_config      # the reference's own path
    from llima_b200 import gguf_conversion as G
    saved = (gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight,
             gc.GgufModel.__dict__.get("__reduce_ex__"), gc.GgufModel.__dict__["model_config"])

    def no_conversion(*a, **k):
        raise AssertionError("a tensor was converted while building the config")

    monkeypatch.setattr(G, "convert_host", no_conversion)
    monkeypatch.setattr(G, "convert_tensors", no_conversion)
    try:
        G.install(gc)
        G.install(gc)                            # a second install wraps nothing twice
        model = gc.GgufModel(path)
        assert model.model_config == want and model.model_config["vocab_size"] == 64
        assert "_llima_b200_shape_only" not in model.__dict__
    finally:
        gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight = saved[:3]
        if saved[3] is None:
            del gc.GgufModel.__reduce_ex__
        else:
            gc.GgufModel.__reduce_ex__ = saved[3]
        gc.GgufModel.model_config = saved[4]


def test_installed_load_weight_reads_ahead_with_the_models_head_counts(tmp_path, monkeypatch):
    """After install, the reference's own GgufModel.load_weight goes through the proxy's
    read-ahead: the first call converts the tensors after it in one batch, with the q/k head
    counts from the model's config (4 and 2 here), and the later calls are handed those
    results without converting (the conversion is replaced by a recorder: no GPU)."""
    gc = _import_reference()
    path = tmp_path / "tiny.gguf"
    _write_gguf(path)
    from llima_b200 import gguf_conversion as G
    saved = (gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight,
             gc.GgufModel.__dict__.get("__reduce_ex__"), gc.GgufModel.__dict__["model_config"])
    batches = []

    def recorder(jobs, force_float=False, device=None):
        batches.append([(t.name, heads) for t, _, heads in jobs])
        out = []
        for t, _, heads in jobs:
            shape = tuple(int(x) for x in t.shape[::-1])
            out.append((np.zeros((int(np.prod(shape)) // 32, 1), np.float32), np.full(shape, heads, np.int8), None))
        return out

    monkeypatch.setattr(G, "convert_tensors", recorder)
    monkeypatch.setenv("LLIMA_B200_READAHEAD_MB", "64")
    try:
        G.install(gc)
        model = gc.GgufModel(path)
        order = [n for n in TENSORS if n != "token_embd.weight"]
        for n in order:
            s, w = model.load_weight(n, is_hf_name=False)
            want = {"blk.0.attn_q.weight": 4, "blk.0.attn_k.weight": 2}.get(n, 0)
            assert w.shape == TENSORS[n][1:] and int(w.flat[0]) == want, n
        assert len(batches) == 1
        assert batches[0] == [(n, {"blk.0.attn_q.weight": 4, "blk.0.attn_k.weight": 2}.get(n, 0)) for n in order]
    finally:
        gc.unpack_gguf_tensor, gc.GgufReaderProxy, gc.GgufModel.load_weight = saved[:3]
        if saved[3] is None:
            del gc.GgufModel.__reduce_ex__
        else:
            gc.GgufModel.__reduce_ex__ = saved[3]
        gc.GgufModel.model_config = saved[4]


# ---------------------------------------------------------------------------------------
# GPU: a stand-in for the reference module
# ---------------------------------------------------------------------------------------

def _fake_module(name: str) -> types.ModuleType:
    """A module shaped like sima_lmm.gguf.gguf_conversion for install(): GgufReaderProxy,
    unpack_gguf_tensor and GgufModel with the attributes load_weight uses and the
    reference's pickling hooks (the reader is dropped and reopened)."""
    m = types.ModuleType(name)

    class GgufModel:
        def __init__(self, path):
            self.file_path = path
            self.gguf_proxy = m.GgufReaderProxy(path)
            self._need_permute_qk_proj = True
            self.model_config = {"num_attention_heads": 4, "num_key_value_heads": 2}

        def convert_hf_weight_name(self, name):
            return name

        def __getstate__(self):
            state = self.__dict__.copy()
            del state["gguf_proxy"]
            return state

        def __setstate__(self, state):
            self.__dict__.update(state)
            self.gguf_proxy = m.GgufReaderProxy(self.file_path)

    GgufModel.__module__ = name
    GgufModel.__qualname__ = "GgufModel"
    m.GgufModel = GgufModel
    m.GgufReaderProxy = None
    m.unpack_gguf_tensor = None
    return m


def _expected(raws, name):
    fmt, rows, cols = TENSORS[name]
    with np.errstate(all="ignore"):
        s, w, _ = O.unpack_tensor(fmt, raws[name].tobytes(), (rows, cols), log=False)
    heads = {"blk.0.attn_q.weight": 4, "blk.0.attn_k.weight": 2}.get(name, 0)
    if heads:
        s, w = O.permute_qk(s, w, heads)
    return s, w


def _child_load(data: bytes, module_name: str, names, queue):
    mod = _fake_module(module_name)
    sys.modules[module_name] = mod
    obj = pickle.loads(data)
    out = {n: obj.load_weight(n, is_hf_name=False) for n in names}
    queue.put({n: (s, np.asarray(w).view(np.uint8)) for n, (s, w) in out.items()})


@pytest.mark.gpu
def test_installed_load_weight_permutes_and_survives_spawn(tmp_path):
    from llima_b200.gguf_conversion import install
    from tests.golden_cases import same_bits
    path = tmp_path / "tiny.gguf"
    raws = _write_gguf(path)
    name = "llima_test_fake_gguf_conversion"
    mod = _fake_module(name)
    sys.modules[name] = mod
    try:
        install(mod)
        model = mod.GgufModel(path)
        for n in TENSORS:
            s, w = model.load_weight(n, is_hf_name=False)
            es, ew = _expected(raws, n)
            assert same_bits(w.view(np.uint8), ew.view(np.uint8)) and same_bits(s, es), n
        data = pickle.dumps(model)
        got = _run_child(_child_load, (data, name, list(TENSORS)))
        for n, (s, w) in got.items():
            es, ew = _expected(raws, n)
            assert same_bits(w, ew.view(np.uint8)) and same_bits(s, es), n
    finally:
        sys.modules.pop(name, None)
