"""Drop-in GGUF tensor decode on B200: the call surface of ``sima_lmm.gguf.gguf_conversion``.

``unpack_gguf_tensor(gguf_tensor, force_float)`` returns exactly what the reference
function of the same name returns (``sima_lmm/gguf/gguf_conversion.py:102-176``): for
quantized types ``(scales f32 (n_blocks, 1), codes (rows, cols))`` with int8 codes (or
ml_dtypes int4 for Q4_0), for ``force_float=True`` ``(None, f32 (rows, cols))`` as
gguf-py's ``dequantize`` computes it, and float tensors unchanged.  The decode runs in
libgguf_b200.so through ``gq_convert_host``; there is no CPU fallback: a type outside
the path (IQ*, TQ*, MXFP4 ...) raises ``NotImplementedError``, and Q8_1 raises the
``KeyError`` the reference's format table raises for it (``ggml_quant.py:716``).

``GgufReaderProxy`` mirrors the reference class (``gguf_conversion.py:179-205``), and
``install`` swaps this decode (and the fused q/k head permutation) into an imported
reference module so that ``GgufModel`` and everything above it run unchanged.
"""
from __future__ import annotations

import ctypes
import functools
import logging
import mmap
import os
import threading
import weakref
from pathlib import Path

import numpy as np
from ml_dtypes import bfloat16, int4

from . import _native as N
from .formats import FORMAT_BY_ID, FORMATS

__all__ = ["unpack_gguf_tensor", "load_tensor", "load_partition", "convert_host", "convert_gguf_file",
           "GgufReaderProxy", "install", "requant_warning"]

# Same logger and text as ggml_quant.py:879-880, so log handling stays as it was.
_log = logging.getLogger("sima_lmm.gguf.ggml_quant")

_GPU_TYPES = {"Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"}
_sessions: dict[tuple[int, int], ctypes.c_void_p] = {}
_sessions_lock = threading.Lock()


def _device() -> int:
    env = os.environ.get("LLIMA_B200_DEVICE")
    if env is not None:
        return int(env)
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.current_device()
    except ImportError:
        pass
    return 0


def _session(device: int) -> ctypes.c_void_p:
    """Per-process, per-device session (created lazily, so spawned workers each get their
    own CUDA context, as the reference's process pool needs)."""
    key = (os.getpid(), device)
    with _sessions_lock:
        s = _sessions.get(key)
        if s is None:
            mb = int(os.environ.get("LLIMA_B200_STAGING_MB", "256"))
            s = ctypes.c_void_p()
            N.check(N.lib().gq_session_create(device, mb << 20, ctypes.byref(s)), "gq_session_create")
            _sessions[key] = s
    return s


def requant_warning(round_error: np.float32, clip_error: np.int16) -> None:
    """Log the reference's distortion warning when it would fire (ggml_quant.py:879-880)."""
    if clip_error > 0 or round_error > 0.5:
        _log.warning(f"Distortion from requantization: rounding {round_error}, clipping {clip_error}")


def _host_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


_HUGE_MIN = 8 << 20


_PINNED_MIN = 1 << 20


class _PinnedBlock:
    """Owner of one page-locked buffer from the library's result arena (gq_host_alloc): the
    arrays viewing it keep it alive, and the buffer goes back to the arena for the next
    result of its size once the last of them is gone."""
    __slots__ = ("ptr", "nbytes", "__weakref__")

    def __init__(self, ptr: int, nbytes: int):
        self.ptr = ptr
        self.nbytes = nbytes
        weakref.finalize(self, _pinned_release, ptr).atexit = False

    @property
    def __array_interface__(self):
        # numpy keeps the object that exports the buffer as the array's base
        return {"shape": (self.nbytes,), "typestr": "|u1", "data": (self.ptr, False), "version": 3}


def _pinned_release(ptr: int) -> None:
    try:
        N.lib().gq_host_free(ptr)
    except Exception:   # interpreter shutdown: the process frees everything anyway
        pass


def _pinned_empty(shape, dtype: np.dtype, n: int):
    """A result array in a recycled page-locked buffer, or None when the arena is full or
    turned off (LLIMA_B200_PINNED_RESULTS_MB=0)."""
    ptr = ctypes.c_void_p()
    if N.lib().gq_host_alloc(n, ctypes.byref(ptr)) != N.GQ_OK or not ptr.value:
        return None
    return np.asarray(_PinnedBlock(ptr.value, n)).view(dtype).reshape(shape)


def _host_empty(shape, dtype) -> np.ndarray:
    """An uninitialised host array for a conversion result.  From 1 MiB on it lives in a
    page-locked buffer of the library's recycled result arena, which the copy engines write
    directly (no page faults, no host copy); when the arena is full, large arrays are
    backed by an anonymous mapping with transparent huge pages requested, so that the first
    writes (by the library's copy threads) fault in 2 MiB pages instead of 4 KiB ones; the
    array owns its memory and frees it (or returns it to the arena) with itself."""
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    if n >= _PINNED_MIN:
        arr = _pinned_empty(shape, dtype, n)
        if arr is not None:
            return arr
    if n < _HUGE_MIN:
        return np.empty(shape, dtype=dtype)
    m = mmap.mmap(-1, n, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
    if hasattr(m, "madvise") and hasattr(mmap, "MADV_HUGEPAGE"):
        try:
            m.madvise(mmap.MADV_HUGEPAGE)
        except OSError:
            pass
    return np.frombuffer(m, dtype=dtype, count=n // dtype.itemsize).reshape(shape)


def convert_host(fmt: str, raw: np.ndarray, rows: int, cols: int, force_float: bool = False,
                 perm_heads: int = 0, device: int | None = None):
    """GGUF bytes in host memory -> (scales | None, weights) in host memory, on the GPU.
    Returns (scales, weights, (round_error, clip_error) | None)."""
    f = FORMATS[fmt]
    raw = np.ascontiguousarray(raw).reshape(-1).view(np.uint8)
    n_values = rows * cols
    if f.asymmetric and not force_float and n_values == 0:
        # the reference's np.max over an empty requantization raises (ggml_quant.py:868)
        raise ValueError("zero-size array to reduction operation maximum which has no identity")
    rec = N.Tensor()
    rec.type = f.type_id
    rec.perm_heads = perm_heads
    rec.rows = rows
    rec.cols = cols
    rec.src = _host_ptr(raw)
    rec.src_bytes = raw.size
    scales = codes = values = None
    if force_float:
        values = _host_empty((rows, cols), np.float32)
        rec.values = _host_ptr(values)
        mask = N.OUT_F32
    else:
        codes = _host_empty((rows, cols), np.int8)
        scales = _host_empty((n_values // f.block_values, 1), np.float32)
        rec.codes = _host_ptr(codes)
        rec.scales = _host_ptr(scales)
        mask = N.OUT_CODES
    diag = N.Diag()
    dev = _device() if device is None else device
    N.check(N.lib().gq_convert_host(_session(dev), ctypes.byref(rec), 1, mask, ctypes.byref(diag)),
            "gq_convert_host")
    if force_float:
        return None, values, None
    d = None
    if f.asymmetric:
        d = (np.array([diag.round_err_bits], dtype=np.uint32).view(np.float32)[0], np.int16(diag.clip_err))
    if fmt == "Q4_0":
        codes = codes.view(np.uint8).view(int4)
    return scales, codes, d


def convert_gguf_file(path, names=None, force_float: bool = False, permute_qk: bool | None = None,
                      device: int | None = None, reader=None) -> dict:
    """Every quantized tensor of a GGUF file (or the ``names`` given) in one host-buffer
    call, so that the copies, the kernels and the result copies of all tensors overlap:
    ``{name: (scales | None, weights)}`` with the values ``unpack_gguf_tensor`` returns for
    each tensor (float tensors are passed through on the host as it does).

    ``permute_qk``: apply the llama / mistral q/k head permutation to ``attn_q`` / ``attn_k``
    weights and biases as ``GgufModel.load_weight`` does (``gguf_conversion.py:285-332``);
    ``None`` decides from the file's ``general.architecture`` (``llama``).  The
    requantization warning is logged per tensor, as the reference logs it per call."""
    if reader is None:
        from gguf import GGUFReader
        reader = GGUFReader(path)
    fields = reader.fields

    def field(key):
        f = fields.get(key)
        if f is None:
            return None
        v = f.contents()
        if isinstance(v, (list, np.ndarray)):
            return int(np.max(v))
        return v

    arch = field("general.architecture")
    if permute_qk is None:
        permute_qk = arch == "llama"
    n_head = field(f"{arch}.attention.head_count") if arch else None
    n_kv = field(f"{arch}.attention.head_count_kv") if arch else None
    wanted = None if names is None else set(names)
    out: dict = {}
    jobs = []
    for t in reader.tensors:
        if wanted is not None and t.name not in wanted:
            continue
        heads = 0
        if permute_qk and n_head:
            if t.name.endswith(("attn_q.weight", "attn_q.bias")):
                heads = int(n_head)
            elif t.name.endswith(("attn_k.weight", "attn_k.bias")):
                heads = int(n_kv or n_head)
        fmt = _type_name(t.tensor_type)
        if fmt in ("F32", "F16", "BF16"):
            out[t.name] = load_tensor(t, force_float, heads)
            continue
        if fmt == "Q8_1" and not force_float:
            raise KeyError("Q8_1")
        if fmt not in _GPU_TYPES:
            raise NotImplementedError(f"GGML type {fmt} is not handled by the B200 GGUF path")
        jobs.append((t, fmt, heads))
    for (t, _, _), (scales, w, d) in zip(jobs, convert_tensors(jobs, force_float, device)):
        if d is not None:
            requant_warning(*d)
        out[t.name] = (scales, w)
    return out


def convert_tensors(jobs, force_float: bool = False, device: int | None = None) -> list:
    """GGUF reader tensors ``[(tensor, fmt, perm_heads)]`` (quantized types on the path) in
    one host-buffer call: ``[(scales | None, weights, (round_error, clip_error) | None)]`` in
    order, each as ``load_tensor`` returns it, with the requantization diagnostics handed
    back instead of logged."""
    if not jobs:
        return []
    recs = (N.Tensor * len(jobs))()
    diags = (N.Diag * len(jobs))()
    results = []
    for i, (t, fmt, heads) in enumerate(jobs):
        f = FORMATS[fmt]
        shape = tuple(int(x) for x in t.shape[::-1])
        rows = shape[0]
        cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
        if f.asymmetric and not force_float and rows * cols == 0:
            raise ValueError("zero-size array to reduction operation maximum which has no identity")
        raw = np.ascontiguousarray(np.asarray(t.data)).reshape(-1).view(np.uint8)
        r = N.Tensor()
        r.type, r.perm_heads, r.rows, r.cols = f.type_id, heads, rows, cols
        r.src, r.src_bytes = _host_ptr(raw), raw.size
        if force_float:
            values = _host_empty((rows, cols), np.float32)
            r.values = _host_ptr(values)
            results.append((fmt, shape, raw, None, values))
        else:
            codes = _host_empty((rows, cols), np.int8)
            scales = _host_empty((rows * cols // f.block_values, 1), np.float32)
            r.codes, r.scales = _host_ptr(codes), _host_ptr(scales)
            results.append((fmt, shape, raw, scales, codes))
        recs[i] = r
    dev = _device() if device is None else device
    mask = N.OUT_F32 if force_float else N.OUT_CODES
    N.check(N.lib().gq_convert_host(_session(dev), recs, len(jobs), mask, diags), "gq_convert_host")
    out = []
    for (fmt, shape, _raw, scales, w), dg in zip(results, diags):
        if force_float:
            out.append((None, w.reshape(shape), None))
            continue
        d = None
        if FORMATS[fmt].asymmetric:
            d = (np.array([dg.round_err_bits], dtype=np.uint32).view(np.float32)[0], np.int16(dg.clip_err))
        if fmt == "Q4_0":
            w = w.view(np.uint8).view(int4)
        out.append((scales, w.reshape(shape), d))
    return out


def _type_name(tensor_type) -> str:
    tid = int(tensor_type)
    f = FORMAT_BY_ID.get(tid)
    if f is not None:
        return f.name
    return getattr(tensor_type, "name", str(tid))


def load_tensor(gguf_tensor, force_float: bool, perm_heads: int = 0):
    """``unpack_gguf_tensor`` plus the llama q/k head permutation fused into the decode
    (``GgufModel.load_weight`` + ``_permute_qk_proj``, gguf_conversion.py:285-332)."""
    name = _type_name(gguf_tensor.tensor_type)
    shape = tuple(int(x) for x in gguf_tensor.shape[::-1])
    if name in ("F32", "F16", "BF16"):
        # float tensors are passed through unchanged (gguf_conversion.py:132-140)
        if name == "F32":
            w = np.asarray(gguf_tensor.data, dtype=np.float32)
        elif name == "F16":
            w = np.asarray(gguf_tensor.data, dtype=np.float16)
        else:
            w = np.frombuffer(gguf_tensor.data.tobytes(), dtype=bfloat16)
        w = w.reshape(shape)
        if perm_heads:
            rows = shape[0]
            w = w.reshape(perm_heads, rows // perm_heads // 2, 2, *shape[1:]).swapaxes(1, 2).reshape(shape)
        return None, w
    if name == "Q8_1" and not force_float:
        raise KeyError("Q8_1")
    if name not in _GPU_TYPES:
        raise NotImplementedError(f"GGML type {name} is not handled by the B200 GGUF path")
    rows = shape[0]
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    s, w, d = convert_host(name, np.asarray(gguf_tensor.data), rows, cols, force_float, perm_heads)
    if d is not None:
        requant_warning(*d)
    return s, w.reshape(shape)


def load_partition(gguf_tensor, count: int, index: int, span: int, force_float: bool = False):
    """A bundled projection's selected rows, decoded on their own.

    ``_build_conv`` decodes the whole bundled tensor (``qkv_proj``, ``gate_up_proj``) for
    each projection and keeps the rows ``_get_array_partition(count, index, span)`` selects,
    from the weights and from the scales reshaped to (rows, blocks per row)
    (model_graph.py:990-998, 1012-1016, 1168-1195).  GGUF stores rows contiguously, so
    only the selected rows' bytes are converted here.  Returns (scales | None, weights) for
    those rows: scales (selected blocks, 1) in row order and weights (r1 - r0, ...), i.e.
    the partition of ``unpack_gguf_tensor``'s result.  The requantization warning then
    covers the decoded rows only."""
    from .layout import array_partition

    name = _type_name(gguf_tensor.tensor_type)
    shape = tuple(int(x) for x in gguf_tensor.shape[::-1])
    r0, r1 = array_partition(shape[0], count, index, span)
    if name in ("F32", "F16", "BF16"):
        s, w = load_tensor(gguf_tensor, force_float, 0)
        return None, w[r0:r1]
    if name == "Q8_1" and not force_float:
        raise KeyError("Q8_1")
    if name not in _GPU_TYPES:
        raise NotImplementedError(f"GGML type {name} is not handled by the B200 GGUF path")
    f = FORMATS[name]
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    row_bytes = cols // f.unit_values * f.unit_bytes
    raw = np.asarray(gguf_tensor.data).reshape(-1).view(np.uint8)[r0 * row_bytes:r1 * row_bytes]
    s, w, d = convert_host(name, raw, r1 - r0, cols, force_float)
    if d is not None:
        requant_warning(*d)
    return s, w.reshape((r1 - r0, *shape[1:]))


def unpack_gguf_tensor(gguf_tensor, force_float: bool):
    """Same inputs and outputs as ``sima_lmm.gguf.gguf_conversion.unpack_gguf_tensor``."""
    return load_tensor(gguf_tensor, force_float, 0)


_READAHEAD_MB_DEFAULT = 1024


def _readahead_bytes() -> int:
    return max(0, int(os.environ.get("LLIMA_B200_READAHEAD_MB", str(_READAHEAD_MB_DEFAULT)))) << 20


class GgufReaderProxy:
    """``GgufReaderProxy`` (gguf_conversion.py:179-205) with the B200 decode.

    ``load_tensor`` of a quantized tensor converts it together with the quantized tensors
    that follow it in the file, up to ``LLIMA_B200_READAHEAD_MB`` (default 1024) MB of GGUF
    bytes, in one host-buffer call, so that the host copies, transfers and kernels of
    successive tensors overlap as in ``convert_gguf_file``.  The tensors read ahead wait in
    the proxy until their own ``load_tensor`` call hands them out (the requantization
    warning is logged then, per call, as the reference logs it), so a loader that asks for
    tensors one at a time in about file order gets whole-file throughput.  At most four
    times the read-ahead budget of results waits at once (the oldest is dropped first, and
    converted again if it is asked for later); if the batch fails, the requested tensor is
    converted on its own, so a call raises only what its own tensor raises.
    ``perm_heads_of(name)`` gives the q/k head
    count the caller will ask for a tensor with (``install`` sets it from the model's
    config); while it is None, ``attn_q`` / ``attn_k`` tensors are not read ahead.
    ``LLIMA_B200_READAHEAD_MB=0`` converts each tensor on its own."""

    def __init__(self, path: Path | str, perm_heads_of=None):
        from collections import OrderedDict
        from gguf import GGUFReader
        self._gguf_reader = GGUFReader(path)
        self._tensor_map = {x.name: idx for idx, x in enumerate(self._gguf_reader.tensors)}
        self.perm_heads_of = perm_heads_of
        self._ahead: OrderedDict = OrderedDict()   # (name, force_float, heads) -> (scales, weights, diag, bytes)
        self._ahead_bytes = 0
        self._lock = threading.Lock()

    def _heads(self, name: str):
        if self.perm_heads_of is not None:
            return int(self.perm_heads_of(name))
        if name.endswith(("attn_q.weight", "attn_q.bias", "attn_k.weight", "attn_k.bias")):
            return None
        return 0

    def load_tensor(self, tensor_name: str, force_float: bool, perm_heads: int = 0):
        assert tensor_name in self._tensor_map, f"Tensor {tensor_name} not exist in tensor map."
        key = (tensor_name, bool(force_float), int(perm_heads))
        with self._lock:
            hit = self._ahead.pop(key, None)
            if hit is not None:
                self._ahead_bytes -= hit[3]
                if hit[2] is not None:
                    requant_warning(*hit[2])
                return hit[0], hit[1]
            idx = self._tensor_map[tensor_name]
            gguf_tensor = self._gguf_reader.get_tensor(idx)
            budget = _readahead_bytes()
            fmt = _type_name(gguf_tensor.tensor_type)
            if budget == 0 or fmt not in _GPU_TYPES or int(gguf_tensor.n_elements) == 0:
                return load_tensor(gguf_tensor, force_float, perm_heads)
            jobs = [(gguf_tensor, fmt, int(perm_heads))]
            keys = [key]
            total = int(gguf_tensor.n_bytes)
            tensors = self._gguf_reader.tensors
            for j in range(idx + 1, len(tensors)):
                if total >= budget:
                    break
                t = tensors[j]
                f = _type_name(t.tensor_type)
                if f not in _GPU_TYPES or int(t.n_elements) == 0:
                    continue
                heads = self._heads(t.name)
                k = (t.name, bool(force_float), heads)
                if heads is None or k in self._ahead:
                    continue
                jobs.append((t, f, heads))
                keys.append(k)
                total += int(t.n_bytes)
            try:
                res = convert_tensors(jobs, force_float)
            except Exception:
                if len(jobs) == 1:
                    raise
                # a tensor read ahead that cannot be converted must not fail this call: the
                # requested tensor alone raises only what its own conversion raises
                jobs, keys = jobs[:1], keys[:1]
                res = convert_tensors(jobs, force_float)
            for k, (sc, w, d) in zip(keys[1:], res[1:]):
                nb = w.nbytes + (sc.nbytes if sc is not None else 0)
                self._ahead[k] = (sc, w, d, nb)
                self._ahead_bytes += nb
            while self._ahead and self._ahead_bytes > 4 * budget:
                self._ahead_bytes -= self._ahead.popitem(last=False)[1][3]
        sc, w, d = res[0]
        if d is not None:
            requant_warning(*d)
        return sc, w

    def get_fields(self) -> dict:
        return dict(self._gguf_reader.fields.items())

    def get_tensor_info(self) -> dict:
        info = {}
        for name, idx in self._tensor_map.items():
            t = self._gguf_reader.get_tensor(idx)
            info[name] = {"gguf_type": t.tensor_type, "shape": tuple(t.shape[::-1])}
        return info


def _qk_heads(model, name: str) -> int:
    """Head count of the llama q/k permutation ``GgufModel.load_weight`` applies to a tensor
    (gguf_conversion.py:285-300), 0 for the others."""
    if model._need_permute_qk_proj:
        if name.endswith(("attn_q.weight", "attn_q.bias")):
            return int(model.model_config["num_attention_heads"])
        if name.endswith(("attn_k.weight", "attn_k.bias")):
            return int(model.model_config["num_key_value_heads"])
    return 0


def _rebuild_model(gguf_module: str, cls_module: str, qualname: str, state: dict):
    """Unpickle a ``GgufModel`` (or subclass) in a worker process: install the B200 path
    into the worker's fresh import of the reference module first, so that the model's
    ``__setstate__`` reopens the file through this module's ``GgufReaderProxy`` and its
    ``load_weight`` converts on the GPU."""
    import importlib
    install(importlib.import_module(gguf_module))
    cls = importlib.import_module(cls_module)
    for part in qualname.split("."):
        cls = getattr(cls, part)
    obj = cls.__new__(cls)
    obj.__setstate__(state)
    return obj


def install(module=None):
    """Route an imported ``sima_lmm.gguf.gguf_conversion`` through the B200 path.

    Replaces the module's ``unpack_gguf_tensor`` and ``GgufReaderProxy`` and makes
    ``GgufModel.load_weight`` apply the llama q/k permutation inside the decode instead
    of on the host afterwards, and ``GgufModel.model_config`` reads the vocabulary size
    from the token embedding's header instead of decoding it.  ``GgufModel`` objects pickled
    for the reference's spawned
    compile workers (``sima_lmm/model/base.py:665-709``) carry the installation with them:
    they unpickle through ``_rebuild_model``, which installs the path in the worker before
    restoring the object.  Returns the module."""
    if module is None:
        import sima_lmm.gguf.gguf_conversion as module  # noqa: PLC0415 (reference package)
    module.unpack_gguf_tensor = unpack_gguf_tensor
    module.GgufReaderProxy = GgufReaderProxy
    model_cls = module.GgufModel
    module_name = module.__name__

    def __reduce_ex__(self, protocol):
        cls = type(self)
        return (_rebuild_model, (module_name, cls.__module__, cls.__qualname__, self.__getstate__()))

    model_cls.__reduce_ex__ = __reduce_ex__

    # model_config decodes the whole token embedding only to read the vocabulary size
    # (gguf_conversion.py:436-437): while it runs, that one load returns an array of the
    # tensor's shape with no columns, read from the tensor's header
    prop = model_cls.__dict__.get("model_config")
    if isinstance(prop, functools.cached_property) and not getattr(prop.func, "_llima_b200", False):
        compute = prop.func

        def model_config(self):
            self._llima_b200_shape_only = True
            try:
                return compute(self)
            finally:
                self.__dict__.pop("_llima_b200_shape_only", None)

        model_config._llima_b200 = True
        model_config.__doc__ = compute.__doc__
        wrapped = functools.cached_property(model_config)
        wrapped.__set_name__(model_cls, "model_config")
        model_cls.model_config = wrapped

    def load_weight(self, name: str, is_hf_name: bool = True, force_float: bool = False):
        if is_hf_name:
            name = self.convert_hf_weight_name(name)
        if name == "token_embd.weight" and self.__dict__.get("_llima_b200_shape_only"):
            return None, np.empty((int(self.tensor_info[name]["shape"][0]), 0), dtype=np.float32)
        proxy = self.gguf_proxy
        if getattr(proxy, "perm_heads_of", 0) is None:
            # the proxy reads ahead with the head counts this model will ask for
            proxy.perm_heads_of = functools.partial(_qk_heads, self)
        return proxy.load_tensor(name, force_float, _qk_heads(self, name))

    model_cls.load_weight = load_weight
    return module
