"""Parity of the CUDA path (through the C ABI) with the reference.

* every golden vector produced by the reference itself (tests/golden/);
* the CPU oracle on seeded inputs at the BASELINE tensor shapes (config 1: Q8_0
  4096x4096; config 2: Q4_0 and Q4_K 11008x4096; Q5_K and Q6_K alike);
* the host-buffer path (gq_convert_host) against the device path;
* the standalone requantization scheme against the oracle.

Integer codes, f32 scales and f32 values are compared bit for bit (NaN == NaN).
"""
import ctypes

import ml_dtypes
import numpy as np
import pytest
import torch

from llima_b200 import _native as N
from llima_b200.device import DeviceTensor, alloc_outputs, convert, diag_values
from llima_b200.formats import FORMATS
from llima_b200.synth import gen_tensor_bytes
from oracle import ggml_oracle as O
from tests.golden_cases import case_names, load_case, same_bits

pytestmark = pytest.mark.gpu
BOTH = N.OUT_CODES | N.OUT_F32


def _dev(raw: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(raw).copy()).cuda()


def _codes_np(t: DeviceTensor) -> np.ndarray:
    return t.codes.cpu().numpy()


def _run(fmt, raw, rows, cols, mask=BOTH, heads=0):
    t = DeviceTensor(fmt, rows, cols, _dev(raw), heads)
    alloc_outputs(t, mask)
    convert(t, mask)
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("case", case_names())
def test_golden(case):
    g = load_case(case)
    fmt, rows, cols = g["fmt"], g["rows"], g["cols"]
    heads = g.get("perm_heads", 0)
    if FORMATS[fmt].block_values == 0:
        t = _run(fmt, g["raw"], rows, cols, N.OUT_CODES, heads)
        want = g["perm_codes"] if heads else g["codes"]
        assert same_bits(t.values.cpu().numpy().reshape(want.shape), want)
        return
    t = _run(fmt, g["raw"], rows, cols, BOTH, heads)
    codes = _codes_np(t)
    want_codes = g["perm_codes"] if heads else g["codes"]
    want_scales = g["perm_scales"] if heads else g["scales"]
    assert same_bits(codes.view(np.uint8), want_codes.view(np.uint8)), case
    assert same_bits(t.scales.cpu().numpy(), want_scales), case
    if not heads:
        assert same_bits(t.values.cpu().numpy(), g["f32"]), case
    if FORMATS[fmt].asymmetric:
        with np.errstate(all="ignore"):
            _, _, d = O.unpack_tensor(fmt, g["raw"].tobytes(), (rows, cols), log=False)
        r, c = diag_values(t.diag)
        assert same_bits(np.float32(r), np.float32(d.round_error))
        assert int(c) == int(d.clip_error)


# BASELINE configs 1 and 2 at full size, plus the other two K formats at the same shape
FULL = [("Q8_0", 4096, 4096), ("Q4_0", 11008, 4096), ("Q4_K", 11008, 4096),
        ("Q5_K", 11008, 4096), ("Q6_K", 11008, 4096), ("Q4_1", 4096, 4096), ("Q5_0", 4096, 4096),
        ("Q5_1", 4096, 4096), ("Q2_K", 4096, 4096), ("Q3_K", 4096, 4096)]


@pytest.mark.parametrize("fmt,rows,cols", FULL, ids=[f[0] for f in FULL])
def test_full_size_vs_oracle(fmt, rows, cols):
    raw = gen_tensor_bytes(fmt, rows * cols, 2024)
    t = _run(fmt, raw, rows, cols, BOTH)
    with np.errstate(all="ignore"):
        s, w, d = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
        f32 = O.gguf_dequantize(raw.tobytes(), fmt).reshape(rows, cols)
    wv = w.view(np.uint8) if w.dtype == ml_dtypes.int4 else w
    assert same_bits(_codes_np(t).view(np.uint8), wv.view(np.uint8))
    assert same_bits(t.scales.cpu().numpy(), s)
    assert same_bits(t.values.cpu().numpy(), f32)
    if d is not None:
        r, c = diag_values(t.diag)
        assert same_bits(np.float32(r), np.float32(d.round_error)) and int(c) == int(d.clip_error)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K"])
@pytest.mark.parametrize("mask", [N.OUT_CODES, N.OUT_F32])
def test_single_output_modes_match_both(fmt, mask):
    rows, cols = 64, 2048
    raw = gen_tensor_bytes(fmt, rows * cols, 99)
    both = _run(fmt, raw, rows, cols, BOTH)
    one = _run(fmt, raw, rows, cols, mask)
    if mask == N.OUT_CODES:
        assert torch.equal(one.codes, both.codes) and torch.equal(one.scales.view(torch.int32),
                                                                   both.scales.view(torch.int32))
        assert one.values is None
    else:
        assert torch.equal(one.values.view(torch.int32), both.values.view(torch.int32))
        assert one.codes is None


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K"])
def test_uniform_random_bytes_vs_oracle(fmt):
    # every f16 field random: NaN, inf, subnormal and huge constants
    f = FORMATS[fmt]
    rows, cols = 128, 2048
    n = rows * cols // f.unit_values
    raw = np.frombuffer(np.random.default_rng(5).bytes(n * f.unit_bytes), dtype=np.uint8).copy()
    t = _run(fmt, raw, rows, cols, BOTH)
    with np.errstate(all="ignore"):
        s, w, d = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
        f32 = O.gguf_dequantize(raw.tobytes(), fmt).reshape(rows, cols)
    assert same_bits(_codes_np(t), w)
    assert same_bits(t.scales.cpu().numpy(), s)
    assert same_bits(t.values.cpu().numpy(), f32)


def test_batch_matches_single_and_accumulates_diag():
    from llima_b200.device import DeviceBatch
    specs = [("Q4_K", 48, 1024, 0), ("Q6_K", 40, 512, 0), ("Q4_K", 64, 512, 4), ("Q5_K", 16, 256, 0),
             ("Q8_0", 33, 64, 0), ("Q4_0", 7, 96, 0), ("F32", 64, 1, 4), ("Q6_K", 32, 256, 2)]
    singles, batch = [], []
    for i, (fmt, r, c, h) in enumerate(specs):
        raw = gen_tensor_bytes(fmt, r * c, 300 + i, "bias")
        singles.append(_run(fmt, raw, r, c, N.OUT_CODES, h))
        batch.append(alloc_outputs(DeviceTensor(fmt, r, c, _dev(raw), h), N.OUT_CODES))
    b = DeviceBatch(batch, N.OUT_CODES)
    b.run()
    torch.cuda.synchronize()
    for s, t in zip(singles, batch):
        for name in ("codes", "scales", "values"):
            a, bb = getattr(s, name), getattr(t, name)
            assert (a is None) == (bb is None)
            if a is not None:
                assert torch.equal(a.view(torch.uint8), bb.view(torch.uint8)), (t.fmt, name)
    for i, (s, (fmt, *_)) in enumerate(zip(singles, specs)):
        if FORMATS[fmt].asymmetric:
            assert torch.equal(b.diags[i], s.diag)


def test_permutation_matches_oracle_full_model_shapes():
    # Llama-3-8B attn_q (32 heads) and attn_k (8 heads) at full size
    for rows, heads in ((4096, 32), (1024, 8)):
        raw = gen_tensor_bytes("Q4_K", rows * 4096, rows)
        t = _run("Q4_K", raw, rows, 4096, N.OUT_CODES, heads)
        with np.errstate(all="ignore"):
            s, w, _ = O.unpack_tensor("Q4_K", raw.tobytes(), (rows, 4096), log=False)
        ps, pw = O.permute_qk(s, w, heads)
        assert same_bits(_codes_np(t), pw) and same_bits(t.scales.cpu().numpy(), ps)


@pytest.mark.parametrize("fmt,rows,cols", [("Q4_K", 300, 4096), ("Q6_K", 257, 1024), ("Q8_0", 513, 4096),
                                           ("F32", 4096, 1)])
def test_host_path_matches_device(fmt, rows, cols):
    from llima_b200.gguf_conversion import convert_host
    raw = gen_tensor_bytes(fmt, rows * cols, 7, "norm")
    if fmt == "F32":
        return
    t = _run(fmt, raw, rows, cols, BOTH)
    s, w, d = convert_host(fmt, raw, rows, cols, False)
    _, f, _ = convert_host(fmt, raw, rows, cols, True)
    assert same_bits(w.view(np.uint8), _codes_np(t).view(np.uint8))
    assert same_bits(s, t.scales.cpu().numpy())
    assert same_bits(f, t.values.cpu().numpy())
    if d is not None:
        r, c = diag_values(t.diag)
        assert same_bits(np.float32(d[0]), np.float32(r)) and int(d[1]) == int(c)


def test_host_path_small_staging_splits_tensors(monkeypatch):
    # a 1 MiB staging slot forces pieces: large tensors are split, small ones packed
    from llima_b200 import gguf_conversion as G
    monkeypatch.setenv("LLIMA_B200_STAGING_MB", "1")
    monkeypatch.setattr(G, "_sessions", {})
    raw = gen_tensor_bytes("Q4_K", 2048 * 4096, 8)
    s, w, _ = G.convert_host("Q4_K", raw, 2048, 4096, False)
    with np.errstate(all="ignore"):
        s2, w2, _ = O.unpack_tensor("Q4_K", raw.tobytes(), (2048, 4096), log=False)
    assert same_bits(w, w2) and same_bits(s, s2)


@pytest.mark.parametrize("layout", ["pageable", "pinned", "pinned_in", "pinned_out"])
def test_host_path_pinned_and_pageable_buffers(layout):
    """gq_convert_host with pageable buffers (bounced through the session's pinned slots
    and host copy threads), pinned buffers (copied directly) and both mixed, on a 4 MiB
    staging session so that pieces rotate through every slot several times; results and
    diagnostics equal the device path bit for bit."""
    specs = [("Q4_K", 700, 4096, 0), ("Q6_K", 300, 2048, 0), ("Q4_K", 256, 512, 4), ("Q8_0", 77, 1024, 0),
             ("Q5_K", 33, 2560, 0), ("F32", 5000, 1, 0), ("Q4_0", 129, 96, 0)]
    pin_in = layout in ("pinned", "pinned_in")
    pin_out = layout in ("pinned", "pinned_out")

    def host(shape, dtype, pinned):
        t = torch.empty(shape, dtype=dtype, pin_memory=pinned)
        return t

    recs = (N.Tensor * len(specs))()
    keep, outs, dev = [], [], []
    for i, (fmt, rows, cols, heads) in enumerate(specs):
        f = FORMATS[fmt]
        raw = gen_tensor_bytes(fmt, rows * cols, 50 + i, "norm")
        src = host((raw.size,), torch.uint8, pin_in)
        src.numpy()[:] = raw
        keep.append(src)
        r = N.Tensor()
        r.type, r.perm_heads, r.rows, r.cols = f.type_id, heads, rows, cols
        r.src, r.src_bytes = src.data_ptr(), raw.size
        o = {}
        if f.block_values == 0:
            o["values"] = host((rows, cols), torch.float32, pin_out)
        else:
            o["codes"] = host((rows, cols), torch.int8, pin_out)
            o["scales"] = host((rows * cols // f.block_values, 1), torch.float32, pin_out)
            o["values"] = host((rows, cols), torch.float32, pin_out)
        for name, t in o.items():
            setattr(r, name, t.data_ptr())
        outs.append(o)
        recs[i] = r
        dev.append(_run(fmt, raw, rows, cols, N.OUT_CODES if f.block_values == 0 else BOTH, heads))
    diags = (N.Diag * len(specs))()
    sess = ctypes.c_void_p()
    N.check(N.lib().gq_session_create(0, 4 << 20, ctypes.byref(sess)), "gq_session_create")
    try:
        for _ in range(2):   # a second call reuses the slots and the bounce buffers
            N.check(N.lib().gq_convert_host(sess, recs, len(specs), BOTH, diags), "gq_convert_host")
            for (fmt, *_), o, t, dg in zip(specs, outs, dev, diags):
                for name, h in o.items():
                    want = getattr(t, name)
                    assert torch.equal(h.view(torch.uint8), want.cpu().view(torch.uint8)), (layout, fmt, name)
                if FORMATS[fmt].asymmetric:
                    r, c = diag_values(t.diag)
                    assert np.uint32(dg.round_err_bits) == np.float32(r).view(np.uint32) and dg.clip_err == int(c)
    finally:
        N.lib().gq_session_destroy(sess)


@pytest.mark.parametrize("layout", ["row_slice", "fortran", "step"])
def test_unpack_gguf_tensor_non_contiguous_views(layout):
    """A reader tensor whose data is not one contiguous block (rows cut out of a wider
    buffer, Fortran order, every other row of an interleaved buffer): the result equals
    the oracle on the same bytes."""
    import types
    from llima_b200.gguf_conversion import unpack_gguf_tensor
    fmt, rows, cols = "Q4_K", 64, 512
    raw = gen_tensor_bytes(fmt, rows * cols, 91)
    rb = raw.size // rows
    if layout == "row_slice":
        wide = np.zeros((rows, rb + 48), dtype=np.uint8)
        wide[:, :rb] = raw.reshape(rows, rb)
        data = wide[:, :rb]
    elif layout == "fortran":
        data = np.asfortranarray(raw.reshape(rows, rb))
    else:
        both = np.zeros((2 * rows, rb), dtype=np.uint8)
        both[::2] = raw.reshape(rows, rb)
        data = both[::2]
    assert not data.flags.c_contiguous
    t = types.SimpleNamespace(tensor_type=FORMATS[fmt].type_id, data=data,
                              shape=np.array([cols, rows], dtype=np.uint64))
    s, w = unpack_gguf_tensor(t, False)
    with np.errstate(all="ignore"):
        s2, w2, _ = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
    assert same_bits(w, w2) and same_bits(s, s2)


@pytest.mark.parametrize("heads,staging_mb", [(32, 4), (8, 12), (32, 256)])
def test_host_path_permuted_tensor_larger_than_a_slot(heads, staging_mb):
    """A q/k-permuted tensor larger than the session's staging slot is cut into pieces of
    whole heads (the permutation never crosses a head): the Llama-3-8B attn_q (32 heads)
    and attn_k shapes, codes and f32 values, against the device path."""
    rows = 4096 if heads == 32 else 1024
    raw = gen_tensor_bytes("Q4_K", rows * 4096, heads + staging_mb)
    t = _run("Q4_K", raw, rows, 4096, BOTH, heads)
    rec = N.Tensor()
    rec.type, rec.perm_heads, rec.rows, rec.cols = FORMATS["Q4_K"].type_id, heads, rows, 4096
    rec.src, rec.src_bytes = raw.ctypes.data, raw.size
    codes = np.empty((rows, 4096), dtype=np.int8)
    scales = np.empty((rows * 4096 // 32, 1), dtype=np.float32)
    values = np.empty((rows, 4096), dtype=np.float32)
    rec.codes, rec.scales, rec.values = codes.ctypes.data, scales.ctypes.data, values.ctypes.data
    diag = N.Diag()
    sess = ctypes.c_void_p()
    N.check(N.lib().gq_session_create(0, staging_mb << 20, ctypes.byref(sess)), "gq_session_create")
    try:
        N.check(N.lib().gq_convert_host(sess, ctypes.byref(rec), 1, BOTH, ctypes.byref(diag)), "gq_convert_host")
    finally:
        N.lib().gq_session_destroy(sess)
    assert same_bits(codes, _codes_np(t)) and same_bits(scales, t.scales.cpu().numpy())
    assert same_bits(values, t.values.cpu().numpy())
    r, c = diag_values(t.diag)
    assert np.uint32(diag.round_err_bits) == np.float32(r).view(np.uint32) and diag.clip_err == int(c)


def test_host_path_head_larger_than_a_slot_is_refused():
    rec = N.Tensor()
    rec.type, rec.perm_heads, rec.rows, rec.cols = FORMATS["Q4_K"].type_id, 2, 4096, 4096
    raw = np.zeros(4096 * 16 * 144, dtype=np.uint8)
    out = np.zeros(4096 * 4096, dtype=np.int8)
    sc = np.zeros(4096 * 128, dtype=np.float32)
    rec.src, rec.src_bytes, rec.codes, rec.scales = raw.ctypes.data, raw.size, out.ctypes.data, sc.ctypes.data
    sess = ctypes.c_void_p()
    N.check(N.lib().gq_session_create(0, 4 << 20, ctypes.byref(sess)), "gq_session_create")
    try:
        # one head is 2048 rows x 4096 columns: about 15 MB of slot footprint
        assert N.lib().gq_convert_host(sess, ctypes.byref(rec), 1, N.OUT_CODES, None) == -2
    finally:
        N.lib().gq_session_destroy(sess)


def test_convert_gguf_file_matches_per_tensor_decode(tmp_path):
    """convert_gguf_file: every tensor of a llama GGUF file in one host call, with the q/k
    permutation taken from the file's architecture and head counts, equal to the oracle's
    unpack (+ _permute_qk_proj) of each tensor; a subset by name; force_float."""
    gguf = pytest.importorskip("gguf")
    from llima_b200.gguf_conversion import convert_gguf_file
    path = tmp_path / "m.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(1)
    w.add_head_count(8)
    w.add_head_count_kv(2)
    specs = {"token_embd.weight": ("Q6_K", 96, 512), "blk.0.attn_q.weight": ("Q4_K", 512, 512),
             "blk.0.attn_k.weight": ("Q5_K", 128, 512), "blk.0.attn_v.weight": ("Q8_0", 128, 512),
             "blk.0.ffn_up.weight": ("Q4_0", 300, 512), "blk.0.ffn_down.weight": ("Q2_K", 512, 768)}
    raws = {}
    for i, (name, (fmt, r, c)) in enumerate(specs.items()):
        raw = gen_tensor_bytes(fmt, r * c, 60 + i)
        w.add_tensor(name, raw.reshape(r, -1), raw_shape=(r, raw.size // r),
                     raw_dtype=getattr(gguf.GGMLQuantizationType, fmt))
        raws[name] = raw
    norm = np.random.default_rng(2).normal(1, 0.02, 512).astype(np.float32)
    w.add_tensor("blk.0.attn_norm.weight", norm)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    got = convert_gguf_file(path)
    assert set(got) == set(specs) | {"blk.0.attn_norm.weight"}
    heads = {"blk.0.attn_q.weight": 8, "blk.0.attn_k.weight": 2}
    for name, (fmt, r, c) in specs.items():
        with np.errstate(all="ignore"):
            s2, q2, _ = O.unpack_tensor(fmt, raws[name].tobytes(), (r, c), log=False)
        if name in heads:
            s2, q2 = O.permute_qk(s2, q2, heads[name])
        s, q = got[name]
        assert q.dtype == q2.dtype and q.shape == (r, c), name
        assert same_bits(q.view(np.uint8), q2.view(np.uint8)) and same_bits(s, s2), name
    assert got["blk.0.attn_norm.weight"][0] is None
    assert np.array_equal(got["blk.0.attn_norm.weight"][1], norm)
    sub = convert_gguf_file(path, names=["blk.0.attn_v.weight"], permute_qk=False)
    assert list(sub) == ["blk.0.attn_v.weight"]
    ff = convert_gguf_file(path, names=["blk.0.ffn_down.weight"], force_float=True)
    want = O.gguf_dequantize(raws["blk.0.ffn_down.weight"].tobytes(), "Q2_K").reshape(512, 768)
    assert ff["blk.0.ffn_down.weight"][0] is None and same_bits(ff["blk.0.ffn_down.weight"][1], want)


def test_unpack_gguf_tensor_dropin_reader(tmp_path):
    gguf = pytest.importorskip("gguf")
    from llima_b200.gguf_conversion import GgufReaderProxy
    path = tmp_path / "t.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    tensors = {}
    for i, (fmt, r, c) in enumerate([("Q4_K", 8, 512), ("Q6_K", 4, 256), ("Q8_0", 6, 64), ("Q4_0", 3, 32)]):
        raw = gen_tensor_bytes(fmt, r * c, 40 + i)
        name = f"blk.0.t{i}.weight"
        w.add_tensor(name, raw.reshape(r, -1), raw_shape=(r, raw.size // r),
                     raw_dtype=getattr(gguf.GGMLQuantizationType, fmt))
        tensors[name] = (fmt, raw, r, c)
    norm = np.random.default_rng(1).normal(1, 0.02, 64).astype(np.float32)
    w.add_tensor("blk.0.attn_norm.weight", norm)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    proxy = GgufReaderProxy(path)
    for name, (fmt, raw, r, c) in tensors.items():
        s, q = proxy.load_tensor(name, False)
        with np.errstate(all="ignore"):
            s2, q2, _ = O.unpack_tensor(fmt, raw.tobytes(), (r, c), log=False)
        assert q.dtype == q2.dtype and q.shape == (r, c)
        assert same_bits(q.view(np.uint8), q2.view(np.uint8)) and same_bits(s, s2)
        _, f = proxy.load_tensor(name, True)
        assert same_bits(f, O.gguf_dequantize(raw.tobytes(), fmt).reshape(r, c))
    s, n = proxy.load_tensor("blk.0.attn_norm.weight", False)
    assert s is None and np.array_equal(n, norm)


def test_requantize_symmetric_scheme_vs_oracle():
    rng = np.random.default_rng(11)
    n, block = 5000, 32
    bc = np.stack([rng.uniform(-1e-2, 1e-2, n), -rng.uniform(0, 0.3, n)], 1).astype(np.float32)
    bc[::17, 0] = 0
    bc[::23, 1] = 0
    q = rng.integers(0, 32, size=(n, block), dtype=np.int8)
    dq, dbc = torch.from_numpy(q).cuda(), torch.from_numpy(bc).cuda()
    out_s = torch.empty(n, dtype=torch.float32, device="cuda")
    out_q = torch.empty((n, block), dtype=torch.int8, device="cuda")
    diag = torch.zeros(2, dtype=torch.int32, device="cuda")
    N.check(N.lib().gq_requantize_symmetric(dbc.data_ptr(), dq.data_ptr(), n, block, 8, out_s.data_ptr(),
                                            out_q.data_ptr(), diag.data_ptr(), None), "requant")
    torch.cuda.synchronize()
    with np.errstate(all="ignore"):
        s, q2, d = O.requantize_symmetric(bc, q, 8, np.int8, log=False)
    assert same_bits(out_s.cpu().numpy().reshape(-1, 1), s)
    assert same_bits(out_q.cpu().numpy(), q2)
    r, c = diag_values(diag)
    assert same_bits(np.float32(r), np.float32(d.round_error)) and int(c) == int(d.clip_error)


def test_invalid_arguments_return_errors_without_launch():
    lib = N.lib()
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    t = N.Tensor()
    t.type, t.rows, t.cols = 12, 1, 256
    t.src, t.src_bytes = buf.data_ptr() + 1, 144   # misaligned source
    t.codes, t.scales = buf.data_ptr() + 1024, buf.data_ptr() + 2048
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == -3
    t.src = buf.data_ptr()
    t.src_bytes = 100                               # too short
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == -2
    t.src_bytes = 144
    t.scales = None                                 # missing output
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == -4
    t.scales = buf.data_ptr() + 2048
    assert lib.gq_convert(ctypes.byref(t), 7, None) == -5
    t.perm_heads = 3                                # rows not divisible by 2*heads
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == -5
    t.perm_heads = 0
    t.type = 9                                      # Q8_1: not on this path
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == -1
    t.type, t.rows = 12, 0                          # empty tensor: nothing to do
    assert lib.gq_convert(ctypes.byref(t), N.OUT_CODES, None) == 0
    torch.cuda.synchronize()


def test_empty_asymmetric_tensor_raises_like_reference():
    from llima_b200.gguf_conversion import convert_host
    with pytest.raises(ValueError, match="zero-size array"):
        convert_host("Q4_K", np.zeros(0, dtype=np.uint8), 0, 256)
    s, w, _ = convert_host("Q6_K", np.zeros(0, dtype=np.uint8), 0, 256)
    assert s.shape == (0, 1) and w.shape == (0, 256)


def _force_rare(raw: np.ndarray, fmt: str, rows: int, cols: int, seed: int) -> np.ndarray:
    """Q4_K / Q5_K bytes in which chosen super-blocks have d = f16(1e-4), every 6-bit scale 1
    and every min 63, so that |M/S| >= 63 and nearly all their blocks need a scale factor
    below 0.98 (blocks the fast path leaves).  The density changes by row quarter: 1%, 30%
    (more such blocks per sub-tile than the kernel's queue holds), 3% with one in seven of
    them given an inf or NaN d, and none."""
    f = FORMATS[fmt]
    u = raw.reshape(-1, f.unit_bytes)
    rng = np.random.default_rng(seed)
    quarter = (np.arange(u.shape[0]) // (cols // 256)) * 4 // rows
    pick = rng.random(u.shape[0]) < np.array([0.01, 0.30, 0.03, 0.0])[quarter]
    u[pick, 0:2] = np.frombuffer(np.float16(1e-4).tobytes(), np.uint8)
    u[pick, 4:8] = 0x01
    u[pick, 8:12] = 0xFF
    u[pick, 12:16] = 0xF1
    odd = pick & (quarter == 2) & (rng.random(u.shape[0]) < 1 / 7)
    u[odd, 0:2] = np.frombuffer(np.array([np.inf], np.float16).tobytes(), np.uint8)
    u[odd & (rng.random(u.shape[0]) < 0.5), 0:2] = np.frombuffer(np.array([np.nan], np.float16).tobytes(), np.uint8)
    return raw


@pytest.mark.parametrize("fmt", ["Q4_K", "Q5_K"])
@pytest.mark.parametrize("rows,heads", [(2048, 0), (2048, 16), (65536, 0), (65536, 512)])
def test_rare_blocks_dense_and_sparse(fmt, rows, heads):
    """Blocks that the integer-scale-factor path leaves, sparse (finished in batches from a
    per-warp queue), dense (past the queue: finished one warp pass each) and with non-finite
    constants, at a size that takes the small tiles (2048 rows) and one that takes the large
    tiles (65536 rows), with and without the q/k head permutation: codes, scales and the
    diagnostics equal the oracle's bit for bit (the oracle runs on row chunks of whole heads)."""
    cols = 4096
    raw = _force_rare(gen_tensor_bytes(fmt, rows * cols, 4321 + rows), fmt, rows, cols, rows + heads)
    t = _run(fmt, raw, rows, cols, N.OUT_CODES, heads)
    codes = _codes_np(t)
    scales = t.scales.cpu().numpy().reshape(rows, cols // 32)
    f = FORMATS[fmt]
    row_bytes = cols // 256 * f.unit_bytes
    chunk = 4096 if heads == 0 else max(4096 // (rows // heads), 1) * (rows // heads)
    chunk = min(chunk, rows)
    round_err, clip_err = np.float32(0), 0
    for r0 in range(0, rows, chunk):
        part = raw[r0 * row_bytes:(r0 + chunk) * row_bytes]
        with np.errstate(all="ignore"):
            s, w, d = O.unpack_tensor(fmt, part.tobytes(), (chunk, cols), log=False)
        if heads:
            s, w = O.permute_qk(s, w, chunk // (rows // heads))
        assert same_bits(codes[r0:r0 + chunk], w), (fmt, rows, heads, r0)
        assert same_bits(scales[r0:r0 + chunk], s.reshape(chunk, cols // 32)), (fmt, rows, heads, r0)
        if np.isnan(d.round_error) or d.round_error.view(np.uint32) > round_err.view(np.uint32):
            round_err = np.float32(d.round_error)
        clip_err = max(clip_err, int(d.clip_error))
    r, c = diag_values(t.diag)
    assert same_bits(np.float32(r), round_err) and int(c) == clip_err
