"""Modalix layout kernel (gq_modalix_layout) against the numpy restatement of
ModelGraph._build_conv (model_graph.py:1012-1079), bit for bit."""
import numpy as np
import pytest
import torch
from ml_dtypes import int4

from llima_b200.layout import modalix_layout, modalix_layout_device, padded_output_channels
from oracle import ggml_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("out_ch,in_ch,block", [(4096, 4096, 32), (1024, 4096, 32), (4096, 14336, 16),
                                                (97, 96, 32), (528, 256, 32), (130, 512, 16), (1, 32, 32)])
def test_layout_matches_build_conv(out_ch, in_ch, block):
    rng = np.random.default_rng(out_ch + in_ch)
    codes = rng.integers(-128, 128, size=(out_ch, in_ch), dtype=np.int8)
    scales = rng.random((out_ch * in_ch // block, 1), dtype=np.float32)
    s, w = modalix_layout(scales, codes)
    s2, w2 = O.modalix_layout(scales, codes, out_ch)
    assert w.shape == w2.shape and s.shape == s2.shape
    assert np.array_equal(w, w2) and np.array_equal(s.view(np.uint32), s2.view(np.uint32))


@pytest.mark.parametrize("out_ch", [528, 784, 1040])
def test_int4_output_padding(out_ch):
    rng = np.random.default_rng(out_ch)
    in_ch = 256
    codes = rng.integers(-8, 8, size=(out_ch, in_ch), dtype=np.int8).astype(int4)
    scales = rng.random((out_ch * in_ch // 32, 1), dtype=np.float32)
    padded = padded_output_channels(out_ch, True)
    assert padded == O.padded_output_channels(out_ch, True) and padded > out_ch
    s, w = modalix_layout(scales, codes, pad_output=True)
    s2, w2 = O.modalix_layout(scales, codes, padded)
    assert w.dtype == int4 and w.shape == (1, 1, in_ch, 1, padded)
    assert np.array_equal(w.view(np.uint8), w2.view(np.uint8))
    assert np.array_equal(s, s2)


def test_layout_of_converted_tensor_on_device():
    from llima_b200 import _native as N
    from llima_b200.device import DeviceTensor, alloc_outputs, convert
    from llima_b200.synth import gen_tensor_bytes
    raw = gen_tensor_bytes("Q4_K", 1024 * 4096, 5)
    t = alloc_outputs(DeviceTensor("Q4_K", 1024, 4096, torch.from_numpy(raw.copy()).cuda()), N.OUT_CODES)
    convert(t, N.OUT_CODES)
    s, c = modalix_layout_device(t.scales, t.codes)
    torch.cuda.synchronize()
    with np.errstate(all="ignore"):
        s0, w0, _ = O.unpack_tensor("Q4_K", raw.tobytes(), (1024, 4096), log=False)
    s2, w2 = O.modalix_layout(s0, w0, 1024)
    assert np.array_equal(c.cpu().numpy(), w2.reshape(4096, 1024))
    assert np.array_equal(s.cpu().numpy(), s2)


def test_layout_against_reference_layout_array_golden():
    from tests.golden_cases import GOLDEN, layout_cases
    for name in layout_cases():
        with np.load(GOLDEN / f"{name}.npz") as z:
            s, w = modalix_layout(z["scales"], z["codes"])
            assert np.array_equal(w, z["out_weight"]) and np.array_equal(s, z["out_scales"])


@pytest.mark.parametrize("fmt,q_size,kv_size,element", [("Q4_K", 4, 2, 8), ("Q6_K", 3, 1, 16), ("Q8_0", 4, 4, 2),
                                                        ("Q4_0", 2, 1, 16), ("Q5_K", 4, 2, 4)])
def test_bundled_qkv_rows_decoded_on_their_own(fmt, q_size, kv_size, element):
    # load_partition(qkv_proj, ...) == _get_array_partition applied to the full decode
    # (model_graph.py:990-998, 1012-1016, 1168-1248), weights and reshaped scales
    import types

    from llima_b200.formats import FORMATS
    from llima_b200.gguf_conversion import load_partition
    from llima_b200.layout import alternate_weight, array_partition
    from llima_b200.synth import gen_tensor_bytes

    f = FORMATS[fmt]
    rows, cols = (q_size + 2 * kv_size) * element, 2 * f.unit_values
    raw = gen_tensor_bytes(fmt, rows * cols, rows + cols)
    tensor = types.SimpleNamespace(tensor_type=f.type_id, data=raw.reshape(rows, -1),
                                   shape=np.array([cols, rows], dtype=np.uint64))
    full_s, full_w, _ = O.unpack_tensor(fmt, raw, (rows, cols), log=False)
    for proj in ("q_proj", "k_proj", "v_proj"):
        fused, count, index, span = alternate_weight(f"blk.0.self_attn.{proj}.weight", q_size, kv_size)
        assert fused == "blk.0.self_attn.qkv_proj.weight"
        r0, r1 = array_partition(rows, count, index, span)
        s, w = load_partition(tensor, count, index, span)
        assert w.shape == (r1 - r0, cols)
        assert np.array_equal(np.asarray(w).view(np.uint8), np.asarray(full_w[r0:r1]).view(np.uint8))
        want_s = np.reshape(full_s, (rows, -1))[r0:r1]
        assert np.array_equal(np.reshape(s, want_s.shape).view(np.uint32), want_s.view(np.uint32))
        _, v = load_partition(tensor, count, index, span, force_float=True)
        full_f = O.gguf_dequantize(raw, fmt).reshape(rows, cols)
        assert np.array_equal(v.view(np.uint32), full_f[r0:r1].view(np.uint32))


def test_bundled_gate_up_and_float_tensors():
    import types

    from llima_b200.formats import FORMATS
    from llima_b200.gguf_conversion import load_partition
    from llima_b200.layout import alternate_weight
    from llima_b200.synth import gen_tensor_bytes

    rows, cols = 48, 512
    raw = gen_tensor_bytes("Q4_K", rows * cols, 9)
    tensor = types.SimpleNamespace(tensor_type=FORMATS["Q4_K"].type_id, data=raw.reshape(rows, -1),
                                   shape=np.array([cols, rows], dtype=np.uint64))
    full_s, full_w, _ = O.unpack_tensor("Q4_K", raw, (rows, cols), log=False)
    for proj, (r0, r1) in (("gate_proj", (0, 24)), ("up_proj", (24, 48))):
        fused, count, index, span = alternate_weight(f"blk.2.mlp.{proj}.weight", None, None)
        assert fused == "blk.2.mlp.gate_up_proj.weight"
        s, w = load_partition(tensor, count, index, span)
        assert np.array_equal(w, full_w[r0:r1])
        assert np.array_equal(np.reshape(s, (24, -1)), np.reshape(full_s, (rows, -1))[r0:r1])
    bias = np.random.default_rng(3).normal(0, 0.02, 96).astype(np.float32)
    bt = types.SimpleNamespace(tensor_type=FORMATS["F32"].type_id, data=bias, shape=np.array([96], dtype=np.uint64))
    s, b = load_partition(bt, 6, 2, 2)
    assert s is None and np.array_equal(b, bias[32:64])
    with pytest.raises(AssertionError):
        load_partition(bt, 7, 0, 1)


# ---------------------------------------------------------------------------------------
# conversion fused with the layout (gq_convert_modalix)
# ---------------------------------------------------------------------------------------

def _fused_case(fmt, rows, cols, heads=0, padded=None, seed=0, expect_fused=True):
    import ctypes

    from llima_b200 import _native as N
    from llima_b200.formats import FORMATS
    from llima_b200.layout import convert_modalix_device
    from llima_b200.synth import gen_tensor_bytes
    from tests.golden_cases import same_bits
    raw = gen_tensor_bytes(fmt, rows * cols, seed + rows + cols)
    src = torch.from_numpy(raw.copy()).cuda()
    padded = rows if padded is None else padded
    if expect_fused is not None:
        # whether the one-pass kernel takes this shape (else the wrapper converts, then lays out)
        f = FORMATS[fmt]
        rec = N.Tensor()
        rec.type, rec.perm_heads, rec.rows, rec.cols = f.type_id, heads, rows, cols
        rec.src, rec.src_bytes = src.data_ptr(), src.numel()
        oc = torch.empty((cols, padded), dtype=torch.int8, device="cuda")
        os_ = torch.empty((cols // f.block_values, padded), dtype=torch.float32, device="cuda")
        rec.codes, rec.scales = oc.data_ptr(), os_.data_ptr()
        st = N.lib().gq_convert_modalix(ctypes.byref(rec), padded, torch.cuda.current_stream().cuda_stream)
        assert (st == 0) == expect_fused, (fmt, rows, cols, st)
    s, c, d = convert_modalix_device(fmt, src, rows, cols, heads, padded)
    torch.cuda.synchronize()
    with np.errstate(all="ignore"):
        s0, w0, dg = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
    if heads:
        s0, w0 = O.permute_qk(s0, w0, heads)
    s2, w2 = O.modalix_layout(s0, w0.view(np.uint8) if fmt == "Q4_0" else w0, padded)
    got_c = c.cpu().numpy().view(np.uint8)
    assert got_c.shape == (cols, padded)
    assert np.array_equal(got_c, w2.reshape(cols, padded).view(np.uint8)), (fmt, rows, cols, heads)
    assert same_bits(s.cpu().numpy(), s2), (fmt, rows, cols, heads)
    if dg is not None:
        from llima_b200.device import diag_values
        r, cl = diag_values(d)
        assert same_bits(np.float32(r), np.float32(dg.round_error)) and int(cl) == int(dg.clip_error)


@pytest.mark.parametrize("fmt,cols", [("Q4_K", 4096), ("Q5_K", 1024), ("Q6_K", 2048), ("Q8_0", 512),
                                      ("Q4_0", 256), ("Q4_1", 512), ("Q5_0", 256), ("Q5_1", 768),
                                      ("Q2_K", 1024), ("Q3_K", 2048)])
@pytest.mark.parametrize("rows", [128, 300, 37, 1])
def test_fused_layout_matches_oracle(fmt, cols, rows):
    _fused_case(fmt, rows, cols)


@pytest.mark.parametrize("fmt,rows,cols,heads", [("Q4_K", 256, 1024, 2), ("Q4_K", 512, 512, 2),
                                                 ("Q6_K", 256, 2048, 8), ("Q8_0", 192, 256, 6),
                                                 ("Q4_K", 4096, 4096, 32), ("Q4_K", 1024, 4096, 8)])
def test_fused_layout_with_head_permutation(fmt, rows, cols, heads):
    # head dims 128, 256 (a head spans two tiles), 32, 32; the Llama-3-8B attn_q / attn_k
    _fused_case(fmt, rows, cols, heads)


@pytest.mark.parametrize("fmt,rows,padded", [("Q4_0", 528, 544), ("Q4_0", 1040, 1056), ("Q4_K", 300, 320)])
def test_fused_layout_output_padding(fmt, rows, padded):
    _fused_case(fmt, rows, 512, padded=padded)


@pytest.mark.parametrize("fmt,rows,cols", [("Q8_0", 40, 96), ("Q6_K", 64, 256), ("Q3_K", 16, 768),
                                           ("Q2_K", 8, 512)])
def test_fused_layout_unsupported_shapes_fall_back(fmt, rows, cols):
    # cols not a multiple of 256, or rows that do not start on 16-byte boundaries: the
    # wrapper converts, then lays out, with the same result
    _fused_case(fmt, rows, cols, expect_fused=False)


def test_fused_layout_full_size_llama_ffn():
    # Llama-3-8B ffn_gate (Q4_K 14336 x 4096) and ffn_down (Q6_K 4096 x 14336)
    _fused_case("Q4_K", 14336, 4096)
    _fused_case("Q6_K", 4096, 14336)


def test_fused_layout_batch_matches_single_calls():
    """gq_convert_modalix_batch over tensors of several types (permuted, padded, ragged rows):
    the same bytes and diagnostics as one gq_convert_modalix call per tensor."""
    import ctypes

    from llima_b200 import _native as N
    from llima_b200.formats import FORMATS
    from llima_b200.synth import gen_tensor_bytes
    specs = [("Q4_K", 256, 1024, 2, 256), ("Q6_K", 300, 2048, 0, 300), ("Q4_K", 37, 512, 0, 37),
             ("Q8_0", 77, 256, 0, 77), ("Q4_0", 528, 512, 0, 544), ("Q5_K", 128, 512, 0, 128),
             ("Q4_K", 1024, 4096, 8, 1024), ("Q6_K", 1, 2048, 0, 1)]
    bufs, singles = [], []
    recs = (N.Tensor * len(specs))()
    padded = (ctypes.c_int64 * len(specs))()
    stream = torch.cuda.current_stream().cuda_stream
    for i, (fmt, rows, cols, heads, pad) in enumerate(specs):
        f = FORMATS[fmt]
        raw = gen_tensor_bytes(fmt, rows * cols, 900 + i)
        src = torch.from_numpy(raw.copy()).cuda()
        outs = []
        for _ in range(2):
            oc = torch.empty((cols, pad), dtype=torch.int8, device="cuda")
            os_ = torch.empty((cols // f.block_values, pad), dtype=torch.float32, device="cuda")
            dg = torch.full((2,), 7, dtype=torch.int32, device="cuda")
            r = N.Tensor()
            r.type, r.perm_heads, r.rows, r.cols = f.type_id, heads, rows, cols
            r.src, r.src_bytes = src.data_ptr(), src.numel()
            r.codes, r.scales, r.diag = oc.data_ptr(), os_.data_ptr(), dg.data_ptr()
            outs.append((r, oc, os_, dg))
        bufs.append((src, outs))
        recs[i] = outs[0][0]
        padded[i] = pad
        N.check(N.lib().gq_convert_modalix(ctypes.byref(outs[1][0]), pad, stream), "gq_convert_modalix")
    N.check(N.lib().gq_convert_modalix_batch(recs, padded, len(specs), stream), "gq_convert_modalix_batch")
    torch.cuda.synchronize()
    for (fmt, *_), (src, outs) in zip(specs, bufs):
        (_, c0, s0, d0), (_, c1, s1, d1) = outs
        assert torch.equal(c0, c1) and torch.equal(s0.view(torch.int32), s1.view(torch.int32)), fmt
        assert torch.equal(d0, d1), fmt
    # and through the Python wrapper's oracle comparison for two of them
    _fused_case("Q5_K", 128, 512)
    _fused_case("Q4_0", 528, 512, padded=544)
