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
