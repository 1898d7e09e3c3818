"""Parity of whole benchmark model sets through the batch API, at full size.

Every tensor of the Llama-3-8B Q4_K_M set and of the Qwen2.5-7B Q5_K / Q8_0 set, and of
a four-layer cut of the Llama-3-70B set (its hidden, FFN, head and vocabulary shapes), is
converted in one ``gq_convert_batch`` call, the way ``bench.py`` times it: one launch per
GGML type holding up to 128 tensors, so the 160 Q4_K tensors of the 8B set take two.  The
oracle cannot convert 5-6 GB in test time, but rows convert independently: a row's codes
and block scales depend only on that row's GGUF bytes (``unpack_gguf_tensor`` reshapes
row-major blocks, ``gguf_conversion.py:174-176``).  So a seeded sample of rows of every
tensor -- always including its first and last row -- is compared bit for bit with the
CPU oracle, permuted q/k rows at their permuted place (``gguf_conversion.py:314-332``).
The diagnostics of each tensor (maxima over all its blocks) must be at least those of its
sampled rows.
"""
import numpy as np
import pytest
import torch

from llima_b200 import _native as N
from llima_b200.device import DeviceBatch, DeviceTensor, alloc_outputs, diag_values
from llima_b200.formats import FORMATS
from llima_b200.synth import gen_tensor_bytes_torch, head_count_for, model_specs
from oracle import ggml_oracle as O
from tests.golden_cases import same_bits

ROWS_PER_TENSOR = 12


def _specs(model: str, layers: int | None):
    sp = model_specs(model)
    if layers is None:
        return sp
    keep = {f"blk.{i}." for i in range(layers)}
    return [s for s in sp if not s.name.startswith("blk.") or any(s.name.startswith(k) for k in keep)]


def _permuted_row(r: int, rows: int, heads: int) -> int:
    # rows (H, D/2, 2) -> (H, 2, D/2): source row h*D + 2a + t lands on h*D + t*D/2 + a
    d = rows // heads
    h, rem = divmod(r, d)
    a, t = divmod(rem, 2)
    return h * d + t * (d // 2) + a


def test_sampled_rows_premise_on_cpu():
    """The premise above, on the CPU: the oracle on a few rows equals those rows of the
    whole tensor's conversion, and _permuted_row finds them after the q/k permutation."""
    from llima_b200.synth import gen_tensor_bytes
    rows, cols, heads = 64, 512, 4
    for fmt in ("Q4_K", "Q6_K", "Q5_K", "Q8_0"):
        f = FORMATS[fmt]
        raw = gen_tensor_bytes(fmt, rows * cols, 11)
        with np.errstate(all="ignore"):
            s_all, w_all, _ = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
        s_perm, w_perm = O.permute_qk(s_all, w_all, heads)
        row_bytes = cols // f.unit_values * f.unit_bytes
        pick = np.array([0, 5, 17, 32, 63])
        sub = raw.reshape(rows, row_bytes)[pick]
        with np.errstate(all="ignore"):
            s_sub, w_sub, _ = O.unpack_tensor(fmt, sub.tobytes(), (len(pick), cols), log=False)
        out = np.array([_permuted_row(int(r), rows, heads) for r in pick])
        assert same_bits(w_perm.reshape(rows, cols)[out].view(np.uint8), w_sub.view(np.uint8))
        assert same_bits(s_perm.reshape(rows, -1)[out], s_sub.reshape(len(pick), -1))


@pytest.mark.gpu
@pytest.mark.parametrize("model,layers", [("llama3-8b", None), ("qwen2.5-7b", None), ("llama3-70b", 4)],
                         ids=["llama3-8b", "qwen2.5-7b", "llama3-70b-4layers"])
def test_model_set_sampled_rows_vs_oracle(model, layers):
    dev = torch.device("cuda", 0)
    specs = _specs(model, layers)
    tensors = []
    for s in specs:
        src = gen_tensor_bytes_torch(s.fmt, s.n_values, s.seed, dev, s.kind)
        t = DeviceTensor(s.fmt, s.rows, s.cols, src, head_count_for(model, s.name), name=s.name)
        tensors.append(alloc_outputs(t, N.OUT_CODES))
    batch = DeviceBatch(tensors, N.OUT_CODES)
    batch.run()
    torch.cuda.synchronize()
    assert any(t.perm_heads for t in tensors) == model.startswith("llama")

    rng = np.random.default_rng(7)
    checked = 0
    for i, t in enumerate(tensors):
        f = FORMATS[t.fmt]
        row_bytes = t.cols // f.unit_values * f.unit_bytes
        rows = np.unique(np.concatenate([[0, t.rows - 1], rng.integers(0, t.rows, ROWS_PER_TENSOR - 2)]))
        src = t.src[:t.rows * row_bytes].view(t.rows, row_bytes)[torch.from_numpy(rows).to(dev)].cpu().numpy()
        out_rows = rows if not t.perm_heads else np.array([_permuted_row(int(r), t.rows, t.perm_heads)
                                                           for r in rows])
        sel = torch.from_numpy(out_rows).to(dev)
        with np.errstate(all="ignore"):
            s_ref, w_ref, d_ref = O.unpack_tensor(t.fmt, src.tobytes(), (len(rows), t.cols), log=False)
        if f.block_values == 0:
            got = t.values[sel].cpu().numpy()
            assert same_bits(got.reshape(w_ref.shape), w_ref), t.name
        else:
            codes = t.codes[sel].cpu().numpy().view(np.uint8)
            scales = t.scales.view(t.rows, -1)[sel].cpu().numpy()
            assert same_bits(codes, w_ref.view(np.uint8).reshape(codes.shape)), t.name
            assert same_bits(scales, s_ref.reshape(scales.shape)), t.name
            if d_ref is not None:
                r_all, c_all = diag_values(batch.diags[i])
                assert r_all >= d_ref.round_error and int(c_all) >= int(d_ref.clip_error), t.name
        checked += len(rows)
    assert checked >= 2 * len(tensors)
    del tensors, batch
    torch.cuda.empty_cache()
