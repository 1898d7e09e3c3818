"""Seeded synthetic GGUF tensors and model-shaped tensor sets.

The reference publishes no benchmark data for this path, so the benchmark configs are
seeded synthetic tensors with the shapes and value distributions of real GGUF files:

* Q8_0: per 32-value block an f16 scale d ~ U[1e-4, 1e-2] and 32 int8 ~ U[-127, 127].
* Q4_0: f16 d ~ U[1e-4, 1e-2] and 16 bytes of uniform nibbles.
* Q4_K / Q5_K: f16 d and dmin ~ U[1e-4, 1e-2], 8 (scale, min) pairs ~ U{0..63} packed
  into 12 bytes (the inverse of the 6-bit unpack in ``sima_lmm/gguf/ggml_quant.py:352-375``),
  uniform nibble bytes and (Q5_K) uniform high-bit bytes.
* Q6_K: uniform ql/qh bytes, 16 int8 sub-scales ~ U[-64, 63], f16 d ~ U[1e-4, 1e-2].
* F32 norm weights ~ N(1, 0.02), biases ~ N(0, 0.02).

Model sets follow the layer shapes of Llama-3-8B, Qwen2.5-7B and Llama-3-70B with the
per-tensor formats of a Q4_K_M / mixed Q5_K-Q8_0 file.  Tensor names use GGUF naming
(``blk.N.attn_q.weight`` ...) and shapes are (rows, cols) as the reference returns them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .formats import FORMATS

__all__ = ["TensorSpec", "model_specs", "gen_tensor_bytes", "MODEL_SETS"]


@dataclass(frozen=True)
class TensorSpec:
    name: str
    fmt: str
    rows: int
    cols: int              # 1-D tensors: rows = length, cols = 1
    seed: int
    kind: str = "weight"   # "weight" | "norm" | "bias"

    @property
    def n_values(self) -> int:
        return self.rows * self.cols

    @property
    def nbytes(self) -> int:
        f = FORMATS[self.fmt]
        return self.n_values // f.unit_values * f.unit_bytes


def _f16_uniform(rng, n, lo=1e-4, hi=1e-2) -> np.ndarray:
    return rng.uniform(lo, hi, n).astype(np.float16).view(np.uint8).reshape(n, 2)


def _pack_6bit(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """8 scales and 8 mins (each 0..63) -> 12 bytes; inverse of the reference's 6-bit unpack."""
    out = np.empty((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, :4] & 0x3F) | ((sc[:, 4:] >> 4) << 6)
    out[:, 4:8] = (mn[:, :4] & 0x3F) | ((mn[:, 4:] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:] & 0x0F) | ((mn[:, 4:] & 0x0F) << 4)
    return out


def gen_tensor_bytes(fmt: str, n_values: int, seed: int, kind: str = "weight") -> np.ndarray:
    """Raw GGUF bytes (uint8, flat) of one synthetic tensor."""
    rng = np.random.default_rng(seed)
    f = FORMATS[fmt]
    if fmt == "F32":
        mean = 1.0 if kind == "norm" else 0.0
        return rng.normal(mean, 0.02, n_values).astype(np.float32).view(np.uint8)
    if fmt in ("F16", "BF16"):
        raise ValueError("no synthetic generator for 16-bit float tensors")
    n = n_values // f.unit_values
    u = np.frombuffer(rng.bytes(n * f.unit_bytes), dtype=np.uint8).reshape(n, f.unit_bytes).copy()
    if fmt == "Q8_0":
        u[:, 0:2] = _f16_uniform(rng, n)
        u[:, 2:34] = rng.integers(-127, 128, size=(n, 32), dtype=np.int8).view(np.uint8)
    elif fmt == "Q4_0":
        u[:, 0:2] = _f16_uniform(rng, n)
    elif fmt in ("Q4_K", "Q5_K"):
        u[:, 0:2] = _f16_uniform(rng, n)
        u[:, 2:4] = _f16_uniform(rng, n)
        sc = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        u[:, 4:16] = _pack_6bit(sc, mn)
    elif fmt == "Q6_K":
        u[:, 192:208] = rng.integers(-64, 64, size=(n, 16), dtype=np.int8).view(np.uint8)
        u[:, 208:210] = _f16_uniform(rng, n)
    elif fmt in ("Q4_1", "Q5_1"):
        u[:, 0:2] = _f16_uniform(rng, n)
        u[:, 2:4] = _f16_uniform(rng, n, -0.15, 0.0)    # the block minimum
    elif fmt == "Q5_0":
        u[:, 0:2] = _f16_uniform(rng, n)
    elif fmt == "Q2_K":
        u[:, 80:82] = _f16_uniform(rng, n)
        u[:, 82:84] = _f16_uniform(rng, n)
    elif fmt == "Q3_K":
        u[:, 108:110] = _f16_uniform(rng, n)
    else:
        raise ValueError(f"unsupported synthetic format {fmt}")
    return u.reshape(-1)


def gen_tensor_bytes_torch(fmt: str, n_values: int, seed: int, device, kind: str = "weight"):
    """Same distributions as ``gen_tensor_bytes``, generated with torch on `device` (the
    byte streams differ from the numpy generator's).  Uniform bytes in the 12 packed
    scale bytes of Q4_K/Q5_K are exactly uniform (scale, min) pairs, since the 6-bit
    packing is a bijection between 16 six-bit values and 12 bytes."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    f = FORMATS[fmt]
    if fmt == "F32":
        mean = 1.0 if kind == "norm" else 0.0
        x = torch.empty(n_values, dtype=torch.float32, device=device).normal_(mean, 0.02, generator=g)
        return x.view(torch.uint8)
    n = n_values // f.unit_values
    u = torch.randint(0, 256, (n, f.unit_bytes), dtype=torch.uint8, device=device, generator=g)

    def f16_field():
        x = torch.empty(n, dtype=torch.float32, device=device).uniform_(1e-4, 1e-2, generator=g)
        return x.to(torch.float16).view(torch.uint8).view(n, 2)

    if fmt == "Q8_0":
        u[:, 0:2] = f16_field()
        u[:, 2:34] = torch.randint(-127, 128, (n, 32), dtype=torch.int8, device=device, generator=g).view(torch.uint8)
    elif fmt == "Q4_0":
        u[:, 0:2] = f16_field()
    elif fmt in ("Q4_K", "Q5_K"):
        u[:, 0:2] = f16_field()
        u[:, 2:4] = f16_field()
    elif fmt == "Q6_K":
        u[:, 192:208] = ((u[:, 192:208] & 0x7F).to(torch.int16) - 64).to(torch.int8).view(torch.uint8)
        u[:, 208:210] = f16_field()
    else:
        raise ValueError(f"unsupported synthetic format {fmt}")
    return u.reshape(-1)


@dataclass(frozen=True)
class ModelShape:
    layers: int
    hidden: int
    ffn: int
    n_head: int
    n_kv: int
    head_dim: int
    vocab: int
    proj_fmt: dict           # tensor role -> format
    embd_fmt: str
    out_fmt: str
    qkv_bias: bool


_Q4KM = {"attn_q": "Q4_K", "attn_k": "Q4_K", "attn_v": "Q6_K", "attn_output": "Q4_K",
         "ffn_gate": "Q4_K", "ffn_up": "Q4_K", "ffn_down": "Q6_K"}
_Q5K = {r: "Q5_K" for r in _Q4KM}

MODEL_SETS: dict[str, ModelShape] = {
    "llama3-8b": ModelShape(32, 4096, 14336, 32, 8, 128, 128256, _Q4KM, "Q6_K", "Q6_K", False),
    "qwen2.5-7b": ModelShape(28, 3584, 18944, 28, 4, 128, 152064, _Q5K, "Q8_0", "Q8_0", True),
    "llama3-70b": ModelShape(80, 8192, 28672, 64, 8, 128, 128256, _Q4KM, "Q6_K", "Q6_K", False),
}


def model_specs(model: "str | ModelShape", seed: int = 0) -> list[TensorSpec]:
    """Tensor list of a model-shaped set (a MODEL_SETS name or a ModelShape), in GGUF
    file order."""
    m = MODEL_SETS[model] if isinstance(model, str) else model
    q_rows = m.n_head * m.head_dim
    kv_rows = m.n_kv * m.head_dim
    specs: list[TensorSpec] = []

    def add(name, fmt, rows, cols, kind="weight"):
        specs.append(TensorSpec(name, fmt, rows, cols, seed * 1_000_003 + len(specs), kind))

    add("token_embd.weight", m.embd_fmt, m.vocab, m.hidden)
    for i in range(m.layers):
        p = f"blk.{i}."
        add(p + "attn_norm.weight", "F32", m.hidden, 1, "norm")
        add(p + "attn_q.weight", m.proj_fmt["attn_q"], q_rows, m.hidden)
        add(p + "attn_k.weight", m.proj_fmt["attn_k"], kv_rows, m.hidden)
        add(p + "attn_v.weight", m.proj_fmt["attn_v"], kv_rows, m.hidden)
        if m.qkv_bias:
            add(p + "attn_q.bias", "F32", q_rows, 1, "bias")
            add(p + "attn_k.bias", "F32", kv_rows, 1, "bias")
            add(p + "attn_v.bias", "F32", kv_rows, 1, "bias")
        add(p + "attn_output.weight", m.proj_fmt["attn_output"], m.hidden, q_rows)
        add(p + "ffn_norm.weight", "F32", m.hidden, 1, "norm")
        add(p + "ffn_gate.weight", m.proj_fmt["ffn_gate"], m.ffn, m.hidden)
        add(p + "ffn_up.weight", m.proj_fmt["ffn_up"], m.ffn, m.hidden)
        add(p + "ffn_down.weight", m.proj_fmt["ffn_down"], m.hidden, m.ffn)
    add("output_norm.weight", "F32", m.hidden, 1, "norm")
    add("output.weight", m.out_fmt, m.vocab, m.hidden)
    return specs


def head_count_for(model: "str | ModelShape", tensor_name: str, llama: bool | None = None) -> int:
    """Heads of the Llama q/k row permutation (0 when the tensor is not permuted).
    ``sima_lmm/gguf/gguf_conversion.py:291-299`` applies it to attn_q/attn_k of llama models."""
    if llama is None:
        llama = isinstance(model, str) and model.startswith("llama")
    if not llama:
        return 0
    m = MODEL_SETS[model] if isinstance(model, str) else model
    if tensor_name.endswith(("attn_q.weight", "attn_q.bias")):
        return m.n_head
    if tensor_name.endswith(("attn_k.weight", "attn_k.bias")):
        return m.n_kv
    return 0
