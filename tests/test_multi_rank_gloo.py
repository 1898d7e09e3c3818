"""Multi-rank sharding on CPU: world size 2 over gloo.

Each rank plans the shards of a small llama-shaped model (``llima_b200.shard``), converts
its own pieces with the CPU oracle, and the per-row results gathered from both ranks must
equal a single-process conversion of the whole model; the timing reduction is the max
over ranks, as in bench.py.  No GPU is involved (the oracle stands in for the kernels,
whose parity is tested separately).
"""
import hashlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llima_b200.formats import FORMATS
from llima_b200.shard import plan_shards
from llima_b200.synth import ModelShape, gen_tensor_bytes, head_count_for, model_specs

_Q4KM = {"attn_q": "Q4_K", "attn_k": "Q4_K", "attn_v": "Q6_K", "attn_output": "Q4_K",
         "ffn_gate": "Q4_K", "ffn_up": "Q4_K", "ffn_down": "Q6_K"}
TINY = ModelShape(2, 256, 512, 4, 2, 64, 384, _Q4KM, "Q6_K", "Q8_0", False)


def _convert_rows(spec, r0, r1):
    """Oracle conversion of rows [r0, r1) of a tensor: digest of codes and scales per row."""
    from oracle import ggml_oracle as O
    f = FORMATS[spec.fmt]
    raw = gen_tensor_bytes(spec.fmt, spec.n_values, spec.seed, spec.kind)
    row_bytes = spec.cols // f.unit_values * f.unit_bytes
    part = raw[r0 * row_bytes:r1 * row_bytes].tobytes()
    with np.errstate(all="ignore"):
        s, w, _ = O.unpack_tensor(spec.fmt, part, (r1 - r0, spec.cols), log=False)
    heads = head_count_for(TINY, spec.name, llama=True)
    if heads and (r0, r1) == (0, spec.rows):
        s, w = O.permute_qk(s, w, heads)
    w = np.ascontiguousarray(w).view(np.uint8).reshape(r1 - r0, -1)
    s = None if s is None else np.ascontiguousarray(s).reshape(r1 - r0, -1)
    rows = []
    for i in range(r1 - r0):
        h = hashlib.sha256(w[i].tobytes())
        if s is not None:
            h.update(s[i].tobytes())
        rows.append(h.hexdigest())
    return rows


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        specs = model_specs(TINY, seed=3)
        items = [(s.fmt, s.rows, s.cols, head_count_for(TINY, s.name, llama=True) > 0) for s in specs]
        plan = plan_shards(items, world)
        mine = {}
        for p in plan[rank]:
            mine[(p.index, p.row0, p.row1)] = _convert_rows(specs[p.index], p.row0, p.row1)
        gathered = [None] * world
        dist.all_gather_object(gathered, {"plan": plan, "rows": mine})
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out.put((gathered, float(t.item())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_cover_the_model_exactly_once():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=600)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert tmax == float(world)
    # every rank derived the same plan
    assert all(g["plan"] == gathered[0]["plan"] for g in gathered)
    specs = model_specs(TINY, seed=3)
    merged = {i: [None] * s.rows for i, s in enumerate(specs)}
    for g in gathered:
        for (idx, r0, r1), rows in g["rows"].items():
            for k, h in enumerate(rows):
                assert merged[idx][r0 + k] is None, "row converted twice"
                merged[idx][r0 + k] = h
    for i, s in enumerate(specs):
        assert merged[i] == _convert_rows(s, 0, s.rows), s.name
