"""Tensor sharding across the GPUs of one node.

Every GGUF block converts independently, so a model's tensors are split over ranks
with no collective on the data path: each rank converts its own pieces.  Assignment is
longest-processing-time first on the bytes a piece moves (GGUF bytes read plus output
bytes written).  Tensors larger than a rank's fair share are cut into row ranges first
(never the q/k tensors whose head permutation moves rows across the whole tensor, and
never below whole stored units).
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

from .formats import FORMATS, output_layout

__all__ = ["Piece", "piece_cost", "plan_shards"]


@dataclass(frozen=True)
class Piece:
    index: int          # tensor index in the model list
    row0: int
    row1: int           # exclusive

    @property
    def rows(self) -> int:
        return self.row1 - self.row0


def piece_cost(fmt: str, rows: int, cols: int, out: str = "codes") -> int:
    """Bytes read + written converting `rows` rows (the HBM traffic of the piece)."""
    f = FORMATS[fmt]
    n = rows * cols
    lay = output_layout(fmt, n)
    read = n // f.unit_values * f.unit_bytes
    if f.block_values == 0:
        return read + lay["values"]
    if out == "codes":
        return read + lay["codes"] + lay["scales"]
    if out == "f32":
        return read + lay["values"]
    return read + lay["codes"] + lay["scales"] + lay["values"]


def plan_shards(tensors: list[tuple[str, int, int, bool]], world: int, out: str = "codes") -> list[list[Piece]]:
    """tensors: (fmt, rows, cols, permuted) per tensor.  Returns the pieces of each rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    total = sum(piece_cost(f, r, c, out) for f, r, c, _ in tensors)
    share = total / world
    pieces: list[tuple[int, Piece]] = []
    for i, (fmt, rows, cols, permuted) in enumerate(tensors):
        cost = piece_cost(fmt, rows, cols, out)
        n_split = 1
        if world > 1 and not permuted and cost > share / 2 and rows > 1:
            n_split = min(rows, world * 2 if cost > share else world)
        step = -(-rows // n_split)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            pieces.append((piece_cost(fmt, r1 - r0, cols, out), Piece(i, r0, r1)))
    pieces.sort(key=lambda cp: (-cp[0], cp[1].index, cp[1].row0))
    heap = [(0, r) for r in range(world)]
    out_lists: list[list[Piece]] = [[] for _ in range(world)]
    for cost, p in pieces:
        load, r = heapq.heappop(heap)
        out_lists[r].append(p)
        heapq.heappush(heap, (load + cost, r))
    for lst in out_lists:
        lst.sort(key=lambda p: (p.index, p.row0))
    return out_lists
