"""How the multi-GPU paths split work across ranks (one process per GPU).

Row-sharded projections: rank r of G holds output rows [r N/G, (r+1) N/G) of
a dense tensor; its bytes are one contiguous slice because every row is a
whole number of blocks. Expert parallelism: rank r holds experts
[r E/G, (r+1) E/G) of each expert tensor, again one contiguous slice of the
[E][rows][cols] layout. Both splits need N (or E) divisible by G.
"""
from __future__ import annotations

import numpy as np

from synth import BLOCK


def row_bytes(quant: int, cols: int) -> int:
    bs, ts = BLOCK[quant]
    return cols // bs * ts


def row_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    if n_rows % world:
        raise ValueError(f"{n_rows} rows do not split over {world} ranks")
    per = n_rows // world
    return rank * per, (rank + 1) * per


def expert_range(n_expert: int, world: int, rank: int) -> tuple[int, int]:
    return row_range(n_expert, world, rank)


def row_shard(data: np.ndarray, quant: int, rows: int, cols: int, world: int, rank: int) -> np.ndarray:
    """The bytes of this rank's rows of a dense [rows][cols] tensor."""
    r0, r1 = row_range(rows, world, rank)
    rb = row_bytes(quant, cols)
    return np.ascontiguousarray(data[r0 * rb:r1 * rb])


def expert_shard(data: np.ndarray, n_expert: int, world: int, rank: int) -> np.ndarray:
    """The bytes of this rank's experts of an [n_expert][rows][cols] tensor."""
    e0, e1 = expert_range(n_expert, world, rank)
    per = data.size // n_expert
    return np.ascontiguousarray(data[e0 * per:e1 * per])


def row_shard_view(model, name: str, world: int, rank: int):
    """This rank's rows of a dense tensor of an opened GGUF model, as an upload
    item pointing into the mapping (only those bytes are read from the file)."""
    rows = model.find(name).shape[1]
    r0, r1 = row_range(rows, world, rank)
    return model.view(name, r0, r1 - r0)


def expert_shard_view(model, name: str, world: int, rank: int):
    """This rank's experts of an [n_expert][rows][cols] tensor of an opened GGUF model."""
    e0, e1 = expert_range(model.find(name).shape[2], world, rank)
    return model.view(name, e0, e1 - e0)
