"""Output-row sharding of a projection across ranks (the 7B-shaped layer).

Rank g of G owns rows [g*N/G, (g+1)*N/G) of every weight: a contiguous byte
range of the GGUF tensor, since GGUF stores whole rows of blocks.  Each rank
computes Y_g = X W_g^T as [B][N/G]; an all-gather over ranks gives
[G][B][N/G], and hd_gather_columns reorders it into Y [B][N].
"""
from __future__ import annotations

import numpy as np

from .synth import BLOCK


def row_range(N: int, rank: int, world: int) -> tuple[int, int]:
    if N % world:
        raise ValueError(f"{N} rows do not split evenly over {world} ranks")
    n = N // world
    return rank * n, (rank + 1) * n


def row_slice(raw: np.ndarray, ggml_type: int, N: int, K: int, rank: int, world: int) -> np.ndarray:
    """GGUF bytes of this rank's rows (raw is [N, row_bytes] or flat)."""
    be, bb = BLOCK[ggml_type]
    row_bytes = (K // be) * bb
    r0, r1 = row_range(N, rank, world)
    return np.ascontiguousarray(np.asarray(raw, np.uint8).reshape(N, row_bytes)[r0:r1])


def gather_columns_reference(gathered: np.ndarray, world: int, B: int, n_shard: int) -> np.ndarray:
    """[G][B][n] -> [B][G*n] (what hd_gather_columns computes on the device)."""
    return np.ascontiguousarray(gathered.reshape(world, B, n_shard).transpose(1, 0, 2).reshape(B, world * n_shard))
