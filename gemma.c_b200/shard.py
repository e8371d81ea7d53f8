"""Row partition of the sharded W8A8 matmuls (lm_head, FFN at 4B/12B).

Every output row of gemm_int8 / gemv_int8 (gemma.c:2754-2788, 3937-4054) is
independent, so rank r of `world` owns weight rows [r*n/world, (r+1)*n/world)
and computes that slice of the output; an all-gather then yields, for m
tokens, a buffer laid out [world][m][n/world] which is re-laid out to the
reference's [m][n].  libgcu.so's gcu_dev_gemm_int8_rowshard implements this
on the GPU (NCCL all-gather, then one 2-D copy per rank); the helpers here
state the same convention for callers that slice weights per rank.
"""
from __future__ import annotations

import numpy as np


def row_slice(n: int, rank: int, world: int) -> slice:
    """The rows of an n-row weight owned by `rank` (n divisible by world)."""
    if n % world:
        raise ValueError(f"{n} rows do not split over {world} ranks")
    nl = n // world
    return slice(rank * nl, (rank + 1) * nl)


def relayout(gathered: np.ndarray, m: int, n: int, world: int) -> np.ndarray:
    """[world][m][n/world] (all-gather order) -> [m][n]."""
    nl = n // world
    return np.ascontiguousarray(gathered.reshape(world, m, nl).transpose(1, 0, 2).reshape(m, n))
